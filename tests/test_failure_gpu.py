"""Failure detection on the GPU without a GPU fault: a bounded device wait that can never be
satisfied expires, the kernel records it and returns, the host reads the status through the
C ABI, and the context stays usable for the next scan. Also: after normal persistent
forward / backward launches the status check reports no expired wait, and the opt-in
check of the Python ops (MWC_CHECK_WAITS) runs clean."""
import ctypes

import pytest
import torch

from _helpers import assert_fp32, make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def test_expired_wait_is_reported_and_context_survives():
    _need_gpu()
    from mamba_windows_cuda import _lib, _ops
    lib = _lib.load()
    word = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = lib.mwc_selftest_wait_timeout(ctypes.c_void_p(word.data_ptr()), stream)
    assert rc == 5, (rc, lib.mwc_last_error())
    assert b"expired" in lib.mwc_last_error()
    assert int(word.item()) == 1          # ERR_WAIT_TMA recorded by the kernel
    # the context is intact: a scan still runs and is right
    x = make_inputs(1, 64, 32, torch.float32, seed=3, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, _, _, _ = _ops.ss_forward(*args)
    o64, _ = O.ss_fwd(*[np64(t) for t in args])
    assert_fp32(out, o64, what="out after the self-test")


def test_persistent_launches_report_no_expired_wait(monkeypatch):
    _need_gpu()
    from mamba_windows_cuda import _lib, _ops
    lib = _lib.load()
    monkeypatch.setattr(_ops, "CHECK_WAITS", True)
    # many channels: the persistent TMA kernels (the ones with device waits) run
    x = make_inputs(4, 256, 5120, torch.float16, seed=4, dist="c3", device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    assert lib.mwc_ss_fwd_workspace_bytes(4, 256, 5120, 1) > 0
    out, _, ck, _ = _ops.ss_forward(*args, want_ckpt=True)
    _ops.ss_backward(*args, None, x["g"], None, ck)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert lib.mwc_check_last_launch(stream) == 0
