"""GPU test of mwc_ss_fwd_noalloc, the forward entry point for callers that cannot
allocate device memory (bindings that only own their input / output buffers, loops that
must not call cudaMalloc). It keeps the L-segment carries in a fixed device array inside
the library instead of a caller workspace.

The test calls it through the C ABI (ctypes) twice in a row on different inputs, with a
shape whose forward is split into L-segments (so the fixed array is actually used), and
checks each result against the regular workspace entry point mwc_ss_fwd within the fp32
tolerance of the other tests (normwise 1e-4) and against the float64 oracle (fp32: normwise
1e-4; fp16: elementwise atol 2e-2 / rtol 1e-2). The file name
makes pytest collect it last.
"""
import ctypes

import pytest
import torch

from _helpers import assert_fp16, assert_fp32, make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_noalloc_forward_matches_workspace_forward(dtype):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from mamba_windows_cuda import _lib, _ops
    lib = _lib.load()
    B, L, D = 1, 8192, 64   # few channels, long sequence: the forward runs in L-segments
    code = 1 if dtype == torch.float16 else 0
    assert lib.mwc_ss_fwd_workspace_bytes(B, L, D, code) > 0, "shape must use segment carries"
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    for call, seed in enumerate((101, 202)):
        x = make_inputs(B, L, D, dtype, seed=seed, with_state=True, dist="c4", device="cuda")
        args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
        out = torch.empty_like(x["u"])
        h_last = torch.empty(B, D, 16, dtype=dtype, device="cuda")
        ckpt = torch.empty(B, _ops.ckpt_count(L), D, 16, dtype=torch.float32, device="cuda")
        decay = torch.empty(B, D, 16, dtype=torch.float32, device="cuda")
        rc = lib.mwc_ss_fwd_noalloc(*[_p(t) for t in args], _p(x["h_prev"]), _p(out), _p(h_last),
                                    _p(ckpt), _p(decay), B, L, D, code, stream)
        assert rc == 0, lib.mwc_last_error()
        ref_out, ref_h, ref_ck, ref_dc = _ops.ss_forward(*args, x["h_prev"], want_h_last=True,
                                                         want_ckpt=True, want_decay=True)
        torch.cuda.synchronize()
        tol = 1e-4 if dtype == torch.float32 else 1e-3
        assert_fp32(out, ref_out.double().cpu().numpy(), tol=tol, what=f"out (call {call})")
        assert_fp32(h_last, ref_h.double().cpu().numpy(), tol=tol, what=f"h_last (call {call})")
        assert_fp32(ckpt, ref_ck.double().cpu().numpy(), tol=1e-4, what=f"ckpt (call {call})")
        assert_fp32(decay, ref_dc.double().cpu().numpy(), tol=1e-4, what=f"decay (call {call})")
        o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
        if dtype == torch.float32:
            assert_fp32(out, o64, what=f"out vs oracle (call {call})")
            assert_fp32(h_last, h64, what=f"h_last vs oracle (call {call})")
        else:   # float64 on the same fp16 inputs, elementwise atol 2e-2 / rtol 1e-2
            assert_fp16(out, o64, f"out vs oracle (call {call})")
            assert_fp16(h_last, h64, f"h_last vs oracle (call {call})")


def test_noalloc_forward_rejects_bad_arguments():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from mamba_windows_cuda import _lib
    lib = _lib.load()
    fake = ctypes.c_void_p(16)
    rc = lib.mwc_ss_fwd_noalloc(fake, fake, fake, fake, fake, fake, None, fake, None, None, None,
                                1, 16, 16, 9, None)
    assert rc == 1 and b"float32/float16" in lib.mwc_last_error()
