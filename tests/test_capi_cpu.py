"""CPU-only checks of the native boundary and the host logic (no GPU compute).

* libmwc_b200.so loads and exports every entry point include/mwc_b200.h declares;
* host-side validation returns the documented status codes before touching the GPU;
* the Python API raises RuntimeError like the reference's TORCH_CHECKs;
* the plain-PyTorch API functions kept from the reference (selective_scan_ref,
  selective_scan_backward, parallel_scan_ref) agree with the oracle.
"""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

from _helpers import make_inputs, np64, rel_err
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mwc_b200.h")


def header_functions():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"MWC_API\s+[\w\s\*]+?\b(mwc_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from mamba_windows_cuda import _lib
    return _lib.load()


def test_library_exports_every_header_symbol(lib):
    from mamba_windows_cuda import _lib
    names = header_functions()
    assert len(names) >= 11
    raw = ctypes.CDLL(_lib.LIB_PATH)
    for n in names:
        assert hasattr(raw, n), f"{n} missing from {_lib.LIB_NAME}"
    assert set(names) == set(_lib.SIGNATURES), "ctypes signatures out of sync with the header"


def test_library_identity(lib):
    assert lib.mwc_abi_version() == 1
    assert b"sm_100a" in lib.mwc_build_info()


def test_size_queries(lib):
    assert lib.mwc_ss_ckpt_count(1) == 1
    assert lib.mwc_ss_ckpt_count(16) == 1
    assert lib.mwc_ss_ckpt_count(17) == 2
    assert lib.mwc_ss_ckpt_count(0) == 0
    ws = lib.mwc_ss_bwd_workspace_bytes(4, 2048, 5120, 1)
    assert ws > 4 * 5120 * 17 * 4 and ws % 256 == 0
    # a long sequence with few channels is scanned in parallel segments (carry space);
    # many channels run the persistent queue (flags + segment hand-off states)
    assert lib.mwc_ss_fwd_workspace_bytes(1, 65536, 2048, 0) > 0
    assert lib.mwc_ss_fwd_workspace_bytes(4, 2048, 5120, 1) > 0
    # few channels and a short sequence: one pass, no workspace
    assert lib.mwc_ss_fwd_workspace_bytes(1, 256, 128, 0) == 0


def test_plan_query(lib):
    """mwc_ss_plan reports the path the entry points take (148 SMs assumed without a GPU):
    the benchmark's config 3 and config 2 run the chained persistent kernels, config 4's
    chunk the few-chain split passes, short few-channel shapes the generic kernels. The
    chained forward gives each SM one run of the chains' concatenated 32-step tiles (seg =
    the longest run); K = 2 when a run boundary cuts a chain, 1 when every run is whole
    chains. The chained backward cuts each chain into K segments of seg 16-step tiles."""
    from mamba_windows_cuda import _ops
    f16 = torch.float16
    p3f, p3b = _ops.plan(4, 2048, 5120, f16), _ops.plan(4, 2048, 5120, f16, backward=True)
    # config 3: 160 chains x 64 tiles over 148 runs of 69-70 tiles
    assert p3f == {"path": "chained", "K": 2, "seg": 70, "grid": 148}, p3f
    assert p3b["path"] == "chained" and p3b["K"] > 1 and p3b["K"] * p3b["seg"] * 16 >= 2048
    assert _ops.plan(8, 2048, 4096, f16)["K"] == 2
    # one chain per SM: whole chains, nothing handed over
    assert _ops.plan(4, 2048, 4736, f16) == {"path": "chained", "K": 1, "seg": 64, "grid": 148}
    assert _ops.plan(2, 4096, 18944, f16) == {"path": "chained", "K": 1, "seg": 256, "grid": 148}
    assert _ops.plan(1, 65536, 2048, torch.float32)["path"] == "split"
    assert _ops.plan(2, 256, 5120, f16)["path"] == "generic"
    # rows of D x 2 bytes that are not a multiple of 16 bytes never take the TMA paths
    assert _ops.plan(4, 2048, 5121, f16)["path"] == "generic"
    info = (ctypes.c_int32 * 4)()
    assert lib.mwc_ss_plan(1, 16, 16, 7, 0, info) == 1


def test_c_abi_rejects_bad_arguments_without_touching_the_gpu(lib):
    nul = None
    fake = ctypes.c_void_p(16)  # never dereferenced: validation fails first
    rc = lib.mwc_ss_fwd(fake, fake, fake, fake, fake, fake, nul, fake, nul, nul, nul, nul, 0,
                        1, 16, 16, 7, nul)
    assert rc == 1 and b"float32/float16" in lib.mwc_last_error()
    rc = lib.mwc_ss_fwd(nul, fake, fake, fake, fake, fake, nul, fake, nul, nul, nul, nul, 0,
                        1, 16, 16, 0, nul)
    assert rc == 1 and b"required" in lib.mwc_last_error()
    rc = lib.mwc_ss_fwd(fake, fake, fake, fake, fake, fake, nul, nul, nul, nul, nul, nul, 0,
                        1, 16, 16, 0, nul)
    assert rc == 1 and b"no output" in lib.mwc_last_error()
    rc = lib.mwc_ss_fwd(fake, fake, fake, fake, fake, fake, nul, fake, nul, nul, nul, nul, 0,
                        1, 0, 16, 0, nul)
    assert rc == 1 and b"empty" in lib.mwc_last_error()
    rc = lib.mwc_ss_bwd(*([fake] * 6), nul, fake, nul, nul, *([fake] * 6), nul, fake, 1 << 40,
                        1, 64, 16, 0, nul)
    assert rc == 1 and b"checkpoint" in lib.mwc_last_error()
    rc = lib.mwc_ss_bwd(*([fake] * 6), nul, fake, nul, fake, *([fake] * 6), nul, fake, 8,
                        1, 64, 16, 0, nul)
    assert rc == 3 and b"workspace" in lib.mwc_last_error()
    rc = lib.mwc_ss_fixup(fake, fake, nul, fake, nul, fake, nul, nul, 1, 16, 16, 0, nul)
    assert rc == 1 and b"C_ssm" in lib.mwc_last_error()
    rc = lib.mwc_lin_scan_fwd(fake, nul, fake, 1, 16, 1, 0, nul)
    assert rc == 1


def test_failure_entry_points_without_a_launch(lib):
    # nothing launched on this thread (or the last call failed validation): nothing to
    # check, and the device is not touched
    fake = ctypes.c_void_p(16)
    lib.mwc_ss_fwd(fake, fake, fake, fake, fake, fake, None, fake, None, None, None, None, 0,
                   1, 16, 16, 7, None)
    assert lib.mwc_check_last_launch(None) == 0
    assert lib.mwc_selftest_wait_timeout(None, None) == 1
    assert b"dev_word" in lib.mwc_last_error()


def test_python_api_rejects_cpu_tensors_like_the_reference():
    import mamba_windows_cuda as m
    x = make_inputs(1, 8, 4)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        m.SelectiveScanCuda()(x["u"], x["delta"], x["A"], x["Bm"], x["Cm"], x["Dv"])
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        m.SelectiveScanCuda().forward_with_state(x["u"], x["delta"], x["A"], x["Bm"], x["Cm"],
                                                 x["Dv"])
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        m.parallel_scan_fn(torch.rand(1, 2, 8, 1), torch.rand(1, 2, 8, 1))


def test_added_python_apis_reject_cpu_tensors():
    from mamba_windows_cuda.grouped import selective_scan_grouped
    from mamba_windows_cuda.nstate import selective_scan_forward_nstate
    x = make_inputs(1, 8, 4)
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        selective_scan_grouped(*args[:3], x["Bm"].unsqueeze(2), x["Cm"].unsqueeze(2), args[5])
    with pytest.raises(RuntimeError, match="CUDA tensors"), torch.no_grad():
        selective_scan_forward_nstate(*args)


def test_nstate_workspace_query(lib):
    # N = 32 / 64: the generic forward's segment carries (N + 1 floats per channel and segment)
    # for a long sequence over few channels, none for a short one; other N: none
    assert lib.mwc_ss_fwd_nstate_workspace_bytes(1, 65536, 64, 32, 0) > 0
    assert lib.mwc_ss_fwd_nstate_workspace_bytes(1, 65536, 64, 64, 0) > \
        lib.mwc_ss_fwd_nstate_workspace_bytes(1, 65536, 64, 32, 0)
    assert lib.mwc_ss_fwd_nstate_workspace_bytes(1, 256, 64, 32, 0) == 0
    assert lib.mwc_ss_fwd_nstate_workspace_bytes(1, 65536, 64, 48, 0) == 0
    assert lib.mwc_ss_fwd_nstate_workspace_bytes(4, 2048, 5120, 16, 1) == \
        lib.mwc_ss_fwd_workspace_bytes(4, 2048, 5120, 1)


def test_selective_scan_ref_and_backward_match_oracle():
    from mamba_windows_cuda.mamba_cuda import selective_scan_backward, selective_scan_ref
    x = make_inputs(2, 40, 12, torch.float64, seed=4, with_state=True)
    out, h_last, inter = selective_scan_ref(x["u"], x["delta"], x["A"], x["Bm"], x["Cm"], x["Dv"],
                                            x["h_prev"], return_intermediates=True)
    ref_out, ref_h = O.ss_fwd(*[np64(x[k]) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")],
                              np64(x["h_prev"]))
    assert rel_err(out, ref_out) < 1e-12 and rel_err(h_last, ref_h) < 1e-12
    g = selective_scan_backward(x["g"], x["gh"], inter, x["Dv"])
    ref = O.ss_bwd(*[np64(x[k]) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")], np64(x["g"]),
                   np64(x["h_prev"]), np64(x["gh"]))
    for got, k in zip(g, ("du", "ddelta", "dA", "dB", "dC", "dD", "dh_prev")):
        assert rel_err(got, ref[k]) < 1e-10, k


def test_parallel_scan_ref_matches_oracle():
    from mamba_windows_cuda import parallel_scan_ref
    g = torch.Generator().manual_seed(0)
    A = torch.rand(2, 3, 50, 4, generator=g, dtype=torch.float64)
    X = torch.randn(2, 3, 50, 4, generator=g, dtype=torch.float64)
    assert rel_err(parallel_scan_ref(A, X), O.lin_fwd(A, X)) < 1e-14
