"""GPU parity at the full sizes of BASELINE.json's configurations, against the float64 oracle
on the same seeded inputs (the reference semantics: mamba_windows_cuda/mamba_cuda.py:93-174
forward, :669-745 backward, :1172-1219 module; selective_scan_cuda_ext.py:562-677 checkpoint
levels; pscan.py:153-171 linear recurrence).

These shapes run the kernels the benchmark times: the chained persistent forward with K > 1
time segments per 128-channel chain (config 3: K = 8, config 2: K = 4, asserted through
mwc_ss_plan), the chained persistent backward, and the few-chain split passes (config 4's
65,536-step chunk).

Tolerances:
* float16 per-element results (out, h_last, du, ddelta, dh_prev): elementwise atol 2e-2 /
  rtol 1e-2 against float64 on the same fp16 inputs;
* float16 reductions (dA over B x L terms, dB / dC over D channels, dD over B x L): the
  same check with atol scaled by max(1, max|ref|), since each is a sum of thousands of
  float32 products before its final rounding to fp16;
* float32: normwise max relative error < 1e-4; parallel_scan_fn float32 normwise < 1e-5.
"""
import numpy as np
import pytest
import torch

from _helpers import assert_fp16, assert_fp32, make_inputs, np64, rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GRADS = ("du", "ddelta", "dA", "dB", "dC", "dD")
REDUCED = ("dA", "dB", "dC", "dD")
KEYS = ("u", "delta", "A", "Bm", "Cm", "Dv")


@pytest.fixture(scope="module")
def mwc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import mamba_windows_cuda
    from mamba_windows_cuda import _lib
    _lib.load()
    return mamba_windows_cuda


def _check_fp16_grads(grads, ref, names=GRADS):
    for k in names:
        assert grads[k].dtype == torch.float16, k
        if k in REDUCED:
            scale = max(1.0, float(np.abs(ref[k]).max()))
            assert_fp16(grads[k], ref[k], k, atol=2e-2 * scale, rtol=1e-2)
        else:
            assert_fp16(grads[k], ref[k], k)


def _oracle_bwd(x, h_prev=None, gh=None):
    return O.ss_bwd(*[np64(x[k]) for k in KEYS], np64(x["g"]), np64(h_prev), np64(gh))


def test_config3_fwd_bwd_chained_path(mwc):
    """Config 3 (B=4, L=2048, D=5120, fp16), fwd + bwd through SelectiveScanCuda (V2 path):
    the benchmark's workload, on the chained persistent kernels with K > 1 segments."""
    from mamba_windows_cuda import _ops
    B, L, D = 4, 2048, 5120
    pf = _ops.plan(B, L, D, torch.float16)
    pb = _ops.plan(B, L, D, torch.float16, backward=True)
    assert pf["path"] == "chained" and pf["K"] > 1, pf
    assert pb["path"] == "chained" and pb["K"] > 1, pb
    x = make_inputs(B, L, D, torch.float16, seed=31, dist="c3", device="cuda")
    leaves = {k: x[k].clone().requires_grad_(True) for k in KEYS}
    out = mwc.SelectiveScanCuda()(*[leaves[k] for k in KEYS])
    out.backward(x["g"])
    torch.cuda.synchronize()
    ref_out, _ = O.ss_fwd(*[np64(x[k]) for k in KEYS])
    assert_fp16(out, ref_out, "out")
    ref = _oracle_bwd(x)
    _check_fp16_grads({n: leaves[k].grad for k, n in zip(KEYS, GRADS)}, ref)


@pytest.mark.parametrize("lvl", [0, 1])
def test_config3_checkpoint_levels_stateful(mwc, lvl):
    """Config 3 through FusedSelectiveScan(checkpoint_lvl) with h_prev ~ N(0, 0.1) and a
    gradient on h_last: the stateful CUDA backward at full size."""
    from mamba_windows_cuda.selective_scan_cuda_ext import FusedSelectiveScan
    B, L, D = 4, 2048, 5120
    x = make_inputs(B, L, D, torch.float16, seed=37 + lvl, dist="c3", with_state=True, device="cuda")
    leaves = {k: x[k].clone().requires_grad_(True) for k in KEYS + ("h_prev",)}
    out, h_last = FusedSelectiveScan(checkpoint_lvl=lvl).forward_with_state(
        *[leaves[k] for k in KEYS + ("h_prev",)])
    torch.autograd.backward([out, h_last], [x["g"], x["gh"]])
    torch.cuda.synchronize()
    ref_out, ref_h = O.ss_fwd(*[np64(x[k]) for k in KEYS], np64(x["h_prev"]))
    assert_fp16(out, ref_out, "out")
    assert_fp16(h_last, ref_h, "h_last")
    ref = _oracle_bwd(x, x["h_prev"], x["gh"])
    grads = {n: leaves[k].grad for k, n in zip(KEYS, GRADS)}
    grads["dh_prev"] = leaves["h_prev"].grad
    _check_fp16_grads(grads, ref, GRADS + ("dh_prev",))


def test_config2_forward_with_state(mwc):
    """Config 2 (B=8, L=2048, D=4096, fp16) inference: forward_with_state from h0 = 0,
    returning out and h_last, on the chained persistent forward with K > 1."""
    from mamba_windows_cuda import _ops
    B, L, D = 8, 2048, 4096
    pf = _ops.plan(B, L, D, torch.float16)
    assert pf["path"] == "chained" and pf["K"] > 1, pf
    x = make_inputs(B, L, D, torch.float16, seed=41, dist="c2", device="cuda")
    with torch.no_grad():
        out, h_last = mwc.SelectiveScanCuda().forward_with_state(*[x[k] for k in KEYS])
    torch.cuda.synchronize()
    ref_out, ref_h = O.ss_fwd(*[np64(x[k]) for k in KEYS])
    assert_fp16(out, ref_out, "out")
    assert_fp16(h_last, ref_h, "h_last")


def test_config4_chunk_streamed_twice(mwc):
    """Config 4's streaming contract at its full chunk size: two 65,536-step fp32 chunks
    (B=1, D=2048) chained through h_prev -> h_last, against one float64 scan of the
    131,072-step sequence (README.md:90-106 of the reference; the split passes run here)."""
    from mamba_windows_cuda import _ops
    B, Lc, D = 1, 65536, 2048
    assert _ops.plan(B, Lc, D, torch.float32)["path"] == "split"
    x = make_inputs(B, 2 * Lc, D, torch.float32, seed=43, dist="c4")
    mod = mwc.SelectiveScanCuda()
    h = torch.zeros(B, D, 16, device="cuda")
    outs = []
    with torch.no_grad():
        for c in range(2):
            sl = slice(c * Lc, (c + 1) * Lc)
            o, h = mod.forward_with_state(*[x[k][:, sl].contiguous().cuda() if x[k].dim() == 3
                                            else x[k].cuda() for k in KEYS], h)
            outs.append(o.cpu())
    ref_out, ref_h = O.ss_fwd(*[np64(x[k]) for k in KEYS])
    assert_fp32(torch.cat(outs, dim=1), ref_out, what="out (2 chunks)")
    assert_fp32(h, ref_h, what="h_last after 2 chunks")


def test_config5_parallel_scan_fp32_full(mwc):
    """Config 5: parallel_scan_fn on (16, 1024, 16384, 1) fp32, a ~ U(0.9, 1), b ~ N(0, 1),
    against the float64 sequential recurrence (parallel_scan_ref's semantics), normwise 1e-5."""
    g = torch.Generator(device="cuda").manual_seed(47)
    a = torch.rand(16, 1024, 16384, 1, generator=g, device="cuda") * 0.1 + 0.9
    b = torch.randn(16, 1024, 16384, 1, generator=g, device="cuda")
    h = mwc.parallel_scan_fn(a, b)
    torch.cuda.synchronize()
    ref = O.lin_fwd(np64(a), np64(b))
    e = rel_err(h, ref)
    assert e < 1e-5, f"normwise relative error {e:.3e}"


def test_config5_parallel_scan_fp16_long(mwc):
    """Config 5': parallel_scan_fn on (16, 1024, 65536, 1) fp16, a ~ U(0.99, 1). The whole
    tensor is scanned on the GPU; 512 of its 16,384 rows (full length each, rows are
    independent) are checked elementwise (atol 2e-2 / rtol 1e-2) against float64 on the same
    fp16 inputs, and every row is checked finite."""
    g = torch.Generator(device="cuda").manual_seed(53)
    a = (torch.rand(16, 1024, 65536, 1, generator=g, device="cuda") * 0.01 + 0.99).half()
    b = torch.randn(16, 1024, 65536, 1, generator=g, device="cuda").half()
    h = mwc.parallel_scan_fn(a, b)
    torch.cuda.synchronize()
    assert h.dtype == torch.float16 and bool(torch.isfinite(h).all())
    rows = torch.randperm(16 * 1024, generator=torch.Generator().manual_seed(0))[:512]
    a2, b2, h2 = (t.view(16 * 1024, 65536)[rows.cuda()] for t in (a, b, h))
    ref = O.lin_fwd(np64(a2).reshape(1, 512, 65536, 1), np64(b2).reshape(1, 512, 65536, 1))
    assert_fp16(h2.reshape(1, 512, 65536, 1), ref, "h (sampled rows)")
