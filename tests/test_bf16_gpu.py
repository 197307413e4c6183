"""bfloat16 I/O (an addition: the reference takes float32 / float16) through the same
kernels: the generic segmented kernels, the persistent TMA kernels (bf16 tensor maps), the
stateful path and parallel_scan_fn. Parity is against the float64 oracle run on the same
bf16-valued inputs.

Tolerance: arithmetic is float32 throughout and every output / gradient is rounded to
bf16 once (unit roundoff 2^-8, so about 2^-9 relative); elementwise
|x - ref| <= 1e-2 * max|ref| + 1e-2 * |ref|.
"""
import numpy as np
import pytest
import torch

from _helpers import make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def assert_bf16(x, ref, what, rtol=1e-2, atol_frac=1e-2):
    x = x.detach().float().cpu().double().numpy()
    ref = np.asarray(ref, np.float64)
    tol = atol_frac * max(np.abs(ref).max(), 1e-30) + rtol * np.abs(ref)
    bad = np.abs(x - ref) > tol
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {bad.size} elements outside bf16 "
                           f"tolerance; max abs err {np.abs(x - ref).max():.3e}")


SHAPES = [
    (2, 200, 64),      # generic kernels, one pass
    (1, 8192, 64),     # generic kernels, L-segmented forward
    (3, 130, 40),      # ragged
    (4, 256, 5120),    # persistent TMA kernels (160 chains)
]


@pytest.mark.parametrize("B,L,D", SHAPES)
def test_bf16_forward_backward(B, L, D):
    _need_gpu()
    from mamba_windows_cuda import _ops
    x = make_inputs(B, L, D, torch.bfloat16, seed=41, dist="c3", device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, _, ck, _ = _ops.ss_forward(*args, want_ckpt=True)
    du, ddelta, dA, dB, dC, dD, _ = _ops.ss_backward(*args, None, x["g"], None, ck)
    torch.cuda.synchronize()
    n = [np64(t) for t in args]
    o64, _ = O.ss_fwd(*n)
    g64 = O.ss_bwd(*n, np64(x["g"]))
    assert_bf16(out, o64, "out")
    for name, t in (("du", du), ("ddelta", ddelta), ("dA", dA), ("dB", dB), ("dC", dC), ("dD", dD)):
        assert_bf16(t, g64[name], name)


def test_bf16_stateful_module_with_h_prev():
    _need_gpu()
    import mamba_windows_cuda as mwc
    x = make_inputs(2, 300, 96, torch.bfloat16, seed=42, dist="c4", with_state=True, device="cuda")
    args = [x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    hp = x["h_prev"].clone().requires_grad_(True)
    out, h_last = mwc.SelectiveScanCuda().forward_with_state(*args, hp)
    (out * x["g"]).sum().backward()
    n = [np64(t) for t in args]
    o64, h64 = O.ss_fwd(*n, np64(hp))
    g64 = O.ss_bwd(*n, np64(x["g"]), h_prev=np64(hp))
    assert_bf16(out, o64, "out")
    assert_bf16(h_last, h64, "h_last")
    assert_bf16(args[0].grad, g64["du"], "du")
    assert_bf16(hp.grad, g64["dh_prev"], "dh_prev")


def test_bf16_parallel_scan():
    _need_gpu()
    from mamba_windows_cuda import parallel_scan_fn
    g = torch.Generator().manual_seed(7)
    A = (torch.rand(4, 64, 512, 1, generator=g) * 0.5 + 0.5).to(torch.bfloat16).cuda()
    X = torch.randn(4, 64, 512, 1, generator=g).to(torch.bfloat16).cuda()
    H = parallel_scan_fn(A, X)
    assert_bf16(H, O.lin_fwd(np64(A), np64(X)), "parallel_scan_fn")
