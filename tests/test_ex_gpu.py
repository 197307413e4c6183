"""GPU parity of the extended scan (selective_scan_fn: delta bias / softplus and the z gate
through mwc_ss_fwd_ex / mwc_ss_bwd_ex) against the float64 oracle composition
(tests/_ex_ref.py): forward output, h_last and every gradient (du, ddelta, dA, dB, dC, dD,
dz, ddelta_bias, dh_prev), on the segmented and the persistent scan kernels.

Tolerances: float32 normwise max relative error < 1e-4; float16 / bfloat16 elementwise
|x - ref| <= atol * max|ref| + rtol * |ref| with (atol, rtol) = (2e-2, 1e-2) for float16 and
(2e-2, 2e-2) for bfloat16 (one rounding of each output to the I/O type)."""
import numpy as np
import pytest
import torch

import _ex_ref as X
from _helpers import assert_fp32, make_inputs, np64

pytestmark = pytest.mark.gpu

TOL = {torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 2e-2)}


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def check(x, ref, dtype, what):
    if ref is None:
        assert x is None, what
        return
    if dtype == torch.float32:
        assert_fp32(x, ref, what=what)
        return
    atol, rtol = TOL[dtype]
    xv = x.detach().float().cpu().double().numpy()
    ref = np.asarray(ref, np.float64)
    bad = np.abs(xv - ref) > atol * max(np.abs(ref).max(), 1e-30) + rtol * np.abs(ref)
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} outside; max err {np.abs(xv - ref).max():.3e}"


CASES = [
    # dtype, B, L, D, z, bias, softplus, h_prev
    (torch.float32, 2, 200, 64, True, True, True, True),
    (torch.float32, 2, 200, 64, False, True, False, False),
    (torch.float32, 2, 200, 64, True, False, False, False),
    (torch.float32, 1, 8192, 64, True, True, True, False),       # L-segmented forward
    (torch.float32, 4, 256, 5120, True, True, True, False),      # persistent kernels
    (torch.float16, 4, 256, 5120, True, True, True, False),
    (torch.bfloat16, 2, 200, 64, True, True, True, True),
    (torch.float16, 3, 130, 40, True, True, True, True),         # ragged
    # the persistent kernels under the transforms: config-3 shape (chained segments), bias
    # without softplus, bfloat16 with h_prev, and the few-chain split passes in float16
    (torch.float16, 4, 2048, 5120, True, True, True, False),
    (torch.float16, 4, 256, 5120, False, True, False, False),
    (torch.bfloat16, 4, 512, 5120, True, True, True, True),
    (torch.float16, 1, 4096, 256, True, True, True, True),
    # ragged L on the persistent kernels (chained segments; split passes; bias only)
    (torch.float16, 4, 2000, 5120, True, True, True, False),
    (torch.float16, 1, 1000, 256, True, True, True, True),
    (torch.float16, 1, 1000, 256, False, True, False, True),
]


@pytest.mark.parametrize("dtype,B,L,D,z_on,bias_on,sp,hp_on", CASES)
def test_extended_scan(dtype, B, L, D, z_on, bias_on, sp, hp_on):
    _need_gpu()
    from mamba_windows_cuda.selective_scan_interface import selective_scan_fn
    x = make_inputs(B, L, D, dtype, seed=51, dist="c1", with_state=True, device="cuda")
    g = torch.Generator().manual_seed(5)
    # with softplus, delta is a pre-activation around zero (both branches of softplus' slope
    # matter); without it delta stays the positive step size (a negative step with A < 0
    # would grow the state without bound), and the bias is non-negative
    raw = (torch.randn(B, L, D, generator=g) * 0.5 - 1.0).to(dtype).cuda()
    delta = raw if sp else x["delta"]
    z = torch.randn(B, L, D, generator=g).to(dtype).cuda() if z_on else None
    b0 = torch.randn(D, generator=g) * 0.3
    bias = (b0 if sp else b0.abs()).to(dtype).cuda() if bias_on else None
    leaves = [t.clone().requires_grad_(True) for t in (x["u"], delta, x["A"], x["Bm"], x["Cm"], x["Dv"])]
    zl = z.clone().requires_grad_(True) if z is not None else None
    bl = bias.clone().requires_grad_(True) if bias is not None else None
    hp = x["h_prev"].clone().requires_grad_(True) if hp_on else None
    out, h_last = selective_scan_fn(*leaves, z=zl, delta_bias=bl, delta_softplus=sp,
                                    return_last_state=True, h_prev=hp)
    (out * x["g"]).sum().backward()
    torch.cuda.synchronize()
    n = [np64(t) for t in leaves]
    kw = dict(z=np64(z) if z is not None else None, bias=np64(bias) if bias is not None else None,
              sp=sp, h_prev=np64(hp) if hp is not None else None)
    o64, _, h64 = X.fwd(*n, **kw)
    g64 = X.bwd(*n, np64(x["g"]), **kw)
    check(out, o64, dtype, "out")
    check(h_last, h64, dtype, "h_last")
    for name, t in zip(("du", "ddelta", "dA", "dB", "dC", "dD"), leaves):
        check(t.grad, g64[name], dtype, name)
    if z is not None:
        check(zl.grad, g64["dz"], dtype, "dz")
    if bias is not None:
        check(bl.grad, g64["dbias"], dtype, "ddelta_bias")
    if hp is not None:
        check(hp.grad, g64["dh_prev"], dtype, "dh_prev")


def test_extended_scan_without_transforms_equals_plain_scan():
    _need_gpu()
    import mamba_windows_cuda as mwc
    from mamba_windows_cuda.selective_scan_interface import selective_scan_fn
    x = make_inputs(2, 300, 96, torch.float32, seed=52, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    a = selective_scan_fn(*args)
    b = mwc.SelectiveScanCuda()(*args)
    assert torch.equal(a, b)


def test_extended_scan_rejects_z_and_bias_off_device():
    """z and delta_bias on the host (with u on the GPU) are rejected before any launch."""
    _need_gpu()
    from mamba_windows_cuda.selective_scan_interface import selective_scan_fn
    x = make_inputs(1, 32, 16, torch.float32, seed=53, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    with pytest.raises(RuntimeError, match="z must match u"):
        selective_scan_fn(*args, z=torch.zeros(1, 32, 16))
    with pytest.raises(RuntimeError, match="delta_bias must be"):
        selective_scan_fn(*args, delta_bias=torch.zeros(16))
