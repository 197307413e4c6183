"""The plain-PyTorch version of the extended scan (selective_scan_ref_ex: delta bias /
softplus and the z gate around the reference's selective_scan_ref) against the float64
oracle composition (tests/_ex_ref.py), forward and all gradients, on CPU."""
import numpy as np
import pytest
import torch

import _ex_ref as X
from _helpers import make_inputs, np64, rel_err


@pytest.mark.parametrize("z_on,bias_on,sp", [(True, True, True), (False, True, False),
                                             (True, False, True), (False, False, False)])
def test_ref_ex_matches_oracle_composition(z_on, bias_on, sp):
    from mamba_windows_cuda.selective_scan_interface import selective_scan_ref_ex
    x = make_inputs(2, 24, 6, torch.float64, seed=9, dist="c1", with_state=True)
    g = torch.Generator().manual_seed(3)
    z = torch.randn(2, 24, 6, generator=g, dtype=torch.float64) if z_on else None
    bias = torch.randn(6, generator=g, dtype=torch.float64) * 0.5 if bias_on else None
    leaves = [x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    zl = z.clone().requires_grad_(True) if z is not None else None
    bl = bias.clone().requires_grad_(True) if bias is not None else None
    hp = x["h_prev"].clone().requires_grad_(True)
    out, h_last = selective_scan_ref_ex(*leaves, z=zl, delta_bias=bl, delta_softplus=sp,
                                        return_last_state=True, h_prev=hp)
    (out * x["g"]).sum().backward()
    n = [np64(t) for t in leaves]
    o64, _, h64 = X.fwd(*n, z=np64(z) if z is not None else None,
                        bias=np64(bias) if bias is not None else None, sp=sp, h_prev=np64(hp))
    g64 = X.bwd(*n, np64(x["g"]), z=np64(z) if z is not None else None,
                bias=np64(bias) if bias is not None else None, sp=sp, h_prev=np64(hp))
    assert rel_err(out, o64) < 1e-10 and rel_err(h_last, h64) < 1e-10
    for name, t in zip(("du", "ddelta", "dA", "dB", "dC", "dD"), leaves):
        assert rel_err(t.grad, g64[name]) < 1e-9, name
    assert rel_err(hp.grad, g64["dh_prev"]) < 1e-9
    if z is not None:
        assert rel_err(zl.grad, g64["dz"]) < 1e-9
    if bias is not None:
        assert rel_err(bl.grad, g64["dbias"]) < 1e-9
