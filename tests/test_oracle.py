"""Pins the CPU oracle to the reference's own outputs (CPU only).

The fixtures in tests/golden were produced by tests/golden/make_golden.py from the
reference's Python functions (selective_scan_ref + torch autograd, the closed form in the
reference's tests, parallel_scan_ref and finite differences of it).
"""
import os

import numpy as np
import pytest

from oracle import oracle as O


def rel(x, ref):
    """Normwise relative error max|x - ref| / max|ref|."""
    return float(np.abs(np.asarray(x, np.float64) - ref).max() / max(np.abs(ref).max(), 1e-300))


GRADS = ("du", "ddelta", "dA", "dB", "dC", "dD")


@pytest.mark.parametrize("name,tol", [("ss_state_f64", 1e-12), ("ss_nostate_f64", 1e-12),
                                      ("ss_state_f32", 2e-6)])
def test_oracle_matches_reference_selective_scan_ref(golden_dir, name, tol):
    z = np.load(os.path.join(golden_dir, name + ".npz"))
    hp = z["h_prev"] if "h_prev" in z else None
    gh = z["gh"] if "gh" in z else None
    args = [z[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last = O.ss_fwd(*args, hp, clamp=False)
    assert rel(out, z["out"]) < tol
    assert rel(h_last, z["h_last"]) < tol
    g = O.ss_bwd(*args, z["g"], hp, gh, clamp=False)
    names = GRADS + (("dh_prev",) if hp is not None else ())
    for k in names:
        assert rel(g[k], z[k]) < tol, k


def test_oracle_matches_reference_closed_form(golden_dir):
    z = np.load(os.path.join(golden_dir, "ss_closed_form_f64.npz"))
    out, h_last = O.ss_fwd(*[z[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")], z["h_prev"])
    assert rel(out, z["out"]) < 1e-12
    assert rel(h_last, z["h_last"]) < 1e-12


def test_oracle_vs_reference_fp16_path(golden_dir):
    """The reference's fp16 PyTorch path vs the float64 oracle on the same fp16 inputs:
    within the fp16 tolerance (atol 2e-2, rtol 1e-2)."""
    z = np.load(os.path.join(golden_dir, "ss_state_f16_fwd.npz"))
    out, h_last = O.ss_fwd(*[z[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")], z["h_prev"])
    np.testing.assert_allclose(z["out"].astype(np.float64), out, atol=2e-2, rtol=1e-2)
    np.testing.assert_allclose(z["h_last"].astype(np.float64), h_last, atol=2e-2, rtol=1e-2)


def test_oracle_matches_parallel_scan_ref(golden_dir):
    z = np.load(os.path.join(golden_dir, "pscan_ref.npz"))
    h = O.lin_fwd(z["a"], z["x"])
    assert rel(h, z["h_f64"]) < 1e-14
    assert rel(h, z["h_f32"]) < 1e-5
    hs = O.lin_fwd(z["a_small"], z["x_small"])
    ga, gx = O.lin_bwd(z["a_small"], hs, z["g_small"])
    np.testing.assert_allclose(ga, z["fd_ga"], atol=1e-7)
    np.testing.assert_allclose(gx, z["fd_gx"], atol=1e-7)


def test_c_oracle_vs_numpy_restatement():
    rng = np.random.default_rng(3)
    B, L, D, N = 2, 33, 5, 16
    u = rng.standard_normal((B, L, D))
    dl = np.log1p(np.exp(rng.normal(-1, .5, (B, L, D))))
    A = -rng.uniform(0.1, 4.0, (D, N))
    Bm, Cm = rng.standard_normal((B, L, N)), rng.standard_normal((B, L, N))
    Dv = rng.uniform(0.5, 1.5, D)
    hp, gh = rng.standard_normal((B, D, N)), rng.standard_normal((B, D, N))
    g = rng.standard_normal((B, L, D))
    o1, h1 = O.ss_fwd(u, dl, A, Bm, Cm, Dv, hp)
    o2, h2 = O.np_ss_fwd(u, dl, A, Bm, Cm, Dv, hp)
    assert rel(o1, o2) < 1e-13 and rel(h1, h2) < 1e-13
    g1 = O.ss_bwd(u, dl, A, Bm, Cm, Dv, g, hp, gh)
    g2 = O.np_ss_bwd(u, dl, A, Bm, Cm, Dv, g, hp, gh)
    for k in GRADS + ("dh_prev",):
        assert rel(g1[k], g2[k]) < 1e-12, k


def test_oracle_streaming_equals_full():
    """Chunked h_prev -> h_last streaming equals one full pass (the property of the
    reference test test_streaming_consistency, tests/test_selective_scan.py:148-193)."""
    rng = np.random.default_rng(11)
    B, L, D, N = 1, 64, 4, 16
    u = rng.standard_normal((B, L, D))
    dl = np.log1p(np.exp(rng.normal(-1, .5, (B, L, D))))
    A = -np.tile(np.arange(1, N + 1, dtype=float), (D, 1))
    Bm, Cm, Dv = rng.standard_normal((B, L, N)), rng.standard_normal((B, L, N)), np.ones(D)
    full, hl = O.ss_fwd(u, dl, A, Bm, Cm, Dv)
    h = None
    outs = []
    for s in range(0, L, 16):
        o, h = O.ss_fwd(u[:, s:s + 16], dl[:, s:s + 16], A, Bm[:, s:s + 16], Cm[:, s:s + 16], Dv, h)
        outs.append(o)
    assert rel(np.concatenate(outs, 1), full) < 1e-13
    assert rel(h, hl) < 1e-13
