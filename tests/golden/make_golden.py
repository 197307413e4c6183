"""Generate the golden fixtures in this directory from the reference's own Python code.

Run once, in a container that has the reference checkout, naming it as the argument or in
``MWC_REFERENCE_ROOT``::

    python tests/golden/make_golden.py REFERENCE_ROOT

It imports the reference package and records inputs and outputs of:

* ``mamba_windows_cuda.mamba_cuda.selective_scan_ref`` (mamba_cuda.py:875-946) forward,
  and its gradients through torch autograd, for loss = sum(out*g) + sum(h_last*gh).
  The reference's einsum at :910 (``'bdl,dn->bdln'``) puts the state axis last while the
  loop at :920-922 indexes the last axis as time, which raises for L != 16. The script
  therefore calls the function unmodified while ``torch.einsum`` is wrapped so that this
  one equation is evaluated as ``'bdl,dn->bdnl'`` (time axis last). No reference source is
  copied or edited.
* ``tests/test_selective_scan.py:8-36`` ``selective_scan_reference`` (the closed form the
  reference's tests use; valid for small |delta*A|).
* ``mamba_windows_cuda.pscan.parallel_scan_ref`` (pscan.py:153-171), plus central
  finite differences of it in float64 as the gradient pin (``PScan.backward`` is
  broken in the reference, and ``parallel_scan_ref`` is not differentiable through its
  in-place writes).

The fixtures are the only part that travels; nothing at test time reads the reference.
"""
from __future__ import annotations

import contextlib
import os
import sys

import numpy as np
import torch

REF_ROOT = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("MWC_REFERENCE_ROOT", "")
OUT_DIR = os.path.dirname(os.path.abspath(__file__))


@contextlib.contextmanager
def time_axis_last_einsum():
    orig = torch.einsum

    def patched(eq, *operands):
        if isinstance(eq, str) and eq.replace(" ", "") == "bdl,dn->bdln":
            eq = "bdl,dn->bdnl"
        return orig(eq, *operands)

    torch.einsum = patched
    try:
        yield
    finally:
        torch.einsum = orig


def c1_inputs(gen, B, L, D, N, dtype, with_state):
    """BASELINE config-1 distributions: u~N(0,1), delta=softplus(N(-1,0.5)),
    A[d,n]=-(n+1), B,C~N(0,1), D=1, g~N(0,1)."""
    u = torch.randn(B, L, D, generator=gen, dtype=torch.float64)
    delta = torch.nn.functional.softplus(
        torch.randn(B, L, D, generator=gen, dtype=torch.float64) * 0.5 - 1.0)
    A = -torch.arange(1, N + 1, dtype=torch.float64).repeat(D, 1)
    Bm = torch.randn(B, L, N, generator=gen, dtype=torch.float64)
    Cm = torch.randn(B, L, N, generator=gen, dtype=torch.float64)
    Dv = torch.ones(D, dtype=torch.float64)
    g = torch.randn(B, L, D, generator=gen, dtype=torch.float64)
    hp = torch.randn(B, D, N, generator=gen, dtype=torch.float64) if with_state else None
    gh = torch.randn(B, D, N, generator=gen, dtype=torch.float64) if with_state else None
    cast = (lambda t: None if t is None else t.to(dtype))
    return [cast(t) for t in (u, delta, A, Bm, Cm, Dv, g, hp, gh)]


def run_ref_fwd_bwd(ref, u, delta, A, Bm, Cm, Dv, g, hp, gh):
    leaves = [t.clone().requires_grad_(True) for t in (u, delta, A, Bm, Cm, Dv)]
    hp_leaf = hp.clone().requires_grad_(True) if hp is not None else None
    with time_axis_last_einsum():
        out, h_last = ref.selective_scan_ref(*leaves, h_prev=hp_leaf)
    loss = (out * g).sum()
    if gh is not None:
        loss = loss + (h_last * gh).sum()
    loss.backward()
    res = {"out": out.detach(), "h_last": h_last.detach()}
    for name, leaf in zip(("du", "ddelta", "dA", "dB", "dC", "dD"), leaves):
        res[name] = leaf.grad
    if hp_leaf is not None:
        res["dh_prev"] = hp_leaf.grad
    return res


def npy(t):
    return None if t is None else t.detach().cpu().numpy()


def save(name, **arrays):
    arrays = {k: v for k, v in arrays.items() if v is not None}
    path = os.path.join(OUT_DIR, name)
    np.savez_compressed(path, **arrays)
    print(f"wrote {path} ({os.path.getsize(path)} bytes)")


def main():
    if not REF_ROOT or not os.path.isdir(os.path.join(REF_ROOT, "mamba_windows_cuda")):
        raise SystemExit("usage: make_golden.py REFERENCE_ROOT (or set MWC_REFERENCE_ROOT)")
    sys.path.insert(0, REF_ROOT)
    import mamba_windows_cuda.mamba_cuda as ref
    import mamba_windows_cuda.pscan as ref_pscan
    sys.path.insert(0, os.path.join(REF_ROOT, "mamba_windows_cuda", "tests"))
    from test_selective_scan import selective_scan_reference  # noqa: E402

    N = 16
    # (1) stateful fwd+bwd, float64 and float32, config-1 distributions
    for dtype, tag in ((torch.float64, "f64"), (torch.float32, "f32")):
        gen = torch.Generator().manual_seed(1234)
        ins = c1_inputs(gen, 2, 48, 24, N, dtype, with_state=True)
        res = run_ref_fwd_bwd(ref, *ins)
        u, delta, A, Bm, Cm, Dv, g, hp, gh = ins
        save(f"ss_state_{tag}.npz", u=npy(u), delta=npy(delta), A=npy(A), Bm=npy(Bm),
             Cm=npy(Cm), Dv=npy(Dv), g=npy(g), h_prev=npy(hp), gh=npy(gh),
             **{k: npy(v) for k, v in res.items()})

    # (2) stateless fwd+bwd (h_prev=None), float64, a longer sequence
    gen = torch.Generator().manual_seed(99)
    ins = c1_inputs(gen, 1, 160, 16, N, torch.float64, with_state=False)
    res = run_ref_fwd_bwd(ref, *ins)
    u, delta, A, Bm, Cm, Dv, g, _, _ = ins
    save("ss_nostate_f64.npz", u=npy(u), delta=npy(delta), A=npy(A), Bm=npy(Bm),
         Cm=npy(Cm), Dv=npy(Dv), g=npy(g), **{k: npy(v) for k, v in res.items()})

    # (3) the reference tests' closed form at their own distributions
    #     (tests/test_selective_scan.py:51-59): u~0.1N, delta=0.01, A=-0.1U, B,C~0.1N, D=0.1
    gen = torch.Generator().manual_seed(42)
    B, L, D = 1, 256, 32
    u = torch.randn(B, L, D, generator=gen, dtype=torch.float64) * 0.1
    delta = torch.full((B, L, D), 0.01, dtype=torch.float64)
    A = -torch.rand(D, N, generator=gen, dtype=torch.float64) * 0.1
    Bm = torch.randn(B, L, N, generator=gen, dtype=torch.float64) * 0.1
    Cm = torch.randn(B, L, N, generator=gen, dtype=torch.float64) * 0.1
    Dv = torch.full((D,), 0.1, dtype=torch.float64)
    hp = torch.randn(B, D, N, generator=gen, dtype=torch.float64)
    out_cf, h_cf = selective_scan_reference(u, delta, A, Bm, Cm, Dv, hp)
    save("ss_closed_form_f64.npz", u=npy(u), delta=npy(delta), A=npy(A), Bm=npy(Bm),
         Cm=npy(Cm), Dv=npy(Dv), h_prev=npy(hp), out=npy(out_cf), h_last=npy(h_cf))

    # (4) fp16 forward through the reference's PyTorch path (CPU half arithmetic)
    gen = torch.Generator().manual_seed(7)
    ins = c1_inputs(gen, 1, 64, 16, N, torch.float16, with_state=True)
    u, delta, A, Bm, Cm, Dv, g, hp, gh = ins
    with torch.no_grad(), time_axis_last_einsum():
        out16, hl16 = ref.selective_scan_ref(u, delta, A, Bm, Cm, Dv, h_prev=hp)
    save("ss_state_f16_fwd.npz", u=npy(u), delta=npy(delta), A=npy(A), Bm=npy(Bm),
         Cm=npy(Cm), Dv=npy(Dv), h_prev=npy(hp), out=npy(out16), h_last=npy(hl16))

    # (5) parallel_scan_ref forward (fp32 and fp64) + finite-difference gradient (fp64)
    gen = torch.Generator().manual_seed(5)
    shape = (2, 3, 40, 4)
    a = torch.rand(shape, generator=gen, dtype=torch.float64) * 0.1 + 0.9
    x = torch.randn(shape, generator=gen, dtype=torch.float64)
    g = torch.randn(shape, generator=gen, dtype=torch.float64)
    h64 = ref_pscan.parallel_scan_ref(a, x)
    h32 = ref_pscan.parallel_scan_ref(a.float(), x.float())
    small = (1, 2, 12, 3)
    a_s, x_s, g_s = a[:1, :2, :12, :3].clone(), x[:1, :2, :12, :3].clone(), g[:1, :2, :12, :3].clone()
    eps = 1e-6
    fd_a = torch.zeros(small, dtype=torch.float64)
    fd_x = torch.zeros(small, dtype=torch.float64)
    for idx in np.ndindex(*small):
        for src, dst in ((a_s, fd_a), (x_s, fd_x)):
            old = src[idx].item()
            src[idx] = old + eps
            fp = (ref_pscan.parallel_scan_ref(a_s, x_s) * g_s).sum().item()
            src[idx] = old - eps
            fm = (ref_pscan.parallel_scan_ref(a_s, x_s) * g_s).sum().item()
            src[idx] = old
            dst[idx] = (fp - fm) / (2 * eps)
    save("pscan_ref.npz", a=npy(a), x=npy(x), h_f64=npy(h64), h_f32=npy(h32),
         a_small=npy(a_s), x_small=npy(x_s), g_small=npy(g_s), fd_ga=npy(fd_a), fd_gx=npy(fd_x))


if __name__ == "__main__":
    main()
