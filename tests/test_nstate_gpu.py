"""GPU parity of the N = 32 / 64 forward scan (selective_scan_forward_nstate through
mwc_ss_fwd_nstate) against the float64 oracle, which takes any N: out, h_last, the float32
checkpoints and the segment decay, on single-pass and L-segmented shapes (segment scans from
zero, carry fold, fixup), float32 / float16 / bfloat16.

The reference supports N = 16 only; N = 16 through the new entry point must equal the regular
forward bitwise. Tolerances as the other scan tests: float32 normwise 1e-4; 16-bit elementwise
atol 2e-2 * max(1, max|ref|) + rtol (1e-2 fp16, 2e-2 bf16)."""
import numpy as np
import pytest
import torch

from _helpers import assert_fp16, assert_fp32, make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def nstate_inputs(B, L, D, N, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    n = torch.arange(1, N + 1, dtype=torch.float32)
    x = {
        "u": torch.randn(B, L, D, generator=g),
        "delta": torch.nn.functional.softplus(torch.randn(B, L, D, generator=g) * 0.5 - 1.0),
        "A": -(n * (1 + 0.1 * torch.rand(D, N, generator=g))),
        "Bm": torch.randn(B, L, N, generator=g),
        "Cm": torch.randn(B, L, N, generator=g),
        "Dv": torch.rand(D, generator=g) + 0.5,
        "h_prev": torch.randn(B, D, N, generator=g) * 0.1,
    }
    return {k: v.to(dtype).cuda() for k, v in x.items()}


CASES = [
    (torch.float32, 2, 300, 96, 32),      # one pass
    (torch.float32, 1, 4096, 64, 64),     # L-segmented
    (torch.float16, 2, 2000, 128, 32),    # L-segmented, ragged L
    (torch.bfloat16, 1, 1024, 256, 64),
]


@pytest.mark.parametrize("dtype,B,L,D,N", CASES)
def test_forward_nstate_matches_oracle(dtype, B, L, D, N):
    _need_gpu()
    from mamba_windows_cuda import _ops
    from mamba_windows_cuda.nstate import selective_scan_forward_nstate
    x = nstate_inputs(B, L, D, N, dtype, seed=N + L)
    names = ("u", "delta", "A", "Bm", "Cm", "Dv")
    with torch.no_grad():
        out, h_last = selective_scan_forward_nstate(*[x[k] for k in names], h_prev=x["h_prev"],
                                                    return_last_state=True)
        _, _, ckpt, decay = _ops.ss_forward(*[x[k] for k in names], x["h_prev"], want_out=False,
                                            want_h_last=True, want_ckpt=True, want_decay=True)
    torch.cuda.synchronize()
    ref_out, ref_h = O.ss_fwd(*[np64(x[k]) for k in names], np64(x["h_prev"]))
    f32 = dtype == torch.float32
    rtol = 1e-2 if dtype == torch.float16 else 2e-2

    def check(a, r, what, tol32=1e-4):
        if f32:
            assert_fp32(a, r, tol=tol32, what=what)
        else:
            scale = max(1.0, float(np.abs(r).max()))
            assert_fp16(a, r, what, atol=2e-2 * scale, rtol=rtol)

    check(out, ref_out, "out")
    check(h_last, ref_h, "h_last")
    k = (L - 1) // 16 // 2
    _, h_k = O.ss_fwd(*[np64(x[n][:, :16 * (k + 1)] if n in ("u", "delta", "Bm", "Cm") else x[n])
                        for n in names], np64(x["h_prev"]))
    assert_fp32(ckpt[:, k], h_k, tol=1e-4 if f32 else rtol, what="ckpt")
    ref_decay = torch.exp(x["delta"].double().sum(1).unsqueeze(-1) * x["A"].double().unsqueeze(0))
    assert_fp32(decay, ref_decay.cpu().numpy(), tol=1e-4 if f32 else rtol, what="decay")


def test_forward_nstate_16_equals_regular_forward():
    _need_gpu()
    from mamba_windows_cuda import _ops
    from mamba_windows_cuda.nstate import selective_scan_forward_nstate
    x = make_inputs(2, 700, 256, torch.float16, seed=81, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    with torch.no_grad():
        a, ha = selective_scan_forward_nstate(*args, h_prev=x["h_prev"], return_last_state=True)
        b, hb, _, _ = _ops.ss_forward(*args, x["h_prev"], want_h_last=True)
    assert torch.equal(a, b) and torch.equal(ha, hb)


def test_forward_nstate_rejects_unsupported():
    _need_gpu()
    from mamba_windows_cuda.nstate import selective_scan_forward_nstate
    x = nstate_inputs(1, 64, 32, 48, torch.float32, seed=82)
    names = ("u", "delta", "A", "Bm", "Cm", "Dv")
    with torch.no_grad(), pytest.raises(RuntimeError, match="N must be one of"):
        selective_scan_forward_nstate(*[x[k] for k in names])
    x = nstate_inputs(1, 64, 32, 32, torch.float32, seed=83)
    u = x["u"].clone().requires_grad_(True)
    with pytest.raises(RuntimeError, match="forward only"):
        selective_scan_forward_nstate(u, *[x[k] for k in names[1:]])


GRAD_CASES = [
    (torch.float32, 1, 1024, 256, 64),    # few chains: the split passes on each 16-state slice
    (torch.float16, 4, 256, 5120, 32),    # many chains: the chained persistent kernels
    (torch.bfloat16, 2, 600, 384, 32),
]


@pytest.mark.parametrize("dtype,B,L,D,N", GRAD_CASES)
def test_nstate_forward_backward_matches_oracle(dtype, B, L, D, N):
    """selective_scan_nstate: N / 16 slices of 16 states on the regular kernels, summed and
    concatenated; every output and gradient against the float64 N-state oracle."""
    _need_gpu()
    from mamba_windows_cuda.nstate import selective_scan_nstate
    x = nstate_inputs(B, L, D, N, dtype, seed=N + D)
    g = torch.Generator(device="cuda").manual_seed(N)
    gy = torch.randn(B, L, D, generator=g, device="cuda").to(dtype)
    gh = torch.randn(B, D, N, generator=g, device="cuda").to(dtype)
    names = ("u", "delta", "A", "Bm", "Cm", "Dv", "h_prev")
    leaves = {k: x[k].clone().requires_grad_(True) for k in names}
    out, h_last = selective_scan_nstate(*[leaves[k] for k in names[:6]], h_prev=leaves["h_prev"],
                                        return_last_state=True)
    ((out.float() * gy.float()).sum() + (h_last.float() * gh.float()).sum()).backward()
    torch.cuda.synchronize()
    n64 = [np64(x[k]) for k in names[:6]]
    ref_out, ref_h = O.ss_fwd(*n64, np64(x["h_prev"]))
    ref = O.ss_bwd(*n64, np64(gy), np64(x["h_prev"]), np64(gh))
    f32 = dtype == torch.float32
    rtol = 1e-2 if dtype == torch.float16 else 2e-2

    def check(a, r, what):
        if f32:
            assert_fp32(a, r, what=what)
        else:
            scale = max(1.0, float(np.abs(r).max()))
            assert_fp16(a, r, what, atol=2e-2 * scale, rtol=rtol)

    check(out, ref_out, "out")
    check(h_last, ref_h, "h_last")
    for k, name in zip(("du", "ddelta", "dA", "dB", "dC", "dD", "dh_prev"), names):
        check(leaves[name].grad, ref[k], k)


def test_nstate_16_equals_regular_scan():
    _need_gpu()
    import mamba_windows_cuda as mwc
    from mamba_windows_cuda.nstate import selective_scan_nstate
    x = make_inputs(2, 300, 256, torch.float32, seed=84, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    a = selective_scan_nstate(*args)
    b = mwc.SelectiveScanCuda()(*args)
    assert torch.equal(a, b)
