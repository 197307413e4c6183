"""GPU parity of the grouped-B / C scan (selective_scan_grouped through mwc_ss_fwd_grouped /
mwc_ss_bwd_grouped): B, C (batch, seqlen, G, 16), channel d reads group d // (D // G).

The reference has no grouped layout, so the oracle is the float64 restatement of the
reference's scan applied to each group's channels with that group's B / C rows: out, h_last,
du, ddelta, dA, dD and dh_prev are that group's slices, and dB / dC of group g are the slice
call's dB / dC (sums over the group's channels only). Cases cover the chained persistent
path (B*D/128 >= SMs) and the few-chain split path, float32 / float16 / bfloat16, a ragged L.

Tolerances as the other scan tests: float32 normwise 1e-4; 16-bit elementwise
atol 2e-2 * max(1, max|ref|) + rtol (1e-2 fp16, 2e-2 bf16)."""
import numpy as np
import pytest
import torch

from _helpers import assert_fp16, assert_fp32, make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GRADS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dh_prev")


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def grouped_inputs(B, L, D, G, dtype, seed):
    x = make_inputs(B, L, D, dtype, seed=seed, with_state=True, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    x["Bm"] = torch.randn(B, L, G, 16, generator=g, device="cuda").to(dtype)
    x["Cm"] = torch.randn(B, L, G, 16, generator=g, device="cuda").to(dtype)
    return x


def oracle_grouped(x, G):
    D = x["u"].shape[2]
    cpg = D // G
    outs, hs, grads = [], [], {k: [] for k in GRADS}
    for gi in range(G):
        sl = slice(gi * cpg, (gi + 1) * cpg)
        args = [np64(x["u"][..., sl]), np64(x["delta"][..., sl]), np64(x["A"][sl]),
                np64(x["Bm"][:, :, gi]), np64(x["Cm"][:, :, gi]), np64(x["Dv"][sl])]
        o, h = O.ss_fwd(*args, np64(x["h_prev"][:, sl]))
        gr = O.ss_bwd(*args, np64(x["g"][..., sl]), np64(x["h_prev"][:, sl]), np64(x["gh"][:, sl]))
        outs.append(o)
        hs.append(h)
        for k in GRADS:
            grads[k].append(gr[k])
    cat = {"du": 2, "ddelta": 2, "dA": 0, "dD": 0, "dh_prev": 1}
    ref = {k: np.concatenate(v, axis=cat[k]) for k, v in grads.items() if k in cat}
    ref["dB"] = np.stack(grads["dB"], axis=2)
    ref["dC"] = np.stack(grads["dC"], axis=2)
    return np.concatenate(outs, axis=2), np.concatenate(hs, axis=1), ref


CASES = [
    # dtype, B, L, D, G: chained path (160 chains) and the few-chain split path
    (torch.float32, 4, 256, 5120, 4),
    (torch.float16, 1, 2048, 1024, 2),
    (torch.bfloat16, 2, 1000, 512, 4),
]


@pytest.mark.parametrize("dtype,B,L,D,G", CASES)
def test_grouped_scan_matches_oracle(dtype, B, L, D, G):
    _need_gpu()
    from mamba_windows_cuda.grouped import selective_scan_grouped
    x = grouped_inputs(B, L, D, G, dtype, seed=71 + G)
    names = ("u", "delta", "A", "Bm", "Cm", "Dv", "h_prev")
    leaves = {k: x[k].clone().requires_grad_(True) for k in names}
    out, h_last = selective_scan_grouped(*[leaves[k] for k in names[:6]], h_prev=leaves["h_prev"],
                                         return_last_state=True)
    ((out.float() * x["g"].float()).sum() + (h_last.float() * x["gh"].float()).sum()).backward()
    torch.cuda.synchronize()
    ref_out, ref_h, ref = oracle_grouped(x, G)
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
    for k, name in zip(GRADS, names):
        check(leaves[name].grad, ref[k], k)


def test_grouped_with_one_group_equals_plain_scan():
    _need_gpu()
    from mamba_windows_cuda import _ops
    x = make_inputs(4, 300, 5120, torch.float16, seed=72, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    g4 = list(args)
    g4[3], g4[4] = args[3].unsqueeze(2), args[4].unsqueeze(2)   # (B, L, 1, 16)
    o1, h1, c1, _ = _ops.ss_forward(*args, x["h_prev"], want_h_last=True, want_ckpt=True)
    o2, h2, c2, _ = _ops.ss_forward(*g4, x["h_prev"], want_h_last=True, want_ckpt=True)
    assert torch.equal(o1, o2) and torch.equal(h1, h2) and torch.equal(c1, c2)
    r1 = _ops.ss_backward(*args, x["h_prev"], x["g"], x["gh"], c1, want_dh_prev=True)
    r2 = _ops.ss_backward(*g4, x["h_prev"], x["g"], x["gh"], c2, want_dh_prev=True)
    for a, b in zip(r1, r2):
        assert torch.equal(a, b.reshape(a.shape))


def test_grouped_rejects_unsupported_shapes():
    _need_gpu()
    from mamba_windows_cuda.grouped import selective_scan_grouped
    x = grouped_inputs(2, 256, 192, 2, torch.float32, seed=73)   # D / G = 96: not a 128 multiple
    with pytest.raises(RuntimeError, match="multiple of 128"):
        selective_scan_grouped(*[x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")])
    x = grouped_inputs(1, 128, 256, 2, torch.float32, seed=74)   # few chains and L < 512
    with pytest.raises(RuntimeError, match="persistent path"):
        selective_scan_grouped(*[x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")])
