"""GPU parity tests: the sm_100a kernels (through the reference-named Python API and the
C ABI) against the float64 CPU oracle on identical seeded inputs.

Tolerances:
* float32: normwise max relative error < 1e-4 for outputs, h_last and every gradient;
* float16: elementwise atol 2e-2 / rtol 1e-2 against float64 run on the same fp16 inputs;
* parallel_scan_fn float32: normwise 1e-5 against parallel_scan_ref / the oracle.
"""
import numpy as np
import pytest
import torch

from _helpers import assert_fp16, assert_fp32, make_inputs, np64, rel_err
from oracle import oracle as O

pytestmark = pytest.mark.gpu

GRADS = ("du", "ddelta", "dA", "dB", "dC", "dD")


@pytest.fixture(scope="module")
def mwc():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import mamba_windows_cuda
    from mamba_windows_cuda import _lib
    _lib.load()
    return mamba_windows_cuda


def oracle_fwd(x, h_prev=None):
    return O.ss_fwd(np64(x["u"]), np64(x["delta"]), np64(x["A"]), np64(x["Bm"]), np64(x["Cm"]),
                    np64(x["Dv"]), np64(h_prev))


def oracle_bwd(x, h_prev=None, gh=None):
    return O.ss_bwd(np64(x["u"]), np64(x["delta"]), np64(x["A"]), np64(x["Bm"]), np64(x["Cm"]),
                    np64(x["Dv"]), np64(x["g"]), np64(h_prev), np64(gh))


def run_stateful(mwc, x, h_prev, gh, grad=True):
    from mamba_windows_cuda.mamba_cuda import SelectiveScanCudaFunction
    leaves = {k: x[k].clone().requires_grad_(grad) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")}
    hp = h_prev.clone().requires_grad_(grad) if h_prev is not None else None
    out, h_last = SelectiveScanCudaFunction.apply(leaves["u"], leaves["delta"], leaves["A"],
                                                  leaves["Bm"], leaves["Cm"], leaves["Dv"], hp)
    grads = {}
    if grad:
        loss = (out.float() * x["g"].float()).sum()
        if gh is not None:
            loss = loss + (h_last.float() * gh.float()).sum()
        loss.backward()
        for k, name in zip(("u", "delta", "A", "Bm", "Cm", "Dv"), GRADS):
            grads[name] = leaves[k].grad
        if hp is not None:
            grads["dh_prev"] = hp.grad
    return out, h_last, grads


SHAPES = [
    (1, 1024, 256),   # BASELINE config 1 (the parity config)
    (2, 100, 40),     # ragged L (not a multiple of 16) and D (not a multiple of the tile)
    (3, 17, 8),
    (1, 1, 16),       # single step
    (2, 16, 129),
]


@pytest.mark.parametrize("B,L,D", SHAPES)
@pytest.mark.parametrize("state", [False, True])
def test_fp32_forward_backward_matches_oracle(mwc, B, L, D, state):
    x = make_inputs(B, L, D, torch.float32, seed=B * 1000 + L + D, with_state=state,
                    device="cuda")
    hp, gh = (x["h_prev"], x["gh"]) if state else (None, None)
    out, h_last, grads = run_stateful(mwc, x, hp, gh)
    ref_out, ref_h = oracle_fwd(x, hp)
    assert_fp32(out, ref_out, what="out")
    assert_fp32(h_last, ref_h, what="h_last")
    ref = oracle_bwd(x, hp, gh)
    for k in GRADS:
        assert_fp32(grads[k], ref[k], what=k)
    if state:
        assert_fp32(grads["dh_prev"], ref["dh_prev"], what="dh_prev")


@pytest.mark.parametrize("B,L,D", [(1, 1024, 256), (2, 100, 40), (1, 300, 64)])
def test_fp16_forward_backward_matches_oracle(mwc, B, L, D):
    x = make_inputs(B, L, D, torch.float16, seed=7 + L, with_state=True, device="cuda")
    out, h_last, grads = run_stateful(mwc, x, x["h_prev"], x["gh"])
    assert out.dtype == torch.float16 and h_last.dtype == torch.float16
    ref_out, ref_h = oracle_fwd(x, x["h_prev"])
    assert_fp16(out, ref_out, "out")
    assert_fp16(h_last, ref_h, "h_last")
    ref = oracle_bwd(x, x["h_prev"], x["gh"])
    for k in GRADS + ("dh_prev",):
        assert grads[k].dtype == torch.float16
        # gradients that are sums over many terms: tolerance relative to their scale
        scale = max(1.0, float(np.abs(ref[k]).max()))
        assert_fp16(grads[k], ref[k], k, atol=2e-2 * scale, rtol=1e-2)


def test_default_module_path_v2(mwc):
    """SelectiveScanCuda.forward without h_prev (SelectiveScanFnV2) on config 1."""
    x = make_inputs(1, 1024, 256, torch.float32, seed=0, device="cuda")
    leaves = {k: x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")}
    out = mwc.SelectiveScanCuda()(leaves["u"], leaves["delta"], leaves["A"], leaves["Bm"],
                                  leaves["Cm"], leaves["Dv"])
    (out * x["g"]).sum().backward()
    ref_out, _ = oracle_fwd(x)
    assert_fp32(out, ref_out, what="out")
    ref = oracle_bwd(x)
    for k, name in zip(("u", "delta", "A", "Bm", "Cm", "Dv"), GRADS):
        assert_fp32(leaves[k].grad, ref[name], what=name)


def test_v1_recompute_path_equals_v2(mwc):
    from mamba_windows_cuda.mamba_cuda import SelectiveScanFn, SelectiveScanFnV2
    x = make_inputs(2, 200, 48, torch.float32, seed=3, device="cuda")
    res = []
    for fn in (SelectiveScanFn, SelectiveScanFnV2):
        leaves = [x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
        out = fn.apply(*leaves)
        (out * x["g"]).sum().backward()
        res.append([out] + [t.grad for t in leaves])
    for a, b in zip(*res):
        assert torch.equal(a, b)


@pytest.mark.parametrize("lvl", [0, 1])
def test_checkpoint_levels(mwc, lvl):
    from mamba_windows_cuda.selective_scan_cuda_ext import FusedSelectiveScan
    x = make_inputs(2, 150, 40, torch.float32, seed=11, with_state=True, device="cuda")
    leaves = {k: x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv",
                                                             "h_prev")}
    mod = FusedSelectiveScan(checkpoint_lvl=lvl)
    out, h_last = mod.forward_with_state(leaves["u"], leaves["delta"], leaves["A"], leaves["Bm"],
                                         leaves["Cm"], leaves["Dv"], leaves["h_prev"])
    ((out * x["g"]).sum() + (h_last * x["gh"]).sum()).backward()
    ref = oracle_bwd(x, x["h_prev"], x["gh"])
    for k, name in zip(("u", "delta", "A", "Bm", "Cm", "Dv", "h_prev"), GRADS + ("dh_prev",)):
        assert_fp32(leaves[k].grad, ref[name], what=name)


def test_backward_is_deterministic(mwc):
    x = make_inputs(2, 300, 96, torch.float32, seed=5, with_state=True, device="cuda")
    _, _, g1 = run_stateful(mwc, x, x["h_prev"], x["gh"])
    _, _, g2 = run_stateful(mwc, x, x["h_prev"], x["gh"])
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_segmented_long_sequence_forward(mwc):
    """Few channels, long L: the forward splits L into segments (scan from zero + carry
    fold + fixup). Output, h_last and the checkpoints the backward consumes must match."""
    B, L, D = 1, 12000, 32
    x = make_inputs(B, L, D, torch.float32, seed=21, with_state=True, dist="c4", device="cuda")
    from mamba_windows_cuda import _lib, _ops
    assert _lib.load().mwc_ss_fwd_workspace_bytes(B, L, D, 0) > 0, "segmented mode not taken"
    out, h_last, ckpt, decay = _ops.ss_forward(x["u"], x["delta"], x["A"], x["Bm"], x["Cm"],
                                               x["Dv"], x["h_prev"], want_h_last=True,
                                               want_ckpt=True, want_decay=True)
    ref_out, ref_h = oracle_fwd(x, x["h_prev"])
    assert_fp32(out, ref_out, what="out")
    assert_fp32(h_last, ref_h, what="h_last")
    # checkpoint k = state after step 16k+15: compare with the oracle prefix
    k = 500
    _, h_k = O.ss_fwd(*[np64(x[n][:, :16 * (k + 1)] if n in ("u", "delta", "Bm", "Cm") else x[n])
                        for n in ("u", "delta", "A", "Bm", "Cm", "Dv")], np64(x["h_prev"]))
    assert_fp32(ckpt[:, k], h_k, what="ckpt")
    dsum = x["delta"].double().sum(1)                       # (B, D)
    ref_decay = torch.exp(dsum.unsqueeze(-1) * x["A"].double().unsqueeze(0))
    assert_fp32(decay, ref_decay.cpu().numpy(), what="decay")
    # gradients through the segmented forward's checkpoints
    _, _, grads = run_stateful(mwc, x, x["h_prev"], x["gh"])
    ref = oracle_bwd(x, x["h_prev"], x["gh"])
    for k2 in GRADS + ("dh_prev",):
        assert_fp32(grads[k2], ref[k2], what=k2)


def test_streaming_equals_full(mwc):
    """Reference test_streaming_consistency (tests/test_selective_scan.py:148-193)."""
    m = mwc.SelectiveScanCuda()
    x = make_inputs(1, 2048, 256, torch.float16, seed=789, dist="reftest", device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    with torch.no_grad():
        full, h_full = m.forward_with_state(*args)
        h = torch.zeros(1, 256, 16, device="cuda", dtype=torch.float16)
        outs = []
        for s in range(0, 2048, 1024):
            o, h = m.forward_with_state(x["u"][:, s:s + 1024], x["delta"][:, s:s + 1024], x["A"],
                                        x["Bm"][:, s:s + 1024], x["Cm"][:, s:s + 1024], x["Dv"],
                                        h_prev=h)
            outs.append(o)
    assert (full.float() - torch.cat(outs, 1).float()).abs().max().item() < 1e-3
    assert (h_full.float() - h.float()).abs().max().item() < 1e-3


def test_reference_closed_form_small_delta(mwc):
    """The reference tests' closed form (tests/test_selective_scan.py:8-36) at their
    distributions, fp16 and fp32, max abs diff < 1e-3 (their bar)."""
    for dt, seed in ((torch.float16, 0), (torch.float32, 42)):
        x = make_inputs(1, 1024, 256, dt, seed=seed, dist="reftest", with_state=True,
                        device="cuda")
        hp = x["h_prev"]
        with torch.no_grad():
            out = mwc.SelectiveScanCuda()(x["u"], x["delta"], x["A"], x["Bm"], x["Cm"], x["Dv"], hp)
        ref_out, _ = oracle_fwd(x, hp)
        assert np.abs(out.double().cpu().numpy() - ref_out).max() < 1e-3


def test_extreme_delta_is_finite(mwc):
    """Reference test_numerical_stability_extreme_values (delta = 10)."""
    x = make_inputs(1, 512, 64, torch.float16, seed=999, dist="reftest", device="cuda")
    delta = torch.full_like(x["delta"], 10.0)
    with torch.no_grad():
        out = mwc.SelectiveScanCuda()(x["u"], delta, x["A"], x["Bm"], x["Cm"], x["Dv"],
                                      torch.zeros(1, 64, 16, device="cuda", dtype=torch.float16))
    assert torch.isfinite(out).all()


def test_positive_exponent_is_clamped_like_safe_exp(mwc):
    """A*delta > 88 is clamped to exp(88) as in the reference's safe_exp."""
    x = make_inputs(1, 1, 16, torch.float32, seed=1, device="cuda")
    A = torch.full_like(x["A"], 50.0)
    delta = torch.full_like(x["delta"], 2.0)   # A*delta = 100 > 88
    u = torch.zeros_like(x["u"])
    with torch.no_grad():
        out, h = mwc.SelectiveScanCuda().forward_with_state(
            u, delta, A, x["Bm"], x["Cm"], x["Dv"], torch.full((1, 16, 16), 1e-36, device="cuda"))
    ref_out, ref_h = O.ss_fwd(np64(u), np64(delta), np64(A), np64(x["Bm"]), np64(x["Cm"]),
                              np64(x["Dv"]), np.full((1, 16, 16), 1e-36), clamp=True)
    assert rel_err(h, ref_h) < 1e-4


def test_input_validation_raises_runtime_error(mwc):
    """Reference test_input_validation (tests/test_selective_scan.py:239-262) and the
    TORCH_CHECK contract (mamba_cuda.py:186-238)."""
    m = mwc.SelectiveScanCuda()
    x = make_inputs(1, 64, 32, torch.float16, seed=0, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    with pytest.raises(RuntimeError):
        m(*args, torch.randn(1, 32, 17, device="cuda").half())
    with pytest.raises(RuntimeError):
        m(*args, torch.randn(2, 32, 16, device="cuda").half())
    with pytest.raises(RuntimeError):
        m(x["u"].float(), *args[1:])
    with pytest.raises(RuntimeError):
        m(args[0].cpu(), *args[1:])
    with pytest.raises(RuntimeError):
        m(args[0], args[1], torch.randn(32, 8, device="cuda").half(), *args[3:])


def test_large_shapes_finite(mwc):
    """Reduced version of test_large_shapes_and_streaming (finiteness, long L, D=2048)."""
    m = mwc.SelectiveScanCuda()
    for (B, L, D) in ((1, 16384, 768), (1, 32768, 2048)):
        x = make_inputs(B, L, D, torch.float16, seed=123, dist="reftest", device="cuda")
        with torch.no_grad():
            out = m(x["u"], x["delta"], x["A"], x["Bm"], x["Cm"], x["Dv"], None)
        assert torch.isfinite(out).all()


def test_fixup_c_abi_split_equals_full(mwc):
    """Scan the second half from zero, fold the first half's state with mwc_ss_fixup:
    equals the unsplit scan (the L-sharding primitive)."""
    from mamba_windows_cuda import _ops
    B, L, D = 2, 4096, 64
    x = make_inputs(B, L, D, torch.float32, seed=8, dist="c4", device="cuda")
    a = {k: x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")}
    full, h_full, ck_full, _ = _ops.ss_forward(*a.values(), want_h_last=True, want_ckpt=True)
    half = L // 2
    s1 = {k: (v[:, :half].contiguous() if k in ("u", "delta", "Bm", "Cm") else v) for k, v in a.items()}
    s2 = {k: (v[:, half:].contiguous() if k in ("u", "delta", "Bm", "Cm") else v) for k, v in a.items()}
    _, h1, _, _ = _ops.ss_forward(*s1.values(), want_out=False, want_h_last=True)
    out2, h2, ck2, dec2 = _ops.ss_forward(*s2.values(), want_h_last=True, want_ckpt=True,
                                          want_decay=True)
    _ops.ss_fixup(s2["delta"], s2["A"], s2["Cm"], h1.float().contiguous(), dec2, out2, h2, ck2)
    assert_fp32(out2, full[:, half:], what="out")
    assert_fp32(h2, h_full, what="h_last")
    assert_fp32(ck2, ck_full[:, half // 16:], what="ckpt")


# ----------------------------------------------------------------------------- pscan

@pytest.mark.parametrize("shape", [(2, 32, 128, 16), (2, 8, 1000, 1), (1, 3, 77, 5),
                                   (4, 64, 4096, 1)])
def test_parallel_scan_fp32(mwc, shape):
    from mamba_windows_cuda import parallel_scan_fn, parallel_scan_ref
    g = torch.Generator().manual_seed(42)
    A = (torch.rand(shape, generator=g) * 0.1 + 0.9).cuda()
    X = torch.randn(shape, generator=g).cuda()
    H = parallel_scan_fn(A, X)
    ref = O.lin_fwd(np64(A), np64(X))
    assert rel_err(H, ref) < 1e-5
    if shape[2] <= 1000:
        assert rel_err(H, parallel_scan_ref(A, X)) < 1e-5


@pytest.mark.parametrize("shape", [(2, 8, 333, 1), (1, 4, 64, 16), (2, 2, 100, 3)])
def test_parallel_scan_grad(mwc, shape):
    from mamba_windows_cuda import parallel_scan_fn
    g = torch.Generator().manual_seed(1)
    A = (torch.rand(shape, generator=g) * 0.1 + 0.9).cuda().requires_grad_(True)
    X = torch.randn(shape, generator=g).cuda().requires_grad_(True)
    G = torch.randn(shape, generator=g).cuda()
    H = parallel_scan_fn(A, X)
    (H * G).sum().backward()
    Href = O.lin_fwd(np64(A), np64(X))
    ga, gx = O.lin_bwd(np64(A), Href, np64(G))
    assert rel_err(X.grad, gx) < 1e-5
    assert rel_err(A.grad, ga) < 1e-5


def test_parallel_scan_fp16_long(mwc):
    from mamba_windows_cuda import parallel_scan_fn
    g = torch.Generator().manual_seed(2)
    shape = (2, 16, 65536, 1)
    A = (torch.rand(shape, generator=g) * 0.01 + 0.99).half().cuda()
    X = torch.randn(shape, generator=g).half().cuda()
    H = parallel_scan_fn(A, X)
    ref = O.lin_fwd(np64(A), np64(X))
    assert_fp16(H, ref, "pscan fp16")


def test_parallel_scan_reference_test_shape(mwc):
    """Reference test_parallel_scan_correctness (tests/test_pscan.py:14-35): |A| < 1
    random, (2, 32, 128, 16), max abs diff < 1e-4 against parallel_scan_ref."""
    from mamba_windows_cuda import parallel_scan_fn, parallel_scan_ref
    torch.manual_seed(42)
    A = torch.randn(2, 32, 128, 16, device="cuda").abs() * 0.1
    X = torch.randn(2, 32, 128, 16, device="cuda")
    assert (parallel_scan_fn(A, X) - parallel_scan_ref(A, X)).abs().max().item() < 1e-4


# ------------------------------------------------------------- many-chain (persistent) path

@pytest.mark.parametrize("dtype,D,L", [(torch.float32, 5120, 250), (torch.float16, 5120, 256),
                                       (torch.float32, 5100, 200)])
def test_persistent_forward_many_chains(mwc, dtype, D, L):
    """B*D/128 >= #SMs: the forward runs as a persistent TMA kernel over a queue of
    (128-channel block, L-segment) units with state hand-off between segments."""
    from mamba_windows_cuda import _lib, _ops
    B = 4
    dt = 1 if dtype == torch.float16 else 0
    assert _lib.load().mwc_ss_fwd_workspace_bytes(B, L, D, dt) > 0
    x = make_inputs(B, L, D, dtype, seed=31 + D + L, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last, ckpt, decay = _ops.ss_forward(*args, x["h_prev"], want_h_last=True,
                                               want_ckpt=True, want_decay=True)
    ref_out, ref_h = oracle_fwd(x, x["h_prev"])
    check = (lambda a, r, w: assert_fp32(a, r, what=w)) if dtype == torch.float32 else \
        (lambda a, r, w: assert_fp16(a, r, w))
    check(out, ref_out, "out")
    check(h_last, ref_h, "h_last")
    k = (L - 1) // 16 // 2
    _, h_k = O.ss_fwd(*[np64(x[n][:, :16 * (k + 1)] if n in ("u", "delta", "Bm", "Cm") else x[n])
                        for n in ("u", "delta", "A", "Bm", "Cm", "Dv")], np64(x["h_prev"]))
    assert_fp32(ckpt[:, k], h_k, tol=1e-4 if dtype == torch.float32 else 1e-2, what="ckpt")
    ref_decay = torch.exp(x["delta"].double().sum(1).unsqueeze(-1) * x["A"].double().unsqueeze(0))
    assert_fp32(decay, ref_decay.cpu().numpy(), tol=1e-4 if dtype == torch.float32 else 1e-2,
                what="decay")
    assert _lib.load().mwc_ss_bwd_workspace_bytes(B, L, D, dt) > 0
    _, _, grads = run_stateful(mwc, x, x["h_prev"], x["gh"])
    ref = oracle_bwd(x, x["h_prev"], x["gh"])
    for k2 in GRADS + ("dh_prev",):
        if dtype == torch.float32:
            assert_fp32(grads[k2], ref[k2], what=k2)
        else:
            scale = max(1.0, float(np.abs(ref[k2]).max()))
            assert_fp16(grads[k2], ref[k2], k2, atol=2e-2 * scale, rtol=1e-2)


@pytest.mark.parametrize("extra,B", [(0, 2), (1, 1), (37, 1)])
def test_persistent_forward_static_runs_edges(mwc, extra, B):
    """The chained forward gives each SM one equal run of the chains' concatenated tiles. With
    exactly one chain per SM no chain is cut (K = 1); with one chain more than the SMs some
    runs are exactly one chain long, so a tail waits for a head finished at the same time;
    with 37 more, runs end and start inside chains throughout. Forward and gradients
    against the float64 oracle, fp32."""
    from mamba_windows_cuda import _ops
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    chains = sms + extra
    if chains % B:
        pytest.skip("chain count not divisible by the batch")
    D, L = chains // B * 128, 512
    plan = _ops.plan(B, L, D, torch.float32)
    assert plan["path"] == "chained" and plan["K"] == (1 if extra == 0 else 2), plan
    x = make_inputs(B, L, D, torch.float32, seed=41 + extra, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last, _, _ = _ops.ss_forward(*args, x["h_prev"], want_h_last=True)
    ref_out, ref_h = oracle_fwd(x, x["h_prev"])
    assert_fp32(out, ref_out, what="out")
    assert_fp32(h_last, ref_h, what="h_last")
    _, _, grads = run_stateful(mwc, x, x["h_prev"], x["gh"])
    ref = oracle_bwd(x, x["h_prev"], x["gh"])
    for k2 in GRADS + ("dh_prev",):
        assert_fp32(grads[k2], ref[k2], what=k2)


@pytest.mark.parametrize("dtype,B,L,D,dist", [(torch.float32, 1, 4096, 2048, "c4"),
                                               (torch.float16, 2, 3000, 640, "c1"),
                                               (torch.bfloat16, 1, 2048, 1024, "c1")])
def test_persistent_forward_few_chains(mwc, dtype, B, L, D, dist):
    """B*D/128 < #SMs: the persistent kernel scans independent L-segments for their end
    states, a fold kernel chains them (segment decay exp(A * sum delta)), and a seeded pass
    writes y, the checkpoints, h_last and the decay. Checked against the oracle, including the
    gradients the backward computes from those checkpoints."""
    from mamba_windows_cuda import _lib, _ops
    dt = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}[dtype]
    assert _lib.load().mwc_ss_fwd_workspace_bytes(B, L, D, dt) > 0
    x = make_inputs(B, L, D, dtype, seed=41 + L, with_state=True, dist=dist, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last, ckpt, decay = _ops.ss_forward(*args, x["h_prev"], want_h_last=True,
                                               want_ckpt=True, want_decay=True)
    ref_out, ref_h = oracle_fwd(x, x["h_prev"])
    f32 = dtype == torch.float32
    tol16 = 2e-2 if dtype == torch.bfloat16 else 1e-2
    check = (lambda a, r, w: assert_fp32(a, r, what=w)) if f32 else \
        (lambda a, r, w: assert_fp16(a, r, w, rtol=tol16))
    check(out, ref_out, "out")
    check(h_last, ref_h, "h_last")
    for k in ((L - 1) // 16 // 3, (L - 1) // 16 - 1):
        _, h_k = O.ss_fwd(*[np64(x[n][:, :16 * (k + 1)] if n in ("u", "delta", "Bm", "Cm") else x[n])
                            for n in ("u", "delta", "A", "Bm", "Cm", "Dv")], np64(x["h_prev"]))
        assert_fp32(ckpt[:, k], h_k, tol=1e-4 if f32 else tol16, what=f"ckpt {k}")
    ref_decay = torch.exp(x["delta"].double().sum(1).unsqueeze(-1) * x["A"].double().unsqueeze(0))
    assert_fp32(decay, ref_decay.cpu().numpy(), tol=1e-4 if f32 else tol16, what="decay")
    _, _, grads = run_stateful(mwc, x, x["h_prev"], x["gh"])
    ref = oracle_bwd(x, x["h_prev"], x["gh"])
    for k2 in GRADS + ("dh_prev",):
        if f32:
            assert_fp32(grads[k2], ref[k2], what=k2)
        else:
            scale = max(1.0, float(np.abs(ref[k2]).max()))
            assert_fp16(grads[k2], ref[k2], k2, atol=2e-2 * scale, rtol=tol16)


def test_persistent_forward_few_chains_deterministic(mwc):
    from mamba_windows_cuda import _ops
    x = make_inputs(1, 4096, 1024, torch.float16, seed=8, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    o1, h1, c1, _ = _ops.ss_forward(*args, x["h_prev"], want_h_last=True, want_ckpt=True)
    o2, h2, c2, _ = _ops.ss_forward(*args, x["h_prev"], want_h_last=True, want_ckpt=True)
    assert torch.equal(o1, o2) and torch.equal(h1, h2) and torch.equal(c1, c2)


def test_persistent_backward_few_chains_deterministic(mwc):
    """Few chains: adjoint-only pass, fold and seeded backward; bitwise repeatable."""
    x = make_inputs(1, 2048, 1024, torch.float16, seed=12, with_state=True, device="cuda")
    _, _, g1 = run_stateful(mwc, x, x["h_prev"], x["gh"])
    _, _, g2 = run_stateful(mwc, x, x["h_prev"], x["gh"])
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_persistent_backward_is_deterministic(mwc):
    x = make_inputs(4, 300, 5120, torch.float16, seed=9, with_state=True, device="cuda")
    _, _, g1 = run_stateful(mwc, x, x["h_prev"], x["gh"])
    _, _, g2 = run_stateful(mwc, x, x["h_prev"], x["gh"])
    for k in g1:
        assert torch.equal(g1[k], g2[k]), k


def test_persistent_forward_is_deterministic_and_ckpt_only(mwc):
    from mamba_windows_cuda import _ops
    x = make_inputs(4, 512, 5120, torch.float16, seed=2, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    o1, h1, c1, _ = _ops.ss_forward(*args, want_h_last=True, want_ckpt=True)
    o2, h2, c2, _ = _ops.ss_forward(*args, want_h_last=True, want_ckpt=True)
    _, h3, c3, _ = _ops.ss_forward(*args, want_out=False, want_h_last=True, want_ckpt=True)
    assert torch.equal(o1, o2) and torch.equal(h1, h2) and torch.equal(c1, c2)
    assert torch.equal(h1, h3) and torch.equal(c1, c3)


@pytest.mark.parametrize("B,L,D,case", [(4, 512, 5120, "posA"), (1, 4096, 512, "posA"),
                                        (4, 512, 5120, "negdelta"), (1, 4096, 512, "negdelta")])
def test_persistent_paths_with_positive_exponents(mwc, B, L, D, case):
    """The clamped copies of the persistent step loops (chosen per tile when some A > 0 or
    some delta < 0 makes an exponent positive): chained segments (160 chains) and the
    few-chain split passes, float32 fwd + bwd against the oracle with the clamp."""
    from mamba_windows_cuda import _ops
    path = _ops.plan(B, L, D, torch.float32)["path"]
    assert path == ("chained" if B * D // 128 >= 148 else "split")
    g = torch.Generator().manual_seed(61)
    x = make_inputs(B, L, D, torch.float32, seed=61, dist="c1", with_state=True)
    if case == "posA":   # small positive A on some states: slow growth, no overflow over L
        x["A"] = -torch.rand(D, 16, generator=g) + 0.02
        x["delta"] = torch.nn.functional.softplus(torch.randn(B, L, D, generator=g) * 0.5 - 2.0)
    else:                # delta of both signs with A < 0
        x["delta"] = torch.randn(B, L, D, generator=g) * 0.02
    x = {k: v.cuda() for k, v in x.items()}
    leaves = [x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    hp = x["h_prev"].clone().requires_grad_(True)
    out, h_last = mwc.SelectiveScanCuda().forward_with_state(*leaves, hp)
    (out * x["g"]).sum().backward()
    torch.cuda.synchronize()
    n = [np64(t) for t in leaves]
    o64, h64 = O.ss_fwd(*n, np64(hp), clamp=True)
    g64 = O.ss_bwd(*n, np64(x["g"]), np64(hp), None, clamp=True)
    assert_fp32(out, o64, what="out")
    assert_fp32(h_last, h64, what="h_last")
    for name, t in zip(("du", "ddelta", "dA", "dB", "dC", "dD"), leaves):
        assert_fp32(t.grad, g64[name], what=name)
    assert_fp32(hp.grad, g64["dh_prev"], what="dh_prev")


@pytest.mark.parametrize("B,L,D", [(4, 512, 5064), (1, 2048, 1000)])
def test_persistent_fp16_partial_channel_block(mwc, B, L, D):
    """D not a multiple of 128 (the last 128-channel block partial) on the persistent
    kernels in float16: chained segments (160 chains) and the few-chain split passes, fwd +
    bwd against the oracle (per-element results elementwise atol 2e-2 / rtol 1e-2, the sums
    dA / dB / dC / dD with atol scaled by their magnitude)."""
    from mamba_windows_cuda import _ops
    assert _ops.plan(B, L, D, torch.float16)["path"] != "generic"
    x = make_inputs(B, L, D, torch.float16, seed=67, dist="c3", with_state=True, device="cuda")
    leaves = [x[k].clone().requires_grad_(True) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    hp = x["h_prev"].clone().requires_grad_(True)
    out, h_last = mwc.SelectiveScanCuda().forward_with_state(*leaves, hp)
    (out * x["g"]).sum().backward()
    torch.cuda.synchronize()
    n = [np64(t) for t in leaves]
    o64, h64 = O.ss_fwd(*n, np64(hp))
    g64 = O.ss_bwd(*n, np64(x["g"]), np64(hp), None)
    assert_fp16(out, o64, what="out")
    assert_fp16(h_last, h64, what="h_last")
    for name, t in zip(("du", "ddelta"), leaves[:2]):
        assert_fp16(t.grad, g64[name], what=name)
    for name, t in zip(("dA", "dB", "dC", "dD"), leaves[2:]):
        ref = g64[name]
        assert_fp16(t.grad, ref, what=name, atol=2e-2 * max(1.0, float(np.abs(ref).max())))
    assert_fp16(hp.grad, g64["dh_prev"], what="dh_prev")
