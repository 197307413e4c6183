"""Causal conv1d on the GPU (mwc_conv1d_fwd / _bwd through causal_conv1d_fn) against the
plain-PyTorch definition run in float64 on CPU: y and the gradients dx, dweight, dbias,
dx_prev, for widths 1-4, both activations, float32 / float16 / bfloat16, the TMA-staged path
(rows a multiple of 16 bytes, aligned) and the element path, lengths that are not a multiple
of the 64-step tile, channel counts that end inside a channel block, and chunked streaming.
At the benchmark's shape (4 x 2048 x 5120, several ring passes per CTA) the reference is the
same definition in float32 on the GPU.

Tolerance: float32 normwise 1e-5; float16 / bfloat16 elementwise atol 2e-2 * max|ref| +
rtol 1e-2 (2e-2 for bf16) * |ref| (one rounding of each result to the I/O type)."""
import numpy as np
import pytest
import torch

from mamba_windows_cuda.causal_conv1d import causal_conv1d_fn, causal_conv1d_ref, conv_state

pytestmark = pytest.mark.gpu


def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")


def check(x, ref, dtype, what):
    xv = x.detach().double().cpu().numpy()
    rv = ref.detach().double().cpu().numpy()
    if dtype == torch.float32:
        e = np.abs(xv - rv).max() / max(np.abs(rv).max(), 1e-30)
        assert e < 1e-5, f"{what}: normwise error {e:.3e}"
        return
    rtol = 1e-2 if dtype == torch.float16 else 2e-2
    bad = np.abs(xv - rv) > 2e-2 * max(np.abs(rv).max(), 1e-30) + rtol * np.abs(rv)
    assert not bad.any(), f"{what}: {int(bad.sum())} of {bad.size} outside; max {np.abs(xv - rv).max():.3e}"


CASES = [
    (torch.float32, 2, 200, 64, 4, "silu", True),
    (torch.float32, 2, 200, 37, 4, "silu", True),     # element path
    (torch.float32, 1, 64, 16, 3, None, False),
    (torch.float32, 3, 10, 8, 2, "silu", True),       # shorter than one run
    (torch.float32, 2, 130, 24, 1, None, False),
    (torch.float16, 2, 300, 128, 4, "silu", True),
    (torch.bfloat16, 2, 300, 128, 4, "silu", False),
    (torch.float16, 1, 129, 40, 3, "silu", True),
]


@pytest.mark.parametrize("dtype,B,L,D,W,act,with_prev", CASES)
def test_conv1d(dtype, B, L, D, W, act, with_prev):
    _need_gpu()
    g = torch.Generator().manual_seed(L + D + W)
    x = torch.randn(B, L, D, generator=g)
    w = torch.randn(D, W, generator=g) * 0.5
    b = torch.randn(D, generator=g) * 0.1
    xp = torch.randn(B, W - 1, D, generator=g) if with_prev and W > 1 else None
    dy = torch.randn(B, L, D, generator=g)
    dev = [t.to(dtype).cuda().requires_grad_(True) if t is not None else None for t in (x, w, b, xp)]
    y = causal_conv1d_fn(dev[0], dev[1], dev[2], act, dev[3])
    y.backward(dy.to(dtype).cuda())
    # float64 reference on the same (rounded) inputs
    ref_in = [t.detach().double().cpu().requires_grad_(True) if t is not None else None for t in dev]
    yr = causal_conv1d_ref(ref_in[0], ref_in[1], ref_in[2], act, ref_in[3])
    yr.backward(dy.to(dtype).double())
    check(y, yr, dtype, "y")
    for name, a, r in zip(("dx", "dweight", "dbias", "dx_prev"), dev, ref_in):
        if a is not None:
            check(a.grad, r.grad, dtype, name)


def test_conv1d_streaming_chunks():
    _need_gpu()
    g = torch.Generator().manual_seed(3)
    x = torch.randn(2, 300, 64, generator=g).cuda()
    w = torch.randn(64, 4, generator=g).cuda()
    y = causal_conv1d_fn(x, w, None, "silu")
    y1 = causal_conv1d_fn(x[:, :170].contiguous(), w, None, "silu")
    y2 = causal_conv1d_fn(x[:, 170:].contiguous(), w, None, "silu", conv_state(x[:, :170], 4).contiguous())
    assert torch.allclose(torch.cat([y1, y2], 1), y, atol=1e-5, rtol=1e-5)


def test_conv1d_full_size_fp16():
    """Benchmark shape: 40 channel blocks x 128 tiles, so each CTA passes its ring several times."""
    _need_gpu()
    g = torch.Generator(device="cuda").manual_seed(11)
    Bb, L, D, W = 4, 2048, 5120, 4
    x = torch.randn(Bb, L, D, generator=g, device="cuda").half()
    w = (torch.randn(D, W, generator=g, device="cuda") * 0.5).half()
    b = (torch.randn(D, generator=g, device="cuda") * 0.1).half()
    xp = torch.randn(Bb, W - 1, D, generator=g, device="cuda").half()
    dy = torch.randn(Bb, L, D, generator=g, device="cuda").half()
    dev = [t.clone().requires_grad_(True) for t in (x, w, b, xp)]
    y = causal_conv1d_fn(dev[0], dev[1], dev[2], "silu", dev[3])
    y.backward(dy)
    ref = [t.float().requires_grad_(True) for t in (x, w, b, xp)]
    yr = causal_conv1d_ref(ref[0], ref[1], ref[2], "silu", ref[3])
    yr.backward(dy.float())
    check(y, yr, torch.float16, "y")
    for name, a, r in zip(("dx", "dweight", "dbias", "dx_prev"), dev, ref):
        check(a.grad, r.grad, torch.float16, name)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16])
def test_conv1d_paths_agree(dtype):
    """The TMA-staged path (aligned rows) and the element path (x one element off a 16-byte
    boundary) compute each y and dx element with the same operations: bitwise equal. dweight /
    dbias sum in a different order: close."""
    _need_gpu()
    g = torch.Generator(device="cuda").manual_seed(12)
    Bb, L, D, W = 2, 333, 264, 4
    x = torch.randn(Bb, L, D, generator=g, device="cuda").to(dtype)
    w = (torch.randn(D, W, generator=g, device="cuda") * 0.5).to(dtype)
    b = (torch.randn(D, generator=g, device="cuda") * 0.1).to(dtype)
    xp = torch.randn(Bb, W - 1, D, generator=g, device="cuda").to(dtype)
    dy = torch.randn(Bb, L, D, generator=g, device="cuda").to(dtype)
    outs = []
    for off in (0, 1):
        store = torch.empty(Bb * L * D + off, dtype=dtype, device="cuda")
        xv = store[off:].view(Bb, L, D)
        xv.copy_(x)
        assert (xv.data_ptr() % 16 == 0) == (off == 0)
        xl = xv.detach().requires_grad_(True)
        wl, bl, pl = (t.clone().requires_grad_(True) for t in (w, b, xp))
        y = causal_conv1d_fn(xl, wl, bl, "silu", pl)
        y.backward(dy)
        outs.append((y.detach(), xl.grad, pl.grad, wl.grad, bl.grad))
    for name, a, c in zip(("y", "dx", "dx_prev"), outs[0][:3], outs[1][:3]):
        assert torch.equal(a, c), name
    for name, a, c in zip(("dweight", "dbias"), outs[0][3:], outs[1][3:]):
        check(a, c.double(), dtype, name)


def test_conv1d_backward_deterministic():
    _need_gpu()
    g = torch.Generator(device="cuda").manual_seed(13)
    x = torch.randn(3, 1500, 1000, generator=g, device="cuda").half()
    w = torch.randn(1000, 4, generator=g, device="cuda").half()
    b = torch.randn(1000, generator=g, device="cuda").half()
    dy = torch.randn(3, 1500, 1000, generator=g, device="cuda").half()
    grads = []
    for _ in range(2):
        wl, bl = w.clone().requires_grad_(True), b.clone().requires_grad_(True)
        causal_conv1d_fn(x, wl, bl, "silu").backward(dy)
        grads.append((wl.grad, bl.grad))
    assert torch.equal(grads[0][0], grads[1][0]) and torch.equal(grads[0][1], grads[1][1])
