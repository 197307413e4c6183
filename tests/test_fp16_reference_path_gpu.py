"""float16 accuracy against the reference's own float16 PyTorch path, on identical inputs.

The reference's float16 CUDA backward cannot be run as a comparator (its kernels call
__shfl_sync with a member mask that leaves out lanes that execute it), so the float16
result of the reference's algorithm is taken from its PyTorch path: selective_scan_ref
(mamba_windows_cuda/mamba_cuda.py:875-946, the einsum axis fixed) evaluated in float16 on
the GPU, with torch autograd for the gradients. Both it and this library's kernels are
compared with the float64 oracle on the same float16 inputs, output by output, as
max |x - ref| / max |ref|.

The check: this library's error is no larger than the reference path's (plus a floor of one
float16 rounding, 2^-11), for every output and gradient, the sums dA / dB / dC / dD
included. The float16 reductions need the atol scaled by max|ref| that the parity tests
use; this test shows the reference's own float16 path needs it as well.
"""
import numpy as np
import pytest
import torch

from _helpers import make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu

KEYS = ("u", "delta", "A", "Bm", "Cm", "Dv")
GRADS = ("du", "ddelta", "dA", "dB", "dC", "dD")
FLOOR = 2.0 ** -11


def _err(x, ref):
    x = x.detach().double().cpu().numpy()
    return float(np.abs(x - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("B,L,D", [(2, 512, 128), (1, 1024, 256)])
def test_fp16_errors_no_larger_than_reference_fp16_path(B, L, D):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    import mamba_windows_cuda as mwc
    from mamba_windows_cuda.mamba_cuda import selective_scan_ref
    x = make_inputs(B, L, D, torch.float16, seed=83, dist="c3", with_state=True, device="cuda")
    g = x["g"]

    def run(fn):
        leaves = [x[k].clone().requires_grad_(True) for k in KEYS]
        hp = x["h_prev"].clone().requires_grad_(True)
        out, h_last = fn(*leaves, hp)
        (out.float() * g.float()).sum().backward()
        torch.cuda.synchronize()
        return out, h_last, [t.grad for t in leaves], hp.grad

    ours = run(mwc.SelectiveScanCuda().forward_with_state)
    theirs = run(selective_scan_ref)
    n = [np64(x[k]) for k in KEYS]
    o64, h64 = O.ss_fwd(*n, np64(x["h_prev"]))
    g64 = O.ss_bwd(*n, np64(g), np64(x["h_prev"]), None)
    refs = [("out", o64), ("h_last", h64)] + [(k, g64[k]) for k in GRADS] + [("dh_prev", g64["dh_prev"])]
    got_ours = [ours[0], ours[1]] + ours[2] + [ours[3]]
    got_theirs = [theirs[0], theirs[1]] + theirs[2] + [theirs[3]]
    for (name, ref), a, b in zip(refs, got_ours, got_theirs):
        e_ours, e_ref = _err(a, ref), _err(b, ref)
        print(f"({B},{L},{D}) {name}: this library {e_ours:.2e}, reference float16 path {e_ref:.2e}")
        assert e_ours <= e_ref + FLOOR, (f"{name}: this library {e_ours:.3e} vs the reference's "
                                         f"float16 path {e_ref:.3e} (relative to max|ref|)")
