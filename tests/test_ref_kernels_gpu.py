"""Forward parity against the reference's own CUDA kernel (selective_scan_fwd_kernel_v4 behind
selective_scan_cuda_forward_with_state, mamba_windows_cuda/mamba_cuda.py:93-174 and
:271-359), built from the reference's source by oracle/build_ref.py, on identical seeded
inputs. Both results are also checked against the float64 oracle.

Tolerances: fp16 elementwise atol 2e-2 / rtol 1e-2 between this
library's fp16 result and the reference kernel's fp16 result, and each against float64 on
the same fp16 inputs; fp32 normwise 1e-4.

Only the reference's forward kernel runs here. Its other kernels (the store-forward and both
backward kernels, mamba_cuda.py:364-562 and :611-745) call __shfl_sync with the member mask
0xFFFF from all 32 lanes of a warp, lanes 16-31 outside the mask: undefined behaviour that
may hang a GPU, so the gradient parity stays against the float64 oracle. The forward kernel
returns before a __syncthreads when D is not a multiple of its 8 warps per block, so every
shape here has D % 8 == 0.
"""
import os
import sys

import pytest
import torch

from _helpers import assert_fp16, assert_fp32, make_inputs, np64
from oracle import oracle as O

pytestmark = pytest.mark.gpu

KEYS = ("u", "delta", "A", "Bm", "Cm", "Dv")


@pytest.fixture(scope="module")
def ref():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle"))
    import build_ref
    mod = build_ref.load()
    if mod is None:
        pytest.skip("reference module not built (python oracle/build_ref.py REFERENCE_ROOT)")
    return mod


CASES = [
    # (B, L, D, dtype, dist, with h_prev)
    (1, 1024, 256, torch.float16, "c1", True),     # config 1 shape
    (8, 2048, 4096, torch.float16, "c2", False),   # config 2 (inference, h0 = 0)
    (4, 2048, 5120, torch.float16, "c3", True),    # config 3 shape, h_prev ~ N(0, 0.1)
    (1, 1024, 256, torch.float32, "c1", True),
]


@pytest.mark.parametrize("B,L,D,dtype,dist,state", CASES)
def test_forward_matches_reference_kernel(ref, B, L, D, dtype, dist, state):
    import mamba_windows_cuda as mwc
    x = make_inputs(B, L, D, dtype, seed=71 + L + D, dist=dist, with_state=state, device="cuda")
    args = [x[k] for k in KEYS]
    hp = x["h_prev"] if state else None
    with torch.no_grad():
        out, h_last = mwc.SelectiveScanCuda().forward_with_state(*args, hp)
    r_out, r_h = ref.selective_scan_cuda_forward_with_state(*args, hp)
    torch.cuda.synchronize()
    o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(hp))
    if dtype == torch.float16:
        assert r_out.dtype == torch.float16 and r_h.dtype == torch.float16
        assert_fp16(out, r_out.double().cpu().numpy(), "out vs the reference kernel")
        assert_fp16(h_last, r_h.double().cpu().numpy(), "h_last vs the reference kernel")
        assert_fp16(out, o64, "out vs float64")
        assert_fp16(h_last, h64, "h_last vs float64")
        assert_fp16(r_out, o64, "reference kernel out vs float64")
        assert_fp16(r_h, h64, "reference kernel h_last vs float64")
    else:
        assert_fp32(out, r_out.double().cpu().numpy(), what="out vs the reference kernel")
        assert_fp32(h_last, r_h.double().cpu().numpy(), what="h_last vs the reference kernel")
        assert_fp32(out, o64, what="out vs float64")
        assert_fp32(r_out, o64, what="reference kernel out vs float64")
