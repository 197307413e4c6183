"""The reference's op-module handle (mamba_windows_cuda/mamba_cuda.py:835-872,
:1106-1111, :1185-1188): callers that reach the host ops through
``_get_selective_scan_cuda_module()`` or ``SelectiveScanCuda()._get_module()`` get the five
entry points (declarations at mamba_cuda.py:793-830), checked here against the float64
oracle (fp32 tolerance: normwise 1e-4)."""
import pytest
import torch

from _helpers import assert_fp32, make_inputs, np64
from oracle import oracle as O

KEYS = ("u", "delta", "A", "Bm", "Cm", "Dv")
GRADS = ("du", "ddelta", "dA", "dB", "dC", "dD")


def test_module_handle_has_reference_entry_points():
    from mamba_windows_cuda import SelectiveScanCuda
    from mamba_windows_cuda.mamba_cuda import (SelectiveScanFn, SelectiveScanFnV2,
                                               _get_selective_scan_cuda_module)
    mod = _get_selective_scan_cuda_module()
    for name in ("selective_scan_cuda_forward", "selective_scan_cuda_forward_with_state",
                 "selective_scan_cuda_backward", "selective_scan_cuda_forward_store",
                 "selective_scan_cuda_backward_direct"):
        assert callable(getattr(mod, name)), name
    assert SelectiveScanCuda()._get_module() is mod
    assert SelectiveScanFn._get_module() is mod and SelectiveScanFnV2._get_module() is mod


@pytest.mark.gpu
def test_module_entry_points_match_oracle():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA GPU")
    from mamba_windows_cuda.mamba_cuda import _get_selective_scan_cuda_module
    mod = _get_selective_scan_cuda_module()
    x = make_inputs(2, 300, 96, torch.float32, seed=61, with_state=True, device="cuda")
    args = [x[k] for k in KEYS]
    n64 = [np64(t) for t in args]
    ref_out0, _ = O.ss_fwd(*n64)
    ref_out, ref_h = O.ss_fwd(*n64, np64(x["h_prev"]))
    assert_fp32(mod.selective_scan_cuda_forward(*args, None), ref_out0, what="forward")
    out, h_last = mod.selective_scan_cuda_forward_with_state(*args, x["h_prev"])
    assert_fp32(out, ref_out, what="forward_with_state out")
    assert_fp32(h_last, ref_h, what="forward_with_state h_last")
    ref = O.ss_bwd(*n64, np64(x["g"]))
    g1 = mod.selective_scan_cuda_backward(*args, x["g"])
    out2, bank = mod.selective_scan_cuda_forward_store(*args)
    assert_fp32(out2, ref_out0, what="forward_store out")
    g2 = mod.selective_scan_cuda_backward_direct(*args, x["g"], bank)
    for k, a, b in zip(GRADS, g1, g2):
        assert_fp32(a, ref[k], what=f"backward {k}")
        assert torch.equal(a, b), k   # same kernels, same checkpoints: bitwise equal
    with pytest.raises(RuntimeError):
        mod.selective_scan_cuda_backward_direct(*args, x["g"], bank[:, :1])
    with pytest.raises(RuntimeError):
        mod.selective_scan_cuda_forward(x["u"].cpu(), *args[1:], None)
