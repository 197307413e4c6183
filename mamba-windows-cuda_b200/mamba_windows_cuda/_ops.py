"""Tensor-level wrappers around the C ABI: validation, allocation, stream and device.

Every tensor (outputs and workspaces) is allocated here with the PyTorch caching
allocator and handed to libmwc_b200.so as a raw pointer together with
``torch.cuda.current_stream()``; the library itself allocates nothing.

Validation mirrors the reference's host checks (mamba_windows_cuda/mamba_cuda.py:186-238)
and raises RuntimeError with the same messages.
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib

NSTATE = 16
CK = 16

_DTYPES = {torch.float32: _lib.MWC_F32, torch.float16: _lib.MWC_F16,
           torch.bfloat16: _lib.MWC_BF16}


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPES[t.dtype]
    except KeyError:
        raise RuntimeError("u must be float32/float16/bfloat16") from None


def _p(t):
    # a plain int: the entry points declare c_void_p arguments, which take ints and None
    return None if t is None else t.data_ptr()


# MWC_CHECK_WAITS=1: after every forward / backward call, wait for the stream and raise if a
# bounded device wait of the persistent kernel gave up (costs a synchronisation per call).
CHECK_WAITS = os.environ.get("MWC_CHECK_WAITS", "0") == "1"


def _check_waits(lib, dev, what):
    if CHECK_WAITS:
        _lib.check(lib.mwc_check_last_launch(_stream(dev)), what)


def _index(device) -> int:
    return device.index if device.index is not None else torch._C._cuda_getDevice()


def _stream(device) -> int:
    """The raw cudaStream_t of the current stream of ``device`` (what
    torch.cuda.current_stream(device).cuda_stream returns, without building the Stream
    object: this is on every call's path)."""
    return torch._C._cuda_getCurrentRawStream(_index(device))


_WS_BYTES = {}


def _ws_bytes(lib, name, *shape):
    """Workspace bytes of an entry point for a shape on the current device, queried once:
    the sizes depend only on the shape and the device's SM count."""
    key = (name, torch._C._cuda_getDevice()) + shape
    v = _WS_BYTES.get(key)
    if v is None:
        v = _WS_BYTES[key] = int(getattr(lib, name)(*shape))
    return v


class _on_device:
    """Make ``device`` the current CUDA device for the block (torch.cuda.device's exchange,
    without its argument normalisation; a no-op exchange when it already is current)."""
    __slots__ = ("idx", "prev")

    def __init__(self, device):
        self.idx = _index(device)

    def __enter__(self):
        self.prev = torch._C._cuda_exchangeDevice(self.idx)

    def __exit__(self, *exc):
        torch._C._cuda_maybeExchangeDevice(self.prev)
        return False


def check_ss_inputs(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None):
    """The reference's TORCH_CHECKs for the selective-scan forward (mamba_cuda.py:186-238)."""
    named = (("u", u), ("delta", delta), ("A", A), ("B_ssm", B_ssm), ("C_ssm", C_ssm),
             ("D_ssm", D_ssm))
    for name, t in named:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
    if u.dtype not in _DTYPES:
        raise RuntimeError("u must be float32/float16/bfloat16")
    for name, t in named[1:]:
        if t.dtype != u.dtype:
            raise RuntimeError(f"{name} dtype must match u dtype")
    if u.dim() != 3:
        raise RuntimeError("u must be 3D (batch, seqlen, dim)")
    if A.dim() != 2:
        raise RuntimeError("A must be 2D (dim, state)")
    Bb, L, D = u.shape
    N = A.size(1)
    if N != NSTATE:
        raise RuntimeError("Only N=16 is supported")
    if delta.dim() != 3:
        raise RuntimeError("delta must be 3D (batch, seqlen, dim)")
    if B_ssm.dim() != 3:
        raise RuntimeError("B_ssm must be 3D (batch, seqlen, state)")
    if C_ssm.dim() != 3:
        raise RuntimeError("C_ssm must be 3D (batch, seqlen, state)")
    if D_ssm.dim() != 1:
        raise RuntimeError("D_ssm must be 1D (dim)")
    if tuple(delta.shape) != (Bb, L, D):
        raise RuntimeError("delta shape mismatch")
    if tuple(A.shape) != (D, N):
        raise RuntimeError("A shape mismatch")
    if tuple(B_ssm.shape) != (Bb, L, N):
        raise RuntimeError("B_ssm shape mismatch")
    if tuple(C_ssm.shape) != (Bb, L, N):
        raise RuntimeError("C_ssm shape mismatch")
    if tuple(D_ssm.shape) != (D,):
        raise RuntimeError("D_ssm shape mismatch")
    if h_prev is not None:
        if not isinstance(h_prev, torch.Tensor) or not h_prev.is_cuda:
            raise RuntimeError("h_prev must be a CUDA tensor")
        if h_prev.dtype != u.dtype:
            raise RuntimeError("h_prev dtype must match u dtype")
        if h_prev.dim() != 3:
            raise RuntimeError("h_prev must be 3D (batch, dim, state)")
        if tuple(h_prev.shape) != (Bb, D, N):
            raise RuntimeError("h_prev shape must be (B, D, N)")
    dev = u.device
    for name, t in named + (("h_prev", h_prev),):
        if t is not None and t.device != dev:
            raise RuntimeError(f"{name} must be on the same device as u")


def ckpt_count(L: int) -> int:
    return (L + CK - 1) // CK


PATHS = {0: "generic", 1: "chained", 2: "split"}


def plan(B: int, L: int, D: int, dtype: torch.dtype, backward: bool = False) -> dict:
    """The launch plan the forward (or backward) picks for (B, L, D) on the current device,
    for 16-byte-aligned buffers (mwc_ss_plan): path ("chained": persistent kernel over
    chained 128-channel chains; "split": independent segments + fold; "generic": the
    non-TMA kernels), K, seg, CTAs. Chained forward: one run of the chains' concatenated
    32-step tiles per CTA, seg = the longest run, K = 2 when a run boundary cuts a chain
    (else 1). Chained backward and split paths: K time segments of seg tiles per chain."""
    lib = _lib.load()
    info = (ctypes.c_int32 * 4)()
    _lib.check(lib.mwc_ss_plan(B, L, D, _DTYPES[dtype], int(bool(backward)), info), "plan query")
    return {"path": PATHS[info[0]], "K": info[1], "seg": info[2], "grid": info[3]}


def ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None, *, want_out=True,
               want_h_last=False, want_ckpt=False, want_decay=False, dprefix=None):
    """Run the forward scan. Inputs must be contiguous and validated.

    Returns (out, h_last, ckpt, decay); entries not requested are None. ``dprefix``: a float32
    (B, mwc_ss_dprefix_count(L), D, 2) buffer to receive the delta prefix records of a
    sequence-sharded local scan (mwc_ss_fwd_seq; needs want_decay and the persistent path).
    """
    Bb, L, D = u.shape
    N = A.shape[1]   # 16 everywhere except the N = 32 / 64 forward (mwc_ss_fwd_nstate)
    dev = u.device
    out = torch.empty_like(u) if want_out else None
    h_last = torch.empty((Bb, D, N), dtype=u.dtype, device=dev) if want_h_last else None
    ckpt = (torch.empty((Bb, ckpt_count(L), D, N), dtype=torch.float32, device=dev)
            if want_ckpt else None)
    decay = (torch.empty((Bb, D, N), dtype=torch.float32, device=dev)
             if want_decay else None)
    if L == 0 or Bb == 0 or D == 0:
        if h_last is not None:
            h_last.copy_(h_prev) if h_prev is not None else h_last.zero_()
        if decay is not None:
            decay.fill_(1.0)
        return out, h_last, ckpt, decay
    lib = _lib.load()
    dt = dtype_code(u)
    with _on_device(dev):
        if N != NSTATE:
            ws_bytes = _ws_bytes(lib, "mwc_ss_fwd_nstate_workspace_bytes", Bb, L, D, N, dt)
        else:
            ws_bytes = _ws_bytes(lib, "mwc_ss_fwd_workspace_bytes", Bb, L, D, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
        if N != NSTATE:
            rc = lib.mwc_ss_fwd_nstate(_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm),
                                       _p(h_prev), _p(out), _p(h_last), _p(ckpt), _p(decay), _p(ws),
                                       ws_bytes, Bb, L, D, N, dt, _stream(dev))
        elif dprefix is not None:
            rc = lib.mwc_ss_fwd_seq(_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm),
                                    _p(h_prev), _p(out), _p(h_last), _p(ckpt), _p(decay), _p(dprefix),
                                    _p(ws), ws_bytes, Bb, L, D, dt, _stream(dev))
        elif B_ssm.dim() == 4:   # grouped B / C (B, L, G, 16)
            rc = lib.mwc_ss_fwd_grouped(_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm),
                                        _p(h_prev), _p(out), _p(h_last), _p(ckpt), _p(decay), _p(ws),
                                        ws_bytes, Bb, L, D, B_ssm.shape[2], dt, _stream(dev))
        else:
            rc = lib.mwc_ss_fwd(_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm),
                                _p(h_prev), _p(out), _p(h_last), _p(ckpt), _p(decay), _p(ws),
                                ws_bytes, Bb, L, D, dt, _stream(dev))
    _lib.check(rc, "selective_scan forward")
    _check_waits(lib, dev, "selective_scan forward")
    return out, h_last, ckpt, decay


def ss_backward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, dout, dh_last, ckpt,
                want_dh_prev=False, carry32=False):
    """Reverse scan. dout (B,L,D) and dh_last (B,D,16) may be None (zero).

    Returns (du, ddelta, dA, dB, dC, dD, dh_prev) in the input dtype. With ``carry32``
    (mwc_ss_bwd_seq, the sequence-sharded backward) h_prev, dh_last and dh_prev are float32.
    """
    Bb, L, D = u.shape
    dev = u.device
    if dout is None:
        dout = torch.zeros_like(u)
    du = torch.empty_like(u)
    ddelta = torch.empty_like(delta)
    dA = torch.empty_like(A)
    dB = torch.empty_like(B_ssm)
    dC = torch.empty_like(C_ssm)
    dD = torch.empty_like(D_ssm)
    carry_dtype = torch.float32 if carry32 else u.dtype
    dh_prev = torch.empty((Bb, D, NSTATE), dtype=carry_dtype, device=dev) if want_dh_prev else None
    if L == 0 or Bb == 0 or D == 0:
        for t in (du, ddelta, dA, dB, dC, dD):
            t.zero_()
        if dh_prev is not None:
            dh_prev.copy_(dh_last) if dh_last is not None else dh_prev.zero_()
        return du, ddelta, dA, dB, dC, dD, dh_prev
    lib = _lib.load()
    dt = dtype_code(u)
    with _on_device(dev):
        ws_bytes = _ws_bytes(lib, "mwc_ss_bwd_workspace_bytes", Bb, L, D, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        args = (_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm), _p(h_prev), _p(dout),
                _p(dh_last), _p(ckpt), _p(du), _p(ddelta), _p(dA), _p(dB), _p(dC), _p(dD),
                _p(dh_prev), _p(ws), ws_bytes, Bb, L, D)
        if B_ssm.dim() == 4:   # grouped B / C: dB, dC (B, L, G, 16)
            rc = lib.mwc_ss_bwd_grouped(*args, B_ssm.shape[2], dt, _stream(dev))
        elif carry32:
            rc = lib.mwc_ss_bwd_seq(*args, dt, _stream(dev))
        else:
            rc = lib.mwc_ss_bwd(*args, dt, _stream(dev))
    _lib.check(rc, "selective_scan backward")
    _check_waits(lib, dev, "selective_scan backward")
    return du, ddelta, dA, dB, dC, dD, dh_prev


def ss_adjoint(delta, A, C_ssm, dout, q_in=None):
    """Adjoint state at the start of a time range (mwc_ss_adjoint_seq): float32 (B, D, 16),
    from the adjoint ``q_in`` (float32, or None for zero) entering at the range end and the
    range's output gradient ``dout``."""
    Bb, L, D = delta.shape
    dev = delta.device
    q_out = torch.empty((Bb, D, NSTATE), dtype=torch.float32, device=dev)
    if L == 0 or Bb == 0 or D == 0:
        q_out.copy_(q_in) if q_in is not None else q_out.zero_()
        return q_out
    lib = _lib.load()
    dt = dtype_code(delta)
    with _on_device(dev):
        ws_bytes = _ws_bytes(lib, "mwc_ss_adjoint_seq_workspace_bytes", Bb, L, D)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        rc = lib.mwc_ss_adjoint_seq(_p(delta), _p(A), _p(C_ssm), _p(dout), _p(q_in), _p(q_out), _p(ws),
                                    ws_bytes, Bb, L, D, dt, _stream(dev))
    _lib.check(rc, "selective_scan range adjoint")
    return q_out


def ss_forward_ex(u, delta, A, B_ssm, C_ssm, D_ssm, z=None, delta_bias=None,
                  delta_softplus=False, h_prev=None, *, want_h_last=False, want_ckpt=False):
    """Forward scan with the delta transform (bias, softplus) and the z gate
    (mwc_ss_fwd_ex). Returns (out, out_z, h_last, ckpt): out is the ungated scan output,
    out_z = out * silu(z) when z is given (else None)."""
    Bb, L, D = u.shape
    dev = u.device
    out = torch.empty_like(u)
    out_z = torch.empty_like(u) if z is not None else None
    h_last = torch.empty((Bb, D, NSTATE), dtype=u.dtype, device=dev) if want_h_last else None
    ckpt = (torch.empty((Bb, ckpt_count(L), D, NSTATE), dtype=torch.float32, device=dev)
            if want_ckpt else None)
    if L == 0 or Bb == 0 or D == 0:
        if h_last is not None:
            h_last.copy_(h_prev) if h_prev is not None else h_last.zero_()
        return out, out_z, h_last, ckpt
    lib = _lib.load()
    dt = dtype_code(u)
    with _on_device(dev):
        ws_bytes = _ws_bytes(lib, "mwc_ss_fwd_ex_workspace_bytes", Bb, L, D, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev) if ws_bytes > 0 else None
        rc = lib.mwc_ss_fwd_ex(_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm), _p(z),
                               _p(delta_bias), int(bool(delta_softplus)), _p(h_prev), _p(out),
                               _p(out_z), _p(h_last), _p(ckpt), _p(ws), ws_bytes, Bb, L, D, dt,
                               _stream(dev))
    _lib.check(rc, "selective_scan forward (extended)")
    _check_waits(lib, dev, "selective_scan forward (extended)")
    return out, out_z, h_last, ckpt


def ss_backward_ex(u, delta, A, B_ssm, C_ssm, D_ssm, z, delta_bias, delta_softplus, h_prev,
                   out, dout, dh_last, ckpt, want_dbias=False, want_dh_prev=False):
    """Reverse scan with the delta transform and the z gate (mwc_ss_bwd_ex). dout is the
    gradient of out_z when z is given, else of out. Returns
    (du, ddelta, dA, dB, dC, dD, ddelta_bias, dz, dh_prev); unrequested entries are None."""
    Bb, L, D = u.shape
    dev = u.device
    if dout is None:
        dout = torch.zeros_like(u)
    du = torch.empty_like(u)
    ddelta = torch.empty_like(delta)
    dA = torch.empty_like(A)
    dB = torch.empty_like(B_ssm)
    dC = torch.empty_like(C_ssm)
    dD = torch.empty_like(D_ssm)
    dbias = torch.empty(D, dtype=u.dtype, device=dev) if want_dbias else None
    dz = torch.empty_like(u) if z is not None else None
    dh_prev = torch.empty((Bb, D, NSTATE), dtype=u.dtype, device=dev) if want_dh_prev else None
    if L == 0 or Bb == 0 or D == 0:
        for t in (du, ddelta, dA, dB, dC, dD, dbias, dz):
            if t is not None:
                t.zero_()
        if dh_prev is not None:
            dh_prev.copy_(dh_last) if dh_last is not None else dh_prev.zero_()
        return du, ddelta, dA, dB, dC, dD, dbias, dz, dh_prev
    lib = _lib.load()
    dt = dtype_code(u)
    with _on_device(dev):
        ws_bytes = _ws_bytes(lib, "mwc_ss_bwd_ex_workspace_bytes", Bb, L, D, dt)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        rc = lib.mwc_ss_bwd_ex(_p(u), _p(delta), _p(A), _p(B_ssm), _p(C_ssm), _p(D_ssm), _p(z),
                               _p(delta_bias), int(bool(delta_softplus)), _p(h_prev), _p(out),
                               _p(dout), _p(dh_last), _p(ckpt), _p(du), _p(ddelta), _p(dA),
                               _p(dB), _p(dC), _p(dD), _p(dbias), _p(dz), _p(dh_prev), _p(ws),
                               ws_bytes, Bb, L, D, dt, _stream(dev))
    _lib.check(rc, "selective_scan backward (extended)")
    _check_waits(lib, dev, "selective_scan backward (extended)")
    return du, ddelta, dA, dB, dC, dD, dbias, dz, dh_prev


def dprefix_count(L: int) -> int:
    """Delta prefix records per channel of a sequence-sharded local scan (one per 32 steps)."""
    return (L + 31) // 32


def ss_fixup(delta, A, C_ssm, h_in, decay=None, out=None, h_last=None, ckpt=None, dprefix=None):
    """Fold an incoming float32 state h_in (B, D, 16) into a scan run from zero, in place.
    With the local scan's ``dprefix`` records the time range is processed in parallel chunks
    that are skipped once h_in has decayed (mwc_ss_fixup_chunked); without them, one pass
    per channel that stops at the decay horizon (mwc_ss_fixup)."""
    Bb, L, D = delta.shape
    if L == 0 or Bb == 0 or D == 0:
        if h_last is not None and decay is not None:
            h_last.copy_((decay * h_in + h_last.float()).to(h_last.dtype))
        return
    lib = _lib.load()
    dt = dtype_code(delta)
    dev = delta.device
    with _on_device(dev):
        if dprefix is not None:
            rc = lib.mwc_ss_fixup_chunked(_p(delta), _p(A), _p(C_ssm), _p(h_in), _p(decay), _p(dprefix),
                                          _p(out), _p(h_last), _p(ckpt), Bb, L, D, dt, _stream(dev))
        else:
            rc = lib.mwc_ss_fixup(_p(delta), _p(A), _p(C_ssm), _p(h_in), _p(decay), _p(out),
                                  _p(h_last), _p(ckpt), Bb, L, D, dt, _stream(dev))
    _lib.check(rc, "selective_scan fixup")


def lin_scan_forward(a, x):
    """h_0 = x_0, h_t = a_t h_{t-1} + x_t along dim 2 of contiguous (B, D, L, N) tensors."""
    Bb, Dd, L, N = x.shape
    h = torch.empty_like(x)
    if h.numel() == 0:
        return h
    lib = _lib.load()
    dev = x.device
    with _on_device(dev):
        rc = lib.mwc_lin_scan_fwd(_p(a), _p(x), _p(h), Bb * Dd, L, N, dtype_code(x),
                                  _stream(dev))
    _lib.check(rc, "parallel_scan forward")
    return h


def lin_scan_backward(a, h, g):
    Bb, Dd, L, N = g.shape
    ga = torch.empty_like(g)
    gx = torch.empty_like(g)
    if g.numel() == 0:
        return ga, gx
    lib = _lib.load()
    dev = g.device
    with _on_device(dev):
        rc = lib.mwc_lin_scan_bwd(_p(a), _p(h), _p(g), _p(ga), _p(gx), Bb * Dd, L, N,
                                  dtype_code(g), _stream(dev))
    _lib.check(rc, "parallel_scan backward")
    return ga, gx
