"""Float64 stand-ins for the CUDA local scan and carry fixup, injected into the sharding
host logic by the CPU tests (test infrastructure: the product path never uses them). The
local scan is the float64 oracle; decay and fixup restate the definitions of
``mwc_ss_fwd``'s ``decay`` output and of ``mwc_ss_fixup`` (include/mwc_b200.h), with the
reference's exponent clamp (``safe_exp``, mamba_cuda.py:65-70)."""
from __future__ import annotations

import numpy as np
import torch

from oracle import oracle as O

ARG_HI = 88.0


def _np(t):
    return None if t is None else t.detach().cpu().double().numpy()


def _log_factors(delta, A):
    """min(delta_t * A, 88) for every (b, t, d, n)."""
    return np.minimum(delta[:, :, :, None] * A[None, None], ARG_HI)


def local_scan(u, delta, A, Bm, Cm, Dv, h_prev):
    out, h_last = O.ss_fwd(_np(u), _np(delta), _np(A), _np(Bm), _np(Cm), _np(Dv), _np(h_prev))
    decay = np.exp(_log_factors(_np(delta), _np(A)).sum(axis=1))
    return (torch.from_numpy(out), torch.from_numpy(h_last), torch.from_numpy(decay))


def fixup(delta, A, Cm, h_in, decay, out, h_last):
    """In place: out_t += <C_t, Pcum_t * h_in>; h_last = decay * h_in + h_last."""
    pcum = np.exp(np.cumsum(_log_factors(_np(delta), _np(A)), axis=1))   # (B, L, D, N)
    hi = _np(h_in)
    corr = np.einsum("bldn,bdn,bln->bld", pcum, hi, _np(Cm))
    out += torch.from_numpy(corr).to(out.dtype)
    h_last.copy_(torch.from_numpy(_np(decay) * hi + _np(h_last)).to(h_last.dtype))


# ---- stand-ins for the hooks of sequence-sharded training (sharding.sequence_sharded_scan) ----

def train_local_forward(u, delta, A, Bm, Cm, Dv, h_prev):
    out, h_last, decay = local_scan(u, delta, A, Bm, Cm, Dv, h_prev)
    return {"out": out, "h_last": h_last, "ckpt": None, "decay": decay, "end": h_last.clone(),
            "dpre": None}


def train_fixup(delta, A, Cm, h_in, st):
    fixup(delta, A, Cm, h_in, st["decay"], st["out"], st["h_last"])


def train_local_backward(u, delta, A, Bm, Cm, Dv, h_start, ckpt, dout, dh_last):
    """float64 oracle reverse scan of one range from its incoming state (ckpt unused)."""
    g = O.ss_bwd(_np(u), _np(delta), _np(A), _np(Bm), _np(Cm), _np(Dv), _np(dout), _np(h_start),
                 _np(dh_last))
    return tuple(torch.from_numpy(g[k]) for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dh_prev"))


TRAIN_HOOKS = dict(local_forward=train_local_forward, fixup=train_fixup,
                   local_backward=train_local_backward)


def train_local_adjoint(u, delta, A, Bm, Cm, Dv, dout, dh_last):
    """Adjoint at the range start from a zero state's reverse scan (the oracle's dh_prev; the
    adjoint does not depend on the forward states)."""
    g = O.ss_bwd(_np(u), _np(delta), _np(A), _np(Bm), _np(Cm), _np(Dv), _np(dout), None, _np(dh_last))
    return torch.from_numpy(g["dh_prev"])


TRAIN_HOOKS["local_adjoint"] = train_local_adjoint
