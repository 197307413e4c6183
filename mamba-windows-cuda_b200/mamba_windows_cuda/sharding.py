"""Multi-GPU partitioning of the selective scan, one process per GPU (torch.distributed:
NCCL between B200s, gloo in the CPU tests).

Two modes.

* Batch / channel sharding (``split_range``, ``shard``): every rank scans its own slice of
  the batch rows or channels with the single-GPU entry points; there is no exchange, so it
  scales as independent replicas.

* Sequence sharding (``sequence_sharded_forward``): rank r owns the contiguous time range
  ``split_range(L_total, world, r)``. Each rank scans its range from a zero state (rank 0 from
  the caller's ``h_prev``), producing its local output, its segment decay
  ``P_r = prod_t exp(min(delta_t * A, 88))`` and its end state ``S_r`` (float32, B x D x 16).
  The ranks all-gather ``(P_r, S_r)`` (2 x B x D x 16 float32 per rank); rank r folds the
  carries of the ranks before it, ``h_in = P_{r-1} * (... (P_0 * 0 + S_0) ...) + S_{r-1}``,
  and folds ``h_in`` into its own range with the carry fixup (``mwc_ss_fixup``):
  ``y_t += <C_t, Pcum_t * h_in>``, ``h_last = P_r * h_in + S_r``. The last rank then holds
  the h_last of the whole sequence, so chunked streaming (``h_prev`` -> ``h_last``) keeps its
  meaning across the sharded sequence (``broadcast_h_last`` hands it to every rank).

The reference runs on one GPU and has neither mode; the local scans are the reference's
forward (``selective_scan_cuda_forward_with_state``, ``mamba_cuda.py:176-359``). Only the
forward is sequence-sharded; gradients of a sequence-sharded scan are not provided.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple

import torch

NSTATE = 16


def split_range(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Contiguous, balanced [start, stop) share of ``n`` items for ``rank`` of ``world``
    (the first ``n % world`` ranks take one item more)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = divmod(int(n), world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def shard(x: torch.Tensor, dim: int, world: int, rank: int) -> torch.Tensor:
    """This rank's contiguous slice of ``x`` along ``dim`` (batch rows: dim 0; channels of a
    (B, L, D) tensor: dim 2), for batch / channel sharding."""
    a, b = split_range(x.shape[dim], world, rank)
    return x.narrow(dim, a, b - a)


def fold_carries(decays: torch.Tensor, states: torch.Tensor, upto: int) -> torch.Tensor:
    """State entering segment ``upto`` of a sequence cut into segments that were each scanned
    from zero: ``h = 0; for j < upto: h = decays[j] * h + states[j]`` (float32).

    On CUDA tensors this is one launch of the linear-recurrence scan behind
    ``parallel_scan_fn`` (x_t = a_t x_{t-1} + b_t along the segment axis), the same combine
    the single-GPU few-chain split uses; elsewhere a loop over the segments."""
    if upto <= 0:
        return torch.zeros_like(states[0], dtype=torch.float32)
    if decays.is_cuda:
        from . import _ops
        n = states[0].numel()
        a = decays[:upto].float().reshape(1, 1, upto, n).contiguous()
        x = states[:upto].float().reshape(1, 1, upto, n).contiguous()
        return _ops.lin_scan_forward(a, x)[0, 0, upto - 1].reshape(states[0].shape)
    h = torch.zeros_like(states[0], dtype=torch.float32)
    for j in range(upto):
        h = decays[j].float() * h + states[j].float()
    return h


def _cuda_local_scan(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev):
    """Local scan of a rank's range: (out, h_last, decay, end, dprefix). ``end`` is the
    float32 end state: with 16-bit I/O, h_last is rounded to the I/O type, so the end state
    comes from the last float32 checkpoint instead (the state after the range's last step),
    and the carries travel and fold in float32 as in the single-GPU scan's segment hand-off.
    ``dprefix`` holds the range's delta prefix records when the persistent kernel runs the
    scan (None otherwise); the chunked fixup uses them."""
    from . import _ops
    half = u.dtype != torch.float32
    Bb, L, D = u.shape
    dpre = None
    if _ops.plan(Bb, L, D, u.dtype)["path"] != "generic" and all(
            t.data_ptr() % 16 == 0 for t in (u, delta, A, B_ssm, C_ssm, D_ssm)):
        dpre = torch.empty((Bb, _ops.dprefix_count(L), D, 2), dtype=torch.float32, device=u.device)
    out, h_last, ckpt, decay = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                               want_h_last=True, want_ckpt=half, want_decay=True,
                                               dprefix=dpre)
    end = ckpt[:, -1].contiguous() if half else h_last
    return out, h_last, decay, end, dpre


def _cuda_fixup(delta, A, C_ssm, h_in, decay, out, h_last, end=None, dpre=None):
    """Folds h_in into the rank's output in place; h_last = decay * h_in + end, computed in
    float32 from the float32 end state when one is given (16-bit I/O)."""
    from . import _ops
    if end is not None and h_last.dtype != torch.float32:
        _ops.ss_fixup(delta, A, C_ssm, h_in, decay, out, None, dprefix=dpre)
        h_last.copy_((decay * h_in + end).to(h_last.dtype))
    else:
        _ops.ss_fixup(delta, A, C_ssm, h_in, decay, out, h_last, dprefix=dpre)


def _split_local(res):
    """(out, h_last, decay, end32, dprefix) from a local scan's result; stand-ins that return
    three values give their h_last as the end state and no prefix records."""
    if len(res) == 5:
        return res
    if len(res) == 4:
        return tuple(res) + (None,)
    out, h_last, decay = res
    return out, h_last, decay, None, None


def _fix(fixup, delta, A, C_ssm, h_in, decay, out, h_last, end, dpre):
    if fixup is _cuda_fixup:
        fixup(delta, A, C_ssm, h_in, decay, out, h_last, end, dpre)
    else:
        fixup(delta, A, C_ssm, h_in, decay, out, h_last)


def _all_gather(payload: torch.Tensor, world: int, group) -> torch.Tensor:
    import torch.distributed as dist
    out = torch.empty((world,) + tuple(payload.shape), dtype=payload.dtype, device=payload.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, payload, group=group)
    else:
        dist.all_gather(list(out.unbind(0)), payload, group=group)
    return out


def sequence_sharded_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None, *, group=None,
                             broadcast_h_last: bool = False,
                             local_scan: Optional[Callable] = None,
                             fixup: Optional[Callable] = None,
                             phase_hook: Optional[Callable[[str], None]] = None):
    """Forward scan of a sequence split along L across the ranks of ``group``.

    Every rank passes its own contiguous time range of ``u, delta, B_ssm, C_ssm`` ((B, L_r, D)
    and (B, L_r, 16); ranges in rank order, see ``split_range``) and the full ``A``, ``D_ssm``;
    ``h_prev`` is used on rank 0 only. Returns ``(out, h_last)``: this rank's output range and
    the state after it (after the last range on the last rank; on every rank with
    ``broadcast_h_last``).

    ``local_scan(u, delta, A, B, C, D, h_prev) -> (out, h_last, decay[, end32])`` and
    ``fixup(delta, A, C, h_in, decay, out, h_last)`` default to the CUDA entry points (the
    CPU tests pass float64 restatements). The carries are exchanged and folded in float32;
    with 16-bit I/O the CUDA local scan supplies a float32 end state for them.
    ``phase_hook(name)``, when given, is called after each phase ("local", "gather", "fold",
    "fixup") so a caller can record timing events between them.
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    local_scan = local_scan or _cuda_local_scan
    fixup = fixup or _cuda_fixup

    hook = phase_hook or (lambda name: None)
    out, h_last, decay, end, dpre = _split_local(
        local_scan(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev if rank == 0 else None))
    payload = torch.stack([decay.float(), (end if end is not None else h_last).float()]).contiguous()
    hook("local")
    gathered = _all_gather(payload, world, group)
    hook("gather")
    if rank > 0:
        h_in = fold_carries(gathered[:, 0], gathered[:, 1], rank).contiguous()
        hook("fold")
        _fix(fixup, delta, A, C_ssm, h_in, decay, out, h_last, end, dpre)
    else:
        hook("fold")
    hook("fixup")
    if broadcast_h_last and world > 1:
        src = world - 1 if group is None else dist.get_global_rank(group, world - 1)
        dist.broadcast(h_last, src=src, group=group)
    return out, h_last


def emulated_sequence_sharded_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None, *, world: int,
                                      local_scan: Optional[Callable] = None,
                                      fixup: Optional[Callable] = None):
    """The sequence-sharded forward with ``world`` ranks emulated in one process on one device
    (same local scans, carry fold and fixup as the multi-process path; for tests and for
    checking the fixup without several GPUs). Takes the whole sequence; returns
    ``(out, h_last)`` of the whole sequence."""
    local_scan = local_scan or _cuda_local_scan
    fixup = fixup or _cuda_fixup
    L = u.shape[1]
    ranges = [split_range(L, world, r) for r in range(world)]
    parts = []
    for r, (a, b) in enumerate(ranges):
        sl = (slice(None), slice(a, b))
        parts.append((u[sl].contiguous(), delta[sl].contiguous(), B_ssm[sl].contiguous(),
                      C_ssm[sl].contiguous()))
    locals_ = [_split_local(local_scan(p[0], p[1], A, p[2], p[3], D_ssm, h_prev if r == 0 else None))
               for r, p in enumerate(parts)]
    payloads = [torch.stack([dc.float(), (e if e is not None else hl).float()])
                for (_, hl, dc, e, _) in locals_]
    outs, h_last = [], None
    for r, ((o, hl, dc, e, dp), p) in enumerate(zip(locals_, parts)):
        if r > 0:
            h_in = fold_carries(torch.stack([q[0] for q in payloads]),
                                torch.stack([q[1] for q in payloads]), r).contiguous()
            _fix(fixup, p[1], A, p[3], h_in, dc, o, hl, e, dp)
        outs.append(o)
        h_last = hl
    return torch.cat(outs, dim=1), h_last
