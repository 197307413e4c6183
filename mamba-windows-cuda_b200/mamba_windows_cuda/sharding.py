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

* Sequence-sharded training (``sequence_sharded_scan``): the same forward keeping float32
  checkpoints of each range, and a backward across the ranks (local reverse scans, one
  all-gather of the adjoint carries, a reverse fold, and a second reverse scan on every rank
  but the last; see the section below).

The reference runs on one GPU and has none of these modes; the local scans are the
reference's forward and backward (``selective_scan_cuda_forward_with_state``,
``mamba_cuda.py:176-359``; ``selective_scan_cuda_backward_direct``, ``:766-790``).
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


def _prep_cuda(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev):
    """The reference's input checks (mamba_cuda.py:186-238: CUDA tensors, one dtype, the
    shapes) and contiguous copies where needed, as the single-GPU ops do: the CUDA entry points
    take raw pointers of contiguous tensors (a time slice of a (B, L, D) tensor with B > 1 is
    not contiguous)."""
    from . import _ops
    _ops.check_ss_inputs(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
    return [t.contiguous() for t in (u, delta, A, B_ssm, C_ssm, D_ssm)] + [
        h_prev.contiguous() if h_prev is not None else None]


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
    if local_scan is None and fixup is None:
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev = _prep_cuda(u, delta, A, B_ssm, C_ssm, D_ssm,
                                                               h_prev if rank == 0 else None)
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
    if local_scan is None and fixup is None:
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev = _prep_cuda(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
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


# ---------------------------------------------------------------------------
# Sequence-sharded training: the forward above keeping what the backward needs, and the
# backward of the sharded scan.
#
# The adjoint is linear in (dout, dh_last) for fixed forward states, so its carries fold
# like the forward's. Each rank first finds q0_r, the adjoint at its range start from the
# range's own terms (its dout, and dh_last on its h_last) with a zero adjoint at the range
# end: the last rank by its full reverse scan, which already gives its final gradients; the
# others by the range-adjoint pass (mwc_ss_adjoint_seq), which computes only that adjoint.
# The adjoint that enters range r at its end from the later ranks is
# Q_r = q0_{r+1} + P_{r+1} * Q_{r+1} (Q_{last} = 0; P_r is the range's decay, the same
# factor the forward carries use), one reverse fold of the all-gathered (P_r, q0_r). Every
# rank but the last then runs its reverse scan with the adjoint dh_last + Q_r entering at the
# end, which gives its gradients.
# ---------------------------------------------------------------------------

def _cuda_train_forward_local(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev):
    """Local scan of a rank's range for training: output, h_last, the float32 checkpoints the
    backward recomputes from, the range decay, the float32 end state and (persistent path)
    the delta prefix records."""
    from . import _ops
    Bb, L, D = u.shape
    dpre = None
    if L > 0 and _ops.plan(Bb, L, D, u.dtype)["path"] != "generic" and all(
            t.data_ptr() % 16 == 0 for t in (u, delta, A, B_ssm, C_ssm, D_ssm)):
        dpre = torch.empty((Bb, _ops.dprefix_count(L), D, 2), dtype=torch.float32, device=u.device)
    out, h_last, ckpt, decay = _ops.ss_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev,
                                               want_h_last=True, want_ckpt=True, want_decay=True,
                                               dprefix=dpre)
    # the end state travels in float32: with 16-bit I/O from the last checkpoint (the state
    # after the range's last step); copied, since the fixup updates the checkpoints in place
    end = ckpt[:, -1].clone() if (u.dtype != torch.float32 and L > 0) else h_last.float().clone()
    return {"out": out, "h_last": h_last, "ckpt": ckpt, "decay": decay, "end": end, "dpre": dpre}


def _cuda_train_fixup(delta, A, C_ssm, h_in, st):
    """Folds h_in into a training local scan in place: output, checkpoints and h_last."""
    from . import _ops
    h_last = st["h_last"]
    half = h_last.dtype != torch.float32
    _ops.ss_fixup(delta, A, C_ssm, h_in, st["decay"], st["out"], None if half else h_last, st["ckpt"],
                  dprefix=st["dpre"])
    if half:
        h_last.copy_((st["decay"] * h_in + st["end"]).to(h_last.dtype))


def _cuda_train_backward_local(u, delta, A, B_ssm, C_ssm, D_ssm, h_start, ckpt, dout, dh_last):
    """Reverse scan of a rank's range from its true incoming state ``h_start`` (None: zero)
    and the adjoint ``dh_last`` entering at its end (mwc_ss_bwd_seq: both, and the returned
    adjoint at the range start, in float32, like the forward's carries): (du, ddelta, dA,
    dB, dC, dD in the input dtype, dh_prev float32)."""
    from . import _ops
    hp = h_start.float().contiguous() if h_start is not None else None
    dh = dh_last.float().contiguous() if dh_last is not None else None
    return _ops.ss_backward(u, delta, A, B_ssm, C_ssm, D_ssm, hp, dout, dh, ckpt, want_dh_prev=True,
                            carry32=True)


def _cuda_train_adjoint_local(u, delta, A, B_ssm, C_ssm, D_ssm, dout, dh_last):
    """Adjoint at the start of a rank's range from its own dout and the adjoint ``dh_last``
    entering at its end (mwc_ss_adjoint_seq, float32): the first backward pass of the ranks
    before the last, which only hand this adjoint on."""
    from . import _ops
    q_in = dh_last.float().contiguous() if dh_last is not None else None
    return _ops.ss_adjoint(delta, A, C_ssm, dout, q_in)


def _train_fwd_phase2(rank, gathered, delta, A, C_ssm, st, fixup):
    """After the all-gather of (decay, end) records: this rank's incoming state (None on rank
    0), folded into its local scan."""
    if rank == 0:
        return None
    h_in = fold_carries(gathered[:, 0], gathered[:, 1], rank).contiguous()
    fixup(delta, A, C_ssm, h_in, st)
    return h_in


def _train_bwd_phase1(rank, world, ins, h_start, ckpt, dout, dh_last, local_backward, local_adjoint):
    """Before the all-gather: (gradients or None, q0). The last rank's reverse scan is already
    final; the others only need q0 here, the adjoint at their range start from their own
    terms, which the range-adjoint pass gives without a full reverse scan."""
    if rank == world - 1:
        grads = local_backward(*ins, h_start, ckpt, dout, dh_last)
        return grads, grads[6]
    return None, local_adjoint(*ins, dout, dh_last)


def _train_bwd_phase2(rank, world, gathered, ins, h_start, ckpt, grads, dout, dh_last, local_backward):
    """After the all-gather of (decay, q0) records: this rank's gradients. The last rank's
    local reverse scan is already complete. Every other rank runs its reverse scan now, with
    the whole adjoint entering at the range end, dh_last + Q (float32), in one scan rather
    than as a scan of its own terms plus a scan of Q's share: the two shares can be large
    with opposite signs next to the range end, and rounding each to a 16-bit type before the
    sum would lose the difference."""
    if rank >= world - 1:
        return list(grads)
    later = torch.flip(gathered[rank + 1:], dims=[0])   # ranks world-1 .. rank+1
    Q = fold_carries(later[:, 0], later[:, 1], world - 1 - rank)
    if dh_last is not None:
        Q = Q + dh_last.float()
    return list(local_backward(*ins, h_start, ckpt, dout, Q.contiguous()))


class _SequenceShardedScanFn(torch.autograd.Function):
    """(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev) of this rank's range -> (out, h_last),
    with the backward across the ranks. Collectives, the same on every rank: forward one
    all-gather; backward one all-gather and one all-reduce (dA, dD)."""

    @staticmethod
    def forward(ctx, u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, group, hooks):
        import torch.distributed as dist
        world, rank = dist.get_world_size(group), dist.get_rank(group)
        local_forward, fixup, local_backward, local_adjoint = hooks
        st = local_forward(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev if rank == 0 else None)
        payload = torch.stack([st["decay"].float(), st["end"].float()]).contiguous()
        gathered = _all_gather(payload, world, group)
        h_in = _train_fwd_phase2(rank, gathered, delta, A, C_ssm, st, fixup)
        h_start = h_in if rank > 0 else h_prev
        ctx.group, ctx.world, ctx.rank = group, world, rank
        ctx.local_backward, ctx.local_adjoint = local_backward, local_adjoint
        ctx.h_prev_grad = rank == 0 and h_prev is not None
        ctx.save_for_backward(u, delta, A, B_ssm, C_ssm, D_ssm, h_start, st["ckpt"], st["decay"])
        return st["out"], st["h_last"]

    @staticmethod
    def backward(ctx, dout, dh_last):
        import torch.distributed as dist
        u, delta, A, B_ssm, C_ssm, D_ssm, h_start, ckpt, decay = ctx.saved_tensors
        ins = (u, delta, A, B_ssm, C_ssm, D_ssm)
        dout = dout.contiguous() if dout is not None else torch.zeros_like(u)
        dh = dh_last.contiguous() if dh_last is not None else None
        grads, q0 = _train_bwd_phase1(ctx.rank, ctx.world, ins, h_start, ckpt, dout, dh,
                                      ctx.local_backward, ctx.local_adjoint)
        payload = torch.stack([decay.float(), q0.float()]).contiguous()
        gathered = _all_gather(payload, ctx.world, ctx.group)
        du, ddelta, dA, dB, dC, dD, dh_prev = _train_bwd_phase2(
            ctx.rank, ctx.world, gathered, ins, h_start, ckpt, grads, dout, dh, ctx.local_backward)
        # A and D are the same on every rank: their gradient is the sum of the ranks' shares
        pack = torch.cat([dA.float().reshape(-1), dD.float().reshape(-1)])
        dist.all_reduce(pack, group=ctx.group)
        dA = pack[:dA.numel()].reshape(dA.shape).to(dA.dtype)
        dD = pack[dA.numel():].reshape(dD.shape).to(dD.dtype)
        dh_prev = dh_prev.to(h_start.dtype) if ctx.h_prev_grad else None
        return (du, ddelta, dA, dB, dC, dD, dh_prev, None, None)


def sequence_sharded_scan(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev=None, *, group=None,
                          local_forward: Optional[Callable] = None, fixup: Optional[Callable] = None,
                          local_backward: Optional[Callable] = None,
                          local_adjoint: Optional[Callable] = None):
    """Selective scan of a sequence split along L across the ranks of ``group``, with
    gradients (training on sequences sharded over GPUs).

    Arguments as ``sequence_sharded_forward``: this rank's time range of ``u, delta, B_ssm,
    C_ssm`` (ranges in rank order, see ``split_range``), the full ``A`` and ``D_ssm``, and
    ``h_prev`` (used on rank 0). Returns ``(out, h_last)``: this rank's output range and the
    state after it. ``backward`` gives every rank the gradients of its own ranges (du, ddelta,
    dB, dC), the whole sequence's dA and dD (summed over the ranks, as for any replicated
    parameter: average them with a data-parallel wrapper, do not sum them again), and, on
    rank 0, the gradient of ``h_prev``. The forward keeps float32 checkpoints of its range
    (like the single-GPU training forward). ``local_forward``, ``fixup``, ``local_backward``
    and ``local_adjoint`` default to the CUDA entry points; the CPU tests pass float64
    stand-ins."""
    if local_forward is None and fixup is None and local_backward is None and local_adjoint is None:
        import torch.distributed as dist
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev = _prep_cuda(
            u, delta, A, B_ssm, C_ssm, D_ssm, h_prev if dist.get_rank(group) == 0 else None)
    hooks = (local_forward or _cuda_train_forward_local, fixup or _cuda_train_fixup,
             local_backward or _cuda_train_backward_local, local_adjoint or _cuda_train_adjoint_local)
    return _SequenceShardedScanFn.apply(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, group, hooks)


def emulated_sequence_sharded_training(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev, dout, dh_last=None,
                                       *, world: int, local_forward: Optional[Callable] = None,
                                       fixup: Optional[Callable] = None,
                                       local_backward: Optional[Callable] = None,
                                       local_adjoint: Optional[Callable] = None):
    """Forward and backward of the sequence-sharded scan with ``world`` ranks emulated in one
    process on one device (the same phases as ``sequence_sharded_scan``; for tests). Takes the
    whole sequence, ``dout`` for the whole output and ``dh_last`` for the sequence's h_last.
    Returns ``(out, h_last, grads)`` with grads a dict of du, ddelta, dA, dB, dC, dD, dh_prev."""
    if local_forward is None and fixup is None and local_backward is None and local_adjoint is None:
        u, delta, A, B_ssm, C_ssm, D_ssm, h_prev = _prep_cuda(u, delta, A, B_ssm, C_ssm, D_ssm, h_prev)
        dout = dout.contiguous()
    lf = local_forward or _cuda_train_forward_local
    fx = fixup or _cuda_train_fixup
    lb = local_backward or _cuda_train_backward_local
    la = local_adjoint or _cuda_train_adjoint_local
    L = u.shape[1]
    ranges = [split_range(L, world, r) for r in range(world)]

    def part(t, a, b):
        return t[:, a:b].contiguous()

    ins = [(part(u, a, b), part(delta, a, b), A, part(B_ssm, a, b), part(C_ssm, a, b), D_ssm)
           for a, b in ranges]
    sts = [lf(*x, h_prev if r == 0 else None) for r, x in enumerate(ins)]
    gathered = torch.stack([torch.stack([s["decay"].float(), s["end"].float()]) for s in sts])
    h_starts = []
    for r, (x, s) in enumerate(zip(ins, sts)):
        h_in = _train_fwd_phase2(r, gathered, x[1], A, x[4], s, fx)
        h_starts.append(h_in if r > 0 else h_prev)
    douts = [part(dout, a, b) for a, b in ranges]
    dhs = [dh_last if r == world - 1 else None for r in range(world)]
    ph1 = [_train_bwd_phase1(r, world, x, h_starts[r], sts[r]["ckpt"], douts[r], dhs[r], lb, la)
           for r, x in enumerate(ins)]
    locals_ = [p[0] for p in ph1]
    gathered_b = torch.stack([torch.stack([s["decay"].float(), p[1].float()]) for s, p in zip(sts, ph1)])
    fin = [_train_bwd_phase2(r, world, gathered_b, x, h_starts[r], sts[r]["ckpt"], locals_[r], douts[r],
                             dhs[r], lb)
           for r, x in enumerate(ins)]
    grads = {
        "du": torch.cat([f[0] for f in fin], dim=1), "ddelta": torch.cat([f[1] for f in fin], dim=1),
        "dA": sum(f[2].float() for f in fin), "dB": torch.cat([f[3] for f in fin], dim=1),
        "dC": torch.cat([f[4] for f in fin], dim=1), "dD": sum(f[5].float() for f in fin),
        "dh_prev": fin[0][6] if h_prev is not None else None,
    }
    out = torch.cat([s["out"] for s in sts], dim=1)
    return out, sts[-1]["h_last"], grads
