"""GPU tests of sequence sharding through the CUDA entry points (local scans with the
segment decay, carry fold, mwc_ss_fixup), against the single-call CUDA scan of the whole
sequence and the float64 oracle. Ranks are emulated in one process on one GPU; the NCCL
test with one process per GPU runs when two or more GPUs are visible."""
from __future__ import annotations

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from _helpers import assert_fp16, assert_fp32, make_inputs, np64
from mamba_windows_cuda import _ops
from mamba_windows_cuda import sharding as S
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _need_gpu(n=1):
    if not torch.cuda.is_available() or torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} CUDA GPU(s)")


CASES = [
    # (dtype, B, L, D, world, dist)
    (torch.float32, 1, 8192, 256, 4, "c4"),
    (torch.float32, 1, 8192, 256, 8, "c4"),
    (torch.float32, 2, 3000, 96, 3, "c1"),      # ragged ranges, strong decay
    (torch.float16, 1, 8192, 256, 8, "c4"),
    (torch.float32, 1, 65536, 2048, 8, "c4"),   # config-4 chunk spread over 8 ranks
]


@pytest.mark.parametrize("dtype,B,L,D,world,dist", CASES)
def test_emulated_sequence_sharding(dtype, B, L, D, world, dist):
    _need_gpu()
    x = make_inputs(B, L, D, dtype, seed=21, dist=dist, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last = S.emulated_sequence_sharded_forward(*args, x["h_prev"], world=world)
    ref_out, ref_h, _, _ = _ops.ss_forward(*args, x["h_prev"], want_h_last=True)
    torch.cuda.synchronize()
    if dtype == torch.float32:
        assert_fp32(out, ref_out.double().cpu().numpy(), what="out vs single-call scan")
        assert_fp32(h_last, ref_h.double().cpu().numpy(), what="h_last vs single-call scan")
        if L * D <= 8192 * 256:
            o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
            assert_fp32(out, o64, what="out vs oracle")
            assert_fp32(h_last, h64, what="h_last vs oracle")
    else:
        o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
        assert_fp16(out, o64, what="out vs oracle")
        assert_fp16(h_last, h64, what="h_last vs oracle")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _nccl_worker(rank, world, port, outdir):
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        x = make_inputs(1, 16384, 512, torch.float32, seed=31, dist="c4", with_state=True,
                        device=f"cuda:{rank}")
        args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
        a, b = S.split_range(x["u"].shape[1], world, rank)
        part = [t[:, a:b].contiguous() if t.dim() == 3 else t for t in args]
        out, h_last = S.sequence_sharded_forward(*part, x["h_prev"], broadcast_h_last=True)
        torch.cuda.synchronize()
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.double().cpu().numpy())
        np.save(os.path.join(outdir, f"h{rank}.npy"), h_last.double().cpu().numpy())
    finally:
        dist.destroy_process_group()


def test_nccl_sequence_sharding_two_ranks():
    _need_gpu(2)
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_nccl_worker, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn", join=True)
        out = np.concatenate([np.load(os.path.join(d, f"out{r}.npy")) for r in range(world)], axis=1)
        hs = [np.load(os.path.join(d, f"h{r}.npy")) for r in range(world)]
    x = make_inputs(1, 16384, 512, torch.float32, seed=31, dist="c4", with_state=True)
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
    assert_fp32(out, o64, what="out")
    for r in range(world):
        assert_fp32(hs[r], h64, what=f"h_last on rank {r}")


@pytest.mark.parametrize("neg", [False, True])
def test_chunked_fixup_matches_serial_fixup(neg):
    """mwc_ss_fixup_chunked (parallel 256-step chunks started from the local scan's delta
    prefix records, skipped once h_in has decayed) against mwc_ss_fixup (one pass per channel
    up to the decay horizon) on the same local scan, including a stretch of negative deltas,
    where the incoming state grows again after having decayed."""
    _need_gpu()
    B, L, D = 1, 8192, 256
    x = make_inputs(B, L, D, torch.float32, seed=23, dist="c4", with_state=True, device="cuda")
    x["delta"] *= 4   # decay horizon ~2.2k steps: most chunks are skipped
    if neg:
        x["delta"][:, 6000:6040] = -0.25
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    assert _ops.plan(B, L, D, torch.float32)["path"] != "generic"
    dpre = torch.empty(B, _ops.dprefix_count(L), D, 2, device="cuda")
    out, h_last, ckpt, decay = _ops.ss_forward(*args, want_h_last=True, want_ckpt=True, want_decay=True,
                                               dprefix=dpre)
    h_in = x["h_prev"].float().contiguous()
    res = []
    for dp in (dpre, None):
        o, h, c = out.clone(), h_last.clone(), ckpt.clone()
        _ops.ss_fixup(x["delta"], x["A"], x["Cm"], h_in, decay, o, h, c, dprefix=dp)
        res.append((o, h, c))
    torch.cuda.synchronize()
    for a, b, what in zip(res[0], res[1], ("out", "h_last", "ckpt")):
        assert_fp32(a, b.double().cpu().numpy(), tol=1e-5, what=what)
    # and against the oracle scan started from h_in
    o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(h_in))
    assert_fp32(res[0][0], o64, what="out vs oracle")
    assert_fp32(res[0][1], h64, what="h_last vs oracle")


# ---- sequence-sharded training (forward + backward across the ranks) ----
# Tolerances: float32 normwise 1e-4; 16-bit per-element gradients (du, ddelta, dh_prev)
# elementwise atol 2e-2 / rtol 1e-2 (bfloat16: rtol 2e-2), the sums (dA, dB, dC, dD) with
# atol scaled by max(1, max|ref|), as in the single-GPU parity tests.

TRAIN_CASES = [
    # (dtype, B, L, D, world, dist)
    (torch.float32, 1, 8192, 256, 4, "c4"),    # few chains: split passes per range; slow decay
    (torch.float32, 2, 3000, 96, 3, "c1"),     # ragged ranges on the generic kernels
    (torch.float16, 1, 8192, 256, 2, "c4"),
    (torch.bfloat16, 1, 4096, 256, 3, "c4"),
    (torch.float16, 4, 1024, 5120, 2, "c3"),   # chained persistent kernels per range
    (torch.float32, 2, 13, 64, 8, "c1"),       # ranges of 0-2 steps (empty ranges too)
    (torch.float16, 2, 1000, 36, 3, "c1"),     # generic kernels (72-byte rows), ranges ending mid-chunk
]
PER_ELEMENT = ("du", "ddelta", "dh_prev")


def _check_grad(x, ref, dtype, what, reduced):
    if dtype == torch.float32:
        assert_fp32(x, ref, what=what)
        return
    atol = 2e-2 * (max(1.0, float(np.abs(ref).max())) if reduced else 1.0)
    rtol = 2e-2 if dtype == torch.bfloat16 else 1e-2
    assert_fp16(x.float(), ref, what=what, atol=atol, rtol=rtol)


@pytest.mark.parametrize("dtype,B,L,D,world,dist", TRAIN_CASES)
def test_emulated_sequence_training(dtype, B, L, D, world, dist):
    _need_gpu()
    x = make_inputs(B, L, D, dtype, seed=23, dist=dist, with_state=True, device="cuda")
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    g = torch.Generator(device="cuda").manual_seed(77)
    dout = torch.randn(B, L, D, generator=g, device="cuda").to(dtype)
    dh_last = torch.randn(B, D, 16, generator=g, device="cuda").to(dtype)
    out, h_last, grads = S.emulated_sequence_sharded_training(*args, x["h_prev"], dout, dh_last,
                                                              world=world)
    torch.cuda.synchronize()
    n = [np64(t) for t in args]
    o64, h64 = O.ss_fwd(*n, np64(x["h_prev"]))
    ref = O.ss_bwd(*n, np64(dout), np64(x["h_prev"]), np64(dh_last))
    _check_grad(out, o64, dtype, "out", False)
    _check_grad(h_last, h64, dtype, "h_last", False)
    for k in ("du", "ddelta", "dA", "dB", "dC", "dD", "dh_prev"):
        _check_grad(grads[k], ref[k], dtype, k, k not in PER_ELEMENT)


def _nccl_train_worker(rank, world, port, outdir):
    import datetime
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        dev = f"cuda:{rank}"
        x = make_inputs(1, 16384, 512, torch.float32, seed=33, dist="c4", with_state=True, device=dev)
        g = torch.Generator(device=dev).manual_seed(79)
        dout = torch.randn(1, 16384, 512, generator=g, device=dev)
        dh_last = torch.randn(1, 512, 16, generator=g, device=dev)
        a, b = S.split_range(16384, world, rank)
        leaves = [(x[k][:, a:b] if x[k].dim() == 3 else x[k]).clone().requires_grad_(True)
                  for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
        hp = x["h_prev"].clone().requires_grad_(True)
        out, h_last = S.sequence_sharded_scan(*leaves, hp)
        loss = (out * dout[:, a:b]).sum()
        if rank == world - 1:
            loss = loss + (h_last * dh_last).sum()
        loss.backward()
        torch.cuda.synchronize()
        for k, t in zip(("du", "ddelta", "dA", "dB", "dC", "dD"), leaves):
            np.save(os.path.join(outdir, f"{k}{rank}.npy"), t.grad.double().cpu().numpy())
        if rank == 0:
            np.save(os.path.join(outdir, "dh_prev.npy"), hp.grad.double().cpu().numpy())
    finally:
        dist.destroy_process_group()


def test_nccl_sequence_training_two_ranks():
    _need_gpu(2)
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_nccl_train_worker, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn", join=True)
        got = {k: [np.load(os.path.join(d, f"{k}{r}.npy")) for r in range(world)]
               for k in ("du", "ddelta", "dA", "dB", "dC", "dD")}
        dhp = np.load(os.path.join(d, "dh_prev.npy"))
    x = make_inputs(1, 16384, 512, torch.float32, seed=33, dist="c4", with_state=True, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(79)
    dout = torch.randn(1, 16384, 512, generator=g, device="cuda")
    dh_last = torch.randn(1, 512, 16, generator=g, device="cuda")
    args = [np64(x[k]) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    ref = O.ss_bwd(*args, np64(dout), np64(x["h_prev"]), np64(dh_last))
    for k in ("du", "ddelta", "dB", "dC"):
        assert_fp32(np.concatenate(got[k], axis=1), ref[k], what=k)
    for r in range(world):
        assert_fp32(got["dA"][r], ref["dA"], what=f"dA on rank {r}")
        assert_fp32(got["dD"][r], ref["dD"], what=f"dD on rank {r}")
    assert_fp32(dhp, ref["dh_prev"], what="dh_prev")


@pytest.mark.parametrize("dtype,B,L,D,with_q", [
    (torch.float32, 2, 1000, 96, True),     # ragged last chunk
    (torch.float32, 1, 100, 40, False),     # one partial chunk
    (torch.float16, 1, 4096, 256, True),
    (torch.bfloat16, 2, 777, 64, True),
])
def test_range_adjoint_matches_oracle(dtype, B, L, D, with_q):
    """mwc_ss_adjoint_seq: the adjoint at the range start against the float64 oracle's
    dh_prev (the adjoint does not depend on the forward states)."""
    _need_gpu()
    x = make_inputs(B, L, D, dtype, seed=41, dist="c4", device="cuda")
    g = torch.Generator(device="cuda").manual_seed(43)
    dout = torch.randn(B, L, D, generator=g, device="cuda").to(dtype)
    q_in = torch.randn(B, D, 16, generator=g, device="cuda") if with_q else None
    q0 = _ops.ss_adjoint(x["delta"], x["A"], x["Cm"], dout, q_in)
    torch.cuda.synchronize()
    args = [np64(x[k]) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    ref = O.ss_bwd(*args, np64(dout), None, np64(q_in) if with_q else None)["dh_prev"]
    assert q0.dtype == torch.float32
    assert_fp32(q0, ref, what="range adjoint")
