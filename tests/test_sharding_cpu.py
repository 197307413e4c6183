"""Host logic of the multi-GPU modes, on CPU: range splitting, the carry fold, the sequence-
sharded forward with ranks emulated in one process, and the same path as two gloo ranks
(world_size 2, one process each). The local scans and the fixup are float64 stand-ins
(tests/_sharding_ref.py); results are checked against the float64 oracle run over the whole
sequence (fp32 tolerance, normwise 1e-4)."""
from __future__ import annotations

import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

import _sharding_ref as R
from _helpers import assert_fp32, make_inputs, np64
from mamba_windows_cuda import sharding as S
from oracle import oracle as O


@pytest.mark.parametrize("n,world", [(10, 3), (7, 7), (5, 8), (2 ** 20, 8), (0, 2)])
def test_split_range_covers_contiguously(n, world):
    prev = 0
    sizes = []
    for r in range(world):
        a, b = S.split_range(n, world, r)
        assert a == prev and b >= a
        sizes.append(b - a)
        prev = b
    assert prev == n and max(sizes) - min(sizes) <= 1


def test_split_range_rejects_bad_rank():
    with pytest.raises(ValueError):
        S.split_range(10, 2, 2)


def test_fold_carries_is_sequential_composition():
    g = torch.Generator().manual_seed(3)
    P = torch.rand(4, 2, 3, 16, generator=g)
    Sx = torch.randn(4, 2, 3, 16, generator=g)
    h = torch.zeros(2, 3, 16)
    for r in range(4):
        assert torch.allclose(S.fold_carries(P, Sx, r), h, atol=1e-6)
        h = P[r] * h + Sx[r]


def _inputs(seed=5, B=2, L=48, D=6, with_state=True):
    x = make_inputs(B, L, D, torch.float32, seed=seed, dist="c4", with_state=with_state)
    return x


@pytest.mark.parametrize("world", [1, 2, 3, 5])
def test_emulated_sequence_sharding_matches_full_scan(world):
    x = _inputs()
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last = S.emulated_sequence_sharded_forward(*args, x["h_prev"], world=world,
                                                      local_scan=R.local_scan, fixup=R.fixup)
    o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
    assert_fp32(out, o64, what=f"out (world {world})")
    assert_fp32(h_last, h64, what=f"h_last (world {world})")


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, outdir, mode):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        x = _inputs(seed=11, B=2, L=40, D=6)
        args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
        if mode == "sequence":
            a, b = S.split_range(x["u"].shape[1], world, rank)
            part = [t[:, a:b].contiguous() if t.dim() == 3 else t for t in args]
            out, h_last = S.sequence_sharded_forward(*part, x["h_prev"], broadcast_h_last=True,
                                                     local_scan=R.local_scan, fixup=R.fixup)
        else:   # batch rows: independent scans, no exchange
            part = [S.shard(t, 0, world, rank) if t.dim() == 3 else t for t in args]
            hp = S.shard(x["h_prev"], 0, world, rank)
            out, h_last, _ = R.local_scan(*part, hp)
        np.save(os.path.join(outdir, f"out{rank}.npy"), out.double().numpy())
        np.save(os.path.join(outdir, f"h{rank}.npy"), h_last.double().numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["sequence", "batch"])
def test_gloo_two_ranks_match_full_scan(mode):
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_gloo_worker, args=(world, _free_port(), d, mode), nprocs=world,
                           start_method="spawn", join=True)
        outs = [np.load(os.path.join(d, f"out{r}.npy")) for r in range(world)]
        hs = [np.load(os.path.join(d, f"h{r}.npy")) for r in range(world)]
    x = _inputs(seed=11, B=2, L=40, D=6)
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
    if mode == "sequence":
        assert_fp32(np.concatenate(outs, axis=1), o64, what="out")
        for r in range(world):   # broadcast_h_last: every rank holds the sequence's h_last
            assert_fp32(hs[r], h64, what=f"h_last on rank {r}")
    else:
        assert_fp32(np.concatenate(outs, axis=0), o64, what="out")
        assert_fp32(np.concatenate(hs, axis=0), h64, what="h_last")


# ---- sequence-sharded training: backward across the ranks ----

GRAD_KEYS = ("du", "ddelta", "dA", "dB", "dC", "dD", "dh_prev")


def _train_case(seed=7, B=2, L=48, D=6):
    x = _inputs(seed=seed, B=B, L=L, D=D)
    g = torch.Generator().manual_seed(seed + 1)
    dout = torch.randn(B, L, D, generator=g)
    dh_last = torch.randn(B, D, 16, generator=g)
    return x, dout, dh_last


def _oracle_grads(x, dout, dh_last):
    args = [np64(x[k]) for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    return O.ss_bwd(*args, np64(dout), np64(x["h_prev"]), np64(dh_last))


@pytest.mark.parametrize("world,L", [(1, 48), (2, 48), (3, 48), (5, 48), (5, 3)])
def test_emulated_sequence_training_matches_full_backward(world, L):
    # (5, 3): more ranks than steps, so some ranges are empty
    x, dout, dh_last = _train_case(L=L)
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    out, h_last, grads = S.emulated_sequence_sharded_training(*args, x["h_prev"], dout, dh_last,
                                                              world=world, **R.TRAIN_HOOKS)
    o64, h64 = O.ss_fwd(*[np64(t) for t in args], np64(x["h_prev"]))
    assert_fp32(out, o64, what=f"out (world {world})")
    assert_fp32(h_last, h64, what=f"h_last (world {world})")
    ref = _oracle_grads(x, dout, dh_last)
    for k in GRAD_KEYS:
        assert_fp32(grads[k], ref[k], what=f"{k} (world {world})")


def _gloo_train_worker(rank, world, port, outdir):
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        x, dout, dh_last = _train_case(seed=13, B=2, L=40, D=6)
        a, b = S.split_range(x["u"].shape[1], world, rank)
        leaves = {k: (x[k][:, a:b] if x[k].dim() == 3 else x[k]).clone().requires_grad_(True)
                  for k in ("u", "delta", "A", "Bm", "Cm", "Dv")}
        hp = x["h_prev"].clone().requires_grad_(True)
        out, h_last = S.sequence_sharded_scan(*leaves.values(), hp, **R.TRAIN_HOOKS)
        loss = (out * dout[:, a:b].to(out.dtype)).sum()
        if rank == world - 1:
            loss = loss + (h_last * dh_last.to(h_last.dtype)).sum()
        loss.backward()
        for k, t in leaves.items():
            np.save(os.path.join(outdir, f"{k}{rank}.npy"), t.grad.double().numpy())
        np.save(os.path.join(outdir, f"hp{rank}.npy"),
                hp.grad.double().numpy() if hp.grad is not None else np.zeros(0))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_training_matches_full_backward():
    world = 2
    with tempfile.TemporaryDirectory() as d:
        mp.start_processes(_gloo_train_worker, args=(world, _free_port(), d), nprocs=world,
                           start_method="spawn", join=True)
        got = {k: [np.load(os.path.join(d, f"{k}{r}.npy")) for r in range(world)]
               for k in ("u", "delta", "A", "Bm", "Cm", "Dv", "hp")}
    x, dout, dh_last = _train_case(seed=13, B=2, L=40, D=6)
    ref = _oracle_grads(x, dout, dh_last)
    for name, k in (("du", "u"), ("ddelta", "delta"), ("dB", "Bm"), ("dC", "Cm")):
        assert_fp32(np.concatenate(got[k], axis=1), ref[name], what=name)
    for r in range(world):   # replicated parameters: every rank holds the sum
        assert_fp32(got["A"][r], ref["dA"], what=f"dA on rank {r}")
        assert_fp32(got["Dv"][r], ref["dD"], what=f"dD on rank {r}")
    assert_fp32(got["hp"][0], ref["dh_prev"], what="dh_prev (rank 0)")


def test_cuda_paths_reject_cpu_tensors():
    """With the default (CUDA) hooks the sharded entry points apply the reference's input
    checks (mamba_cuda.py:186-238) before anything reaches the C entry points."""
    x, dout, dh_last = _train_case(L=16)
    args = [x[k] for k in ("u", "delta", "A", "Bm", "Cm", "Dv")]
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        S.emulated_sequence_sharded_forward(*args, x["h_prev"], world=2)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        S.emulated_sequence_sharded_training(*args, x["h_prev"], dout, dh_last, world=2)
