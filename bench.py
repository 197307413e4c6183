#!/usr/bin/env python3
"""Benchmark of the B200 selective scan on BASELINE.json's headline workload.

Default workload (N=1 and per rank for N>1): config 3, the Mamba-2.8B-like training step
of the selective scan, fp16 I/O, B=4, L=2048, D=5120, N=16, forward + backward through
the public API (SelectiveScanCuda -> SelectiveScanFnV2). Metric: GB/s of algorithmic bytes
(fwd reads u, delta, B, C, A, D and writes y; bwd reads u, delta, dy, B, C, A, D and writes
du, ddelta, dA, dB, dC, dD), with the roofline fraction against the slower of HBM
(bytes / measured HBM bandwidth) and MUFU (16 ex2 per (b, l, d) element per pass).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
                  [--config c3|c2|c1|c4|c5]

For N > 1 launch with torchrun (one process per GPU, NCCL): every rank scans its own
batch (weak scaling, no data-path collective); time = max over ranks of the device time.
``--impl reference`` times the reference algorithm's CPU restatement (oracle/, float64,
all host threads) on a bounded sample of the same workload (rank 0 only).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import statistics
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_PARENT = os.path.join(ROOT, "mamba-windows-cuda_b200")
for _p in (ROOT, PKG_PARENT):
    if _p not in sys.path:
        sys.path.insert(0, _p)

import torch  # noqa: E402

METRIC = "selective-scan fwd+bwd GB/s & % of HBM/MUFU roofline, B=4 L=2048 D=5120 fp16"
NSTATE = 16

CONFIGS = {
    "c3": dict(workload="config 3: Mamba-2.8B-like training step, selective scan fwd+bwd "
                        "(SelectiveScanCuda, default V2 path)",
               B=4, L=2048, D=5120, dtype=torch.float16, mode="fwdbwd", dist="c3"),
    "c3bf16": dict(workload="config 3 with bfloat16 I/O (an addition: the reference takes "
                            "float32 / float16)",
                   B=4, L=2048, D=5120, dtype=torch.bfloat16, mode="fwdbwd", dist="c3",
                   metric="selective-scan fwd+bwd GB/s, B=4 L=2048 D=5120 bf16"),
    "c3ex": dict(workload="config 3 shape through selective_scan_fn with Mamba's block transforms "
                          "(delta bias + softplus, z gate; an addition: the reference has neither)",
                 B=4, L=2048, D=5120, dtype=torch.float16, mode="fwdbwd", dist="c3", block=True,
                 metric="selective-scan block op fwd+bwd GB/s (softplus(delta+bias), y*silu(z)), "
                        "B=4 L=2048 D=5120 fp16"),
    "c3b1": dict(workload="config 3 at batch 1 (40 (batch, 128-channel) chains, fewer than the SMs: "
                          "the few-chain split passes of the persistent kernels)",
                 B=1, L=2048, D=5120, dtype=torch.float16, mode="fwdbwd", dist="c3",
                 metric="selective-scan fwd+bwd GB/s, B=1 L=2048 D=5120 fp16"),
    "c3g4": dict(workload="config 3 shape with grouped B / C, G = 4 (B, C of shape (4, 2048, 4, 16); "
                          "an addition: the reference's B / C are one group)",
                 B=4, L=2048, D=5120, dtype=torch.float16, mode="fwdbwd", dist="c3", groups=4,
                 metric="selective-scan fwd+bwd GB/s, B=4 L=2048 D=5120 G=4 fp16"),
    "c3n32": dict(workload="config 3 shape with N = 32 states per channel (selective_scan_nstate: two "
                           "16-state slices; an addition: the reference supports N = 16 only)",
                  B=4, L=2048, D=5120, dtype=torch.float16, mode="fwdbwd", dist="c3", nstate=32,
                  metric="selective-scan fwd+bwd GB/s, B=4 L=2048 D=5120 N=32 fp16"),
    "conv": dict(workload="causal conv1d producer of u (width 4, SiLU) at the config-3 shape, fwd+bwd "
                          "(an addition: the reference has no conv1d)",
                 B=4, L=2048, D=5120, dtype=torch.float16, mode="conv", dist="c3",
                 metric="causal_conv1d fwd+bwd GB/s, (4, 2048, 5120) width 4 SiLU fp16"),
    "c1": dict(workload="config 1: selective scan fwd+bwd fp32 B1 L1024 D256",
               B=1, L=1024, D=256, dtype=torch.float32, mode="fwdbwd", dist="c1",
               metric="selective-scan fwd+bwd GB/s, B=1 L=1024 D=256 fp32"),
    "c2": dict(workload="config 2: Mamba-1.4B-like inference forward_with_state fp16",
               B=8, L=2048, D=4096, dtype=torch.float16, mode="fwd", dist="c2",
               metric="selective-scan inference forward_with_state GB/s, B=8 L=2048 D=4096 fp16"),
    "c4": dict(workload="config 4: streaming scan fp32, 16 chunks of 65536 with h_prev/h_last "
                        "(2^20 tokens; sequence-sharded across ranks for N > 1)",
               B=1, L=65536, D=2048, dtype=torch.float32, mode="stream", dist="c4", chunks=16,
               metric="selective-scan streaming forward GB/s, B=1 L=2^20 (16 x 65536) D=2048 fp32"),
    "c5": dict(workload="config 5: parallel_scan_fn fp32 (B=16, D=1024, L=16384, 1), a~U(0.9,1), "
                        "b~N(0,1)",
               B=16, L=16384, D=1024, dtype=torch.float32, mode="pscan", dist="c5",
               metric="parallel_scan_fn GB/s, (16, 1024, 16384, 1) fp32"),
}


# DRAM bytes (read + write) of one launch of the dominant kernel, from one ncu capture of
# this bench's own command (`--metrics dram__bytes_read.sum,dram__bytes_write.sum` on the
# kernel named below; the capture and its command are kept with the profile summaries).
CAPTURED_TRAFFIC = {
    "c3": {"bytes": 419.284992e6 + 204.703744e6,
           "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one ss_bwd_persistent_kernel "
                     "launch of `python bench.py --steps 3 --warmup 3 --no-cpu-baseline`"},
    "conv": {"bytes": 167.935232e6 + 54.496256e6,
             "source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one conv1d_bwd_tma_kernel "
                       "launch of `python bench.py --config conv --steps 3 --warmup 3 --no-cpu-baseline` "
                       "(part of dx is still in L2 at kernel end)"},
}


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return dict(hbm_gbs=float(pk["hbm_gbs"]), sm_max_mhz=float(pk.get("sm_max_mhz", 1965.0)),
                    source="measured (MEASURED_PEAKS.json)")
    except Exception:
        return dict(hbm_gbs=6650.0, sm_max_mhz=1965.0, source="fallback")


# ----------------------------------------------------------------------------- models

def ss_bytes(B, L, D, es, mode):
    """Algorithmic bytes of one forward (+ backward) pass."""
    E = B * L * D
    bc = B * L * NSTATE * es
    params = (D * NSTATE + D) * es
    fwd = 3 * E * es + 2 * bc + params
    if mode in ("fwd", "stream"):
        return fwd + (2 * B * D * NSTATE * es)  # h_prev in / h_last out
    bwd = 5 * E * es + 4 * bc + 2 * params
    return fwd + bwd


def ss_ex2(B, L, D, mode):
    E = B * L * D
    return 16 * E * (2 if mode == "fwdbwd" else 1)


# ----------------------------------------------------------------------------- inputs

def make_ss_inputs(cfg, dev, seed, L=None, D=None, B=None):
    B = cfg["B"] if B is None else B
    L = cfg["L"] if L is None else L
    D = cfg["D"] if D is None else D
    g = torch.Generator(device=dev).manual_seed(seed)
    f32 = torch.float32
    n1 = torch.arange(1, NSTATE + 1, dtype=f32, device=dev)

    def rn(*s):
        return torch.randn(*s, generator=g, device=dev, dtype=f32)

    dist = cfg["dist"]
    if dist in ("c1", "c3"):
        u, delta = rn(B, L, D), torch.nn.functional.softplus(rn(B, L, D) * 0.5 - 1.0)
        A, Bm, Cm, Dv = -n1.repeat(D, 1), rn(B, L, NSTATE), rn(B, L, NSTATE), torch.ones(D, device=dev)
    elif dist == "c2":
        u, delta = rn(B, L, D), torch.nn.functional.softplus(rn(B, L, D) * 0.5 - 2.0)
        A = -n1.repeat(D, 1) * (1 + 0.1 * torch.rand(D, NSTATE, generator=g, device=dev))
        Bm, Cm = rn(B, L, NSTATE) / 4, rn(B, L, NSTATE) / 4
        Dv = 0.5 + torch.rand(D, generator=g, device=dev)
    else:  # c4
        u, delta = rn(B, L, D), torch.nn.functional.softplus(rn(B, L, D) * 0.5 - 3.0)
        A, Bm, Cm, Dv = -(n1 / 16).repeat(D, 1), rn(B, L, NSTATE), rn(B, L, NSTATE), torch.ones(D, device=dev)
    dt = cfg["dtype"]
    return [t.to(dt).contiguous() for t in (u, delta, A, Bm, Cm, Dv)], rn(B, L, D).to(dt)


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
               0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown",
               0x100: "display_clock_setting"}

    def __init__(self, index):
        self.index = index
        self.samples = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._t = None
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                self.reasons |= nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            except Exception:
                pass
            time.sleep(0.002)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._t is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        names = [n for bit, n in self.REASONS.items() if self.reasons & bit and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


# ----------------------------------------------------------------------------- timing

def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if args.impl == "b200" else "gloo"
        if args.impl == "b200":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return world, rank, local


def barrier_sync(world, dev):
    if world > 1:
        import torch.distributed as dist
        t = torch.zeros(1, device=dev)
        dist.all_reduce(t)
    torch.cuda.synchronize(dev)


def max_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def sum_over_ranks(x, world, dev):
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


# ----------------------------------------------------------------------------- CPU side

def host_threads():
    """Host CPUs this process may run on (the thread count both CPU baselines use: torchrun
    exports OMP_NUM_THREADS=1, so the count is set explicitly, not inherited)."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def cpu_record():
    """The CPU baseline's host record: CPU model, logical CPUs, CPUs available to us."""
    model = ""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    return {"cpu_model": model, "os_cpu_count": os.cpu_count(), "cpus_available": host_threads()}


def oracle_sample(cfg, target_s, seed=0):
    """Time the float64 CPU restatement of the reference path (oracle/, OpenMP over channels,
    all host CPUs) on an L-slice of the workload sized to ~target_s seconds. Returns
    (seconds, bytes, sample_desc, threads)."""
    from oracle import oracle as O
    O.set_threads(host_threads())
    B, D = cfg["B"], cfg["D"]
    es = torch.tensor([], dtype=cfg["dtype"]).element_size()

    def run(Ls):
        if cfg["mode"] == "pscan":   # linear recurrence along L of (B, D, L, 1)
            g = torch.Generator().manual_seed(seed)
            a = (torch.rand(B, D, Ls, 1, generator=g) * 0.1 + 0.9).double().numpy()
            x = torch.randn(B, D, Ls, 1, generator=g).double().numpy()
            t0 = time.perf_counter()
            O.lin_fwd(a, x)
            return time.perf_counter() - t0
        (u, delta, A, Bm, Cm, Dv), gy = make_ss_inputs(cfg, "cpu", seed, L=Ls)
        nst = cfg.get("nstate", NSTATE)
        if nst != NSTATE:   # the N-state workload: A = -(n+1) for n < N, B / C (B, L, N)
            g = torch.Generator().manual_seed(seed + 1)
            A = -torch.arange(1, nst + 1, dtype=torch.float64).repeat(D, 1)
            Bm, Cm = torch.randn(B, Ls, nst, generator=g), torch.randn(B, Ls, nst, generator=g)
        n = [t.double().numpy() for t in (u, delta, A, Bm, Cm, Dv)]
        t0 = time.perf_counter()
        O.ss_fwd(*n)
        if cfg["mode"] == "fwdbwd":
            O.ss_bwd(*n, gy.double().numpy())
        return time.perf_counter() - t0

    probe = 16
    t = run(probe)
    Ls = int(min(cfg["L"], max(16, probe * target_s / max(t, 1e-6))))
    secs = run(Ls)
    if cfg["mode"] == "pscan":
        nbytes = 12 * B * D * Ls
        desc = f"B={B} D={D} L={Ls} (of {cfg['L']}) slice, float64 oracle linear recurrence"
    else:
        nbytes = ss_bytes(B, Ls, D, es, cfg["mode"])
        desc = (f"B={B} L={Ls} (of {cfg['L']}) D={D} slice, float64 oracle on "
                f"{'fp16-valued' if es == 2 else 'fp32'} inputs, fwd{'+bwd' if cfg['mode'] == 'fwdbwd' else ''}")
    return secs, nbytes, desc, O.num_threads()


def torch_ref_sample(cfg, target_s, seed=0):
    """Time the reference's own PyTorch CPU path on an L-slice of the workload: the package's
    restatement of ``selective_scan_ref`` (the reference's mamba_cuda.py:875-946 with the time
    axis of its einsum fixed) run forward and then backward through torch autograd, in float32
    with torch.set_num_threads(all host CPUs); ``parallel_scan_ref`` (pscan.py:153-171) for the
    linear-recurrence workload. Returns (seconds, bytes, sample_desc, threads) with bytes by the
    workload's byte model, so the GB/s compares with the other arms."""
    from mamba_windows_cuda.mamba_cuda import selective_scan_ref
    from mamba_windows_cuda.pscan import parallel_scan_ref
    nthr = host_threads()
    torch.set_num_threads(nthr)
    B, D = cfg["B"], cfg["D"]
    es = torch.tensor([], dtype=cfg["dtype"]).element_size()

    def run(Ls):
        if cfg["mode"] == "pscan":
            g = torch.Generator().manual_seed(seed)
            a = torch.rand(B, D, Ls, 1, generator=g) * 0.1 + 0.9
            x = torch.randn(B, D, Ls, 1, generator=g)
            t0 = time.perf_counter()
            parallel_scan_ref(a, x)
            return time.perf_counter() - t0
        (u, delta, A, Bm, Cm, Dv), gy = make_ss_inputs(cfg, "cpu", seed, L=Ls)
        leaves = [t.float().requires_grad_(cfg["mode"] == "fwdbwd") for t in (u, delta, A, Bm, Cm, Dv)]
        t0 = time.perf_counter()
        out, _ = selective_scan_ref(*leaves)
        if cfg["mode"] == "fwdbwd":
            out.backward(gy.float())
        return time.perf_counter() - t0

    run(8)   # first call: thread pool and allocator warm-up
    # autograd over the Python time loop grows faster than linearly in L: double the slice
    # while it takes under ~40% of the target, and keep the last measurement
    Ls = 16
    secs = run(Ls)
    while secs < 0.4 * target_s and 2 * Ls <= cfg["L"]:
        Ls *= 2
        secs = run(Ls)
    if cfg["mode"] == "pscan":
        nbytes = 12 * B * D * Ls
        desc = f"B={B} D={D} L={Ls} (of {cfg['L']}) slice, parallel_scan_ref float32 on CPU"
    else:
        nbytes = ss_bytes(B, Ls, D, es, cfg["mode"])
        desc = (f"B={B} L={Ls} (of {cfg['L']}) D={D} slice, selective_scan_ref float32 fwd"
                f"{' + autograd bwd' if cfg['mode'] == 'fwdbwd' else ''} on CPU")
    return secs, nbytes, desc, nthr


def cpu_baseline_record(cfg, port_s, torch_s, seed=0):
    """The cpu_baseline object: the oracle port timed on all host CPUs (the reported value),
    with the reference's PyTorch CPU path timed beside it as the anchor and the CPU record."""
    secs, nbytes, desc, threads = oracle_sample(cfg, port_s, seed=seed)
    rec = {"value": nbytes / secs / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
           "sample": desc, **cpu_record(), "torch_threads": torch.get_num_threads()}
    if cfg["mode"] in ("fwdbwd", "fwd", "pscan"):
        ts, tb, tdesc, tthr = torch_ref_sample(cfg, torch_s, seed=seed)
        rec["torch_reference"] = {"value": tb / ts / 1e9, "unit": "GB/s", "threads": tthr,
                                  "sample": tdesc}
        rec["port_over_torch_reference"] = rec["value"] / rec["torch_reference"]["value"]
        rec["torch_threads"] = torch.get_num_threads()
    return rec


def reference_arm(args, cfg):
    """Times the reference algorithm on the host's CPUs: the float64 C port in oracle/ (the
    reference's CPU algorithm, OpenMP over channels) with every available CPU, each step a
    bounded L-slice of the workload; the reference's PyTorch CPU path is timed once beside it."""
    from oracle import oracle as O
    O.build()
    per_step = max(0.2, 90.0 / max(1, args.steps + args.warmup))
    times = []
    for i in range(args.warmup + args.steps):
        s2, b2, desc, threads = oracle_sample(cfg, per_step, seed=i)
        if i >= args.warmup:
            times.append((s2, b2))
    tot_s = sum(t for t, _ in times)
    tot_b = sum(b for _, b in times)
    gbs = tot_b / tot_s / 1e9
    base = {"value": gbs, "unit": "GB/s", "cores": threads, "kind": "port", "sample": desc,
            **cpu_record(), "torch_threads": torch.get_num_threads()}
    if cfg["mode"] in ("fwdbwd", "fwd", "pscan"):
        ts, tb, tdesc, tthr = torch_ref_sample(cfg, 10.0)
        base["torch_reference"] = {"value": tb / ts / 1e9, "unit": "GB/s", "threads": tthr,
                                   "sample": tdesc}
        base["port_over_torch_reference"] = gbs / base["torch_reference"]["value"]
    line = {
        "impl": "reference", "metric": cfg.get("metric", METRIC), "value": gbs, "unit": "GB/s",
        "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * tot_s / len(times),
        "higher_is_better": True, "scaling": "strong" if cfg["mode"] == "stream" else "weak",
        "vs_baseline": None, "dtype": "f64",
        "data": "synthetic (seeded, BASELINE distributions)",
        "config": {"workload": cfg["workload"], "B": cfg["B"], "L": cfg["L"], "D": cfg["D"],
                   "N": NSTATE, "sample_per_step": desc},
        "cpu_baseline": base,
        "e2e": {"value": gbs, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# ----------------------------------------------------------------------------- GPU arms

def scan_launches(B, L, D, es, dev):
    """(forward, backward) kernel launches of one scan call, by the library's own rule:
    B*D/128 chains >= SMs run the chained persistent kernels (1 forward; backward + its
    finalize); fewer chains with 16-byte rows and L >= 512 run the split passes (state-only
    pass, fold, seeded pass; adjoint-only pass, fold, seeded backward, finalize); other
    shapes the generic kernels (forward + fixup when L is segmented; backward + finalize).
    The bench's inputs are 16-byte aligned."""
    from mamba_windows_cuda import _lib
    nch = B * ((D + 127) // 128)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    if nch >= sms:
        return 1, 2
    if (D * es) % 16 == 0 and L >= 512:
        return 3, 4
    seg = int(_lib.load().mwc_ss_fwd_workspace_bytes(B, L, D, 0 if es == 4 else 1)) > 0
    return (2 if seg else 1), 2


def bench_fwdbwd(args, cfg, dev, world, rank, peaks):
    import mamba_windows_cuda as mwc
    B, L, D = cfg["B"], cfg["L"], cfg["D"]
    ins, gy = make_ss_inputs(cfg, dev, seed=1000 + rank)
    es = ins[0].element_size()
    block = cfg.get("block", False)
    nst = cfg.get("nstate", NSTATE)   # states per channel (16 except the N-state config)
    if block:
        # block form: delta is the pre-activation, plus z (B, L, D) and delta_bias (D)
        from mamba_windows_cuda.selective_scan_interface import selective_scan_fn
        gen = torch.Generator(device=dev).manual_seed(2000 + rank)
        ins[1] = (torch.randn(B, L, D, generator=gen, device=dev) * 0.5 - 1.0).to(cfg["dtype"])
        ins = ins + [torch.randn(B, L, D, generator=gen, device=dev).to(cfg["dtype"]),
                     (torch.randn(D, generator=gen, device=dev) * 0.3).to(cfg["dtype"])]

        def mod(*a):
            return selective_scan_fn(*a[:6], z=a[6], delta_bias=a[7], delta_softplus=True)
    elif cfg.get("groups", 1) > 1:
        # grouped B / C (B, L, G, 16): channel d reads group d // (D // G)
        from mamba_windows_cuda.grouped import selective_scan_grouped
        gen = torch.Generator(device=dev).manual_seed(2000 + rank)
        ins[3], ins[4] = [torch.randn(B, L, cfg["groups"], NSTATE, generator=gen, device=dev).to(cfg["dtype"])
                          for _ in range(2)]
        mod = selective_scan_grouped
    elif nst != NSTATE:
        # N states per channel: A = -(n+1) for n < N, B / C (B, L, N); N / 16 slices of 16 states
        from mamba_windows_cuda.nstate import selective_scan_nstate
        gen = torch.Generator(device=dev).manual_seed(2000 + rank)
        n1 = torch.arange(1, nst + 1, dtype=torch.float32, device=dev)
        ins[2] = (-n1.repeat(D, 1)).to(cfg["dtype"])
        ins[3], ins[4] = [torch.randn(B, L, nst, generator=gen, device=dev).to(cfg["dtype"]) for _ in range(2)]
        mod = selective_scan_nstate
    else:
        mod = mwc.SelectiveScanCuda()
    leaves = [t.clone().requires_grad_(True) for t in ins]
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        for t in leaves:
            t.grad = None
        if ev is not None:
            ev[0].record(stream)
        out = mod(*leaves)
        if ev is not None:
            ev[1].record(stream)
        out.backward(gy)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(world, dev)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(evs[i])
        stop.record(stream)
        torch.cuda.synchronize(dev)
    barrier_sync(world, dev)
    ms = start.elapsed_time(stop)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    ms_max = max_over_ranks(ms, world, dev)
    nbytes = ss_bytes(B, L, D, es, "fwdbwd")
    if block:   # + z read and out_z written (fwd); z, ungated out read and dz written (bwd)
        nbytes += 5 * B * L * D * es + 2 * D * es
    value = nbytes * world / (ms_max / args.steps / 1e3) / 1e9
    # our kernels per step: the forward scan (+ its carry fixup on the segmented path), the
    # backward scan + its finalize; the block form adds the delta transform and the gate in
    # both directions and the ddelta / dbias pair
    fk, bk = scan_launches(B, L, D, es, dev)
    launches_per_step = (fk + bk) * (nst // NSTATE) + (6 if block else 0)

    # roofline of the dominant kernel (the backward: reverse scan + its fixed-order reduction)
    mufu_peak = 148 * 16 * peaks["sm_max_mhz"] * 1e6  # ex2 / s at the max SM clock
    E = B * L * D
    bwd_bytes = ss_bytes(B, L, D, es, "fwdbwd") - ss_bytes(B, L, D, es, "fwd") + 2 * B * D * nst * es
    fwd_bytes = nbytes - bwd_bytes

    def roof(nb, nex2, t_ms):
        t = t_ms / 1e3
        return dict(hbm_gbs=nb / t / 1e9, hbm_frac=nb / t / 1e9 / peaks["hbm_gbs"],
                    ex2_per_s=nex2 / t, mufu_frac=nex2 / t / mufu_peak,
                    frac=max(nb / (peaks["hbm_gbs"] * 1e9), nex2 / mufu_peak) / t)

    rb = roof(bwd_bytes, nst * E, bwd_ms)   # one ex2 per element and state in each pass
    rf = roof(fwd_bytes, nst * E, fwd_ms)
    rs = roof(nbytes, 32 * E, ms / args.steps)
    traffic = CAPTURED_TRAFFIC.get(args.config)
    roofline = {
        "kernel": "ss_bwd_persistent_kernel + ss_bwd_persistent_final_kernel (backward op)",
        "bound": "mufu", "achieved": rb["ex2_per_s"] / 1e9, "peak": mufu_peak / 1e9,
        "unit": "Gex2/s", "frac": rb["mufu_frac"],
        "traffic": traffic["bytes"] if traffic else None,
        "traffic_source": traffic["source"] if traffic else None,
        "hbm": {"achieved": rb["hbm_gbs"], "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": rb["hbm_frac"], "peak_source": peaks["source"]},
        "model": f"max(algorithmic bytes / HBM, {nst} ex2 per element / MUFU at 148 SM x 16/clk x sm_max_mhz)",
        "per_op_ms": {"fwd": fwd_ms, "bwd": bwd_ms},
        "fwd_frac": rf["frac"], "step_frac": rs["frac"],
    }

    # e2e through the public API from pinned host memory
    host_in = [t.detach().cpu().pin_memory() for t in ins] + [gy.cpu().pin_memory()]
    host_out = [torch.empty(t.shape, dtype=t.dtype).pin_memory() for t in ins]

    def e2e_op(xs):
        leaves_d = [x.detach().requires_grad_(True) for x in xs[:-1]]
        mod(*leaves_d).backward(xs[-1])
        return [x.grad for x in leaves_d]

    e2e = _e2e(args, world, dev, host_in, host_out, e2e_op, nbytes)
    return dict(value=value, ms_per_step=ms_max / args.steps, roofline=roofline, e2e=e2e,
                clocks=clk.summary(), gpu_launches=launches_per_step * args.steps,
                dtype="f32", io_dtype=str(cfg["dtype"]).replace("torch.", ""))


def bench_stream(args, cfg, dev, world, rank, peaks):
    """Config 4: forward over a 2^20-token sequence (16 chunks of 65536), B=1, D=2048, fp32.

    N=1: the chunks run in order through ``SelectiveScanCuda.forward_with_state`` (h_prev ->
    h_last), the reference's streaming use. N>1: sequence sharding (strong scaling, the
    sequence is fixed): rank r owns chunks split_range(16, N, r) as one contiguous range and
    runs ``sharding.sequence_sharded_forward`` (local scan from zero, NCCL all-gather of the
    float32 (decay, end state) pairs, carry fold, ``mwc_ss_fixup``)."""
    import mamba_windows_cuda as mwc
    from mamba_windows_cuda import sharding as S
    B, Lc, D, nch = cfg["B"], cfg["L"], cfg["D"], cfg["chunks"]
    c0, c1 = S.split_range(nch, world, rank)
    Lr = (c1 - c0) * Lc
    ins, _ = make_ss_inputs(cfg, dev, seed=3000 + rank, L=Lr)
    u, delta, A, Bm, Cm, Dv = ins
    es = u.element_size()
    h0 = torch.zeros(B, D, NSTATE, dtype=cfg["dtype"], device=dev) if rank == 0 else None
    mod = mwc.SelectiveScanCuda()
    stream = torch.cuda.current_stream(dev)

    if world == 1:
        def step():
            h = h0
            with torch.no_grad():
                for c in range(nch):
                    sl = slice(c * Lc, (c + 1) * Lc)
                    _, h = mod.forward_with_state(u[:, sl], delta[:, sl], A, Bm[:, sl], Cm[:, sl], Dv, h)
            return h
        launches = nch * scan_launches(B, Lc, D, es, dev)[0]
    else:
        def step():
            with torch.no_grad():
                _, h = S.sequence_sharded_forward(u, delta, A, Bm, Cm, Dv, h0)
            return h
        launches = scan_launches(B, Lr, D, es, dev)[0] + (1 if rank > 0 else 0)

    for _ in range(args.warmup):
        step()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(world, dev)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        start.record(stream)
        for _ in range(args.steps):
            step()
        stop.record(stream)
        torch.cuda.synchronize(dev)
    barrier_sync(world, dev)
    ms = start.elapsed_time(stop)
    ms_max = max_over_ranks(ms, world, dev)
    Ltot = Lc * nch
    nbytes = ss_bytes(B, Ltot, D, es, "stream")
    value = nbytes / (ms_max / args.steps / 1e3) / 1e9
    mufu_peak = 148 * 16 * peaks["sm_max_mhz"] * 1e6
    t_rank = ms / args.steps / 1e3
    ex2_rank = 16 * B * Lr * D
    bytes_rank = ss_bytes(B, Lr, D, es, "stream")
    roofline = {
        "kernel": "forward scan of this rank's range (ss_fwd_kernel + ss_fixup_kernel, L-segmented)",
        "bound": "mufu", "achieved": ex2_rank / t_rank / 1e9, "peak": mufu_peak / 1e9,
        "unit": "Gex2/s", "frac": ex2_rank / t_rank / mufu_peak, "traffic": None,
        "hbm": {"achieved": bytes_rank / t_rank / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": bytes_rank / t_rank / 1e9 / peaks["hbm_gbs"], "peak_source": peaks["source"]},
        "model": "per rank: 16 ex2 per element of its range / MUFU; step time includes the "
                 "carry exchange and fixup for N > 1",
    }
    e2e = {"value": None, "unit": "GB/s", "h2d_bytes_per_step": None, "d2h_bytes_per_step": None,
           "note": "not measured for config 4: its 25.8 GB of fp32 inputs per step are "
                   "generated on the device; the host-buffer e2e line is config 3's"}
    return dict(value=value, ms_per_step=ms_max / args.steps, roofline=roofline, e2e=e2e,
                clocks=clk.summary(), gpu_launches=launches * args.steps, dtype="f32",
                io_dtype=str(cfg["dtype"]).replace("torch.", ""), scaling="strong",
                parallelism=(f"sequence-sharded x{world}: chunks {c0}..{c1 - 1} on rank {rank}, "
                             "NCCL all-gather of (decay, end state) + carry fixup")
                if world > 1 else "single GPU, 16 chunks chained through h_prev / h_last",
                l2=f"{3 * B * Lr * D * es / 1e9:.1f} GB of u / delta / y per rank per step, "
                   "far above the 126 MB L2; no flush")


def measure_sharded(args, dev, world, rank):
    """The north star's multi-GPU workloads, measured beside the headline at every N (strong
    scaling: the total work is fixed, so ms per step should fall as 1/N).

    * config 4, sequence-sharded: the 2^20-token fp32 streaming forward (B=1, D=2048) split
      along L, rank r owning chunks split_range(16, N, r); per step every rank runs
      sharding.sequence_sharded_forward (local scan from zero, NCCL all-gather of the float32
      (decay, end state) pairs, carry fold, mwc_ss_fixup). Reported: ms per step (max over
      ranks, CUDA events), GB/s of the whole sequence, the per-phase times (max over ranks)
      and the speed-up against the single-GPU run of the same sequence as 16 chained
      forward_with_state calls (the reference's streaming use), timed on rank 0.
    * config 2, batch split: the B=8 inference forward_with_state with batch rows
      split_range(8, N, r) on rank r; no exchange.
    """
    import mamba_windows_cuda as mwc
    from mamba_windows_cuda import sharding as S
    steps, warm = max(3, min(args.steps, 10)), 3
    stream = torch.cuda.current_stream(dev)
    mod = mwc.SelectiveScanCuda()
    out = {}

    # ---- config 4: sequence sharding
    cfg = CONFIGS["c4"]
    B, Lc, D, nch = cfg["B"], cfg["L"], cfg["D"], cfg["chunks"]
    es = torch.tensor([], dtype=cfg["dtype"]).element_size()
    nbytes = ss_bytes(B, Lc * nch, D, es, "stream")

    def chained(u, delta, A, Bm, Cm, Dv):
        h = torch.zeros(B, D, NSTATE, dtype=cfg["dtype"], device=dev)
        with torch.no_grad():
            for c in range(nch):
                sl = slice(c * Lc, (c + 1) * Lc)
                _, h = mod.forward_with_state(u[:, sl], delta[:, sl], A, Bm[:, sl], Cm[:, sl], Dv, h)
        return h

    def time_fn(fn, n=None, w=None):
        n, w = n or steps, w or warm
        for _ in range(w):
            fn()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(n):
            fn()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / n

    t1 = None
    if world == 1 or rank == 0:   # the single-GPU chained run of the whole sequence
        ins, _ = make_ss_inputs(cfg, dev, seed=3000, L=Lc * nch)
        t1 = time_fn(lambda: chained(*ins))
        del ins
        torch.cuda.empty_cache()
    barrier_sync(world, dev)
    rec = {"workload": "config 4: 2^20-token fp32 streaming forward (B=1, D=2048), sequence-sharded "
                       "along L across the ranks",
           "ranks": world, "scaling": "strong", "unit": "GB/s"}
    if world == 1:
        rec.update(ms_per_step=t1, value=nbytes / (t1 / 1e3) / 1e9, one_gpu_chained_ms=t1,
                   speedup_vs_one_gpu_chained=1.0,
                   note="one GPU: the 16 chunks chained through h_prev / h_last")
    else:
        c0, c1 = S.split_range(nch, world, rank)
        ins, _ = make_ss_inputs(cfg, dev, seed=3000 + rank, L=(c1 - c0) * Lc)
        h0 = torch.zeros(B, D, NSTATE, dtype=cfg["dtype"], device=dev) if rank == 0 else None
        names = ("local", "gather", "fold", "fixup")
        evs = [{k: torch.cuda.Event(enable_timing=True) for k in ("start",) + names}
               for _ in range(steps)]

        def sharded(ev=None):
            hook = None
            if ev is not None:
                ev["start"].record(stream)
                hook = lambda name: ev[name].record(stream)   # noqa: E731
            with torch.no_grad():
                S.sequence_sharded_forward(*ins, h0, phase_hook=hook)

        for _ in range(warm):
            sharded()
        barrier_sync(world, dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for i in range(steps):
            sharded(evs[i])
        e1.record(stream)
        torch.cuda.synchronize(dev)
        barrier_sync(world, dev)
        ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
        prev = ("start",) + names
        ph = [statistics.mean(e[prev[j]].elapsed_time(e[prev[j + 1]]) for e in evs) for j in range(4)]
        import torch.distributed as dist
        pt = torch.tensor(ph, dtype=torch.float64, device=dev)
        dist.all_reduce(pt, op=dist.ReduceOp.MAX)
        t1 = max_over_ranks(t1 if t1 is not None else 0.0, world, dev)
        rec.update(ms_per_step=ms, value=nbytes / (ms / 1e3) / 1e9, one_gpu_chained_ms=t1,
                   speedup_vs_one_gpu_chained=t1 / ms,
                   phases_ms_max_over_ranks=dict(zip(names, [float(v) for v in pt.tolist()])),
                   note="phases: local scan of the rank's chunks (+ fp32 carry record), NCCL "
                        "all-gather of (decay, end state), carry fold (one linear-scan launch), "
                        "mwc_ss_fixup; the all-gather includes waiting for the slowest rank")
        del ins
        torch.cuda.empty_cache()
    out["c4_sequence_sharded"] = rec

    # ---- config 4's first TRAIN_CHUNKS chunks trained (forward + backward) across the ranks
    if world > 1:
        out["c4_sequence_sharded_training"] = _sharded_training(cfg, dev, world, rank, steps, warm,
                                                                stream, mod, time_fn)

    # ---- config 2: batch rows split across the ranks
    cfg = CONFIGS["c2"]
    Bt, L, D = cfg["B"], cfg["L"], cfg["D"]
    es = torch.tensor([], dtype=cfg["dtype"]).element_size()
    b0, b1 = S.split_range(Bt, world, rank)
    ms = 0.0
    if b1 > b0:
        ins, _ = make_ss_inputs(cfg, dev, seed=4000 + rank, B=b1 - b0)

        def fwd():
            with torch.no_grad():
                return mod.forward_with_state(*ins)

        ms = time_fn(fwd, n=max(steps, 50), w=10)   # a 0.4 ms step: time as many as the headline
        del ins
    barrier_sync(world, dev)
    ms = max_over_ranks(ms, world, dev)
    out["c2_batch_split"] = {
        "workload": "config 2: B=8 L=2048 D=4096 fp16 inference forward_with_state, batch rows "
                    "split across the ranks (no exchange)",
        "ranks": world, "rows_per_rank": f"{Bt // world}-{-(-Bt // world)}", "scaling": "strong",
        "ms_per_step": ms, "value": ss_bytes(Bt, L, D, es, "fwd") / (ms / 1e3) / 1e9, "unit": "GB/s"}
    return out


TRAIN_CHUNKS = 4   # 2^18 tokens: per-rank ranges up to 2^28 elements at D = 2048


def _sharded_training(cfg, dev, world, rank, steps, warm, stream, mod, time_fn):
    """Forward + backward of sharding.sequence_sharded_scan over config 4's first
    TRAIN_CHUNKS chunks split along L (rank r owns split_range(tokens, N, r)), against the
    same tokens trained on one GPU (rank 0) as TRAIN_CHUNKS chained 65,536-step calls with
    h_prev / h_last and autograd through the chain."""
    from mamba_windows_cuda import sharding as S
    from mamba_windows_cuda.mamba_cuda import SelectiveScanCudaFunction
    B, Lc, D = cfg["B"], cfg["L"], cfg["D"]
    Lt = Lc * TRAIN_CHUNKS
    a, b = S.split_range(Lt, world, rank)
    ins, gy = make_ss_inputs(cfg, dev, seed=3100 + rank, L=b - a)
    leaves = [t.clone().requires_grad_(True) for t in ins]

    def step():
        for t in leaves:
            t.grad = None
        o, _ = S.sequence_sharded_scan(*leaves, None)
        o.backward(gy)

    for _ in range(warm):
        step()
    barrier_sync(world, dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(e0.elapsed_time(e1) / steps, world, dev)
    del ins, gy, leaves
    torch.cuda.empty_cache()
    t1 = 0.0
    if rank == 0:
        ins, gy = make_ss_inputs(cfg, dev, seed=3100, L=Lt)
        leaves = [t.clone().requires_grad_(True) for t in ins]

        def one_gpu():
            for t in leaves:
                t.grad = None
            u, delta, A, Bm, Cm, Dv = leaves
            h, outs = None, []
            for c in range(TRAIN_CHUNKS):
                sl = slice(c * Lc, (c + 1) * Lc)
                o, h = SelectiveScanCudaFunction.apply(u[:, sl], delta[:, sl], A, Bm[:, sl], Cm[:, sl], Dv, h)
                outs.append(o)
            torch.cat(outs, dim=1).backward(gy)

        t1 = time_fn(one_gpu)
        del ins, gy, leaves
        torch.cuda.empty_cache()
    barrier_sync(world, dev)
    t1 = max_over_ranks(t1, world, dev)
    es = torch.tensor([], dtype=cfg["dtype"]).element_size()
    return {"workload": f"config 4's first {TRAIN_CHUNKS} chunks ({Lt} tokens, fp32, B=1, D=2048) trained: "
                        "forward + backward of sharding.sequence_sharded_scan, split along L",
            "ranks": world, "scaling": "strong", "ms_per_step": ms,
            "value": ss_bytes(B, Lt, D, es, "fwdbwd") / (ms / 1e3) / 1e9, "unit": "GB/s",
            "one_gpu_chained_ms": t1, "speedup_vs_one_gpu_chained": t1 / ms if ms > 0 else None,
            "note": "collectives per step: one all-gather (forward), one all-gather and one "
                    "all-reduce (backward); one GPU: the chunks chained through h_prev / h_last"}


_JSON_FD = None


def emit(line):
    """Write the one JSON result line to the process's original stdout."""
    data = (json.dumps(line) + "\n").encode()
    if _JSON_FD is None:
        sys.stdout.write(data.decode())
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, data)


def _timed(args, world, dev, fn):
    """Warm-up, then K timed calls bracketed by events on the current stream; returns the
    max-over-ranks milliseconds of the K calls and the clock summary."""
    stream = torch.cuda.current_stream(dev)
    for _ in range(args.warmup):
        fn()
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(world, dev)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        start.record(stream)
        for _ in range(args.steps):
            fn()
        stop.record(stream)
        torch.cuda.synchronize(dev)
    barrier_sync(world, dev)
    return max_over_ranks(start.elapsed_time(stop), world, dev), clk.summary()


def _e2e(args, world, dev, host_in, host_out, fn_dev, nbytes):
    """Same op through host buffers, as a training or inference loop feeds it: every step
    copies its inputs host -> device from pinned memory, runs the op through the public API
    and copies its results device -> host, all inside the timed region. The copies run on
    their own streams, so step i+1's inputs load (into the other of two device buffer sets)
    while step i computes and step i-1's results drain; PCIe carries both directions at
    once. fn_dev gets the step's device inputs and returns the device outputs."""
    comp = torch.cuda.current_stream(dev)
    s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    bufs = [[torch.empty(h.shape, dtype=h.dtype, device=dev) for h in host_in] for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]

    def load(j):
        with torch.cuda.stream(s_in):
            s_in.wait_event(free[j])   # the op that last read buffer set j is done
            for bd, h in zip(bufs[j], host_in):
                bd.copy_(h, non_blocking=True)
            ready[j].record(s_in)

    def run(n):
        for j in range(2):
            free[j].record(comp)
        s_in.wait_stream(comp)
        load(0)
        for i in range(n):
            j = i % 2
            if i + 1 < n:
                load((i + 1) % 2)
            comp.wait_event(ready[j])
            outs = fn_dev(bufs[j])
            free[j].record(comp)
            s_out.wait_stream(comp)
            with torch.cuda.stream(s_out):
                for ho, o in zip(host_out, outs):
                    o.record_stream(s_out)   # keep the result alive until its copy is done
                    ho.copy_(o, non_blocking=True)
        comp.wait_stream(s_out)

    # 40 steps: the first step's input copy and the last step's result copy are not
    # overlapped, a fixed cost of about one step's copies per run (config 3: 7.9 ms)
    steps = 40
    run(2)
    torch.cuda.synchronize(dev)
    barrier_sync(world, dev)
    s2, t2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s2.record(comp)
    run(steps)
    t2.record(comp)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(s2.elapsed_time(t2), world, dev) / steps
    return {"value": nbytes * world / (ms / 1e3) / 1e9, "unit": "GB/s",
            "h2d_bytes_per_step": sum(t.numel() * t.element_size() for t in host_in),
            "d2h_bytes_per_step": sum(t.numel() * t.element_size() for t in host_out), "ms_per_step": ms,
            "overlap": "step i+1 host->device and step i-1 device->host copies overlap step i"}


def bench_fwd(args, cfg, dev, world, rank, peaks):
    """Config 2: inference forward_with_state (h0 = 0, returns out and h_last), fp16; each
    rank its own batch (batch x D tiles at N GPUs, no exchange)."""
    import mamba_windows_cuda as mwc
    B, L, D = cfg["B"], cfg["L"], cfg["D"]
    ins, _ = make_ss_inputs(cfg, dev, seed=4000 + rank)
    es = ins[0].element_size()
    mod = mwc.SelectiveScanCuda()

    def op(xs):
        with torch.no_grad():
            return mod.forward_with_state(*xs)

    ms, clk = _timed(args, world, dev, lambda: op(ins))
    nbytes = ss_bytes(B, L, D, es, "fwd")
    t = ms / args.steps / 1e3
    mufu_peak = 148 * 16 * peaks["sm_max_mhz"] * 1e6
    ex2 = 16 * B * L * D
    roofline = {"kernel": "ss_fwd_persistent_kernel (forward, h_last out)", "bound": "mufu",
                "achieved": ex2 / t / 1e9, "peak": mufu_peak / 1e9, "unit": "Gex2/s",
                "frac": ex2 / t / mufu_peak, "traffic": None,
                "hbm": {"achieved": nbytes / t / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                        "frac": nbytes / t / 1e9 / peaks["hbm_gbs"], "peak_source": peaks["source"]},
                "model": "max(algorithmic bytes / HBM, 16 ex2 per element / MUFU)"}
    host_in = [x.cpu().pin_memory() for x in ins]
    host_out = [torch.empty(ins[0].shape, dtype=ins[0].dtype).pin_memory(),
                torch.empty((B, D, NSTATE), dtype=ins[0].dtype).pin_memory()]
    e2e = _e2e(args, world, dev, host_in, host_out, op, nbytes)
    return dict(value=nbytes * world / t / 1e9, ms_per_step=ms / args.steps, roofline=roofline,
                e2e=e2e, clocks=clk, gpu_launches=1 * args.steps, dtype="f32",
                io_dtype=str(cfg["dtype"]).replace("torch.", ""),
                parallelism=f"batch tiles x{world}: one independent batch per rank, no collective")


def bench_pscan(args, cfg, dev, world, rank, peaks):
    """Config 5: parallel_scan_fn, H_t = A_t H_{t-1} + X_t along L of (B, D, L, 1), fp32;
    HBM-bound (read A, X, write H: 12 bytes per element)."""
    from mamba_windows_cuda import parallel_scan_fn
    B, L, D = cfg["B"], cfg["L"], cfg["D"]
    gen = torch.Generator(device=dev).manual_seed(5000 + rank)
    A = torch.rand(B, D, L, 1, generator=gen, device=dev) * 0.1 + 0.9
    X = torch.randn(B, D, L, 1, generator=gen, device=dev)

    def op(xs):
        with torch.no_grad():
            return (parallel_scan_fn(*xs),)

    ms, clk = _timed(args, world, dev, lambda: op((A, X)))
    E = B * D * L
    nbytes = 12 * E
    t = ms / args.steps / 1e3
    roofline = {"kernel": "lin_fwd_kernel (warp-shuffle scan of affine maps)", "bound": "hbm",
                "achieved": nbytes / t / 1e9, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": nbytes / t / 1e9 / peaks["hbm_gbs"], "traffic": None,
                "peak_source": peaks["source"], "model": "12 bytes per element (A, X read; H written)"}
    host_in = [A.cpu().pin_memory(), X.cpu().pin_memory()]
    host_out = [torch.empty(A.shape, dtype=A.dtype).pin_memory()]
    e2e = _e2e(args, world, dev, host_in, host_out, op, nbytes)
    return dict(value=nbytes * world / t / 1e9, ms_per_step=ms / args.steps, roofline=roofline,
                e2e=e2e, clocks=clk, gpu_launches=1 * args.steps, dtype="f32", io_dtype="float32",
                l2=f"{nbytes / 1e9:.1f} GB per step, far above the 126 MB L2; no flush",
                parallelism=f"replicas x{world}: one independent scan per rank, no collective")


def bench_conv(args, cfg, dev, world, rank, peaks):
    """Causal conv1d (width 4, SiLU) forward + backward: HBM-bound (x read, y written;
    x, dy read, dx written: 10 bytes per fp16 element, plus the weight / bias partials).
    Roofline: the backward op (TMA-staged kernel + fixed-order weight reduction, the larger
    share of the step), timed with events on the launching stream over back-to-back C-ABI
    calls."""
    from mamba_windows_cuda.causal_conv1d import causal_conv1d_fn
    B, L, D = cfg["B"], cfg["L"], cfg["D"]
    gen = torch.Generator(device=dev).manual_seed(6000 + rank)
    dt = cfg["dtype"]
    x = torch.randn(B, L, D, generator=gen, device=dev).to(dt).requires_grad_(True)
    w = (torch.randn(D, 4, generator=gen, device=dev) * 0.5).to(dt).requires_grad_(True)
    b = (torch.randn(D, generator=gen, device=dev) * 0.1).to(dt).requires_grad_(True)
    dy = torch.randn(B, L, D, generator=gen, device=dev).to(dt)
    stream = torch.cuda.current_stream(dev)

    def step(ev=None):
        for t in (x, w, b):
            t.grad = None
        if ev is not None:
            ev[0].record(stream)
        y = causal_conv1d_fn(x, w, b, "silu")
        if ev is not None:
            ev[1].record(stream)
        y.backward(dy)
        if ev is not None:
            ev[2].record(stream)

    for _ in range(args.warmup):
        step()
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier_sync(world, dev)
    with ClockSampler(dev.index if dev.index is not None else 0) as clk:
        start.record(stream)
        for i in range(args.steps):
            step(evs[i])
        stop.record(stream)
        torch.cuda.synchronize(dev)
    barrier_sync(world, dev)
    ms = max_over_ranks(start.elapsed_time(stop), world, dev)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in evs)
    # The autograd step leaves the GPU idle while Python runs between the two ops, so the
    # kernels' own durations come from back-to-back C-ABI calls on preallocated buffers
    # (the backward op: the TMA kernel + the weight reduction; inputs > L2 between calls).
    from mamba_windows_cuda import _lib
    from mamba_windows_cuda._ops import _p, dtype_code
    lib = _lib.load()
    sh = ctypes.c_void_p(stream.cuda_stream)
    xd, wd, bd = x.detach(), w.detach(), b.detach()
    yk = torch.empty_like(xd)
    dxk, dwk, dbk = torch.empty_like(xd), torch.empty_like(wd), torch.empty_like(bd)
    wsb = int(lib.mwc_conv1d_bwd_workspace_bytes(B, L, D, 4))
    wsk = torch.empty(max(wsb, 1), dtype=torch.uint8, device=dev)
    dc = dtype_code(xd)

    def kfwd():
        return lib.mwc_conv1d_fwd(_p(xd), _p(wd), _p(bd), None, 1, _p(yk), B, L, D, 4, dc, sh)

    def kbwd():
        return lib.mwc_conv1d_bwd(_p(xd), _p(wd), _p(bd), None, 1, _p(dy), _p(dxk), _p(dwk), _p(dbk), None,
                                  _p(wsk), wsb, B, L, D, 4, dc, sh)

    kms = {}
    for name, fn in (("fwd", kfwd), ("bwd", kbwd)):
        for _ in range(3):
            assert fn() == 0, name
        k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        k0.record(stream)
        for _ in range(args.steps):
            fn()
        k1.record(stream)
        torch.cuda.synchronize(dev)
        kms[name] = k0.elapsed_time(k1) / args.steps
    es = x.element_size()
    E = B * L * D
    nbytes = 10 * E * es // 2
    bwd_bytes = 3 * E * es + 4 * D * es * 2   # x, dy read, dx written; weights in, dweight out
    t = ms / args.steps / 1e3
    achieved = bwd_bytes / (kms["bwd"] / 1e3) / 1e9
    roofline = {"kernel": "conv1d_bwd_tma_kernel + conv1d_reduce_kernel (backward op)",
                "bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                "frac": achieved / peaks["hbm_gbs"],
                "traffic": CAPTURED_TRAFFIC["conv"]["bytes"] if args.config == "conv" else None,
                "traffic_source": CAPTURED_TRAFFIC["conv"]["source"] if args.config == "conv" else None,
                "peak_source": peaks["source"],
                "model": "x, dy read + dx written (3 x 2 B per fp16 element)",
                "kernel_ms": kms, "per_op_ms_in_step": {"fwd": fwd_ms, "bwd": bwd_ms},
                "fwd_frac": 2 * E * es / (kms["fwd"] / 1e3) / 1e9 / peaks["hbm_gbs"]}
    xh, dyh = x.detach().cpu().pin_memory(), dy.cpu().pin_memory()
    dxh = torch.empty(x.shape, dtype=dt).pin_memory()

    def op(xs):
        xi = xs[0].detach().requires_grad_(True)
        causal_conv1d_fn(xi, w, b, "silu").backward(xs[1])
        return (xi.grad,)

    e2e = _e2e(args, world, dev, [xh, dyh], [dxh], op, nbytes)
    return dict(value=nbytes * world / t / 1e9, ms_per_step=ms / args.steps, roofline=roofline, e2e=e2e,
                clocks=clk.summary(), gpu_launches=3 * args.steps, dtype="f32",
                io_dtype=str(dt).replace("torch.", ""),
                parallelism=f"replicas x{world}: one independent batch per rank, no collective")


def main():
    global _JSON_FD
    # Keep stdout for the JSON line alone: libraries that print banners to fd 1 (NCCL's
    # version line, for one) are sent to stderr.
    sys.stdout.flush()
    _JSON_FD = os.dup(1)
    os.dup2(2, 1)
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["b200", "reference"], default="b200")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="c3")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the sequence-sharded config-4 and batch-split config-2 measurements")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    world, rank, local = dist_setup(args)
    peaks = load_peaks()

    if args.impl == "reference":
        if rank == 0:
            reference_arm(args, cfg)
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()
        return

    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if cfg["mode"] == "stream":
        res = bench_stream(args, cfg, dev, world, rank, peaks)
    elif cfg["mode"] == "fwd":
        res = bench_fwd(args, cfg, dev, world, rank, peaks)
    elif cfg["mode"] == "pscan":
        res = bench_pscan(args, cfg, dev, world, rank, peaks)
    elif cfg["mode"] == "conv":
        res = bench_conv(args, cfg, dev, world, rank, peaks)
    elif cfg["mode"] == "fwdbwd":
        res = bench_fwdbwd(args, cfg, dev, world, rank, peaks)
    else:
        raise SystemExit(f"--config {args.config}: mode {cfg['mode']} is covered by the tests; "
                         "bench.py measures the fwd+bwd (c1, c3) and streaming (c4) workloads")

    line = {
        "metric": cfg.get("metric", METRIC), "value": res["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": res["ms_per_step"],
        "higher_is_better": True, "scaling": res.get("scaling", "weak"), "vs_baseline": None,
        "dtype": res["dtype"], "data": "synthetic (seeded, BASELINE distributions, generated on device)",
        "config": {"workload": cfg["workload"], "B": cfg["B"], "L": cfg["L"], "D": cfg["D"],
                   "N": cfg.get("nstate", NSTATE), "groups": cfg.get("groups", 1), "io_dtype": res["io_dtype"],
                   "l2": res.get("l2", "inputs + outputs per step (~250 MB at config 3) exceed the "
                                       "126 MB L2; no flush"),
                   "parallelism": res.get("parallelism", f"replicas x{world}: one independent "
                                                         "batch per rank, no collective")},
        "roofline": res["roofline"], "e2e": res["e2e"], "gpu_launches": res["gpu_launches"],
        "clocks": res["clocks"],
    }
    if args.config == "c3" and not args.no_sharded:
        line["sharded"] = measure_sharded(args, dev, world, rank)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_record(cfg, 10.0, 8.0)
    if rank == 0:
        emit(line)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
