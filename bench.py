"""Benchmark of the fused drafter-loss hot path on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Default workload (per GPU): D-PACE forward + backward over fp32 logits
[N=64, B=16, V=128256] ~ N(0, 2^2), uniform targets, per-sequence prefix mask
k ~ U{0..4}, alpha 0.5, loss_type "dpace" -- the Llama-3-vocabulary
configuration the metric is quoted on. With N GPUs every rank holds its own 64
sequences of a 64*N-sequence batch (weak scaling): the loss divisor is the
global N and the only collective is one 4-byte NCCL all_reduce of the loss
per step. A step = forward (+ all_reduce) + backward through the C ABI with
inputs resident in HBM; two input sets alternate, each larger than L2.

Metric: fwd+bwd logits GB/s = 12 * N*B*V bytes (forward read, backward read,
backward write) / step time, summed over GPUs; rows/s alongside.

--impl reference times the reference's CPU path (its torch oracle,
losses/dpace_ref.py, restated in oracle/dpace.py) on the host cores with all
threads, on a bounded sample of the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "cuda-spec-decode_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "fwd+bwd logits GB/s (% of B200 HBM peak) at V=128256; rows/s at 1/2/4/8 GPU"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0


# ----------------------------------------------------------------------------- helpers

def hbm_peak():
    p = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured (MEASURED_PEAKS.json hbm_gbs)"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback (no MEASURED_PEAKS.json)"


def profiled_traffic(kernel: str, workload: str):
    """DRAM bytes per launch from a committed ncu summary (profiles/traffic.txt)."""
    p = os.path.join(REPO, "profiles", "traffic.txt")
    try:
        for line in open(p):
            parts = line.split()
            if len(parts) >= 3 and parts[0] == kernel and parts[1] == workload:
                return float(parts[2])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples while the GPU is under load."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: torch.device):
        uuid = str(getattr(torch.cuda.get_device_properties(device), "uuid", "") or "")
        self.index = (uuid if uuid.startswith("GPU-") else f"GPU-{uuid}") if uuid else str(device.index)
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.QUERY}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.thread.join(timeout=2)
        sm, smax, power, reasons = [], [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
                power.append(float(f[3]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "power_w_max": max(power) if power else None,
                "samples": len(sm), "reasons": sorted(reasons)}


def dpace_inputs(N, B, V, sigma, kmax, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(N, B, V, device=device, generator=g).mul_(sigma)
    t = torch.randint(0, V, (N, B), device=device, generator=g)
    k = torch.randint(0, kmax + 1, (N, 1), device=device, generator=g)
    m = (torch.arange(B, device=device).view(1, B) >= k).float()
    return x, t, m


def dflash_inputs(N, B, V, seed, device):
    g = torch.Generator(device=device).manual_seed(seed)
    x = torch.randn(N, B, V, device=device, generator=g).mul_(2.0)
    y = x + torch.randn(N, B, V, device=device, generator=g)
    return x, y


# ----------------------------------------------------------------------------- reference arm

def cpu_oracle_step_dpace(x, t, m):
    """One fwd+bwd of the reference's torch algorithm; x is a leaf with requires_grad."""
    from oracle.dpace import dpace_loss_torch

    x.grad = None
    loss = dpace_loss_torch(x, t, 0.5, m)
    loss.backward()
    return float(loss.detach())


def cpu_sample(N_s, B, V, seed=0):
    x, t, m = dpace_inputs(N_s, B, V, 2.0, 4, seed, torch.device("cpu"))
    return x.requires_grad_(True), t, m


def time_cpu_baseline(B, V, budget_s=10.0, N_s=4):
    """Reference torch oracle fwd+bwd on the host cores over a bounded sample."""
    torch.set_num_threads(os.cpu_count() or 1)
    x, t, m = cpu_sample(N_s, B, V)
    cpu_oracle_step_dpace(x, t, m)  # warm-up
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        cpu_oracle_step_dpace(x, t, m)
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    E = N_s * B * V
    return {"value": round(12 * E / sec / 1e9, 4), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"D-PACE fwd+bwd via the reference's torch oracle algorithm (oracle/dpace.py) "
                      f"on [{N_s},{B},{V}] of the workload, median of {len(times)} runs",
            "rows_per_s": round(N_s * B / sec, 1), "ms_per_step": round(sec * 1e3, 2)}


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    B, V, N_s = 16, 128256, 4
    x, t, m = cpu_sample(N_s, B, V)
    for _ in range(args.warmup):
        cpu_oracle_step_dpace(x, t, m)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_oracle_step_dpace(x, t, m)
    sec = (time.perf_counter() - t0) / args.steps
    E = N_s * B * V
    val = 12 * E / sec / 1e9
    line = {"metric": METRIC, "value": round(val, 4), "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "dpace_fwd_bwd_llama3_vocab", "N": N_s, "B": B, "V": V,
                       "sigma": 2.0, "mask": "prefix k~U{0..4}", "alpha": 0.5,
                       "loss_type": "dpace", "sample_of": "[64,16,128256] per GPU"},
            "rows_per_s": round(N_s * B / sec, 1),
            "cpu_baseline": {"value": round(val, 4), "unit": UNIT,
                             "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"[{N_s},{B},{V}] of the [64,16,128256] workload per step"},
            "e2e": {"value": round(val, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- our arm

def time_dflash(args, dev, stream, world, n_global, max_over_ranks, barrier):
    """DFlash objective (KL), draft [64, 16, 128256] ~ N(0, 2^2), verifier =
    draft + N(0, 1), gamma 4, anchor slot unscored, every slot masked in.
    Bytes model 20 * N*B*V per step (forward reads both, backward reads both
    and writes the gradient); required bytes skip the zero-weight anchor rows."""
    from specdec import ops

    N, B, V = args.n, 16, 128256
    E = N * B * V
    sets = [dflash_inputs(N, B, V, 2000 * s + int(os.environ.get("RANK", "0")), dev) for s in range(2)]
    grad = torch.empty(N, B, V, device=dev)

    def step(i, ev=None):
        x, y = sets[i & 1]
        if ev is not None:
            ev[0].record(stream)
        loss, _, scale, lzq, lzp, _ = ops.dflash_forward(x, y, None, 4.0, False, 0, B, n_global)
        if ev is not None:
            ev[1].record(stream)
        if world > 1:
            import torch.distributed as dist
            dist.all_reduce(loss)
        if ev is not None:
            ev[2].record(stream)
        ops.dflash_backward(x, y, scale, lzq, lzp, None, None, 0, out=grad)
        if ev is not None:
            ev[3].record(stream)

    for i in range(args.warmup):
        step(i)
    K = args.dflash_steps
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(K)]
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    a.record(stream)
    for k in range(K):
        step(k, evs[k])
    b.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    ms = max_over_ranks(a.elapsed_time(b)) / K
    fwd = max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in evs))
    bwd = max_over_ranks(statistics.mean(e[2].elapsed_time(e[3]) for e in evs))
    live = 15.0 / 16.0
    peak, _ = hbm_peak()
    bwd_bytes = 8.0 * E * live + 4.0 * E
    fwd_bytes = 8.0 * E * live
    wl = f"{N}x{B}x{V}"
    value = 20.0 * E * world / (ms * 1e-3) / 1e9
    return {"metric": "DFlash-KL fwd+bwd logits GB/s (20*N*B*V bytes per GPU-step)",
            "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "rows_per_s": round(N * B * world / (ms * 1e-3), 1),
            "pct_of_hbm_peak": round(100.0 * value / world / peak, 2),
            "fwd_ms": round(fwd, 4), "bwd_ms": round(bwd, 4), "steps": K,
            "config": {"workload": "dflash_kl_fwd_bwd_llama3_vocab", "N_per_gpu": N, "B": B, "V": V,
                       "draft": "N(0, 2^2)", "verifier": "draft + N(0, 1)", "gamma": 4.0,
                       "sample_from_anchor": False, "mask": "all ones"},
            "roofline": {"kernel": "dflash_bwd_ring_kernel<KL>", "bound": "hbm",
                         "achieved": round(bwd_bytes / (bwd * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(bwd_bytes / (bwd * 1e-3) / 1e9 / peak, 4),
                         "traffic": profiled_traffic("dflash_bwd_kl", wl), "bytes_per_launch": bwd_bytes},
            "fwd_roofline": {"kernel": "dflash_fwd_ring_kernel<KL> + finalize",
                             "achieved": round(fwd_bytes / (fwd * 1e-3) / 1e9, 1),
                             "frac": round(fwd_bytes / (fwd * 1e-3) / 1e9 / peak, 4),
                             "traffic": profiled_traffic("dflash_fwd_kl", wl), "bytes_per_launch": fwd_bytes}}


def run_ours(args):
    import torch.distributed as dist
    from datetime import timedelta

    from specdec import _lib, ops

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=120))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    N, B, V = args.n, 16, 128256
    E = N * B * V
    n_global = N * world
    sets = [dpace_inputs(N, B, V, 2.0, 4, 1000 * s + rank, dev) for s in range(2)]
    live = [float(m.sum()) / (N * B) for (_, _, m) in sets]
    grad = torch.empty(N, B, V, device=dev)
    stream = torch.cuda.current_stream(dev)
    # ring kernels (16-byte-aligned inputs): forward = streaming + finalize, backward = 1
    launches_per_step = 3 if all(x.data_ptr() % 16 == 0 for x, _, _ in sets) else 2

    def step(i, ev=None):
        x, t, m = sets[i & 1]
        if ev is not None:
            ev[0].record(stream)
        loss, lse, scale, _ = ops.dpace_forward(x, t, m, 0.5, 0, n_global=n_global, validate=False)
        if ev is not None:
            ev[1].record(stream)
        if world > 1:
            dist.all_reduce(loss)
        if ev is not None:
            ev[2].record(stream)
        ops.dpace_backward(x, t, lse, scale, None, out=grad)
        if ev is not None:
            ev[3].record(stream)
        return loss

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(dev)
    sampler.start()
    t_soak = time.perf_counter() + args.soak
    i = 0
    while time.perf_counter() < t_soak:
        step(i)
        i += 1
        if i % 64 == 0:
            torch.cuda.synchronize(dev)

    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    start.record(stream)
    for k in range(args.steps):
        step(k, evs[k])
    stop.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ms_local = start.elapsed_time(stop)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    ms = max_over_ranks(ms_local)
    fwd_ms_max, bwd_ms_max = max_over_ranks(fwd_ms), max_over_ranks(bwd_ms)
    dflash = None
    if args.dflash_steps > 0:
        dflash = time_dflash(args, dev, stream, world, n_global, max_over_ranks, barrier)
    ms_step = ms / args.steps
    total_bytes = 12.0 * E * world
    value = total_bytes / (ms_step * 1e-3) / 1e9
    rows_s = N * B * world / (ms_step * 1e-3)

    # roofline of the dominant kernel (the backward): bytes it must move per launch
    peak, peak_src = hbm_peak()
    live_frac = statistics.mean(live)
    bwd_bytes = 4.0 * E * live_frac + 4.0 * E
    fwd_bytes = 4.0 * E * live_frac
    wl = f"{N}x{B}x{V}"
    roof_bwd = {"kernel": "dpace_bwd_kernel", "bound": "hbm", "achieved": round(bwd_bytes / (bwd_ms_max * 1e-3) / 1e9, 1),
                "peak": peak, "unit": "GB/s", "traffic": profiled_traffic("dpace_bwd", wl),
                "bytes_per_launch": bwd_bytes, "peak_source": peak_src}
    roof_bwd["frac"] = round(roof_bwd["achieved"] / peak, 4)
    roof_fwd = {"kernel": "dpace_fwd_kernel", "achieved": round(fwd_bytes / (fwd_ms_max * 1e-3) / 1e9, 1),
                "bytes_per_launch": fwd_bytes, "traffic": profiled_traffic("dpace_fwd", wl)}
    roof_fwd["frac"] = round(roof_fwd["achieved"] / peak, 4)

    # end to end through the public API: pinned host inputs -> dpace_loss -> backward -> loss to host
    e2e = None
    if args.e2e_steps > 0:
        from losses import dpace_loss

        hx = [s[0].cpu().pin_memory() for s in sets]
        ht = [s[1].cpu().pin_memory() for s in sets]
        hm = [s[2].cpu().pin_memory() for s in sets]
        hloss = torch.empty((), dtype=torch.float32).pin_memory()

        def e2e_step(i):
            x = hx[i & 1].to(dev, non_blocking=True).requires_grad_(True)
            t = ht[i & 1].to(dev, non_blocking=True)
            m = hm[i & 1].to(dev, non_blocking=True)
            loss = dpace_loss(x, t, 0.5, m)
            loss.backward()
            hloss.copy_(loss.detach(), non_blocking=True)
            return x

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        barrier()
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        for i in range(args.e2e_steps):
            e2e_step(i)
        s1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(s0.elapsed_time(s1)) / args.e2e_steps
        h2d = hx[0].numel() * 4 + ht[0].numel() * 8 + hm[0].numel() * 4
        e2e = {"value": round(total_bytes / (e2e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": 4 + 4,
               "ms_per_step": round(e2e_ms, 3), "steps": args.e2e_steps,
               "path": "losses.dpace.dpace_loss(...).backward() from pinned host buffers; "
                       "includes the target-range check (4-byte read-back)"}

    cpu_base = None
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        cpu_base = time_cpu_baseline(B, V, args.cpu_budget)

    if world > 1:
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {"metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "dpace_fwd_bwd_llama3_vocab", "N_per_gpu": N, "B": B, "V": V,
                       "global_N": n_global, "sigma": 2.0, "mask": "prefix k~U{0..4}",
                       "alpha": 0.5, "loss_type": "dpace", "parallelism": f"dp{world} (N-sharded)",
                       "l2": "two alternating input sets, each 525 MB > 126 MB L2",
                       "bytes_model": "12*N*B*V per GPU-step"},
            "rows_per_s": round(rows_s, 1),
            "pct_of_hbm_peak": round(100.0 * value / world / peak, 2),
            "roofline": roof_bwd,
            "kernels": {"dpace_fwd_ms": round(fwd_ms_max, 4), "dpace_bwd_ms": round(bwd_ms_max, 4),
                        "fwd": roof_fwd,
                        "launches_per_step": launches_per_step,
                        "fwd_note": "forward = streaming kernel + PDL-chained finalize kernel"},
            "dflash_kl": dflash,
            "live_row_fraction": round(live_frac, 4),
            "cpu_baseline": cpu_base, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps, "gpu_launches_scope": "per rank",
            "clocks": clocks}
    print(json.dumps(line), flush=True)
    return 0


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=10)
    p.add_argument("--impl", choices=("ours", "reference"), default="ours")
    p.add_argument("--n", type=int, default=64, help="sequences per GPU")
    p.add_argument("--soak", type=float, default=1.0, help="seconds of untimed load before timing")
    p.add_argument("--e2e-steps", type=int, default=20)
    p.add_argument("--dflash-steps", type=int, default=100,
                   help="timed steps of the DFlash-KL workload (0 = skip)")
    p.add_argument("--cpu-budget", type=float, default=10.0,
                   help="seconds of CPU-oracle timing on rank 0 at N=1 (0 = skip)")
    args = p.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
