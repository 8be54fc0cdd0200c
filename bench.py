"""Benchmark of the fused drafter-loss hot path on B200.

    python bench.py [--gpus N --steps K --warmup W] [--impl ours|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Headline workload (per GPU): D-PACE forward + backward over fp32 logits
[N=64, B=16, V=128256] ~ N(0, 2^2), uniform targets, per-sequence prefix mask
k ~ U{0..4}, alpha 0.5, loss_type "dpace" -- the Llama-3-vocabulary
configuration the metric is quoted on. With N GPUs every rank holds its own 64
sequences of a 64*N-sequence batch (weak scaling): the loss divisor is the
global N and the only collective is one 4-byte NCCL all_reduce of the loss
per step. A step = specdec_dpace_forward_backward through the C ABI (loss and
gradient in one call; the backward is chained to the forward's finalize) with
inputs resident in HBM; two input sets alternate, each larger than L2.

Metric: fwd+bwd logits GB/s = 12 * N*B*V bytes (forward read, backward read,
backward write) / step time, summed over GPUs; rows/s alongside. The bytes a
step actually moves are fewer (unscored rows are never read):
moved_bytes_per_step and pct_of_hbm_peak use those.

Other legs in the same line: the large-batch workload [512, 32, 151936]
~ N(0, 3^2), prefix mask k ~ U{0..8}, its 512 sequences split across the N
GPUs (strong scaling, "c4"); the DFlash objective (KL) at [64, 16, 128256];
bf16 logits; the end-to-end drafter training step; the same D-PACE metric
end to end from pinned host memory through the public API ("e2e").

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
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    # communicator set-up lines (rank count per communicator) in the log; set
    # before torch loads NCCL, which reads them once
    os.environ.setdefault("NCCL_DEBUG", "INFO")
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
sys.path.insert(0, os.path.join(REPO, "cuda-spec-decode_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

from specdec.dist import LossReducer  # noqa: E402

METRIC = "fwd+bwd logits GB/s (% of B200 HBM peak) at V=128256; rows/s at 1/2/4/8 GPU"
UNIT = "GB/s"
FALLBACK_HBM_GBS = 6650.0
# B200 HBM3e data-sheet bandwidth (DGX figure): a second, fixed denominator.
# The measured peak is a device-to-device copy, which this path's read-heavy
# kernels can exceed.
SPEC_HBM_GBS = 8000.0


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


def time_cpu_baseline_dflash(B, V, budget_s=10.0, N_s=4):
    """The reference's DFlash CPU path -- its speculators oracle (loss_function
    + kl_div_loss, models/dflash/tests/test_loss.py:21-49, restated in
    oracle/dflash.py) -- fwd+bwd on the host cores over a bounded sample of
    the DFlash-KL workload; 20*E bytes per step like the GPU leg."""
    from oracle.dflash import dflash_loss_torch

    torch.set_num_threads(os.cpu_count() or 1)
    x, y = dflash_inputs(N_s, B, V, 0, torch.device("cpu"))
    x.requires_grad_(True)

    def step():
        x.grad = None
        loss = dflash_loss_torch(x, y, None, 4.0, False, "kl")
        loss.backward()

    step()
    times = []
    t_end = time.perf_counter() + budget_s
    while time.perf_counter() < t_end or len(times) < 3:
        t0 = time.perf_counter()
        step()
        times.append(time.perf_counter() - t0)
    sec = statistics.median(times)
    E = N_s * B * V
    return {"value": round(20 * E / sec / 1e9, 4), "unit": UNIT, "cores": torch.get_num_threads(),
            "kind": "port",
            "sample": f"DFlash-KL fwd+bwd via the reference's speculators oracle (oracle/dflash.py) on "
                      f"[{N_s},{B},{V}] of the workload, median of {len(times)} runs",
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

def device_barrier_on(world, dev):
    """A 1-element all_reduce on the current stream: every rank's next event
    fires when it completes, so a rank whose host left the barrier late does
    not land its delay inside the other ranks' timed windows."""
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(torch.zeros(1, device=dev))


class Timing:
    """Per-rank timing context: the compute stream, the world, the max-over-
    ranks reduction, the host barrier and the loss reducer (NCCL all_reduce
    of the 4-byte loss on a side stream, or on the compute stream for
    --loss-reduce serial)."""

    def __init__(self, args, dev, world):
        import torch.distributed as dist

        self.args, self.dev, self.world = args, dev, world
        self.stream = torch.cuda.current_stream(dev)
        self.reducer = LossReducer(dev) if world > 1 and args.loss_reduce == "overlap" else None
        self._dist = dist

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=self.dev)
        self._dist.all_reduce(t, op=self._dist.ReduceOp.MAX)
        return float(t.item())

    def barrier(self):
        if self.world > 1:
            self._dist.barrier()

    def reduce(self, loss):
        """Starts the global loss reduction of a step (no-op on one GPU)."""
        if self.world == 1:
            return loss
        if self.reducer is not None:
            return self.reducer.start(loss)
        self._dist.all_reduce(loss)
        return loss

    def settle(self):
        """The compute stream waits for every loss reduction started so far."""
        if self.reducer is not None:
            self.reducer.wait()

    def loop(self, step, steps):
        """args.warmup untimed steps, then `steps` timed steps of step(i) in one
        event pair on the compute stream, behind a host and a device barrier.
        Returns (ms per step max over ranks, this rank's ms per step)."""
        for i in range(self.args.warmup):
            step(i)
        self.settle()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        self.barrier()
        torch.cuda.synchronize(self.dev)
        device_barrier_on(self.world, self.dev)
        a.record(self.stream)
        for k in range(steps):
            step(k)
        self.settle()
        b.record(self.stream)
        torch.cuda.synchronize(self.dev)
        self.barrier()
        local = a.elapsed_time(b) / steps
        return self.max(local), local

    def graphs(self, call, n_sets):
        """CUDA graphs of call(s) (the library launches of one step on input
        set s, returning its loss tensor), one per input set, captured on a
        side stream after eager warm-up calls there (so the workspace and the
        status words for that stream exist before capture). Returns
        step(i) = replay graph i % n_sets, then start the loss reduction
        (eager: no collective inside a graph)."""
        cap = torch.cuda.Stream(self.dev)
        cap.wait_stream(self.stream)
        with torch.cuda.stream(cap):
            for i in range(3 * n_sets):
                call(i % n_sets)
        self.stream.wait_stream(cap)
        torch.cuda.synchronize(self.dev)
        gs, outs = [], []
        for s_ in range(n_sets):
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                outs.append(call(s_))
            gs.append(g)
        torch.cuda.synchronize(self.dev)

        def step(i):
            gs[i % n_sets].replay()
            self.reduce(outs[i % n_sets])

        step.graphs = gs  # kept alive with the step function
        return step

    def split(self, fwd, bwd, steps, n_sets=1):
        """A second, instrumented pass: events around the forward call and the
        backward call of each step (separate calls, so no chaining between
        them). Returns (mean forward ms, mean backward ms), max over ranks.

        With --graphs 1 the forward and the backward of each input set are
        captured as two CUDA graphs of `reps` back-to-back calls each (after
        eager warm-up calls on the capture stream) and replayed between the
        events; a figure is the graph's time / reps, so it holds the calls'
        device time without a graph launch's latency. A ~1 ms device-side
        spin ahead of the first event lets the host's enqueueing run ahead of
        the GPU."""
        reps = 1
        if self.args.graphs:
            reps = 8
            cap = torch.cuda.Stream(self.dev)
            cap.wait_stream(self.stream)
            with torch.cuda.stream(cap):
                for i in range(2 * n_sets):
                    _, st = fwd(i % n_sets)
                    bwd(i % n_sets, st)
            self.stream.wait_stream(cap)
            torch.cuda.synchronize(self.dev)
            gf, gb, outs = [], [], []
            for s_ in range(n_sets):
                g1, g2 = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                with torch.cuda.graph(g1, stream=cap):
                    for _ in range(reps):
                        loss, st = fwd(s_)
                with torch.cuda.graph(g2, stream=cap):
                    for _ in range(reps):
                        bwd(s_, st)
                gf.append(g1)
                gb.append(g2)
                outs.append((loss, st))
            torch.cuda.synchronize(self.dev)

            def run_fwd(k):
                gf[k % n_sets].replay()
                return outs[k % n_sets]

            def run_bwd(k, st):
                gb[k % n_sets].replay()
        else:
            run_fwd, run_bwd = fwd, bwd
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
        torch.cuda._sleep(2_000_000)
        for k in range(steps):
            evs[k][0].record(self.stream)
            loss, state = run_fwd(k)
            evs[k][1].record(self.stream)
            self.reduce(loss)
            evs[k][2].record(self.stream)
            run_bwd(k, state)
            evs[k][3].record(self.stream)
            self.settle()
        torch.cuda.synchronize(self.dev)
        f = statistics.mean(e[0].elapsed_time(e[1]) for e in evs) / reps
        g = statistics.mean(e[2].elapsed_time(e[3]) for e in evs) / reps
        return self.max(f), self.max(g)


def roofline(kernel, nbytes, ms, peak, traffic=None, **extra):
    achieved = nbytes / (ms * 1e-3) / 1e9
    d = {"kernel": kernel, "bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
         "frac": round(achieved / peak, 4), "traffic": traffic, "bytes_per_launch": nbytes}
    d.update(extra)
    return d


def dpace_moved_bytes(E, live, esz):
    """Bytes a D-PACE step moves: forward reads the scored rows, backward
    re-reads them and writes every gradient element."""
    return esz * E * (2.0 * live + 1.0)


def time_dflash(args, T, n_global, dtype=torch.float32, steps=None):
    """DFlash objective (KL), draft [64, 16, 128256] ~ N(0, 2^2), verifier =
    draft + N(0, 1), gamma 4, anchor slot unscored, every slot masked in.
    Bytes model 20 * N*B*V per step for fp32 (forward reads both, backward
    reads both and writes the gradient), 10 * N*B*V for bf16; moved bytes
    skip the zero-weight anchor rows."""
    from specdec import ops

    dev, world = T.dev, T.world
    N, B, V = args.n, 16, 128256
    E = N * B * V
    esz = 2 if dtype == torch.bfloat16 else 4
    sets = []
    for s_ in range(2):
        x, y = dflash_inputs(N, B, V, 2000 * s_ + int(os.environ.get("RANK", "0")), dev)
        sets.append((x.to(dtype), y.to(dtype)))
        del x, y
    grad = torch.empty(N, B, V, device=dev, dtype=dtype)

    def fwd(i):
        x, y = sets[i & 1]
        loss, _, scale, lzq, lzp, _ = ops.dflash_forward(x, y, None, 4.0, False, 0, B, n_global)
        return loss, (scale, lzq, lzp)

    def bwd(i, st):
        x, y = sets[i & 1]
        ops.dflash_backward(x, y, st[0], st[1], st[2], None, None, 0, out=grad)

    def call(i):  # one step's launches: forward then backward (dloss = 1)
        loss, st = fwd(i)
        bwd(i, st)
        return loss

    K = args.dflash_steps if steps is None else steps
    ms, ms_local = T.loop(T.graphs(call, 2) if args.graphs else (lambda i: T.reduce(call(i))), K)
    f, g = T.split(fwd, bwd, K, 2)
    live = 15.0 / 16.0
    peak, _ = hbm_peak()
    bwd_bytes = 2.0 * esz * E * live + esz * E
    fwd_bytes = 2.0 * esz * E * live
    moved = fwd_bytes + bwd_bytes
    model = 5 * esz
    wl = f"{N}x{B}x{V}"
    tag = "_bf16" if esz == 2 else ""
    value = model * E * world / (ms * 1e-3) / 1e9
    del sets, grad
    kname = "bf16" if esz == 2 else "f32"
    return {"metric": f"DFlash-KL fwd+bwd logits GB/s ({model}*N*B*V bytes per GPU-step)",
            "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "ms_per_step_this_rank": round(ms_local, 4),
            "rows_per_s": round(N * B * world / (ms * 1e-3), 1),
            "moved_bytes_per_step": moved,
            "pct_of_hbm_peak": round(100.0 * moved / (ms * 1e-3) / 1e9 / peak, 2),
            "pct_basis": "moved bytes (anchor rows are not read) / ms_per_step / measured HBM peak",
            "pct_of_spec_8000": round(100.0 * moved / (ms * 1e-3) / 1e9 / SPEC_HBM_GBS, 2),
            "fwd_ms": round(f, 4), "bwd_ms": round(g, 4), "steps": K,
            "dtype": "bf16" if esz == 2 else "f32",
            "config": {"workload": f"dflash_kl_fwd_bwd_llama3_vocab{tag}", "N_per_gpu": N, "B": B, "V": V,
                       "draft": "N(0, 2^2)", "verifier": "draft + N(0, 1)", "gamma": 4.0,
                       "sample_from_anchor": False, "mask": "all ones",
                       "logits": "bf16 (fp32 arithmetic)" if esz == 2 else "fp32"},
            "roofline": roofline(f"dflash_bwd_ring_kernel<{kname}, KL>", bwd_bytes, g, peak,
                                 profiled_traffic(f"dflash_bwd_kl{tag}", wl)),
            "fwd_roofline": roofline(f"dflash_fwd_ring_kernel<{kname}, KL> + finalize", fwd_bytes, f, peak,
                                     profiled_traffic(f"dflash_fwd_kl{tag}", wl))}


def dpace_leg(args, T, N, B, V, sigma, kmax, n_global, steps, dtype=torch.float32, sets_n=2, seed0=1000):
    """Times a D-PACE workload: `steps` steps of specdec_dpace_forward_backward
    (plus the loss reduction when world > 1), then the instrumented split pass
    of separate forward / backward calls. Returns a dict of raw figures."""
    from specdec import ops

    dev = T.dev
    rank = int(os.environ.get("RANK", "0"))
    sets = []
    for s_ in range(sets_n):
        x, t, m = dpace_inputs(N, B, V, sigma, kmax, seed0 * s_ + rank, dev)
        sets.append((x if dtype == torch.float32 else x.to(dtype), t, m))
        del x
    live = statistics.mean(float(m.mean()) for _, _, m in sets)
    grad = torch.empty(N, B, V, device=dev, dtype=dtype)

    def call(i):  # one step's launches: specdec_dpace_forward_backward
        x, t, m = sets[i % sets_n]
        loss, _, _, _, _ = ops.dpace_forward_backward(x, t, m, 0.5, 0, n_global=n_global, validate=False,
                                                      out=grad)
        return loss

    step = T.graphs(call, sets_n) if args.graphs else (lambda i: T.reduce(call(i)))

    def fwd(i):
        x, t, m = sets[i % sets_n]
        loss, lse, scale, _ = ops.dpace_forward(x, t, m, 0.5, 0, n_global=n_global, validate=False)
        return loss, (lse, scale)

    def bwd(i, st):
        x, t, _ = sets[i % sets_n]
        ops.dpace_backward(x, t, st[0], st[1], None, out=grad)

    ms, ms_local = T.loop(step, steps)
    f, g = T.split(fwd, bwd, steps, sets_n)
    aligned = all(x.data_ptr() % 16 == 0 for x, _, _ in sets)
    out = {"ms": ms, "ms_local": ms_local, "fwd_ms": f, "bwd_ms": g, "live": live, "aligned": aligned}
    del sets, grad
    torch.cuda.empty_cache()
    return out


def dpace_report(r, N, B, V, world, esz, n_total_rows, peak, scaling, wl_tag=""):
    """Common fields of a D-PACE leg: model bytes 12E (or 6E for bf16) per
    GPU-step summed over GPUs, moved bytes, fractions of the measured peak,
    the backward kernel's roofline."""
    E = N * B * V
    ms = r["ms"]
    model_bytes = 3 * esz * E  # per GPU-step: forward read + backward read + write
    moved = dpace_moved_bytes(E, r["live"], esz)
    bwd_bytes = esz * E * r["live"] + esz * E
    fwd_bytes = esz * E * r["live"]
    kname = "bf16" if esz == 2 else "f32"
    wl = f"{N}x{B}x{V}"
    return {"value": round(model_bytes * world / (ms * 1e-3) / 1e9, 2), "ms_per_step": round(ms, 4),
            "ms_per_step_this_rank": round(r["ms_local"], 4),
            "rows_per_s": round(n_total_rows / (ms * 1e-3), 1),
            "moved_bytes_per_step": moved,
            "pct_of_hbm_peak": round(100.0 * moved / (ms * 1e-3) / 1e9 / peak, 2),
            "pct_basis": "moved bytes per GPU (unscored rows are not read) / ms_per_step / measured HBM peak",
            "pct_of_spec_8000": round(100.0 * moved / (ms * 1e-3) / 1e9 / SPEC_HBM_GBS, 2),
            "live_row_fraction": round(r["live"], 4),
            "roofline": roofline(f"dpace_bwd_ring_kernel<{kname}>", bwd_bytes, r["bwd_ms"], peak,
                                 profiled_traffic("dpace_bwd" + wl_tag, wl)),
            "fwd_roofline": roofline(f"dpace_fwd_ring_kernel<{kname}> + dpace_finalize_kernel", fwd_bytes,
                                     r["fwd_ms"], peak, profiled_traffic("dpace_fwd" + wl_tag, wl)),
            "split_ms": {"fwd": round(r["fwd_ms"], 4), "bwd": round(r["bwd_ms"], 4),
                         "note": "separate forward / backward calls with events between them"},
            "scaling": scaling}


def time_dpace_bf16(args, T, n_global):
    """D-PACE on bf16 logits, the headline workload otherwise: [64, 16, 128256]
    ~ N(0, 2^2) rounded to bf16, prefix mask k ~ U{0..4}, alpha 0.5. Bytes model
    6 * N*B*V per step (2-byte elements: forward read, backward read + write)."""
    N, B, V = args.n, 16, 128256
    r = dpace_leg(args, T, N, B, V, 2.0, 4, n_global, args.bf16_steps, dtype=torch.bfloat16)
    peak, _ = hbm_peak()
    d = {"metric": "D-PACE fwd+bwd bf16 logits GB/s (6*N*B*V bytes per GPU-step)", "unit": "GB/s",
         "steps": args.bf16_steps, "dtype": "bf16",
         "config": {"workload": "dpace_fwd_bwd_llama3_vocab_bf16", "N_per_gpu": N, "B": B, "V": V,
                    "sigma": 2.0, "mask": "prefix k~U{0..4}", "alpha": 0.5, "loss_type": "dpace",
                    "logits": "bf16 (fp32 arithmetic)", "step": "specdec_dpace_forward_backward_bf16"}}
    d.update(dpace_report(r, N, B, V, T.world, 2, N * B * T.world, peak, "weak", "_bf16"))
    return d


def time_c4(args, T):
    """The large-batch workload: [512, 32, 151936] fp32 ~ N(0, 3^2), uniform
    targets, per-sequence prefix mask k ~ U{0..8}, alpha 0.5, the 512
    sequences split contiguously across the ranks (strong scaling: 512/N per
    GPU, loss divisor 512, one 4-byte all_reduce per step). One input set:
    every shard (>= 1.2 GB at N = 8) is larger than L2."""
    from specdec.dist import shard_range

    rank = int(os.environ.get("RANK", "0"))
    NT, B, V = 512, 32, 151936
    lo, hi = shard_range(NT, rank, T.world)
    N = hi - lo
    r = dpace_leg(args, T, N, B, V, 3.0, 8, NT, args.c4_steps, sets_n=1, seed0=4000)
    peak, _ = hbm_peak()
    d = {"metric": "D-PACE fwd+bwd logits GB/s, large batch (12*N*B*V bytes per GPU-step, summed)",
         "unit": "GB/s", "steps": args.c4_steps, "dtype": "f32",
         "config": {"workload": "dpace_large_batch_strong_scaling", "N_total": NT, "N_per_gpu": N, "B": B,
                    "V": V, "sigma": 3.0, "mask": "prefix k~U{0..8}", "alpha": 0.5, "loss_type": "dpace",
                    "shards": f"contiguous, {T.world} ranks", "l2": "one input set, > 126 MB L2 per rank",
                    "step": "specdec_dpace_forward_backward"}}
    d.update(dpace_report(r, N, B, V, T.world, 4, NT, peak, "strong"))
    return d


def torch_ops_dpace_loss(logits, targets, alpha, mask):
    """D-PACE written with plain torch ops on the GPU (cross_entropy, exp,
    cumprod, reversed cumsum), the unfused way a user without this library
    would run the objective; used only as the end-to-end comparison."""
    N, B, V = logits.shape
    ce = torch.nn.functional.cross_entropy(logits.reshape(-1, V).float(), targets.reshape(-1),
                                           reduction="none").view(N, B)
    with torch.no_grad():
        live = (mask > 0).float()
        sm = torch.where(live > 0, (1 - alpha) * torch.exp(-ce) + alpha, torch.ones_like(ce))
        P = torch.cumprod(sm, dim=1)
        w = torch.flip(torch.cumsum(torch.flip(P * live, [1]), 1), [1]) * live
    return (ce * w).sum() / N


def time_drafter_step(args, dev, world, max_over_ranks, barrier):
    """End-to-end drafter training step around the loss hook: the DFlash
    drafter (d_target 4096, d_model 256, 3 layers, 4 heads, block 16) over
    target features [32, 512, 4096] with a frozen random lm_head [128256, 4096],
    D-PACE alpha 0.5 with the anchor slot masked out, AdamW + grad-norm clip
    as the reference pipeline's step; DDP across ranks when world > 1.
    Variants: the fused loss on fp32 logits, the same objective in plain torch
    ops on fp32 logits, a bf16 lm_head feeding the fused bf16-logits loss, and
    the whole drafter under bf16 autocast (fused SDPA kernels, bf16 GEMMs)
    feeding the fused bf16-logits loss. GEMMs run on cuBLAS (TF32 for fp32
    operands)."""
    import torch.nn as nn

    from losses import dpace_loss
    from models.dflash.model import DFlashSpeculator

    Nb, S, D, V, blk = 32, 512, 4096, 128256, 16
    prev_tf32 = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    torch.manual_seed(1234)
    head = nn.Linear(D, V, bias=False).to(dev)
    head_bf16 = nn.Linear(D, V, bias=False, dtype=torch.bfloat16).to(dev)
    with torch.no_grad():
        head_bf16.weight.copy_(head.weight)
    g = torch.Generator(device=dev).manual_seed(99 + int(os.environ.get("RANK", "0")))
    # the verifier's features are bf16; the fp32-logit variants take them widened to fp32 (the
    # reference loss is fp32-only), the bf16-autocast variants as they are
    feats_bf16 = torch.randn(Nb, S, D, device=dev, generator=g, dtype=torch.bfloat16)
    feats = feats_bf16.float()
    tokens = torch.randint(0, V, (Nb, blk), device=dev, generator=g)
    mask = torch.ones(Nb, blk, device=dev)
    mask[:, 0] = 0.0

    def build(lm_head, ddp):
        m = DFlashSpeculator(d_target=D, d_model=256, target_vocab_size=V, block_size=blk, num_layers=3,
                             num_heads=4, target_lm_head=lm_head).to(dev)
        if lm_head.weight.dtype == torch.bfloat16:
            # the drafter body stays fp32; its output feature enters the bf16 head in bf16
            m.final_norm.register_forward_hook(lambda _m, _i, out: out.to(torch.bfloat16))
        if ddp and world > 1:
            # gradients as views of the all-reduce buckets (no copy in or out), no buffer
            # broadcast (the drafter has none), and the same graph every step
            m = nn.parallel.DistributedDataParallel(m, device_ids=[dev.index], broadcast_buffers=False,
                                                    gradient_as_bucket_view=True, static_graph=True)
        return m

    def loss_fused(logits, tok):
        return dpace_loss(logits, tok, 0.5, position_mask=mask)

    def loss_torch(logits, tok):
        return torch_ops_dpace_loss(logits, tok, 0.5, mask)

    from specdec import drafter as layer_kernels
    from specdec.graphs import allreduce_grads

    # (name, lm_head, objective, autocast, the drafter's norms/attention on the library's kernels)
    variants = [("fused_loss_fp32_logits", head, loss_fused, False, True, False),
                ("torch_ops_loss_fp32_logits", head, loss_torch, False, False, False),
                ("fused_loss_bf16_logits", head_bf16, loss_fused, False, True, False),
                ("bf16_autocast_drafter_fused_loss", head_bf16, loss_fused, True, True, False),
                ("bf16_autocast_drafter_torch_layers_fused_loss", head_bf16, loss_fused, True, False, False)]
    # the same step captured once as a CUDA graph (specdec.graphs.GraphedStep) and replayed; with
    # N > 1 the gradient all-reduce (one NCCL call on the flat gradient) is captured with it
    variants.append(("bf16_autocast_drafter_fused_loss_graphed", head_bf16, loss_fused, True, True, True))
    out = {}
    stream = torch.cuda.current_stream(dev)
    for name, lm_head, lfn, autocast, kernels, graphed in variants:
        layer_kernels.set_enabled(kernels)
        model = build(lm_head, ddp=not graphed)
        core = model.module if (world > 1 and not graphed) else model
        params = [p for p in model.parameters() if p.requires_grad]
        # the graphed step runs the fused AdamW kernel (capturable): the capturable foreach form
        # is ~60 elementwise launches per step, ~0.8 ms at this size
        opt = torch.optim.AdamW(params, lr=1e-3, capturable=graphed, fused=graphed)

        def step_fn(f_in, t_in):
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast, cache_enabled=not graphed):
                loss = core.compute_loss(f_in, t_in, loss_fn=lfn) if (world == 1 or graphed) else \
                    lfn(model(f_in), t_in)
            loss.backward()
            if graphed and world > 1:
                allreduce_grads(params)
            torch.nn.utils.clip_grad_norm_(params, 1.0)
            opt.step()
            return loss

        if graphed:
            from specdec.graphs import GraphedStep

            gstep = GraphedStep(step_fn, feats_bf16 if autocast else feats, tokens, optimizers=(opt,))
            step = gstep
        else:
            gstep = None

            def step():
                return step_fn(feats_bf16 if autocast else feats, tokens)

        for _ in range(3):
            step()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize(dev)
        device_barrier_on(world, dev)
        a.record(stream)
        for _ in range(args.drafter_steps):
            loss = step()
        b.record(stream)
        torch.cuda.synchronize(dev)
        barrier()
        if gstep is not None:
            gstep.check()
        ms = max_over_ranks(a.elapsed_time(b)) / args.drafter_steps
        out[name] = {"ms_per_step": round(ms, 3), "rows_per_s": round(Nb * blk * world / (ms * 1e-3), 1),
                     "loss": round(float(loss.detach()), 6), "library_layers": kernels,
                     "cuda_graph": graphed}
        # the graph (with its NCCL all-reduce for N > 1) is released here, well before the
        # process group is destroyed
        del model, core, opt, params, gstep, step, step_fn, loss
        torch.cuda.synchronize(dev)
        torch.cuda.empty_cache()
    layer_kernels.set_enabled(True)
    torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    del head, head_bf16, feats, feats_bf16
    torch.cuda.empty_cache()
    base = out["torch_ops_loss_fp32_logits"]["ms_per_step"]
    for v in out.values():
        v["speedup_vs_torch_ops_loss"] = round(base / v["ms_per_step"], 3)
    return {"metric": "drafter training step (fwd + loss + bwd + AdamW) rows/s",
            "steps": args.drafter_steps,
            "config": {"workload": "dflash_drafter_step", "features": [Nb, S, D],
                       "features_dtype": "bf16, widened to fp32 for the fp32-logit variants", "d_model": 256,
                       "layers": 3,
                       "heads": 4, "block_size": blk, "V": V, "lm_head": "frozen, random",
                       "objective": "dpace alpha 0.5, anchor slot masked", "optimizer": "AdamW lr 1e-3, clip 1.0",
                       "gemms": "cuBLAS, TF32 for fp32", "parallelism": f"ddp{world}",
                       "library_layers": "RMSNorm kernels (fp32/bf16) and, for bf16 q/k/v, the tcgen05 "
                                         "attention forward and backward (specdec.drafter)",
                       "cuda_graph": "the _graphed variant replays the whole step -- forward, loss, "
                                     "backward, the gradient all-reduce (N > 1: one NCCL call on the flat "
                                     "gradient, specdec.graphs.allreduce_grads), clip, AdamW(fused, "
                                     "capturable) -- as one CUDA graph (specdec.graphs.GraphedStep); the "
                                     "others launch eagerly with the default AdamW and, for N > 1, DDP"},
            "variants": out}


def run_ours(args):
    import torch.distributed as dist
    from datetime import timedelta

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if world > 1:
        # high-priority NCCL stream: the loss all_reduce is dispatched ahead of
        # the next kernel's CTAs and overlaps it
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=120), pg_options=opts)
    T = Timing(args, dev, world)

    N, B, V = args.n, 16, 128256
    E = N * B * V
    n_global = N * world
    peak, peak_src = hbm_peak()

    # untimed soak of about args.soak seconds on the headline workload, with
    # the clock sampler running from here through the timed region
    sampler = ClockSampler(dev)
    sampler.start()
    head = None
    if args.soak > 0:
        from specdec import ops

        x, t, m = dpace_inputs(N, B, V, 2.0, 4, rank, dev)
        g = torch.empty_like(x)
        ops.dpace_forward_backward(x, t, m, 0.5, 0, n_global=n_global, validate=False, out=g)
        torch.cuda.synchronize(dev)
        probe = time.perf_counter()
        for _ in range(4):
            ops.dpace_forward_backward(x, t, m, 0.5, 0, n_global=n_global, validate=False, out=g)
        torch.cuda.synchronize(dev)
        per_step = max((time.perf_counter() - probe) / 4, 1e-5)
        soak_steps = int(T.max(float(int(args.soak / per_step))))
        for i in range(soak_steps):
            ops.dpace_forward_backward(x, t, m, 0.5, 0, n_global=n_global, validate=False, out=g)
            if (i + 1) % 64 == 0:
                torch.cuda.synchronize(dev)
        torch.cuda.synchronize(dev)
        del x, t, m, g
    head = dpace_leg(args, T, N, B, V, 2.0, 4, n_global, args.steps)
    clocks = sampler.stop()
    launches_per_step = 3 if head["aligned"] else 2  # ring: stream + finalize + backward

    c4 = time_c4(args, T) if args.c4_steps > 0 else None
    dflash = time_dflash(args, T, n_global) if args.dflash_steps > 0 else None
    drafter = time_drafter_step(args, dev, world, T.max, T.barrier) if args.drafter_steps > 0 else None
    bf16 = None
    if args.bf16_steps > 0:
        bf16 = {"dpace": time_dpace_bf16(args, T, n_global),
                "dflash_kl": time_dflash(args, T, n_global, dtype=torch.bfloat16, steps=args.bf16_steps)}

    # end to end through the public API: pinned host inputs -> dpace_loss ->
    # backward -> loss to host. The next step's inputs are copied on a copy
    # stream while this step computes (double-buffered device inputs).
    e2e = None
    if args.e2e_steps > 0:
        from losses import dpace_loss
        from specdec import ops
        from specdec.dist import sharded_dpace_loss

        hsets = [dpace_inputs(N, B, V, 2.0, 4, 1000 * s_ + rank, torch.device("cpu")) for s_ in range(2)]
        hx = [h[0].pin_memory() for h in hsets]
        ht = [h[1].pin_memory() for h in hsets]
        hm = [h[2].pin_memory() for h in hsets]
        del hsets
        hloss = torch.empty((), dtype=torch.float32).pin_memory()
        bufs = [(torch.empty(N, B, V, device=dev), torch.empty(N, B, dtype=torch.int64, device=dev),
                 torch.empty(N, B, device=dev)) for _ in range(2)]
        copy_stream = torch.cuda.Stream(dev)
        ready = [torch.cuda.Event() for _ in range(2)]
        free = [torch.cuda.Event() for _ in range(2)]
        for ev in free:
            ev.record(T.stream)
        saved_fused = ops.FUSED_BACKWARD
        ops.set_fused_backward(args.e2e_fused)

        def h2d(i):
            j = i & 1
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(free[j])
                for d, h in zip(bufs[j], (hx[j], ht[j], hm[j])):
                    d.copy_(h, non_blocking=True)
                ready[j].record(copy_stream)

        def e2e_step(i, steps):
            j = i & 1
            if i + 1 < steps:
                h2d(i + 1)  # prefetch the next step's inputs
            T.stream.wait_event(ready[j])
            x = bufs[j][0].detach().requires_grad_(True)
            t, m = bufs[j][1], bufs[j][2]
            if world > 1:  # the multi-GPU entry point: this rank's shard, global loss
                loss = sharded_dpace_loss(x, t, 0.5, m, n_global=n_global)
            else:
                loss = dpace_loss(x, t, 0.5, m)
            loss.backward()
            free[j].record(T.stream)
            hloss.copy_(loss.detach(), non_blocking=True)

        h2d(0)
        for i in range(2):
            e2e_step(i, 2)
        torch.cuda.synchronize(dev)
        T.barrier()
        device_barrier_on(world, dev)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(T.stream)
        copy_stream.wait_event(s0)  # every one of the K steps' copies runs inside the timed region
        h2d(0)
        for i in range(args.e2e_steps):
            e2e_step(i, args.e2e_steps)
        s1.record(T.stream)
        torch.cuda.synchronize(dev)
        ops.set_fused_backward(saved_fused)
        e2e_ms = T.max(s0.elapsed_time(s1)) / args.e2e_steps
        h2d_bytes = hx[0].numel() * 4 + ht[0].numel() * 8 + hm[0].numel() * 4
        e2e = {"value": round(12.0 * E * world / (e2e_ms * 1e-3) / 1e9, 2), "unit": UNIT,
               "h2d_bytes_per_step": h2d_bytes, "d2h_bytes_per_step": 4 + 12,
               "ms_per_step": round(e2e_ms, 3), "steps": args.e2e_steps,
               "h2d_gbs": round(h2d_bytes / (e2e_ms * 1e-3) / 1e9, 2),
               "path": ("specdec.dist.sharded_dpace_loss" if world > 1 else "losses.dpace.dpace_loss")
                       + "(...).backward() from pinned host buffers (each step's inputs copied on a copy "
                         "stream while the previous step computes); includes the target-range check "
                         "(12-byte status read-back)"
                       + ("; specdec.ops.set_fused_backward(True)" if args.e2e_fused else "")}
        del bufs, hx, ht, hm

    cpu_base = cpu_dflash = None
    if rank == 0 and world == 1 and args.cpu_budget > 0:
        cpu_base = time_cpu_baseline(B, V, args.cpu_budget)
        cpu_dflash = time_cpu_baseline_dflash(B, V, args.cpu_budget)
        if dflash is not None:
            dflash["cpu_baseline"] = cpu_dflash

    # every rank's own figures, for the scaling record
    mine = {"rank": rank, "ms_per_step": round(head["ms_local"], 4), "clocks": clocks,
            "c4_ms_per_step": None if c4 is None else c4["ms_per_step_this_rank"],
            "dflash_ms_per_step": None if dflash is None else dflash["ms_per_step_this_rank"]}
    per_rank = [None] * world
    if world > 1:
        dist.all_gather_object(per_rank, mine)
        dist.destroy_process_group()
    else:
        per_rank = [mine]
    if rank != 0:
        return 0

    rep = dpace_report(head, N, B, V, world, 4, N * B * world, peak, "weak")
    line = {"metric": METRIC, "value": rep["value"], "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": rep["ms_per_step"],
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "dpace_fwd_bwd_llama3_vocab", "N_per_gpu": N, "B": B, "V": V,
                       "global_N": n_global, "sigma": 2.0, "mask": "prefix k~U{0..4}",
                       "alpha": 0.5, "loss_type": "dpace", "parallelism": f"dp{world} (N-sharded)",
                       "loss_all_reduce": (args.loss_reduce + ", one per step, started after the step's "
                                           "call, waited for once before the stop event") if world > 1
                       else None,
                       "l2": "two alternating input sets, each 525 MB > 126 MB L2",
                       "bytes_model": "12*N*B*V per GPU-step",
                       "step": "specdec_dpace_forward_backward through the C ABI (library level: the "
                               "public API's 4-byte status read-back is timed in e2e)",
                       "launch": "one CUDA graph per step (the step's 3 kernel launches), replayed"
                                 if args.graphs else "eager launches from Python",
                       "split": "forward and backward each captured as a CUDA graph of 8 back-to-back calls, "
                                "replayed between events (time / 8)" if args.graphs else
                                "eager calls between events"},
            "rows_per_s": rep["rows_per_s"],
            "moved_bytes_per_step": rep["moved_bytes_per_step"],
            "pct_of_hbm_peak": rep["pct_of_hbm_peak"], "pct_basis": rep["pct_basis"],
            "pct_of_spec_8000": rep["pct_of_spec_8000"],
            "roofline": dict(rep["roofline"], peak_source=peak_src),
            "kernels": {"fwd": rep["fwd_roofline"], "split_ms": rep["split_ms"],
                        "launches_per_step": launches_per_step,
                        "fwd_note": "forward = streaming kernel + PDL-chained finalize kernel; in the "
                                    "timed step the backward is PDL-chained to the finalize"},
            "live_row_fraction": rep["live_row_fraction"],
            "c4": c4,
            "dflash_kl": dflash,
            "bf16": bf16,
            "drafter_step": drafter,
            "cpu_baseline": cpu_base, "e2e": e2e,
            "gpu_launches": launches_per_step * args.steps, "gpu_launches_scope": "per rank, headline loop",
            "clocks": clocks,
            "per_rank": per_rank}
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
    p.add_argument("--bf16-steps", type=int, default=100,
                   help="timed steps of each bf16-logits workload (0 = skip)")
    p.add_argument("--drafter-steps", type=int, default=10,
                   help="timed end-to-end drafter training steps per variant (0 = skip)")
    p.add_argument("--loss-reduce", choices=("overlap", "serial"), default="overlap",
                   help="N > 1: loss all_reduce on a side stream beside the backward, or between "
                        "forward and backward on the compute stream")
    p.add_argument("--cpu-budget", type=float, default=10.0,
                   help="seconds of CPU-oracle timing per objective on rank 0 at N=1 (0 = skip)")
    p.add_argument("--c4-steps", type=int, default=10,
                   help="timed steps of the large-batch [512,32,151936] workload (0 = skip)")
    p.add_argument("--graphs", type=int, default=1,
                   help="timed loops replay one CUDA graph per step (1) or launch from Python (0)")
    p.add_argument("--e2e-fused", type=int, default=1,
                   help="e2e: specdec.ops.set_fused_backward (1) or the separate backward kernel (0)")
    args = p.parse_args(argv)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
