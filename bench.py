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

from specdec.dist import LossReducer  # noqa: E402

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

def device_barrier_on(world, dev):
    """A 1-element all_reduce on the current stream: every rank's next event
    fires when it completes, so a rank whose host left the barrier late does
    not land its delay inside the other ranks' timed windows."""
    if world > 1:
        import torch.distributed as dist

        dist.all_reduce(torch.zeros(1, device=dev))


def time_pair(args, stream, world, max_over_ranks, barrier, fwd, bwd, steps):
    """Times `steps` steps of fwd(i) (+ the loss all_reduce when world > 1) +
    bwd(i, state) on alternating input sets after args.warmup untimed steps.
    Returns (ms per step, mean forward ms, mean backward ms), max over ranks."""

    reducer = LossReducer(stream.device) if world > 1 and args.loss_reduce == "overlap" else None

    def step(i, ev=None):
        if ev is not None:
            ev[0].record(stream)
        loss, state = fwd(i)
        if ev is not None:
            ev[1].record(stream)
        if reducer is not None:
            reducer.start(loss)
        elif world > 1:
            import torch.distributed as dist
            dist.all_reduce(loss)
        if ev is not None:
            ev[2].record(stream)
        bwd(i, state)
        if ev is not None:
            ev[3].record(stream)
        if reducer is not None:
            reducer.wait()

    for i in range(args.warmup):
        step(i)
    # the step time comes from an uninstrumented loop (events between kernels
    # would break the programmatic-dependent-launch chaining of the kernels)
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    device_barrier_on(world, stream.device)
    a.record(stream)
    for k in range(steps):
        step(k)
    b.record(stream)
    torch.cuda.synchronize()
    barrier()
    ms = max_over_ranks(a.elapsed_time(b)) / steps
    # per-kernel split from a second, instrumented pass
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(steps)]
    for k in range(steps):
        step(k, evs[k])
    torch.cuda.synchronize()
    f = max_over_ranks(statistics.mean(e[0].elapsed_time(e[1]) for e in evs))
    g = max_over_ranks(statistics.mean(e[2].elapsed_time(e[3]) for e in evs))
    return ms, f, g


def time_dflash(args, dev, stream, world, n_global, max_over_ranks, barrier, dtype=torch.float32, steps=None):
    """DFlash objective (KL), draft [64, 16, 128256] ~ N(0, 2^2), verifier =
    draft + N(0, 1), gamma 4, anchor slot unscored, every slot masked in.
    Bytes model 20 * N*B*V per step for fp32 (forward reads both, backward
    reads both and writes the gradient), 10 * N*B*V for bf16; required bytes
    skip the zero-weight anchor rows."""
    from specdec import ops

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

    K = args.dflash_steps if steps is None else steps
    ms, f, g = time_pair(args, stream, world, max_over_ranks, barrier, fwd, bwd, K)
    live = 15.0 / 16.0
    peak, _ = hbm_peak()
    bwd_bytes = 2.0 * esz * E * live + esz * E
    fwd_bytes = 2.0 * esz * E * live
    model = 5 * esz
    wl = f"{N}x{B}x{V}"
    tag = "_bf16" if esz == 2 else ""
    value = model * E * world / (ms * 1e-3) / 1e9
    del sets, grad
    return {"metric": f"DFlash-KL fwd+bwd logits GB/s ({model}*N*B*V bytes per GPU-step)",
            "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "rows_per_s": round(N * B * world / (ms * 1e-3), 1),
            "pct_of_hbm_peak": round(100.0 * value / world / peak, 2),
            "fwd_ms": round(f, 4), "bwd_ms": round(g, 4), "steps": K,
            "dtype": "bf16" if esz == 2 else "f32",
            "config": {"workload": f"dflash_kl_fwd_bwd_llama3_vocab{tag}", "N_per_gpu": N, "B": B, "V": V,
                       "draft": "N(0, 2^2)", "verifier": "draft + N(0, 1)", "gamma": 4.0,
                       "sample_from_anchor": False, "mask": "all ones",
                       "logits": "bf16 (fp32 arithmetic)" if esz == 2 else "fp32"},
            "roofline": {"kernel": f"dflash_bwd_ring_kernel<{'bf16' if esz == 2 else 'f32'}, KL>", "bound": "hbm",
                         "achieved": round(bwd_bytes / (g * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(bwd_bytes / (g * 1e-3) / 1e9 / peak, 4),
                         "traffic": profiled_traffic(f"dflash_bwd_kl{tag}", wl), "bytes_per_launch": bwd_bytes},
            "fwd_roofline": {"kernel": f"dflash_fwd_ring_kernel<{'bf16' if esz == 2 else 'f32'}, KL> + finalize",
                             "achieved": round(fwd_bytes / (f * 1e-3) / 1e9, 1),
                             "frac": round(fwd_bytes / (f * 1e-3) / 1e9 / peak, 4),
                             "traffic": profiled_traffic(f"dflash_fwd_kl{tag}", wl), "bytes_per_launch": fwd_bytes}}


def time_dpace_bf16(args, dev, stream, world, n_global, max_over_ranks, barrier):
    """D-PACE on bf16 logits, the headline workload otherwise: [64, 16, 128256]
    ~ N(0, 2^2) rounded to bf16, prefix mask k ~ U{0..4}, alpha 0.5. Bytes model
    6 * N*B*V per step (2-byte elements: forward read, backward read + write);
    required bytes skip the unscored rows."""
    from specdec import ops

    N, B, V = args.n, 16, 128256
    E = N * B * V
    sets = []
    for s_ in range(2):
        x, t, m = dpace_inputs(N, B, V, 2.0, 4, 1000 * s_ + int(os.environ.get("RANK", "0")), dev)
        sets.append((x.to(torch.bfloat16), t, m))
        del x
    live = statistics.mean(float(m.mean()) for _, _, m in sets)
    grad = torch.empty(N, B, V, device=dev, dtype=torch.bfloat16)

    def fwd(i):
        x, t, m = sets[i & 1]
        loss, lse, scale, _ = ops.dpace_forward(x, t, m, 0.5, 0, n_global=n_global, validate=False)
        return loss, (lse, scale)

    def bwd(i, st):
        x, t, _ = sets[i & 1]
        ops.dpace_backward(x, t, st[0], st[1], None, out=grad)

    K = args.bf16_steps
    ms, f, g = time_pair(args, stream, world, max_over_ranks, barrier, fwd, bwd, K)
    peak, _ = hbm_peak()
    bwd_bytes = 2.0 * E * live + 2.0 * E
    fwd_bytes = 2.0 * E * live
    wl = f"{N}x{B}x{V}"
    value = 6.0 * E * world / (ms * 1e-3) / 1e9
    del sets, grad
    return {"metric": "D-PACE fwd+bwd bf16 logits GB/s (6*N*B*V bytes per GPU-step)",
            "value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 4),
            "rows_per_s": round(N * B * world / (ms * 1e-3), 1),
            "pct_of_hbm_peak": round(100.0 * value / world / peak, 2),
            "fwd_ms": round(f, 4), "bwd_ms": round(g, 4), "steps": K, "dtype": "bf16",
            "config": {"workload": "dpace_fwd_bwd_llama3_vocab_bf16", "N_per_gpu": N, "B": B, "V": V,
                       "sigma": 2.0, "mask": "prefix k~U{0..4}", "alpha": 0.5, "loss_type": "dpace",
                       "logits": "bf16 (fp32 arithmetic)"},
            "roofline": {"kernel": "dpace_bwd_ring_kernel<bf16>", "bound": "hbm",
                         "achieved": round(bwd_bytes / (g * 1e-3) / 1e9, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(bwd_bytes / (g * 1e-3) / 1e9 / peak, 4),
                         "traffic": profiled_traffic("dpace_bwd_bf16", wl), "bytes_per_launch": bwd_bytes},
            "fwd_roofline": {"kernel": "dpace_fwd_ring_kernel<bf16> + finalize",
                             "achieved": round(fwd_bytes / (f * 1e-3) / 1e9, 1),
                             "frac": round(fwd_bytes / (f * 1e-3) / 1e9 / peak, 4),
                             "traffic": profiled_traffic("dpace_fwd_bf16", wl), "bytes_per_launch": fwd_bytes}}


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
    feats = torch.randn(Nb, S, D, device=dev, generator=g, dtype=torch.bfloat16).float()
    tokens = torch.randint(0, V, (Nb, blk), device=dev, generator=g)
    mask = torch.ones(Nb, blk, device=dev)
    mask[:, 0] = 0.0

    def build(lm_head):
        m = DFlashSpeculator(d_target=D, d_model=256, target_vocab_size=V, block_size=blk, num_layers=3,
                             num_heads=4, target_lm_head=lm_head).to(dev)
        if lm_head.weight.dtype == torch.bfloat16:
            # the drafter body stays fp32; its output feature enters the bf16 head in bf16
            m.final_norm.register_forward_hook(lambda _m, _i, out: out.to(torch.bfloat16))
        if world > 1:
            m = nn.parallel.DistributedDataParallel(m, device_ids=[dev.index])
        return m

    def loss_fused(logits, tok):
        return dpace_loss(logits, tok, 0.5, position_mask=mask)

    def loss_torch(logits, tok):
        return torch_ops_dpace_loss(logits, tok, 0.5, mask)

    variants = [("fused_loss_fp32_logits", head, loss_fused, False),
                ("torch_ops_loss_fp32_logits", head, loss_torch, False),
                ("fused_loss_bf16_logits", head_bf16, loss_fused, False),
                ("bf16_autocast_drafter_fused_loss", head_bf16, loss_fused, True)]
    out = {}
    stream = torch.cuda.current_stream(dev)
    for name, lm_head, lfn, autocast in variants:
        model = build(lm_head)
        core = model.module if world > 1 else model
        params = [p for p in model.parameters() if p.requires_grad]
        opt = torch.optim.AdamW(params, lr=1e-3)

        def step():
            opt.zero_grad(set_to_none=True)
            with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
                loss = core.compute_loss(feats, tokens, loss_fn=lfn) if world == 1 else \
                    lfn(model(feats), tokens)
            loss.backward()
            torch.nn.utils.clip_grad_norm_(params, 1.0)
            opt.step()
            return loss

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
        ms = max_over_ranks(a.elapsed_time(b)) / args.drafter_steps
        out[name] = {"ms_per_step": round(ms, 3), "rows_per_s": round(Nb * blk * world / (ms * 1e-3), 1),
                     "loss": round(float(loss.detach()), 6)}
        del model, core, opt, params
    torch.backends.cuda.matmul.allow_tf32 = prev_tf32
    del head, head_bf16, feats
    torch.cuda.empty_cache()
    base = out["torch_ops_loss_fp32_logits"]["ms_per_step"]
    for v in out.values():
        v["speedup_vs_torch_ops_loss"] = round(base / v["ms_per_step"], 3)
    return {"metric": "drafter training step (fwd + loss + bwd + AdamW) rows/s",
            "steps": args.drafter_steps,
            "config": {"workload": "dflash_drafter_step", "features": [Nb, S, D], "d_model": 256, "layers": 3,
                       "heads": 4, "block_size": blk, "V": V, "lm_head": "frozen, random",
                       "objective": "dpace alpha 0.5, anchor slot masked", "optimizer": "AdamW lr 1e-3, clip 1.0",
                       "gemms": "cuBLAS, TF32 for fp32", "parallelism": f"ddp{world}"},
            "variants": out}


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
        # high-priority NCCL stream: the loss all_reduce is dispatched ahead of
        # the backward's CTAs and overlaps it
        opts = dist.ProcessGroupNCCL.Options()
        opts.is_high_priority_stream = True
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=timedelta(seconds=120), pg_options=opts)

    def barrier():
        if world > 1:
            dist.barrier()

    def device_barrier():
        device_barrier_on(world, dev)

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

    reducer = LossReducer(dev) if world > 1 and args.loss_reduce == "overlap" else None

    def step(i, ev=None):
        x, t, m = sets[i & 1]
        if ev is not None:
            ev[0].record(stream)
        loss, lse, scale, _ = ops.dpace_forward(x, t, m, 0.5, 0, n_global=n_global, validate=False)
        if ev is not None:
            ev[1].record(stream)
        if reducer is not None:
            loss = reducer.start(loss)  # global loss, reduced beside the backward
        elif world > 1:
            dist.all_reduce(loss)
        if ev is not None:
            ev[2].record(stream)
        ops.dpace_backward(x, t, lse, scale, None, out=grad)
        if ev is not None:
            ev[3].record(stream)
        if reducer is not None:
            reducer.wait()
        return loss

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize(dev)
    # untimed soak of about args.soak seconds: every step holds a collective
    # when world > 1, so all ranks run the same, agreed number of steps
    probe = time.perf_counter()
    for i in range(4):
        step(i)
    torch.cuda.synchronize(dev)
    per_step = max((time.perf_counter() - probe) / 4, 1e-5)
    soak_steps = int(max_over_ranks(float(int(args.soak / per_step)))) if args.soak > 0 else 0
    sampler = ClockSampler(dev)
    sampler.start()
    for i in range(soak_steps):
        step(i)
        if (i + 1) % 64 == 0:
            torch.cuda.synchronize(dev)

    # timed region: K uninstrumented steps (events between the kernels would
    # break their programmatic-dependent-launch chaining)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize(dev)
    device_barrier()
    start.record(stream)
    for k in range(args.steps):
        step(k)
    stop.record(stream)
    torch.cuda.synchronize(dev)
    barrier()
    clocks = sampler.stop()
    ms_local = start.elapsed_time(stop)
    # per-kernel split (roofline): a second pass with events around each kernel
    evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(args.steps)]
    for k in range(args.steps):
        step(k, evs[k])
    torch.cuda.synchronize(dev)
    fwd_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in evs)
    bwd_ms = statistics.mean(e[2].elapsed_time(e[3]) for e in evs)
    ms = max_over_ranks(ms_local)
    fwd_ms_max, bwd_ms_max = max_over_ranks(fwd_ms), max_over_ranks(bwd_ms)
    dflash = None
    if args.dflash_steps > 0:
        dflash = time_dflash(args, dev, stream, world, n_global, max_over_ranks, barrier)
    drafter = None
    if args.drafter_steps > 0:
        drafter = time_drafter_step(args, dev, world, max_over_ranks, barrier)
    bf16 = None
    if args.bf16_steps > 0:
        bf16 = {"dpace": time_dpace_bf16(args, dev, stream, world, n_global, max_over_ranks, barrier),
                "dflash_kl": time_dflash(args, dev, stream, world, n_global, max_over_ranks, barrier,
                                         dtype=torch.bfloat16, steps=args.bf16_steps)}
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

        from specdec.dist import sharded_dpace_loss

        def e2e_step(i):
            x = hx[i & 1].to(dev, non_blocking=True).requires_grad_(True)
            t = ht[i & 1].to(dev, non_blocking=True)
            m = hm[i & 1].to(dev, non_blocking=True)
            if world > 1:  # the multi-GPU entry point: this rank's shard, global loss
                loss = sharded_dpace_loss(x, t, 0.5, m, n_global=n_global)
            else:
                loss = dpace_loss(x, t, 0.5, m)
            loss.backward()
            hloss.copy_(loss.detach(), non_blocking=True)
            return x

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize(dev)
        barrier()
        device_barrier()
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
               "path": ("specdec.dist.sharded_dpace_loss" if world > 1 else "losses.dpace.dpace_loss")
                       + "(...).backward() from pinned host buffers; includes the target-range check "
                         "(4-byte read-back)"}

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
                       "alpha": 0.5, "loss_type": "dpace", "parallelism": f"dp{world} (N-sharded)", "loss_all_reduce": args.loss_reduce if world > 1 else None,
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
            "bf16": bf16,
            "drafter_step": drafter,
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
    p.add_argument("--bf16-steps", type=int, default=100,
                   help="timed steps of each bf16-logits workload (0 = skip)")
    p.add_argument("--drafter-steps", type=int, default=10,
                   help="timed end-to-end drafter training steps per variant (0 = skip)")
    p.add_argument("--loss-reduce", choices=("overlap", "serial"), default="overlap",
                   help="N > 1: loss all_reduce on a side stream beside the backward, or between "
                        "forward and backward on the compute stream")
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
