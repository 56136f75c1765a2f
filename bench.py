"""Benchmark of the HilbertA paired block-sparse attention on B200.

Metric: ms/call + effective TFLOP/s over ACTIVE 64x64 blocks of
the sparse attention at 2048^2 (128x128 image grid + 512 text tokens = 16896
tokens), 16 tiles, bridge K=3, B=1, 24 heads x 128, bf16 Q/K/V ~ N(0,1) from
torch seed 2707 (the reference benchmark's protocol, hilberta/benchmark.py:24-85).

One step = one attention call for each of the four tile phases; ms/call is
phase-weighted 15/14/14/14 over 57 layers (benchmark.py:76-83).  Every call is
timed with CUDA events on the launching stream after an L2 flush (a 256 MB
write outside the events); ``value`` = active FLOP of the timed calls / their
summed device time (max over ranks).  FLOP per call = H * 4*64*64*D * A, A =
active 64x64 (query-block, key-block) pairs (global rows x all blocks + sum of
kv_counts).  The clocks are sampled through NVML every 2 ms during the timed
region; ``sustained`` repeats the measurement on the 57-call sequence of
denoising steps for about half a second, where the power cap lowers the clock,
against the measured sustained peak.

N > 1 (torchrun): head-parallel, rank r owns heads [r*H/P, (r+1)*H/P); every
call also gathers all ranks' bf16 head outputs on every rank (what the FLUX
block consumes) — inside the attention kernel, which stores each output row to
all ranks over NVLink peer memory (head_parallel.PeerAllGather).  The kernel
followed by an NCCL all-gather is timed beside it (``nccl_path``), and the
link the peer stores use is measured in the run (plain peer copies).

Side fields: ``parity`` (every head's sampled rows of phases 0 and 3, at N > 1
the all-gathered output of every rank, against an fp32 torch reference),
``scaling_4096`` (the 4096^2 t16k3 shape on this run's GPUs), ``e2e`` (host
buffers, copies inside the timed region), ``flux_step`` (one denoising step of a
FLUX.1-architecture transformer with random weights, HilbertA vs dense
attention; tensor-parallel at N > 1), and at N = 1 ``token_order`` (raster
layouts), ``prep`` (Q/K/V preparation), ``cpu_baseline`` and
``triton_reference`` (the reference's own Triton kernel from baseline/_ref on
this GPU, timed by its benchmark's protocol).

``--impl reference`` times the reference's dense-mask CPU path (plan mask +
fp32 SDPA, the computation of hilberta/flux_adapter.py:299-307) restated in
oracle/attention_oracle.py, on bounded row samples, with all host threads.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

CONFIGS = {
    # name: (resolution, tiles, k)
    "1024_t4k1": (1024, 4, 1),
    "1024_t16k3": (1024, 16, 3),
    "2048_t4k1": (2048, 4, 1),
    "2048_t16k3": (2048, 16, 3),
    "4096_t16k3": (4096, 16, 3),
}
WEIGHTS = (15, 14, 14, 14)
# one step = one call per tile phase; ms/call is phase-weighted 15/14/14/14
STEP_PHASES = (0, 1, 2, 3)
# the 57 joint-attention calls of a FLUX.1 denoising step (19 double + 38 single
# blocks), layer i on tile phase i % 4: the reference benchmark's phase weights
# (hilberta/benchmark.py:76-83) as a call sequence, for the sustained timing
DENOISE_PHASES = tuple(layer % 4 for layer in range(57))
L2_FLUSH_BYTES = 256 << 20  # twice the 126 MB L2
METRIC = "ms/call + effective TFLOP/s (active blocks) of sparse attn, 2048² t16k3, 1/2/4/8 B200"
FALLBACK_PEAK_TFLOPS = 1590.0
FALLBACK_SUSTAINED_TFLOPS = 1400.0
FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["native", "reference"], default="native")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="2048_t16k3")
    ap.add_argument("--heads", type=int, default=24)
    ap.add_argument("--layout", choices=["bhnd", "bnhd"], default="bhnd")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="target CPU seconds of the baseline sample")
    ap.add_argument("--tp-chunks", type=int, default=1,
                    help="FLUX step at N > 1: row chunks of each row-parallel GEMM (all-reduce overlap)")
    ap.add_argument("--tp-carveout", type=int, default=0, help="SMs kept free of those GEMMs for the all-reduce")
    ap.add_argument("--tp-sp", type=int, default=None, choices=(0, 1),
                    help="FLUX step at N > 1: sequence parallelism (token-split streams, all-gather/reduce-scatter); "
                    "default: on at 4 or more GPUs (measured 4.7 %% faster there, equal at 2)")
    ap.add_argument("--no-4096", action="store_true", help="skip the 4096^2 t16k3 side timing (scaling_4096)")
    ap.add_argument("--no-sustained", action="store_true", help="skip the sustained 57-call side timing")
    ap.add_argument("--no-triton-reference", action="store_true",
                    help="skip timing the reference's Triton kernel on this GPU (triton_reference)")
    ap.add_argument("--triton-reference-child", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--no-flux-step", action="store_true",
                    help="skip the FLUX.1-architecture denoising step (random weights), HilbertA vs dense attention")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def peaks():
    """(burst bf16 TFLOP/s, HBM GB/s, source, sustained bf16 TFLOP/s)."""
    f = ROOT / "MEASURED_PEAKS.json"
    if f.exists():
        d = json.loads(f.read_text())
        burst = float(d["bf16_tflops"])
        return burst, float(d["hbm_gbs"]), "measured", float(d.get("bf16_tflops_sustained", burst))
    return FALLBACK_PEAK_TFLOPS, FALLBACK_HBM_GBS, "fallback", FALLBACK_SUSTAINED_TFLOPS


def ncu_traffic(config):
    """Per-launch DRAM bytes of k_paired_fwd from the committed ncu summary, if any."""
    f = ROOT / "profiles" / f"paired_fwd_{config}_traffic.txt"
    if not f.exists():
        return None
    for line in f.read_text().splitlines():
        if line.startswith("dram_bytes_per_launch="):
            return float(line.split("=", 1)[1])
    return None


_SAMPLER = r"""
import select, sys, time
import pynvml
pynvml.nvmlInit()
h = pynvml.nvmlDeviceGetHandleByUUID(sys.argv[1])
period = float(sys.argv[2])
get_reasons = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
    pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
print("ready", pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM), flush=True)
out, power, n = [], 0.0, 0
while True:
    try:
        if n % 8 == 0:  # the power reading is the slow query: every 8th sample
            power = pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0
        out.append((time.time(), pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM), get_reasons(h), power))
        n += 1
    except pynvml.NVMLError:
        pass
    if select.select([sys.stdin], [], [], period)[0]:
        break
for x in out:
    print(*x)
"""


class ClockSampler:
    """SM clock, power draw and clock-event reasons of this rank's GPU during the
    timed region, read through NVML (the library behind nvidia-smi's clocks
    query) every `period` seconds by a separate process, so the samples keep
    their pace while this process launches kernels (a thread here would wait
    for the interpreter lock).  Only samples taken between entering and leaving
    the block count.  Falls back to ``nvidia-smi -lms 100`` when NVML cannot be
    opened."""

    QUERY = (
        "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )
    # NVML clock-event reason bits (nvml.h nvmlClocksEventReason*)
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, device, period=0.002):
        self.device, self.period = torch.device(device), period
        self.result, self.proc, self.smi = None, None, None

    def __enter__(self):
        try:
            uuid = "GPU-" + str(torch.cuda.get_device_properties(self.device).uuid)
            self.proc = subprocess.Popen([sys.executable, "-c", _SAMPLER, uuid, str(self.period)],
                                         stdin=subprocess.PIPE, stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                                         text=True)
            first = self.proc.stdout.readline().split()
            if not first or first[0] != "ready":
                raise RuntimeError("NVML sampler did not start")
            self.max_mhz = float(first[1])
        except (OSError, RuntimeError, ValueError, IndexError):
            if self.proc is not None:
                self.proc.kill()
                self.proc.wait()
            self.proc = None
            try:
                self.smi = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-lms", "100",
                     "-i", str(self.device.index)],
                    stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            except (OSError, ValueError):
                self.smi = None
            time.sleep(0.3)
        self.t0 = time.time()
        return self

    def __exit__(self, *exc):
        t1 = time.time()
        if self.proc is not None:
            try:
                out, _ = self.proc.communicate(input="stop\n", timeout=30)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            rows = []
            for line in out.splitlines():
                f = line.split()
                if len(f) == 4:
                    rows.append((float(f[0]), float(f[1]), int(f[2]), float(f[3])))
            inside = [r for r in rows if self.t0 <= r[0] <= t1]
            if inside:
                mhz = [r[1] for r in inside]
                reasons = sorted(n for n, bit in self.REASONS.items() if any(r[2] & bit for r in inside))
                self.result = {"sm_mhz": statistics.median(mhz), "sm_min_mhz": min(mhz), "sm_max_mhz": self.max_mhz,
                               "reasons": reasons, "samples": len(mhz),
                               "power_w_max": round(max(r[3] for r in inside), 1),
                               "window_ms": round(1e3 * (t1 - self.t0), 1),
                               "source": "nvml, separate process, every %g ms (power every 8th)" % (1e3 * self.period)}
            return False
        if self.smi is None:
            return False
        time.sleep(0.2)
        self.smi.terminate()
        try:
            out, _ = self.smi.communicate(timeout=5)
        except subprocess.TimeoutExpired:
            self.smi.kill()
            out, _ = self.smi.communicate()
        mhz, maxmhz, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                mhz.append(float(f[1]))
                maxmhz = max(maxmhz, float(f[2]))
            except ValueError:
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        if mhz:
            self.result = {"sm_mhz": statistics.median(mhz), "sm_min_mhz": min(mhz), "sm_max_mhz": maxmhz,
                           "reasons": sorted(reasons), "samples": len(mhz), "source": "nvidia-smi"}
        return False


def merge_clocks(results):
    """One clocks record over the ranks: the lowest median, every reason seen,
    the samples of all ranks."""
    results = [r for r in results if r]
    if not results:
        return None
    return {"sm_mhz": min(r["sm_mhz"] for r in results), "sm_min_mhz": min(r["sm_min_mhz"] for r in results),
            "sm_max_mhz": max(r["sm_max_mhz"] for r in results),
            "reasons": sorted(set().union(*(r["reasons"] for r in results))),
            "samples": sum(r["samples"] for r in results), "source": results[0]["source"], "ranks": len(results)}


def build_workload(config, heads, layout, device, head_slice=None):
    import hilberta_b200 as hb

    res, tiles, k = CONFIGS[config]
    plan = hb.bridge_k_plan(tiles, k, False, grid_size=res // 16, device=device)
    N, G = plan.total_tokens, plan.global_tokens
    metas, active = [], []
    for p in plan.phases:
        metas.append(hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(device))
        active.append((G // 64) * (N // 64) + int(p.kv_counts.sum()))
    g = torch.Generator(device="cpu").manual_seed(2707)
    shape = (1, heads, N, 128) if layout == "bhnd" else (1, N, heads, 128)
    qkv = [torch.randn(shape, generator=g, dtype=torch.float32).to(torch.bfloat16) for _ in range(3)]
    if layout == "bnhd":
        qkv = [x.transpose(1, 2) for x in qkv]
    if head_slice is not None:
        return plan, metas, active, [x[:, head_slice] for x in qkv], qkv
    return plan, metas, active, qkv, qkv


def flop_per_call(active, heads, D=128):
    return heads * 4 * 64 * 64 * D * active


def run_native(a):
    import torch.distributed as dist

    import hilberta_b200 as hb

    rank, world, local = dist_env()
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    H = a.heads
    if H % world:
        raise SystemExit("heads must divide across ranks")
    hr = H // world
    hs = slice(rank * hr, (rank + 1) * hr)
    plan, metas, active, qkv_host, qkv_all = build_workload(a.config, H, a.layout, dev, head_slice=hs)
    N = plan.total_tokens
    q, k, v = (x.to(dev) for x in qkv_host)
    out = torch.empty_like(q)
    stream = torch.cuda.current_stream(dev)
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    fused = None
    if world > 1:
        from hilberta_b200.head_parallel import PeerAllGather

        fused = PeerAllGather(1, H, N, 128, layout=a.layout, device=dev)

    def call(ph):
        if fused is None:
            hb.paired_attention(q, k, v, metas[ph], out=out, **kw)
        else:
            fused(q, k, v, metas[ph], **kw)

    # L2 flush between calls: at 4-8 GPUs a rank's Q/K/V (78 / 39 MB) would fit in
    # the 126 MB L2, so every call starts from a written-over L2 (outside the
    # per-call events), as it does inside a denoising step between the GEMMs
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)

    def run_steps(n, record, phases=STEP_PHASES):
        evs = []
        for _ in range(n):
            for ph in phases:
                flush.zero_()
                if record:
                    e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    e[0].record(stream)
                call(ph)
                if record:
                    e[1].record(stream)
                    evs.append((ph, e))
        return evs

    with torch.inference_mode():
        run_steps(max(3, a.warmup), False)
        torch.cuda.synchronize()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        # the sampler process starts first (its start-up time differs between
        # ranks), then the barrier lines the ranks up: a fused call waits for
        # every rank's rows, so a rank that starts late would inflate the first call
        with ClockSampler(dev, period=0.001) as clk:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            t0.record(stream)
            evs = run_steps(a.steps, True)
            t1.record(stream)
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
        status = hb.device_status(dev)
    region_ms = t0.elapsed_time(t1)
    per_phase = [[e[0].elapsed_time(e[1]) for p_, e in evs if p_ == ph] for ph in range(4)]
    total_ms = sum(sum(x) for x in per_phase)  # device time of the timed calls (flushes excluded)
    kern_ms = [statistics.mean(x) for x in per_phase]

    def pct(xs, q):  # nearest-rank percentile of one phase's per-call times
        ys = sorted(xs)
        return ys[min(len(ys) - 1, max(0, math.ceil(q * len(ys)) - 1))]

    phase_stats = {
        "median": [round(statistics.median(x), 4) for x in per_phase],
        "p10": [round(pct(x, 0.10), 4) for x in per_phase],
        "p90": [round(pct(x, 0.90), 4) for x in per_phase],
    }
    t = torch.tensor([total_ms, region_ms, *kern_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    total_ms, region_ms, kern_ms = float(t[0]), float(t[1]), [float(x) for x in t[2:]]
    clocks = clk.result
    if world > 1:
        every = [None] * world
        dist.all_gather_object(every, clk.result)
        clocks = merge_clocks(every)
    flops = [flop_per_call(A, H) for A in active]  # whole job (all heads)
    weighted_ms = sum(w * m for w, m in zip(WEIGHTS, kern_ms)) / 57
    weighted_flop = sum(w * f for w, f in zip(WEIGHTS, flops)) / 57
    step_flop = sum(flops[ph] for ph in STEP_PHASES)
    value = step_flop * a.steps / (total_ms * 1e-3) / 1e12

    # sustained: the 57-call sequence of denoising steps back to back for about
    # half a second, long enough for the 1 kW power cap to act (clocks below)
    n_sustain = 0 if a.no_sustained else max(4, int(500.0 / (len(DENOISE_PHASES) * weighted_ms)))
    with torch.inference_mode():
        torch.cuda.synchronize()
        with ClockSampler(dev, period=0.01) as clk_s:
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
            sevs = run_steps(n_sustain, True, DENOISE_PHASES)
            torch.cuda.synchronize()
        status |= hb.device_status(dev)
    s_ms = torch.tensor([sum(e[0].elapsed_time(e[1]) for _, e in sevs)], dtype=torch.float64, device=dev)
    s_clocks = clk_s.result
    if world > 1:
        dist.all_reduce(s_ms, op=dist.ReduceOp.MAX)
        every = [None] * world
        dist.all_gather_object(every, clk_s.result)
        s_clocks = merge_clocks(every)
    s_ms = float(s_ms[0])
    s_flop = n_sustain * sum(flops[ph] for ph in DENOISE_PHASES)
    s_call_ms = s_ms / max(1, len(sevs))
    sustained = None if not sevs else {
        "ms_per_call": round(s_call_ms, 4),
        "value": round(s_flop / (s_ms * 1e-3) / 1e12, 2),
        "steps": n_sustain,
        "calls": len(sevs),
        "clocks": s_clocks,
    }

    with torch.inference_mode():
        outs = {}
        for ph in (0, 3):
            outs[ph] = (hb.paired_attention(q, k, v, metas[ph], **kw) if fused is None else fused(q, k, v, metas[ph], **kw)).clone()
        parity = parity_rows(plan, qkv_all, outs, dev)
        status |= hb.device_status(dev)
    del outs
    if world > 1:
        t = torch.tensor([parity["max_abs"], parity["mean_abs"], 0.0 if parity["ok"] else 1.0], dtype=torch.float64,
                         device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        parity.update(max_abs=float(t[0]), mean_abs=float(t[1]), ok=not bool(t[2]), ranks_checked=world)
    link_gbs = link_ce_gbs = None
    if world > 1:
        t = torch.tensor([fused.measure_link_gbs(method="sm"), fused.measure_link_gbs(method="copy_engine")],
                         dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MIN)
        link_gbs, link_ce_gbs = float(t[0]), float(t[1])
    perm = permutation_side_timing(a, q, k, v, metas, plan, dev, hb) if world == 1 else None
    prep_t = prep_side_timing(plan, H, dev) if world == 1 else None
    flux = None if a.no_flux_step else flux_step_timing(a, dev, world)
    nccl = nccl_side_timing(a, q, k, v, metas, flops, world, dev, hb) if world > 1 else None
    big = None if a.no_4096 or a.config == "4096_t16k3" else scaling_4096_timing(a, world, rank, dev, hb)

    e2e = None
    if not a.no_e2e:
        e2e = run_e2e(a, q, k, v, metas, flops, world, dev, hb, fused)
    peak, hbm, peak_kind, peak_sustained = peaks()
    achieved = weighted_flop / world / (weighted_ms * 1e-3) / 1e12  # one GPU's launch
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = cpu_baseline(a, plan, active, bounded=a.cpu_seconds)
    triton_ref = None
    if rank == 0 and world == 1 and not a.no_triton_reference:
        triton_ref = triton_reference_side(a)
    if world > 1:
        fused.close()
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    traffic = ncu_traffic(a.config)
    line = {
        "metric": METRIC,
        "value": round(value, 2),
        "unit": "TFLOP/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": max(3, a.warmup),
        "ms_per_step": round(total_ms / a.steps, 4),
        "ms_timed_region": round(region_ms, 3),
        "ms_per_call": round(weighted_ms, 4),
        "ms_per_call_by_phase": [round(x, 4) for x in kern_ms],
        "ms_per_call_by_phase_stats": phase_stats,  # this rank's per-call distribution (rank 0)
        "eff_tflops_kernel": round(weighted_flop / (weighted_ms * 1e-3) / 1e12, 2),
        "frac_peak": round(achieved / peak, 4),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) bf16 Q/K/V, reference benchmark protocol)",
        "config": shared_config(a.config, H, N, world, a.layout, active),
        "l2_detail": "this GPU's Q+K+V %.0f MB; the flush is a %d MB write outside the per-call events"
        % (3 * N * hr * 128 * 2 / 1e6, L2_FLUSH_BYTES >> 20),
        "gpu_launches": len(STEP_PHASES) * a.steps,
        "device_status": status,
        "roofline": {
            "bound": "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "peak_source": f"{peak_kind} bf16 dense (MEASURED_PEAKS.json bf16_tflops, burst)" if peak_kind == "measured" else "fallback 1.59 PFLOP/s",
            "traffic": traffic,
            "kernel": "k_paired_fwd",
        },
    }
    if perm is not None:
        line["token_order"] = perm
    if prep_t is not None:
        prep_t["frac_hbm"] = round(prep_t["achieved_gbs"] / hbm, 4)
        prep_t["peak_gbs"] = hbm
        line["prep"] = prep_t
    if world > 1:
        # fused compute + collective: the target is the slower of the tensor time
        # and this GPU's share of the NVLink traffic (its rows to P-1 peers)
        link = link_gbs  # GB/s this rank sends with SM stores, measured in this run (slowest rank)
        nv_bytes = (world - 1) * N * hr * 128 * 2
        t_tensor = weighted_flop / world / (peak * 1e12)
        t_link = nv_bytes / (link * 1e9)
        line["roofline"]["fused_allgather"] = {
            "nvlink_bytes_per_call": nv_bytes,
            "link_gbs": round(link, 1),
            "link_source": "measured now: hb_peer_scatter (SM stores in the fused kernel's pattern) of each rank's "
            "rows to every peer, all ranks at once, best of 3, slowest rank",
            "link_gbs_copy_engine": round(link_ce_gbs, 1),
            "target_ms": round(max(t_tensor, t_link) * 1e3, 4),
            "bound": "tensor" if t_tensor >= t_link else "nvlink",
            "frac": round(max(t_tensor, t_link) * 1e3 / weighted_ms, 4),
        }
        line["nccl_path"] = nccl
        # the north star asks for kernel-only and kernel + gather separately at N > 1
        line["kernel_only"] = {"ms_per_call": nccl["kernel_ms_per_call"], "value": nccl["kernel_only_value"],
                               "unit": "TFLOP/s", "note": "attention launches without the all-gather (nccl_path)"}
    if sustained is not None:
        sustained["frac_sustained_peak"] = round(sustained["value"] / world / peak_sustained, 4)
        sustained["peak_sustained"] = peak_sustained
        sustained["note"] = ("the 57 joint-attention calls of a denoising step (layer i on phase i % 4) back to back, "
                             "per-call events after an L2 flush; frac against the measured sustained bf16 peak "
                             "(MEASURED_PEAKS.json bf16_tflops_sustained), the figure for a kernel inside a long step")
        line["sustained"] = sustained
    line["parity"] = parity
    line["parity_ok"] = parity["ok"]
    if big is not None:
        line["scaling_4096"] = big
    if flux is not None:
        line["flux_step"] = flux
    if e2e is not None:
        line["e2e"] = e2e
    if clocks is not None:
        clocks["ms_per_call_x_sm_mhz"] = round(weighted_ms * clocks["sm_mhz"], 1)
        line["clocks"] = clocks
    if cpu is not None:
        line["cpu_baseline"] = cpu
    if triton_ref is not None:
        line["triton_reference"] = triton_ref
    print(json.dumps(line), flush=True)


def parity_rows(plan, qkv_all, outs, dev, n_random=60, seed=0):
    """Sampled output rows of EVERY head (at N > 1 the all-gathered output this
    rank received) against a plain fp32 torch reference of the same call:
    softmax(Q K^T / sqrt(D) + mask) V with the mask of the plan's rows (global
    rows see every key, hilberta/plan.py:70-84), from the same bf16 inputs.
    Tolerance: the north star's max-abs 2e-2 and mean-abs 2e-3."""
    import numpy as np

    N, G = plan.total_tokens, plan.global_tokens
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, G - 1, G, G + 64, N - 1], rng.integers(0, N, n_random)]))
    sel = torch.from_numpy(rows)
    qf = qkv_all[0][:, :, sel].to(dev, torch.float32)
    kf, vf = (x.to(dev, torch.float32) for x in qkv_all[1:])
    worst_max, worst_mean = 0.0, 0.0
    for ph, got in outs.items():
        p = plan.phases[ph]
        ids, counts = torch.as_tensor(p.kv_indices).cpu(), torch.as_tensor(p.kv_counts).cpu()
        mask = torch.zeros(len(rows), N, dtype=torch.bool)
        for j, r in enumerate(rows.tolist()):
            if r < G:
                mask[j] = True
            else:
                b = (r - G) // 64
                blocks = ids[b, : int(counts[b])].long()
                mask[j, (blocks[:, None] * 64 + torch.arange(64)).reshape(-1)] = True
        mask = mask.to(dev)
        want = torch.empty_like(qf)
        for h in range(qf.shape[1]):  # per head: [R, N] scores
            sc = (qf[0, h] @ kf[0, h].T) * (qf.shape[-1] ** -0.5)
            want[0, h] = torch.softmax(sc.masked_fill(~mask, float("-inf")), dim=-1) @ vf[0, h]
        err = (got[:, :, sel.to(dev)].float() - want).abs()
        worst_max, worst_mean = max(worst_max, float(err.max())), max(worst_mean, float(err.mean()))
    return {"ok": worst_max <= 2e-2 and worst_mean <= 2e-3, "max_abs": worst_max, "mean_abs": worst_mean,
            "phases": sorted(outs), "rows": int(len(rows)), "heads": int(qf.shape[1]),
            "reference": "fp32 torch masked softmax attention on the device, same bf16 inputs"}


def scaling_4096_timing(a, world, rank, dev, hb, steps=3):
    """``north_star``'s scaling shape: 4096^2 16-tile K3 (66048 tokens, 24 heads)
    on this run's GPUs, this rank's heads, fused with the all-gather at N > 1.
    Per-call CUDA events after an L2 flush, steps of one call per phase, max over ranks.
    Inputs are drawn on the device (seeded): a performance-only side timing."""
    import torch.distributed as dist

    H = a.heads
    hr = H // world
    plan = hb.bridge_k_plan(16, 3, False, grid_size=256, device=dev)
    N, G = plan.total_tokens, plan.global_tokens
    metas, active = [], []
    for p in plan.phases:
        metas.append(hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev))
        active.append((G // 64) * (N // 64) + int(p.kv_counts.sum()))
    gen = torch.Generator(device=dev).manual_seed(2707 + rank)
    shape = (1, hr, N, 128) if a.layout == "bhnd" else (1, N, hr, 128)
    q, k, v = (torch.randn(shape, generator=gen, device=dev, dtype=torch.bfloat16) for _ in range(3))
    if a.layout == "bnhd":
        q, k, v = (x.transpose(1, 2) for x in (q, k, v))
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    fused = None
    if world > 1:
        from hilberta_b200.head_parallel import PeerAllGather

        fused = PeerAllGather(1, H, N, 128, layout=a.layout, device=dev)
    out = torch.empty_like(q)
    flush = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=dev)
    stream = torch.cuda.current_stream(dev)
    evs = []
    with torch.inference_mode():
        for rec in (False, True):
            if rec:
                torch.cuda.synchronize()
                if world > 1:
                    dist.barrier()
            for _ in range(steps if rec else 1):
                for ph in STEP_PHASES:
                    flush.zero_()
                    e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                    e[0].record(stream)
                    if fused is None:
                        hb.paired_attention(q, k, v, metas[ph], out=out, **kw)
                    else:
                        fused(q, k, v, metas[ph], **kw)
                    e[1].record(stream)
                    if rec:
                        evs.append((ph, e))
        torch.cuda.synchronize()
        status = hb.device_status(dev)
    per_phase = [statistics.mean(e[0].elapsed_time(e[1]) for p_, e in evs if p_ == ph) for ph in range(4)]
    t = torch.tensor(per_phase + [float(status)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        fused.close()
    per_phase = [float(x) for x in t[:4]]
    ms = sum(w * m for w, m in zip(WEIGHTS, per_phase)) / 57
    flop = sum(w * flop_per_call(x, H) for w, x in zip(WEIGHTS, active)) / 57
    del q, k, v, out, flush
    torch.cuda.empty_cache()
    return {
        "workload": workload_name("4096_t16k3", H, N),
        "heads_per_gpu": hr,
        "ms_per_call": round(ms, 4),
        "ms_per_call_by_phase": [round(x, 4) for x in per_phase],
        "value": round(flop / (ms * 1e-3) / 1e12, 2),
        "unit": "TFLOP/s (whole job, active blocks)",
        "device_status": int(t[4]),
        "path": "paired attention" + (" fused with the NVLink all-gather of all heads" if world > 1 else ""),
        "note": "%d steps of one call per phase, per-call events after an L2 flush, max over ranks; inputs drawn on the device"
        % steps,
    }


def prep_side_timing(plan, H, dev, steps=10, D=128):
    """The processor's Q/K/V preparation at this config (hilberta/flux_adapter.py:
    280-298): hb_norm_rope_pack for Q, K, V against the same steps as eager torch
    ops; HBM bytes = the six projections read + Q/K/V written + cos/sin read by
    the Q and K passes."""
    from hilberta_b200 import prep

    T, N = plan.text_tokens, plan.total_tokens
    n = N - T
    g = torch.Generator(device="cpu").manual_seed(11)
    proj = [torch.randn(1, T if i < 3 else n, H * D, generator=g).to(torch.bfloat16).to(dev) for i in range(6)]
    w = [torch.ones(D, dtype=torch.bfloat16, device=dev) for _ in range(4)]
    ang = torch.rand(N, D // 2, generator=g) * 6.28
    cos = torch.cos(ang).repeat_interleave(2, dim=1).to(dev)
    sin = torch.sin(ang).repeat_interleave(2, dim=1).to(dev)

    def fused():
        prep.prepare_qkv(*proj, heads=H, norm_q=w[0], norm_k=w[1], norm_added_q=w[2], norm_added_k=w[3],
                         rotary=(cos, sin))

    def eager():
        def norm(x, wt):
            x = x.unflatten(-1, (H, -1))
            y = (x * torch.rsqrt(x.float().pow(2).mean(-1, keepdim=True) + 1e-6)).to(x.dtype)
            return y * wt

        def rope(x):
            re, im = x.reshape(*x.shape[:-1], -1, 2).unbind(-1)
            rot = torch.stack([-im, re], dim=-1).flatten(3)
            return (x.float() * cos[None, :, None] + rot.float() * sin[None, :, None]).to(x.dtype)

        qq = rope(torch.cat([norm(proj[0], w[2]), norm(proj[3], w[0])], dim=1))
        kk = rope(torch.cat([norm(proj[1], w[3]), norm(proj[4], w[1])], dim=1))
        vv = torch.cat([proj[2].unflatten(-1, (H, -1)), proj[5].unflatten(-1, (H, -1))], dim=1)
        return qq, kk, vv

    res = {}
    with torch.inference_mode():
        for name, fn in (("ms", fused), ("eager_ms", eager)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                fn()
            e1.record()
            torch.cuda.synchronize()
            res[name] = round(e0.elapsed_time(e1) / steps, 4)
    nbytes = 2 * (3 * N * H * D * 2) + 2 * (2 * N * D * 4)
    res["bytes"] = nbytes
    res["achieved_gbs"] = round(nbytes / (res["ms"] * 1e-3) / 1e9, 1)
    res["note"] = "Q,K,V: per-head RMSNorm + text/image cat + rotary + [B,S,H,D] pack (hb_norm_rope_pack) vs eager torch"
    return res


def flux_step_timing(a, dev, world, steps=3, warmup=2):
    """One denoising step of a FLUX.1-architecture transformer with random
    weights (19 double + 38 single blocks, hidden 3072, 24 x 128 heads, 512 text
    tokens; hilberta_b200/flux_model.py) at this config's resolution, run
    through the reference's adapter entry, ``persistent_flux_attention(model,
    plan, backend="paired")`` (HilbertA in every joint attention, layer i on
    phase i % 4, image tokens gathered into the plan's order at entry and back
    at exit), against the same weights with dense attention outside it.  N > 1:
    tensor-parallel over the ranks (hilberta_b200/flux_tp.py), each rank
    attending over its 24/N heads; times are the max over ranks.  Inputs are
    device-resident.  The attention parts are timed alone: 57 paired calls
    (phases cycled) and 57 dense SDPA calls on this rank's heads."""
    import torch.distributed as dist

    from hilberta_b200 import PlanBank, bridge_k_plan, paired_attention
    from hilberta_b200.flux_adapter import persistent_flux_attention
    from hilberta_b200.flux_model import FluxTransformer, parameter_count, step_inputs

    res_px, tiles, k = CONFIGS[a.config]
    grid = res_px // 16
    plan = bridge_k_plan(tiles, k, False, grid_size=grid)
    tp_sp = (world >= 4) if a.tp_sp is None else bool(a.tp_sp)
    torch.manual_seed(5)  # identical weights on every rank
    model = FluxTransformer(device=dev)
    params = parameter_count(model)
    if world > 1:
        from hilberta_b200.flux_tp import shard_flux_model

        shard_flux_model(model, chunks=a.tp_chunks, carveout=a.tp_carveout or None, sequence_parallel=tp_sp)
    x = step_inputs(grid, plan.text_tokens, dev)
    N, hr = plan.total_tokens, 24 // world
    qkv = [torch.randn(1, hr, N, 128, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    metas = PlanBank(plan).on_device(dev)["paired_phases"]

    def timed(fn, n):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(n):
            fn()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    times, outs = {}, {}
    with torch.inference_mode():
        with persistent_flux_attention(model, plan, backend="paired") as info:
            times["hilberta_ms"] = timed(lambda: model(**x), steps)
            outs["hilberta"] = model(**x).sample.float()
        times["dense_ms"] = timed(lambda: model(**x), steps)
        outs["dense"] = model(**x).sample.float()
        times["attention_ms_hilberta"] = timed(lambda: [paired_attention(*qkv, metas[i % 4]) for i in range(57)], 1)
        times["attention_ms_dense"] = timed(
            lambda: [torch.nn.functional.scaled_dot_product_attention(*qkv) for _ in range(57)], 1)
    vals = torch.tensor(list(times.values()), dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    res = {"workload": f"FLUX.1-architecture step, {a.config}, 19+38 blocks, hidden 3072, random weights",
           "parameters": params,
           "entry": "persistent_flux_attention(model, plan, backend='paired')",
           "parallelism": (f"tensor-parallel x{world} (heads and MLP hidden sharded; "
                           + ("sequence-parallel streams, NCCL all-gather / reduce-scatter)" if tp_sp else
                              f"NCCL all-reduce, {a.tp_chunks} row chunks per row-parallel GEMM, "
                              f"{a.tp_carveout} SMs carved out)"))
           if world > 1 else "single GPU"}
    res.update({key: round(float(v), 2) for key, v in zip(times, vals)})
    res["speedup"] = round(res["dense_ms"] / res["hilberta_ms"], 3)
    res["rel_diff_vs_dense"] = round(float((outs["hilberta"] - outs["dense"]).norm() / outs["dense"].norm()), 4)
    res["adapter_calls"] = {k: info[k] for k in ("transformer_calls", "image_reorder_calls", "image_inverse_calls")}
    res["note"] = ("steps=%d warmup=%d, device-resident inputs, max over ranks; attention_ms_* = 57 calls on this "
                   "rank's heads; rel_diff_vs_dense is the sparse step's relative L2 distance from the dense step "
                   "(a property of the sparse pattern, not an error)" % (steps, warmup))
    del model, outs, qkv
    torch.cuda.empty_cache()
    return res


def nccl_side_timing(a, q, k, v, metas, flops, world, dev, hb, steps=5):
    """The unfused head-parallel path on the same inputs: the kernel into a local
    output, then an NCCL all-gather of every rank's heads (max over ranks)."""
    import torch.distributed as dist

    out = torch.empty_like(q)
    B, hr, N, D = q.shape
    gathered = torch.empty(world, B, hr, N, D, dtype=q.dtype, device=dev)
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    ev = []
    with torch.inference_mode():
        def step(record):
            for ph in range(4):
                e = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) if record else None
                if e:
                    e[0].record()
                hb.paired_attention(q, k, v, metas[ph], out=out, **kw)
                if e:
                    e[1].record()
                    ev.append(e)
                dist.all_gather_into_tensor(gathered.view(-1), out.contiguous().view(-1))

        for _ in range(3):
            step(False)
        torch.cuda.synchronize()
        dist.barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        for _ in range(steps):
            step(True)
        t1.record()
        torch.cuda.synchronize()
    t = torch.tensor([t0.elapsed_time(t1) / steps, statistics.mean(e[0].elapsed_time(e[1]) for e in ev)],
                     dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.barrier()
    return {
        "ms_per_step": round(float(t[0]), 4),
        "kernel_ms_per_call": round(float(t[1]), 4),
        "value": round(sum(flops) / (float(t[0]) * 1e-3) / 1e12, 2),
        "kernel_only_value": round(sum(flops) / len(flops) / (float(t[1]) * 1e-3) / 1e12, 2),
        "note": "paired_attention into a local output, then dist.all_gather_into_tensor (NCCL), per call; "
        "kernel_only_value: whole-job TFLOP/s of the attention launches alone (this rank's heads, max over ranks)",
    }


def permutation_side_timing(a, q, k, v, metas, plan, dev, hb, steps=5):
    """Raster-order Q/K/V (the tensors as given, read as raster token order):
    mean ms per call of the kernel reading/writing raster order in place
    (``token_order``: 8x8-square boxes, and the general row-map gather) against the
    explicit path (index_select of Q/K/V into the plan's order, the kernel,
    scatter of O back; sampling_layout.py:88-116 per call)."""
    from hilberta_b200.paired_kernel import raster_order, token_order_map

    rows = token_order_map(plan, dev)
    squares = raster_order(plan, dev)
    idx = rows.long()
    out = torch.empty_like(q)
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)

    def fused(ph):
        hb.paired_attention(q, k, v, metas[ph], out=out, token_order=squares, **kw)

    def gathered(ph):
        hb.paired_attention(q, k, v, metas[ph], out=out, token_order=rows, **kw)

    def explicit(ph):
        pq, pk, pv = (x.index_select(2, idx) for x in (q, k, v))
        o = hb.paired_attention(pq, pk, pv, metas[ph], **kw)
        out[:, :, idx] = o

    res = {}
    with torch.inference_mode():
        for name, fn in (("fused_ms_per_call", fused), ("gather4_ms_per_call", gathered),
                         ("explicit_ms_per_call", explicit)):
            for ph in range(4):
                fn(ph)
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                for ph in range(4):
                    fn(ph)
            e1.record()
            torch.cuda.synchronize()
            res[name] = round(e0.elapsed_time(e1) / (4 * steps), 4)
    res["note"] = ("Q/K/V in raster token order; fused = one 8x8-square TMA box per key/query block "
                   "(hb_paired_fwd_raster); gather4 = rows through a row map (tile::gather4)")
    return res


def run_e2e(a, q, k, v, metas, flops, world, dev, hb, fused=None):
    """Same metric through the public call with HOST buffers, streamed the way a
    caller feeding the attention from host memory would: call i's Q/K/V go
    host->device (pinned) on a copy stream while call i-1 computes, and call
    i-1's output goes device->host on another copy stream while call i
    computes; device inputs and outputs are double-buffered and ordered by
    events.  Every call's inputs cross PCIe in and its output crosses back out
    inside the timed region.  At N > 1 the attention is this rank's heads fused
    with the all-gather (PeerAllGather) and each rank reads back all heads."""
    import torch.distributed as dist

    hq, hk, hv = (x.detach().cpu().contiguous().pin_memory() for x in (q, k, v))
    B, hr, N, D = q.shape
    hout = [torch.empty((B, hr * world, N, D), dtype=q.dtype).pin_memory() for _ in range(2)]
    dins = [[torch.empty_like(x, device=dev) for x in (hq, hk, hv)] for _ in range(2)]
    douts = [torch.empty((B, hr, N, D), dtype=q.dtype, device=dev) for _ in range(2)]
    steps = max(1, a.steps)
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    compute = torch.cuda.current_stream(dev)
    h2d, d2h = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    ev = lambda: torch.cuda.Event()

    def run(n_calls):
        loaded = [None, None]   # event: inputs of buffer b are on the device
        consumed = [ev(), ev()]  # event: compute finished reading inputs of buffer b
        written = [None, None]  # event: output buffer b holds a result to read back
        drained = [ev(), ev()]  # event: output buffer b was copied to the host
        for e in (*consumed, *drained):
            e.record(compute)
        pending = None
        for i in range(n_calls + 1):
            b = i & 1
            if i < n_calls:  # stage call i's inputs
                with torch.cuda.stream(h2d):
                    h2d.wait_event(consumed[b])
                    for dst, src in zip(dins[b], (hq, hk, hv)):
                        dst.copy_(src, non_blocking=True)
                    loaded[b] = ev()
                    loaded[b].record(h2d)
            if pending is not None:  # read back the previous call's output
                pb, res = pending
                with torch.cuda.stream(d2h):
                    d2h.wait_event(written[pb])
                    hout[pb].copy_(res, non_blocking=True)
                    drained[pb].record(d2h)
                pending = None
            if i < n_calls:  # compute call i
                ph = STEP_PHASES[i % len(STEP_PHASES)]
                compute.wait_event(loaded[b])
                compute.wait_event(drained[b])
                if fused is not None and i > 0:
                    # peers write the buffer of call i-1 again during their call
                    # i+1, which may start once this rank's call i has finished:
                    # its read-back must be ordered before call i
                    compute.wait_event(drained[b ^ 1])
                if fused is None:
                    res = hb.paired_attention(*dins[b], metas[ph], out=douts[b], **kw)
                else:
                    res = fused(*dins[b], metas[ph], **kw)
                consumed[b].record(compute)
                written[b] = ev()
                written[b].record(compute)
                pending = (b, res)
        compute.wait_stream(h2d)
        compute.wait_stream(d2h)

    with torch.inference_mode():
        run(8)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(compute)
        run(len(STEP_PHASES) * steps)
        e1.record(compute)
        torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    ms = float(ms[0])
    calls = len(STEP_PHASES)
    h2d_bytes = sum(x.numel() * x.element_size() for x in (hq, hk, hv)) * calls * world
    d2h_bytes = hout[0].numel() * hout[0].element_size() * calls * world
    return {
        "value": round(sum(flops[ph] for ph in STEP_PHASES) * steps / (ms * 1e-3) / 1e12, 3),
        "unit": "TFLOP/s",
        "ms_per_step": round(ms / steps, 3),
        "h2d_bytes_per_step": h2d_bytes,
        "d2h_bytes_per_step": d2h_bytes,
        "steps": steps,
        "note": "per call: pinned Q/K/V H2D + attention + O D2H through the public API, copies of neighbouring calls "
        "overlapped on two copy streams"
        + (" (head_parallel.PeerAllGather: local heads in, all heads out)" if fused is not None else " (paired_attention)"),
    }


def triton_reference_child(a):
    """Child of ``triton_reference_side``: the reference's own GPU kernel, the
    Triton ``paired_attention`` of hilberta/paired_kernel.py:18-205 from the
    unmodified install in baseline/_ref, called as its benchmark calls it
    (global_strategy="triton", num_warps=8, num_stages=2; hilberta/benchmark.py:
    51-56) on this config, timed like that benchmark (10 warm-up and 30 timed
    launches per phase, CUDA events, median; phase weights 15/14/14/14), next to
    this package's kernel on the same inputs (relative L2 distance of the two
    outputs)."""
    import hilberta_b200 as hb

    sys.path.insert(0, str(ROOT / "baseline" / "_ref"))
    from hilberta.paired_kernel import paired_attention as ref_paired_attention

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    res, tiles, k = CONFIGS[a.config]
    plan = hb.bridge_k_plan(tiles, k, False, grid_size=res // 16)
    N, G = plan.total_tokens, plan.global_tokens
    torch.manual_seed(2707)
    q, kk, v = [torch.randn(1, a.heads, N, 128, device=dev, dtype=torch.bfloat16) for _ in range(3)]
    kw = dict(global_strategy="triton", num_warps=8, num_stages=2)
    med, ours, rel = [], [], []
    with torch.inference_mode():
        for p in plan.phases:
            meta = hb.pair_metadata(p.kv_indices, p.kv_counts, tokens=N, global_tokens=G).to(dev)
            for fn, acc in ((lambda: ref_paired_attention(q, kk, v, meta, **kw), med),
                            (lambda: hb.paired_attention(q, kk, v, meta, **kw), ours)):
                for _ in range(10):
                    fn()
                torch.cuda.synchronize()
                times = []
                for _ in range(30):
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    fn()
                    e1.record()
                    e1.synchronize()
                    times.append(e0.elapsed_time(e1))
                acc.append(statistics.median(times))
            a_out, b_out = ref_paired_attention(q, kk, v, meta, **kw).float(), hb.paired_attention(q, kk, v, meta, **kw).float()
            rel.append(float((a_out - b_out).norm() / a_out.norm()))
    wref = sum(w * m for w, m in zip(WEIGHTS, med)) / 57
    wour = sum(w * m for w, m in zip(WEIGHTS, ours)) / 57
    print(json.dumps({"ms_per_call": round(wref, 4), "ms_per_call_by_phase": [round(x, 4) for x in med],
                      "native_ms_per_call_same_protocol": round(wour, 4), "speedup": round(wref / wour, 3),
                      "rel_l2_vs_native": [round(x, 6) for x in rel]}), flush=True)


def triton_reference_side(a, timeout=900):
    """The reference's Triton kernel on this GPU (``triton_reference_child`` in a
    child process, so its JIT compile and context stay apart from this one),
    or the reason it could not run."""
    if not (ROOT / "baseline" / "_ref" / "hilberta" / "paired_kernel.py").exists():
        return {"unavailable": "reference not installed in baseline/_ref"}
    cmd = [sys.executable, str(ROOT / "bench.py"), "--triton-reference-child", "--config", a.config,
           "--heads", str(a.heads)]
    try:
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, cwd=ROOT,
                             env={**os.environ, "CUDA_VISIBLE_DEVICES": os.environ.get("CUDA_VISIBLE_DEVICES", "0")})
    except subprocess.TimeoutExpired:
        return {"unavailable": f"timed out after {timeout} s"}
    if res.returncode != 0:
        tail = (res.stderr or res.stdout).strip().splitlines()[-3:]
        return {"unavailable": f"exit {res.returncode}: " + " | ".join(tail)[-600:]}
    out = json.loads(res.stdout.strip().splitlines()[-1])
    out["kernel"] = "hilberta.paired_kernel.paired_attention (Triton, baseline/_ref), global_strategy=triton, 8 warps, 2 stages"
    out["protocol"] = "reference benchmark: 10 warm-up + 30 timed launches per phase, CUDA events, median, 15/14/14/14"
    return out


def workload_name(config, heads, tokens):
    """The workload string both arms print (the driver pairs the lines by it)."""
    return f"HilbertA paired sparse attention {config}, B=1, H={heads}, D=128, N={tokens}, G=512"


def shared_config(config, heads, tokens, world, layout, active):
    """The ``config`` object both arms print, identical for the same arguments
    (arm-specific details go in other keys)."""
    return {
        "workload": workload_name(config, heads, tokens),
        "layout": layout,
        "heads_per_gpu": heads // max(1, world),
        "step": "4 calls (tile phases 0-3); ms/call phase-weighted 15/14/14/14"
        + (", each with the all-gather of head outputs" if world > 1 else ""),
        "parallelism": f"head-parallel x{world}" if world > 1 else "single GPU",
        "l2": "GPU arm: L2 flushed before every call; CPU arm: no device cache involved",
        "active_blocks_per_phase": list(active),
    }


class CpuDenseMask:
    """The reference's dense-mask CPU path (plan mask + fp32 SDPA, the
    computation of hilberta/plan.py:70-84 with flux_adapter.py:299-307), as
    restated in oracle/attention_oracle.py, on bounded row samples of the four
    phases' calls, with every host thread.  Inputs follow the benchmark
    protocol (seed 2707, Q/K/V ~ N(0,1) bf16, upcast to fp32)."""

    def __init__(self, plan, heads):
        import numpy as np

        from oracle import attention_oracle as ao

        self.ao, self.np = ao, np
        self.threads = os.cpu_count() or 1
        torch.set_num_threads(self.threads)
        self.H, self.N, self.G = heads, plan.total_tokens, plan.global_tokens
        self.masks = [ao.block_mask_from_rows(np.asarray(p.kv_indices), np.asarray(p.kv_counts), self.N, self.G)
                      for p in plan.phases]
        self.row_active = [m.sum(1).repeat(64) for m in self.masks]  # active key blocks per query row
        g = torch.Generator().manual_seed(2707)
        # bf16 draws upcast to fp32 once, outside the timed samples (a whole
        # call amortises that conversion over every query row)
        self.qkv = [torch.randn(1, heads, self.N, 128, generator=g).to(torch.bfloat16).float() for _ in range(3)]
        self.rng = np.random.default_rng(0)

    def rows_for(self, seconds):
        """Rows per phase so that one sample (all four phases) takes ~`seconds`."""
        probe = self.sample(16)[0]
        per_row = probe / 64
        return int(max(16, min(self.N, seconds / max(per_row, 1e-6) / 4)))

    def sample(self, rows_per_phase):
        """One bounded sample: `rows_per_phase` random query rows of each phase's
        call.  Returns (seconds, active FLOP of the sampled rows)."""
        flop = 0.0
        t = time.perf_counter()
        for ph, mask in enumerate(self.masks):
            rows = self.np.sort(self.rng.choice(self.N, rows_per_phase, replace=False))
            self.ao.masked_attention_fp32(*self.qkv, mask, rows=rows, chunk=256)
            flop += self.H * 4 * 64 * 128 * float(self.row_active[ph][rows].sum())
        return time.perf_counter() - t, flop


def cpu_baseline(a, plan, active, bounded=15.0):
    """The CPU baseline leg of the native line: one bounded sample of the
    reference's dense-mask CPU path (``CpuDenseMask``) on this host."""
    cpu = CpuDenseMask(plan, a.heads)
    n = cpu.rows_for(bounded)
    sec, flop = cpu.sample(n)
    tflops = flop / sec / 1e12
    full_call_s = flop_per_call(sum(w * x for w, x in zip(WEIGHTS, active)) / 57, a.heads) / (tflops * 1e12)
    return {
        "value": round(tflops, 5),
        "unit": "TFLOP/s",
        "cores": cpu.threads,
        "kind": "port",
        "sample": f"{n} of {cpu.N} query rows x {cpu.H} heads of each of the 4 phases' calls, dense-mask fp32 SDPA "
        f"(torch CPU, oracle/attention_oracle.py); {sec:.1f} s; extrapolated {full_call_s:.1f} s per call",
        "ms_per_call_extrapolated": round(full_call_s * 1e3, 1),
    }


def run_reference(a):
    """``--impl reference``: the reference's CPU implementation of the path (its
    dense-mask path, restated as the oracle port; the reference is Python with
    no compiled CPU code) on this host's cores, on the native arm's config and
    metric.  Plans come from the oracle's restatement of the reference builder
    (oracle/plan_oracle.py); nothing of hilberta_b200 is imported.  Each step is
    one bounded sample (random query rows of each of the four phases' calls),
    sized so that warm-up plus timed steps take about two minutes; ``value`` is
    the active-block FLOP of the sampled rows over their wall time.  Under
    torchrun only rank 0 runs."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    from oracle import plan_oracle as po

    res, tiles, k = CONFIGS[a.config]
    plan = po.bridge_k_plan(tiles, k, False, grid_size=res // 16)
    N, G = plan.total_tokens, plan.global_tokens
    active = [(G // 64) * (N // 64) + int(p.kv_counts.sum()) for p in plan.phases]
    cpu = CpuDenseMask(plan, a.heads)
    steps, warmup = max(1, a.steps), max(0, a.warmup)
    per_step = min(a.cpu_seconds, max(0.5, 120.0 / (steps + warmup)))
    n = cpu.rows_for(per_step)
    for _ in range(warmup):
        cpu.sample(n)
    secs, flops = [], []
    for _ in range(steps):
        s, f = cpu.sample(n)
        secs.append(s)
        flops.append(f)
    value = sum(flops) / sum(secs) / 1e12
    ms_step = 1e3 * sum(secs) / steps
    full_step_flop = sum(flop_per_call(x, a.heads) for x in active)
    weighted_call_flop = flop_per_call(sum(w * x for w, x in zip(WEIGHTS, active)) / 57, a.heads)
    sample = (f"{n} of {N} query rows x {a.heads} heads of each of the 4 phases' calls per step, dense-mask fp32 "
              f"SDPA (torch CPU, oracle/attention_oracle.py)")
    line = {
        "metric": METRIC,
        "value": round(value, 5),
        "unit": "TFLOP/s",
        "impl": "reference",
        "n_gpus": a.gpus,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(ms_step, 1),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32 (from bf16 inputs)",
        "data": "synthetic (seeded N(0,1) bf16 Q/K/V, reference benchmark protocol)",
        "config": shared_config(a.config, a.heads, N, a.gpus, a.layout, active),
        "path": "reference dense-mask CPU path (plan.dense_mask + fp32 SDPA), oracle port",
        "step_sample": sample,
        "plan": "oracle/plan_oracle.py bridge_k_plan (restatement of hilberta/bridge_k.py, pinned by goldens)",
        "extrapolated": {
            "ms_per_call": round(weighted_call_flop / (value * 1e12) * 1e3, 1),
            "ms_per_step": round(full_step_flop / (value * 1e12) * 1e3, 1),
            "note": "whole calls (every query row) at the measured rate; not timed",
        },
        "cpu_baseline": {"kind": "port", "cores": cpu.threads, "sample": sample, "value": round(value, 5),
                         "unit": "TFLOP/s"},
        "e2e": {"value": round(value, 5), "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    a = parse()
    if a.triton_reference_child:
        triton_reference_child(a)
    elif a.impl == "reference":
        run_reference(a)
    else:
        run_native(a)


if __name__ == "__main__":
    main()
