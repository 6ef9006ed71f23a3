"""Benchmark of the B200 Gated DeltaNet operator pair (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload per GPU (weak scaling: per-GPU work is fixed as N grows, ranks use seed = rank):
  * headline step: one decode step at B=64 (state [64,8,128,128] fp32, updated in place).
    value = whole-job state HBM GB/s = N * 67,108,864 B / (max over ranks of the device time per step).
    Timed as CUDA-graph replays of K decode launches cycling over 8 state buffers
    (8 x 32 MiB = 256 MiB > the 126 MB L2, so every launch streams its state from HBM).
  * prefill_8k: one 8192-token sequence (cu_seqlens = [0, 8192], initial state N(0, 0.02)),
    tokens/s; L2 flushed before every timed step (a 256 MiB write, then a 256 MiB read of another
    buffer so that the write's dirty lines are written back outside the timed call), per-step
    CUDA events.
  * decode_sweep (config 1): B = 1 .. 512, each over rotating state buffers (>= 384 MiB), beside
    the reference's published latencies.
  * prefill_configs: single sequences of 64 .. 4096 tokens (beside the reference's published table),
    one 1024-token sequence, 1000 x 16 and 4000 x 6 short sequences (the short-sequence kernels), 16 log-uniform varlen sequences (total <= 32768)
    and 8 packed 1024-token sequences per GPU, timed the same way; plus 64 x 4096 tokens split by
    sequence over the ranks (strong scaling; whole-job tokens/s over the slowest rank).
  * e2e: the same two metrics through the public API (gdn.decode.kernel / gdn.prefill.kernel)
    with pinned host buffers: every step copies its inputs host->device and its results back
    (one pinned host arena, one copy each way per step), pipelined over copy-in / compute /
    copy-out streams as a serving loop runs them.
  * cpu_baseline: the CPU oracle (a C restatement of the reference's sequential PyTorch
    loops, all host threads) on a bounded sample of the same workload, rank 0 only.
--impl reference times that same CPU oracle as the reference arm (the reference itself is
Python-only and cannot be installed on the GPU box, so its algorithm runs as the C port).
Multi-GPU: one process per GPU under torchrun; no collective on the data path, a barrier and
a MAX all-reduce of the timings only.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
for _p in (ROOT, os.path.join(ROOT, "gated-delta-network_b200")):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode µs/step + state HBM GB/s at B=64; prefill tokens/s at 8K tokens"
H, HV, D = 4, 8, 128
DECODE_B = 64
PREFILL_T = 8192
STATE_BYTES_PER_ELEM = HV * D * D * 4                     # 524,288 B of fp32 state per batch element
DECODE_STATE_BYTES = DECODE_B * STATE_BYTES_PER_ELEM * 2  # read + write = 67,108,864 B
# algorithmic bytes of one decode launch: state r+w, q,k (2x4x128 bf16), v,out (2x8x128 bf16), a,b, A_log, dt_bias
DECODE_ALG_BYTES = DECODE_B * (2 * STATE_BYTES_PER_ELEM + 2 * H * D * 2 + 2 * HV * D * 2 + 2 * HV * 2) + 2 * HV * 4
# prefill: per token q,k (2x4x128 bf16) + v (8x128 bf16) + a,b (2x8 bf16) + out (8x128 bf16); per sequence state in+out
PREFILL_ALG_BYTES_PER_TOKEN = 2 * H * D * 2 + HV * D * 2 + 2 * HV * 2 + HV * D * 2   # 6,176 B
PREFILL_FLOPS_PER_TOKEN = (10 * 64 * 128 + 6 * 128 * 128) * HV                      # chunked WY form, 1,441,792
N_STATE_BUFS = 8
REPS = 5  # timed repetitions of every measurement; the median is reported
# DRAM bytes per launch measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum), or None.
# Source: the ncu summaries under profiles/ (decode B=64 launch; prefill at T=8192).
# decode: 33.83 MB read; the 33.55 MB of state writes are still dirty in L2 when ncu's replayed launch ends.
# prefill_8k_call: the four launches of one default-route call (prep 60.0 MB, segment-local 88.1, chain 7.6,
# output 52.8), each measured with ncu's per-kernel cache flush.
# prefill_8k_call_warm: the same four launches with ncu's --cache-control none (caches kept between kernels, as
# in the timed call): 256 MB, because write-backs of earlier kernels' dirty lines then land in later kernels
# (prep 100.5 MB, segment-local 111.3, chain 3.2, output 40.8).
NCU_TRAFFIC = {"decode": 33832960, "prefill_8k_call": 208500000, "prefill_8k_call_warm": 255800000}
# Critical path of the 8K call with the current kernels given unlimited SMs (us): one prep item (~11), the local
# chain of one segment (15 chunk steps x ~2.95), the chain over 9 segments (~0.92 each) and one output item (~5),
# from the phase counters and the warm launch list.  The remaining time of the call is throughput: the prep's
# 1024 (chunk, v-head) items take 3.5 waves of two CTAs per SM.
PREFILL_8K_CRITICAL_PATH_US = 68.5


def env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


def load_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            pk = json.load(f)
        return float(pk["hbm_gbs"]), float(pk["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]
        return False

    def summary(self):
        sms, maxs, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sms.append(float(parts[1]))
                maxs.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(nm)
        if not sms:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        return {"sm_mhz": statistics.median(sms), "sm_max_mhz": max(maxs), "reasons": sorted(reasons),
                "samples": len(sms)}


def host_threads():
    """Cores this process may run on (torchrun sets OMP_NUM_THREADS=1, which must not shrink the baseline)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_decode_baseline(budget_s=10.0, threads=0):
    """CPU oracle on decode B=64 (same inputs as the headline), repeated for ~budget_s."""
    from oracle import oracle

    threads = threads or host_threads()
    from tests.golden import inputs as gi

    inp = gi.decode_inputs(DECODE_B, seed=0)
    args = (inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
            inp["scale"])
    oracle.decode(*args, threads=threads)  # warm-up
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.decode(*args, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= budget_s:
            break
    per = el / n
    return {"value": DECODE_STATE_BYTES / per / 1e9, "unit": "GB/s", "cores": threads or oracle.max_threads(),
            "kind": "port", "us_per_step": per * 1e6,
            "sample": f"{n} decode steps at B=64 (CPU oracle, fp32), {el:.1f} s"}


def cpu_prefill_baseline(tokens=1024, threads=0):
    """CPU oracle on the first `tokens` tokens of one sequence: tokens/s (the oracle is linear in T)."""
    from oracle import oracle

    threads = threads or host_threads()
    from tests.golden import inputs as gi

    inp = gi.prefill_inputs([tokens], seed=0, with_state=True)
    t0 = time.perf_counter()
    oracle.prefill(inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"],
                   inp["cu_seqlens"], inp["scale"], threads=threads)
    el = time.perf_counter() - t0
    return {"value": tokens / el, "unit": "tokens/s", "cores": threads or oracle.max_threads(), "kind": "port",
            "sample": f"one {tokens}-token sequence of the 8K workload (CPU oracle), {el:.2f} s; "
                      f"the sequential oracle's cost is linear in tokens"}


def bind_host_to_gpu(dev_index):
    """Restrict this process to the CPUs local to its GPU's PCIe root (sysfs local_cpulist), so
    that pinned host buffers are first touched -- and placed -- on the GPU's own NUMA node.
    Returns a description for the JSON line."""
    import torch

    try:
        pr = torch.cuda.get_device_properties(dev_index)
        bdf = f"{pr.pci_domain_id:04x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
        base = f"/sys/bus/pci/devices/{bdf}"
        with open(base + "/local_cpulist") as f:
            cpulist = f.read().strip()
        try:
            with open(base + "/numa_node") as f:
                node = int(f.read().strip())
        except OSError:
            node = -1
        cpus = set()
        for part in cpulist.split(","):
            lo, _, hi = part.partition("-")
            cpus.update(range(int(lo), int(hi or lo) + 1))
        cpus &= os.sched_getaffinity(0)
        if cpus:
            os.sched_setaffinity(0, cpus)
        return {"pci": bdf, "numa_node": node, "cpus": cpulist}
    except Exception as exc:  # sysfs layout differs: keep the default placement
        return {"unbound": str(exc)[:80]}


def decode_config(world):
    """Workload of the headline line, shared by both arms (the same dict in each)."""
    return {"workload": "decode B=64 per GPU (qk4_v8_d128, k-last fp32 state, in place), one step",
            "global_batch": DECODE_B * world, "seq_len": 1,
            "parallelism": f"dp{world}: the global batch in {world} independent shards"}


def run_reference_arm(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle

    threads = host_threads()
    times = []
    from tests.golden import inputs as gi

    # the same global batch as the GPU arm: B = 64 per GPU x N GPUs, on the host cores
    gb = DECODE_B * world
    inp = gi.decode_inputs(gb, seed=0)
    a = (inp["q"], inp["k"], inp["v"], inp["state"], inp["A_log"], inp["a"], inp["dt_bias"], inp["b"], inp["scale"])
    for _ in range(args.warmup):
        oracle.decode(*a, threads=threads)
    for _ in range(args.steps):
        t0 = time.perf_counter()
        oracle.decode(*a, threads=threads)
        times.append(time.perf_counter() - t0)
    per = sum(times) / len(times)
    val = world * DECODE_STATE_BYTES / per / 1e9
    line = {
        "metric": METRIC, "value": round(val, 3), "unit": "GB/s", "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(per * 1e3, 3), "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": decode_config(world),
        "timing": f"host wall clock (time.perf_counter) per step, mean of --steps steps, rank 0 only",
        "cpu_baseline": {"value": round(val, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{args.steps} full decode steps at B={gb} (the whole global batch) of the C "
                                   f"restatement of reference/gdn_decode_ref.py, {threads} threads"},
        "e2e": {"value": round(val, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def profile_run(args):
    """A few calls of one prefill or decode configuration with the benchmark's input distributions,
    nothing timed: the command that the ncu summaries under profiles/ capture."""
    import torch

    import gdn
    from gdn import prefill as pmod

    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    rn = lambda *sh: torch.randn(*sh, generator=g, device=dev)
    l2n = lambda x: (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)
    # prefill may take other head counts (N,T,FLAGS,H,HV): e.g. the pieces of a head split
    parts = [int(x, 0) for x in args.profile_prefill.split(",")] if args.profile_prefill else []
    nh, nhv = (parts[3], parts[4]) if len(parts) > 4 else (H, HV)
    A_log = torch.rand(nhv, generator=g, device=dev) * math.log(16.0)
    dt_bias = rn(nhv) * 0.1
    if args.profile_decode:
        B = args.profile_decode
        q, k = l2n(rn(B, 1, H, D)), l2n(rn(B, 1, H, D))
        v, a, b = rn(B, 1, HV, D).bfloat16(), rn(B, 1, HV).bfloat16(), rn(B, 1, HV).bfloat16()
        st = rn(B, HV, D, D) * 0.02
        out = torch.empty(B, 1, HV, D, dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            gdn.decode.kernel(q, k, v, st, A_log, a, dt_bias, b, D ** -0.5, out, st)
    else:
        N, T, flags = parts[0], parts[1], (parts[2] if len(parts) > 2 else 0)
        TT = N * T
        q, k = l2n(rn(TT, nh, D)), l2n(rn(TT, nh, D))
        v, a, b = rn(TT, nhv, D).bfloat16(), rn(TT, nhv).bfloat16(), rn(TT, nhv).bfloat16()
        h0 = rn(N, nhv, D, D) * 0.02
        cu = torch.arange(N + 1, dtype=torch.int32, device=dev) * T
        out = torch.empty(TT, nhv, D, dtype=torch.bfloat16, device=dev)
        ns = torch.empty(N, nhv, D, D, device=dev)
        ws = torch.empty(gdn.prefill.workspace_bytes(N, TT, nh, nhv), dtype=torch.uint8, device=dev)
        for _ in range(3):
            pmod._launch(q, k, v, h0, A_log, a, dt_bias, b, cu, D ** -0.5, out, ns, workspace=ws, flags=flags)
    torch.cuda.synchronize()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--prefill-steps", type=int, default=20)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--profile-prefill", metavar="N,T[,FLAGS[,H,HV]]", default=None,
                    help="profiling aid (ncu): run 3 prefill calls of N sequences x T tokens (library flags, "
                         "e.g. 0x8 for the single-pass scan; optional head counts, e.g. 1,2 for a piece of a "
                         "4-way head split) and exit; prints no JSON line")
    ap.add_argument("--profile-decode", metavar="B", type=int, default=None,
                    help="profiling aid (ncu): run 3 decode steps at batch B and exit")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    rank = env_int("RANK", 0)
    world = env_int("WORLD_SIZE", 1)
    local_rank = env_int("LOCAL_RANK", 0)

    if args.impl == "reference":
        run_reference_arm(args, rank, world)
        return
    if args.profile_prefill or args.profile_decode:
        profile_run(args)
        return

    import torch
    import torch.distributed as dist

    import gdn

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    orig_affinity = os.sched_getaffinity(0)
    host_binding = bind_host_to_gpu(local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    hbm_peak, tc_peak, peak_src = load_peaks()
    gen = torch.Generator(device=dev).manual_seed(rank)

    def randn(shape, std=1.0, dtype=torch.float32):
        return (torch.randn(shape, generator=gen, device=dev, dtype=torch.float32) * std).to(dtype)

    def l2n(x):
        return (x / x.norm(dim=-1, keepdim=True)).to(torch.bfloat16)

    # ---------------- decode B=64 ----------------
    B = DECODE_B
    q = l2n(randn((B, 1, H, D)))
    k = l2n(randn((B, 1, H, D)))
    v = randn((B, 1, HV, D), dtype=torch.bfloat16)
    a = randn((B, 1, HV), dtype=torch.bfloat16)
    b = randn((B, 1, HV), dtype=torch.bfloat16)
    A_log = torch.rand(HV, generator=gen, device=dev) * math.log(16.0)
    dt_bias = randn((HV,), 0.1)
    scale = 1.0 / math.sqrt(D)
    states = [randn((B, HV, D, D), 0.02) for _ in range(N_STATE_BUFS)]
    out = torch.empty((B, 1, HV, D), dtype=torch.bfloat16, device=dev)

    def decode_step(i):
        st = states[i % N_STATE_BUFS]
        gdn.decode.kernel(q, k, v, st, A_log, a, dt_bias, b, scale, out, st)

    # CUDA graph of exactly K = --steps launches, cycling over the N_STATE_BUFS state buffers.
    side = torch.cuda.Stream(device=dev)
    side.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(side):
        for i in range(N_STATE_BUFS):
            decode_step(i)
    torch.cuda.current_stream(dev).wait_stream(side)

    def capture(n):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for i in range(n):
                decode_step(i)
        return g

    steps = args.steps
    graph = capture(steps)
    # >= 10 ms of launches in one region, the stability cross-check of the K-step number
    n_long = max(N_STATE_BUFS, -(-int(10e-3 / 11e-6) // N_STATE_BUFS) * N_STATE_BUFS)
    graph_long = capture(n_long)
    for _ in range(args.warmup):
        graph.replay()
    graph_long.replay()
    barrier()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)

    def timed_replay(g, n):
        """Device time per launch of one replay of `g` (n launches).  A ~1 ms sleep kernel queued
        first keeps the GPU busy while the host submits the graph, so the region holds the
        launches back to back and no host submission latency."""
        barrier()
        torch.cuda._sleep(2_000_000)
        ev0.record()
        g.replay()
        ev1.record()
        barrier()
        return ev0.elapsed_time(ev1) / n

    with ClockSampler(local_rank) as clocks:
        rep_ms = [max_over_ranks(timed_replay(graph, steps)) for _ in range(REPS)]
        long_ms = [max_over_ranks(timed_replay(graph_long, n_long)) for _ in range(REPS)]
    dec_ms = statistics.median(rep_ms)
    dec_long_ms = statistics.median(long_ms)
    clock_summary = clocks.summary()
    del graph_long

    # eager launches (Python + ctypes path, no graph)
    barrier()
    ev0.record()
    for i in range(steps):
        decode_step(i)
    ev1.record()
    barrier()
    dec_eager_ms = max_over_ranks(ev0.elapsed_time(ev1) / steps)

    # ---------------- decode batch sweep (config 1), beside the reference's published latencies ----------------
    def time_decode(bs):
        sbytes = bs * STATE_BYTES_PER_ELEM
        nb = max(2, min(768, -(-(384 << 20) // sbytes)))  # rotating state buffers: >= 384 MiB, 3x the L2
        sq, sk = l2n(randn((bs, 1, H, D))), l2n(randn((bs, 1, H, D)))
        sv = randn((bs, 1, HV, D), dtype=torch.bfloat16)
        sa, sb = randn((bs, 1, HV), dtype=torch.bfloat16), randn((bs, 1, HV), dtype=torch.bfloat16)
        sts = [randn((bs, HV, D, D), 0.02) for _ in range(nb)]
        so = torch.empty((bs, 1, HV, D), dtype=torch.bfloat16, device=dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            for st in sts:
                gdn.decode.kernel(sq, sk, sv, st, A_log, sa, dt_bias, sb, scale, so, st)
        torch.cuda.current_stream(dev).wait_stream(side)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g):
            for st in sts:
                gdn.decode.kernel(sq, sk, sv, st, A_log, sa, dt_bias, sb, scale, so, st)
        reps = max(2, 400 // nb)
        g.replay()
        per_rep = []
        for _ in range(REPS):
            barrier()
            torch.cuda._sleep(2_000_000)
            ev0.record()
            for _ in range(reps):
                g.replay()
            ev1.record()
            barrier()
            per_rep.append(max_over_ranks(ev0.elapsed_time(ev1) / (reps * nb)))
        ms = statistics.median(per_rep)
        del g, sts
        return {"us_per_step": round(ms * 1e3, 3), "state_GBps": round(2 * sbytes / (ms * 1e-3) / 1e9, 1),
                "frac_of_hbm_peak": round(2 * sbytes / (ms * 1e-3) / 1e9 / hbm_peak, 4)}

    # the reference's published Triton decode latencies on B200 (README.md:42-49, OPTIMIZATION_LOG.md:44, 56-57)
    ref_decode_us = {1: 26.0, 4: 23.5, 8: 23.5, 16: 23.5, 32: 23.5, 48: 23.5, 64: 23.5, 128: 27.89, 512: 86.79}
    decode_sweep = {}
    for bs in (1, 4, 8, 16, 32, 48, 64, 128, 512):
        decode_sweep[f"B={bs}"] = dict(time_decode(bs), reference_published_us=ref_decode_us[bs])

    # config 4, decode half: B = 512 split by batch over the ranks (strong scaling, no collective);
    # whole-job state traffic over the slowest rank's time per step
    from gdn.shard import batch_shard

    b0, b1 = batch_shard(512, world, rank)
    c4d = time_decode(b1 - b0)
    c4_dec = {"us_per_step": c4d["us_per_step"], "local_batch": b1 - b0,
              "state_GBps_whole_job": round(512 * STATE_BYTES_PER_ELEM * 2 / (c4d["us_per_step"] * 1e-6) / 1e9, 1),
              "frac_of_hbm_peak_per_gpu": c4d["frac_of_hbm_peak"],
              "scaling": "strong: decode B=512 split by batch over the ranks"}

    # ---------------- prefill 8K ----------------
    T = PREFILL_T
    pq = l2n(randn((T, H, D)))
    pk = l2n(randn((T, H, D)))
    pv = randn((T, HV, D), dtype=torch.bfloat16)
    pa = randn((T, HV), dtype=torch.bfloat16)
    pb = randn((T, HV), dtype=torch.bfloat16)
    ph0 = randn((1, HV, D, D), 0.02)
    cu = torch.tensor([0, T], dtype=torch.int32, device=dev)
    pout = torch.empty((T, HV, D), dtype=torch.bfloat16, device=dev)
    pns = torch.empty((1, HV, D, D), dtype=torch.float32, device=dev)
    ws = torch.empty(gdn.prefill.workspace_bytes(1, T), dtype=torch.uint8, device=dev)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    flush_rd = torch.zeros(32 * 1024 * 1024, dtype=torch.int64, device=dev)

    def flush_l2(clean=True):
        # A 256 MiB write evicts everything earlier steps left in L2.  It leaves L2 full of its own
        # dirty lines, whose write-back would then land inside the next timed call (~126 MB, about
        # 20 us of HBM time at 8K); reading another 256 MiB afterwards writes them back here and
        # leaves L2 holding clean, unrelated lines.  clean=False keeps the dirty-L2 variant.
        flush.fill_(1)
        if clean:
            flush_rd.sum()
    from gdn import prefill as pmod

    def prefill_step(flags=0):
        pmod._launch(pq, pk, pv, ph0, A_log, pa, dt_bias, pb, cu, scale, pout, pns, workspace=ws, flags=flags)

    def time_8k(flags, clean=True):
        for _ in range(args.warmup):
            prefill_step(flags)
        barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.prefill_steps)]
        for e0, e1 in evs:
            flush_l2(clean)
            torch.cuda._sleep(2_000_000)  # ~1 ms: the GPU stays busy while the host submits the call
            e0.record()
            prefill_step(flags)
            e1.record()
        barrier()
        return max_over_ranks(statistics.median(e0.elapsed_time(e1) for e0, e1 in evs))

    # Host-side pauses (the interpreter's garbage collector in this large process) inside a timed
    # region would leave the GPU idle between a call's launches: collection is off while the prefill
    # sections run, and each timed call is queued behind a ~1 ms sleep kernel.
    gc.collect()
    gc.disable()
    pre_ms = time_8k(0)  # the library's default route (segmented for one 8192-token sequence)

    # the same sequence split by v-head over the ranks (gdn.shard.head_shard: each rank runs its q/k
    # head group, no exchange), strong scaling; at N = 1 also the pieces a 4- and an 8-GPU split run
    from gdn.shard import head_shard

    def time_8k_heads(world_, rank_):
        h0, h1, v0, v1 = head_shard(H, HV, world_, rank_, prefill=True)
        xq, xk = pq[:, h0:h1].contiguous(), pk[:, h0:h1].contiguous()
        xv, xa, xb = pv[:, v0:v1].contiguous(), pa[:, v0:v1].contiguous(), pb[:, v0:v1].contiguous()
        xh, xA, xdt = ph0[:, v0:v1].contiguous(), A_log[v0:v1].contiguous(), dt_bias[v0:v1].contiguous()
        xo = torch.empty((T, v1 - v0, D), dtype=torch.bfloat16, device=dev)
        xs = torch.empty((1, v1 - v0, D, D), dtype=torch.float32, device=dev)
        xws = torch.empty(gdn.prefill.workspace_bytes(1, T, num_qk_heads=h1 - h0, num_v_heads=v1 - v0), dtype=torch.uint8, device=dev)

        def step():
            pmod._launch(xq, xk, xv, xh, xA, xa, xdt, xb, cu, scale, xo, xs, workspace=xws)

        for _ in range(args.warmup):
            step()
        barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.prefill_steps)]
        for e0, e1 in evs:
            flush_l2()
            torch.cuda._sleep(2_000_000)
            e0.record()
            step()
            e1.record()
        barrier()
        return max_over_ranks(statistics.median(e0.elapsed_time(e1) for e0, e1 in evs)), (h1 - h0, v1 - v0)

    hs_ms, hs_heads = time_8k_heads(world, rank)
    head_split = {"ms_per_step": round(hs_ms, 5), "tokens_per_s": round(T / (hs_ms * 1e-3), 1),
                  "heads_per_rank": {"qk": hs_heads[0], "v": hs_heads[1]},
                  "scaling": "strong: one 8192-token sequence split by v-head over the ranks (gdn.shard.head_shard)"}
    if world == 1:
        head_split["one_rank_of_4_ms"] = round(time_8k_heads(4, 0)[0], 5)
        head_split["one_rank_of_8_ms"] = round(time_8k_heads(8, 0)[0], 5)
    pre_routes = {"segmented_ms": round(time_8k(0x10), 5), "single_pass_scan_ms": round(time_8k(0x8), 5),
                  "dirty_l2_flush_ms": round(time_8k(0, clean=False), 5)}

    # ---------------- other prefill configurations (reported alongside) ----------------
    def time_prefill(lens, with_state, steps=10):
        Tn, Nn = int(sum(lens)), len(lens)
        xq, xk = l2n(randn((Tn, H, D))), l2n(randn((Tn, H, D)))
        xv = randn((Tn, HV, D), dtype=torch.bfloat16)
        xa, xb = randn((Tn, HV), dtype=torch.bfloat16), randn((Tn, HV), dtype=torch.bfloat16)
        xh = randn((Nn, HV, D, D), 0.02) if with_state else None
        xcu = torch.tensor([0] + torch.tensor(lens).cumsum(0).tolist(), dtype=torch.int32, device=dev)
        xo = torch.empty((Tn, HV, D), dtype=torch.bfloat16, device=dev)
        xs = torch.empty((Nn, HV, D, D), dtype=torch.float32, device=dev)
        xws = torch.empty(gdn.prefill.workspace_bytes(Nn, Tn), dtype=torch.uint8, device=dev)

        def step():
            pmod._launch(xq, xk, xv, xh, A_log, xa, dt_bias, xb, xcu, scale, xo, xs, workspace=xws)

        for _ in range(3):
            step()
        barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            flush_l2()
            torch.cuda._sleep(2_000_000)  # ~1 ms: the GPU stays busy while the host submits the call
            e0.record()
            step()
            e1.record()
        barrier()
        ms = max_over_ranks(statistics.median(e0.elapsed_time(e1) for e0, e1 in evs))
        return {"tokens_per_s": round(world * Tn / (ms * 1e-3), 1), "ms_per_step": round(ms, 5), "tokens": Tn,
                "sequences": Nn}

    from tests.golden.inputs import varlen_lengths  # seeded log-uniform lengths (numpy only)

    from gdn.shard import seq_shard

    # config 4: 64 x 4096 tokens partitioned by sequence over the ranks (strong scaling, no collective)
    c4_cu = [4096 * i for i in range(65)]
    _, _, c4_t0, c4_t1, c4_local = seq_shard(c4_cu, world, rank)
    c4 = time_prefill([c4_local[i + 1] - c4_local[i] for i in range(len(c4_local) - 1)], True, steps=3)
    c4["tokens_per_s"] = round(64 * 4096 / (c4["ms_per_step"] * 1e-3), 1)  # whole job over max-rank time
    c4["scaling"] = "strong: 64 sequences x 4096 tokens split over the ranks"

    prefill_more = {
        "1x1024 (config 2, zero initial state)": time_prefill([1024], False),
        # single sequences at the lengths of the reference's published prefill table (README.md:86-90, 106-107)
        "1x64": dict(time_prefill([64], True), reference_published_ms=0.202),
        "1x256": dict(time_prefill([256], True), reference_published_ms=0.204),
        "1x512": dict(time_prefill([512], True), reference_published_ms=0.199),
        "1x2048": dict(time_prefill([2048], True), reference_published_ms=0.229),
        "1x4096": dict(time_prefill([4096], True), reference_published_ms=0.420),
        "16 varlen, log-uniform [6, 8192] (config 3)": time_prefill(varlen_lengths(), True),
        "8x1024 packed": time_prefill([1024] * 8, True),
        # batches of short prompts: the short-sequence kernels (one-chunk tensor-core / token recurrence)
        "1000x16 short sequences": time_prefill([16] * 1000, True),
        "4000x6 short sequences": time_prefill([6] * 4000, True),
        "64x4096 partitioned (config 4)": c4,
    }

    # FlashInfer-Bench style timing: every argument (inputs and the destination tensors) is cloned
    # before each iteration inside the timed region, then the public destination-passing call runs
    # (the reference's published clone-mode table, README.md:115-120).
    def time_prefill_clone(T_, steps=20):
        xq, xk = l2n(randn((T_, H, D))), l2n(randn((T_, H, D)))
        xv = randn((T_, HV, D), dtype=torch.bfloat16)
        xa, xb = randn((T_, HV), dtype=torch.bfloat16), randn((T_, HV), dtype=torch.bfloat16)
        xh = randn((1, HV, D, D), 0.02)
        xcu = torch.tensor([0, T_], dtype=torch.int32, device=dev)
        xo = torch.empty((T_, HV, D), dtype=torch.bfloat16, device=dev)
        xs = torch.empty((1, HV, D, D), dtype=torch.float32, device=dev)
        argl = [xq, xk, xv, xh, A_log, xa, dt_bias, xb, xcu, xo, xs]

        def it():
            c = [t.clone() for t in argl]
            gdn.prefill.kernel(c[0], c[1], c[2], c[3], c[4], c[5], c[6], c[7], c[8], scale, c[9], c[10])

        for _ in range(3):
            it()
        barrier()
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        for e0, e1 in evs:
            e0.record()
            it()
            e1.record()
        barrier()
        ms = max_over_ranks(statistics.median(e0.elapsed_time(e1) for e0, e1 in evs))
        return {"ms_per_step": round(ms, 5), "tokens_per_s": round(world * T_ / (ms * 1e-3), 1)}

    prefill_clone = {
        "1x1024": dict(time_prefill_clone(1024), reference_published_clone_ms=0.546),
        "1x4096": dict(time_prefill_clone(4096), reference_published_clone_ms=0.805),
        "method": "median of 20 iterations; each clones all 11 tensor arguments, then calls gdn.prefill.kernel, "
                  "both inside the CUDA-event region (FlashInfer-Bench do_bench _clone_args)",
    }
    gc.enable()

    # ---------------- e2e through the public API with pinned host buffers ----------------
    # Every step copies its inputs host -> device from pinned memory, runs the public call and
    # copies its results back.  A serving loop stages a step's tensors in one pinned host arena
    # and one device arena per buffer set (the tensors are views into it), so each step is one
    # host -> device copy of [inputs | state] and one device -> host copy of [state or outputs]:
    # six separate copies per step measured ~6% slower on the same box (per-copy setup, and
    # small copies interleaved with the large ones in each direction).  Steps are pipelined:
    # copy-in, compute and copy-out on three streams over a ring of three device arenas, so
    # step i's device -> host copy overlaps step i + 1's host -> device copy (PCIe is full
    # duplex).  The timed region runs from the first copy-in to the last copy-out.
    def arena_layout(specs):
        """specs: (shape, dtype) list -> (byte offsets 256-aligned, total bytes)."""
        offs, off = [], 0
        for shape, dt in specs:
            offs.append(off)
            nbytes = math.prod(shape) * torch.empty((), dtype=dt).element_size()
            off = (off + nbytes + 255) // 256 * 256
        return offs, off

    def arena_views(buf, specs, offs):
        return [buf[o:o + math.prod(sh) * torch.empty((), dtype=dt).element_size()].view(dt).view(sh)
                for (sh, dt), o in zip(specs, offs)]

    def pipelined_e2e(h_in, out_specs, launch, n_steps, inout_last=False, n_bufs=3):
        """h_in: host tensors copied in every step; out_specs: (shape, dtype) of the results copied
        back.  With inout_last the last input is updated in place and copied back too (decode's
        state).  launch(ins, outs) makes the public call on device views."""
        specs = [(tuple(t.shape), t.dtype) for t in h_in] + list(out_specs)
        offs, total = arena_layout(specs)
        n_in = len(h_in)
        h2d_end = offs[n_in - 1] + h_in[-1].numel() * h_in[-1].element_size()
        d2h_begin = offs[n_in - 1] if inout_last else offs[n_in]
        h_arena = torch.empty(total, dtype=torch.uint8).pin_memory()
        for t, v_ in zip(h_in, arena_views(h_arena, specs, offs)):
            v_.copy_(t)
        d_arena = [torch.empty(total, dtype=torch.uint8, device=dev) for _ in range(n_bufs)]
        d_views = [arena_views(d, specs, offs) for d in d_arena]
        h_back = [torch.empty(total - d2h_begin, dtype=torch.uint8).pin_memory() for _ in range(n_bufs)]
        s_in, s_run, s_out = (torch.cuda.Stream(device=dev) for _ in range(3))
        ev_in = [torch.cuda.Event() for _ in range(n_bufs)]
        ev_run = [torch.cuda.Event() for _ in range(n_bufs)]
        ev_out = [torch.cuda.Event() for _ in range(n_bufs)]

        def run(n):
            for i in range(n):
                j = i % n_bufs
                if i >= n_bufs:
                    s_in.wait_event(ev_out[j])  # buffer set j is free again
                with torch.cuda.stream(s_in):
                    d_arena[j][:h2d_end].copy_(h_arena[:h2d_end], non_blocking=True)
                    ev_in[j].record(s_in)
                s_run.wait_event(ev_in[j])
                with torch.cuda.stream(s_run):
                    launch(d_views[j][:n_in], d_views[j][n_in:])
                    ev_run[j].record(s_run)
                s_out.wait_event(ev_run[j])
                with torch.cuda.stream(s_out):
                    h_back[j].copy_(d_arena[j][d2h_begin:], non_blocking=True)
                    ev_out[j].record(s_out)

        cur = torch.cuda.current_stream(dev)
        for st_ in (s_in, s_run, s_out):
            st_.wait_stream(cur)
        run(n_bufs)
        torch.cuda.synchronize()
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record(s_in)
        run(n_steps)
        t1.record(s_out)
        torch.cuda.synchronize()
        barrier()
        return max_over_ranks(t0.elapsed_time(t1) / n_steps), h2d_end, total - d2h_begin

    def host_link_rates(nbytes=64 << 20, reps=5):
        """H2D and D2H copy rates of this rank from pinned memory, all ranks copying at the same
        time (the e2e loop's situation): the per-rank numbers locate a shared host-side limit."""
        hb = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        db = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        out = {}
        for name, fn in (("h2d_GBps", lambda: db.copy_(hb, non_blocking=True)),
                         ("d2h_GBps", lambda: hb.copy_(db, non_blocking=True))):
            fn()
            barrier()
            ev0.record()
            for _ in range(reps):
                fn()
            ev1.record()
            barrier()
            out[name] = round(reps * nbytes / (ev0.elapsed_time(ev1) * 1e-3) / 1e9, 2)
        # both directions at once on two streams (what the pipelined e2e loop does), every rank at once:
        # the sum over ranks of bidir_GBps is the host-side throughput the whole box reached
        hb2 = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
        db2 = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        s_a, s_b = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        cur = torch.cuda.current_stream(dev)
        barrier()
        ev0.record()
        s_a.wait_stream(cur)
        s_b.wait_stream(cur)
        for _ in range(reps):
            with torch.cuda.stream(s_a):
                db.copy_(hb, non_blocking=True)
            with torch.cuda.stream(s_b):
                hb2.copy_(db2, non_blocking=True)
        cur.wait_stream(s_a)
        cur.wait_stream(s_b)
        ev1.record()
        barrier()
        out["bidir_GBps"] = round(2 * reps * nbytes / (ev0.elapsed_time(ev1) * 1e-3) / 1e9, 2)
        return out

    e2e = None
    pre_e2e = None
    link = None
    if not args.no_e2e:
        link = host_link_rates()
        if world > 1:
            allr = [None] * world
            dist.all_gather_object(allr, {**link, **host_binding})
            link = {"per_rank": allr}
        n_e2e = max(6, min(30, args.steps // 8))
        h_dec = [t.cpu() for t in (q, k, v, a, b, states[0])]

        def dec_launch(d, o):  # in place: the state view is also new_state
            gdn.decode.kernel(d[0], d[1], d[2], d[5], A_log, d[3], dt_bias, d[4], scale, o[0], d[5])

        e2e_ms, h2d, d2h = pipelined_e2e(h_dec, [(tuple(out.shape), out.dtype)], dec_launch, n_e2e, inout_last=True)
        e2e = {"value": round(world * DECODE_STATE_BYTES / (e2e_ms * 1e-3) / 1e9, 3), "unit": "GB/s",
               "ms_per_step": round(e2e_ms, 4), "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "pipeline": "copy-in / compute / copy-out streams, 3 device arenas, one pinned host arena: one H2D and one D2H copy per step"}

        hcu = torch.tensor([0, T], dtype=torch.int32)
        h_pre = [t.cpu() for t in (pq, pk, pv, pa, pb, hcu, ph0)]

        def pre_launch(d, o):
            gdn.prefill.kernel(d[0], d[1], d[2], d[6], A_log, d[3], dt_bias, d[4], d[5], scale, o[0], o[1])

        pe_ms, ph2d, pd2h = pipelined_e2e(h_pre, [(tuple(pout.shape), pout.dtype), (tuple(pns.shape), pns.dtype)],
                                          pre_launch, n_e2e)
        pre_e2e = {"value": round(world * T / (pe_ms * 1e-3), 1), "unit": "tokens/s", "ms_per_step": round(pe_ms, 4),
                   "h2d_bytes_per_step": ph2d, "d2h_bytes_per_step": pd2h,
                   "pipeline": "copy-in / compute / copy-out streams, 3 device arenas, one pinned host arena: one H2D and one D2H copy per step"}

    # ---------------- report ----------------
    if rank != 0:
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    cpu = None
    os.sched_setaffinity(0, orig_affinity)  # the CPU baselines use every core this process may run on
    if not args.no_cpu_baseline:
        cpu = cpu_decode_baseline(budget_s=args.cpu_budget)
        cpu_pre = cpu_prefill_baseline(8192)
    dec_us = dec_ms * 1e3
    value = world * DECODE_STATE_BYTES / (dec_ms * 1e-3) / 1e9
    achieved = DECODE_ALG_BYTES / (dec_ms * 1e-3) / 1e9
    pre_bytes = T * PREFILL_ALG_BYTES_PER_TOKEN + 2 * STATE_BYTES_PER_ELEM
    pre_flops = T * PREFILL_FLOPS_PER_TOKEN
    pre_bound_s = max(pre_bytes / (hbm_peak * 1e9), pre_flops / (tc_peak * 1e12))
    line = {
        "metric": METRIC,
        "value": round(value, 3),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": args.warmup,
        "ms_per_step": round(dec_ms, 6),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic",
        "config": decode_config(world),
        "l2": f"{N_STATE_BUFS} rotating state buffers ({N_STATE_BUFS * 32} MiB > 126 MB L2)",
        "timing": f"median of {REPS} timed replays of a CUDA graph of exactly --steps launches "
                  f"(each preceded by a sleep kernel so the launches run back to back), CUDA events, "
                  f"max over ranks",
        "decode_us_per_step": round(dec_us, 3),
        "decode_us_per_rep": [round(x * 1e3, 3) for x in rep_ms],
        "decode_long_us_per_step": round(dec_long_ms * 1e3, 3),
        "decode_long_launches": n_long,
        "decode_eager_us_per_step": round(dec_eager_ms * 1e3, 3),
        "decode_sweep": decode_sweep,
        "decode_config4_b512": c4_dec,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4), "traffic": NCU_TRAFFIC["decode"],
                     "kernel": "gdn_decode_kernel", "peak_source": peak_src},
        "prefill_8k": {
            "tokens_per_s": round(world * T / (pre_ms * 1e-3), 1), "ms_per_step": round(pre_ms, 5),
            "config": "one 8192-token sequence per GPU, cu_seqlens int32, initial state N(0,0.02); L2 flushed (256 MiB write, then a 256 MiB read of another buffer) before each call",
            "roofline": {"bound": "max(hbm, tensor)", "achieved_frac": round(pre_bound_s / (pre_ms * 1e-3), 5),
                         "bound_us": round(pre_bound_s * 1e6, 3), "alg_bytes": pre_bytes, "alg_flops": pre_flops,
                         "traffic": NCU_TRAFFIC["prefill_8k_call"], "traffic_scope": "all kernels of one call",
                         "traffic_warm_caches": NCU_TRAFFIC["prefill_8k_call_warm"],
                         "kernel_us_warm": {"prep": 55.8, "seg_local": 44.2, "seg_chain": 8.3, "seg_out": 17.7},
                         "critical_path_us": PREFILL_8K_CRITICAL_PATH_US,
                         "peak_source": peak_src},
            "routes": pre_routes,
            "head_split": head_split,
            "e2e": pre_e2e,
        },
        "prefill_configs": prefill_more,
        "prefill_clone_mode": prefill_clone,
        "e2e": e2e,
        "host_link": link if world > 1 else ({**link, **host_binding} if link else None),
        "gpu_launches": steps * REPS,
        "clocks": clock_summary,
    }
    if cpu is not None:
        line["cpu_baseline"] = cpu
        line["prefill_8k"]["cpu_baseline"] = cpu_pre
    print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
