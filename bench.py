"""Benchmark of the fused Llama-2 layer-kernel chain on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

A step is one pass of the chain (update lens -> embedding -> RMSNorm -> RoPE +
KV append -> fused scores -> SwiGLU) over one batch of synthetic input
(llama2_b200.workloads). The default workload is 7b-b64: Llama-2-7B dims,
batch 64 decode, fp32 (the reference's precision), KV cache [64, 32, 4096,
128] — the largest single-GPU 7B-dims decode configuration, whose 2.2 GB
step is where the HBM roofline fraction means something (a batch-1 step
moves 9 MB, 1.4 us at the copy peak, under the launch latency).

Under torchrun each rank runs on its own GPU with no collective on the data
path; time is the max over ranks of the summed per-step device time (CUDA
events), and value = tokens of all ranks / that time. Two ways to split:

  default        weak scaling: every rank holds its own batch of the
                 workload's size (its own activations and cache, the same
                 sequence lengths as rank 0, so the ranks' work is equal);
  --shard ORDER  strong scaling: one global seeded batch of the workload's
                 size is split by sequence over the ranks (ORDER contiguous:
                 rank r takes sequences [r*B/N, (r+1)*B/N); balanced: sorted
                 by length and dealt in snake order, equal counts and nearly
                 equal keys per rank). Per-rank step times are reported.

Between timed steps the sequence lengths are restored and the L2 cache is
flushed: a 2 x L2-sized buffer is written, then another one read, so that
L2 holds none of the step's data and the written lines have gone back to
HBM before the next step starts — all outside the timed windows.
`--l2-flush write` flushes by the write alone (its dirty lines are then
written back while the next step runs, which costs short HBM-bound steps
up to 5 %), `--l2-flush auto` skips the flush when a step moves more than
4 x L2; `config.l2` says which was done.

--impl reference times the reference's own CPU implementation of the path
(its CPU test helpers compiled from its sources, oracle/_ref; the C
restatement oracle/liboracle.so where those are absent) on this box's host
cores, rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from llama2_b200.workloads import (WORKLOADS, algorithmic_bytes, host_cache_ok, host_inputs,  # noqa: E402
                                   shard_inputs, shard_rows, with_batch)

FALLBACK_HBM_GBS = 6650.0


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--workload", default="7b-b64", choices=sorted(WORKLOADS))
    ap.add_argument("--shard", default="off", choices=["off", "contiguous", "balanced"],
                    help="split ONE global batch of the workload over the ranks (strong scaling) instead of "
                         "giving every rank a batch of its own (weak scaling)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--cpu-sample-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch", type=int, default=0,
                    help="override the workload's per-GPU batch (small cases for profiling)")
    ap.add_argument("--attention", action="store_true",
                    help="the chain also produces the attention output: P.V (fused into the decode scores; at the "
                         "launch_linear call site for prefill) and the transpose + unpad")
    ap.add_argument("--l2-flush", default="always", choices=["always", "write", "auto"],
                    help="always: before every step, a 2 x L2 write then a 2 x L2 read (the written lines "
                         "go back to HBM before the step); write: the write alone (its dirty lines are "
                         "written back while the next step runs); auto: as always, but no flush when a "
                         "step moves more than 4 x L2")
    ap.add_argument("--unfused", action="store_true",
                    help="run a decode step as the operator sequence instead of the one-launch fused step")
    return ap.parse_args()


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


# ---------------------------------------------------------------------------
# Clock sampling (NVML) during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
        0x10: "sync_boost", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
        0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting",
    }

    def __init__(self, device_index, period=0.002):
        self.samples = []
        self.reasons = set()
        self.max_mhz = None
        self.period = period
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.nvml = None

    def _run(self):
        n = self.nvml
        while not self._stop.is_set():
            self._sample()
            time.sleep(self.period)

    def _sample(self):
        n = self.nvml
        try:
            self.samples.append(n.nvmlDeviceGetClockInfo(self.h, n.NVML_CLOCK_SM))
            r = n.nvmlDeviceGetCurrentClocksEventReasons(self.h)
            for bit, name in self.REASONS.items():
                if r & bit and name != "gpu_idle":
                    self.reasons.add(name)
        except Exception:
            pass

    def start(self):
        if self.nvml:
            self._sample()
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread:
            self._stop.set()
            self._thread.join()
            self._sample()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        return {"sm_mhz": float(statistics.median(self.samples)), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU baselines (oracle / reference helpers) — only the CPU legs touch oracle/
# ---------------------------------------------------------------------------
def cpu_chain_rate(w, inputs, seconds, impl, attention_output=False):
    """tokens/s of the CPU chain on a bounded sample: chain steps over the
    first sequences of the batch (CpuChain.sample_batch) until `seconds`."""
    from oracle import cpu_chain
    runner = cpu_chain.CpuChain(w, inputs, impl=impl, attention_output=attention_output)
    steps, tokens, t0 = 0, 0, time.perf_counter()
    while True:
        tokens += runner.step()
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    nseq = len(runner.sample_batch())
    return {"value": tokens / el, "unit": "tokens/s", "cores": runner.threads, "kind": runner.kind,
            "cpu_model": host_cpu()["model"],
            "sample": f"{steps} chain step(s) over {nseq} of the {w.batch} sequence(s) of {w.name} "
                      f"({tokens} tokens) in {el:.1f} s on {runner.threads} thread(s)"}


# ---------------------------------------------------------------------------
# Our arm
# ---------------------------------------------------------------------------
def bench_config(w_job, args, n_gpus):
    """The workload as both arms describe it (the same dict in the line of
    `--impl ours` and of `--impl reference`)."""
    shard = args.shard != "off"
    per_gpu = w_job.batch // n_gpus if shard else w_job.batch
    flush = {"always": "flushed between timed GPU steps (2 x L2 written, then 2 x L2 read to evict it)",
             "write": "flushed between timed GPU steps (2 x L2 written)",
             "auto": "flushed between timed GPU steps unless a step moves more than 4 x L2 "
                     "(then its inputs alone exceed L2)"}[args.l2_flush]
    return {"workload": w_job.name, "dim": w_job.dim, "heads": w_job.heads, "head_dim": w_job.head_dim,
            "hidden": w_job.hidden, "kv_cache_len": w_job.kv_cache_len, "dtype": w_job.dtype,
            "global_batch": per_gpu * n_gpus, "batch_per_gpu": per_gpu, "prefill_len": w_job.prefill_len,
            "attention_output": bool(args.attention),
            "parallelism": (f"sequence-batch shards x{n_gpus}: one global batch split {args.shard} by sequence"
                            if shard else f"sequence-batch shards x{n_gpus}: a batch of its own per GPU, the "
                                          f"same lengths on every rank"),
            "positions": f"uniform in [{w_job.pos_lo}, {w_job.pos_hi}], seed 0" if w_job.decode
                         else "fresh prefill",
            "l2": flush}


def rank_inputs(args, rank, world):
    """(per-rank workload, per-rank host inputs, the job's workload)."""
    w_job = WORKLOADS[args.workload]
    if args.batch:
        w_job = with_batch(w_job, args.batch)
    if args.shard == "off":
        return w_job, host_inputs(w_job, seed=0, rank=rank, kv_cache=host_cache_ok(w_job)), w_job
    if not w_job.decode:
        raise SystemExit("--shard splits the sequence batch of a decode workload")
    glob = host_inputs(w_job, seed=0, kv_cache=host_cache_ok(w_job))
    rows = shard_rows(glob["kv_lens"], world, rank, args.shard)
    inputs = shard_inputs(w_job, glob, rows)
    if "cache_seed" in inputs:
        inputs["cache_seed"] = rank  # the rank's cache slice, drawn on its device
    return with_batch(w_job, len(rows)), inputs, w_job


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    from llama2_b200.chain import Chain

    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    w, inputs, w_job = rank_inputs(args, rank, world)
    chain = Chain(w, inputs, device=dev, fused=not args.unfused, attention_output=args.attention)

    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    kv_after = inputs["kv_lens"].astype(np.int64) + inputs["q_lens"].astype(np.int64)
    chain_bytes = algorithmic_bytes(w, kv_after, args.attention)
    flush_each = args.l2_flush != "auto" or chain_bytes < 4 * l2
    flush_buf = torch.empty(max(2 * l2, 256 << 20) // 4, dtype=torch.float32, device=dev)
    drain_buf = torch.ones(max(2 * l2, 256 << 20) // 4, dtype=torch.float32, device=dev) \
        if args.l2_flush != "write" else None

    def flush():
        """Evict L2: write a 2 x L2 buffer, then (unless --l2-flush write) read
        another one, so that the written lines are evicted (written back to
        HBM) here, outside the timed window, instead of during the next step."""
        if flush_each:
            flush_buf.zero_()
            if drain_buf is not None:
                drain_buf.sum()

    def barrier():
        if world > 1:
            dist.barrier()

    # The step as the timed loop runs it (`chain.replay`: the one-kernel fused
    # step launched directly, the operator sequence as a CUDA graph), and a
    # graph copy whose dominant kernel (the fused step, or the fused scores)
    # is bracketed by external event-record nodes, replayed in a separate
    # loop so that the event nodes do not add to the step time.
    kev = (torch.cuda.Event(enable_timing=True, external=True), torch.cuda.Event(enable_timing=True, external=True))
    kernel_graph = capture_with_kernel_events(chain, kev)
    chain.capture()

    stream = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]

    def one_step(run, i=None):
        chain.reset_lengths()
        flush()
        if i is not None:
            ev[i][0].record(stream)
        run()
        if i is not None:
            ev[i][1].record(stream)

    for _ in range(max(args.warmup, 3)):
        one_step(chain.replay)
        one_step(kernel_graph.replay)
    torch.cuda.synchronize()

    clocks = ClockSampler(local_rank)
    kernel_ms = []
    barrier()
    torch.cuda.synchronize()
    clocks.start()
    for i in range(args.steps):
        one_step(chain.replay, i)
    torch.cuda.synchronize()
    for i in range(args.steps):
        one_step(kernel_graph.replay)
        kev[1].synchronize()
        kernel_ms.append(kev[0].elapsed_time(kev[1]))
    torch.cuda.synchronize()
    clocks.stop()
    barrier()
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = sum(step_ms)

    # End to end through the public API: H2D of the step's inputs from pinned
    # memory, the chain, D2H of its results, every step. Timed twice: by the
    # host clock from the call to the results being on the host (the stream
    # synchronized after each step, as a caller that reads the results does),
    # and by CUDA events around the same work on the stream.
    chain.host_buffers(inputs)
    h2d, d2h = chain.e2e_bytes()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for _ in range(max(args.warmup, 3)):
        flush()
        chain.step_e2e()
    torch.cuda.synchronize()
    barrier()
    wall_s = 0.0
    for i in range(args.steps):
        flush()
        stream.synchronize()
        t0 = time.perf_counter()
        ev2[i][0].record(stream)
        chain.step_e2e()
        ev2[i][1].record(stream)
        stream.synchronize()
        wall_s += time.perf_counter() - t0
    torch.cuda.synchronize()
    barrier()
    e2e_ms = sum(a.elapsed_time(b) for a, b in ev2)

    # The timed kernel: the fused step (the whole chain), the fused decode
    # attention, or the fused scores.
    if chain.fused:
        kernel_name, kernel_key, kernel_bytes = "fused decode step", "decode_step", chain_bytes
        if args.attention:
            kernel_name, kernel_key = "fused decode step with P.V", "decode_step_attention"
    elif w.decode and args.attention:
        kernel_name, kernel_key = "fused decode attention", "attention_rows_stream"
        kernel_bytes = scores_bytes(w, kv_after, attention_output=True)
    else:
        kernel_name = "fused decode scores" if w.decode else "fused prefill scores"
        kernel_key = "score_rows_stream" if w.decode else "prefill_scores_tc"
        kernel_bytes = scores_bytes(w, kv_after)

    per_rank_ms = gather_over_ranks(total_ms / args.steps, world, dev)
    per_rank_clocks = gather_objects(clocks.summary(), world)
    total_ms, e2e_ms, wall_ms = max_over_ranks([total_ms, e2e_ms, wall_s * 1e3], world, dev)

    result = None
    if rank == 0:
        peak, peak_kind = peaks()
        kmean = float(np.mean(kernel_ms)) if kernel_ms else None
        achieved = kernel_bytes / (kmean * 1e-3) / 1e9 if kmean else None
        result = {
            "metric": "layer-kernel tokens/s at Llama-2-7B dims",
            "value": job_tokens_per_s(w.tokens, world, args.steps, total_ms),
            "unit": "tokens/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": total_ms / args.steps,
            "higher_is_better": True,
            "scaling": "strong" if args.shard != "off" else "weak",
            "vs_baseline": None,
            "dtype": {"f32": "fp32", "bf16": "bf16", "f16": "fp16"}[w.dtype],
            "data": "synthetic (seeded; N(0,1) activations and KV cache, N(0,0.02) embeddings)",
            "config": bench_config(w_job, args, world),
            "launch": ("one kernel per step, launched directly" if chain.fused
                       else f"{chain.kernels_per_step()} kernels per step, one CUDA graph replay"),
            "l2_flushed": bool(flush_each),
            "chain_hbm": {"algorithmic_bytes_per_step": chain_bytes,
                          "achieved_gbs": chain_bytes / (total_ms / args.steps * 1e-3) / 1e9,
                          "frac_of_peak": chain_bytes / (total_ms / args.steps * 1e-3) / 1e9 / peak},
            "roofline": {"kernel": kernel_name,
                         "bound": "hbm", "achieved": achieved, "peak": peak, "peak_kind": peak_kind,
                         "unit": "GB/s", "frac": achieved / peak if achieved else None,
                         "algorithmic_bytes_per_launch": kernel_bytes, "mean_launch_ms": kmean,
                         "traffic": profiled_traffic(kernel_key, w.name if args.shard == "off" else None)},
            "e2e": {"value": job_tokens_per_s(w.tokens, world, args.steps, wall_ms), "unit": "tokens/s",
                    "timing": "host clock from the call to the results on the host, per step",
                    "event_value": job_tokens_per_s(w.tokens, world, args.steps, e2e_ms),
                    "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": chain.kernels_per_step() * args.steps,
            "clocks": clocks.summary(),
        }
        if world > 1:
            result["per_rank"] = {"ms_per_step": per_rank_ms,
                                  "sequences": [w.batch] * world,
                                  "sm_mhz": [c["sm_mhz"] for c in per_rank_clocks],
                                  "reasons": sorted({r for c in per_rank_clocks for r in c["reasons"]})}
        if not args.no_cpu_baseline and world == 1:
            result["cpu_baseline"] = cpu_chain_rate(w, inputs, args.cpu_sample_seconds, impl="port",
                                                    attention_output=args.attention)
    return result


def gather_over_ranks(value, world, device):
    """Every rank's float, in rank order (every rank calls it)."""
    if world == 1:
        return [value]
    import torch
    import torch.distributed as dist
    t = torch.tensor([value], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def gather_objects(obj, world):
    """Every rank's picklable object, in rank order (every rank calls it)."""
    if world == 1:
        return [obj]
    import torch.distributed as dist
    out = [None] * world
    dist.all_gather_object(out, obj)
    return out


def max_over_ranks(values, world, device):
    """Element-wise maximum over all ranks of a list of floats (every rank
    calls it, in the same order): the job's time is its slowest rank's."""
    if world == 1:
        return list(values)
    import torch
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def job_tokens_per_s(tokens_per_rank_step, world, steps, max_ms):
    """Whole-job throughput: every rank's tokens over the slowest rank's time."""
    return tokens_per_rank_step * world * steps / (max_ms * 1e-3)


def capture_with_kernel_events(chain, kev):
    """Capture chain.step() as a graph with event-record nodes around the
    dominant kernel (the fused decode step, or the fused scores)."""
    from llama2_b200 import ops

    names = ("decode_step", "decode_step_attention", "decode_attention_scores", "decode_attention",
             "prefill_attention_scores")
    orig = {n: getattr(ops, n) for n in names}

    def wrap(fn):
        def inner(*a, **k):
            kev[0].record()
            fn(*a, **k)
            kev[1].record()
        return inner

    for n in names:
        setattr(ops, n, wrap(orig[n]))
    try:
        return chain.capture()
    finally:
        for n in names:
            setattr(ops, n, orig[n])


def scores_bytes(w, kv_after, attention_output=False):
    """Algorithmic bytes of one fused-scores launch: q, K rows 0..pos, score rows
    (and for the fused decode attention also V rows 0..pos and the output)."""
    s = 2 if w.dtype in ("bf16", "f16") else 4
    kv = np.asarray(kv_after, np.int64)
    max_kv = int(kv.max())
    if w.decode:
        pv = (kv.sum() * w.dim * s + w.batch * w.dim * s) if attention_output else 0
        return int(w.batch * w.dim * s + kv.sum() * w.dim * s + w.batch * w.heads * max_kv * s + pv)
    q = w.prefill_len
    return int(w.tokens * w.dim * s + kv.sum() * w.dim * s + w.batch * w.heads * q * max_kv * s)


def profiled_traffic(kernel_key, workload):
    """DRAM bytes (read + write) per launch of the timed kernel on this
    workload, from the committed ncu summaries; None if not profiled."""
    path = os.path.join(ROOT, "profiles", "traffic.json")
    try:
        with open(path) as f:
            return json.load(f).get(f"{kernel_key}:{workload}")
    except Exception:
        return None


# ---------------------------------------------------------------------------
# Reference arm: the reference's CPU implementation on the host cores
# ---------------------------------------------------------------------------
def host_cpu():
    """The host's CPU model (from /proc/cpuinfo) and the logical CPUs this
    process may run on."""
    model = None
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    model = line.split(":", 1)[1].strip()
                    break
    except OSError:
        pass
    try:
        usable = len(os.sched_getaffinity(0))
    except AttributeError:
        usable = os.cpu_count()
    return {"model": model or "unknown", "logical_cpus": os.cpu_count(), "usable_cpus": usable}


def run_reference(args):
    from oracle import cpu_chain

    w_job = WORKLOADS[args.workload]
    if args.batch:
        w_job = with_batch(w_job, args.batch)
    inputs = host_inputs(w_job, seed=0, kv_cache=host_cache_ok(w_job))
    impl = "ref" if cpu_chain.ref_available() else "port"
    cpu = host_cpu()
    threads = cpu["usable_cpus"]
    # A decode step samples up to 16 sequences: 16 x heads (sequence, head)
    # score rows keep every host thread busy in the dominant part.
    runner = cpu_chain.CpuChain(w_job, inputs, impl=impl, threads=threads, attention_output=args.attention,
                                max_sequences=16)
    sample = runner.sample_batch()
    # Prefill: the scores of every 16th query row are computed and their time is
    # scaled by 16 (a full 2048-row step of the CPU helpers takes many seconds).
    stride = 1 if w_job.decode else 16
    for _ in range(max(args.warmup, 1)):
        runner.step(sample, row_stride=stride)
    el = 0.0
    for _ in range(args.steps):
        runner.step(sample, row_stride=stride)
        el += runner.last_times["other"] + runner.last_times["scores"] * stride
    tokens = len(sample) * (w_job.prefill_len or 1) * args.steps
    value = tokens / el
    rows = len(sample) * w_job.heads
    return {
        "impl": "reference",
        "metric": "layer-kernel tokens/s at Llama-2-7B dims",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if args.shard != "off" else "weak", "vs_baseline": None,
        "dtype": {"f32": "fp32", "bf16": "bf16", "f16": "fp16"}[w_job.dtype],
        "data": "synthetic (seeded; N(0,1) activations and KV cache, N(0,0.02) embeddings)",
        "config": bench_config(w_job, args, args.gpus),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": runner.kind,
                         "cpu_model": cpu["model"], "logical_cpus": cpu["logical_cpus"],
                         "sample": f"{len(sample)} of {w_job.batch} sequence(s) per step, {args.steps} steps; "
                                   f"{rows} (sequence, head) RoPE and score rows per step spread over "
                                   f"{threads} thread(s), embedding/RMSNorm/SwiGLU over "
                                   f"{min(threads, len(sample) * (w_job.prefill_len or 1))} row block(s)" +
                                   (f"; scores of every {stride}th query row, their time x{stride}" if stride > 1
                                    else "") +
                                   ("" if impl == "ref" else "; the reference helpers are not built here: the C "
                                                             "restatement ran")},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            print(json.dumps(run_reference(args)))
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
    try:
        res = run_ours(args, rank, world, local_rank)
        if rank == 0:
            print(json.dumps(res))
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
