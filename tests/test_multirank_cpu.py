"""The multi-rank host logic of bench.py on CPU: two gloo ranks (world 2).

Each rank owns its own sequence-batch shard (seeded by rank, no exchange on
the data path); the job's time is the maximum over ranks, and its throughput
is every rank's tokens over that time."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench
from llama2_b200.workloads import WORKLOADS, host_inputs, with_batch


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # rank-dependent step times: the job's time is the slowest rank's
        got = bench.max_over_ranks([1.0 + rank, 10.0 - rank], world, "cpu")
        w = with_batch(WORKLOADS["tiny"], 2)
        inp = host_inputs(w, seed=0, rank=rank)
        digest = float(np.asarray(inp["qkv"], np.float64).sum())
        d = torch.tensor([digest], dtype=torch.float64)
        all_d = [torch.zeros(1, dtype=torch.float64) for _ in range(world)]
        dist.all_gather(all_d, d)
        out.put((rank, got, [x.item() for x in all_d]))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, got, digests in res:
        assert got == [2.0, 10.0]
        assert digests[0] != digests[1]  # each rank has its own shard


def test_shards_are_deterministic_per_rank():
    w = with_batch(WORKLOADS["tiny"], 2)
    a, b = host_inputs(w, seed=0, rank=1), host_inputs(w, seed=0, rank=1)
    for k in ("ids", "qkv", "kv_lens", "k_cache"):
        assert np.array_equal(a[k], b[k])


def test_job_throughput_counts_every_rank():
    # 4 ranks x 64 tokens x 10 steps over a slowest-rank time of 2 ms
    assert bench.job_tokens_per_s(64, 4, 10, 2.0) == 64 * 4 * 10 / 2e-3
    assert bench.max_over_ranks([3.0, 1.0], 1, "cpu") == [3.0, 1.0]


def test_reference_arm_json_line():
    """`bench.py --impl reference` (the reference's CPU path on host cores)
    prints one JSON line with the keys the bench contract names."""
    import json
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", "tiny", "--steps", "1",
                          "--warmup", "1"], cwd=root, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1
    res = json.loads(lines[0])
    for key in ("impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in res, key
    assert res["impl"] == "reference" and res["value"] > 0 and res["config"]["workload"] == "tiny"
    assert {"value", "unit", "cores", "kind", "sample"} <= set(res["cpu_baseline"])
    assert res["e2e"]["h2d_bytes_per_step"] == 0 and res["e2e"]["d2h_bytes_per_step"] == 0


def test_decode_algorithmic_bytes_by_operator():
    """The bytes behind every decode roofline figure, recounted operator by
    operator (each tensor read or written once) for the 7B batch-64 bf16 step
    at seeded lengths: the same total as workloads.algorithmic_bytes."""
    from llama2_b200.workloads import algorithmic_bytes

    w = WORKLOADS["7b-b64-bf16"]
    s, d, f, h, b = 2, w.dim, w.hidden, w.heads, w.batch
    kv = np.random.default_rng(3).integers(1, w.kv_cache_len, b) + 1
    embedding = b * d * s + b * d * s                  # gathered rows read, x written
    rmsnorm = b * d * s + b * d * s + d * s            # x read, normed written, weight read
    rope = b * 3 * d * s + b * d * s + 2 * b * d * s   # qkv read; q, K row, V row written
    scores = b * d * s + int(kv.sum()) * d * s + b * h * int(kv.max()) * s  # q, K rows 0..pos, score rows
    swiglu = b * 2 * f * s + b * f * s                 # gate/up read, output written
    assert algorithmic_bytes(w, kv) == embedding + rmsnorm + rope + scores + swiglu
    pv = int(kv.sum()) * d * s + b * d * s             # V rows 0..pos read, attention output written
    assert algorithmic_bytes(w, kv, attention_output=True) == embedding + rmsnorm + rope + scores + swiglu + pv
