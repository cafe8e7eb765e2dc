"""The multi-rank host logic of bench.py on CPU: two gloo ranks (world 2).

Weak scaling: each rank owns a batch of its own (seeded by rank, no exchange
on the data path) with the same multiset of sequence lengths. Strong scaling
(--shard): one global batch split by sequence over the ranks. The job's time
is the maximum over ranks, and its throughput is every rank's tokens over
that time."""
import os
import socket

import numpy as np
import pytest
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
        per_rank = bench.gather_over_ranks(float(rank + 1), world, "cpu")
        objs = bench.gather_objects({"rank": rank}, world)
        # strong scaling: this rank's rows of one global batch, as bench.rank_inputs picks them
        args = bench.argparse.Namespace(workload="tiny", batch=8, shard="balanced")
        w_rank, inp_rank, w_job = bench.rank_inputs(args, rank, world)
        rows = bench.shard_rows(host_inputs(w_job, seed=0, kv_cache=False)["kv_lens"], world, rank, "balanced")
        out.put((rank, got, [x.item() for x in all_d], per_rank, objs, rows.tolist(), w_rank.batch,
                 inp_rank["kv_lens"].tolist()))
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
    glob = host_inputs(with_batch(WORKLOADS["tiny"], 8), seed=0, kv_cache=False)["kv_lens"]
    all_rows = []
    for rank, got, digests, per_rank, objs, rows, batch, kv in res:
        assert got == [2.0, 10.0]
        assert digests[0] != digests[1]  # each rank has its own shard
        assert per_rank == [1.0, 2.0] and objs == [{"rank": 0}, {"rank": 1}]
        assert batch == 4 and kv == glob[rows].tolist()
        all_rows += rows
    assert sorted(all_rows) == list(range(8))  # every sequence of the global batch on exactly one rank


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
    args = bench.argparse.Namespace(workload="tiny", batch=0, shard="off", attention=False, l2_flush="always")
    assert res["config"] == bench.bench_config(WORKLOADS["tiny"], args, 1)
    assert {"value", "unit", "cores", "kind", "sample", "cpu_model"} <= set(res["cpu_baseline"])
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


def test_weak_scaling_ranks_hold_the_same_lengths():
    """Every rank's positions are rank 0's (equal work per rank) while its
    activations are its own (different sequences)."""
    w = with_batch(WORKLOADS["tiny"], 16)
    base = host_inputs(w, seed=0, rank=0, kv_cache=False)
    for rank in (1, 2, 7):
        other = host_inputs(w, seed=0, rank=rank, kv_cache=False)
        assert np.array_equal(other["kv_lens"], base["kv_lens"])
        assert not np.array_equal(other["qkv"], base["qkv"])


@pytest.mark.parametrize("order", ["contiguous", "balanced"])
@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_shard_rows_partition_the_global_batch(order, world):
    from llama2_b200.workloads import shard_rows
    w = WORKLOADS["13b-b256"]
    kv = np.random.default_rng(5).integers(w.pos_lo, w.pos_hi + 1, w.batch, dtype=np.uint32)
    parts = [shard_rows(kv, world, r, order) for r in range(world)]
    assert all(len(p) == 256 // world for p in parts)
    assert sorted(np.concatenate(parts).tolist()) == list(range(256))
    if order == "contiguous":
        assert all(np.array_equal(p, np.arange(r * len(p), (r + 1) * len(p))) for r, p in enumerate(parts))
    else:
        keys = [int(kv[p].astype(np.int64).sum()) for p in parts]
        assert max(keys) <= 1.01 * (sum(keys) / world)  # snake dealing keeps the ranks' keys within 1 %
    with pytest.raises(ValueError):
        shard_rows(kv[:255], 2, 0, order)


def test_both_arms_describe_the_same_config():
    """The reference arm's config is the dict the GPU arm prints for the same
    arguments (so the two lines compare)."""
    args = bench.argparse.Namespace(workload="7b-b64", batch=0, shard="off", attention=False, l2_flush="always")
    a = bench.bench_config(WORKLOADS["7b-b64"], args, 1)
    assert a["workload"] == "7b-b64" and a["global_batch"] == 64 and a["batch_per_gpu"] == 64
    args.shard = "contiguous"
    b = bench.bench_config(WORKLOADS["13b-b256"], args, 8)
    assert b["global_batch"] == 256 and b["batch_per_gpu"] == 32 and "split contiguous" in b["parallelism"]
