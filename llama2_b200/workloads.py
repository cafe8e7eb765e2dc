"""Workload definitions (Llama-2 layer-kernel shapes) and seeded synthetic inputs.

The five workloads are the reference path's benchmark configurations:

  tiny      dim 288, 6 heads of 48, hidden 768, cache 256, batch 1, fp32 decode
  7b-b1     Llama-2-7B dims (4096, 32 x 128, hidden 11008), cache 4096, batch 1, fp32 decode
  7b-b64    7B dims, batch 64 decode (fp32, or bf16 I/O)
  7b-prefill 7B dims, 8 x 2048-token prefill, bf16 I/O, causal scores [8,32,2048,2048]
  13b-b256  Llama-2-13B dims (5120, 40 x 128, hidden 13824), batch 256 decode, fp16

Inputs follow the stated distributions: token ids U[0, 32000), embedding
table N(0, 0.02), RMSNorm weight U(0.5, 1.5), q/k/v and gate/up activations
N(0, 1) (standing in for the projection outputs), KV cache N(0, 1), and one
position per sequence uniform in [1, 4095] ([0, 255] for tiny). Generated on
the host with numpy's seeded Generator (so CPU oracles see identical bits)
and copied once to the device.
"""
from __future__ import annotations

import dataclasses

import numpy as np


@dataclasses.dataclass(frozen=True)
class Workload:
    name: str
    dim: int
    heads: int
    head_dim: int
    hidden: int
    vocab: int
    kv_cache_len: int
    batch: int
    dtype: str          # "f32" | "bf16" | "f16"
    pairing: int        # 0 interleaved, 1 half (the reference's "_llama2")
    prefill_len: int = 0  # tokens per sequence for prefill workloads (0 = decode)
    pos_lo: int = 1
    pos_hi: int = 4095

    @property
    def decode(self) -> bool:
        return self.prefill_len == 0

    @property
    def tokens(self) -> int:
        return self.batch * (self.prefill_len or 1)


WORKLOADS = {
    "tiny": Workload("tiny", 288, 6, 48, 768, 32000, 256, 1, "f32", 0, pos_lo=0, pos_hi=255),
    "7b-b1": Workload("7b-b1", 4096, 32, 128, 11008, 32000, 4096, 1, "f32", 1),
    "7b-b64": Workload("7b-b64", 4096, 32, 128, 11008, 32000, 4096, 64, "f32", 1),
    "7b-b64-bf16": Workload("7b-b64-bf16", 4096, 32, 128, 11008, 32000, 4096, 64, "bf16", 1),
    "7b-prefill": Workload("7b-prefill", 4096, 32, 128, 11008, 32000, 2048, 8, "bf16", 1, prefill_len=2048),
    "13b-b256": Workload("13b-b256", 5120, 40, 128, 13824, 32000, 4096, 256, "f16", 1),
}


def with_batch(w: Workload, batch: int) -> Workload:
    return dataclasses.replace(w, batch=batch)


def np_dtype(dt: str):
    return np.float32


def host_inputs(w: Workload, seed: int = 0, rank: int = 0, kv_cache: bool = True) -> dict:
    """Seeded float32 / uint32 host arrays for one step of workload `w`.

    Decode: positions p ~ U[pos_lo, pos_hi]; kv_lens holds p (the length
    before this step's token), and the length update makes it p + 1.
    Prefill: a fresh prefill (kv_lens = 0 before the update, q_lens = prefill_len).

    Every rank draws its own activations, ids and cache from the seed
    sequence [seed, rank]. The positions of rank r > 0 are rank 0's draw
    (`rank_positions`), so the ranks of a weak-scaling job hold different
    sequences with the same lengths in the same order: equal work per rank.
    """
    rng = np.random.default_rng([seed, rank])
    d, h, hd, f, s = w.dim, w.heads, w.head_dim, w.hidden, w.kv_cache_len
    t = w.tokens
    out = {
        "embed_table": (rng.standard_normal((w.vocab, d), dtype=np.float32) * np.float32(0.02)),
        "norm_weight": rng.uniform(0.5, 1.5, d).astype(np.float32),
        "ids": rng.integers(0, w.vocab, t, dtype=np.uint32),
        "qkv": rng.standard_normal((t, 3 * d), dtype=np.float32),
        "gate_up": rng.standard_normal((t, 2 * f), dtype=np.float32),
        "is_done": np.zeros(w.batch, np.uint8),
    }
    if w.decode:
        out["q_lens"] = np.ones(w.batch, np.uint32)
        out["kv_lens"] = rng.integers(w.pos_lo, w.pos_hi + 1, w.batch, dtype=np.uint32)
        if rank:
            out["kv_lens"] = rank_positions(w, seed, rank)
    else:
        out["q_lens"] = np.full(w.batch, w.prefill_len, np.uint32)
        out["kv_lens"] = np.zeros(w.batch, np.uint32)
    if kv_cache:
        out["k_cache"] = rng.standard_normal((w.batch, h, s, hd), dtype=np.float32)
        out["v_cache"] = rng.standard_normal((w.batch, h, s, hd), dtype=np.float32)
    else:
        out["cache_seed"] = seed * 1000003 + rank
    return out


def rank_positions(w: Workload, seed: int, rank: int) -> np.ndarray:
    """Rank 0's seeded positions (the same draw host_inputs makes for rank 0,
    replayed from its seed sequence). Every rank of a weak-scaling job thus
    holds sequences of the same lengths in the same order (the fused step
    schedules its rows in sequence order, so a reordering alone moves a
    rank's time by a few per cent)."""
    rng = np.random.default_rng([seed, 0])
    d, f, t = w.dim, w.hidden, w.tokens
    # replay rank 0's draws up to its positions (same order and sizes as host_inputs)
    rng.standard_normal((w.vocab, d), dtype=np.float32)
    rng.uniform(0.5, 1.5, d)
    rng.integers(0, w.vocab, t, dtype=np.uint32)
    rng.standard_normal((t, 3 * d), dtype=np.float32)
    rng.standard_normal((t, 2 * f), dtype=np.float32)
    return rng.integers(w.pos_lo, w.pos_hi + 1, w.batch, dtype=np.uint32)


def shard_rows(positions, world: int, rank: int, order: str = "contiguous") -> np.ndarray:
    """Sequence indices of one global batch that rank `rank` of `world` owns.

    contiguous: the slice [rank*B/world, (rank+1)*B/world) — the rank's part
    of the (batch, kv_head, kv_cache_len, head_dim) cache cut along batch.
    balanced: sequences sorted by length (longest first) and dealt to the
    ranks in snake order (0..N-1, N-1..0, ...): every rank gets B/world
    sequences and nearly the same number of keys, so the slowest rank (which
    sets the job's time) is not held up by a run of long sequences."""
    b = len(positions)
    if b % world:
        raise ValueError(f"global batch {b} does not split evenly over {world} ranks")
    if order == "contiguous":
        per = b // world
        return np.arange(rank * per, (rank + 1) * per)
    if order != "balanced":
        raise ValueError(f"unknown shard order {order!r}")
    idx = np.argsort(-np.asarray(positions, np.int64), kind="stable")
    lanes = np.concatenate([np.arange(world), np.arange(world)[::-1]])
    owner = lanes[np.arange(b) % (2 * world)]
    return np.sort(idx[owner == rank])


def shard_inputs(w: Workload, inputs: dict, rows) -> dict:
    """The per-step inputs of the sequences `rows` of a global batch (decode)."""
    rows = np.asarray(rows, np.int64)
    out = {k: v for k, v in inputs.items() if k in ("embed_table", "norm_weight")}
    for k in ("ids", "qkv", "gate_up", "is_done", "q_lens", "kv_lens"):
        out[k] = np.ascontiguousarray(inputs[k][rows])
    for k in ("k_cache", "v_cache"):
        if k in inputs:
            out[k] = np.ascontiguousarray(inputs[k][rows])
    if "cache_seed" in inputs:
        out["cache_seed"] = inputs["cache_seed"]
    return out


def host_cache_ok(w: Workload, limit_elems: int = 1 << 28) -> bool:
    """Whether the KV cache is small enough to draw on the host (<= 1 GiB fp32 each)."""
    return w.batch * w.heads * w.kv_cache_len * w.head_dim <= limit_elems


def algorithmic_bytes(w: Workload, kv_lens_after: np.ndarray, attention_output: bool = False) -> int:
    """Mandatory HBM bytes of one chain step (reads + writes, no intermediates):
    embedding 2*D*s per token, RMSNorm 2*D*s per token + D*s weight,
    RoPE/KV 6*D*s per token (read q, k, v; write q, k row, v row), scores
    D*s (q) + K rows 0..pos (D*s per key) + H*s per score written (all keys
    < max_kv of each row are written), SwiGLU 3*F*s per token.
    attention_output adds, for decode, the V rows 0..pos (D*s per key) and
    the output (D*s per sequence); for prefill, the P.V call site (read the
    score matrix and V rows < max_kv, write max_q padded rows of D*s) and the
    unpad (read and write D*s per token)."""
    s = 2 if w.dtype in ("bf16", "f16") else 4
    d, f, h = w.dim, w.hidden, w.heads
    t = w.tokens
    kv = np.asarray(kv_lens_after, np.int64)
    max_kv = int(kv.max()) if kv.size else 0
    per_tok = 2 * d * s + 2 * d * s + 6 * d * s + 3 * f * s
    total = t * per_tok + d * s
    if w.decode:
        total += w.batch * d * s                  # q read by the scores
        total += int(kv.sum()) * d * s            # K rows 0..pos of every head
        total += w.batch * h * max_kv * s         # score rows written
        if attention_output:
            total += int(kv.sum()) * d * s        # V rows 0..pos
            total += w.batch * d * s              # attention output
    else:
        q = w.prefill_len
        total += t * d * s                        # q read
        total += w.batch * max_kv * d * s         # K read
        total += w.batch * h * q * max_kv * s     # score matrix written (zeros included)
        if attention_output:
            total += w.batch * h * q * max_kv * s  # score matrix read by P.V
            total += w.batch * max_kv * d * s      # V read
            total += w.batch * q * d * s           # padded P.V rows written
            total += 2 * t * d * s                 # unpad: read and write
    return int(total)
