"""CPU oracle of the whole layer-kernel chain — TEST INFRASTRUCTURE ONLY.

Composes the restated reference helpers (oracle.port) in the chain order,
with the intended "positions 0..pos" mask for the scores. For 16-bit
workloads every tensor is rounded to the storage type wherever the device
data flow stores it (inputs, RMSNorm output, rotated q/k, scores, SwiGLU
output) and the arithmetic is fp32 — the "fp32 oracle on rounded inputs"
semantics the bf16/f16 parity tolerance is stated against.
"""
from __future__ import annotations

import numpy as np
import torch

from oracle import port

_TORCH = {"bf16": torch.bfloat16, "f16": torch.float16}


def rounder(dtype: str):
    if dtype == "f32":
        return lambda a: np.ascontiguousarray(a, np.float32)
    td = _TORCH[dtype]
    return lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(td).float().numpy()


def intended_mask(q_lens, kv_lens, max_q, max_kv, q_cache_len, kv_cache_len):
    m = np.zeros((len(q_lens), q_cache_len, kv_cache_len), np.uint8)
    port.build_intended_mask(q_lens, kv_lens, max_q, max_kv, m)
    return m


def decode_step(w, inp: dict, qk_init=None, attention_output: bool = False) -> dict:
    """One decode chain step on host copies. Returns every output tensor; with
    attention_output also "attn_out" (B, D): P.V of the fp32 probabilities
    (the fused decode attention keeps them in fp32), rounded once."""
    r = rounder(w.dtype)
    b, h, hd, s = w.batch, w.heads, w.head_dim, w.kv_cache_len
    table = r(inp["embed_table"])
    weight = r(inp["norm_weight"])
    qkv = r(inp["qkv"])
    gate_up = r(inp["gate_up"])
    k = r(inp["k_cache"]).copy()
    v = r(inp["v_cache"]).copy()
    kv, mq, mkv = port.update_q_kv_lens(inp["q_lens"], inp["kv_lens"])
    x = port.embedding(inp["ids"], table)
    _, normed = port.fused_add_residual_rmsnorm(x, np.zeros_like(x), weight, False)
    normed = r(normed)
    q = np.zeros((b, h, 1, hd), np.float32)
    port.rope_kvcache_decode(w.pairing, qkv, inp["is_done"], kv, q, k, v)
    q, k = r(q), r(k)
    qk = np.zeros((b, h, 1, s), np.float32) if qk_init is None else np.array(qk_init, np.float32)
    port.qk_scores(q, k, 1, mkv, qk)
    mask = intended_mask(inp["q_lens"], kv, 1, mkv, 1, s)
    port.masked_attention_score(qk, mask, inp["q_lens"], mkv, hd)
    out = {}
    if attention_output:
        attn = np.zeros((b, h, 1, hd), np.float32)
        port.attention_qkv(qk, v, 1, mkv, attn)
        out["attn_out"] = r(attn.reshape(b, h * hd))
    qk = r(qk)
    ffn = r(port.swiglu(gate_up))
    out.update({"x": x, "normed": normed, "q": q, "k": k, "v": v, "qk": qk, "ffn_out": ffn, "kv_lens": kv,
                "max_q": mq, "max_kv": mkv})
    return out


def prefill_step(w, inp: dict, attention_output: bool = False) -> dict:
    """One prefill chain pass on host copies; with attention_output also
    "attn_out" (tokens, D): P.V of the stored (rounded) probabilities over keys
    < max_kv for rows < max_q (the launch_linear call site), rounded, then
    transposed and unpadded."""
    r = rounder(w.dtype)
    b, h, hd, s, qc = w.batch, w.heads, w.head_dim, w.kv_cache_len, w.prefill_len
    table = r(inp["embed_table"])
    weight = r(inp["norm_weight"])
    qkv = r(inp["qkv"])
    gate_up = r(inp["gate_up"])
    k = r(inp["k_cache"]).copy()
    v = r(inp["v_cache"]).copy()
    kv, mq, mkv = port.update_q_kv_lens(inp["q_lens"], inp["kv_lens"])
    unpad, offs = port.build_padding_index_maps(inp["q_lens"], qc)
    x = port.embedding(inp["ids"], table)
    _, normed = port.fused_add_residual_rmsnorm(x, np.zeros_like(x), weight, False)
    normed = r(normed)
    q = np.zeros((b, h, qc, hd), np.float32)
    port.rope_kvcache_prefill(w.pairing, qkv, inp["q_lens"], kv, unpad, q, k, v)
    q, k = r(q), r(k)
    qk = np.zeros((b, h, qc, s), np.float32)
    port.qk_scores(q, k, mq, mkv, qk)
    mask = intended_mask(inp["q_lens"], kv, mq, mkv, qc, s)
    port.masked_attention_score(qk, mask, inp["q_lens"], mkv, hd)
    qk = r(qk)
    out = {}
    if attention_output:
        attn = np.zeros((b, h, qc, hd), np.float32)
        port.attention_qkv(qk, v, mq, mkv, attn)
        out["attn_out"] = port.transpose_unpad(r(attn), unpad, int(np.asarray(inp["q_lens"], np.int64).sum()))
    ffn = r(port.swiglu(gate_up))
    out.update({"x": x, "normed": normed, "q": q, "k": k, "v": v, "qk": qk, "ffn_out": ffn, "kv_lens": kv,
                "max_q": mq, "max_kv": mkv, "unpad_to_pad": unpad, "seq_offsets": offs})
    return out


def score_row(q_row, k_rows, keep_upto, head_dim):
    """One softmax score row: q_row (hd,), k_rows (n, hd); keys 0..keep_upto kept.
    Same helpers (and accumulation order) as the full oracle."""
    n = k_rows.shape[0]
    qk = np.zeros((1, 1, 1, n), np.float32)
    port.qk_scores(np.ascontiguousarray(q_row, np.float32).reshape(1, 1, 1, -1),
                   np.ascontiguousarray(k_rows, np.float32).reshape(1, 1, n, -1), 1, n, qk)
    mask = np.zeros((1, 1, n), np.uint8)
    mask[0, 0, :keep_upto + 1] = 1
    port.masked_attention_score(qk, mask, np.ones(1, np.uint32), n, head_dim)
    return qk.reshape(-1)
