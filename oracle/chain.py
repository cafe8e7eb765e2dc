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


def decode_layer(wts: dict, x, pending, kv_lens, max_kv, is_done, k, v, pairing: int, dtype: str) -> dict:
    """One decoder-layer decode step (llama2_b200.layer.DecoderLayer.decode)
    composed from the restated helpers: add-residual RMSNorm
    (test_fused_add_residual_rmsnorm.cu:21-52), compute_expected_linear
    (test_linear.cu:78-108) for the projections, the decode RoPE + append,
    QK^T + the intended mask + softmax, P.V of the fp32 probabilities, SwiGLU.
    Every tensor the device stores in 16 bits is rounded there. k, v are
    updated in place (float32). kv_lens are the updated lengths."""
    r = rounder(dtype)
    w = {n: r(np.asarray(a, np.float32)) for n, a in wts.items()}
    x = r(x)
    b, d = x.shape
    hd = k.shape[3]
    hq = d // hd
    s = k.shape[2]
    f = w["w_down"].shape[0]
    if pending is None:
        x1, h = port.fused_add_residual_rmsnorm(x, np.zeros_like(x), w["w_attn_norm"], False)
    else:
        x1, h = port.fused_add_residual_rmsnorm(x, r(pending), w["w_attn_norm"], True)
    x1, h = r(x1), r(h)
    n_qkv = w["w_qkv"].shape[1]
    qkv = r(port.linear(h, w["w_qkv"], False, False, b, n_qkv, d))
    q = np.zeros((b, hq, 1, hd), np.float32)
    port.rope_kvcache_decode(pairing, qkv, is_done, kv_lens, q, k, v)
    q = r(q)
    k[...] = r(k)
    v[...] = r(v)
    qk = np.zeros((b, hq, 1, s), np.float32)
    port.qk_scores(q, k, 1, max_kv, qk)
    ones = np.ones(b, np.uint32)
    mask = intended_mask(ones, kv_lens, 1, max_kv, 1, s)
    port.masked_attention_score(qk, mask, ones, max_kv, hd)
    attn = np.zeros((b, hq, 1, hd), np.float32)
    port.attention_qkv(qk, v, 1, max_kv, attn)
    attn = r(attn.reshape(b, d))
    o = r(port.linear(attn, w["w_o"], False, False, b, d, d))
    x2, h2 = port.fused_add_residual_rmsnorm(x1, o, w["w_ffn_norm"], True)
    x2, h2 = r(x2), r(h2)
    gu = r(port.linear(h2, w["w_gate_up"], False, False, b, 2 * f, d))
    act = r(port.swiglu(gu))
    down = r(port.linear(act, w["w_down"], False, False, b, d, f))
    return {"x": x2, "down": down, "qk": r(qk), "attn": attn, "h": h, "qkv": qkv}


def prefill_layer(wts: dict, x, pending, q_lens, kv_lens, max_q, max_kv, unpad, k, v, q_cache_len: int,
                  pairing: int, dtype: str) -> dict:
    """One decoder-layer prefill pass (llama2_b200.layer.DecoderLayer.prefill)
    composed from the restated helpers: add-residual RMSNorm, the QKV
    projection, the padded RoPE + append, QK^T + the intended causal mask +
    softmax, P.V of the stored (rounded) probabilities over keys < max_kv for
    rows < max_q (the launch_linear call site), transpose + unpad, the O
    projection, the second norm, gate/up, SwiGLU, down. k, v are updated in
    place (float32); kv_lens are the updated lengths."""
    r = rounder(dtype)
    w = {n: r(np.asarray(a, np.float32)) for n, a in wts.items()}
    x = r(x)
    t, d = x.shape
    b = len(q_lens)
    hd = k.shape[3]
    hq = d // hd
    s = k.shape[2]
    f = w["w_down"].shape[0]
    if pending is None:
        x1, h = port.fused_add_residual_rmsnorm(x, np.zeros_like(x), w["w_attn_norm"], False)
    else:
        x1, h = port.fused_add_residual_rmsnorm(x, r(pending), w["w_attn_norm"], True)
    x1, h = r(x1), r(h)
    qkv = r(port.linear(h, w["w_qkv"], False, False, t, w["w_qkv"].shape[1], d))
    q = np.zeros((b, hq, q_cache_len, hd), np.float32)
    port.rope_kvcache_prefill(pairing, qkv, q_lens, kv_lens, unpad, q, k, v)
    q = r(q)
    k[...] = r(k)
    v[...] = r(v)
    qk = np.zeros((b, hq, q_cache_len, s), np.float32)
    port.qk_scores(q, k, max_q, max_kv, qk)
    mask = intended_mask(q_lens, kv_lens, max_q, max_kv, q_cache_len, s)
    port.masked_attention_score(qk, mask, q_lens, max_kv, hd)
    qk = r(qk)
    pv = np.zeros((b, hq, q_cache_len, hd), np.float32)
    port.attention_qkv(qk, v, max_q, max_kv, pv)
    attn = port.transpose_unpad(r(pv), unpad, t)
    o = r(port.linear(attn, w["w_o"], False, False, t, d, d))
    x2, h2 = port.fused_add_residual_rmsnorm(x1, o, w["w_ffn_norm"], True)
    x2, h2 = r(x2), r(h2)
    gu = r(port.linear(h2, w["w_gate_up"], False, False, t, 2 * f, d))
    act = r(port.swiglu(gu))
    down = r(port.linear(act, w["w_down"], False, False, t, d, f))
    return {"x": x2, "down": down, "qk": qk, "attn": attn}
