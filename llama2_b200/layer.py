"""One Llama-2 decoder layer over this library's kernels — the layer driver
the reference leaves out (its src/core holds only a timer; its kernels are
called only by their tests).

A decode step of one layer for a batch of sequences, one new token each,
in the reference's operator API (a residual stream x and a pending addend,
with the fused add-residual RMSNorm at both norms,
include/kernel/fused_add_residual_rmsnorm.h:6-19):

    x, h   = x + pending, RMSNorm(x + pending)   (first layer: h = RMSNorm(x))
    qkv    = h Wqkv                               launch_linear (tcgen05, 16-bit)
    q, K/V = RoPE at kv_len - 1, append           launch_fused_reshape_rope_kvcache[_llama2]_decode
    p, a   = softmax(q K^T / sqrt(hd)), p V       fused decode attention (one pass over K and V)
    o      = a Wo                                 launch_linear
    x, h2  = x + o, RMSNorm(x + o)
    g      = h2 Wgu ; s = silu(g[:F]) * g[F:]     launch_linear, launch_swiglu
    pending = s Wdown                             launch_linear

The lengths are updated once per model step (launch_update_q_kv_lens) before
the first layer; each layer reads the updated kv_lens and the device max.
Weights are [in, out] row-major (the MN-major B operand of the tensor-core
GEMM). Nine launches per layer as listed (seven with the fused epilogues
below); ``capture_decode`` records a layer step as a CUDA graph. ``prefill``
runs the same layer over the new tokens of a batch of prompts (eleven
launches, nine fused: the scores, P.V and the unpad replace the fused decode
attention).

With 16-bit weights and more than 8 rows (where launch_linear runs on the
tensor cores) the QKV projection takes the RoPE + K/V append into its
epilogue and the gate/up projection the SwiGLU (``fuse_epilogues``, on by
default): two launches fewer and neither product goes to HBM, with results
bit-identical to the separate launches.
"""
from __future__ import annotations

import math

import torch

from . import ops


class DecoderLayer:
    def __init__(self, dim: int, heads: int, kv_heads: int, hidden: int, kv_cache_len: int, batch: int,
                 dtype=torch.bfloat16, device="cuda", seed: int = 0, pairing: int = 1, fuse_epilogues: bool = True):
        if dim % heads or heads % kv_heads:
            raise ValueError("dim must be a multiple of heads, heads of kv_heads")
        self.dim, self.heads, self.kv_heads, self.hidden = dim, heads, kv_heads, hidden
        self.head_dim = dim // heads
        self.kv_cache_len, self.batch, self.dtype, self.pairing = kv_cache_len, batch, dtype, pairing
        # the epilogue kernels' shape rules (16-bit, head_dim 64 or 128, F % 8 == 0)
        self.fuse_epilogues = (fuse_epilogues and dtype != torch.float32 and self.head_dim in (64, 128)
                               and hidden % 8 == 0)
        self.device = torch.device(device)
        hd, d, f = self.head_dim, dim, hidden
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)

        def weight(n_in, n_out):
            w = torch.randn(n_in, n_out, generator=g, device=self.device) / math.sqrt(n_in)
            return w.to(dtype).contiguous()

        self.w_attn_norm = (torch.rand(d, generator=g, device=self.device) + 0.5).to(dtype)
        self.w_qkv = weight(d, (heads + 2 * kv_heads) * hd)
        self.w_o = weight(d, d)
        self.w_ffn_norm = (torch.rand(d, generator=g, device=self.device) + 0.5).to(dtype)
        self.w_gate_up = weight(d, 2 * f)
        self.w_down = weight(f, d)
        self.k_cache = torch.randn(batch, kv_heads, kv_cache_len, hd, generator=g, device=self.device).to(dtype)
        self.v_cache = torch.randn(batch, kv_heads, kv_cache_len, hd, generator=g, device=self.device).to(dtype)
        # activations of one step
        e = dict(dtype=dtype, device=self.device)
        self.h = torch.empty(batch, d, **e)
        unfused = not self._fused(batch)  # products the epilogue kernels do not store
        self.qkv = torch.empty(batch if unfused else 0, (heads + 2 * kv_heads) * hd, **e)
        self.q = torch.zeros(batch, heads, 1, hd, **e)  # finished sequences keep this (RoPE skips them)
        self.qk = torch.zeros(batch, heads, 1, kv_cache_len, **e)
        self.attn = torch.empty(batch, heads, 1, hd, **e)
        self.o = torch.empty(batch, d, **e)
        self.gate_up = torch.empty(batch if unfused else 0, 2 * f, **e)
        self.act = torch.empty(batch, f, **e)
        self.down = torch.empty(batch, d, **e)
        ops.rope_table(hd, self.device)  # built before any graph capture

    def weights(self) -> dict:
        return {"w_attn_norm": self.w_attn_norm, "w_qkv": self.w_qkv, "w_o": self.w_o,
                "w_ffn_norm": self.w_ffn_norm, "w_gate_up": self.w_gate_up, "w_down": self.w_down}

    def decode(self, x: torch.Tensor, pending, kv_lens: torch.Tensor, max_kv_len: torch.Tensor,
               is_done: torch.Tensor) -> torch.Tensor:
        """One decode step of this layer. x: the residual stream [B, D],
        updated in place; pending: the previous layer's addend [B, D] or None
        (first layer). Returns this layer's addend (self.down)."""
        b, d, f = self.batch, self.dim, self.hidden
        if pending is None:
            ops.launch_fused_add_residual_rmsnorm(self.w_attn_norm, x, self.h, False)
            h = self.h
        else:
            ops.launch_fused_add_residual_rmsnorm(self.w_attn_norm, x, pending, True)
            h = pending  # the normed rows land in the residual argument
        fuse = self._fused(b)
        if fuse:
            ops.linear_rope_kvcache_decode(h, self.w_qkv, is_done, kv_lens, self.q, self.k_cache, self.v_cache,
                                           pairing=self.pairing)
        else:
            ops.launch_linear(False, False, b, self.qkv.shape[1], d, h, self.w_qkv, self.qkv)
            rope = (ops.launch_fused_reshape_rope_kvcache_llama2_decode if self.pairing
                    else ops.launch_fused_reshape_rope_kvcache_decode)
            rope(self.qkv, is_done, kv_lens, self.q, self.k_cache, self.v_cache)
        ops.decode_attention(self.q, self.k_cache, self.v_cache, kv_lens, max_kv_len, self.qk, self.attn)
        ops.launch_linear(False, False, b, d, d, self.attn.view(b, d), self.w_o, self.o)
        ops.launch_fused_add_residual_rmsnorm(self.w_ffn_norm, x, self.o, True)
        self._gate_up_swiglu(b, self.o, self.gate_up, self.act, fuse)
        ops.launch_linear(False, False, b, d, f, self.act, self.w_down, self.down)
        return self.down

    def _fused(self, rows: int) -> bool:
        """Whether this pass uses the epilogue kernels: above 8 rows, where
        launch_linear itself runs on the tensor cores."""
        return self.fuse_epilogues and rows > 8

    def _gate_up_swiglu(self, rows, h, gate_up, act, fuse):
        if fuse:
            ops.linear_swiglu(h, self.w_gate_up, act)
        else:
            ops.launch_linear(False, False, rows, 2 * self.hidden, self.dim, h, self.w_gate_up, gate_up)
            ops.launch_swiglu(gate_up, act)

    def capture_decode(self, x, pending, kv_lens, max_kv_len, is_done):
        """A CUDA graph of one decode() call on these tensors."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.decode(x.clone(), None if pending is None else pending.clone(), kv_lens, max_kv_len, is_done)
        torch.cuda.current_stream(self.device).wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            self.decode(x, pending, kv_lens, max_kv_len, is_done)
        return graph

    def prefill(self, x: torch.Tensor, pending, q_lens: torch.Tensor, kv_lens: torch.Tensor, max_q: int,
                max_kv: int, unpad_to_pad: torch.Tensor) -> torch.Tensor:
        """One prefill pass of this layer over T new tokens (sequence-major,
        unpadded). x: the residual stream [T, D], updated in place; pending:
        the previous layer's addend [T, D] or None; kv_lens: the updated
        lengths; max_q / max_kv: their maxima (host ints, as the reference
        passes them); unpad_to_pad: the token -> padded slot map
        (launch_build_padding_index_maps). Returns this layer's addend [T, D].

        qkv -> padded RoPE + append -> tcgen05 scores (QK^T, causal mask,
        softmax) -> P.V at the launch_linear site -> transpose + unpad -> O,
        then the feed-forward half as in decode()."""
        t, d, f = x.shape[0], self.dim, self.hidden
        qc = unpad_to_pad.numel() // self.batch
        buf = self._prefill_buffers(t, qc)
        if pending is None:
            ops.launch_fused_add_residual_rmsnorm(self.w_attn_norm, x, buf["h"], False)
            h = buf["h"]
        else:
            ops.launch_fused_add_residual_rmsnorm(self.w_attn_norm, x, pending, True)
            h = pending
        fuse = self._fused(t)
        if fuse:
            ops.linear_pad_rope_kvcache_prefill(h, self.w_qkv, q_lens, kv_lens, unpad_to_pad.view(-1), buf["q"],
                                                self.k_cache, self.v_cache, pairing=self.pairing)
        else:
            ops.launch_linear(False, False, t, buf["qkv"].shape[1], d, h, self.w_qkv, buf["qkv"])
            rope = (ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2 if self.pairing
                    else ops.launch_fused_pad_reshape_transpose_rope_kvcache)
            rope(buf["qkv"], q_lens, kv_lens, unpad_to_pad.view(-1), buf["q"], self.k_cache, self.v_cache)
        ops.prefill_attention_scores(buf["q"], self.k_cache, q_lens, kv_lens, max_q, max_kv, buf["qk"])
        ops.launch_attention_qkv(buf["qk"], self.v_cache, buf["pv"], max_q, max_kv)
        ops.launch_fused_transpose_unpad(t, buf["pv"], unpad_to_pad.view(-1), buf["attn"])
        ops.launch_linear(False, False, t, d, d, buf["attn"], self.w_o, buf["o"])
        ops.launch_fused_add_residual_rmsnorm(self.w_ffn_norm, x, buf["o"], True)
        self._gate_up_swiglu(t, buf["o"], buf["gate_up"], buf["act"], fuse)
        ops.launch_linear(False, False, t, d, f, buf["act"], self.w_down, buf["down"])
        return buf["down"]

    def _prefill_buffers(self, t: int, qc: int) -> dict:
        key = (t, qc)
        if getattr(self, "_pf_key", None) != key:
            b, h, kvh, hd, d, f = self.batch, self.heads, self.kv_heads, self.head_dim, self.dim, self.hidden
            e = dict(dtype=self.dtype, device=self.device)
            # the products that the epilogue kernels never store are not allocated for them
            unfused = not self._fused(t)
            self._pf = {"h": torch.empty(t, d, **e), "qkv": torch.empty(t if unfused else 0, (h + 2 * kvh) * hd, **e),
                        "q": torch.zeros(b, h, qc, hd, **e), "qk": torch.zeros(b, h, qc, self.kv_cache_len, **e),
                        "pv": torch.zeros(b, h, qc, hd, **e), "attn": torch.empty(t, d, **e),
                        "o": torch.empty(t, d, **e), "gate_up": torch.empty(t if unfused else 0, 2 * f, **e),
                        "act": torch.empty(t, f, **e), "down": torch.empty(t, d, **e)}
            self._pf_key = key
        return self._pf

    def launches_per_step(self) -> int:
        return 7 if self._fused(self.batch) else 9

    def launches_per_prefill(self, tokens: int) -> int:
        return 9 if self._fused(tokens) else 11
