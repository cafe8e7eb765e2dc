"""The layer-kernel chain: one decode step or one prefill pass over a batch.

This composes the operators in the order the reference's tests exercise them
(there is no layer code in the reference; src/main.cpp is a stub):

  decode:  update lens -> embedding -> RMSNorm -> RoPE + KV append
           -> fused scores (QK^T, scale, mask, softmax) -> SwiGLU
  prefill: update lens -> padding maps -> embedding -> RMSNorm
           -> prefill RoPE + KV append -> fused prefill scores -> SwiGLU

The q/k/v and gate/up activations are inputs (the projection GEMMs are not
on this path). A decode step runs as ONE launch (ops.decode_step, the fused
decode-step kernel) whenever its shapes are supported, else as the operator
sequence above. All buffers live on one device; ``step()`` only enqueues
work on the current stream, and ``capture()`` records the step as a CUDA
graph so a step costs one graph launch. ``step_e2e()`` is the host-facing
form: copy this step's inputs from pinned host memory, run, copy the results
back.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from .workloads import Workload

_TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


class Chain:
    def __init__(self, w: Workload, inputs: dict, device="cuda", use_table: bool = True, fused: bool = True):
        self.w = w
        self.device = torch.device(device)
        dt = _TORCH[w.dtype]
        self.dtype = dt
        d, h, hd, f, s = w.dim, w.heads, w.head_dim, w.hidden, w.kv_cache_len
        b, t = w.batch, w.tokens

        def put(a, dtype=None):
            x = torch.from_numpy(np.ascontiguousarray(a))
            return (x.to(dtype) if dtype is not None else x).to(self.device)

        # resident state
        self.embed_table = put(inputs["embed_table"], dt)
        self.norm_weight = put(inputs["norm_weight"], dt)
        if "k_cache" in inputs:
            self.k_cache = put(inputs["k_cache"], dt)
            self.v_cache = put(inputs["v_cache"], dt)
        else:
            # Large caches are drawn N(0, 1) on the device (seeded) instead of on the host.
            g = torch.Generator(device=self.device)
            g.manual_seed(int(inputs.get("cache_seed", 0)))
            self.k_cache = torch.randn(b, h, s, hd, generator=g, dtype=dt, device=self.device)
            self.v_cache = torch.randn(b, h, s, hd, generator=g, dtype=dt, device=self.device)
        # per-step inputs
        self.ids = put(inputs["ids"])
        self.q_lens = put(inputs["q_lens"])
        self.kv_lens = put(inputs["kv_lens"])
        self.kv_lens_initial = self.kv_lens.clone()
        self.is_done = put(inputs["is_done"])
        self.qkv = put(inputs["qkv"], dt)
        self.gate_up = put(inputs["gate_up"], dt)
        # outputs / intermediates
        self.x = torch.empty(t, d, dtype=dt, device=self.device)
        self.normed = torch.empty(t, d, dtype=dt, device=self.device)
        qc = w.prefill_len or 1
        self.q = torch.zeros(b, h, qc, hd, dtype=dt, device=self.device)
        self.qk = torch.zeros(b, h, qc, s, dtype=dt, device=self.device)
        self.ffn_out = torch.empty(t, f, dtype=dt, device=self.device)
        self.max_lens = torch.zeros(2, dtype=torch.uint32, device=self.device)
        if not w.decode:
            self.unpad_to_pad = torch.zeros(b, qc, dtype=torch.uint32, device=self.device)
            self.seq_offsets = torch.zeros(b, dtype=torch.uint32, device=self.device)
            ql = np.asarray(inputs["q_lens"], np.int64)
            self.max_q = int(ql.max())
            self.max_kv = int((np.asarray(inputs["kv_lens"], np.int64) + ql).max())
        self.use_table = use_table
        if use_table:
            ops.rope_table(hd, self.device)  # build before any graph capture
        # Decode runs as one fused launch (ops.decode_step) whenever the shapes
        # allow it; otherwise, and for prefill, as the sequence of operators.
        self.fused = False
        if w.decode and fused:
            self.workspace = ops.decode_step_workspace(self.device)
            self.fused = ops.decode_step_supported(**self._step_tensors())
        self.graph = None
        self._pinned = None

    def _step_tensors(self) -> dict:
        return dict(q_lens=self.q_lens, kv_lens=self.kv_lens, max_lens=self.max_lens, input_ids=self.ids,
                    embed_table=self.embed_table, norm_weight=self.norm_weight, x=self.x, normed=self.normed,
                    qkv=self.qkv, is_done=self.is_done, q=self.q, k_cache=self.k_cache, v_cache=self.v_cache,
                    qk=self.qk, gate_up=self.gate_up, ffn_out=self.ffn_out, pairing=self.w.pairing,
                    use_table=self.use_table)

    # ------------------------------------------------------------------
    def step(self, branches=None):
        """Enqueue one chain step on the current stream.

        branches: optional pair of side streams. The lengths update (and the
        padding maps) run first on the current stream; then embedding ->
        RMSNorm runs on branches[0], SwiGLU on branches[1] and RoPE -> scores
        on the current stream, which finally waits for both branches. The
        three sub-chains share no data, so the step's critical path is the
        longest of them instead of their sum."""
        w = self.w
        if self.fused:
            ops.decode_step(**self._step_tensors(), workspace=self.workspace)
            return
        main = torch.cuda.current_stream(self.device)
        ops.launch_update_q_kv_lens(self.q_lens, self.kv_lens, self.max_lens[0:1], self.max_lens[1:2])
        if not w.decode:
            ops.launch_build_padding_index_maps(w.tokens, self.q_lens, self.unpad_to_pad, self.seq_offsets)
        if branches:
            for s in branches:
                s.wait_stream(main)
            with torch.cuda.stream(branches[0]):
                ops.launch_embedding(self.ids, self.embed_table, self.x)
                ops.launch_fused_add_residual_rmsnorm(self.norm_weight, self.x, self.normed, False)
            with torch.cuda.stream(branches[1]):
                ops.launch_swiglu(self.gate_up, self.ffn_out)
        else:
            ops.launch_embedding(self.ids, self.embed_table, self.x)
            ops.launch_fused_add_residual_rmsnorm(self.norm_weight, self.x, self.normed, False)
        if w.decode:
            rope = (ops.launch_fused_reshape_rope_kvcache_llama2_decode if w.pairing
                    else ops.launch_fused_reshape_rope_kvcache_decode)
            rope(self.qkv, self.is_done, self.kv_lens, self.q, self.k_cache, self.v_cache, use_table=self.use_table)
            ops.decode_attention_scores(self.q, self.k_cache, self.kv_lens, self.max_lens[1:2], self.qk)
        else:
            rope = (ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2 if w.pairing
                    else ops.launch_fused_pad_reshape_transpose_rope_kvcache)
            rope(self.qkv, self.q_lens, self.kv_lens, self.unpad_to_pad.view(-1), self.q, self.k_cache, self.v_cache,
                 use_table=self.use_table)
            ops.prefill_attention_scores(self.q, self.k_cache, self.q_lens, self.kv_lens, self.max_q, self.max_kv,
                                         self.qk)
        if branches:
            for s in branches:
                main.wait_stream(s)
        else:
            ops.launch_swiglu(self.gate_up, self.ffn_out)

    def kernels_per_step(self) -> int:
        """Kernel launches of this library per step."""
        if self.fused:
            return 1
        if self.w.decode:
            return 6
        # lens, maps, embedding, norm, rope, scores (+ masked softmax for fp32), swiglu
        return 8 if self.w.dtype == "f32" else 7

    def reset_lengths(self):
        """Restore the pre-step kv_lens (so a step can be repeated)."""
        self.kv_lens.copy_(self.kv_lens_initial, non_blocking=True)

    def capture(self):
        """Record step() as a CUDA graph with its three independent sub-chains as
        parallel branches; replay() then launches the whole step at once."""
        s = torch.cuda.Stream(device=self.device)
        s.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(s):
            self.step()  # warm-up outside capture (lazy attribute setup)
            self.reset_lengths()
        torch.cuda.current_stream(self.device).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        branches = (torch.cuda.Stream(device=self.device), torch.cuda.Stream(device=self.device))
        with torch.cuda.graph(g):
            self.step(branches)
        self.graph = g
        self.reset_lengths()
        return g

    def replay(self):
        if self.graph is None:
            self.capture()
        self.graph.replay()

    # ------------------------------------------------------------------
    def host_buffers(self, inputs: dict):
        """Pinned host copies of the per-step inputs and the step's results."""
        pin = lambda a, dt=None: (torch.from_numpy(np.ascontiguousarray(a)).to(dt) if dt else
                                  torch.from_numpy(np.ascontiguousarray(a))).pin_memory()
        ins = {
            "ids": pin(inputs["ids"]), "q_lens": pin(inputs["q_lens"]), "kv_lens": pin(inputs["kv_lens"]),
            "is_done": pin(inputs["is_done"]), "qkv": pin(inputs["qkv"], self.dtype),
            "gate_up": pin(inputs["gate_up"], self.dtype),
        }
        outs = {
            "normed": torch.empty_like(self.normed, device="cpu").pin_memory(),
            "qk": torch.empty_like(self.qk, device="cpu").pin_memory(),
            "ffn_out": torch.empty_like(self.ffn_out, device="cpu").pin_memory(),
            "max_lens": torch.empty_like(self.max_lens, device="cpu").pin_memory(),
        }
        self._pinned = (ins, outs)
        return ins, outs

    def e2e_bytes(self):
        ins, outs = self._pinned
        return (sum(t.numel() * t.element_size() for t in ins.values()),
                sum(t.numel() * t.element_size() for t in outs.values()))

    def step_e2e(self):
        """H2D of the step inputs, the chain (graph replay), D2H of the results."""
        ins, outs = self._pinned
        dsts = {"ids": self.ids, "q_lens": self.q_lens, "kv_lens": self.kv_lens, "is_done": self.is_done,
                "qkv": self.qkv, "gate_up": self.gate_up}
        for k, t in ins.items():
            dsts[k].copy_(t, non_blocking=True)
        self.replay()
        outs["normed"].copy_(self.normed, non_blocking=True)
        outs["qk"].copy_(self.qk, non_blocking=True)
        outs["ffn_out"].copy_(self.ffn_out, non_blocking=True)
        outs["max_lens"].copy_(self.max_lens, non_blocking=True)
