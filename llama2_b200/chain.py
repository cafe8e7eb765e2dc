"""The layer-kernel chain: one decode step or one prefill pass over a batch.

This composes the operators in the order the reference's tests exercise them
(there is no layer code in the reference; src/main.cpp is a stub):

  decode:  update lens -> embedding -> RMSNorm -> RoPE + KV append
           -> fused scores (QK^T, scale, mask, softmax) -> SwiGLU
  prefill: update lens -> padding maps -> embedding -> RMSNorm
           -> prefill RoPE + KV append -> fused prefill scores -> SwiGLU

With ``attention_output=True`` the chain also produces the attention output
(tokens, D): the one-launch decode step computes it in the same pass
(l2k_decode_step_attention; the operator sequence runs the fused decode
attention in place of the scores); prefill follows the scores with P.V at
the launch_linear call site (tensor cores for 16-bit) and the transpose +
unpad.

The q/k/v and gate/up activations are inputs (the projection GEMMs are not
on this path). A decode step runs as ONE launch (ops.decode_step, the fused
decode-step kernel) whenever its shapes are supported, else as the operator
sequence above. All buffers live on one device; ``step()`` only enqueues
work on the current stream, and ``capture()`` records the step as a CUDA
graph so a step costs one graph launch; ``replay()`` launches the one-kernel
step directly and replays the graph otherwise. ``step_e2e()`` is the host-facing
form: copy this step's inputs from pinned host memory, run, copy the results
back.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from .workloads import Workload

_TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


class Packed:
    """Several tensors as 256-byte aligned views of one contiguous buffer, so
    that a step's inputs (or results) cross PCIe in one copy."""

    def __init__(self, specs, device, pin=False):
        offs, off = [], 0
        for _, shape, dt in specs:
            off = (off + 255) // 256 * 256
            n = int(np.prod(shape)) * torch.empty((), dtype=dt).element_size()
            offs.append((off, n))
            off += n
        self.buf = torch.zeros(off, dtype=torch.uint8, device=device)
        if pin:
            self.buf = self.buf.pin_memory()
        self.offsets = {name: o for (name, _, _), (o, _) in zip(specs, offs)}
        self.views = {name: self.buf[o:o + n].view(dt).view(shape)
                      for (name, shape, dt), (o, n) in zip(specs, offs)}

    def __getitem__(self, name):
        return self.views[name]


class Chain:
    def __init__(self, w: Workload, inputs: dict, device="cuda", use_table: bool = True, fused: bool = True,
                 attention_output: bool = False):
        self.w = w
        self.attention_output = attention_output
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
        # per-step inputs, packed (one host-to-device copy per step)
        qc = w.prefill_len or 1
        self.in_specs = [("ids", (t,), torch.uint32), ("q_lens", (b,), torch.uint32),
                         ("kv_lens", (b,), torch.uint32), ("is_done", (b,), torch.uint8),
                         ("qkv", (t, 3 * d), dt), ("gate_up", (t, 2 * f), dt)]
        self.inputs = Packed(self.in_specs, self.device)
        for name, _, tdt in self.in_specs:
            self.inputs[name].copy_(torch.from_numpy(np.ascontiguousarray(inputs[name])).to(tdt))
        self.ids, self.q_lens, self.kv_lens = self.inputs["ids"], self.inputs["q_lens"], self.inputs["kv_lens"]
        self.is_done, self.qkv, self.gate_up = self.inputs["is_done"], self.inputs["qkv"], self.inputs["gate_up"]
        self.kv_lens_initial = self.kv_lens.clone()
        # results, packed (the small ones in one device-to-host copy per step,
        # the score rows last), and intermediates
        self.out_specs = [("max_lens", (2,), torch.uint32), ("normed", (t, d), dt), ("ffn_out", (t, f), dt)]
        if attention_output:
            self.out_specs.append(("attn_out", (t, d), dt))
        self.out_specs.append(("qk", (b, h, qc, s), dt))
        self.outputs = Packed(self.out_specs, self.device)
        self.max_lens, self.normed = self.outputs["max_lens"], self.outputs["normed"]
        self.ffn_out, self.qk = self.outputs["ffn_out"], self.outputs["qk"]
        self.attn_out = self.outputs["attn_out"] if attention_output else None
        if attention_output and not w.decode:
            self.qkv_pad = torch.empty(b, h, qc, hd, dtype=dt, device=self.device)  # P.V before the unpad
        self.x = torch.empty(t, d, dtype=dt, device=self.device)
        self.q = torch.zeros(b, h, qc, hd, dtype=dt, device=self.device)
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
        self._launch = None  # the one-kernel step, launched directly (no graph)
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
            if self.attention_output:
                ops.decode_step_attention(**self._step_tensors(), workspace=self.workspace,
                                          attn_out=self.attn_out.view(w.batch, w.heads, 1, w.head_dim))
            else:
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
            if self.attention_output:
                ops.decode_attention(self.q, self.k_cache, self.v_cache, self.kv_lens, self.max_lens[1:2], self.qk,
                                     self.attn_out.view(w.batch, w.heads, 1, w.head_dim))
            else:
                ops.decode_attention_scores(self.q, self.k_cache, self.kv_lens, self.max_lens[1:2], self.qk)
        else:
            rope = (ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2 if w.pairing
                    else ops.launch_fused_pad_reshape_transpose_rope_kvcache)
            rope(self.qkv, self.q_lens, self.kv_lens, self.unpad_to_pad.view(-1), self.q, self.k_cache, self.v_cache,
                 use_table=self.use_table)
            ops.prefill_attention_scores(self.q, self.k_cache, self.q_lens, self.kv_lens, self.max_q, self.max_kv,
                                         self.qk)
            if self.attention_output:
                ops.launch_attention_qkv(self.qk, self.v_cache, self.qkv_pad, self.max_q, self.max_kv)
                ops.launch_fused_transpose_unpad(w.tokens, self.qkv_pad, self.unpad_to_pad.view(-1), self.attn_out)
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
        # lens, maps, embedding, norm, rope, scores (+ masked softmax for fp32), swiglu (+ P.V, unpad)
        return (8 if self.w.dtype == "f32" else 7) + (2 if self.attention_output else 0)

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
        """Enqueue one step: the one-kernel fused step is launched directly
        (a CUDA graph adds its launch cost and saves nothing for one kernel);
        the operator sequence replays its graph."""
        if self.fused:
            if self._launch is None:
                w = self.w
                attn = (self.attn_out.view(w.batch, w.heads, 1, w.head_dim) if self.attention_output else None)
                self._launch = ops.decode_step_launcher(**self._step_tensors(), workspace=self.workspace,
                                                        attn_out=attn)
            self._launch()
            return
        if self.graph is None:
            self.capture()
        self.graph.replay()

    # ------------------------------------------------------------------
    def host_buffers(self, inputs: dict):
        """Pinned host images of the packed per-step inputs (filled from
        `inputs`) and of the packed results."""
        hin = Packed(self.in_specs, "cpu", pin=True)
        for name, _, tdt in self.in_specs:
            hin[name].copy_(torch.from_numpy(np.ascontiguousarray(inputs[name])).to(tdt))
        hout = Packed(self.out_specs, "cpu", pin=True)
        # A step writes keys [0, M) of every score row, M = the largest updated length.
        kv = np.asarray(inputs["kv_lens"], np.int64) + np.asarray(inputs["q_lens"], np.int64)
        self._m_written = int(min(kv.max() if kv.size else 0, self.w.kv_cache_len))
        self._pinned = (hin, hout)
        return hin, hout

    def _one_copy(self) -> bool:
        """Whether the results come back in ONE device-to-host copy (the small
        outputs and every score row whole) rather than two (the small outputs,
        then a 2-D copy of the written keys [0, M) of every row): one copy
        when the written part is at least half of each row, where the unwritten
        tail costs less than a second copy's latency."""
        return 2 * self._m_written >= self.qk.shape[3]

    def e2e_bytes(self):
        hin, hout = self._pinned
        qk = self.qk
        small = hout.offsets["qk"]
        rows = qk.shape[0] * qk.shape[1] * qk.shape[2]
        cols = qk.shape[3] if self._one_copy() else self._m_written
        return hin.buf.numel(), small + rows * cols * qk.element_size()

    def step_e2e(self):
        """One copy of the step's inputs to the device, the step (replay()),
        then its results back to pinned host memory: either one copy of the
        lengths maxima, normed rows, SwiGLU output and the whole score rows,
        or one copy of the small results and one 2-D copy of the written part
        (keys [0, M)) of every score row, whichever moves less (_one_copy)."""
        from cuda.bindings import runtime as cudart

        hin, hout = self._pinned
        self.inputs.buf.copy_(hin.buf, non_blocking=True)
        self.replay()
        small = hout.offsets["qk"]
        qk, hqk = self.qk, hout["qk"]
        if self._one_copy():
            n = small + qk.numel() * qk.element_size()
            hout.buf[:n].copy_(self.outputs.buf[:n], non_blocking=True)
            return
        hout.buf[:small].copy_(self.outputs.buf[:small], non_blocking=True)
        es = qk.element_size()
        rows = qk.shape[0] * qk.shape[1] * qk.shape[2]
        if self._m_written and rows:
            pitch = qk.shape[3] * es
            err, = cudart.cudaMemcpy2DAsync(hqk.data_ptr(), pitch, qk.data_ptr(), pitch, self._m_written * es, rows,
                                            cudart.cudaMemcpyKind.cudaMemcpyDeviceToHost,
                                            torch.cuda.current_stream(self.device).cuda_stream)
            if err != cudart.cudaError_t.cudaSuccess:
                raise RuntimeError(f"score rows device-to-host copy failed: {err}")
