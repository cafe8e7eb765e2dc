"""The layer-kernel chain on the host CPU — TEST/BASELINE INFRASTRUCTURE ONLY.

Used by bench.py's CPU legs: ``cpu_baseline`` (impl="port": the C
restatement, oracle/liboracle.so, one thread) and ``--impl reference``
(impl="ref": the reference's own CPU test helpers compiled from its sources,
oracle/_ref/libref_oracle.so, on every host thread). Work is split over
(sequence, head) score rows and row blocks with a thread pool; ctypes
releases the GIL during the C calls, so threads run in parallel.

The reference helpers take std::vector arguments; the glue copies each
argument into a vector on every call, as a caller of those helpers must.
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes

import numpy as np

import oracle

u = ctypes.c_uint
P = lambda a: ctypes.c_void_p(a.ctypes.data)


def ref_available() -> bool:
    return oracle.ref_available()


class CpuChain:
    def __init__(self, w, inputs: dict, impl: str = "port", threads: int = 1, seed: int = 0,
                 attention_output: bool = False, max_sequences: int = 8):
        self.w = w
        self.max_sequences = max(1, int(max_sequences))
        self.attention_output = attention_output
        self.impl = impl
        self.kind = "reference" if impl == "ref" else "port"
        self.threads = max(1, int(threads or 1))
        self.pool = cf.ThreadPoolExecutor(self.threads) if self.threads > 1 else None
        self.lib = oracle.ref_lib() if impl == "ref" else oracle.port_lib()
        if self.lib is None:
            raise RuntimeError("reference helpers are not built (make -C oracle ref)")
        self.inp = inputs
        b, h, hd, s = w.batch, w.heads, w.head_dim, w.kv_cache_len
        sample = self.sample_batch()
        if "k_cache" in inputs:
            self.k = np.ascontiguousarray(inputs["k_cache"][sample])
            self.v = np.ascontiguousarray(inputs["v_cache"][sample])
        else:
            rng = np.random.default_rng(seed)
            self.k = rng.standard_normal((len(sample), h, s, hd), dtype=np.float32)
            self.v = rng.standard_normal((len(sample), h, s, hd), dtype=np.float32)
        self._sample = sample

    def sample_batch(self):
        """Sequences processed per step: the first max_sequences of a decode
        batch (8 by default), one prefill sequence."""
        w = self.w
        return list(range(min(w.batch, self.max_sequences))) if w.decode else [0]

    def _map(self, fn, items):
        if self.pool is None:
            for it in items:
                fn(it)
        else:
            list(self.pool.map(fn, items))

    def step(self, sample=None, row_stride=1):
        """One chain step on the sample. row_stride > 1 computes the scores of
        every row_stride-th query row only (prefill); self.last_times then
        holds the seconds spent outside and inside the scores, so a caller can
        extrapolate the full step as other + scores * row_stride."""
        import time as _time
        t_start = _time.perf_counter()
        w = self.w
        lib = self.lib
        sample = self._sample if sample is None else sample
        nb = len(sample)
        qlen = w.prefill_len or 1
        d, h, hd, s, f = w.dim, w.heads, w.head_dim, w.kv_cache_len, w.hidden
        q_lens = np.ascontiguousarray(self.inp["q_lens"][sample])
        kv0 = np.ascontiguousarray(self.inp["kv_lens"][sample])
        tok = np.concatenate([np.arange(i * qlen, (i + 1) * qlen) for i in sample])
        ids = np.ascontiguousarray(self.inp["ids"][tok])
        qkv = np.ascontiguousarray(self.inp["qkv"][tok])
        gate_up = np.ascontiguousarray(self.inp["gate_up"][tok])
        t = len(tok)
        table = self.inp["embed_table"]
        weight = self.inp["norm_weight"]
        # lens
        kv = np.empty_like(kv0)
        mq, mkv = ctypes.c_uint(), ctypes.c_uint()
        if self.impl == "ref":
            lib.ref_update_q_kv_lens(P(q_lens), P(kv0), u(nb), P(kv), ctypes.byref(mq), ctypes.byref(mkv))
        else:
            kv[:] = kv0
            lib.orc_update_q_kv_lens(P(q_lens), P(kv), ctypes.c_int64(nb), ctypes.byref(mq), ctypes.byref(mkv))
        max_kv = mkv.value
        # embedding + RMSNorm (row blocks)
        x = np.empty((t, d), np.float32)
        xa = np.empty_like(x)
        normed = np.empty_like(x)
        zeros = np.zeros_like(x)
        blocks = [(r0, min(t, r0 + max(1, t // self.threads))) for r0 in range(0, t, max(1, t // self.threads))]

        def emb_norm(blk):
            r0, r1 = blk
            n = r1 - r0
            ids_b = np.ascontiguousarray(ids[r0:r1])
            xb, xab, nb_, zb = x[r0:r1], xa[r0:r1], normed[r0:r1], zeros[r0:r1]
            if self.impl == "ref":
                lib.ref_embedding(P(ids_b), u(n), P(table), u(d), P(xb))
                lib.ref_fused_add_residual_rmsnorm(P(xb), P(zb), P(weight), u(n), u(d), ctypes.c_int(0), P(xab),
                                                   P(nb_))
            else:
                lib.orc_embedding(P(ids_b), ctypes.c_int64(n), P(table), ctypes.c_int64(d), ctypes.c_int64(4), P(xb))
                lib.orc_fused_add_residual_rmsnorm(P(xb), P(zb), P(weight), ctypes.c_int64(n), ctypes.c_int64(d),
                                                   ctypes.c_int(0), P(xab), P(nb_))

        self._map(emb_norm, blocks)
        # RoPE + KV append, then scores per (sequence, head)
        q = np.zeros((nb, h, qlen, hd), np.float32)
        qk = np.zeros((nb, h, qlen, s), np.float32)
        attn = np.zeros((nb, h, qlen, hd), np.float32) if self.attention_output else None

        def head_work(item):
            si, hh = item
            kvl = int(kv[si])
            hist = kvl - int(q_lens[si])
            if not self._rope_only:
                return score_work(si, hh, kvl, hist)
            for ti in range(int(q_lens[si])):
                pos = hist + ti
                row = qkv[si * qlen + ti]
                qh = np.ascontiguousarray(row[hh * hd:(hh + 1) * hd])
                kh = np.ascontiguousarray(row[(h + hh) * hd:(h + hh + 1) * hd])
                vh = row[(2 * h + hh) * hd:(2 * h + hh + 1) * hd]
                if self.impl == "ref":
                    rot = lib.ref_rotate_head_llama2 if w.pairing else lib.ref_rotate_head
                    qo = np.empty(hd, np.float32)
                    ko = np.empty(hd, np.float32)
                    rot(P(qh), u(hd), u(pos), u(kvl), P(qo))
                    rot(P(kh), u(hd), u(pos), u(kvl), P(ko))
                    q[si, hh, ti] = qo
                    self.k[si, hh, pos] = ko
                else:
                    qo = np.empty(hd, np.float32)
                    ko = np.empty(hd, np.float32)
                    lib.orc_rotate_one_head(ctypes.c_int(w.pairing), P(qh), ctypes.c_int64(hd), u(pos), u(kvl), P(qo))
                    lib.orc_rotate_one_head(ctypes.c_int(w.pairing), P(kh), ctypes.c_int64(hd), u(pos), u(kvl), P(ko))
                    q[si, hh, ti] = qo
                    self.k[si, hh, pos] = ko
                self.v[si, hh, pos] = vh

        def score_work(si, hh, kvl, hist):
            # scores: QK^T over keys < max_kv, intended mask, softmax
            kslice = np.ascontiguousarray(self.k[si, hh, :max_kv])
            for ti in range(0, int(q_lens[si]), row_stride):
                qrow = np.ascontiguousarray(q[si, hh, ti])
                logits = np.zeros(max_kv, np.float32)
                mask = np.zeros(max_kv, np.uint8)
                mask[:hist + ti + 1] = 1
                if self.impl == "ref":
                    lib.ref_linear(P(qrow), P(kslice), ctypes.c_int(0), ctypes.c_int(1), u(1), u(max_kv), u(hd),
                                   P(logits))
                    out = np.zeros(max_kv, np.float32)
                    one = np.ones(1, np.uint32)
                    lib.ref_masked_attention_score_f32(P(logits), P(mask), P(one), u(1), u(1), u(1), u(max_kv),
                                                       u(max_kv), u(hd), P(out))
                    qk[si, hh, ti, :max_kv] = out
                else:
                    lib.orc_linear(P(qrow), P(kslice), ctypes.c_int(0), ctypes.c_int(1), ctypes.c_int64(1),
                                   ctypes.c_int64(max_kv), ctypes.c_int64(hd), P(logits))
                    one = np.ones(1, np.uint32)
                    lib.orc_masked_attention_score(P(logits), P(mask), P(one), ctypes.c_int64(1), ctypes.c_int64(1),
                                                   ctypes.c_int64(1), ctypes.c_int64(max_kv), ctypes.c_int64(max_kv),
                                                   ctypes.c_int64(hd))
                    qk[si, hh, ti, :max_kv] = logits
                if attn is not None:
                    # P.V of this row: the launch_linear helper on (1 x max_kv) x (max_kv x hd)
                    prow = np.ascontiguousarray(qk[si, hh, ti, :max_kv])
                    vslice = np.ascontiguousarray(self.v[si, hh, :max_kv])
                    orow = np.zeros(hd, np.float32)
                    if self.impl == "ref":
                        lib.ref_linear(P(prow), P(vslice), ctypes.c_int(0), ctypes.c_int(0), u(1), u(hd), u(max_kv),
                                       P(orow))
                    else:
                        lib.orc_linear(P(prow), P(vslice), ctypes.c_int(0), ctypes.c_int(0), ctypes.c_int64(1),
                                       ctypes.c_int64(hd), ctypes.c_int64(max_kv), P(orow))
                    attn[si, hh, ti] = orow

        self._rope_only = True
        self._map(head_work, [(si, hh) for si in range(nb) for hh in range(h)])
        t_scores = _time.perf_counter()
        self._rope_only = False
        self._map(head_work, [(si, hh) for si in range(nb) for hh in range(h)])
        t_scores_end = _time.perf_counter()
        # SwiGLU (row blocks)
        ffn = np.empty((t, f), np.float32)

        def swiglu(blk):
            r0, r1 = blk
            gb = np.ascontiguousarray(gate_up[r0:r1])
            ob = ffn[r0:r1]
            if self.impl == "ref":
                lib.ref_swiglu(P(gb), u(r1 - r0), u(f), P(ob))
            else:
                lib.orc_swiglu(P(gb), ctypes.c_int64(r1 - r0), ctypes.c_int64(f), P(ob))

        self._map(swiglu, blocks)
        t_end = _time.perf_counter()
        self.last = {"normed": normed, "q": q, "qk": qk, "ffn_out": ffn, "kv_lens": kv}
        if attn is not None:
            # transpose + unpad: token rows (sequence-major) of H * hd
            self.last["attn_out"] = np.ascontiguousarray(attn.transpose(0, 2, 1, 3)).reshape(nb * qlen, h * hd)
        self.last_times = {"other": (t_scores - t_start) + (t_end - t_scores_end),
                           "scores": t_scores_end - t_scores}
        return nb * qlen
