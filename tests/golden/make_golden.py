"""Generate the golden fixtures under tests/golden/ from the reference itself.

Each fixture file holds the reference's own unit-test cases (pentatracy5/llama2,
test/kernel/*.cu): the inputs each TEST builds, restated here case by case with
the file:line of the TEST, and the outputs of the reference's own CPU helper
(compute_expected_* etc.) on those inputs. The helpers are compiled from the
reference's test sources in place (``make -C oracle ref``) and called through
``oracle/_ref/libref_oracle.so``.

Run from the repository root, where the reference sources are present:

    python tests/golden/make_golden.py [--ref-root DIR]   (default: $L2K_REFERENCE_ROOT, else ../reference)

The fixtures are committed; nothing at test time needs the reference.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

F32 = np.float32
U32 = np.uint32


def P(a):
    return ctypes.c_void_p(a.ctypes.data)


def pattern(n, mod, mul, sub):
    """static_cast<float>(i % mod) * mul - sub, in float32 like the tests."""
    i = np.arange(n, dtype=np.int64)
    base = (i % mod).astype(F32) if mod else i.astype(F32)
    return (base * F32(mul) - F32(sub)).astype(F32)


class Writer:
    def __init__(self, family):
        self.family = family
        self.arrays = {}
        self.meta = {}

    def case(self, name, params, **arrays):
        self.meta[name] = params
        for k, v in arrays.items():
            self.arrays[f"{name}__{k}"] = np.ascontiguousarray(v)

    def save(self):
        path = os.path.join(HERE, f"{self.family}.npz")
        np.savez_compressed(path, __meta__=np.array(json.dumps(self.meta, sort_keys=True)), **self.arrays)
        print(f"wrote {path}: {len(self.meta)} cases")


def gen_embedding(lib):
    w = Writer("embedding")
    cases = [
        # name, vocab, dim, ids, table start, test_embedding.cu line
        ("BasicLookup", 4, 8, [0, 2, 1, 3], 0.1, 21),
        ("SingleTokenFourDim", 3, 4, [2], 0.0, 64),
        ("RepeatedIndex", 5, 4, [1, 1, 3, 3, 1, 3], 0.0, 98),
        ("MultiTokenBatch", 10, 16, [i % 10 for i in range(32)], 0.5, 136),
    ]
    for name, vocab, dim, ids, start, line in cases:
        table = np.zeros(vocab * dim, dtype=F32)
        lib.ref_fill_sequential(P(table), ctypes.c_uint(table.size), ctypes.c_float(start))
        ids = np.array(ids, dtype=U32)
        out = np.zeros(ids.size * dim, dtype=F32)
        lib.ref_embedding(P(ids), ctypes.c_uint(ids.size), P(table), ctypes.c_uint(dim), P(out))
        w.case(name, {"line": f"test_embedding.cu:{line}", "vocab": vocab, "dim": dim},
               ids=ids, table=table.reshape(vocab, dim), out=out.reshape(ids.size, dim))
    w.save()


def gen_rmsnorm(lib):
    w = Writer("rmsnorm")
    # Decimal literals such as 0.3f: round(0.1 * 3, 6) is the double nearest 0.3,
    # whose float32 rounding is the literal's value.
    x_rows3 = np.array([round(0.1 * (i + 1), 6) for i in range(16)] + [round(-0.1 * (i + 1), 6) for i in range(16)] +
                       [2.0] * 16, dtype=F32)
    res_rows3 = np.array(
        [round(v, 6) for i in range(8) for v in (-0.1 * (i + 1), 0.1 * (i + 1))] +
        [round(v, 6) for i in range(8) for v in (0.1 * (i + 1), -0.1 * (i + 1))] +
        [v for _ in range(8) for v in (1.0, -1.0)], dtype=F32)
    x8 = np.arange(1, 9, dtype=F32)
    res8 = np.array([0.5, -0.5, 1.0, -1.0, 0.25, -0.25, 0.125, -0.125], dtype=F32)
    w16 = np.arange(1, 17, dtype=F32)

    def fixed(name, dtype, add, t, d, x, res, wt, tol, line):
        xa = np.zeros(t * d, F32)
        ro = np.zeros(t * d, F32)
        lib.ref_fused_add_residual_rmsnorm(P(x), P(res), P(wt), ctypes.c_uint(t), ctypes.c_uint(d),
                                           ctypes.c_int(int(add)), P(xa), P(ro))
        w.case(name, {"line": f"test_fused_add_residual_rmsnorm.cu:{line}", "dtype": dtype, "add": add,
                      "tokens": t, "dim": d, "tol": tol},
               x=x.reshape(t, d), residual=res.reshape(t, d), w=wt, x_after=xa.reshape(t, d),
               residual_out=ro.reshape(t, d))

    def rnd(name, dtype, add, seed, tol, line):
        t = d = 64
        x = np.zeros(t * d, F32)
        res = np.zeros(t * d, F32)
        wt = np.zeros(d, F32)
        lib.ref_rmsnorm_random_inputs(ctypes.c_uint(seed), ctypes.c_int(int(add)), ctypes.c_uint(t),
                                      ctypes.c_uint(d), P(x), P(res), P(wt))
        fixed(name, dtype, add, t, d, x, res, wt, tol, line)

    small4 = np.array([1.0, 0.0, -1.0, 2.0, 3.0, 1.0, -2.0, 0.5, 0.0, 0.0, 0.0, 0.0, -0.5, -1.5, 2.5, -3.5], F32)
    for dtype, base, lines in (("f32", "RMSNormTest", (170, 182, 206, 218, 234)),
                               ("f16", "RMSNormHalfTest", (350, 362, 386, None, 398))):
        tols = (1e-4, 1e-4, 1e-4, 1e-4, 1e-3) if dtype == "f32" else (1e-3, 2e-2, 1e-3, None, 1e-2)
        fixed(f"{base}.SingleTokenUnitWeights", dtype, False, 1, 8, x8, np.zeros(8, F32), np.ones(8, F32),
              tols[0], lines[0])
        fixed(f"{base}.MultipleTokensWithWeights", dtype, False, 3, 16, x_rows3, np.zeros(48, F32), w16, tols[1],
              lines[1])
        fixed(f"{base}.ConstantInputAndWeights", dtype, False, 5, 32, np.full(160, 2.0, F32), np.zeros(160, F32),
              np.full(32, 0.5, F32), tols[2], lines[2])
        if lines[3]:
            fixed(f"{base}.SmallDimMultipleOfVecLen", dtype, False, 4, 4, small4, np.zeros(16, F32),
                  np.array([0.5, 1.0, 1.5, 2.0], F32), tols[3], lines[3])
        rnd(f"{base}.LargeBatchRandomValues", dtype, False, 42, tols[4], lines[4])
    for dtype, base, lines in (("f32", "FusedAddResidualRMSNormTest", (261, 274, 307, 322)),
                               ("f16", "FusedAddResidualRMSNormHalfTest", (425, 438, None, 471))):
        tols = (1e-4, 1e-4, 1e-4, 1e-3) if dtype == "f32" else (1e-3, 5e-2, None, 1e-2)
        fixed(f"{base}.SingleToken", dtype, True, 1, 8, x8, res8, np.ones(8, F32), tols[0], lines[0])
        fixed(f"{base}.MultipleTokensWithWeights", dtype, True, 3, 16, x_rows3, res_rows3, w16, tols[1], lines[1])
        if lines[2]:
            fixed(f"{base}.ResidualCancelsX", dtype, True, 2, 8, np.full(16, 1.5, F32), np.full(16, -1.5, F32),
                  np.full(8, 2.0, F32), tols[2], lines[2])
        rnd(f"{base}.LargeBatchRandomValues", dtype, True, 123 if dtype == "f32" else 456, tols[3], lines[3])
    w.save()


def gen_rope_decode(lib):
    w = Writer("rope_decode")
    generic = [
        # name, B, Hq, Hkv, hd, S, is_done, kv_lens, (mod, mul, sub), line
        ("BasicTwoSequences", 2, 4, 2, 64, 64, [0, 0], [3, 6], (17, 0.1, 0.8), 102),
        ("FirstDecodeStep", 1, 8, 4, 32, 32, [0], [1], (0, 0.005, 0.5), 159),
        ("WithDoneSequences", 4, 8, 4, 64, 64, [0, 1, 0, 1], [4, 9, 15, 20], (23, 0.05, 0.5), 216),
        ("LargeBatchLoopOverGrid", 300, 4, 2, 64, 128, [0] * 300, [(i % 63) + 1 for i in range(300)],
         (31, 0.03, 0.4), 273),
        ("LoopOverHeads", 2, 16, 8, 64, 64, [0, 0], [5, 10], (19, 0.07, 0.6), 333),
    ]
    llama2 = [
        ("BasicTwoSequences", 2, 4, 2, 128, 64, [0, 0], [3, 6], (17, 0.1, 0.8), 103),
        ("FirstDecodeStep", 1, 8, 4, 128, 32, [0], [1], (0, 0.005, 0.5), 160),
        ("WithDoneSequences", 4, 8, 4, 128, 64, [0, 1, 0, 1], [4, 9, 15, 20], (23, 0.05, 0.5), 217),
        ("LargeBatchLoopOverGrid", 300, 4, 2, 128, 128, [0] * 300, [(i % 63) + 1 for i in range(300)],
         (31, 0.03, 0.4), 274),
    ]
    for pairing, table, fname in ((0, generic, "test_fused_reshape_rope_kvcache_decode.cu"),
                                  (1, llama2, "test_fused_reshape_rope_kvcache_llama2_decode.cu")):
        for name, b, hq, hkv, hd, s, done, kvl, pat, line in table:
            inp = pattern(b * (hq + 2 * hkv) * hd, *pat)
            done = np.array(done, np.uint8)
            kvl = np.array(kvl, U32)
            q = np.zeros(b * hq * hd, F32)
            k = np.zeros(b * hkv * s * hd, F32)
            v = np.zeros(b * hkv * s * hd, F32)
            if pairing == 0:
                lib.ref_rope_kvcache_decode(P(inp), P(done), P(kvl), *(ctypes.c_uint(x) for x in (b, hq, hkv, hd, s)),
                                            P(q), P(k), P(v))
            else:
                lib.ref_rope_kvcache_llama2_decode(P(inp), P(done), P(kvl), *(ctypes.c_uint(x) for x in (b, hq, hkv, s)),
                                                   P(q), P(k), P(v))
            w.case(f"{'llama2' if pairing else 'generic'}.{name}",
                   {"line": f"{fname}:{line}", "pairing": pairing, "batch": b, "q_heads": hq, "kv_heads": hkv,
                    "head_dim": hd, "kv_cache_len": s, "tol_qk": 1e-3, "tol_v": 1e-4},
                   input=inp.reshape(b, -1), is_done=done, kv_lens=kvl, q=q.reshape(b, hq, 1, hd),
                   k=k.reshape(b, hkv, s, hd), v=v.reshape(b, hkv, s, hd))
    w.save()


def gen_rope_prefill(lib):
    w = Writer("rope_prefill")
    generic = [
        # name, B, Hq, Hkv, hd, Qc, S, q_lens, kv_lens, pattern, line
        ("BasicTwoSequences", 2, 2, 1, 8, 16, 32, [2, 3], [3, 6], (17, 0.1, 0.8), 129),
        ("SingleSequenceFirstForward", 1, 2, 2, 4, 8, 16, [3], [3], (0, 0.05, 0.5), 197),
        ("IncrementalDecoding", 3, 4, 2, 8, 8, 32, [1, 1, 1], [4, 9, 15], (23, 0.05, 0.5), 265),
    ]
    llama2 = [
        ("BasicTwoSequences", 2, 4, 2, 128, 16, 64, [2, 3], [3, 6], (17, 0.1, 0.8), 132),
        ("SingleSequenceFirstForward", 1, 8, 4, 128, 16, 32, [5], [5], (0, 0.005, 0.5), 200),
        ("IncrementalDecoding", 3, 8, 4, 128, 8, 64, [1, 1, 1], [4, 9, 15], (23, 0.05, 0.5), 268),
    ]
    for pairing, table, fname in ((0, generic, "test_fused_pad_reshape_transpose_rope_kvcache.cu"),
                                  (1, llama2, "test_fused_pad_reshape_transpose_rope_kvcache_llama2.cu")):
        for name, b, hq, hkv, hd, qc, s, ql, kvl, pat, line in table:
            ql = np.array(ql, U32)
            kvl = np.array(kvl, U32)
            t = int(ql.sum())
            unpad = np.zeros(t, U32)
            lib.ref_prefill_unpad_to_pad_idx(P(ql), ctypes.c_uint(b), ctypes.c_uint(qc), P(unpad))
            inp = pattern(t * (hq + 2 * hkv) * hd, *pat)
            q = np.zeros(b * hq * qc * hd, F32)
            k = np.zeros(b * hkv * s * hd, F32)
            v = np.zeros(b * hkv * s * hd, F32)
            if pairing == 0:
                lib.ref_rope_kvcache_prefill(P(inp), P(ql), P(kvl), P(unpad),
                                             *(ctypes.c_uint(x) for x in (t, b, hq, hkv, hd, qc, s)), P(q), P(k), P(v))
            else:
                lib.ref_rope_kvcache_llama2_prefill(P(inp), P(ql), P(kvl), P(unpad),
                                                    *(ctypes.c_uint(x) for x in (t, b, hq, hkv, qc, s)),
                                                    P(q), P(k), P(v))
            tol_qk = 1e-4 if pairing == 0 else 1e-3
            w.case(f"{'llama2' if pairing else 'generic'}.{name}",
                   {"line": f"{fname}:{line}", "pairing": pairing, "batch": b, "q_heads": hq, "kv_heads": hkv,
                    "head_dim": hd, "q_cache_len": qc, "kv_cache_len": s, "tol_qk": tol_qk, "tol_v": 1e-4},
                   input=inp.reshape(t, -1), q_lens=ql, kv_lens=kvl, unpad_to_pad=unpad,
                   q=q.reshape(b, hq, qc, hd), k=k.reshape(b, hkv, s, hd), v=v.reshape(b, hkv, s, hd))
    w.save()


def gen_integer(lib):
    w = Writer("integer")
    masks = [
        # name, q_lens, kv_lens, max_q, max_kv, Qc, S, line
        ("BasicTwoSequences", [2, 3], [4, 5], 3, 5, 3, 5, 49),
        ("EqualQueryAndKVLengths", [3, 4], [3, 4], 4, 4, 4, 4, 82),
        ("SingleToken", [1], [1], 4, 4, 4, 4, 115),
        ("IncrementalDecoding", [1, 1, 1], [3, 5, 7], 1, 8, 1, 8, 148),
        ("LargeBatchRandomLengths", [(i % 16) + 1 for i in range(32)],
         [(i % 16) + 1 + (i % 17) for i in range(32)], 16, 32, 16, 32, 182),
        ("CacheLargerThanActual", [2, 3], [4, 5], 3, 5, 4, 6, 221),
    ]
    for name, ql, kvl, mq, mkv, qc, s, line in masks:
        ql, kvl = np.array(ql, U32), np.array(kvl, U32)
        b = ql.size
        m = np.zeros(b * qc * s, np.uint8)
        lib.ref_build_causal_mask(P(ql), P(kvl), ctypes.c_uint(b), ctypes.c_uint(mq), ctypes.c_uint(mkv),
                                  ctypes.c_uint(qc), ctypes.c_uint(s), P(m))
        w.case(f"mask.{name}", {"line": f"test_build_causal_mask.cu:{line}", "max_q": mq, "max_kv": mkv,
                                "q_cache_len": qc, "kv_cache_len": s},
               q_lens=ql, kv_lens=kvl, mask=m.reshape(b, qc, s))
    maps = [
        ("BasicTwoSequences", 5, [2, 3], 39),
        ("SingleTokenSingleSequence", 4, [1], 77),
        ("UnequalLengths", 8, [1, 4, 2, 3], 106),
        ("LargeBatch", 16, [(i % 16) + 1 for i in range(32)], 144),
    ]
    for name, qc, lens, line in maps:
        lens = np.array(lens, U32)
        t = int(lens.sum())
        u = np.zeros(t, U32)
        o = np.zeros(lens.size, U32)
        lib.ref_build_padding_index_maps(P(lens), ctypes.c_uint(lens.size), ctypes.c_uint(qc), P(u), P(o))
        w.case(f"maps.{name}", {"line": f"test_build_padding_index_maps.cu:{line}", "q_cache_len": qc},
               seq_lens=lens, unpad_to_pad=u, seq_offsets=o)
    lens_cases = [
        ("BasicTwoSequences", [2, 3], [4, 5], 33),
        ("SingleSequence", [3], [7], 71),
        ("FirstTokenZeroKVCache", [2, 5, 3], [0, 0, 0], 105),
        ("IncrementalDecoding", [1, 1, 1, 1], [3, 5, 7, 2], 144),
        ("LargeBatch", [(i % 8) + 1 for i in range(64)], [(i % 16) * 2 for i in range(64)], 183),
    ]
    for name, ql, kvl, line in lens_cases:
        ql, kvl = np.array(ql, U32), np.array(kvl, U32)
        out = np.zeros_like(kvl)
        mq, mkv = ctypes.c_uint(), ctypes.c_uint()
        lib.ref_update_q_kv_lens(P(ql), P(kvl), ctypes.c_uint(ql.size), P(out), ctypes.byref(mq), ctypes.byref(mkv))
        w.case(f"lens.{name}", {"line": f"test_update_q_kv_lens.cu:{line}"},
               q_lens=ql, kv_lens=kvl, kv_lens_out=out, max_q=np.array(mq.value, U32),
               max_kv=np.array(mkv.value, U32))
    # Pointer-array cases (test_build_q_k_v_qk_qkv_array.cu:133-207). The test
    # computes expectations inline (:84-130); the fixture stores the case
    # shapes, and the expectation is recomputed from them.
    ptr_cases = [
        ("MhaSingleBatch", 1, 4, 4, 8, 16, 32, 4, 133),
        ("GqaSingleBatch", 1, 8, 2, 4, 8, 16, 4, 144),
        ("GqaMultiBatch", 3, 6, 2, 4, 10, 8, 4, 155),
        ("ManyQueryHeadsPerKvHead", 2, 64, 1, 2, 4, 8, 4, 165),
        ("ManyKvHeads", 2, 64, 64, 2, 4, 8, 4, 176),
        ("LargeBatch", 300, 4, 2, 4, 8, 16, 4, 187),
        ("HalfPrecision", 2, 8, 2, 4, 8, 16, 2, 198),
    ]
    for name, b, hq, hkv, qc, s, hs, es, line in ptr_cases:
        w.case(f"ptr.{name}", {"line": f"test_build_q_k_v_qk_qkv_array.cu:{line}", "batch": b, "q_heads": hq,
                               "kv_heads": hkv, "q_cache_len": qc, "kv_cache_len": s, "head_size": hs,
                               "elem_size": es}, dummy=np.zeros(1, np.uint8))
    w.save()


def gen_linear(lib):
    w = Writer("linear")
    two_d = [((False, False, 3, 4, 5), 1e-4, 1e-2), ((True, False, 3, 4, 5), 1e-4, 1e-2),
             ((False, True, 3, 4, 5), 1e-4, 1e-2), ((True, True, 3, 4, 5), 1e-4, 1e-2),
             ((False, False, 1, 1, 1), 1e-4, None), ((False, False, 4, 6, 64), 1e-3, 2e-2)]
    batched = [((False, False, 3, 4, 5, 6), 1e-4, 1e-2), ((True, False, 2, 4, 5, 6), 1e-4, 1e-2),
               ((False, True, 2, 4, 5, 6), 1e-4, 1e-2), ((True, True, 2, 4, 5, 6), 1e-4, 1e-2),
               ((False, False, 1, 4, 5, 6), 1e-4, None), ((False, False, 32, 4, 5, 6), 1e-3, 2e-2)]
    for dtype in ("f32", "f16"):
        scale = F32(1.0 / 16.0) if dtype == "f16" else F32(1.0)
        for (ta, tb, m, n, k), tol32, tol16 in two_d:
            tol = tol32 if dtype == "f32" else tol16
            if tol is None:
                continue
            a = (((np.arange(m * k) % 7) - 3).astype(F32) * scale).astype(F32)
            bm = (((np.arange(n * k) % 5) - 2).astype(F32) * scale).astype(F32)
            c = np.zeros(m * n, F32)
            lib.ref_linear(P(a), P(bm), ctypes.c_int(ta), ctypes.c_int(tb), ctypes.c_uint(m), ctypes.c_uint(n),
                           ctypes.c_uint(k), P(c))
            w.case(f"{dtype}.2d.{int(ta)}{int(tb)}.{m}x{n}x{k}",
                   {"line": "test_linear.cu:289-406", "dtype": dtype, "batch": 0, "trans_a": ta, "trans_b": tb,
                    "M": m, "N": n, "K": k, "tol": tol},
                   A=a.reshape((k, m) if ta else (m, k)), B=bm.reshape((n, k) if tb else (k, n)),
                   C=c.reshape(m, n))
        for (ta, tb, bt, m, n, k), tol32, tol16 in batched:
            tol = tol32 if dtype == "f32" else tol16
            if tol is None:
                continue
            a = (((np.arange(bt * m * k) % 7) - 3).astype(F32) * scale).astype(F32)
            bm = (((np.arange(bt * n * k) % 5) - 2).astype(F32) * scale).astype(F32)
            c = np.zeros(bt * m * n, F32)
            for i in range(bt):
                ai = np.ascontiguousarray(a[i * m * k:(i + 1) * m * k])
                bi = np.ascontiguousarray(bm[i * n * k:(i + 1) * n * k])
                ci = np.zeros(m * n, F32)
                lib.ref_linear(P(ai), P(bi), ctypes.c_int(ta), ctypes.c_int(tb), ctypes.c_uint(m), ctypes.c_uint(n),
                               ctypes.c_uint(k), P(ci))
                c[i * m * n:(i + 1) * m * n] = ci
            w.case(f"{dtype}.batched.{int(ta)}{int(tb)}.{bt}x{m}x{n}x{k}",
                   {"line": "test_linear.cu:289-406", "dtype": dtype, "batch": bt, "trans_a": ta, "trans_b": tb,
                    "M": m, "N": n, "K": k, "tol": tol},
                   A=a.reshape((bt, k, m) if ta else (bt, m, k)), B=bm.reshape((bt, n, k) if tb else (bt, k, n)),
                   C=c.reshape(bt, m, n))
    w.save()


def gen_score(lib):
    w = Writer("score")

    def tri(b, qc, s, ql, mkv):
        m = np.zeros((b, qc, s), np.uint8)
        for si in range(b):
            for qi in range(ql[si] if ql else qc):
                for ki in range(min(qi + 1, mkv)):
                    m[si, qi, ki] = 1
        return m

    cases = []
    cases.append(("BasicAllValidFloat", "f32", 1, 1, 4, 4, 4, 4, 8, [4], np.ones((1, 4, 4), np.uint8), 1e-5, 191))
    cases.append(("PartialMaskFloat", "f32", 1, 2, 4, 6, 4, 6, 16, [4], tri(1, 4, 6, None, 6), 1e-5, 214))
    m = np.zeros((3, 8, 8), np.uint8)
    for si, ql in enumerate([3, 6, 2]):
        for qi in range(ql):
            m[si, qi, 0::2] = 1
    cases.append(("BatchWithPaddingFloat", "f32", 3, 2, 8, 8, 6, 8, 32, [3, 6, 2], m, 1e-4, 246))
    cases.append(("AllMaskedFloat", "f32", 2, 2, 4, 4, 4, 4, 8, [4, 4], np.zeros((2, 4, 4), np.uint8), 1e-6, 284))
    m = np.zeros((1, 4, 8), np.uint8)
    m[0, :, :5] = 1
    cases.append(("MaxKVSsmallerThanKVCacheFloat", "f32", 1, 1, 4, 8, 4, 5, 8, [4], m, 1e-5, 307))
    cases.append(("BasicHalf", "f16", 2, 4, 4, 4, 4, 4, 16, [3, 4], tri(2, 4, 4, [3, 4], 4), 1e-3, 338))
    cases.append(("SingleTokenFloat", "f32", 1, 1, 1, 1, 1, 1, 8, [1], np.ones((1, 1, 1), np.uint8), 1e-5, 372))
    for name, dtype, b, h, qc, s, mq, mkv, hd, ql, mask, tol, line in cases:
        n = b * h * qc * s
        ql = np.array(ql, U32)
        valid = np.zeros((b, h, qc, s), bool)
        for si in range(b):
            valid[si, :, :ql[si], :mkv] = True
        if dtype == "f32":
            qk = np.zeros(n, F32)
            lib.ref_fill_random_qk_f32(P(qk), ctypes.c_uint(n))
            qk = np.where(valid.reshape(-1), qk, F32(0)).astype(F32)
            exp = np.zeros(n, F32)
            lib.ref_masked_attention_score_f32(P(qk), P(mask), P(ql), *(ctypes.c_uint(x) for x in (b, h, qc, s, mkv, hd)),
                                               P(exp))
        else:
            qk = np.zeros(n, np.uint16)
            lib.ref_fill_random_qk_f16(P(qk), ctypes.c_uint(n))
            qk = np.where(valid.reshape(-1), qk, np.uint16(0)).astype(np.uint16)
            exp = np.zeros(n, np.uint16)
            lib.ref_masked_attention_score_f16(P(qk), P(mask), P(ql), *(ctypes.c_uint(x) for x in (b, h, qc, s, mkv, hd)),
                                               P(exp))
            qk = qk.view(np.float16)
            exp = exp.view(np.float16)
        w.case(name, {"line": f"test_compute_masked_attention_score.cu:{line}", "dtype": dtype, "batch": b,
                      "q_heads": h, "q_cache_len": qc, "kv_cache_len": s, "max_q": mq, "max_kv": mkv,
                      "head_dim": hd, "tol": tol},
               qk=qk.reshape(b, h, qc, s), mask=mask, q_lens=ql, expected=exp.reshape(b, h, qc, s))
    w.save()


def gen_swiglu(lib):
    w = Writer("swiglu")
    single = np.array([0.0, 1.0, -1.0, 2.0, -2.0, 0.5, -0.5, 1.5, 1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0], F32)
    multi = np.concatenate([np.concatenate([pattern(16, 0, 0.1, 0.8), np.arange(1, 17, dtype=F32)])
                            for _ in range(3)])
    for dtype, base, lines, seed in (("f32", "SwiGLUTest", (136, 149, 167), 42),
                                     ("f16", "SwiGLUHalfTest", (186, 198, 216), 123)):
        tols = (1e-4, 1e-4, 1e-3) if dtype == "f32" else (1e-2, 1e-2, 1e-2)
        rnd = np.zeros(64 * 128, F32)
        lib.ref_swiglu_random_inputs(ctypes.c_uint(seed), ctypes.c_uint(rnd.size), P(rnd))
        for (name, t, f, inp), tol, line in zip((("SingleToken", 1, 8, single), ("MultipleTokens", 3, 16, multi),
                                                 ("LargeBatchRandomValues", 64, 64, rnd)), tols, lines):
            out = np.zeros(t * f, F32)
            lib.ref_swiglu(P(inp), ctypes.c_uint(t), ctypes.c_uint(f), P(out))
            w.case(f"{base}.{name}", {"line": f"test_swiglu.cu:{line}", "dtype": dtype, "tol": tol},
                   input=inp.reshape(t, 2 * f), out=out.reshape(t, f))
    w.save()


def gen_unpad(lib):
    """test_fused_transpose_unpad.cu: the index map from the reference helper
    compute_unpad_to_pad_idx (:78-93), the input pattern of the runner
    (:115-117, i % 53 * 0.1 - 1, rounded through half for the half case), and
    the expected rows of the runner's inline loop (:148-167), restated here
    because that loop is not a callable helper."""
    w = Writer("unpad")
    cases = [("BasicTwoSequences", 3, 4, 16, 16, [2, 5, 3], "f32", 180),
             ("SingleSequence", 1, 2, 8, 16, [6], "f32", 192),
             ("IncrementalDecoding", 4, 2, 8, 16, [1, 1, 1, 1], "f32", 204),
             ("LargerHeadDim", 2, 2, 32, 64, [7, 9], "f32", 217),
             ("HalfBasic", 2, 2, 8, 16, [3, 4], "f16", 233)]
    for name, b, h, qc, hd, q_lens, dtype, line in cases:
        q_lens = np.array(q_lens, U32)
        t = int(q_lens.sum())
        idx = np.zeros(b * qc, U32)
        lib.ref_unpad_to_pad_idx(P(q_lens), ctypes.c_uint(b), ctypes.c_uint(qc), P(idx))
        qkv = pattern(b * h * qc * hd, 53, 0.1, 1.0)
        if dtype == "f16":
            qkv = qkv.astype(np.float16).astype(F32)
        qkv = qkv.reshape(b, h, qc, hd)
        out = np.zeros((t, h * hd), F32)
        off = 0
        for s, n in enumerate(q_lens):
            for i in range(int(n)):
                out[off + i] = qkv[s, :, i, :].reshape(-1)
            off += int(n)
        w.case(f"unpad.{name}", {"line": f"test_fused_transpose_unpad.cu:{line}", "dtype": dtype,
                                 "num_input_tokens": t},
               q_lens=q_lens, unpad_to_pad=idx.reshape(b, qc), qkv=qkv, out=out)
    w.save()


def gen_attention_qkv(lib):
    """P.V at the launch_linear call site (trans_A = trans_B = false): per
    (b, q head) the reference helper compute_expected_linear
    (test_linear.cu:78-108) on the slice qk[b, h, :m, :n] x v[b, h / g, :n, :].
    The shapes are the decode and prefill call sites with grouped heads."""
    w = Writer("attention_qkv")
    rng = np.random.default_rng(7)
    cases = [("decode_mha", 2, 3, 3, 1, 40, 16, 1, 33),
             ("decode_gqa", 2, 4, 2, 1, 64, 32, 1, 64),
             ("prefill_gqa", 1, 4, 1, 8, 24, 16, 5, 20),
             ("prefill_full", 2, 2, 2, 6, 12, 8, 6, 12)]
    for name, b, hq, hkv, qc, s, hd, m, n in cases:
        qk = rng.random((b, hq, qc, s), dtype=F32)
        v = rng.standard_normal((b, hkv, s, hd), dtype=F32)
        out = np.full((b, hq, qc, hd), -7.0, F32)
        g = hq // hkv
        for bi in range(b):
            for h in range(hq):
                a_s = np.ascontiguousarray(qk[bi, h, :m, :n])
                b_s = np.ascontiguousarray(v[bi, h // g, :n, :])
                c = np.zeros((m, hd), F32)
                lib.ref_linear(P(a_s), P(b_s), 0, 0, ctypes.c_uint(m), ctypes.c_uint(hd), ctypes.c_uint(n), P(c))
                out[bi, h, :m] = c
        w.case(name, {"line": "test_linear.cu:78-108", "m": m, "n": n}, qk=qk, v=v, qkv=out)
    w.save()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", default=None, help="the reference sources (default: oracle.reference_root())")
    args = ap.parse_args()
    oracle.build_ref(args.ref_root)
    lib = oracle.ref_lib()
    if lib is None:
        sys.exit("reference helpers are not built; the reference sources are needed")
    for fn in (gen_embedding, gen_rmsnorm, gen_rope_decode, gen_rope_prefill, gen_integer, gen_linear, gen_score,
               gen_swiglu, gen_unpad, gen_attention_qkv):
        fn(lib)


if __name__ == "__main__":
    main()
