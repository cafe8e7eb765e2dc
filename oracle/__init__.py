"""CPU oracle for the fused Llama-2 layer-kernel path — TEST INFRASTRUCTURE ONLY.

Two oracles live here, both used only by ``tests/``, ``__graft_entry__.smoke()``
and the ``cpu_baseline`` / ``--impl reference`` legs of ``bench.py``:

* ``port`` — ``oracle.c``: a plain-C restatement of the reference's CPU test
  helpers (``test/kernel/*.cu`` in pentatracy5/llama2), built into
  ``liboracle.so``. It is the checker every CUDA kernel is compared against.
* ``ref``  — ``_ref/libref_oracle.so``: the reference's own CPU test helpers,
  compiled from the reference's test sources where they lie (``make ref``),
  exposed through ``ref_glue/``. It pins ``port`` (and generated the golden
  fixtures under ``tests/golden/``). It is absent wherever the reference
  sources are absent; ``ref_available()`` says whether it loaded.

Nothing in the product package imports this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_PORT_SO = os.path.join(_HERE, "liboracle.so")
_REF_SO = os.path.join(_HERE, "_ref", "libref_oracle.so")

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_u32 = ctypes.c_uint32
_int = ctypes.c_int


def _ptr(a: np.ndarray) -> ctypes.c_void_p:
    assert a.flags["C_CONTIGUOUS"], "oracle inputs must be C-contiguous"
    return ctypes.c_void_p(a.ctypes.data)


def _load_port() -> ctypes.CDLL:
    if not os.path.exists(_PORT_SO):
        subprocess.run(["make", "-s", "-C", _HERE, "liboracle.so"], check=True)
    lib = ctypes.CDLL(_PORT_SO)
    for name in [n for n in dir(lib) if n.startswith("orc_")]:
        getattr(lib, name).restype = None
    return lib


_port = None
_ref = None


def port_lib() -> ctypes.CDLL:
    global _port
    if _port is None:
        _port = _load_port()
    return _port


def ref_lib():
    """The reference's own helpers, or None when they were not built here."""
    global _ref
    if _ref is None and os.path.exists(_REF_SO):
        _ref = ctypes.CDLL(_REF_SO)
    return _ref


def ref_available() -> bool:
    return ref_lib() is not None


def reference_root() -> str:
    """Where the reference sources are: $L2K_REFERENCE_ROOT when set, else a
    checkout named "reference" beside this repository."""
    return os.environ.get("L2K_REFERENCE_ROOT") or os.path.join(os.path.dirname(os.path.dirname(_HERE)), "reference")


def build_ref(ref_root: str | None = None) -> bool:
    """Compile the reference helpers when the reference sources are present."""
    ref_root = ref_root or reference_root()
    if not os.path.isdir(ref_root):
        return False
    subprocess.run(["make", "-s", "-C", _HERE, "ref", f"REF_ROOT={ref_root}"], check=True)
    return True


def f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


def u32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint32)


def u8(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.uint8)


class port:
    """numpy front end of oracle.c (the restated reference helpers)."""

    @staticmethod
    def embedding(ids, table):
        ids = u32(ids)
        table = np.ascontiguousarray(table)
        out = np.empty((ids.shape[0], table.shape[1]), dtype=table.dtype)
        port_lib().orc_embedding(_ptr(ids), _i64(ids.shape[0]), _ptr(table), _i64(table.shape[1]),
                                 _i64(table.itemsize), _ptr(out))
        return out

    @staticmethod
    def fused_add_residual_rmsnorm(x, residual, w, add_residual):
        x, residual, w = f32(x), f32(residual), f32(w)
        t, d = x.shape
        x_after = np.empty_like(x)
        res_out = np.empty_like(x)
        port_lib().orc_fused_add_residual_rmsnorm(_ptr(x), _ptr(residual), _ptr(w), _i64(t), _i64(d),
                                                  _int(int(add_residual)), _ptr(x_after), _ptr(res_out))
        return x_after, res_out

    @staticmethod
    def rope_cos_sin(i, head_dim, pos, seq_len):
        c, s = ctypes.c_float(), ctypes.c_float()
        port_lib().orc_rope_cos_sin(_u32(i), _u32(head_dim), _u32(pos), _u32(seq_len), ctypes.byref(c),
                                    ctypes.byref(s))
        return c.value, s.value

    @staticmethod
    def rotate_one_head(pairing, head, pos, seq_len):
        """One head (head_dim floats) rotated at `pos` with the length `seq_len`
        the angle's scale uses: the per-head step of rope_kvcache_decode."""
        head = f32(head)
        out = np.empty_like(head)
        port_lib().orc_rotate_one_head(_int(pairing), _ptr(head), _i64(head.shape[0]), _u32(pos), _u32(seq_len),
                                       _ptr(out))
        return out

    @staticmethod
    def rope_kvcache_decode(pairing, inp, is_done, kv_lens, q, k, v):
        """In place on q, k, v (float32, [B,Hq,1,hd] / [B,Hkv,S,hd])."""
        inp, is_done, kv_lens = f32(inp), u8(is_done), u32(kv_lens)
        b, hq, _, hd = q.shape
        hkv, s = k.shape[1], k.shape[2]
        port_lib().orc_rope_kvcache_decode(_int(pairing), _ptr(inp), _ptr(is_done), _ptr(kv_lens), _i64(b),
                                           _i64(hq), _i64(hkv), _i64(hd), _i64(s), _ptr(q), _ptr(k), _ptr(v))

    @staticmethod
    def rope_kvcache_prefill(pairing, inp, q_lens, kv_lens, unpad_to_pad, q, k, v):
        """In place on q [B,Hq,Qc,hd], k, v [B,Hkv,S,hd] (float32)."""
        inp, q_lens, kv_lens, unpad_to_pad = f32(inp), u32(q_lens), u32(kv_lens), u32(unpad_to_pad)
        _, hq, qc, hd = q.shape
        hkv, s = k.shape[1], k.shape[2]
        port_lib().orc_rope_kvcache_prefill(_int(pairing), _ptr(inp), _ptr(q_lens), _ptr(kv_lens),
                                            _ptr(unpad_to_pad), _i64(inp.shape[0]), _i64(hq), _i64(hkv),
                                            _i64(hd), _i64(qc), _i64(s), _ptr(q), _ptr(k), _ptr(v))

    @staticmethod
    def update_q_kv_lens(q_lens, kv_lens):
        q_lens = u32(q_lens)
        kv = u32(kv_lens).copy()
        mq, mkv = ctypes.c_uint32(), ctypes.c_uint32()
        port_lib().orc_update_q_kv_lens(_ptr(q_lens), _ptr(kv), _i64(q_lens.shape[0]), ctypes.byref(mq),
                                        ctypes.byref(mkv))
        return kv, mq.value, mkv.value

    @staticmethod
    def build_causal_mask(q_lens, kv_lens, max_q, max_kv, mask):
        """In place on mask [B, Qc, S] u8 (reference unsigned-wrap expression)."""
        q_lens, kv_lens = u32(q_lens), u32(kv_lens)
        b, qc, s = mask.shape
        port_lib().orc_build_causal_mask(_ptr(q_lens), _ptr(kv_lens), _i64(b), _u32(max_q), _u32(max_kv),
                                         _i64(qc), _i64(s), _ptr(mask))

    @staticmethod
    def build_intended_mask(q_lens, kv_lens, max_q, max_kv, mask):
        """In place on mask [B, Qc, S] u8 (positions 0..pos)."""
        q_lens, kv_lens = u32(q_lens), u32(kv_lens)
        b, qc, s = mask.shape
        port_lib().orc_build_intended_mask(_ptr(q_lens), _ptr(kv_lens), _i64(b), _u32(max_q), _u32(max_kv),
                                           _i64(qc), _i64(s), _ptr(mask))

    @staticmethod
    def build_padding_index_maps(seq_lens, q_cache_len):
        seq_lens = u32(seq_lens)
        n_tokens = int(seq_lens.astype(np.int64).sum())
        unpad = np.zeros(max(n_tokens, 1), dtype=np.uint32)[:n_tokens]
        offs = np.zeros(seq_lens.shape[0], dtype=np.uint32)
        port_lib().orc_build_padding_index_maps(_ptr(seq_lens), _i64(seq_lens.shape[0]), _i64(q_cache_len),
                                                _ptr(unpad) if n_tokens else _c_void_p(0), _ptr(offs))
        return unpad, offs

    @staticmethod
    def build_ptr_arrays(bases, strides, batch, q_heads, kv_heads):
        bases = np.ascontiguousarray(bases, dtype=np.uint64)
        strides = np.ascontiguousarray(strides, dtype=np.uint64)
        out = np.zeros((8, batch * q_heads), dtype=np.uint64)
        port_lib().orc_build_ptr_arrays(_ptr(bases), _ptr(strides), _i64(batch), _i64(q_heads), _i64(kv_heads),
                                        _ptr(out))
        return out

    @staticmethod
    def linear(a, b, trans_a, trans_b, m, n, k):
        a, b = f32(a), f32(b)
        c = np.zeros((m, n), dtype=np.float32)
        port_lib().orc_linear(_ptr(a), _ptr(b), _int(int(trans_a)), _int(int(trans_b)), _i64(m), _i64(n), _i64(k),
                              _ptr(c))
        return c

    @staticmethod
    def qk_scores(q, k, m, n, qk):
        """In place on qk [B,Hq,Qc,S]: rows < m, keys < n."""
        q, k = f32(q), f32(k)
        b, hq, qc, hd = q.shape
        hkv, s = k.shape[1], k.shape[2]
        port_lib().orc_qk_scores(_ptr(q), _ptr(k), _i64(b), _i64(hq), _i64(hkv), _i64(qc), _i64(s), _i64(hd),
                                 _i64(m), _i64(n), _ptr(qk))

    @staticmethod
    def masked_attention_score(qk, mask, q_lens, max_kv, head_dim):
        """In place on qk [B,H,Qc,S] float32."""
        mask, q_lens = u8(mask), u32(q_lens)
        b, h, qc, s = qk.shape
        port_lib().orc_masked_attention_score(_ptr(qk), _ptr(mask), _ptr(q_lens), _i64(b), _i64(h), _i64(qc),
                                              _i64(s), _i64(max_kv), _i64(head_dim))

    @staticmethod
    def swiglu(inp):
        inp = f32(inp)
        t, two_f = inp.shape
        out = np.empty((t, two_f // 2), dtype=np.float32)
        port_lib().orc_swiglu(_ptr(inp), _i64(t), _i64(two_f // 2), _ptr(out))
        return out

    @staticmethod
    def transpose_unpad(qkv, unpad_to_pad, n_tokens):
        """qkv (B, H, Qc, hd) of any dtype -> (n_tokens, H * hd)."""
        qkv = np.ascontiguousarray(qkv)
        unpad_to_pad = u32(unpad_to_pad)
        b, h, qc, hd = qkv.shape
        out = np.empty((n_tokens, h * hd), dtype=qkv.dtype)
        if n_tokens:
            port_lib().orc_transpose_unpad(_ptr(qkv), _ptr(unpad_to_pad), _i64(n_tokens), _i64(b), _i64(h),
                                           _i64(qc), _i64(hd), _i64(qkv.dtype.itemsize), _ptr(out))
        return out

    @staticmethod
    def e4m3_from_f32(x, scale):
        """Bytes of x / scale (x * float32(1 / scale)) rounded to e4m3, saturating."""
        x = f32(x)
        inv = np.float32(1.0) / np.float32(scale)
        out = np.empty(x.shape, np.uint8)
        port_lib().orc_e4m3_from_f32(_ptr(x), _i64(x.size), ctypes.c_float(inv), _ptr(out))
        return out

    @staticmethod
    def e4m3_to_f32(b, scale):
        """The values scale * e4m3(b) of a uint8 array."""
        b = u8(b)
        out = np.empty(b.shape, np.float32)
        port_lib().orc_e4m3_to_f32(_ptr(b), _i64(b.size), ctypes.c_float(scale), _ptr(out))
        return out

    @staticmethod
    def attention_qkv(qk, v, m, n, qkv):
        """In place on qkv (B, Hq, Qc, hd) float32: rows < m, keys < n."""
        qk, v = f32(qk), f32(v)
        b, hq, qc, s = qk.shape
        hkv, hd = v.shape[1], v.shape[3]
        port_lib().orc_attention_qkv(_ptr(qk), _ptr(v), _i64(b), _i64(hq), _i64(hkv), _i64(qc), _i64(s), _i64(hd),
                                     _i64(m), _i64(n), _ptr(qkv))
