"""ctypes binding of the C ABI in include/llama2_b200.h.

Loads llama2_b200/libllama2_b200.so (built by ``python -m llama2_b200.build``)
and declares every entry point's argument types. There is no fallback: if
the library is missing, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "libllama2_b200.so")

L2K_F32, L2K_F16, L2K_BF16 = 0, 1, 2
L2K_ROPE_INTERLEAVED, L2K_ROPE_HALF = 0, 1
STATUS = {0: "ok", 1: "invalid argument", 2: "unsupported dtype", 3: "unsupported shape", 4: "CUDA error"}

vp = ctypes.c_void_p
i64 = ctypes.c_int64
u32 = ctypes.c_uint32
cint = ctypes.c_int
f32 = ctypes.c_float


class DecodeStepArgs(ctypes.Structure):
    """l2k_decode_step_args (include/llama2_b200.h), field for field."""
    _fields_ = [
        ("q_lens", vp), ("kv_lens", vp), ("max_lens", vp),
        ("input_ids", vp), ("embed_table", vp), ("norm_weight", vp), ("x", vp), ("normed", vp),
        ("qkv", vp), ("is_done", vp), ("q", vp), ("k_cache", vp), ("v_cache", vp), ("qk", vp),
        ("rope_table", vp), ("rope_table_positions", i64),
        ("gate_up", vp), ("ffn_out", vp),
        ("batch", i64), ("vocab_size", i64), ("dim", i64), ("q_head_num", i64), ("kv_head_num", i64),
        ("head_dim", i64), ("kv_cache_len", i64), ("hidden", i64),
        ("pairing", cint), ("dtype", cint),
    ]


# name -> argument types (restype int unless noted)
SIGNATURES = {
    "l2k_status_string": ([cint], ctypes.c_char_p),
    "l2k_last_error_message": ([], ctypes.c_char_p),
    "l2k_abi_version": ([], cint),
    "l2k_embedding": [vp, i64, vp, i64, i64, vp, cint, vp],
    "l2k_fused_add_residual_rmsnorm": [vp, vp, vp, i64, i64, cint, cint, vp],
    "l2k_rope_table_floats": ([i64, i64], i64),
    "l2k_rope_table_fill": [vp, i64, i64],
    "l2k_fused_reshape_rope_kvcache_decode": [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, vp, i64, cint, vp],
    "l2k_fused_reshape_rope_kvcache_llama2_decode": [vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, vp, i64, cint,
                                                     vp],
    "l2k_fused_pad_reshape_transpose_rope_kvcache": [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, vp,
                                                     i64, cint, vp],
    "l2k_fused_pad_reshape_transpose_rope_kvcache_llama2": [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64,
                                                            i64, vp, i64, cint, vp],
    "l2k_update_q_kv_lens": [vp, vp, i64, vp, vp, vp],
    "l2k_build_causal_mask": [u32, u32, vp, vp, vp, i64, i64, i64, vp],
    "l2k_build_padding_index_maps": [i64, vp, i64, i64, vp, vp, vp],
    "l2k_build_q_k_v_qk_qkv_array": [ctypes.POINTER(vp), ctypes.POINTER(i64), i64, i64, i64, i64, ctypes.POINTER(vp),
                                     vp],
    "l2k_linear": [cint, cint, i64, i64, i64, vp, i64, vp, i64, vp, i64, i64, vp, vp, vp, cint, vp],
    "l2k_qk_scores": [vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, cint, vp],
    "l2k_attention_qkv": [vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i64, cint, vp],
    "l2k_compute_masked_attention_score": [i64, u32, u32, vp, vp, vp, i64, i64, i64, i64, cint, vp],
    "l2k_swiglu": [vp, vp, i64, i64, cint, vp],
    "l2k_linear_swiglu": [cint, i64, i64, i64, vp, i64, vp, i64, vp, i64, cint, vp],
    "l2k_linear_rope_kvcache_decode": [cint, vp, i64, vp, i64, i64, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64,
                                       vp, i64, cint, cint, vp],
    "l2k_linear_pad_rope_kvcache_prefill": [cint, vp, i64, vp, i64, i64, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64,
                                            i64, i64, i64, vp, i64, cint, cint, vp],
    "l2k_fused_transpose_unpad": [i64, vp, vp, vp, i64, i64, i64, i64, cint, vp],
    "l2k_decode_attention_scores": [vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, cint, vp],
    "l2k_decode_attention": [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, cint, vp],
    "l2k_paged_block_rows": ([i64, cint], i64),
    "l2k_fused_reshape_rope_kvcache_paged_decode": [vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64,
                                                    vp, i64, cint, cint, vp],
    "l2k_decode_attention_paged": [vp, vp, vp, vp, i64, i64, vp, vp, vp, vp, i64, i64, i64, i64, cint, vp],
    "l2k_prefill_attention_scores": [vp, vp, vp, vp, u32, u32, vp, i64, i64, i64, i64, i64, i64, cint, vp],
    "l2k_fused_pad_reshape_transpose_rope_kvcache_paged": [vp, vp, vp, vp, vp, vp, vp, vp, i64, i64, i64, i64, i64,
                                                           i64, i64, i64, i64, vp, i64, cint, cint, vp],
    "l2k_prefill_attention_scores_paged": [vp, vp, vp, i64, i64, vp, vp, u32, u32, vp, i64, i64, i64, i64, i64, cint,
                                           vp],
    "l2k_attention_qkv_paged": [vp, vp, vp, i64, i64, vp, vp, i64, i64, i64, i64, i64, i64, i64, cint, vp],
    "l2k_fused_reshape_rope_kvcache_fp8_decode": [vp, vp, vp, vp, vp, vp, f32, f32, i64, i64, i64, i64, i64, vp, i64,
                                                  cint, cint, vp],
    "l2k_decode_attention_fp8": [vp, vp, vp, f32, f32, vp, vp, vp, vp, i64, i64, i64, i64, i64, cint, vp],
    "l2k_decode_attention_fp8_paged": [vp, vp, vp, f32, f32, vp, i64, i64, vp, vp, vp, vp, i64, i64, i64, i64, cint,
                                       vp],
    "l2k_decode_step_workspace_bytes": ([], i64),
    "l2k_decode_step_supported": [ctypes.POINTER(DecodeStepArgs)],
    "l2k_decode_step": [ctypes.POINTER(DecodeStepArgs), vp, vp],
    "l2k_decode_step_attention": [ctypes.POINTER(DecodeStepArgs), vp, vp, vp],
    "l2k_decode_step_paged": [ctypes.POINTER(DecodeStepArgs), vp, i64, i64, vp, vp],
    "l2k_decode_step_attention_paged": [ctypes.POINTER(DecodeStepArgs), vp, i64, i64, vp, vp, vp],
    "l2k_decode_step_attention_no_alloc": [ctypes.POINTER(DecodeStepArgs), vp, vp],
    "l2k_decode_step_no_alloc": [ctypes.POINTER(DecodeStepArgs), vp],
    "l2k_device_error": ([cint], cint),
}

_lib = None


class L2KError(RuntimeError):
    def __init__(self, name, status, message):
        super().__init__(f"{name}: {STATUS.get(status, status)}: {message}")
        self.status = status


def lib() -> ctypes.CDLL:
    """The loaded kernel library; raises if it was not built."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing; build it with `python -m llama2_b200.build`")
        handle = ctypes.CDLL(LIB_PATH)
        for name, sig in SIGNATURES.items():
            fn = getattr(handle, name)
            if isinstance(sig, tuple):
                fn.argtypes, fn.restype = sig
            else:
                fn.argtypes, fn.restype = sig, cint
        _lib = handle
    return _lib


def call(name: str, *args) -> None:
    """Calls an int-returning entry point and raises L2KError on failure."""
    status = getattr(lib(), name)(*args)
    if status != 0:
        raise L2KError(name, status, lib().l2k_last_error_message().decode())


def exported_names():
    return list(SIGNATURES)
