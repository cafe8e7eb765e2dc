"""The C-ABI library on the CPU: it loads, exports every entry point that
include/llama2_b200.h declares, and rejects bad arguments before launching
anything (these calls never reach the GPU)."""
import ctypes
import os
import re

import numpy as np
import pytest

from llama2_b200 import capi
from oracle import port

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "llama2_b200.h")


def declared_names():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(l2k_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_entry_points():
    names = declared_names()
    assert "l2k_embedding" in names and "l2k_decode_attention_scores" in names
    assert len(names) >= 20


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(capi.LIB_PATH)
    missing = [n for n in declared_names() if not hasattr(lib, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert sorted(capi.exported_names()) == declared_names()


def test_status_strings():
    lib = capi.lib()
    assert lib.l2k_status_string(0) == b"ok"
    assert lib.l2k_status_string(3) == b"unsupported shape"
    assert lib.l2k_abi_version() == 1


@pytest.mark.parametrize("call,args,status", [
    ("l2k_embedding", (None, -1, None, 10, 8, None, 0, None), 1),
    ("l2k_embedding", (None, 4, None, 10, 8, None, 7, None), 1),
    ("l2k_swiglu", (None, None, 2, -4, 0, None), 1),
    ("l2k_swiglu", (None, None, 2, 4, 0, None), 1),
    ("l2k_fused_add_residual_rmsnorm", (None, None, None, 2, 8, 0, 0, None), 1),
    ("l2k_fused_reshape_rope_kvcache_decode", (None, None, None, None, None, None, 1, 2, 2, 7, 8, None, 0, 0, None), 1),
    ("l2k_build_causal_mask", (5, 2, None, None, None, 1, 4, 4, None), 1),
    ("l2k_build_padding_index_maps", (4, None, 20000, 4, None, None, None), 3),
    ("l2k_decode_attention_scores", (None, None, None, None, None, 1, 3, 2, 16, 8, 0, None), 1),
    ("l2k_prefill_attention_scores", (None, None, None, None, 9, 4, None, 1, 2, 2, 8, 8, 16, 0, None), 1),
    ("l2k_compute_masked_attention_score", (16, 4, 4, None, None, None, 1, 1, 4, 4, 9, None), 1),
    ("l2k_fused_transpose_unpad", (3, None, None, None, 2, 4, 8, 16, 0, None), 1),   # null pointers
    ("l2k_fused_transpose_unpad", (17, None, None, None, 2, 4, 8, 16, 0, None), 1),  # more tokens than slots
    ("l2k_fused_transpose_unpad", (1, None, None, None, 2, 4, 8, 16, 5, None), 1),   # dtype
    ("l2k_attention_qkv", (None, None, None, 2, 4, 2, 8, 16, 128, 4, 8, 2, None), 1),  # null pointers
    ("l2k_attention_qkv", (None, None, None, 2, 4, 2, 8, 16, 128, 9, 8, 2, None), 1),  # m > q_cache_len
    ("l2k_attention_qkv", (None, None, None, 2, 4, 3, 8, 16, 128, 4, 8, 2, None), 1),  # Hq % Hkv
    ("l2k_decode_attention", (None, None, None, None, None, None, None, 2, 4, 2, 64, 128, 0, None), 1),
    ("l2k_decode_attention", (None, None, None, None, None, None, None, 2, 4, 3, 64, 128, 0, None), 1),
    ("l2k_decode_attention", (None, None, None, None, None, None, None, 2, 4, 2, 64, 0, 0, None), 1),
    ("l2k_linear_swiglu", (0, 16, 8, 64, None, 64, None, 16, None, 8, 2, None), 1),  # null pointers
    ("l2k_linear_swiglu", (0, 16, 8, 64, 16, 64, 16, 8, 16, 8, 2, None), 1),        # ldb < 2 inter
    ("l2k_linear_swiglu", (0, 16, 8, 64, 16, 64, 16, 16, 16, 8, 0, None), 2),       # f32
    ("l2k_linear_rope_kvcache_decode", (0, None, 64, None, 512, 64, None, None, None, None, None, 2, 2, 1, 128,
                                        16, None, 0, 1, 2, None), 1),                  # null pointers
    ("l2k_linear_rope_kvcache_decode", (0, 16, 64, 16, 512, 64, 16, 16, 16, 16, 16, 2, 2, 1, 128,
                                        16, None, 0, 7, 2, None), 1),                  # pairing
    ("l2k_linear_pad_rope_kvcache_prefill", (0, 16, 64, 16, 512, 64, 16, 16, 16, 16, 16, 16, 5, 2, 2, 1, 128,
                                             0, 16, None, 0, 1, 2, None), 1),          # q_cache_len 0
])
def test_bad_arguments_are_rejected(call, args, status):
    with pytest.raises(capi.L2KError) as e:
        capi.call(call, *args)
    assert e.value.status == status
    assert capi.lib().l2k_last_error_message()


def test_empty_inputs_are_noops():
    # Zero-sized work returns before touching any pointer or the device.
    capi.call("l2k_embedding", None, 0, None, 10, 8, None, 0, None)
    capi.call("l2k_swiglu", None, None, 0, 16, 2, None)
    capi.call("l2k_fused_add_residual_rmsnorm", None, None, None, 0, 64, 1, 1, None)
    capi.call("l2k_fused_transpose_unpad", 0, None, None, None, 2, 4, 8, 16, 1, None)
    capi.call("l2k_attention_qkv", None, None, None, 0, 4, 2, 8, 16, 128, 4, 8, 2, None)
    capi.call("l2k_decode_attention", None, None, None, None, None, None, None, 0, 4, 2, 64, 128, 2, None)


@pytest.mark.parametrize("hd", [2, 4, 48, 64, 128])
def test_rope_table_matches_oracle_bitwise(hd):
    n_pos = 512
    n = capi.lib().l2k_rope_table_floats(hd, n_pos)
    assert n == n_pos * hd
    t = np.zeros(n, np.float32)
    capi.call("l2k_rope_table_fill", t.ctypes.data, hd, n_pos)
    t = t.reshape(n_pos, hd // 2, 2)
    for pos in range(0, n_pos, 37):
        for i in range(hd // 2):
            c, s = port.rope_cos_sin(i, hd, pos, pos + 1)
            assert t[pos, i, 0] == np.float32(c) and t[pos, i, 1] == np.float32(s), (pos, i)


def _step_args(**over):
    """l2k_decode_step_args with fake 16-byte aligned (never dereferenced) pointers."""
    a = capi.DecodeStepArgs()
    for i, (name, typ) in enumerate(capi.DecodeStepArgs._fields_):
        if typ is capi.vp:
            setattr(a, name, 0x10000 + 0x100 * i)
    a.batch, a.vocab_size, a.dim, a.q_head_num, a.kv_head_num = 1, 32000, 4096, 32, 32
    a.head_dim, a.kv_cache_len, a.hidden, a.pairing, a.dtype = 128, 4096, 11008, 1, 0
    a.rope_table_positions = 4096
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,status", [
    (dict(head_dim=48), 3),               # 192-byte K rows: not a streaming row size
    (dict(head_dim=96, dtype=2), 3),      # 192-byte rows in bf16
    (dict(dim=4094), 3),                  # dim not a multiple of 16 bytes
    (dict(qkv=0x10008), 3),               # misaligned tensor
    (dict(kv_head_num=5), 1),             # q_head_num not a multiple of kv_head_num
    (dict(head_dim=127), 1),              # odd head_dim
    (dict(dtype=9), 1),
    (dict(pairing=2), 1),
    (dict(kv_lens=None), 1),
    (dict(normed=0x10000, x=0x10000), 1), # x and normed alias
])
def test_decode_step_rejects_before_launch(over, status):
    assert capi.lib().l2k_decode_step_supported(ctypes.byref(_step_args(**over))) == status
    assert capi.lib().l2k_last_error_message()


def test_decode_step_null_args_and_workspace():
    assert capi.lib().l2k_decode_step(None, None, None) == 1
    assert capi.lib().l2k_decode_step(ctypes.byref(_step_args()), None, None) == 1
    assert capi.lib().l2k_decode_step_workspace_bytes() >= 4


def test_decode_step_empty_batch_is_noop():
    ws = np.zeros(4, np.uint32)
    assert capi.lib().l2k_decode_step(ctypes.byref(_step_args(batch=0)), ws.ctypes.data, None) == 0
