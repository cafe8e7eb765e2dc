"""Python mirror of the reference operator API (include/kernel/*.h of
pentatracy5/llama2) over torch CUDA tensors.

Each ``launch_*`` function keeps the reference function's name, argument
order and meaning; tensors replace ``Tensor<T>``. Shapes are read from the
tensors exactly as the reference's host wrappers read ``Tensor::shape()``,
and the reference's ``assert``s become ``ValueError``s raised before anything
is launched. Work is enqueued on torch's current CUDA stream through the C
ABI (llama2_b200.capi); nothing here computes on the CPU.

Integer tensors (ids, lengths, index maps) are 4-byte (torch.uint32 or
torch.int32, read as unsigned); masks and done flags are torch.uint8.
"""
from __future__ import annotations

import ctypes
import threading

import torch

from . import capi

_DT = {torch.float32: capi.L2K_F32, torch.float16: capi.L2K_F16, torch.bfloat16: capi.L2K_BF16}
_U32 = (torch.uint32, torch.int32)

ROPE_TABLE_POSITIONS = 4096  # positions covered by the host-built cos/sin table


def _code(t: torch.Tensor) -> int:
    try:
        return _DT[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def _dev(*ts):
    for t in ts:
        if not t.is_cuda:
            raise ValueError("tensors must be on a CUDA device")
        if not t.is_contiguous():
            raise ValueError("tensors must be contiguous")


def _u32(t, name):
    if t.dtype not in _U32:
        raise ValueError(f"{name} must be a 4-byte integer tensor, got {t.dtype}")


def _same(a, b, name):
    if a.dtype != b.dtype:
        raise ValueError(f"{name}: dtype mismatch {a.dtype} vs {b.dtype}")


def _require(cond, msg):
    if not cond:
        raise ValueError(msg)


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


# --------------------------------------------------------------------------
# RoPE cos/sin tables, one per (device, head_dim), built once on the host.
# --------------------------------------------------------------------------
_tables = {}
_tables_lock = threading.Lock()


def rope_table(head_dim: int, device: torch.device) -> torch.Tensor:
    key = (torch.device(device), head_dim)
    with _tables_lock:
        t = _tables.get(key)
        if t is None:
            n = capi.lib().l2k_rope_table_floats(head_dim, ROPE_TABLE_POSITIONS)
            host = torch.empty(n, dtype=torch.float32)
            capi.call("l2k_rope_table_fill", host.data_ptr(), head_dim, ROPE_TABLE_POSITIONS)
            t = host.to(device)
            _tables[key] = t
    return t


# --------------------------------------------------------------------------
# Operators
# --------------------------------------------------------------------------
def launch_embedding(input_ids, embed_table, output):
    """include/kernel/embedding.h:6-9"""
    _dev(input_ids, embed_table, output)
    _u32(input_ids, "input_ids")
    _same(embed_table, output, "launch_embedding")
    n, (vocab, dim) = input_ids.shape[0], embed_table.shape
    _require(tuple(output.shape) == (n, dim), "Incorrect output size")
    capi.call("l2k_embedding", input_ids.data_ptr(), n, embed_table.data_ptr(), vocab, dim, output.data_ptr(),
              _code(output), _stream())


def launch_fused_add_residual_rmsnorm(weights, x, residual, add_residual: bool):
    """include/kernel/fused_add_residual_rmsnorm.h:16-19 (add_residual is the template flag)."""
    _dev(weights, x, residual)
    _same(x, residual, "launch_fused_add_residual_rmsnorm")
    _same(x, weights, "launch_fused_add_residual_rmsnorm")
    n, dim = x.shape
    _require(tuple(residual.shape) == (n, dim), "Incorrect residual size")
    _require(tuple(weights.shape) == (dim,), "Incorrect rmsnorm weight size")
    capi.call("l2k_fused_add_residual_rmsnorm", weights.data_ptr(), x.data_ptr(), residual.data_ptr(), n, dim,
              int(bool(add_residual)), _code(x), _stream())


def _rope_decode(name, input, is_done, kv_lens, q, k, v, table):
    _dev(input, is_done, kv_lens, q, k, v)
    _u32(kv_lens, "kv_lens")
    for t in (q, k, v):
        _same(input, t, name)
    b, hq, one, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    _require(hd % 2 == 0, "Head dim should be even")
    _require(k.shape[3] == hd and v.shape[3] == hd, "Head dim of q k v do not match")
    _require(v.shape[1] == hkv, "Head num of k v do not match")
    _require(input.shape[1] == (hq + 2 * hkv) * hd, "Incorrect embedding dim")
    _require(input.shape[0] == b and is_done.shape[0] == b and kv_lens.shape[0] == b, "Incorrect batch size")
    _require(k.shape[0] == b and v.shape[0] == b, "Batch size of k v do not match")
    _require(one == 1, "Incorrect q cache length")
    _require(v.shape[2] == s, "k v cache length do not match")
    tab = rope_table(hd, q.device) if table else None
    capi.call(name, input.data_ptr(), is_done.data_ptr(), kv_lens.data_ptr(), q.data_ptr(), k.data_ptr(),
              v.data_ptr(), b, hq, hkv, hd, s, tab.data_ptr() if tab is not None else None,
              ROPE_TABLE_POSITIONS if tab is not None else 0, _code(q), _stream())


def launch_fused_reshape_rope_kvcache_decode(input, is_done, kv_lens, q, k, v, *, use_table=True):
    """include/kernel/fused_reshape_rope_kvcache_decode.h:6-12 (pairs (2i, 2i+1))."""
    _rope_decode("l2k_fused_reshape_rope_kvcache_decode", input, is_done, kv_lens, q, k, v, use_table)


def launch_fused_reshape_rope_kvcache_llama2_decode(input, is_done, kv_lens, q, k, v, *, use_table=True):
    """include/kernel/fused_reshape_rope_kvcache_llama2_decode.h:6-12 (pairs (i, i + hd/2))."""
    _rope_decode("l2k_fused_reshape_rope_kvcache_llama2_decode", input, is_done, kv_lens, q, k, v, use_table)


def _rope_prefill(name, input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v, table):
    _dev(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v)
    for t, nm in ((q_lens, "q_lens"), (kv_lens, "kv_lens"), (unpad_to_pad_idx, "unpad_to_pad_idx")):
        _u32(t, nm)
    for t in (q, k, v):
        _same(input, t, name)
    n = input.shape[0]
    b, hq, qc, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    _require(hd % 2 == 0, "Head dim should be even")
    _require(k.shape[3] == hd and v.shape[3] == hd, "Head dim of q k v do not match")
    _require(v.shape[1] == hkv, "Head num of k v do not match")
    _require(input.shape[1] == (hq + 2 * hkv) * hd, "Incorrect embedding dim")
    _require(q_lens.shape[0] == b and kv_lens.shape[0] == b, "Incorrect batch size of sequence length")
    _require(k.shape[0] == b and v.shape[0] == b, "Batch size of k v do not match")
    _require(v.shape[2] == s, "k v cache length do not match")
    _require(unpad_to_pad_idx.numel() >= n, "unpad_to_pad_idx too small")
    tab = rope_table(hd, q.device) if table else None
    capi.call(name, input.data_ptr(), q_lens.data_ptr(), kv_lens.data_ptr(), unpad_to_pad_idx.data_ptr(),
              q.data_ptr(), k.data_ptr(), v.data_ptr(), n, b, hq, hkv, hd, qc, s,
              tab.data_ptr() if tab is not None else None, ROPE_TABLE_POSITIONS if tab is not None else 0, _code(q),
              _stream())


def launch_fused_pad_reshape_transpose_rope_kvcache(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v, *,
                                                    use_table=True):
    """include/kernel/fused_pad_reshape_transpose_rope_kvcache.h:6-13"""
    _rope_prefill("l2k_fused_pad_reshape_transpose_rope_kvcache", input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v,
                  use_table)


def launch_fused_pad_reshape_transpose_rope_kvcache_llama2(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v, *,
                                                           use_table=True):
    """include/kernel/fused_pad_reshape_transpose_rope_kvcache_llama2.h:6-13"""
    _rope_prefill("l2k_fused_pad_reshape_transpose_rope_kvcache_llama2", input, q_lens, kv_lens, unpad_to_pad_idx,
                  q, k, v, use_table)


def launch_update_q_kv_lens(q_lens, kv_lens, max_q_len, max_kv_len):
    """include/kernel/update_q_kv_lens.h:6-9.

    max_q_len / max_kv_len are 1-element tensors. On the device the results
    stay there (no synchronization). On the host, as in the reference
    (src/kernel/update_q_kv_lens.cu:52-61), the call synchronizes and the
    results land in them.
    """
    _dev(q_lens, kv_lens)
    _u32(q_lens, "q_lens")
    _u32(kv_lens, "kv_lens")
    b = q_lens.shape[0]
    _require(kv_lens.shape[0] == b, "Incorrect kv_lens size")
    if max_q_len.is_cuda and max_kv_len.is_cuda:
        capi.call("l2k_update_q_kv_lens", q_lens.data_ptr(), kv_lens.data_ptr(), b, max_q_len.data_ptr(),
                  max_kv_len.data_ptr(), _stream())
        return
    dev = torch.empty(2, dtype=torch.uint32, device=q_lens.device)
    capi.call("l2k_update_q_kv_lens", q_lens.data_ptr(), kv_lens.data_ptr(), b, dev.data_ptr(), dev.data_ptr() + 4,
              _stream())
    host = dev.cpu()
    max_q_len.view(-1)[0] = host[0].to(max_q_len.dtype)
    max_kv_len.view(-1)[0] = host[1].to(max_kv_len.dtype)


def launch_build_causal_mask(max_q_len, max_kv_len, q_lens, kv_lens, mask):
    """include/kernel/build_causal_mask.h:6-11 (the reference's unsigned-wrap expression)."""
    _dev(q_lens, kv_lens, mask)
    _require(mask.dtype == torch.uint8, "mask must be uint8")
    b, qc, s = mask.shape
    capi.call("l2k_build_causal_mask", int(max_q_len), int(max_kv_len), q_lens.data_ptr(), kv_lens.data_ptr(),
              mask.data_ptr(), b, qc, s, _stream())


def launch_build_padding_index_maps(num_input_tokens, seq_lens, unpad_to_pad_idx, seq_offsets):
    """include/kernel/build_padding_index_maps.h:6-10 (unpad_to_pad_idx is (batch, q_cache_len))."""
    _dev(seq_lens, unpad_to_pad_idx, seq_offsets)
    b = seq_lens.shape[0]
    qc = unpad_to_pad_idx.shape[1] if unpad_to_pad_idx.dim() == 2 else unpad_to_pad_idx.shape[0]
    _require(unpad_to_pad_idx.numel() >= num_input_tokens, "unpad_to_pad_idx too small")
    _require(seq_offsets.shape[0] == b, "Incorrect seq_offsets size")
    capi.call("l2k_build_padding_index_maps", int(num_input_tokens), seq_lens.data_ptr(), b, qc,
              unpad_to_pad_idx.data_ptr(), seq_offsets.data_ptr(), _stream())


def launch_build_q_k_v_qk_qkv_array(q, q_decode, k, v, qk, qk_decode, qkv, qkv_decode, q_array, q_decode_array,
                                    k_array, v_array, qk_array, qk_decode_array, qkv_array, qkv_decode_array):
    """include/kernel/build_q_k_v_qk_qkv_array.h:6-22 (arrays: int64 tensors of batch * q_head_num)."""
    tensors = (q, q_decode, k, v, qk, qk_decode, qkv, qkv_decode)
    arrays = (q_array, q_decode_array, k_array, v_array, qk_array, qk_decode_array, qkv_array, qkv_decode_array)
    _dev(*tensors, *arrays)
    b, hq = q.shape[0], q.shape[1]
    hkv = k.shape[1]
    _require(hq % hkv == 0, "q_head_num is not divisible by kv_head_num")
    for a in arrays:
        _require(a.numel() == b * hq and a.element_size() == 8, "Incorrect pointer array size")
    bases = (capi.vp * 8)(*[t.data_ptr() for t in tensors])
    slices = (capi.i64 * 8)(*[t.shape[2] * t.shape[3] for t in tensors])
    outs = (capi.vp * 8)(*[a.data_ptr() for a in arrays])
    capi.call("l2k_build_q_k_v_qk_qkv_array", bases, slices, q.element_size(), b, hq, hkv, outs, _stream())


def launch_linear(trans_A, trans_B, M, N, K, A, B, C, A_array=None, B_array=None, C_array=None):
    """include/kernel/linear.h:9-24 (no cuBLAS handle: the library's own kernel runs)."""
    _dev(A, B, C)
    _same(A, C, "launch_linear")
    _same(B, C, "launch_linear")
    dim = C.dim()
    _require(dim >= 2 and A.dim() == dim and B.dim() == dim, "Matrix dim do not match")
    lda, ldb, ldc = A.shape[-1], B.shape[-1], C.shape[-1]
    if dim > 2:
        batch = 1
        for s in C.shape[:-2]:
            batch *= s
        for arr in (A_array, B_array, C_array):
            _require(arr is not None and arr.numel() == batch, "Illegal pointer array size")
        capi.call("l2k_linear", int(trans_A), int(trans_B), M, N, K, None, lda, None, ldb, None, ldc, batch,
                  A_array.data_ptr(), B_array.data_ptr(), C_array.data_ptr(), _code(C), _stream())
    else:
        capi.call("l2k_linear", int(trans_A), int(trans_B), M, N, K, A.data_ptr(), lda, B.data_ptr(), ldb,
                  C.data_ptr(), ldc, 0, None, None, None, _code(C), _stream())


def launch_qk_scores(q, k, qk, M, N):
    """QK^T at the launch_linear call site, per (seq, head) with grouped KV heads."""
    _dev(q, k, qk)
    _same(q, k, "launch_qk_scores")
    _same(q, qk, "launch_qk_scores")
    b, hq, qc, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    _require(tuple(qk.shape) == (b, hq, qc, s), "Incorrect qk size")
    capi.call("l2k_qk_scores", q.data_ptr(), k.data_ptr(), qk.data_ptr(), b, hq, hkv, qc, s, hd, M, N, _code(q),
              _stream())


def launch_attention_qkv(qk, v, qkv, M, N):
    """P.V at the launch_linear call site (qk x v), per (seq, head) with grouped KV heads."""
    _dev(qk, v, qkv)
    _same(qk, v, "launch_attention_qkv")
    _same(qk, qkv, "launch_attention_qkv")
    b, hq, qc, s = qk.shape
    hkv, hd = v.shape[1], v.shape[3]
    _require(tuple(v.shape) == (b, hkv, s, hd), "Incorrect v size")
    _require(tuple(qkv.shape) == (b, hq, qc, hd), "Incorrect qkv size")
    capi.call("l2k_attention_qkv", qk.data_ptr(), v.data_ptr(), qkv.data_ptr(), b, hq, hkv, qc, s, hd, M, N,
              _code(qk), _stream())


def launch_compute_masked_attention_score(head_dim, max_q_len, max_kv_len, q_lens, mask, qk):
    """include/kernel/compute_masked_attention_score.h:6-12"""
    _dev(q_lens, mask, qk)
    b, hq, qc, s = qk.shape
    _require(q_lens.shape[0] == b, "Incorrect q_lens size")
    _require(tuple(mask.shape) == (b, qc, s), "Incorrect mask size")
    _require(max_q_len <= qc and max_kv_len <= s, "Incorrect max_q_len / max_kv_len")
    capi.call("l2k_compute_masked_attention_score", head_dim, int(max_q_len), int(max_kv_len), q_lens.data_ptr(),
              mask.data_ptr(), qk.data_ptr(), b, hq, qc, s, _code(qk), _stream())


def launch_swiglu(input, output):
    """include/kernel/swiglu.h:6-8"""
    _dev(input, output)
    _same(input, output, "launch_swiglu")
    n, f = output.shape
    _require(tuple(input.shape) == (n, 2 * f), "Incorrect input size")
    capi.call("l2k_swiglu", input.data_ptr(), output.data_ptr(), n, f, _code(output), _stream())


def linear_swiglu(A, B, out, *, trans_B=False):
    """out = swiglu(A op(B)) in one launch: the gate/up projection with
    launch_swiglu in its epilogue (A [T, K]; B [K, 2F], or [2F, K] with
    trans_B; out [T, F]). Raises capi.L2KError (status 3) for shapes the
    tensor-core kernel does not take."""
    _dev(A, B, out)
    _same(A, B, "linear_swiglu")
    _same(A, out, "linear_swiglu")
    t, k = A.shape
    f = out.shape[1]
    _require(out.shape[0] == t, "Incorrect output size")
    _require(tuple(B.shape) == ((2 * f, k) if trans_B else (k, 2 * f)), "Incorrect weight size")
    capi.call("l2k_linear_swiglu", int(bool(trans_B)), t, f, k, A.data_ptr(), A.stride(0), B.data_ptr(), B.stride(0),
              out.data_ptr(), out.stride(0), _code(out), _stream())


def linear_rope_kvcache_decode(A, B, is_done, kv_lens, q, k, v, *, pairing, trans_B=False, use_table=True):
    """The QKV projection of a decode step with the decode RoPE + K/V append
    in its epilogue: P = A op(B) (A [B, D]; B [D, (Hq + 2 Hkv) hd] or its
    transpose), then launch_fused_reshape_rope_kvcache[_llama2]_decode(P, ...)
    without storing P."""
    _dev(A, B, is_done, kv_lens, q, k, v)
    _u32(kv_lens, "kv_lens")
    for t in (B, q, k, v):
        _same(A, t, "linear_rope_kvcache_decode")
    b, hq, one, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    n = (hq + 2 * hkv) * hd
    _require(one == 1 and A.shape[0] == b, "Incorrect batch size")
    _require(tuple(B.shape) == ((n, A.shape[1]) if trans_B else (A.shape[1], n)), "Incorrect weight size")
    _require(tuple(k.shape) == (b, hkv, s, hd) and tuple(v.shape) == (b, hkv, s, hd), "Incorrect k v cache size")
    tab = rope_table(hd, q.device) if use_table else None
    capi.call("l2k_linear_rope_kvcache_decode", int(bool(trans_B)), A.data_ptr(), A.stride(0), B.data_ptr(),
              B.stride(0), A.shape[1], is_done.data_ptr(), kv_lens.data_ptr(), q.data_ptr(), k.data_ptr(),
              v.data_ptr(), b, hq, hkv, hd, s, tab.data_ptr() if tab is not None else None,
              ROPE_TABLE_POSITIONS if tab is not None else 0, int(pairing), _code(q), _stream())


def linear_pad_rope_kvcache_prefill(A, B, q_lens, kv_lens, unpad_to_pad_idx, q, k, v, *, pairing, trans_B=False,
                                    use_table=True):
    """The QKV projection of a prefill pass with the padded RoPE + K/V append
    in its epilogue: P = A op(B) over the T unpadded token rows, then
    launch_fused_pad_reshape_transpose_rope_kvcache[_llama2](P, ...) without
    storing P."""
    _dev(A, B, q_lens, kv_lens, unpad_to_pad_idx, q, k, v)
    for t, nm in ((q_lens, "q_lens"), (kv_lens, "kv_lens"), (unpad_to_pad_idx, "unpad_to_pad_idx")):
        _u32(t, nm)
    for t in (B, q, k, v):
        _same(A, t, "linear_pad_rope_kvcache_prefill")
    tokens = A.shape[0]
    b, hq, qc, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    n = (hq + 2 * hkv) * hd
    _require(tuple(B.shape) == ((n, A.shape[1]) if trans_B else (A.shape[1], n)), "Incorrect weight size")
    _require(tuple(k.shape) == (b, hkv, s, hd) and tuple(v.shape) == (b, hkv, s, hd), "Incorrect k v cache size")
    _require(q_lens.shape[0] == b and kv_lens.shape[0] == b, "Incorrect batch size of sequence length")
    _require(unpad_to_pad_idx.numel() >= tokens, "unpad_to_pad_idx too small")
    tab = rope_table(hd, q.device) if use_table else None
    capi.call("l2k_linear_pad_rope_kvcache_prefill", int(bool(trans_B)), A.data_ptr(), A.stride(0), B.data_ptr(),
              B.stride(0), A.shape[1], q_lens.data_ptr(), kv_lens.data_ptr(), unpad_to_pad_idx.data_ptr(),
              q.data_ptr(), k.data_ptr(), v.data_ptr(), tokens, b, hq, hkv, hd, qc, s,
              tab.data_ptr() if tab is not None else None, ROPE_TABLE_POSITIONS if tab is not None else 0,
              int(pairing), _code(q), _stream())


def launch_fused_transpose_unpad(num_input_tokens, qkv, unpad_to_pad_idx, unpad_qkv):
    """include/kernel/fused_transpose_unpad.h:6-11 (qkv (B, H, Qc, hd) -> unpad_qkv (T, H * hd))."""
    _dev(qkv, unpad_to_pad_idx, unpad_qkv)
    _same(qkv, unpad_qkv, "launch_fused_transpose_unpad")
    _u32(unpad_to_pad_idx, "unpad_to_pad_idx")
    b, h, qc, hd = qkv.shape
    _require(unpad_qkv.dim() == 2 and unpad_qkv.shape[1] == h * hd, "Incorrect embed dim")
    _require(unpad_qkv.shape[0] >= num_input_tokens, "unpad_qkv has too few rows")
    _require(unpad_to_pad_idx.numel() >= num_input_tokens, "unpad_to_pad_idx too small")
    capi.call("l2k_fused_transpose_unpad", int(num_input_tokens), qkv.data_ptr(), unpad_to_pad_idx.data_ptr(),
              unpad_qkv.data_ptr(), b, h, qc, hd, _code(qkv), _stream())


def decode_attention_scores(q, k, kv_lens, max_kv_len, qk):
    """Fused QK^T + scale + length mask + softmax for one query token per sequence.

    q (B, Hq, 1, hd); k (B, Hkv, S, hd); qk (B, Hq, 1, S); max_kv_len: 1-element
    device tensor (e.g. written by launch_update_q_kv_lens)."""
    _dev(q, k, kv_lens, max_kv_len, qk)
    _same(q, k, "decode_attention_scores")
    _same(q, qk, "decode_attention_scores")
    b, hq, one, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    _require(one == 1 and tuple(qk.shape) == (b, hq, 1, s), "Incorrect q / qk size")
    capi.call("l2k_decode_attention_scores", q.data_ptr(), k.data_ptr(), kv_lens.data_ptr(), max_kv_len.data_ptr(),
              qk.data_ptr(), b, hq, hkv, s, hd, _code(q), _stream())


def decode_attention(q, k, v, kv_lens, max_kv_len, qk, qkv):
    """Fused decode attention: the decode_attention_scores probabilities (into qk)
    and the attention output P.V (into qkv (B, Hq, 1, hd)) in one pass."""
    _dev(q, k, v, kv_lens, max_kv_len, qk, qkv)
    for t in (k, v, qk, qkv):
        _same(q, t, "decode_attention")
    b, hq, one, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    _require(one == 1 and tuple(qk.shape) == (b, hq, 1, s), "Incorrect q / qk size")
    _require(tuple(v.shape) == tuple(k.shape), "Incorrect v size")
    _require(tuple(qkv.shape) == (b, hq, 1, hd), "Incorrect qkv size")
    capi.call("l2k_decode_attention", q.data_ptr(), k.data_ptr(), v.data_ptr(), kv_lens.data_ptr(),
              max_kv_len.data_ptr(), qk.data_ptr(), qkv.data_ptr(), b, hq, hkv, s, hd, _code(q), _stream())


def paged_block_rows(head_dim: int, dtype: torch.dtype) -> int:
    """Rows per page (and kv head) of the paged caches: one 16 KB streamed block."""
    return int(capi.lib().l2k_paged_block_rows(head_dim, _DT[dtype]))


def launch_rope_kvcache_paged_decode(input, is_done, kv_lens, q, k_pages, v_pages, block_table, *, pairing,
                                     use_table=True):
    """Decode RoPE + K/V append into paged caches k_pages / v_pages
    (num_pages, Hkv, page_rows, hd); block_table (B, max_pages) u32."""
    _dev(input, is_done, kv_lens, q, k_pages, v_pages, block_table)
    _u32(block_table, "block_table")
    b, hq, _, hd = q.shape
    n_pages, hkv, page_rows, _ = k_pages.shape
    _require(tuple(v_pages.shape) == tuple(k_pages.shape), "Incorrect v_pages size")
    table = rope_table(hd, q.device) if use_table else None
    capi.call("l2k_fused_reshape_rope_kvcache_paged_decode", input.data_ptr(), is_done.data_ptr(),
              kv_lens.data_ptr(), q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(),
              block_table.shape[1], n_pages, page_rows, b, hq, hkv, hd,
              table.data_ptr() if table is not None else None, ROPE_TABLE_POSITIONS if table is not None else 0,
              int(pairing), _code(q), _stream())


def decode_attention_paged(q, k_pages, v_pages, block_table, kv_lens, max_kv_len, qk, qkv):
    """decode_attention over paged caches (num_pages, Hkv, page_rows, hd)
    with page_rows = paged_block_rows(hd, dtype); qk (B, Hq, 1, max_pages * page_rows)."""
    _dev(q, k_pages, v_pages, block_table, kv_lens, max_kv_len, qk, qkv)
    _u32(block_table, "block_table")
    b, hq, _, hd = q.shape
    n_pages, hkv, page_rows, _ = k_pages.shape
    _require(page_rows == paged_block_rows(hd, q.dtype), "page_rows must be paged_block_rows(head_dim, dtype)")
    max_pages = block_table.shape[1]
    _require(tuple(qk.shape) == (b, hq, 1, max_pages * page_rows), "Incorrect qk size")
    _require(tuple(qkv.shape) == (b, hq, 1, hd), "Incorrect qkv size")
    capi.call("l2k_decode_attention_paged", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
              block_table.data_ptr(), max_pages, n_pages, kv_lens.data_ptr(), max_kv_len.data_ptr(), qk.data_ptr(),
              qkv.data_ptr(), b, hq, hkv, hd, _code(q), _stream())


def launch_rope_kvcache_paged_prefill(input, q_lens, kv_lens, unpad_to_pad_idx, q, k_pages, v_pages, block_table, *,
                                      pairing, use_table=True):
    """Prefill RoPE + K/V append (the padded q of
    launch_fused_pad_reshape_transpose_rope_kvcache[_llama2]) into paged caches
    k_pages / v_pages (num_pages, Hkv, page_rows, hd); block_table (B, max_pages) u32."""
    _dev(input, q_lens, kv_lens, unpad_to_pad_idx, q, k_pages, v_pages, block_table)
    for t, nm in ((q_lens, "q_lens"), (kv_lens, "kv_lens"), (unpad_to_pad_idx, "unpad_to_pad_idx"),
                  (block_table, "block_table")):
        _u32(t, nm)
    for t in (q, k_pages, v_pages):
        _same(input, t, "launch_rope_kvcache_paged_prefill")
    n = input.shape[0]
    b, hq, qc, hd = q.shape
    n_pages, hkv, page_rows, _ = k_pages.shape
    _require(tuple(v_pages.shape) == tuple(k_pages.shape), "Incorrect v_pages size")
    _require(input.shape[1] == (hq + 2 * hkv) * hd, "Incorrect embedding dim")
    _require(block_table.shape[0] == b and q_lens.shape[0] == b and kv_lens.shape[0] == b, "Incorrect batch size")
    _require(unpad_to_pad_idx.numel() >= n, "unpad_to_pad_idx too small")
    table = rope_table(hd, q.device) if use_table else None
    capi.call("l2k_fused_pad_reshape_transpose_rope_kvcache_paged", input.data_ptr(), q_lens.data_ptr(),
              kv_lens.data_ptr(), unpad_to_pad_idx.data_ptr(), q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(),
              block_table.data_ptr(), block_table.shape[1], n_pages, page_rows, n, b, hq, hkv, hd, qc,
              table.data_ptr() if table is not None else None, ROPE_TABLE_POSITIONS if table is not None else 0,
              int(pairing), _code(q), _stream())


def prefill_attention_scores_paged(q, k_pages, block_table, q_lens, kv_lens, max_q_len, max_kv_len, qk):
    """prefill_attention_scores over a paged K cache (num_pages, Hkv, 64, 128),
    16-bit; qk (B, Hq, q_cache_len, max_pages * 64)."""
    _dev(q, k_pages, block_table, q_lens, kv_lens, qk)
    _u32(block_table, "block_table")
    _same(q, k_pages, "prefill_attention_scores_paged")
    _same(q, qk, "prefill_attention_scores_paged")
    b, hq, qc, hd = q.shape
    n_pages, hkv = k_pages.shape[0], k_pages.shape[1]
    max_pages = block_table.shape[1]
    _require(tuple(qk.shape) == (b, hq, qc, max_pages * 64), "Incorrect qk size")
    capi.call("l2k_prefill_attention_scores_paged", q.data_ptr(), k_pages.data_ptr(), block_table.data_ptr(),
              max_pages, n_pages, q_lens.data_ptr(), kv_lens.data_ptr(), int(max_q_len), int(max_kv_len),
              qk.data_ptr(), b, hq, hkv, qc, hd, _code(q), _stream())


def launch_attention_qkv_paged(qk, v_pages, block_table, kv_lens, qkv, M, N):
    """launch_attention_qkv over a paged V cache (num_pages, Hkv, 64, 128), 16-bit."""
    _dev(qk, v_pages, block_table, kv_lens, qkv)
    _u32(block_table, "block_table")
    _same(qk, v_pages, "launch_attention_qkv_paged")
    _same(qk, qkv, "launch_attention_qkv_paged")
    b, hq, qc, s = qk.shape
    n_pages, hkv, _, hd = v_pages.shape
    max_pages = block_table.shape[1]
    _require(s == max_pages * 64, "Incorrect qk size")
    _require(tuple(qkv.shape) == (b, hq, qc, hd), "Incorrect qkv size")
    capi.call("l2k_attention_qkv_paged", qk.data_ptr(), v_pages.data_ptr(), block_table.data_ptr(), max_pages,
              n_pages, kv_lens.data_ptr(), qkv.data_ptr(), b, hq, hkv, qc, hd, int(M), int(N), _code(qk), _stream())


def launch_rope_kvcache_fp8_decode(input, is_done, kv_lens, q, k_cache, v_cache, k_scale, v_scale, *, pairing,
                                   use_table=True):
    """Decode RoPE + K/V append into fp8 (e4m3) caches k_cache / v_cache:
    uint8 tensors (B, Hkv, S, hd) holding value / scale rounded to e4m3; q
    (B, Hq, 1, hd) in the 16-bit activation type of input."""
    _dev(input, is_done, kv_lens, q, k_cache, v_cache)
    _same(input, q, "launch_rope_kvcache_fp8_decode")
    _require(k_cache.dtype == torch.uint8 and v_cache.dtype == torch.uint8, "fp8 caches are uint8 tensors")
    b, hq, _, hd = q.shape
    hkv, s = k_cache.shape[1], k_cache.shape[2]
    _require(tuple(v_cache.shape) == tuple(k_cache.shape) and k_cache.shape[3] == hd and k_cache.shape[0] == b,
             "Incorrect cache size")
    _require(input.shape[1] == (hq + 2 * hkv) * hd, "Incorrect embedding dim")
    table = rope_table(hd, q.device) if use_table else None
    capi.call("l2k_fused_reshape_rope_kvcache_fp8_decode", input.data_ptr(), is_done.data_ptr(), kv_lens.data_ptr(),
              q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), float(k_scale), float(v_scale), b, hq, hkv, hd, s,
              table.data_ptr() if table is not None else None, ROPE_TABLE_POSITIONS if table is not None else 0,
              int(pairing), _code(q), _stream())


def decode_attention_fp8(q, k_cache, v_cache, k_scale, v_scale, kv_lens, max_kv_len, qk, qkv):
    """decode_attention over fp8 (e4m3, uint8 storage) caches (B, Hkv, S, hd)."""
    _dev(q, k_cache, v_cache, kv_lens, max_kv_len, qk, qkv)
    _same(q, qk, "decode_attention_fp8")
    _same(q, qkv, "decode_attention_fp8")
    b, hq, _, hd = q.shape
    hkv, s = k_cache.shape[1], k_cache.shape[2]
    _require(k_cache.dtype == torch.uint8 and tuple(v_cache.shape) == tuple(k_cache.shape), "Incorrect caches")
    _require(tuple(qk.shape) == (b, hq, 1, s) and tuple(qkv.shape) == (b, hq, 1, hd), "Incorrect qk / qkv size")
    capi.call("l2k_decode_attention_fp8", q.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), float(k_scale),
              float(v_scale), kv_lens.data_ptr(), max_kv_len.data_ptr(), qk.data_ptr(), qkv.data_ptr(), b, hq, hkv, s,
              hd, _code(q), _stream())


def decode_attention_fp8_paged(q, k_pages, v_pages, k_scale, v_scale, block_table, kv_lens, max_kv_len, qk, qkv):
    """decode_attention_fp8 over page pools (num_pages, Hkv, 16384 / hd, hd) of e4m3 bytes."""
    _dev(q, k_pages, v_pages, block_table, kv_lens, max_kv_len, qk, qkv)
    _u32(block_table, "block_table")
    b, hq, _, hd = q.shape
    n_pages, hkv, rows, _ = k_pages.shape
    max_pages = block_table.shape[1]
    _require(rows == 16384 // hd and k_pages.dtype == torch.uint8, "pages must be uint8 (num_pages, Hkv, 16384/hd, hd)")
    _require(tuple(qk.shape) == (b, hq, 1, max_pages * rows), "Incorrect qk size")
    capi.call("l2k_decode_attention_fp8_paged", q.data_ptr(), k_pages.data_ptr(), v_pages.data_ptr(), float(k_scale),
              float(v_scale), block_table.data_ptr(), max_pages, n_pages, kv_lens.data_ptr(), max_kv_len.data_ptr(),
              qk.data_ptr(), qkv.data_ptr(), b, hq, hkv, hd, _code(q), _stream())


def prefill_attention_scores(q, k, q_lens, kv_lens, max_q_len, max_kv_len, qk):
    """Fused QK^T + scale + causal mask + softmax for q_len query rows per sequence."""
    _dev(q, k, q_lens, kv_lens, qk)
    _same(q, k, "prefill_attention_scores")
    _same(q, qk, "prefill_attention_scores")
    b, hq, qc, hd = q.shape
    hkv, s = k.shape[1], k.shape[2]
    _require(tuple(qk.shape) == (b, hq, qc, s), "Incorrect qk size")
    capi.call("l2k_prefill_attention_scores", q.data_ptr(), k.data_ptr(), q_lens.data_ptr(), kv_lens.data_ptr(),
              int(max_q_len), int(max_kv_len), qk.data_ptr(), b, hq, hkv, qc, s, hd, _code(q), _stream())


# --------------------------------------------------------------------------
# Fused decode step (one launch for the whole decode chain)
# --------------------------------------------------------------------------
def decode_step_workspace(device) -> torch.Tensor:
    """Zeroed workspace for decode_step (one per step that may run concurrently)."""
    n = int(capi.lib().l2k_decode_step_workspace_bytes())
    return torch.zeros((n + 3) // 4, dtype=torch.uint32, device=device)


def _decode_step_args(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done, q,
                      k_cache, v_cache, qk, gate_up, ffn_out, pairing, use_table, block_table=None):
    _dev(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done, q, k_cache, v_cache,
         qk, gate_up, ffn_out)
    for t, n in ((q_lens, "q_lens"), (kv_lens, "kv_lens"), (max_lens, "max_lens"), (input_ids, "input_ids")):
        _u32(t, n)
    for t in (norm_weight, x, normed, qkv, q, k_cache, v_cache, qk, gate_up, ffn_out):
        _same(embed_table, t, "decode_step")
    b = input_ids.numel()
    vocab, dim = embed_table.shape
    _, hq, one, hd = q.shape
    hkv, s = k_cache.shape[1], k_cache.shape[2]
    hidden = ffn_out.shape[-1]
    _require(one == 1 and q.shape[0] == b, "Incorrect q size")
    if block_table is None:
        _require(tuple(k_cache.shape) == (b, hkv, s, hd) and tuple(v_cache.shape) == (b, hkv, s, hd),
                 "Incorrect k/v cache size")
    else:
        # page pools (num_pages, Hkv, page_rows, hd); s = the logical cache length
        _dev(block_table)
        _u32(block_table, "block_table")
        page_rows = k_cache.shape[2]
        _require(page_rows == paged_block_rows(hd, q.dtype), "page_rows must be paged_block_rows(head_dim, dtype)")
        _require(tuple(v_cache.shape) == tuple(k_cache.shape) and k_cache.shape[3] == hd, "Incorrect k/v pool size")
        _require(block_table.dim() == 2 and block_table.shape[0] == b, "Incorrect block_table size")
        s = block_table.shape[1] * page_rows
    _require(tuple(qk.shape) == (b, hq, 1, s), "Incorrect qk size")
    _require(qkv.numel() == b * (hq + 2 * hkv) * hd, "Incorrect qkv size")
    _require(x.numel() == b * dim and normed.numel() == b * dim and norm_weight.numel() == dim, "Incorrect x size")
    _require(gate_up.numel() == 2 * b * hidden and ffn_out.numel() == b * hidden, "Incorrect gate_up size")
    _require(q_lens.numel() == b and kv_lens.numel() == b and is_done.numel() == b and max_lens.numel() >= 2,
             "Incorrect lens size")
    table = rope_table(hd, q.device) if use_table else None
    return capi.DecodeStepArgs(
        q_lens.data_ptr(), kv_lens.data_ptr(), max_lens.data_ptr(), input_ids.data_ptr(), embed_table.data_ptr(),
        norm_weight.data_ptr(), x.data_ptr(), normed.data_ptr(), qkv.data_ptr(), is_done.data_ptr(), q.data_ptr(),
        k_cache.data_ptr(), v_cache.data_ptr(), qk.data_ptr(), table.data_ptr() if table is not None else None,
        ROPE_TABLE_POSITIONS if table is not None else 0, gate_up.data_ptr(), ffn_out.data_ptr(), b, vocab, dim, hq,
        hkv, hd, s, hidden, int(pairing), _code(embed_table))


def decode_step(*, q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done, q,
                k_cache, v_cache, qk, gate_up, ffn_out, workspace, pairing, use_table=True):
    """The decode chain of one layer step in one launch (l2k_decode_step):
    lengths update, embedding, RMSNorm, RoPE + KV append, fused scores, SwiGLU.
    max_lens: 2-element u32 device tensor (max q_len, max kv_len)."""
    args = _decode_step_args(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done,
                             q, k_cache, v_cache, qk, gate_up, ffn_out, pairing, use_table)
    _dev(workspace)
    capi.call("l2k_decode_step", ctypes.byref(args), workspace.data_ptr(), _stream())


def decode_step_paged(*, q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done, q,
                      k_pages, v_pages, block_table, qk, gate_up, ffn_out, workspace, pairing, use_table=True,
                      attn_out=None):
    """decode_step (or, with attn_out, decode_step_attention) over paged caches
    k_pages / v_pages (num_pages, Hkv, page_rows, hd), page_rows =
    paged_block_rows(hd, dtype); block_table (B, max_pages) u32; qk
    (B, Hq, 1, max_pages * page_rows) (l2k_decode_step[_attention]_paged)."""
    args = _decode_step_args(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done,
                             q, k_pages, v_pages, qk, gate_up, ffn_out, pairing, use_table, block_table=block_table)
    _dev(workspace)
    max_pages, num_pages = block_table.shape[1], k_pages.shape[0]
    if attn_out is None:
        capi.call("l2k_decode_step_paged", ctypes.byref(args), block_table.data_ptr(), max_pages, num_pages,
                  workspace.data_ptr(), _stream())
        return
    _dev(attn_out)
    _same(qk, attn_out, "decode_step_paged")
    _require(attn_out.numel() == q.numel(), "attn_out must hold (batch, Hq, 1, head_dim)")
    capi.call("l2k_decode_step_attention_paged", ctypes.byref(args), block_table.data_ptr(), max_pages, num_pages,
              attn_out.data_ptr(), workspace.data_ptr(), _stream())


def decode_step_attention(*, q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv,
                          is_done, q, k_cache, v_cache, qk, gate_up, ffn_out, attn_out, workspace, pairing,
                          use_table=True):
    """decode_step plus the attention output attn_out (B, Hq, 1, hd) = P.V over
    the appended V cache, in the same launch (l2k_decode_step_attention)."""
    args = _decode_step_args(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done,
                             q, k_cache, v_cache, qk, gate_up, ffn_out, pairing, use_table)
    _dev(workspace, attn_out)
    _same(qk, attn_out, "decode_step_attention")
    _require(attn_out.numel() == q.numel(), "attn_out must hold (batch, Hq, 1, head_dim)")
    capi.call("l2k_decode_step_attention", ctypes.byref(args), attn_out.data_ptr(), workspace.data_ptr(), _stream())


def decode_step_launcher(*, workspace, attn_out=None, **kw):
    """decode_step (or, with attn_out, decode_step_attention) with its
    arguments checked and packed once: returns a function that enqueues the
    step on the current stream. For a caller that repeats the step over the
    same tensors: the step is one kernel, so a direct launch costs less than
    replaying it from a CUDA graph."""
    kw.setdefault("use_table", True)
    args = _decode_step_args(**kw)
    _dev(workspace)
    ws = workspace.data_ptr()
    lib = capi.lib()
    if attn_out is None:
        name, fn, extra = "l2k_decode_step", lib.l2k_decode_step, ()
    else:
        _dev(attn_out)
        _same(kw["qk"], attn_out, "decode_step_attention")
        _require(attn_out.numel() == kw["q"].numel(), "attn_out must hold (batch, Hq, 1, head_dim)")
        name, fn, extra = "l2k_decode_step_attention", lib.l2k_decode_step_attention, (attn_out.data_ptr(),)
    ref = ctypes.byref(args)

    def launch():
        status = fn(ref, *extra, ws, _stream())
        if status != 0:
            raise capi.L2KError(name, status, lib.l2k_last_error_message().decode())

    launch.args = args  # keeps the packed arguments alive with the launcher
    return launch


def decode_step_no_alloc(*, q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv,
                         is_done, q, k_cache, v_cache, qk, gate_up, ffn_out, pairing, use_table=True):
    """decode_step with the library's own static scratch as workspace
    (l2k_decode_step_no_alloc): no workspace argument, nothing allocated;
    steps on one device must not overlap."""
    args = _decode_step_args(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done,
                             q, k_cache, v_cache, qk, gate_up, ffn_out, pairing, use_table)
    capi.call("l2k_decode_step_no_alloc", ctypes.byref(args), _stream())


def decode_step_attention_no_alloc(*, q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed,
                                   qkv, is_done, q, k_cache, v_cache, qk, gate_up, ffn_out, attn_out, pairing,
                                   use_table=True):
    """decode_step_attention on the library's static scratch
    (l2k_decode_step_attention_no_alloc); steps on one device must not
    overlap."""
    args = _decode_step_args(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x, normed, qkv, is_done,
                             q, k_cache, v_cache, qk, gate_up, ffn_out, pairing, use_table)
    _dev(attn_out)
    _same(qk, attn_out, "decode_step_attention_no_alloc")
    _require(attn_out.numel() == q.numel(), "attn_out must hold (batch, Hq, 1, head_dim)")
    capi.call("l2k_decode_step_attention_no_alloc", ctypes.byref(args), attn_out.data_ptr(), _stream())


def decode_step_supported(**kw) -> bool:
    """Whether decode_step takes these tensors (shape and alignment support)."""
    kw.pop("workspace", None)
    kw.setdefault("use_table", True)
    args = _decode_step_args(**kw)
    return capi.lib().l2k_decode_step_supported(ctypes.byref(args)) == 0
