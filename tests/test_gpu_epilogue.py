"""Projection GEMMs with the next operator in the tensor-core epilogue:
gate/up + SwiGLU (l2k_linear_swiglu) and QKV + RoPE + K/V append, decode and
prefill (l2k_linear_rope_kvcache_decode, l2k_linear_pad_rope_kvcache_prefill).

Bar: bit-identical to the unfused pair (l2k_linear on its tensor-core path,
i.e. more than 8 rows, then launch_swiglu / the fused RoPE operator on the
stored product), every element of q and of both caches compared; at few
rows (where l2k_linear streams B on the CUDA cores instead) and against the
oracle composition (oracle GEMM, rounded to 16 bits, then the oracle's
SwiGLU / RoPE): 1e-2 relative to each output row's largest magnitude.
"""
import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from oracle import port
from tests.gpu_util import bits_equal, host, round_to

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def _row_rel_err(got, want):
    got = np.asarray(got, np.float64).reshape(-1, np.asarray(got).shape[-1])
    want = np.asarray(want, np.float64).reshape(got.shape)
    scale = np.maximum(np.abs(want).max(axis=-1, keepdims=True), 1e-30)
    return float((np.abs(got - want) / scale).max())


def _randn(g, *shape, dtype, scale=1.0):
    return (torch.randn(*shape, generator=g, device="cuda") * scale).to(dtype)


# ---------------------------------------------------------------- SwiGLU
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("m,f,k,trans_b", [
    (64, 11008, 4096, 0),   # 7B decode batch 64: one row tile, 172 column tiles
    (16, 384, 1000, 0),     # k split over a cluster of 8, ragged last k block
    (300, 200, 136, 1),     # B stored 2F x K, F not a multiple of the tile's 128 outputs
    (1024, 11008, 4096, 0), # 128 x 256 tiles (128 gate + 128 up columns)
])
def test_linear_swiglu_bit_identical_to_linear_then_swiglu(dtype, m, f, k, trans_b):
    g = torch.Generator(device="cuda")
    g.manual_seed(m + f + k)
    a = _randn(g, m, k, dtype=dtype)
    w = _randn(g, *((2 * f, k) if trans_b else (k, 2 * f)), dtype=dtype, scale=k ** -0.5)
    gate_up = torch.empty(m, 2 * f, dtype=dtype, device="cuda")
    want = torch.empty(m, f, dtype=dtype, device="cuda")
    got = torch.full((m, f), 7.0, dtype=dtype, device="cuda")
    ops.launch_linear(False, bool(trans_b), m, 2 * f, k, a, w, gate_up)
    ops.launch_swiglu(gate_up, want)
    ops.linear_swiglu(a, w, got, trans_B=bool(trans_b))
    torch.cuda.synchronize()
    assert bits_equal(host(got), host(want))


@pytest.mark.parametrize("m", [3, 12])
def test_linear_swiglu_against_oracle(m):
    """Few rows (the unfused GEMM would take the CUDA-core path) and a small
    tile, against the oracle's GEMM rounded to bf16 and its SwiGLU."""
    f, k, dtype = 256, 192, torch.bfloat16
    g = torch.Generator(device="cuda")
    g.manual_seed(m)
    a = _randn(g, m, k, dtype=dtype)
    w = _randn(g, k, 2 * f, dtype=dtype, scale=k ** -0.5)
    got = torch.empty(m, f, dtype=dtype, device="cuda")
    ops.linear_swiglu(a, w, got)
    torch.cuda.synchronize()
    prod = round_to(port.linear(host(a), host(w), False, False, m, 2 * f, k), dtype)
    assert _row_rel_err(host(got), port.swiglu(prod)) <= 1e-2


def test_linear_swiglu_rejects_what_it_does_not_take():
    a = torch.zeros(16, 64, dtype=torch.bfloat16, device="cuda")
    w = torch.zeros(64, 2 * 12, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(16, 12, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(capi.L2KError) as e:
        ops.linear_swiglu(a, w, out)  # F = 12: not a multiple of 8
    assert e.value.status == 3


# ---------------------------------------------------------------- RoPE, decode
def _decode_case(dtype, b, hq, hkv, hd, s, dim, seed, edges=True):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    n = (hq + 2 * hkv) * hd
    a = _randn(g, b, dim, dtype=dtype)
    w = _randn(g, dim, n, dtype=dtype, scale=dim ** -0.5)
    k = _randn(g, b, hkv, s, hd, dtype=dtype)
    v = _randn(g, b, hkv, s, hd, dtype=dtype)
    lens = torch.randint(1, s + 1, (b,), generator=torch.Generator().manual_seed(seed))
    lens[0] = s               # the last cache row
    if edges and b > 3:
        lens[1] = 0           # position wraps below zero: nothing written
        lens[2] = s + 1       # past the cache: nothing written (the oracle, like the reference, would write there)
    done = torch.zeros(b, dtype=torch.uint8)
    done[3 % b] = 1
    return a, w, k, v, lens.to(torch.uint32).cuda(), done.cuda()


@pytest.mark.parametrize("dtype,b,hq,hkv,hd,s,dim,pairing,table", [
    (torch.bfloat16, 64, 32, 32, 128, 512, 4096, 1, True),    # 7B decode batch 64 (k split over 2)
    (torch.float16, 64, 32, 8, 128, 300, 1024, 0, True),      # grouped KV heads, interleaved pairs
    (torch.bfloat16, 20, 8, 2, 64, 100, 256, 1, True),        # head_dim 64: two heads per tile
    (torch.bfloat16, 200, 8, 4, 128, 64, 512, 0, True),       # 128 x 256 tiles: two heads per tile
    (torch.bfloat16, 24, 4, 2, 128, 64, 256, 1, False),       # angles evaluated on the device
])
def test_linear_rope_decode_bit_identical_to_linear_then_rope(dtype, b, hq, hkv, hd, s, dim, pairing, table):
    a, w, k1, v1, kv_lens, is_done = _decode_case(dtype, b, hq, hkv, hd, s, dim, seed=b + hq + hd)
    k2, v2 = k1.clone(), v1.clone()
    q1 = torch.full((b, hq, 1, hd), 3.0, dtype=dtype, device="cuda")
    q2 = q1.clone()
    qkv = torch.empty(b, (hq + 2 * hkv) * hd, dtype=dtype, device="cuda")
    ops.launch_linear(False, False, b, qkv.shape[1], dim, a, w, qkv)
    rope = (ops.launch_fused_reshape_rope_kvcache_llama2_decode if pairing
            else ops.launch_fused_reshape_rope_kvcache_decode)
    rope(qkv, is_done, kv_lens, q1, k1, v1, use_table=table)
    ops.linear_rope_kvcache_decode(a, w, is_done, kv_lens, q2, k2, v2, pairing=pairing, use_table=table)
    torch.cuda.synchronize()
    assert bits_equal(host(q2), host(q1))
    assert bits_equal(host(k2), host(k1))
    assert bits_equal(host(v2), host(v1))


@pytest.mark.parametrize("pairing", [0, 1])
def test_linear_rope_decode_against_oracle(pairing):
    dtype, b, hq, hkv, hd, s, dim = torch.bfloat16, 12, 4, 2, 128, 48, 256
    a, w, k, v, kv_lens, is_done = _decode_case(dtype, b, hq, hkv, hd, s, dim, seed=5, edges=False)
    q = torch.zeros(b, hq, 1, hd, dtype=dtype, device="cuda")
    kr, vr, qr = host(k).copy(), host(v).copy(), host(q).copy()
    ops.linear_rope_kvcache_decode(a, w, is_done, kv_lens, q, k, v, pairing=pairing)
    torch.cuda.synchronize()
    prod = round_to(port.linear(host(a), host(w), False, False, b, w.shape[1], dim), dtype)
    port.rope_kvcache_decode(pairing, prod, host(is_done), host(kv_lens), qr, kr, vr)
    assert _row_rel_err(host(q), qr) <= 1e-2
    assert _row_rel_err(host(k), kr) <= 1e-2
    assert _row_rel_err(host(v), vr) <= 1e-2  # the 16-bit product may differ by an ulp from the oracle's


# ---------------------------------------------------------------- RoPE, prefill
def _prefill_case(dtype, q_lens_h, cached_h, qc, s, hq, hkv, hd, dim, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    b = len(q_lens_h)
    t = int(sum(q_lens_h))
    n = (hq + 2 * hkv) * hd
    a = _randn(g, t, dim, dtype=dtype)
    w = _randn(g, dim, n, dtype=dtype, scale=dim ** -0.5)
    k = _randn(g, b, hkv, s, hd, dtype=dtype)
    v = _randn(g, b, hkv, s, hd, dtype=dtype)
    q_lens = torch.tensor(q_lens_h, dtype=torch.uint32, device="cuda")
    kv_lens = torch.tensor([c + q for c, q in zip(cached_h, q_lens_h)], dtype=torch.uint32, device="cuda")
    unpad = torch.zeros(b, qc, dtype=torch.uint32, device="cuda")
    offsets = torch.zeros(b, dtype=torch.uint32, device="cuda")
    ops.launch_build_padding_index_maps(t, q_lens, unpad, offsets)
    return a, w, k, v, q_lens, kv_lens, unpad.view(-1)


@pytest.mark.parametrize("dtype,q_lens_h,cached_h,pairing", [
    (torch.bfloat16, [100, 37, 1], [0, 20, 60], 1),   # 138 token rows: 128 x 256 tiles
    (torch.float16, [64, 40], [0, 10], 0),            # 104 rows: one row tile, k split over a cluster
    (torch.bfloat16, [128, 100, 90], [0, 20, 60], 1), # 318 rows: 256 x 256 tiles over CTA pairs
])
def test_linear_rope_prefill_bit_identical_to_linear_then_rope(dtype, q_lens_h, cached_h, pairing):
    hq, hkv, hd, dim, qc, s = 8, 4, 128, 512, 128, 256
    a, w, k1, v1, q_lens, kv_lens, unpad = _prefill_case(dtype, q_lens_h, cached_h, qc, s, hq, hkv, hd, dim, 11)
    b, t = len(q_lens_h), a.shape[0]
    k2, v2 = k1.clone(), v1.clone()
    q1 = torch.full((b, hq, qc, hd), 3.0, dtype=dtype, device="cuda")
    q2 = q1.clone()
    qkv = torch.empty(t, w.shape[1], dtype=dtype, device="cuda")
    ops.launch_linear(False, False, t, w.shape[1], dim, a, w, qkv)
    rope = (ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2 if pairing
            else ops.launch_fused_pad_reshape_transpose_rope_kvcache)
    rope(qkv, q_lens, kv_lens, unpad, q1, k1, v1)
    ops.linear_pad_rope_kvcache_prefill(a, w, q_lens, kv_lens, unpad, q2, k2, v2, pairing=pairing)
    torch.cuda.synchronize()
    assert bits_equal(host(q2), host(q1))
    assert bits_equal(host(k2), host(k1))
    assert bits_equal(host(v2), host(v1))


def test_linear_rope_prefill_against_oracle():
    dtype, hq, hkv, hd, dim, qc, s = torch.bfloat16, 4, 2, 128, 256, 32, 64
    q_lens_h, cached_h = [20, 7], [0, 30]
    a, w, k, v, q_lens, kv_lens, unpad = _prefill_case(dtype, q_lens_h, cached_h, qc, s, hq, hkv, hd, dim, 3)
    t = a.shape[0]
    q = torch.zeros(2, hq, qc, hd, dtype=dtype, device="cuda")
    kr, vr, qr = host(k).copy(), host(v).copy(), host(q).copy()
    ops.linear_pad_rope_kvcache_prefill(a, w, q_lens, kv_lens, unpad, q, k, v, pairing=1)
    torch.cuda.synchronize()
    prod = round_to(port.linear(host(a), host(w), False, False, t, w.shape[1], dim), dtype)
    port.rope_kvcache_prefill(1, prod, q_lens_h, host(kv_lens), host(unpad)[:t], qr, kr, vr)
    assert _row_rel_err(host(q), qr) <= 1e-2
    assert _row_rel_err(host(k), kr) <= 1e-2
    assert _row_rel_err(host(v), vr) <= 1e-2  # the 16-bit product may differ by an ulp from the oracle's
