"""fp8 (e4m3) K/V caches for decode: the RoPE + append into byte caches and
the streaming decode attention that dequantizes its K/V blocks in shared
memory, against the oracle on the same bytes.

Bars: q (16-bit) bit-identical to the 16-bit operator's; appended K/V bytes
bit-exact against the oracle's e4m3 rounding of the same fp32 values
(oracle.port.e4m3_from_f32); untouched cache rows unchanged. Scores and the
attention output against the oracle's fp32 softmax and P.V over the
dequantized caches (scale * e4m3 value), max relative error <= 1e-2 (the
16-bit-I/O bar; the output relative to each row's largest magnitude). Paged
caches bit-identical to the contiguous ones.
"""
import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from oracle import chain as ochain
from oracle import port
from tests.gpu_util import bits_equal, host, max_rel_err

pytestmark = pytest.mark.gpu

TORCH = {"bf16": torch.bfloat16, "f16": torch.float16}


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield
    assert capi.lib().l2k_device_error(1) == 0


def _cache_bytes(shape, scale, seed):
    """A cache of e4m3 bytes holding N(0, 1) values quantized at `scale`."""
    x = np.random.default_rng(seed).standard_normal(shape, dtype=np.float32)
    return port.e4m3_from_f32(x, scale)


@pytest.mark.parametrize("dtype,pairing,k_scale,v_scale", [("bf16", 1, 0.25, 0.5), ("f16", 1, 0.037, 0.11),
                                                           ("bf16", 0, 1.0, 1.0)])
def test_fp8_rope_append_matches_oracle(dtype, pairing, k_scale, v_scale):
    b, hq, hkv, hd, s = 4, 8, 2, 128, 256
    td = TORCH[dtype]
    r = ochain.rounder(dtype)
    g = np.random.default_rng(1)
    qkv = r(g.standard_normal((b, (hq + 2 * hkv) * hd), dtype=np.float32))
    kv_lens = np.array([s, 1, 100, 37], np.uint32)        # after the update: rows 255, 0, 99, 36
    is_done = np.array([0, 0, 0, 1], np.uint8)
    k8 = _cache_bytes((b, hkv, s, hd), k_scale, 2)
    v8 = _cache_bytes((b, hkv, s, hd), v_scale, 3)
    dk, dv = torch.from_numpy(k8).cuda(), torch.from_numpy(v8).cuda()
    dqkv = torch.from_numpy(qkv).cuda().to(td)
    dkl, ddone = torch.from_numpy(kv_lens).cuda(), torch.from_numpy(is_done).cuda()
    q8 = torch.zeros(b, hq, 1, hd, dtype=td, device="cuda")
    ops.launch_rope_kvcache_fp8_decode(dqkv, ddone, dkl, q8, dk, dv, k_scale, v_scale, pairing=pairing)
    # the 16-bit operator's q on the same input
    q16 = torch.zeros_like(q8)
    k16 = torch.zeros(b, hkv, s, hd, dtype=td, device="cuda")
    rope = ops.launch_fused_reshape_rope_kvcache_llama2_decode if pairing else ops.launch_fused_reshape_rope_kvcache_decode
    rope(dqkv, ddone, dkl, q16, k16, torch.zeros_like(k16))
    torch.cuda.synchronize()
    assert bits_equal(host(q8), host(q16))
    want_k, want_v = k8.copy(), v8.copy()
    heads = qkv.reshape(b, hq + 2 * hkv, hd)
    for i in range(b):
        if is_done[i]:
            continue
        pos = int(kv_lens[i]) - 1
        for j in range(hkv):
            rot = port.rotate_one_head(pairing, heads[i, hq + j], pos, int(kv_lens[i]))
            want_k[i, j, pos] = port.e4m3_from_f32(rot, k_scale)
            want_v[i, j, pos] = port.e4m3_from_f32(heads[i, hq + hkv + j], v_scale)
    assert bits_equal(host(dk), want_k)
    assert bits_equal(host(dv), want_v)


@pytest.mark.parametrize("dtype,hd,b,hq,hkv,kv", [
    ("bf16", 128, 4, 8, 2, [4096, 1, 2000, 129]),   # 7B-length rows, GQA, a single key, a partial block
    ("f16", 128, 2, 4, 4, [333, 1024]),
    ("bf16", 64, 2, 4, 1, [700, 64]),               # 64-byte rows (256 rows per block)
])
def test_fp8_decode_attention_matches_oracle(dtype, hd, b, hq, hkv, kv):
    s = max(4096, max(kv))
    td = TORCH[dtype]
    r = ochain.rounder(dtype)
    k_scale, v_scale = 0.21, 0.6
    k8 = _cache_bytes((b, hkv, s, hd), k_scale, 5)
    v8 = _cache_bytes((b, hkv, s, hd), v_scale, 6)
    q = r(np.random.default_rng(7).standard_normal((b, hq, 1, hd), dtype=np.float32))
    dq = torch.from_numpy(q).cuda().to(td)
    kv_lens = torch.tensor(kv, dtype=torch.uint32, device="cuda")
    mx = torch.tensor([max(kv)], dtype=torch.uint32, device="cuda")
    qk = torch.full((b, hq, 1, s), 5.0, dtype=td, device="cuda")
    out = torch.zeros(b, hq, 1, hd, dtype=td, device="cuda")
    ops.decode_attention_fp8(dq, torch.from_numpy(k8).cuda(), torch.from_numpy(v8).cuda(), k_scale, v_scale, kv_lens,
                             mx, qk, out)
    torch.cuda.synchronize()
    got_qk, got_o = host(qk), host(out)
    group = hq // hkv
    for i in range(b):
        n = kv[i]
        for h in range(hq):
            kd = port.e4m3_to_f32(k8[i, h // group, :n], k_scale)
            vd = port.e4m3_to_f32(v8[i, h // group, :n], v_scale)
            want = ochain.score_row(q[i, h, 0], kd, n - 1, hd)
            assert max_rel_err(got_qk[i, h, 0, :n], r(want)) <= 1e-2, (i, h)
            assert not np.any(got_qk[i, h, 0, n:max(kv)]), "keys past the row's length are written as 0"
            o = port.linear(want.reshape(1, -1), vd, False, False, 1, hd, n).reshape(-1)
            err = float(np.abs(got_o[i, h, 0] - r(o)).max() / max(np.abs(o).max(), 1e-30))
            assert err <= 1e-2, (i, h, err)
    assert np.all(got_qk[..., max(kv):] == 5.0), "keys past max_kv are not written"


def test_fp8_paged_matches_contiguous():
    b, hq, hkv, hd, max_pages = 3, 8, 2, 128, 12
    rows = 16384 // hd
    assert int(capi.lib().l2k_paged_block_rows(hd, 3)) == rows
    s = max_pages * rows
    k8 = _cache_bytes((b, hkv, s, hd), 0.3, 8)
    v8 = _cache_bytes((b, hkv, s, hd), 0.4, 9)
    n_pages = b * max_pages + 4
    perm = np.random.default_rng(10).permutation(n_pages)[: b * max_pages].reshape(b, max_pages).astype(np.uint32)
    kp = _cache_bytes((n_pages, hkv, rows, hd), 1.0, 11)
    vp = _cache_bytes((n_pages, hkv, rows, hd), 1.0, 12)
    for i in range(b):
        for j in range(max_pages):
            kp[perm[i, j]] = k8[i, :, j * rows:(j + 1) * rows]
            vp[perm[i, j]] = v8[i, :, j * rows:(j + 1) * rows]
    q = torch.randn(b, hq, 1, hd, device="cuda").to(torch.bfloat16)
    kv = [s, 3, rows + 17]
    kv_lens = torch.tensor(kv, dtype=torch.uint32, device="cuda")
    mx = torch.tensor([max(kv)], dtype=torch.uint32, device="cuda")
    qk1 = torch.zeros(b, hq, 1, s, dtype=torch.bfloat16, device="cuda")
    qk2 = torch.zeros_like(qk1)
    o1 = torch.zeros(b, hq, 1, hd, dtype=torch.bfloat16, device="cuda")
    o2 = torch.zeros_like(o1)
    ops.decode_attention_fp8(q, torch.from_numpy(k8).cuda(), torch.from_numpy(v8).cuda(), 0.3, 0.4, kv_lens, mx, qk1,
                             o1)
    ops.decode_attention_fp8_paged(q, torch.from_numpy(kp).cuda(), torch.from_numpy(vp).cuda(), 0.3, 0.4,
                                   torch.from_numpy(perm).cuda(), kv_lens, mx, qk2, o2)
    torch.cuda.synchronize()
    assert bits_equal(host(qk1), host(qk2))
    assert bits_equal(host(o1), host(o2))


def test_fp8_rejects_bad_arguments():
    b, hq, hkv, hd, s = 1, 2, 2, 96, 64
    q = torch.zeros(b, hq, 1, hd, dtype=torch.bfloat16, device="cuda")
    k = torch.zeros(b, hkv, s, hd, dtype=torch.uint8, device="cuda")
    kv = torch.ones(1, dtype=torch.uint32, device="cuda")
    qk = torch.zeros(b, hq, 1, s, dtype=torch.bfloat16, device="cuda")
    o = torch.zeros_like(q)
    with pytest.raises(capi.L2KError):   # head_dim 96: not a whole number of 16-byte slices per lane group
        ops.decode_attention_fp8(q, k, k, 1.0, 1.0, kv, kv, qk, o)
    with pytest.raises(capi.L2KError):   # scale must be positive
        ops.decode_attention_fp8(q[..., :64].contiguous(), k[..., :64].contiguous(), k[..., :64].contiguous(), 0.0,
                                 1.0, kv, kv, qk, o[..., :64].contiguous())


def test_fp8_attention_q_values_outside_the_f16_range():
    """The K dot product takes q as f16 pairs only when every value of a
    lane's slice converts exactly; slices holding values below the normal f16
    range or above its largest value take the fp32 path. Both against the
    oracle."""
    b, hq, hkv, hd = 1, 4, 1, 128
    s, n = 512, 300
    r = ochain.rounder("bf16")
    k8 = _cache_bytes((b, hkv, s, hd), 0.002, 13)
    v8 = _cache_bytes((b, hkv, s, hd), 0.5, 14)
    q = np.random.default_rng(15).standard_normal((b, hq, 1, hd), dtype=np.float32) * 0.01
    q[0, 1, 0, 3] = 3e-6          # below the normal f16 range
    q[0, 2, 0, 70] = 9.0e4        # above the largest f16 value
    q[0, 3, 0, :] = 0.0           # all zero: uniform probabilities
    q = r(q)
    qk = torch.zeros(b, hq, 1, s, dtype=torch.bfloat16, device="cuda")
    out = torch.zeros(b, hq, 1, hd, dtype=torch.bfloat16, device="cuda")
    kv = torch.tensor([n], dtype=torch.uint32, device="cuda")
    ops.decode_attention_fp8(torch.from_numpy(q).cuda().to(torch.bfloat16), torch.from_numpy(k8).cuda(),
                             torch.from_numpy(v8).cuda(), 0.002, 0.5, kv, kv, qk, out)
    torch.cuda.synchronize()
    for h in range(hq):
        kd = port.e4m3_to_f32(k8[0, 0, :n], 0.002)
        want = ochain.score_row(q[0, h, 0], kd, n - 1, hd)
        assert max_rel_err(host(qk)[0, h, 0, :n], r(want)) <= 1e-2, h
