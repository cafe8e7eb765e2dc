"""Paged K/V caches (decode): the paged RoPE + append and the paged fused
decode attention against the contiguous operators on the same data.

A pool of pages (num_pages, Hkv, page_rows, hd) holds each sequence's cache
in pages scattered by a shuffled block table; gathering the pages back into
the (B, Hkv, S, hd) layout must give exactly the contiguous cache, and the
attention over the pages exactly the contiguous attention's bits (the same
blocks are streamed in the same order).
"""
import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from tests.gpu_util import bits_equal, host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    rows = ops.paged_block_rows(hd, dtype)
    s = max_pages * rows
    k = torch.randn(b, hkv, s, hd, generator=g, device="cuda").to(dtype)
    v = torch.randn(b, hkv, s, hd, generator=g, device="cuda").to(dtype)
    n_pages = b * max_pages + spare
    perm = torch.randperm(n_pages, generator=torch.Generator().manual_seed(seed))[: b * max_pages]
    table = perm.view(b, max_pages).to(torch.int32)
    kp = torch.randn(n_pages, hkv, rows, hd, generator=g, device="cuda").to(dtype)
    vp = torch.randn(n_pages, hkv, rows, hd, generator=g, device="cuda").to(dtype)
    for bi in range(b):
        for j in range(max_pages):
            p = int(table[bi, j])
            kp[p] = k[bi, :, j * rows:(j + 1) * rows]
            vp[p] = v[bi, :, j * rows:(j + 1) * rows]
    return k, v, kp, vp, table.cuda(), rows


def _gather(pages, table, rows):
    b, max_pages = table.shape
    out = []
    for bi in range(b):
        out.append(torch.cat([pages[int(table[bi, j])] for j in range(max_pages)], dim=1))
    return torch.stack(out)


@pytest.mark.parametrize("dtype,pairing", [(torch.float32, 1), (torch.bfloat16, 1), (torch.bfloat16, 0)])
def test_paged_rope_append_matches_contiguous(dtype, pairing):
    b, hq, hkv, hd, max_pages = 3, 8, 2, 128, 6
    k, v, kp, vp, table, rows = _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare=5, seed=1)
    s = max_pages * rows
    g = torch.Generator(device="cuda")
    g.manual_seed(3)
    qkv = torch.randn(b, (hq + 2 * hkv) * hd, generator=g, device="cuda").to(dtype)
    kv_lens = torch.tensor([s, 1, rows + 5], dtype=torch.uint32, device="cuda")   # last row, first row, page 2
    is_done = torch.tensor([0, 0, 0], dtype=torch.uint8, device="cuda")
    q1 = torch.zeros(b, hq, 1, hd, dtype=dtype, device="cuda")
    q2 = torch.zeros_like(q1)
    rope = ops.launch_fused_reshape_rope_kvcache_llama2_decode if pairing else ops.launch_fused_reshape_rope_kvcache_decode
    rope(qkv, is_done, kv_lens, q1, k, v)
    ops.launch_rope_kvcache_paged_decode(qkv, is_done, kv_lens, q2, kp, vp, table, pairing=pairing)
    torch.cuda.synchronize()
    assert bits_equal(host(q1), host(q2))
    assert bits_equal(host(_gather(kp, table, rows)), host(k))
    assert bits_equal(host(_gather(vp, table, rows)), host(v))


@pytest.mark.parametrize("dtype,b,hq,hkv,max_pages,kv", [
    (torch.float32, 3, 4, 4, 40, [1280, 7, 640]),     # 32-row pages, a full cache, one partial page
    (torch.bfloat16, 4, 8, 2, 64, [4096, 1, 2000, 64]),  # 64-row pages, GQA, 7B-length caches
])
def test_paged_attention_matches_contiguous(dtype, b, hq, hkv, max_pages, kv):
    hd = 128
    k, v, kp, vp, table, rows = _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare=3, seed=7)
    s = max_pages * rows
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    q = torch.randn(b, hq, 1, hd, generator=g, device="cuda").to(dtype)
    kv_lens = torch.tensor(kv, dtype=torch.uint32, device="cuda")
    mx = torch.tensor([max(kv)], dtype=torch.uint32, device="cuda")
    qk1 = torch.full((b, hq, 1, s), 7.0, dtype=dtype, device="cuda")
    qk2 = torch.full_like(qk1, 7.0)
    o1 = torch.empty(b, hq, 1, hd, dtype=dtype, device="cuda")
    o2 = torch.empty_like(o1)
    ops.decode_attention(q, k, v, kv_lens, mx, qk1, o1)
    ops.decode_attention_paged(q, kp, vp, table, kv_lens, mx, qk2, o2)
    torch.cuda.synchronize()
    assert bits_equal(host(qk1), host(qk2))
    assert bits_equal(host(o1), host(o2))


def test_paged_attention_page_past_the_pool_is_an_error_not_a_read():
    """A block-table entry past the pool reads page 0 and records an error
    code (l2k_device_error), without touching memory outside the pool."""
    dtype, b, hq, hkv, hd, max_pages = torch.float32, 2, 2, 2, 128, 4
    k, v, kp, vp, table, rows = _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare=0, seed=2)
    capi.lib().l2k_device_error(1)
    table[1, 1] = 1 << 20  # used by sequence 1 (kv_len covers page 1)
    q = torch.randn(b, hq, 1, hd, device="cuda")
    kv_lens = torch.tensor([rows, 2 * rows], dtype=torch.uint32, device="cuda")
    mx = torch.tensor([2 * rows], dtype=torch.uint32, device="cuda")
    qk = torch.zeros(b, hq, 1, max_pages * rows, device="cuda")
    o = torch.empty(b, hq, 1, hd, device="cuda")
    ops.decode_attention_paged(q, kp, vp, table, kv_lens, mx, qk, o)
    torch.cuda.synchronize()
    assert capi.lib().l2k_device_error(1) == 0x206
    assert np.isfinite(host(qk)).all() and np.isfinite(host(o)).all()


# ---------------------------------------------------------------------------
# Paged prefill: RoPE + append, tensor-core scores and P.V over paged caches
# ---------------------------------------------------------------------------
def _prefill_inputs(dtype, q_lens, hist, hq, hkv, hd, seed):
    from oracle import port
    b = len(q_lens)
    qc = max(q_lens)
    ql = np.asarray(q_lens, np.uint32)
    unpad, _ = port.build_padding_index_maps(ql, qc)
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    t = int(ql.sum())
    qkv = torch.randn(t, (hq + 2 * hkv) * hd, generator=g, device="cuda").to(dtype)
    q_lens_d = torch.tensor(q_lens, dtype=torch.uint32, device="cuda")
    kv_lens_d = torch.tensor([h + q for h, q in zip(hist, q_lens)], dtype=torch.uint32, device="cuda")
    return qkv, q_lens_d, kv_lens_d, torch.from_numpy(unpad.astype(np.uint32)).cuda(), qc


@pytest.mark.parametrize("dtype,pairing", [(torch.bfloat16, 1), (torch.float32, 0), (torch.float16, 1)])
def test_paged_prefill_rope_append_matches_contiguous(dtype, pairing):
    """Ragged prompts after a history: every token's K/V row lands on its page
    and q is the padded q of the contiguous operator, bit for bit."""
    b, hq, hkv, hd, max_pages = 3, 8, 2, 128, 8
    k, v, kp, vp, table, rows = _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare=4, seed=11)
    s = max_pages * rows
    q_lens, hist = [5, rows + 7, 2 * rows], [0, rows - 3, s - 2 * rows]
    qkv, ql, kl, unpad, qc = _prefill_inputs(dtype, q_lens, hist, hq, hkv, hd, seed=12)
    q1 = torch.zeros(b, hq, qc, hd, dtype=dtype, device="cuda")
    q2 = torch.zeros_like(q1)
    rope = (ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2 if pairing
            else ops.launch_fused_pad_reshape_transpose_rope_kvcache)
    rope(qkv, ql, kl, unpad, q1, k, v)
    ops.launch_rope_kvcache_paged_prefill(qkv, ql, kl, unpad, q2, kp, vp, table, pairing=pairing)
    torch.cuda.synchronize()
    assert bits_equal(host(q1), host(q2))
    assert bits_equal(host(_gather(kp, table, rows)), host(k))
    assert bits_equal(host(_gather(vp, table, rows)), host(v))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("q_lens,hist", [([128, 77, 300], [0, 100, 212]),   # ragged, with history
                                         ([256, 256], [0, 0])])              # fresh prompts, whole tiles
def test_paged_prefill_scores_and_pv_match_contiguous(dtype, q_lens, hist):
    """The tensor-core scores over a shuffled page pool equal the contiguous
    scores bit for bit (the same tiles, two pages per 128-key tile), and P.V
    over paged V equals the contiguous P.V."""
    b, hq, hkv, hd, max_pages = len(q_lens), 8, 2, 128, 10
    k, v, kp, vp, table, rows = _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare=5, seed=21)
    assert rows == 64
    s = max_pages * rows
    qc = max(q_lens)
    g = torch.Generator(device="cuda")
    g.manual_seed(22)
    q = torch.randn(b, hq, qc, hd, generator=g, device="cuda").to(dtype)
    ql = torch.tensor(q_lens, dtype=torch.uint32, device="cuda")
    kv = [h + x for h, x in zip(hist, q_lens)]
    kl = torch.tensor(kv, dtype=torch.uint32, device="cuda")
    max_q, max_kv = max(q_lens), max(kv)
    p1 = torch.full((b, hq, qc, s), 3.0, dtype=dtype, device="cuda")
    p2 = p1.clone()
    ops.prefill_attention_scores(q, k, ql, kl, max_q, max_kv, p1)
    ops.prefill_attention_scores_paged(q, kp, table, ql, kl, max_q, max_kv, p2)
    torch.cuda.synchronize()
    assert bits_equal(host(p1), host(p2))
    o1 = torch.zeros(b, hq, qc, hd, dtype=dtype, device="cuda")
    o2 = torch.zeros_like(o1)
    ops.launch_attention_qkv(p1, v, o1, max_q, max_kv)
    ops.launch_attention_qkv_paged(p2, vp, table, kl, o2, max_q, max_kv)
    torch.cuda.synchronize()
    # Rows i < q_len of each sequence (the rows the scores defined; rows past
    # q_len hold whatever the buffer held, so their products are unspecified),
    # equal as numbers.
    for bi, n in enumerate(q_lens):
        assert torch.equal(o1[bi, :, :n].float(), o2[bi, :, :n].float()), bi
    assert capi.lib().l2k_device_error(1) == 0


def test_paged_prefill_rejects_shapes_the_tensor_cores_do_not_take():
    b, hq, hkv, hd = 1, 2, 2, 64
    kp = torch.zeros(4, hkv, 64, hd, dtype=torch.bfloat16, device="cuda")
    table = torch.zeros(b, 2, dtype=torch.uint32, device="cuda")
    q = torch.zeros(b, hq, 64, hd, dtype=torch.bfloat16, device="cuda")
    ql = torch.tensor([64], dtype=torch.uint32, device="cuda")
    qk = torch.zeros(b, hq, 64, 128, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(capi.L2KError):
        ops.prefill_attention_scores_paged(q, kp, table, ql, ql, 64, 64, qk)


@pytest.mark.parametrize("dtype,b,hq,hkv,max_pages,kv,attention,pairing", [
    (torch.float32, 3, 4, 4, 12, [383, 0, 31], False, 1),            # last position, first, a page's last row
    (torch.bfloat16, 4, 8, 2, 16, [1023, 64, 500, 7], False, 1),     # GQA, a fresh page at 64
    (torch.bfloat16, 4, 8, 8, 16, [1000, 63, 1023, 300], True, 0),   # with the attention output, interleaved pairs
    (torch.float32, 2, 4, 2, 10, [319, 32], True, 1),
])
def test_paged_decode_step_matches_contiguous(dtype, b, hq, hkv, max_pages, kv, attention, pairing):
    """The one-launch decode step over page pools (shuffled block table)
    against the same step on the contiguous caches the pages form: every
    output bit-identical, and the appended K/V rows land in the right page."""
    hd, F, V = 128, 256, 500
    D = hq * hd
    k, v, kp, vp, table, rows = _paged_setup(dtype, b, hq, hkv, hd, max_pages, spare=4, seed=b + hkv)
    s = max_pages * rows
    g = torch.Generator(device="cuda")
    g.manual_seed(11)

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device="cuda") * scale).to(dtype)

    base = dict(q_lens=torch.ones(b, dtype=torch.uint32, device="cuda"),
                input_ids=torch.randint(0, V, (b,), generator=torch.Generator().manual_seed(2)).to(torch.uint32).cuda(),
                embed_table=rnd(V, D, scale=0.02), norm_weight=(torch.rand(D, generator=g, device="cuda") + 0.5).to(dtype),
                qkv=rnd(b, (hq + 2 * hkv) * hd), is_done=torch.zeros(b, dtype=torch.uint8, device="cuda"),
                gate_up=rnd(b, 2 * F))
    base["is_done"][-1] = 1  # a finished sequence: not rotated or appended
    kv0 = torch.tensor(kv, dtype=torch.uint32, device="cuda")

    def outs():
        return dict(kv_lens=kv0.clone(), max_lens=torch.zeros(2, dtype=torch.uint32, device="cuda"),
                    x=torch.empty(b, D, dtype=dtype, device="cuda"), normed=torch.empty(b, D, dtype=dtype, device="cuda"),
                    q=torch.zeros(b, hq, 1, hd, dtype=dtype, device="cuda"),
                    qk=torch.full((b, hq, 1, s), 7.0, dtype=dtype, device="cuda"),
                    ffn_out=torch.empty(b, F, dtype=dtype, device="cuda"))

    ws = ops.decode_step_workspace(torch.device("cuda"))
    c, p = outs(), outs()
    attn_c = torch.zeros(b, hq, 1, hd, dtype=dtype, device="cuda") if attention else None
    attn_p = torch.zeros_like(attn_c) if attention else None
    if attention:
        ops.decode_step_attention(**base, **c, k_cache=k, v_cache=v, workspace=ws, pairing=pairing, attn_out=attn_c)
    else:
        ops.decode_step(**base, **c, k_cache=k, v_cache=v, workspace=ws, pairing=pairing)
    ops.decode_step_paged(**base, **p, k_pages=kp, v_pages=vp, block_table=table, workspace=ws, pairing=pairing,
                          attn_out=attn_p)
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "normed", "q", "qk", "ffn_out"):
        assert bits_equal(host(c[n]), host(p[n])), n
    if attention:
        assert bits_equal(host(attn_c), host(attn_p))
    assert bits_equal(host(_gather(kp, table, rows)), host(k))
    assert bits_equal(host(_gather(vp, table, rows)), host(v))
    assert int(host(ws).astype(np.int64).sum()) == 0
    assert capi.lib().l2k_device_error(1) == 0
