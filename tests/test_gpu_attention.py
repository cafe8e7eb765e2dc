"""Attention output on the GPU: the transpose + unpad copy and P.V, through
the C ABI, against the oracle (oracle/oracle.c) and the reference's own
test cases (tests/golden/unpad.npz, attention_qkv.npz).

Bars: the unpad copy is byte-exact; P.V is within 1e-5 relative (fp32) or
1e-2 (16-bit I/O) of the oracle, relative to the largest magnitude of the
output row (the terms of a P.V sum have both signs, so single elements can
cancel to near zero).
"""
import numpy as np
import pytest
import torch

from llama2_b200 import ops
from oracle import chain as ochain
from oracle import port
from tests import golden_io
from tests.gpu_util import TORCH, dev, host, max_rel_err

pytestmark = pytest.mark.gpu

@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


# ---------------------------------------------------------------------------
# transpose + unpad
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("case", golden_io.case_ids("unpad"))
def test_unpad_golden(case):
    p, a = golden_io.load("unpad")[case]
    dt = TORCH[p["dtype"]]
    qkv = dev(a["qkv"], dt)
    idx = dev(a["unpad_to_pad"].reshape(-1))
    t = p["num_input_tokens"]
    out = torch.zeros(t, qkv.shape[1] * qkv.shape[3], dtype=dt, device="cuda")
    ops.launch_fused_transpose_unpad(t, qkv, idx, out)
    assert np.array_equal(host(out), a["out"])


def _slots(q_lens, qc):
    """unpad_to_pad_idx as the reference builds it: token t of sequence b -> b * qc + t."""
    out = np.zeros(len(q_lens) * qc, np.uint32)
    off = 0
    for b, n in enumerate(q_lens):
        out[off:off + n] = b * qc + np.arange(n, dtype=np.uint32)
        off += n
    return out, off


def _bits(t):
    t = t.detach().cpu()
    if t.dtype == torch.float32:
        return t.view(torch.int32).numpy()
    return t.view(torch.int16).numpy()


@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
@pytest.mark.parametrize("b,h,qc,hd,lens", [
    (3, 4, 16, 16, [2, 5, 3]),
    (8, 32, 64, 128, [64, 1, 17, 0, 33, 64, 5, 2]),   # 7B heads, ragged, an empty sequence
    (2, 3, 5, 6, [5, 4]),                             # 12- and 24-byte head rows: the 2-byte path
    (64, 32, 1, 128, [1] * 64),                       # decode: one token per sequence
])
def test_unpad_matches_oracle(dt, b, h, qc, hd, lens):
    g = torch.Generator().manual_seed(0)
    qkv = torch.randn(b, h, qc, hd, generator=g).to(TORCH[dt]).cuda()
    slots, t = _slots(lens, qc)
    out = torch.full((max(t, 1), h * hd), 7.0, dtype=TORCH[dt], device="cuda")
    ops.launch_fused_transpose_unpad(t, qkv, dev(slots), out)
    torch.cuda.synchronize()
    want = port.transpose_unpad(_bits(qkv), slots, t)
    assert np.array_equal(_bits(out)[:t], want)
    if t == 0:
        assert torch.all(out == 7.0)


def test_unpad_out_of_range_slot_gives_zero_row():
    qkv = torch.randn(2, 2, 4, 8, device="cuda")
    slots = np.array([1, 9, 4, 7], np.uint32)  # 9 >= batch * q_cache_len = 8
    out = torch.full((4, 16), 3.0, device="cuda")
    ops.launch_fused_transpose_unpad(4, qkv, dev(slots), out)
    got = host(out)
    want = port.transpose_unpad(host(qkv), slots, 4)
    assert np.array_equal(got, want)
    assert not got[1].any()


def test_unpad_unaligned_base_takes_the_narrow_path():
    # A view whose base is 4 bytes past a 16-byte boundary (fp32, hd = 8).
    buf = torch.randn(1 + 2 * 3 * 4 * 8, device="cuda")
    qkv = buf[1:].view(2, 3, 4, 8)
    slots = np.array([0, 1, 4, 6, 7], np.uint32)
    out = torch.empty(5, 24, device="cuda")
    ops.launch_fused_transpose_unpad(5, qkv, dev(slots), out)
    assert np.array_equal(host(out), port.transpose_unpad(host(qkv), slots, 5))


def test_unpad_full_prefill_size_round_trip():
    # 8 x 2048 tokens at 7B dims in bf16 (268 MB each way): every output row
    # is the padded row its slot names (a torch gather of the same rows).
    b, h, qc, hd = 8, 32, 2048, 128
    qkv = torch.randn(b, h, qc, hd, device="cuda", dtype=torch.bfloat16)
    lens = [2048, 1500, 2048, 7, 2048, 1024, 2048, 333]
    slots, t = _slots(lens, qc)
    out = torch.empty(t, h * hd, device="cuda", dtype=torch.bfloat16)
    ops.launch_fused_transpose_unpad(t, qkv, dev(slots), out)
    s = torch.from_numpy(slots[:t].astype(np.int64)).cuda()
    want = qkv.permute(0, 2, 1, 3).reshape(b * qc, h * hd).index_select(0, s)
    assert torch.equal(out, want)


# ---------------------------------------------------------------------------
# P.V and the fused decode attention
# ---------------------------------------------------------------------------
REL = {"f32": 1e-5, "bf16": 1e-2, "f16": 1e-2}


def _row_rel_err(got, want):
    """max |got - want| / max |want| per output row (the last axis)."""
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.maximum(np.abs(want).max(axis=-1, keepdims=True), 1e-30)
    return float((np.abs(got - want) / scale).max()) if want.size else 0.0


@pytest.mark.parametrize("case", golden_io.case_ids("attention_qkv"))
def test_attention_qkv_golden(case):
    p, a = golden_io.load("attention_qkv")[case]
    qk, v = dev(a["qk"]), dev(a["v"])
    out = torch.full(a["qkv"].shape, -7.0, device="cuda")
    ops.launch_attention_qkv(qk, v, out, p["m"], p["n"])
    got = host(out)
    assert _row_rel_err(got, a["qkv"]) <= 1e-5
    assert np.all(got[:, :, p["m"]:] == -7.0), "rows >= m are left as is"


def _attention_oracle(q, k, v, kv_lens, max_kv):
    """Probabilities (keys < max_kv) and P.V of the chain oracle's helpers."""
    b, hq, _, hd = q.shape
    s = k.shape[2]
    ones = np.ones(b, np.uint32)
    qk = np.zeros((b, hq, 1, s), np.float32)
    port.qk_scores(q, k, 1, max_kv, qk)
    mask = ochain.intended_mask(ones, kv_lens, 1, max_kv, 1, s)
    port.masked_attention_score(qk, mask, ones, max_kv, hd)
    out = np.zeros((b, hq, 1, hd), np.float32)
    port.attention_qkv(qk, v, 1, max_kv, out)
    return qk, out


def _run_decode_attention(dt, b, hq, hkv, s, hd, kv_lens, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    td = TORCH[dt]
    q = torch.randn(b, hq, 1, hd, generator=g, device="cuda").to(td)
    k = torch.randn(b, hkv, s, hd, generator=g, device="cuda").to(td)
    v = torch.randn(b, hkv, s, hd, generator=g, device="cuda").to(td)
    kv = torch.tensor(kv_lens, dtype=torch.uint32, device="cuda")
    mx = torch.tensor([max(kv_lens)], dtype=torch.uint32, device="cuda")
    qk = torch.full((b, hq, 1, s), 7.0, dtype=td, device="cuda")
    qkv = torch.full((b, hq, 1, hd), 7.0, dtype=td, device="cuda")
    ops.decode_attention(q, k, v, kv, mx, qk, qkv)
    torch.cuda.synchronize()
    return q, k, v, kv, mx, qk, qkv


@pytest.mark.parametrize("dt,b,hq,hkv,s,hd,kv_lens", [
    ("f32", 3, 4, 4, 1000, 128, [700, 3, 1000]),       # 512-byte K/V rows, a row at the cache end
    ("bf16", 2, 8, 2, 4096, 128, [4096, 1]),           # 256-byte rows, GQA, one key
    ("f16", 3, 4, 2, 777, 64, [777, 400, 33]),         # 128-byte rows, a ragged last block
    ("f32", 2, 2, 1, 300, 16, [300, 17]),              # 64-byte rows
    ("f32", 2, 6, 6, 256, 48, [200, 256]),             # 192-byte rows: score operator + P.V kernel
    ("bf16", 3, 4, 4, 512, 128, [0, 512, 5]),          # a sequence with no keys: a zero row
])
def test_decode_attention_matches_oracle(dt, b, hq, hkv, s, hd, kv_lens):
    q, k, v, kv, mx, qk, qkv = _run_decode_attention(dt, b, hq, hkv, s, hd, kv_lens)
    m = max(kv_lens)
    want_qk, want_out = _attention_oracle(host(q), host(k), host(v), np.array(kv_lens, np.uint32), m)
    got_qk = host(qk)
    tol = REL[dt]
    assert max_rel_err(got_qk[..., :m], want_qk[..., :m]) <= tol
    assert np.all(got_qk[..., m:] == 7.0), "keys >= max_kv_len are left as is"
    got = host(qkv)
    assert _row_rel_err(got, want_out) <= tol
    for bi, n in enumerate(kv_lens):
        if n == 0:
            assert not got[bi].any() and not got_qk[bi, ..., :m].any()


@pytest.mark.parametrize("dt", ["f32", "bf16"])
def test_decode_attention_is_scores_plus_attention_qkv(dt):
    """The fused operator's probabilities are bit-identical to the score
    operator's; its output equals P.V of those probabilities through the
    launch_linear call-site operator (within the fp32 summation-order bar)."""
    b, hq, hkv, s, hd = 4, 8, 8, 2048, 128
    kv_lens = [2048, 1500, 2, 999]
    q, k, v, kv, mx, qk, qkv = _run_decode_attention(dt, b, hq, hkv, s, hd, kv_lens, seed=3)
    qk2 = torch.full_like(qk, 7.0)
    ops.decode_attention_scores(q, k, kv, mx, qk2)
    out2 = torch.empty_like(qkv)
    ops.launch_attention_qkv(qk2, v, out2, 1, max(kv_lens))
    torch.cuda.synchronize()
    assert torch.equal(qk, qk2)
    # 16-bit: the fused output uses the fp32 probabilities, the call site the stored ones
    assert _row_rel_err(host(qkv), host(out2)) <= (1e-5 if dt == "f32" else 1e-2)


def test_decode_attention_7b_dims_against_oracle():
    """7B dims (32 heads x 128, 4096-key cache) at four sequences, bf16."""
    kv_lens = [4096, 2048, 1, 3333]
    q, k, v, kv, mx, qk, qkv = _run_decode_attention("bf16", 4, 32, 32, 4096, 128, kv_lens, seed=11)
    want_qk, want_out = _attention_oracle(host(q), host(k), host(v), np.array(kv_lens, np.uint32), 4096)
    assert max_rel_err(host(qk), want_qk) <= 1e-2
    assert _row_rel_err(host(qkv), want_out) <= 1e-2


def test_decode_attention_repeatable():
    """Fixed-order reductions: two runs give identical bits."""
    r1 = _run_decode_attention("f32", 8, 32, 32, 4096, 128, [4096] * 8, seed=5)
    r2 = _run_decode_attention("f32", 8, 32, 32, 4096, 128, [4096] * 8, seed=5)
    assert torch.equal(r1[-1], r2[-1]) and torch.equal(r1[-2], r2[-2])


# ---------------------------------------------------------------------------
# P.V on the tensor cores (16-bit, head_dim 128)
# ---------------------------------------------------------------------------
@pytest.mark.parametrize("dt,b,hq,hkv,qc,s,m,n", [
    ("bf16", 2, 4, 2, 256, 512, 256, 300),   # GQA, n not a multiple of the 64-key block
    ("f16", 1, 2, 2, 300, 256, 200, 64),     # a partial 128-row tile, one key block
    ("bf16", 3, 2, 1, 1, 1024, 1, 777),      # the decode call site (one row per head)
    ("f16", 2, 2, 2, 128, 64, 128, 1),       # one key
])
def test_attention_qkv_tensor_cores_against_oracle(dt, b, hq, hkv, qc, s, m, n):
    g = torch.Generator(device="cuda")
    g.manual_seed(n + qc)
    td = TORCH[dt]
    qk = torch.rand(b, hq, qc, s, generator=g, device="cuda").to(td)
    v = torch.randn(b, hkv, s, 128, generator=g, device="cuda").to(td)
    # entries the product must not read: keys >= n of qk and V rows >= n
    qk[..., n:] = float("nan")
    v[:, :, n:] = float("nan")
    out = torch.full((b, hq, qc, 128), 7.0, dtype=td, device="cuda")
    ops.launch_attention_qkv(qk, v, out, m, n)
    torch.cuda.synchronize()
    want = np.full((b, hq, qc, 128), 7.0, np.float32)
    port.attention_qkv(host(qk), host(v), m, n, want)
    got = host(out)
    assert np.isfinite(got).all()
    assert _row_rel_err(got[:, :, :m], want[:, :, :m]) <= 1e-2
    assert np.all(got[:, :, m:] == 7.0), "rows >= m are left as is"


def test_attention_qkv_tensor_cores_prefill_size_one_hot():
    """7B prefill shape (8 x 32 heads, 2048 x 2048 probabilities, bf16): with
    one-hot probability rows the product is exactly the selected V rows, so
    the whole output is checked bit for bit at full size."""
    b, h, qc, s = 8, 32, 2048, 2048
    g = torch.Generator(device="cuda")
    g.manual_seed(1)
    v = torch.randn(b, h, s, 128, generator=g, device="cuda", dtype=torch.bfloat16)
    sel = torch.randint(0, s, (b, h, qc), generator=g, device="cuda")
    qk = torch.zeros(b, h, qc, s, device="cuda", dtype=torch.bfloat16)
    qk.scatter_(3, sel.unsqueeze(-1), 1.0)
    out = torch.empty(b, h, qc, 128, device="cuda", dtype=torch.bfloat16)
    ops.launch_attention_qkv(qk, v, out, qc, s)
    want = torch.gather(v, 2, sel.unsqueeze(-1).expand(b, h, qc, 128))
    assert torch.equal(out, want)
