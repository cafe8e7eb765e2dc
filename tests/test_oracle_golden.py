"""The oracle (oracle/oracle.c) against the reference's own outputs.

The fixtures in tests/golden/ were produced by the reference's CPU test
helpers compiled from its own sources (tests/golden/make_golden.py). The C
restatement must reproduce every one of them bit-exactly: same inputs, same
float operation order, same libm. CPU only.
"""
import numpy as np
import pytest

from oracle import port
from tests import golden_io

F32 = np.float32


def _bits_equal(a, b):
    a = np.ascontiguousarray(a)
    b = np.ascontiguousarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype, (a.shape, b.shape, a.dtype, b.dtype)
    return np.array_equal(a.view(np.uint8), b.view(np.uint8))


@pytest.mark.parametrize("case", golden_io.case_ids("embedding"))
def test_embedding(case):
    _, a = golden_io.load("embedding")[case]
    assert _bits_equal(port.embedding(a["ids"], a["table"]), a["out"])


@pytest.mark.parametrize("case", golden_io.case_ids("rmsnorm"))
def test_rmsnorm(case):
    p, a = golden_io.load("rmsnorm")[case]
    x_after, res_out = port.fused_add_residual_rmsnorm(a["x"], a["residual"], a["w"], p["add"])
    assert _bits_equal(x_after, a["x_after"])
    assert _bits_equal(res_out, a["residual_out"])


@pytest.mark.parametrize("case", golden_io.case_ids("rope_decode"))
def test_rope_decode(case):
    p, a = golden_io.load("rope_decode")[case]
    q = np.zeros_like(a["q"])
    k = np.zeros_like(a["k"])
    v = np.zeros_like(a["v"])
    port.rope_kvcache_decode(p["pairing"], a["input"], a["is_done"], a["kv_lens"], q, k, v)
    for got, want in ((q, a["q"]), (k, a["k"]), (v, a["v"])):
        assert _bits_equal(got, want)


@pytest.mark.parametrize("case", golden_io.case_ids("rope_prefill"))
def test_rope_prefill(case):
    p, a = golden_io.load("rope_prefill")[case]
    unpad, _ = port.build_padding_index_maps(a["q_lens"], p["q_cache_len"])
    assert _bits_equal(unpad, a["unpad_to_pad"])
    q = np.zeros_like(a["q"])
    k = np.zeros_like(a["k"])
    v = np.zeros_like(a["v"])
    port.rope_kvcache_prefill(p["pairing"], a["input"], a["q_lens"], a["kv_lens"], a["unpad_to_pad"], q, k, v)
    for got, want in ((q, a["q"]), (k, a["k"]), (v, a["v"])):
        assert _bits_equal(got, want)


INTEGER = golden_io.load("integer")


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("mask.")))
def test_causal_mask(case):
    p, a = INTEGER[case]
    mask = np.zeros_like(a["mask"])
    port.build_causal_mask(a["q_lens"], a["kv_lens"], p["max_q"], p["max_kv"], mask)
    assert _bits_equal(mask, a["mask"])


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("maps.")))
def test_padding_maps(case):
    p, a = INTEGER[case]
    unpad, offs = port.build_padding_index_maps(a["seq_lens"], p["q_cache_len"])
    assert _bits_equal(unpad, a["unpad_to_pad"])
    assert _bits_equal(offs, a["seq_offsets"])


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("lens.")))
def test_update_lens(case):
    _, a = INTEGER[case]
    kv, mq, mkv = port.update_q_kv_lens(a["q_lens"], a["kv_lens"])
    assert _bits_equal(kv, a["kv_lens_out"])
    assert (mq, mkv) == (int(a["max_q"]), int(a["max_kv"]))


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("ptr.")))
def test_ptr_arrays(case):
    """Pointer expectations of test_build_q_k_v_qk_qkv_array.cu:84-130, recomputed."""
    p, _ = INTEGER[case]
    b, hq, hkv, qc, s, hs, es = (p[k] for k in ("batch", "q_heads", "kv_heads", "q_cache_len", "kv_cache_len",
                                                "head_size", "elem_size"))
    bases = np.arange(1, 9, dtype=np.uint64) << np.uint64(40)
    strides = np.array([qc * hs, hs, s * hs, s * hs, qc * s, s, qc * hs, hs], dtype=np.uint64) * np.uint64(es)
    out = port.build_ptr_arrays(bases, strides, b, hq, hkv)
    group = hq // hkv
    for bi in range(b):
        for qh in range(hq):
            idx = bi * hq + qh
            kv_idx = bi * hkv + qh // group
            assert out[0, idx] == bases[0] + idx * strides[0]
            assert out[2, idx] == bases[2] + kv_idx * strides[2]
            assert out[3, idx] == bases[3] + kv_idx * strides[3]
            assert out[5, idx] == bases[5] + idx * strides[5]


@pytest.mark.parametrize("case", golden_io.case_ids("linear"))
def test_linear(case):
    p, a = golden_io.load("linear")[case]
    m, n, k = p["M"], p["N"], p["K"]
    if p["batch"] == 0:
        got = port.linear(a["A"], a["B"], p["trans_a"], p["trans_b"], m, n, k)
    else:
        got = np.stack([port.linear(a["A"][i], a["B"][i], p["trans_a"], p["trans_b"], m, n, k)
                        for i in range(p["batch"])])
    assert _bits_equal(got, a["C"])


@pytest.mark.parametrize("case", golden_io.case_ids("score"))
def test_masked_attention_score(case):
    p, a = golden_io.load("score")[case]
    qk = a["qk"].astype(F32)
    port.masked_attention_score(qk, a["mask"], a["q_lens"], p["max_kv"], p["head_dim"])
    if p["dtype"] == "f32":
        assert _bits_equal(qk, a["expected"])
    else:
        # The f16 helper rounds each output to half; the oracle works in fp32.
        assert _bits_equal(qk.astype(np.float16), a["expected"])


@pytest.mark.parametrize("case", golden_io.case_ids("swiglu"))
def test_swiglu(case):
    _, a = golden_io.load("swiglu")[case]
    assert _bits_equal(port.swiglu(a["input"]), a["out"])


@pytest.mark.parametrize("case", golden_io.case_ids("unpad"))
def test_transpose_unpad(case):
    p, a = golden_io.load("unpad")[case]
    qkv = a["qkv"].astype(np.float16) if p["dtype"] == "f16" else a["qkv"]
    got = port.transpose_unpad(qkv, a["unpad_to_pad"].reshape(-1), p["num_input_tokens"])
    assert _bits_equal(got.astype(F32), a["out"])


@pytest.mark.parametrize("case", golden_io.case_ids("attention_qkv"))
def test_attention_qkv(case):
    p, a = golden_io.load("attention_qkv")[case]
    got = np.full_like(a["qkv"], -7.0)
    port.attention_qkv(a["qk"], a["v"], p["m"], p["n"], got)
    assert _bits_equal(got, a["qkv"])


def test_e4m3_oracle_rounding():
    """The oracle's e4m3 rounding (round to nearest even, saturating) against
    torch's float8_e4m3fn conversion on in-range values (normals, subnormals,
    ties), and its exact decoding of every byte."""
    import torch

    from oracle import port

    rng = np.random.default_rng(0)
    x = (rng.standard_normal(100000) * np.exp(rng.uniform(-14, 6, 100000))).astype(np.float32)
    ties = np.array([m * 2.0 ** -9 for m in np.arange(0.5, 8, 1.0)] + [1.0625, 1.1875, 240.0, 416.0], np.float32)
    for scale in (1.0, 0.37, 3.1):
        inv = np.float32(1) / np.float32(scale)
        xs = np.concatenate([x[np.abs(x * inv) < 448], ties * np.float32(scale)])
        want = torch.from_numpy(xs * inv).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
        assert np.array_equal(port.e4m3_from_f32(xs, scale), want)
    assert port.e4m3_from_f32(np.array([500.0, -1e6, 448.0], np.float32), 1.0).tolist() == [0x7E, 0xFE, 0x7E]
    vals = port.e4m3_to_f32(np.arange(256, dtype=np.uint8), 1.0)
    want = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).float().numpy()
    assert np.array_equal(np.isnan(vals), np.isnan(want)) and np.array_equal(vals[~np.isnan(vals)], want[~np.isnan(want)])
