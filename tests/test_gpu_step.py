"""The one-launch decode step (l2k_decode_step) on the GPU.

Against the chain oracle for consecutive steps and edge lengths, and against
this library's own operator sequence (each operator parity-tested against
the oracle elsewhere) for shapes the chain workloads do not cover (GQA).
Bars: bit-exact for the embedding rows, RoPE q, K/V cache rows, lengths and
maxima; max relative error <= 1e-5 fp32 / 1e-2 16-bit for RMSNorm, scores
and SwiGLU.
"""
import dataclasses

import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from llama2_b200.chain import Chain
from llama2_b200.workloads import WORKLOADS, host_inputs, with_batch
from oracle import chain as ochain
from tests.gpu_util import bits_equal, host, max_rel_err

pytestmark = pytest.mark.gpu

REL = {"f32": 1e-5, "bf16": 1e-2, "f16": 1e-2}


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield
    assert capi.lib().l2k_device_error(1) == 0


def check_against(ch, ref, tol, qk=True):
    assert bits_equal(host(ch.kv_lens).astype(np.uint32), ref["kv_lens"])
    mx = host(ch.max_lens)
    assert int(mx[0]) == ref["max_q"] and int(mx[1]) == ref["max_kv"]
    assert bits_equal(host(ch.x), ref["x"])
    assert max_rel_err(host(ch.normed), ref["normed"]) <= tol
    assert bits_equal(host(ch.q), ref["q"])
    assert bits_equal(host(ch.k_cache), ref["k"])
    assert bits_equal(host(ch.v_cache), ref["v"])
    if qk:
        assert max_rel_err(host(ch.qk), ref["qk"]) <= tol
    assert max_rel_err(host(ch.ffn_out), ref["ffn_out"], floor=1e-30) <= tol


@pytest.mark.parametrize("name,batch", [("7b-b1", 1), ("7b-b64", 3), ("7b-b64-bf16", 3)])
def test_consecutive_steps(name, batch):
    """Two steps back to back: the lengths advance twice, the second step sees
    the first step's K/V rows, and the workspace counter returns to zero."""
    w = with_batch(WORKLOADS[name], batch)
    inp = host_inputs(w, seed=11)
    ch = Chain(w, inp)
    assert ch.fused
    ch.step()
    ch.step()
    torch.cuda.synchronize()
    ref1 = ochain.decode_step(w, inp)
    inp2 = dict(inp, kv_lens=ref1["kv_lens"], k_cache=ref1["k"], v_cache=ref1["v"])
    ref2 = ochain.decode_step(w, inp2, qk_init=ref1["qk"])
    check_against(ch, ref2, REL[w.dtype])
    assert int(host(ch.workspace).astype(np.int64).sum()) == 0


@pytest.mark.parametrize("name", ["7b-b1", "7b-b64", "7b-b64-bf16", "13b-b256"])
def test_fused_equals_operator_sequence(name):
    """Bitwise equal to the operator sequence, except RMSNorm (different
    summation order, tolerance) — same kernels' arithmetic in one launch."""
    w = with_batch(WORKLOADS[name], 1 if name == "7b-b1" else 3)
    inp = host_inputs(w, seed=2)
    a, b = Chain(w, inp, fused=True), Chain(w, inp, fused=False)
    assert a.fused and not b.fused
    a.step()
    b.step()
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(getattr(a, n)), host(getattr(b, n))), n
    assert max_rel_err(host(a.normed), host(b.normed)) <= REL[w.dtype]


def test_edge_lengths():
    """Last cache row, an empty history, a finished sequence."""
    w = dataclasses.replace(with_batch(WORKLOADS["7b-b64"], 3), kv_cache_len=512)
    inp = host_inputs(w, seed=4)
    inp["kv_lens"] = np.array([511, 0, 100], np.uint32)
    inp["is_done"] = np.array([0, 0, 1], np.uint8)
    ch = Chain(w, inp)
    assert ch.fused
    ch.step()
    torch.cuda.synchronize()
    check_against(ch, ochain.decode_step(w, inp), 1e-5)


def test_position_past_cache_end_matches_operator_sequence():
    """kv_len + 1 > kv_cache_len: the token is not rotated or appended (the
    reference would write past the cache) and the row covers the whole cache."""
    w = dataclasses.replace(with_batch(WORKLOADS["7b-b64"], 4), kv_cache_len=256)
    inp = host_inputs(w, seed=6)
    inp["kv_lens"] = np.array([255, 256, 0, 100], np.uint32)
    inp["is_done"] = np.array([0, 0, 0, 1], np.uint8)
    a, b = Chain(w, inp, fused=True), Chain(w, inp, fused=False)
    a.step()
    b.step()
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(getattr(a, n)), host(getattr(b, n))), n


@pytest.mark.parametrize("dtype,pairing", [(torch.bfloat16, 1), (torch.float32, 0), (torch.float16, 1)])
def test_gqa_against_operator_sequence(dtype, pairing):
    """Grouped K/V heads (Hq = 8, Hkv = 2): the appended rows are written once
    per K/V head and every q head of the group scores against them."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    B, Hq, Hkv, hd, S, D, F, V = 3, 8, 2, 128, 1024, 1024, 512, 1000

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)

    base = dict(
        q_lens=torch.ones(B, dtype=torch.uint32, device=dev),
        input_ids=torch.tensor([5, 999, 1234], dtype=torch.uint32, device=dev),  # 1234 >= vocab: zero row
        embed_table=rnd(V, D, scale=0.02),
        norm_weight=(torch.rand(D, generator=g, device=dev) + 0.5).to(dtype),
        qkv=rnd(B, (Hq + 2 * Hkv) * hd),
        is_done=torch.tensor([0, 0, 1], dtype=torch.uint8, device=dev),
        gate_up=rnd(B, 2 * F),
    )
    kv0 = torch.tensor([700, 3, 1023], dtype=torch.uint32, device=dev)
    k0, v0 = rnd(B, Hkv, S, hd), rnd(B, Hkv, S, hd)

    def fresh():
        return dict(kv_lens=kv0.clone(), max_lens=torch.zeros(2, dtype=torch.uint32, device=dev),
                    x=torch.empty(B, D, dtype=dtype, device=dev), normed=torch.empty(B, D, dtype=dtype, device=dev),
                    q=torch.zeros(B, Hq, 1, hd, dtype=dtype, device=dev), k_cache=k0.clone(), v_cache=v0.clone(),
                    qk=torch.full((B, Hq, 1, S), 7.0, dtype=dtype, device=dev),
                    ffn_out=torch.empty(B, F, dtype=dtype, device=dev))

    f = fresh()
    ops.decode_step(**base, **f, workspace=ops.decode_step_workspace(dev), pairing=pairing)
    u = fresh()
    ops.launch_update_q_kv_lens(base["q_lens"], u["kv_lens"], u["max_lens"][0:1], u["max_lens"][1:2])
    ops.launch_embedding(base["input_ids"], base["embed_table"], u["x"])
    ops.launch_fused_add_residual_rmsnorm(base["norm_weight"], u["x"], u["normed"], False)
    rope = ops.launch_fused_reshape_rope_kvcache_llama2_decode if pairing else ops.launch_fused_reshape_rope_kvcache_decode
    rope(base["qkv"], base["is_done"], u["kv_lens"], u["q"], u["k_cache"], u["v_cache"])
    ops.decode_attention_scores(u["q"], u["k_cache"], u["kv_lens"], u["max_lens"][1:2], u["qk"])
    ops.launch_swiglu(base["gate_up"], u["ffn_out"])
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(f[n]), host(u[n])), n
    assert max_rel_err(host(f["normed"]), host(u["normed"])) <= (1e-5 if dtype == torch.float32 else 1e-2)
    assert np.all(host(f["x"])[2] == 0)


def test_unsupported_head_size_runs_operator_sequence():
    """head_dim 48 fp32 (192-byte K rows) is outside the fused step: the chain
    runs the operators instead, with the same results."""
    ch = Chain(WORKLOADS["tiny"], host_inputs(WORKLOADS["tiny"], seed=0))
    assert not ch.fused
    assert ch.kernels_per_step() == 6


@pytest.mark.parametrize("dtype,hd,pairing,S", [
    (torch.float32, 64, 1, 700),    # 256-byte K rows
    (torch.float32, 32, 0, 300),    # 128-byte K rows
    (torch.float16, 64, 0, 1000),   # 128-byte K rows, 16-bit
    (torch.bfloat16, 256, 1, 512),  # 512-byte K rows, 16-bit
    (torch.float16, 32, 1, 2048),   # 64-byte K rows
])
def test_row_widths_against_operator_sequence(dtype, hd, pairing, S):
    """Every K-row width the fused step takes (64 to 512 bytes: the four
    streaming-row instantiations), both pairings, against the operator
    sequence on the same buffers."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(hd * 7 + S)
    B, H, F, V = 3, 4, 256, 500
    D = H * hd

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)

    base = dict(q_lens=torch.ones(B, dtype=torch.uint32, device=dev),
                input_ids=torch.tensor([3, 499, 250], dtype=torch.uint32, device=dev),
                embed_table=rnd(V, D, scale=0.02), norm_weight=(torch.rand(D, generator=g, device=dev) + 0.5).to(dtype),
                qkv=rnd(B, 3 * D), is_done=torch.tensor([0, 1, 0], dtype=torch.uint8, device=dev), gate_up=rnd(B, 2 * F))
    kv0 = torch.tensor([S // 2, 5, S - 1], dtype=torch.uint32, device=dev)
    k0, v0 = rnd(B, H, S, hd), rnd(B, H, S, hd)

    def fresh():
        return dict(kv_lens=kv0.clone(), max_lens=torch.zeros(2, dtype=torch.uint32, device=dev),
                    x=torch.empty(B, D, dtype=dtype, device=dev), normed=torch.empty(B, D, dtype=dtype, device=dev),
                    q=torch.zeros(B, H, 1, hd, dtype=dtype, device=dev), k_cache=k0.clone(), v_cache=v0.clone(),
                    qk=torch.full((B, H, 1, S), 7.0, dtype=dtype, device=dev),
                    ffn_out=torch.empty(B, F, dtype=dtype, device=dev))

    f = fresh()
    assert ops.decode_step_supported(**base, **f, pairing=pairing)
    ops.decode_step(**base, **f, workspace=ops.decode_step_workspace(dev), pairing=pairing)
    u = fresh()
    ops.launch_update_q_kv_lens(base["q_lens"], u["kv_lens"], u["max_lens"][0:1], u["max_lens"][1:2])
    ops.launch_embedding(base["input_ids"], base["embed_table"], u["x"])
    ops.launch_fused_add_residual_rmsnorm(base["norm_weight"], u["x"], u["normed"], False)
    rope = ops.launch_fused_reshape_rope_kvcache_llama2_decode if pairing else ops.launch_fused_reshape_rope_kvcache_decode
    rope(base["qkv"], base["is_done"], u["kv_lens"], u["q"], u["k_cache"], u["v_cache"])
    ops.decode_attention_scores(u["q"], u["k_cache"], u["kv_lens"], u["max_lens"][1:2], u["qk"])
    ops.launch_swiglu(base["gate_up"], u["ffn_out"])
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(f[n]), host(u[n])), n
    assert max_rel_err(host(f["normed"]), host(u["normed"])) <= (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype,hd,pairing,S,hq,hkv", [
    (torch.float32, 128, 1, 4096, 8, 8),    # 512-byte rows (7B head)
    (torch.bfloat16, 128, 1, 2048, 8, 2),   # 256-byte rows, GQA
    (torch.float16, 64, 0, 1000, 4, 4),     # 128-byte rows, ragged last block
    (torch.float32, 16, 1, 300, 4, 2),      # 64-byte rows
])
def test_step_attention_matches_operator_sequence(dtype, hd, pairing, S, hq, hkv):
    """l2k_decode_step_attention against the operator sequence with the fused
    decode attention in place of the scores: every output bit-identical (the
    new V row is patched into its block exactly as the cache receives it),
    RMSNorm within its tolerance."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(hd + S + hkv)
    B, F, V = 3, 256, 500
    D = hq * hd

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)

    base = dict(q_lens=torch.ones(B, dtype=torch.uint32, device=dev),
                input_ids=torch.tensor([3, 499, 250], dtype=torch.uint32, device=dev),
                embed_table=rnd(V, D, scale=0.02), norm_weight=(torch.rand(D, generator=g, device=dev) + 0.5).to(dtype),
                qkv=rnd(B, (hq + 2 * hkv) * hd), is_done=torch.tensor([0, 1, 0], dtype=torch.uint8, device=dev),
                gate_up=rnd(B, 2 * F))
    kv0 = torch.tensor([S // 2, 5, S - 1], dtype=torch.uint32, device=dev)
    k0, v0 = rnd(B, hkv, S, hd), rnd(B, hkv, S, hd)

    def fresh():
        return dict(kv_lens=kv0.clone(), max_lens=torch.zeros(2, dtype=torch.uint32, device=dev),
                    x=torch.empty(B, D, dtype=dtype, device=dev), normed=torch.empty(B, D, dtype=dtype, device=dev),
                    q=torch.zeros(B, hq, 1, hd, dtype=dtype, device=dev), k_cache=k0.clone(), v_cache=v0.clone(),
                    qk=torch.full((B, hq, 1, S), 7.0, dtype=dtype, device=dev),
                    ffn_out=torch.empty(B, F, dtype=dtype, device=dev))

    f = fresh()
    out_f = torch.full((B, hq, 1, hd), 7.0, dtype=dtype, device=dev)
    assert ops.decode_step_supported(**base, **f, pairing=pairing)
    ops.decode_step_attention(**base, **f, attn_out=out_f, workspace=ops.decode_step_workspace(dev), pairing=pairing)
    u = fresh()
    out_u = torch.full((B, hq, 1, hd), 7.0, dtype=dtype, device=dev)
    ops.launch_update_q_kv_lens(base["q_lens"], u["kv_lens"], u["max_lens"][0:1], u["max_lens"][1:2])
    ops.launch_embedding(base["input_ids"], base["embed_table"], u["x"])
    ops.launch_fused_add_residual_rmsnorm(base["norm_weight"], u["x"], u["normed"], False)
    rope = ops.launch_fused_reshape_rope_kvcache_llama2_decode if pairing else ops.launch_fused_reshape_rope_kvcache_decode
    rope(base["qkv"], base["is_done"], u["kv_lens"], u["q"], u["k_cache"], u["v_cache"])
    ops.decode_attention(u["q"], u["k_cache"], u["v_cache"], u["kv_lens"], u["max_lens"][1:2], u["qk"], out_u)
    ops.launch_swiglu(base["gate_up"], u["ffn_out"])
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(f[n]), host(u[n])), n
    assert bits_equal(host(out_f), host(out_u)), "attention output"
    assert max_rel_err(host(f["normed"]), host(u["normed"])) <= (1e-5 if dtype == torch.float32 else 1e-2)


@pytest.mark.parametrize("dtype,use_table,S,kv", [
    (torch.bfloat16, False, 512, [255, 7, 511]),     # no host table: angles on the device
    (torch.float32, True, 4608, [4200, 4095, 30]),   # lengths past 4096: the length-scaled angles on the device
    (torch.bfloat16, True, 4608, [4200, 100, 4607]),
    (torch.bfloat16, True, 4096, [4095, 0, 2000]),   # every position in the table: the table-only kernel
])
def test_step_angle_sources_against_operator_sequence(dtype, use_table, S, kv):
    """The fused step has a kernel for launches whose every position is in the
    host cos/sin table and one that may evaluate angles on the device; each
    is bit-identical to the operator sequence with the same angle source."""
    dev = torch.device("cuda")
    g = torch.Generator(device=dev)
    g.manual_seed(S + len(kv) + int(use_table))
    B, H, hd, F, V = 3, 4, 128, 256, 500
    D = H * hd

    def rnd(*shape, scale=1.0):
        return (torch.randn(*shape, generator=g, device=dev) * scale).to(dtype)

    base = dict(q_lens=torch.ones(B, dtype=torch.uint32, device=dev),
                input_ids=torch.tensor([3, 499, 250], dtype=torch.uint32, device=dev),
                embed_table=rnd(V, D, scale=0.02), norm_weight=(torch.rand(D, generator=g, device=dev) + 0.5).to(dtype),
                qkv=rnd(B, 3 * D), is_done=torch.zeros(B, dtype=torch.uint8, device=dev), gate_up=rnd(B, 2 * F))
    kv0 = torch.tensor(kv, dtype=torch.uint32, device=dev)
    k0, v0 = rnd(B, H, S, hd), rnd(B, H, S, hd)

    def fresh():
        return dict(kv_lens=kv0.clone(), max_lens=torch.zeros(2, dtype=torch.uint32, device=dev),
                    x=torch.empty(B, D, dtype=dtype, device=dev), normed=torch.empty(B, D, dtype=dtype, device=dev),
                    q=torch.zeros(B, H, 1, hd, dtype=dtype, device=dev), k_cache=k0.clone(), v_cache=v0.clone(),
                    qk=torch.full((B, H, 1, S), 7.0, dtype=dtype, device=dev),
                    ffn_out=torch.empty(B, F, dtype=dtype, device=dev))

    f = fresh()
    ops.decode_step(**base, **f, workspace=ops.decode_step_workspace(dev), pairing=1, use_table=use_table)
    u = fresh()
    ops.launch_update_q_kv_lens(base["q_lens"], u["kv_lens"], u["max_lens"][0:1], u["max_lens"][1:2])
    ops.launch_embedding(base["input_ids"], base["embed_table"], u["x"])
    ops.launch_fused_add_residual_rmsnorm(base["norm_weight"], u["x"], u["normed"], False)
    ops.launch_fused_reshape_rope_kvcache_llama2_decode(base["qkv"], base["is_done"], u["kv_lens"], u["q"],
                                                        u["k_cache"], u["v_cache"], use_table=use_table)
    ops.decode_attention_scores(u["q"], u["k_cache"], u["kv_lens"], u["max_lens"][1:2], u["qk"])
    ops.launch_swiglu(base["gate_up"], u["ffn_out"])
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(f[n]), host(u[n])), n
    assert max_rel_err(host(f["normed"]), host(u["normed"])) <= (1e-5 if dtype == torch.float32 else 1e-2)
