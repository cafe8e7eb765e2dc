"""Whole-chain parity on the GPU at the workload shapes (batch trimmed where
the CPU oracle would take too long), against the chain oracle on the same
seeded inputs.

Bars: bit-exact for the embedding gather, the KV-cache
rows/positions, the lengths and the RoPE outputs (host-built angle table);
max relative error <= 1e-5 for fp32 and <= 1e-2 for 16-bit I/O elsewhere.
"""
import dataclasses

import numpy as np
import pytest
import torch

from llama2_b200.chain import Chain
from llama2_b200.workloads import WORKLOADS, host_inputs, with_batch
from oracle import chain as ochain
from tests.gpu_util import bits_equal, host, max_rel_err

pytestmark = pytest.mark.gpu

REL = {"f32": 1e-5, "bf16": 1e-2, "f16": 1e-2}


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def run_and_check(w, seed=0, fused=True):
    inp = host_inputs(w, seed=seed)
    ch = Chain(w, inp, fused=fused)
    ch.step()
    torch.cuda.synchronize()
    ref = ochain.decode_step(w, inp) if w.decode else ochain.prefill_step(w, inp)
    tol = REL[w.dtype]
    assert bits_equal(host(ch.kv_lens).astype(np.uint32), ref["kv_lens"])
    mx = host(ch.max_lens)
    assert int(mx[0]) == ref["max_q"] and int(mx[1]) == ref["max_kv"]
    assert bits_equal(host(ch.x), ref["x"]), "embedding gather must be bit-exact"
    assert max_rel_err(host(ch.normed), ref["normed"]) <= tol
    assert bits_equal(host(ch.q), ref["q"]), "RoPE q must be bit-exact (host angle table)"
    assert bits_equal(host(ch.k_cache), ref["k"]), "K cache rows must be bit-exact"
    assert bits_equal(host(ch.v_cache), ref["v"]), "V cache rows must be bit-exact"
    got_qk = host(ch.qk)
    if w.decode:
        assert max_rel_err(got_qk, ref["qk"]) <= tol
    else:
        # rows >= q_len are not part of the fused kernel's output; all rows are valid here
        assert max_rel_err(got_qk, ref["qk"]) <= tol
    assert max_rel_err(host(ch.ffn_out), ref["ffn_out"], floor=1e-30) <= tol
    return ch, ref


def test_tiny_decode_fp32():
    run_and_check(WORKLOADS["tiny"])


# fused=True runs the one-launch decode step, fused=False the operator sequence.
@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("seed", [0, 1])
def test_7b_b1_decode_fp32(seed, fused):
    ch, _ = run_and_check(WORKLOADS["7b-b1"], seed=seed, fused=fused)
    assert ch.fused == fused


@pytest.mark.parametrize("fused", [True, False])
def test_7b_batched_decode_fp32(fused):
    ch, _ = run_and_check(with_batch(WORKLOADS["7b-b64"], 4), fused=fused)
    assert ch.fused == fused


@pytest.mark.parametrize("fused", [True, False])
def test_7b_batched_decode_bf16(fused):
    ch, _ = run_and_check(with_batch(WORKLOADS["7b-b64-bf16"], 4), fused=fused)
    assert ch.fused == fused


@pytest.mark.parametrize("fused", [True, False])
def test_13b_decode_fp16(fused):
    ch, _ = run_and_check(with_batch(WORKLOADS["13b-b256"], 2), fused=fused)
    assert ch.fused == fused


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_prefill_small(dtype):
    w = dataclasses.replace(WORKLOADS["7b-prefill"], batch=2, prefill_len=192, kv_cache_len=256, dtype=dtype)
    run_and_check(w)


@pytest.mark.parametrize("fused", [True, False])
def test_decode_interleaved_pairs_hd128(fused):
    w = dataclasses.replace(with_batch(WORKLOADS["7b-b64"], 2), pairing=0)
    run_and_check(w, fused=fused)


@pytest.mark.parametrize("fused", [True, False])
def test_decode_done_sequences_untouched(fused):
    w = with_batch(WORKLOADS["7b-b64"], 3)
    inp = host_inputs(w, seed=5)
    inp["is_done"] = np.array([0, 1, 0], np.uint8)
    ch = Chain(w, inp, fused=fused)
    ch.step()
    torch.cuda.synchronize()
    ref = ochain.decode_step(w, inp)
    assert bits_equal(host(ch.k_cache), ref["k"]) and bits_equal(host(ch.v_cache), ref["v"])
    assert bits_equal(host(ch.q), ref["q"])
    assert max_rel_err(host(ch.qk), ref["qk"]) <= 1e-5


def test_graph_replay_matches_eager():
    w = WORKLOADS["7b-b1"]
    inp = host_inputs(w, seed=3)
    ch = Chain(w, inp)
    ch.capture()
    ch.replay()
    torch.cuda.synchronize()
    ref = ochain.decode_step(w, inp)
    assert max_rel_err(host(ch.qk), ref["qk"]) <= 1e-5
    assert bits_equal(host(ch.k_cache), ref["k"])


@pytest.mark.parametrize("name,batch", [("7b-b1", 1), ("7b-b64-bf16", 3)])
def test_end_to_end_step_reads_back_results(name, batch):
    """step_e2e: one packed upload, the step, the results back on the host —
    the score rows' written keys [0, M) and the small outputs, equal to the
    device's."""
    w = with_batch(WORKLOADS[name], batch)
    inp = host_inputs(w, seed=9)
    ch = Chain(w, inp)
    ch.capture()
    hin, hout = ch.host_buffers(inp)
    ch.step_e2e()
    torch.cuda.synchronize()
    m = ch._m_written
    assert m == min(int((inp["kv_lens"].astype(np.int64) + 1).max()), w.kv_cache_len)
    assert bits_equal(host(hout["qk"])[..., :m], host(ch.qk)[..., :m])
    for n in ("normed", "ffn_out", "max_lens"):
        assert bits_equal(host(hout[n]), host(getattr(ch, n))), n
    ref = ochain.decode_step(w, inp)
    assert max_rel_err(host(hout["qk"])[..., :m], ref["qk"][..., :m]) <= REL[w.dtype]
    h2d, d2h = ch.e2e_bytes()
    assert h2d == hin.buf.numel()
    # one copy of everything when keys [0, M) are at least half of each row, else the written part only
    assert (d2h == hout.buf.numel()) == (2 * m >= w.kv_cache_len) and d2h <= hout.buf.numel()


# ---------------------------------------------------------------------------
# The chain with the attention output (P.V and the transpose + unpad)
# ---------------------------------------------------------------------------
def _row_rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.maximum(np.abs(want).max(axis=-1, keepdims=True), 1e-30)
    return float((np.abs(got - want) / scale).max())


@pytest.mark.parametrize("fused", [True, False])
@pytest.mark.parametrize("name,batch", [("7b-b1", 1), ("7b-b64", 3), ("7b-b64-bf16", 4), ("tiny", 1)])
def test_decode_chain_with_attention_output(name, batch, fused):
    w = with_batch(WORKLOADS[name], batch)
    inp = host_inputs(w, seed=2)
    ch = Chain(w, inp, attention_output=True, fused=fused)
    # the one-launch step (with its P.V) wherever it takes the shapes (head_dim 48 of "tiny" it does not)
    assert ch.fused == (fused and w.head_dim == 128)
    ch.capture()
    ch.replay()
    torch.cuda.synchronize()
    ref = ochain.decode_step(w, inp, attention_output=True)
    tol = REL[w.dtype]
    assert max_rel_err(host(ch.qk), ref["qk"]) <= tol
    assert bits_equal(host(ch.v_cache), ref["v"])
    assert _row_rel_err(host(ch.attn_out), ref["attn_out"]) <= tol


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_prefill_chain_with_attention_output(dtype):
    w = dataclasses.replace(WORKLOADS["7b-prefill"], batch=2, prefill_len=192, kv_cache_len=256, dtype=dtype)
    inp = host_inputs(w, seed=4)
    ch = Chain(w, inp, attention_output=True)
    assert ch.kernels_per_step() == (10 if dtype == "f32" else 9)
    ch.step()
    torch.cuda.synchronize()
    ref = ochain.prefill_step(w, inp, attention_output=True)
    tol = REL[w.dtype]
    assert max_rel_err(host(ch.qk), ref["qk"]) <= tol
    assert _row_rel_err(host(ch.attn_out), ref["attn_out"]) <= tol
