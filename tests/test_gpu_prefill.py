"""Fused prefill attention scores (tcgen05 tensor-core path and the cluster
score-row path) against the oracle: QK^T (test_linear.cu:78-108 order) +
intended causal mask + masked softmax (test_compute_masked_attention_score.cu:21-89).

16-bit I/O bar: max relative error <= 1e-2 on every written score. Entries
the operator must not touch (rows >= q_len, keys >= max_kv) are filled with a
sentinel beforehand and must keep it.
"""
import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from oracle import chain as ochain
from oracle import port
from tests.gpu_util import host, max_rel_err

pytestmark = pytest.mark.gpu

SENTINEL = 7.0


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield
    assert capi.lib().l2k_device_error(1) == 0, "a kernel recorded a device-side wait timeout"


def make_case(b, hq, hkv, hd, qc, s, q_lens, kv_lens, dtype, seed=0):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn(b, hq, qc, hd, generator=g, device="cuda").to(dtype)
    k = torch.randn(b, hkv, s, hd, generator=g, device="cuda").to(dtype)
    qk = torch.full((b, hq, qc, s), SENTINEL, dtype=dtype, device="cuda")
    ql = torch.tensor(q_lens, dtype=torch.uint32, device="cuda")
    kl = torch.tensor(kv_lens, dtype=torch.uint32, device="cuda")
    return q, k, qk, ql, kl


def oracle_scores(q, k, q_lens, kv_lens, max_q, max_kv):
    qf, kf = host(q), host(k)
    b, hq, qc, hd = qf.shape
    s = kf.shape[2]
    ref = np.full((b, hq, qc, s), SENTINEL, np.float32)
    port.qk_scores(qf, kf, max_q, max_kv, ref)
    mask = ochain.intended_mask(np.array(q_lens, np.uint32), np.array(kv_lens, np.uint32), max_q, max_kv, qc, s)
    port.masked_attention_score(ref, mask, np.array(q_lens, np.uint32), max_kv, hd)
    # rows >= q_len keep the sentinel in the fused operator
    for bi, ql in enumerate(q_lens):
        ref[bi, :, ql:, :] = SENTINEL
    return ref


def check(q, k, qk, q_lens, kv_lens, tol=1e-2):
    max_q, max_kv = max(q_lens), max(kv_lens)
    ops.prefill_attention_scores(q, k, torch.tensor(q_lens, dtype=torch.uint32, device="cuda"),
                                 torch.tensor(kv_lens, dtype=torch.uint32, device="cuda"), max_q, max_kv, qk)
    torch.cuda.synchronize()
    got = host(qk)
    ref = oracle_scores(q, k, q_lens, kv_lens, max_q, max_kv)
    assert np.all(got[..., max_kv:] == SENTINEL), "keys >= max_kv must be untouched"
    for bi, ql in enumerate(q_lens):
        assert np.all(got[bi, :, ql:, :] == SENTINEL), "rows >= q_len must be untouched"
    err = max_rel_err(got, ref)
    assert err <= tol, err


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_tc_uniform_full_tiles(dtype):
    q, k, qk, _, _ = make_case(2, 4, 4, 128, 256, 256, [256, 256], [256, 256], dtype)
    check(q, k, qk, [256, 256], [256, 256])


def test_tc_ragged_rows_and_history():
    # q_len 130 straddles a 128-row tile; sequence 2 is a chunked prefill with
    # history (kv_len - q_len = 299); max_kv = 300 is not a tile multiple.
    q_lens, kv_lens = [256, 130, 1], [256, 200, 300]
    q, k, qk, _, _ = make_case(3, 4, 4, 128, 256, 384, q_lens, kv_lens, torch.bfloat16, seed=1)
    check(q, k, qk, q_lens, kv_lens)


def test_tc_grouped_kv_heads():
    q_lens, kv_lens = [192, 192], [192, 192]
    q, k, qk, _, _ = make_case(2, 8, 2, 128, 192, 200, q_lens, kv_lens, torch.bfloat16, seed=2)
    check(q, k, qk, q_lens, kv_lens)


def test_row_kernel_other_head_dim():
    # head_dim 64: not the tensor-core shape; cluster score-row path
    q_lens, kv_lens = [100, 37], [100, 64]
    q, k, qk, _, _ = make_case(2, 2, 2, 64, 128, 128, q_lens, kv_lens, torch.bfloat16, seed=3)
    check(q, k, qk, q_lens, kv_lens)


def test_fp32_unfused_path():
    q_lens, kv_lens = [70, 128], [90, 128]
    q, k, qk, _, _ = make_case(2, 2, 2, 128, 128, 160, q_lens, kv_lens, torch.float32, seed=4)
    check(q, k, qk, q_lens, kv_lens, tol=1e-5)


def test_full_size_prefill_properties():
    """[8, 32, 2048, 2048] bf16 causal scores: size-independent properties on
    every row, and 64 sampled rows against the oracle."""
    b, h, qc, hd = 8, 32, 2048, 128
    q, k, qk, ql, kl = make_case(b, h, h, hd, qc, qc, [qc] * b, [qc] * b, torch.bfloat16, seed=5)
    ops.prefill_attention_scores(q, k, ql, kl, qc, qc, qk)
    torch.cuda.synchronize()
    # upper triangle exactly zero, row sums 1 within bf16 rounding
    tri = torch.triu(torch.ones(qc, qc, dtype=torch.bool, device="cuda"), diagonal=1)
    assert not torch.any(qk[:, :, tri] != 0)
    sums = qk.float().sum(-1)
    assert torch.max(torch.abs(sums - 1.0)).item() < 1e-2
    rng = np.random.default_rng(0)
    for _ in range(64):
        bi, hi, i = rng.integers(0, b), rng.integers(0, h), rng.integers(0, qc)
        want = ochain.score_row(host(q[bi, hi, i]), host(k[bi, hi, :i + 1]), i, hd)
        got = host(qk[bi, hi, i, :i + 1])
        assert max_rel_err(got, want) <= 1e-2, (bi, hi, i)
