"""launch_linear's own kernels for plain 16-bit GEMMs with A not transposed
(tcgen05 tensor cores; the CUDA-core B stream for at most 8 rows)
against the oracle's restatement of the reference helper
(compute_expected_linear, test/kernel/test_linear.cu:78-108) and, at sizes
the CPU oracle cannot finish in seconds, against a torch fp32 product of the
same 16-bit operands.

Bar: 1e-2 relative to the largest magnitude of each output row (16-bit I/O;
the products of a GEMM row cancel, so single elements can be near zero).
"""
import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from oracle import port
from tests.gpu_util import TORCH, host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def _row_rel_err(got, want):
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    scale = np.maximum(np.abs(want).max(axis=-1, keepdims=True), 1e-30)
    return float((np.abs(got - want) / scale).max())


def _operands(dt, m, n, k, trans_b, seed, pad=0):
    """A (m x k) and B (n x k if trans_b else k x n) as views with row strides
    padded by `pad` elements (a multiple of 8 keeps the rows 16-byte aligned)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    a_full = torch.randn(m, k + pad, generator=g, device="cuda").to(TORCH[dt])
    b_rows, b_cols = (n, k) if trans_b else (k, n)
    b_full = torch.randn(b_rows, b_cols + pad, generator=g, device="cuda").to(TORCH[dt])
    return a_full[:, :k], b_full[:, :b_cols]


def _call(a, b, c, trans_b, m, n, k):
    capi.call("l2k_linear", 0, int(trans_b), m, n, k, a.data_ptr(), a.stride(0), b.data_ptr(), b.stride(0),
              c.data_ptr(), c.stride(0), 0, None, None, None, {torch.bfloat16: 2, torch.float16: 1}[a.dtype],
              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("trans_b", [0, 1])
@pytest.mark.parametrize("m,n,k,pad", [
    (128, 128, 64, 0),     # one tile, one k block
    (300, 200, 136, 8),    # partial tiles in every dimension, padded row strides
    (1, 512, 4096, 0),     # a decode-shaped product (one row): k split over a cluster of 8
    (257, 384, 320, 16),
    (64, 1024, 2048, 0),   # a batch-64 decode product: k split over a cluster of 2
    (16, 384, 1000, 8),    # a ragged last k block with the split
    (3, 300, 1000, 4),     # few rows: the CUDA-core B stream (K x N layout; N x K falls back: unaligned rows)
    (8, 996, 2048, 4),     # few rows, a ragged last column vector
    (5, 4096, 11008, 0),   # few rows, the down projection's k split over a cluster of 8
    (1, 12288, 4096, 0),   # one row, the QKV projection
])
def test_linear_tensor_cores_against_oracle(dt, trans_b, m, n, k, pad):
    a, b = _operands(dt, m, n, k, trans_b, seed=m + n + k + trans_b, pad=pad)
    c_full = torch.full((m, n + pad), 7.0, dtype=TORCH[dt], device="cuda")
    _call(a, b, c_full, trans_b, m, n, k)
    torch.cuda.synchronize()
    want = port.linear(host(a), host(b), False, bool(trans_b), m, n, k)
    got = host(c_full)
    assert _row_rel_err(got[:, :n], want) <= 1e-2
    assert np.all(got[:, n:] == 7.0), "columns past n are left as is"


@pytest.mark.parametrize("trans_b", [0, 1])
def test_linear_tensor_cores_large_against_torch_fp32(trans_b):
    """4096 x 4096 x 4096 bf16 against torch's fp32 product of the same operands."""
    m = n = k = 4096
    a, b = _operands("bf16", m, n, k, trans_b, seed=5)
    c = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    _call(a, b, c, trans_b, m, n, k)
    bb = b.float().t() if trans_b else b.float()
    want = (a.float() @ bb).cpu().numpy()
    assert _row_rel_err(host(c), want) <= 1e-2


def test_launch_linear_routes_plain_16bit_to_the_same_results():
    """ops.launch_linear (the reference API) on a 2-D bf16 product equals the
    direct C-ABI call (the tensor-core path) bit for bit."""
    m, n, k = 192, 320, 256
    a, b = _operands("bf16", m, n, k, 0, seed=3)
    a, b = a.contiguous(), b.contiguous()
    c1 = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    c2 = torch.empty_like(c1)
    ops.launch_linear(False, False, m, n, k, a, b, c1)
    _call(a, b, c2, 0, m, n, k)
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
