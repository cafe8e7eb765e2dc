"""Parity of the one-launch decode step at the FULL sizes of the batched
decode workloads, against the oracle, on the bench's own seed-0 inputs.

  7b-b64        Llama-2-7B dims, 64 sequences, fp32 K/V cache [64, 32, 4096, 128] (4.3 GB each)
  7b-b64-bf16   the same with bf16 I/O
  13b-b256      Llama-2-13B dims, 256 sequences, fp16 cache [256, 40, 4096, 128]: 5.37 G elements per
                cache, so the planes of sequences >= 205 (and heads >= 32 of sequence 204) start past
                element 2^32 — the 64-bit offset path the reference's 32-bit indexing cannot reach

Checked for EVERY sequence and head: the lengths and maxima (exact), the
embedding rows (bit-exact), RMSNorm rows and SwiGLU rows (tolerance), the
rotated q rows (bit-exact), the appended K and V rows (bit-exact) and that
no other cache row changed (on the device, whole caches), every score row's
keys past its position are zero and every row sums to 1. Checked for sampled
(sequence, head) pairs — the first, middle and last sequences, the planes on
both sides of the 2^32-element boundary, and seeded random pairs — the score
row against the oracle's softmax row over the post-step cache plane, and
with the attention output, P.V of that row against the oracle's.

Bars (the oracle's fp32 arithmetic on the 16-bit-rounded data for 16-bit
I/O): max relative error <= 1e-5 for fp32 and <= 1e-2 for 16-bit; the
attention output relative to each output row's largest magnitude.
"""
import numpy as np
import pytest
import torch

from llama2_b200 import capi
from llama2_b200.chain import Chain
from llama2_b200.workloads import WORKLOADS, host_inputs
from oracle import chain as ochain
from oracle import port
from tests.gpu_util import bits_equal, host, max_rel_err

pytestmark = pytest.mark.gpu

REL = {"f32": 1e-5, "bf16": 1e-2, "f16": 1e-2}
SUM_TOL = {"f32": 1e-4, "bf16": 1e-2, "f16": 1e-2}


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield
    assert capi.lib().l2k_device_error(1) == 0
    torch.cuda.empty_cache()


def sampled_pairs(b, h, plane_elems):
    """(sequence, head) pairs for the oracle score rows: the corners, the
    planes either side of element 2^32 (where one exists), and 12 seeded
    random pairs."""
    pairs = {(0, 0), (0, h - 1), (1, h // 2), (b // 2, 0), (b - 2, h // 2), (b - 1, 0), (b - 1, h - 1)}
    boundary = (1 << 32) // plane_elems  # first plane index whose first element is >= 2^32
    if boundary < b * h:
        for idx in (boundary - 1, boundary, boundary + 1, b * h - 1):
            pairs.add(divmod(idx, h))
    rng = np.random.default_rng(123)
    for _ in range(12):
        pairs.add((int(rng.integers(b)), int(rng.integers(h))))
    return sorted(pairs)


@pytest.mark.parametrize("name,attention", [("7b-b64", False), ("7b-b64-bf16", False), ("13b-b256", False),
                                            ("7b-b64", True), ("7b-b64-bf16", True)])
def test_full_size_decode_step(name, attention):
    w = WORKLOADS[name]
    b, h, hd, s = w.batch, w.heads, w.head_dim, w.kv_cache_len
    inp = host_inputs(w, seed=0, kv_cache=False)
    r = ochain.rounder(w.dtype)
    tol = REL[w.dtype]
    ch = Chain(w, inp, attention_output=attention)
    assert ch.fused
    k_before, v_before = ch.k_cache.clone(), ch.v_cache.clone()
    ch.step()
    torch.cuda.synchronize()

    pos = inp["kv_lens"].astype(np.int64)          # row each sequence appends (its length before the step)
    kv_after = pos + 1
    max_kv = int(kv_after.max())
    assert bits_equal(host(ch.kv_lens).astype(np.uint32), kv_after.astype(np.uint32))
    assert host(ch.max_lens).tolist() == [1, max_kv]

    # embedding, RMSNorm, SwiGLU: every token
    x = port.embedding(inp["ids"], r(inp["embed_table"]))
    assert bits_equal(host(ch.x), x)
    _, normed = port.fused_add_residual_rmsnorm(x, np.zeros_like(x), r(inp["norm_weight"]), False)
    assert max_rel_err(host(ch.normed), r(normed)) <= tol
    assert max_rel_err(host(ch.ffn_out), r(port.swiglu(r(inp["gate_up"]))), floor=1e-30) <= tol

    # rotated q and the appended K / V rows: every sequence and head, bit-exact
    qkv = r(inp["qkv"]).reshape(b, 3 * h, hd)
    want_q = np.empty((b, h, hd), np.float32)
    want_k = np.empty((b, h, hd), np.float32)
    for i in range(b):
        p = int(pos[i])
        for j in range(h):
            want_q[i, j] = port.rotate_one_head(w.pairing, qkv[i, j], p, p + 1)
            want_k[i, j] = port.rotate_one_head(w.pairing, qkv[i, h + j], p, p + 1)
    want_q, want_k = r(want_q), r(want_k)
    assert bits_equal(host(ch.q).reshape(b, h, hd), want_q)
    dev_pos = torch.from_numpy(pos).to(ch.k_cache.device)
    bi = torch.arange(b, device=dev_pos.device)[:, None]
    hi = torch.arange(h, device=dev_pos.device)[None, :]
    assert bits_equal(host(ch.k_cache[bi, hi, dev_pos[:, None]]), want_k)
    assert bits_equal(host(ch.v_cache[bi, hi, dev_pos[:, None]]), np.ascontiguousarray(qkv[:, 2 * h:]))

    # no other cache row changed (whole caches, on the device, 8 sequences at a time)
    rows = torch.arange(s, device=dev_pos.device)
    for c0 in range(0, b, 8):
        c1 = min(b, c0 + 8)
        own = (rows[None, :] == dev_pos[c0:c1, None])[:, None, :]          # [c, 1, S]
        for after, before in ((ch.k_cache, k_before), (ch.v_cache, v_before)):
            changed = (after[c0:c1] != before[c0:c1]).any(-1)                # [c, H, S]
            assert not bool((changed & ~own).any()), f"cache rows outside the appended row changed in [{c0}, {c1})"
    del k_before, v_before

    # every score row: zero past its position, sums to 1 over the kept keys
    qk = ch.qk.view(b, h, s).float()
    keys = torch.arange(s, device=qk.device)
    past = keys[None, None, :] > dev_pos[:, None, None]
    assert not bool((torch.where(past, qk, torch.zeros_like(qk)) != 0).any()), "keys past a row's position must be 0"
    sums = qk.sum(-1)
    assert float((sums - 1).abs().max()) <= SUM_TOL[w.dtype]

    # sampled rows against the oracle (the post-step plane holds the appended key)
    pairs = sampled_pairs(b, h, s * hd)
    if name == "13b-b256":
        assert any((i * h + j) * s * hd >= (1 << 32) for i, j in pairs)
    for i, j in pairs:
        p = int(pos[i])
        k_rows = host(ch.k_cache[i, j, :p + 1])
        want = ochain.score_row(want_q[i, j], k_rows, p, hd)
        got = host(ch.qk[i, j, 0, :p + 1])
        assert max_rel_err(got, r(want)) <= tol, f"score row ({i}, {j})"
        if attention:
            v_rows = host(ch.v_cache[i, j, :p + 1])
            out = r(port.linear(want.reshape(1, -1), v_rows, False, False, 1, hd, p + 1)).reshape(-1)
            got_o = host(ch.attn_out[i, j * hd:(j + 1) * hd]).astype(np.float64)
            err = float(np.abs(got_o - out).max() / max(np.abs(out).max(), 1e-30))
            assert err <= tol, f"attention output ({i}, {j}): {err:.3g}"
