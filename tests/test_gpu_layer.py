"""The decoder-layer driver (llama2_b200.layer) on the GPU against the oracle
composition of the same restated helpers (oracle/chain.py decode_layer):
two consecutive layers of a decode step, fp32 and bf16.

Bars: 1e-5 (fp32) / 2e-2 (bf16, four chained 16-bit projections and two
norms) relative to the largest magnitude of each row, the appended K rows
included (they are RoPE of the QKV projection); every other cache row
bit-exact.
"""
import numpy as np
import pytest
import torch

from llama2_b200 import ops
from llama2_b200.layer import DecoderLayer
from oracle import chain as ochain
from tests.gpu_util import bits_equal, host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def _row_rel_err(got, want):
    got = np.asarray(got, np.float64).reshape(got.shape[0], -1)
    want = np.asarray(want, np.float64).reshape(want.shape[0], -1)
    scale = np.maximum(np.abs(want).max(axis=-1, keepdims=True), 1e-30)
    return float((np.abs(got - want) / scale).max())


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
@pytest.mark.parametrize("graph", [False, True])
def test_two_decode_layers_against_oracle(dtype, tol, graph):
    b, d, heads, kvh, f, s = 3, 256, 2, 2, 512, 512
    dev = torch.device("cuda")
    layers = [DecoderLayer(d, heads, kvh, f, s, b, dtype=dtype, seed=10 + i) for i in range(2)]
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    x = torch.randn(b, d, generator=g, device=dev).to(dtype)
    q_lens = torch.ones(b, dtype=torch.uint32, device=dev)
    kv_lens = torch.tensor([100, 7, 511], dtype=torch.uint32, device=dev)
    max_lens = torch.zeros(2, dtype=torch.uint32, device=dev)
    is_done = torch.tensor([0, 1, 0], dtype=torch.uint8, device=dev)
    ops.launch_update_q_kv_lens(q_lens, kv_lens, max_lens[0:1], max_lens[1:2])
    torch.cuda.synchronize()
    kv_host = host(kv_lens).astype(np.uint32)
    max_kv = int(host(max_lens)[1])
    x0 = host(x)
    caches = [(host(L.k_cache).copy(), host(L.v_cache).copy()) for L in layers]
    wts = [{n: host(t) for n, t in L.weights().items()} for L in layers]

    if graph:
        g0 = layers[0].capture_decode(x, None, kv_lens, max_lens[1:2], is_done)
        g0.replay()
        g1 = layers[1].capture_decode(x, layers[0].down, kv_lens, max_lens[1:2], is_done)
        g1.replay()
        pending = layers[1].down
    else:
        pending = None
        for L in layers:
            pending = L.decode(x, pending, kv_lens, max_lens[1:2], is_done)
    torch.cuda.synchronize()

    dt = "f32" if dtype == torch.float32 else "bf16"
    xr, pend = x0, None
    for i, L in enumerate(layers):
        k, v = caches[i]
        ref = ochain.decode_layer(wts[i], xr, pend, kv_host, max_kv, host(is_done), k, v, 1, dt)
        got_k = host(L.k_cache)
        # rows this step does not append are untouched; the appended rows are
        # RoPE of the QKV projection, within the projection's tolerance
        assert _row_rel_err(got_k.reshape(-1, got_k.shape[-1]), k.reshape(-1, k.shape[-1])) <= tol, f"layer {i} K"
        for bi, kvl in enumerate(kv_host):
            keep = np.ones(got_k.shape[2], bool)
            keep[int(kvl) - 1] = False
            assert bits_equal(got_k[bi][:, keep], k[bi][:, keep]), f"layer {i} K rows other than the new one"
        assert _row_rel_err(host(L.qk), ref["qk"]) <= tol, f"layer {i} scores"
        xr, pend = ref["x"], ref["down"]
    assert _row_rel_err(host(x), xr) <= tol
    assert _row_rel_err(host(pending), pend) <= tol


@pytest.mark.parametrize("dtype,tol", [(torch.float32, 1e-5), (torch.bfloat16, 2e-2)])
def test_two_prefill_layers_against_oracle(dtype, tol):
    """Two layers over a batch of two prompts (64 and 40 new tokens after
    0 and 10 cached ones), ragged, causal, against the oracle composition."""
    b, d, heads, kvh, f, s, qc = 2, 256, 2, 2, 512, 128, 64
    dev = torch.device("cuda")
    layers = [DecoderLayer(d, heads, kvh, f, s, b, dtype=dtype, seed=20 + i) for i in range(2)]
    q_lens_h = np.array([64, 40], np.uint32)
    kv0_h = np.array([0, 10], np.uint32)
    t = int(q_lens_h.sum())
    g = torch.Generator(device=dev)
    g.manual_seed(2)
    x = torch.randn(t, d, generator=g, device=dev).to(dtype)
    q_lens = torch.from_numpy(q_lens_h).cuda()
    kv_lens = torch.from_numpy(kv0_h).cuda()
    max_lens = torch.zeros(2, dtype=torch.uint32, device=dev)
    unpad = torch.zeros(b, qc, dtype=torch.uint32, device=dev)
    offsets = torch.zeros(b, dtype=torch.uint32, device=dev)
    ops.launch_update_q_kv_lens(q_lens, kv_lens, max_lens[0:1], max_lens[1:2])
    ops.launch_build_padding_index_maps(t, q_lens, unpad, offsets)
    torch.cuda.synchronize()
    kv_h = host(kv_lens).astype(np.uint32)
    max_q, max_kv = int(host(max_lens)[0]), int(host(max_lens)[1])
    unpad_h = host(unpad).reshape(-1)[:t].astype(np.uint32)
    x0 = host(x)
    caches = [(host(L.k_cache).copy(), host(L.v_cache).copy()) for L in layers]
    wts = [{n: host(w) for n, w in L.weights().items()} for L in layers]

    pending = None
    for L in layers:
        pending = L.prefill(x, pending, q_lens, kv_lens, max_q, max_kv, unpad)
    torch.cuda.synchronize()

    dt = "f32" if dtype == torch.float32 else "bf16"
    xr, pend = x0, None
    for i, L in enumerate(layers):
        k, v = caches[i]
        ref = ochain.prefill_layer(wts[i], xr, pend, q_lens_h, kv_h, max_q, max_kv, unpad_h, k, v, qc, 1, dt)
        assert _row_rel_err(host(L.k_cache).reshape(-1, 128), k.reshape(-1, 128)) <= tol, f"layer {i} K"
        xr, pend = ref["x"], ref["down"]
    assert _row_rel_err(host(x), xr) <= tol
    assert _row_rel_err(host(pending), pend) <= tol


@pytest.mark.parametrize("pairing", [0, 1])
def test_fused_epilogues_bit_identical_to_separate_launches(pairing):
    """A bf16 layer whose QKV projection carries the RoPE + K/V append and
    whose gate/up projection carries the SwiGLU (7 decode launches, 9
    prefill) against the same layer with the separate launches (9 and 11):
    a decode step of 12 sequences, then a prefill pass of 104 tokens, every
    output and both caches bit for bit."""
    b, d, heads, kvh, f, s, qc = 12, 512, 4, 2, 1024, 256, 64
    dev = torch.device("cuda")
    runs = []
    for fuse in (False, True):
        L = DecoderLayer(d, heads, kvh, f, s, b, dtype=torch.bfloat16, seed=3, pairing=pairing,
                         fuse_epilogues=fuse)
        assert L.launches_per_step() == (7 if fuse else 9)
        g = torch.Generator(device=dev)
        g.manual_seed(4)
        x = torch.randn(b, d, generator=g, device=dev).to(torch.bfloat16)
        pending = torch.randn(b, d, generator=g, device=dev).to(torch.bfloat16)
        lens = torch.randint(1, s, (b,), generator=torch.Generator().manual_seed(5))
        kv_lens = lens.to(torch.uint32).cuda()
        max_kv = torch.tensor([int(lens.max())], dtype=torch.uint32, device=dev)
        is_done = torch.zeros(b, dtype=torch.uint8, device=dev)
        is_done[2] = 1
        down = L.decode(x, pending, kv_lens, max_kv, is_done)
        out = [host(x), host(down), host(L.qk), host(L.act)]

        # prefill: two prompts (64 and 40 new tokens after 0 and 10 cached) of the first two sequences
        q_lens = torch.tensor([64, 40] + [0] * (b - 2), dtype=torch.uint32, device=dev)
        kv_p = torch.tensor([64, 50] + [0] * (b - 2), dtype=torch.uint32, device=dev)
        t = 104
        unpad = torch.zeros(b, qc, dtype=torch.uint32, device=dev)
        offsets = torch.zeros(b, dtype=torch.uint32, device=dev)
        ops.launch_build_padding_index_maps(t, q_lens, unpad, offsets)
        xp = torch.randn(t, d, generator=g, device=dev).to(torch.bfloat16)
        assert L.launches_per_prefill(t) == (9 if fuse else 11)
        down_p = L.prefill(xp, None, q_lens, kv_p, 64, 64, unpad)
        torch.cuda.synchronize()
        out += [host(xp), host(down_p), host(L.k_cache), host(L.v_cache)]
        runs.append(out)
    names = ["x", "down", "scores", "swiglu", "prefill x", "prefill down", "K cache", "V cache"]
    for name, a, c in zip(names, *runs):
        assert bits_equal(a, c), name
