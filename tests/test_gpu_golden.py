"""Every reference unit-test case, run through the C ABI on the GPU and
checked against the reference's own CPU-helper outputs (tests/golden/).

Tolerances: the reference test's own (absolute, per case) always; in
addition fp32 results must be within 1e-5 relative of the reference output
(the parity bar), and RoPE / integer / copy results must be bit-identical.
"""
import numpy as np
import pytest
import torch

from llama2_b200 import ops
from oracle import port
from tests import golden_io
from tests.gpu_util import TORCH, bits_equal, dev, host, max_rel_err, round_to

pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


@pytest.mark.parametrize("case", golden_io.case_ids("embedding"))
@pytest.mark.parametrize("dt", ["f32", "f16", "bf16"])
def test_embedding(case, dt):
    _, a = golden_io.load("embedding")[case]
    table = dev(a["table"], TORCH[dt])
    ids = dev(a["ids"])
    out = torch.empty(ids.shape[0], table.shape[1], dtype=table.dtype, device="cuda")
    ops.launch_embedding(ids, table, out)
    want = torch.from_numpy(a["out"]).to(TORCH[dt])
    assert torch.equal(out.cpu(), want)


@pytest.mark.parametrize("case", golden_io.case_ids("rmsnorm"))
def test_rmsnorm(case):
    p, a = golden_io.load("rmsnorm")[case]
    dt = TORCH[p["dtype"]]
    x = dev(a["x"], dt)
    r = dev(a["residual"], dt)
    w = dev(a["w"], dt)
    ops.launch_fused_add_residual_rmsnorm(w, x, r, p["add"])
    tol = p["tol"]
    assert np.max(np.abs(host(x) - a["x_after"])) <= tol
    assert np.max(np.abs(host(r) - a["residual_out"])) <= tol
    if p["dtype"] == "f32":
        assert max_rel_err(host(r), a["residual_out"]) <= 1e-5
        assert bits_equal(host(x), a["x_after"])


@pytest.mark.parametrize("case", golden_io.case_ids("rope_decode"))
@pytest.mark.parametrize("use_table", [True, False])
def test_rope_decode(case, use_table):
    p, a = golden_io.load("rope_decode")[case]
    q = torch.zeros(a["q"].shape, device="cuda")
    k = torch.zeros(a["k"].shape, device="cuda")
    v = torch.zeros(a["v"].shape, device="cuda")
    fn = (ops.launch_fused_reshape_rope_kvcache_llama2_decode if p["pairing"]
          else ops.launch_fused_reshape_rope_kvcache_decode)
    fn(dev(a["input"]), dev(a["is_done"]), dev(a["kv_lens"]), q, k, v, use_table=use_table)
    if use_table:
        # Host-built angles + unfused products: identical to the reference's CPU oracle.
        assert bits_equal(host(q), a["q"]) and bits_equal(host(k), a["k"]) and bits_equal(host(v), a["v"])
    else:
        assert np.max(np.abs(host(q) - a["q"])) <= p["tol_qk"]
        assert np.max(np.abs(host(k) - a["k"])) <= p["tol_qk"]
        assert bits_equal(host(v), a["v"])


@pytest.mark.parametrize("case", golden_io.case_ids("rope_prefill"))
@pytest.mark.parametrize("use_table", [True, False])
def test_rope_prefill(case, use_table):
    p, a = golden_io.load("rope_prefill")[case]
    b = a["q_lens"].shape[0]
    unpad = torch.zeros(b, p["q_cache_len"], dtype=torch.uint32, device="cuda")
    offs = torch.zeros(b, dtype=torch.uint32, device="cuda")
    n = a["input"].shape[0]
    ops.launch_build_padding_index_maps(n, dev(a["q_lens"]), unpad, offs)
    assert bits_equal(host(unpad).reshape(-1)[:n], a["unpad_to_pad"])
    q = torch.zeros(a["q"].shape, device="cuda")
    k = torch.zeros(a["k"].shape, device="cuda")
    v = torch.zeros(a["v"].shape, device="cuda")
    fn = (ops.launch_fused_pad_reshape_transpose_rope_kvcache_llama2 if p["pairing"]
          else ops.launch_fused_pad_reshape_transpose_rope_kvcache)
    fn(dev(a["input"]), dev(a["q_lens"]), dev(a["kv_lens"]), unpad.view(-1), q, k, v, use_table=use_table)
    if use_table:
        assert bits_equal(host(q), a["q"]) and bits_equal(host(k), a["k"]) and bits_equal(host(v), a["v"])
    else:
        assert np.max(np.abs(host(q) - a["q"])) <= p["tol_qk"]
        assert np.max(np.abs(host(k) - a["k"])) <= p["tol_qk"]
        assert bits_equal(host(v), a["v"])


INTEGER = golden_io.load("integer")


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("mask.")))
def test_causal_mask(case):
    p, a = INTEGER[case]
    mask = torch.zeros(a["mask"].shape, dtype=torch.uint8, device="cuda")
    ops.launch_build_causal_mask(p["max_q"], p["max_kv"], dev(a["q_lens"]), dev(a["kv_lens"]), mask)
    assert bits_equal(host(mask), a["mask"])


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("maps.")))
def test_padding_maps(case):
    p, a = INTEGER[case]
    b = a["seq_lens"].shape[0]
    n = a["unpad_to_pad"].shape[0]
    unpad = torch.zeros(b, p["q_cache_len"], dtype=torch.uint32, device="cuda")
    offs = torch.full((b,), 7, dtype=torch.uint32, device="cuda")
    ops.launch_build_padding_index_maps(n, dev(a["seq_lens"]), unpad, offs)
    assert bits_equal(host(unpad).reshape(-1)[:n], a["unpad_to_pad"])
    assert bits_equal(host(offs), a["seq_offsets"])


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("lens.")))
@pytest.mark.parametrize("max_on_device", [True, False])
def test_update_lens(case, max_on_device):
    _, a = INTEGER[case]
    kv = dev(a["kv_lens"])
    if max_on_device:
        mq = torch.zeros(1, dtype=torch.uint32, device="cuda")
        mkv = torch.zeros(1, dtype=torch.uint32, device="cuda")
    else:
        mq = torch.zeros(1, dtype=torch.uint32)
        mkv = torch.zeros(1, dtype=torch.uint32)
    ops.launch_update_q_kv_lens(dev(a["q_lens"]), kv, mq, mkv)
    assert bits_equal(host(kv), a["kv_lens_out"])
    assert int(mq.cpu()[0]) == int(a["max_q"]) and int(mkv.cpu()[0]) == int(a["max_kv"])


@pytest.mark.parametrize("case", sorted(c for c in INTEGER if c.startswith("ptr.")))
def test_ptr_arrays(case):
    p, _ = INTEGER[case]
    b, hq, hkv, qc, s, hs = (p[k] for k in ("batch", "q_heads", "kv_heads", "q_cache_len", "kv_cache_len",
                                            "head_size"))
    dt = torch.float32 if p["elem_size"] == 4 else torch.float16
    shapes = [(b, hq, qc, hs), (b, hq, 1, hs), (b, hkv, s, hs), (b, hkv, s, hs), (b, hq, qc, s), (b, hq, 1, s),
              (b, hq, qc, hs), (b, hq, 1, hs)]
    ts = [torch.zeros(sh, dtype=dt, device="cuda") for sh in shapes]
    arrays = [torch.zeros(b * hq, dtype=torch.int64, device="cuda") for _ in range(8)]
    ops.launch_build_q_k_v_qk_qkv_array(*ts, *arrays)
    bases = [t.data_ptr() for t in ts]
    strides = [sh[2] * sh[3] * p["elem_size"] for sh in shapes]
    want = port.build_ptr_arrays(bases, strides, b, hq, hkv)
    got = np.stack([host(x).astype(np.uint64) for x in arrays])
    assert np.array_equal(got, want)


@pytest.mark.parametrize("case", golden_io.case_ids("linear"))
def test_linear(case):
    p, a = golden_io.load("linear")[case]
    dt = TORCH[p["dtype"]]
    A, B = dev(a["A"], dt), dev(a["B"], dt)
    m, n, k = p["M"], p["N"], p["K"]
    if p["batch"] == 0:
        C = torch.zeros(m, n, dtype=dt, device="cuda")
        ops.launch_linear(p["trans_a"], p["trans_b"], m, n, k, A, B, C)
    else:
        bt = p["batch"]
        C = torch.zeros(bt, m, n, dtype=dt, device="cuda")
        ptr = lambda t: torch.tensor([t[i].data_ptr() for i in range(bt)], dtype=torch.int64, device="cuda")
        ops.launch_linear(p["trans_a"], p["trans_b"], m, n, k, A, B, C, ptr(A), ptr(B), ptr(C))
    assert np.max(np.abs(host(C) - a["C"])) <= p["tol"]
    if p["dtype"] == "f32":
        # Small integers: fp32 accumulation is exact in any order.
        assert bits_equal(host(C), a["C"])


@pytest.mark.parametrize("case", golden_io.case_ids("score"))
def test_masked_attention_score(case):
    p, a = golden_io.load("score")[case]
    dt = TORCH[p["dtype"]]
    qk = dev(a["qk"].astype(np.float32), dt)
    ops.launch_compute_masked_attention_score(p["head_dim"], p["max_q"], p["max_kv"], dev(a["q_lens"]),
                                              dev(a["mask"]), qk)
    exp = a["expected"].astype(np.float32)
    assert np.max(np.abs(host(qk) - exp)) <= p["tol"]
    if p["dtype"] == "f32":
        assert max_rel_err(host(qk), exp) <= 1e-5


@pytest.mark.parametrize("case", golden_io.case_ids("swiglu"))
def test_swiglu(case):
    p, a = golden_io.load("swiglu")[case]
    dt = TORCH[p["dtype"]]
    inp = dev(a["input"], dt)
    out = torch.empty(inp.shape[0], inp.shape[1] // 2, dtype=dt, device="cuda")
    ops.launch_swiglu(inp, out)
    assert np.max(np.abs(host(out) - a["out"])) <= p["tol"]
    if p["dtype"] == "f32":
        assert max_rel_err(host(out), a["out"]) <= 1e-5
    else:
        # 16-bit I/O: against the oracle on the rounded inputs, 1e-2 relative.
        ref = port.swiglu(round_to(a["input"], dt))
        assert max_rel_err(host(out), round_to(ref, dt), floor=1e-3) <= 1e-2
