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
from oracle import port
from tests import golden_io
from tests.gpu_util import TORCH, dev, host

pytestmark = pytest.mark.gpu

F32 = np.float32


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield


def _np_dtype(dt):
    return {"f32": np.float32, "f16": np.float16}.get(dt)


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
    # is the padded row it names, checked as a checksum of row checksums.
    b, h, qc, hd = 8, 32, 2048, 128
    qkv = torch.randn(b, h, qc, hd, device="cuda", dtype=torch.bfloat16)
    lens = [2048, 1500, 2048, 7, 2048, 1024, 2048, 333]
    slots, t = _slots(lens, qc)
    out = torch.empty(t, h * hd, device="cuda", dtype=torch.bfloat16)
    ops.launch_fused_transpose_unpad(t, qkv, dev(slots), out)
    s = torch.from_numpy(slots[:t].astype(np.int64)).cuda()
    want = qkv.permute(0, 2, 1, 3).reshape(b * qc, h * hd).index_select(0, s)
    assert torch.equal(out, want)
