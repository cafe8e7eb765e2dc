"""l2k_decode_step_no_alloc and l2k_decode_step_attention_no_alloc (the
library's static scratch, no workspace argument) against l2k_decode_step /
l2k_decode_step_attention (caller workspace) on the same inputs: two steps
in a row, bitwise equal outputs. Named to be collected last; also passes
alone. The entries serve callers that cannot hand the library device memory
(a binding that passes only the tensors it already has)."""
import ctypes

import numpy as np
import pytest
import torch

from llama2_b200 import capi, ops
from llama2_b200.chain import Chain
from llama2_b200.workloads import WORKLOADS, host_inputs, with_batch
from tests.gpu_util import bits_equal, host

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _lib(cuda_lib):
    yield
    assert capi.lib().l2k_device_error(1) == 0


@pytest.mark.parametrize("attention", [False, True])
@pytest.mark.parametrize("name,batch", [("7b-b1", 1), ("7b-b64-bf16", 5)])
def test_no_alloc_matches_workspace_entry(name, batch, attention):
    w = with_batch(WORKLOADS[name], batch)
    inp = host_inputs(w, seed=21)
    ref = Chain(w, inp, fused=False, attention_output=attention)  # buffers only; stepped through ops below
    new = Chain(w, inp, fused=False, attention_output=attention)
    ws = ops.decode_step_workspace(ref.device)
    shape = (w.batch, w.heads, 1, w.head_dim)
    for _ in range(2):
        if attention:
            ops.decode_step_attention(**ref._step_tensors(), workspace=ws, attn_out=ref.attn_out.view(shape))
            ops.decode_step_attention_no_alloc(**new._step_tensors(), attn_out=new.attn_out.view(shape))
        else:
            ops.decode_step(**ref._step_tensors(), workspace=ws)
            ops.decode_step_no_alloc(**new._step_tensors())
    torch.cuda.synchronize()
    names = ["kv_lens", "max_lens", "x", "normed", "q", "k_cache", "v_cache", "qk", "ffn_out"]
    for n in names + (["attn_out"] if attention else []):
        assert bits_equal(host(getattr(new, n)), host(getattr(ref, n))), n
    assert int(host(ws).astype(np.int64).sum()) == 0
    # both steps advanced every length by one: the scratch counter was zero before each step
    for ch in (ref, new):
        assert int(host(ch.kv_lens).astype(np.int64).sum()) == int(inp["kv_lens"].astype(np.int64).sum()) + 2 * batch


def test_no_alloc_rejects_a_stream_of_another_device():
    """A stream of a device that is not current is refused before anything
    runs (the scratch is per device); needs two visible devices."""
    if torch.cuda.device_count() < 2:
        pytest.skip("one visible device")
    w = with_batch(WORKLOADS["7b-b1"], 1)
    ch = Chain(w, host_inputs(w, seed=3), device="cuda:0", fused=False)
    other = torch.cuda.Stream(device=1)
    t = ch._step_tensors()
    with torch.cuda.device(0):
        args = ops._decode_step_args(*(t[k] for k in (
            "q_lens", "kv_lens", "max_lens", "input_ids", "embed_table", "norm_weight", "x", "normed", "qkv",
            "is_done", "q", "k_cache", "v_cache", "qk", "gate_up", "ffn_out", "pairing", "use_table")))
        st = capi.lib().l2k_decode_step_no_alloc(ctypes.byref(args), ctypes.c_void_p(other.cuda_stream))
    assert st == 1  # L2K_ERR_INVALID_ARGUMENT
    assert b"belongs to device 1" in capi.lib().l2k_last_error_message()
