"""l2k_decode_step_no_alloc (static scratch, no workspace argument) against
l2k_decode_step (caller workspace) on the same inputs: two steps in a row,
bitwise equal outputs. Named to be collected last; also passes alone."""
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


@pytest.mark.parametrize("name,batch", [("7b-b1", 1), ("7b-b64-bf16", 5)])
def test_no_alloc_matches_workspace_entry(name, batch):
    w = with_batch(WORKLOADS[name], batch)
    inp = host_inputs(w, seed=21)
    ref = Chain(w, inp, fused=False)   # buffers only; stepped through ops.decode_step below
    new = Chain(w, inp, fused=False)
    ws = ops.decode_step_workspace(ref.device)
    for _ in range(2):
        ops.decode_step(**ref._step_tensors(), workspace=ws)
        ops.decode_step_no_alloc(**new._step_tensors())
    torch.cuda.synchronize()
    for n in ("kv_lens", "max_lens", "x", "normed", "q", "k_cache", "v_cache", "qk", "ffn_out"):
        assert bits_equal(host(getattr(new, n)), host(getattr(ref, n))), n
    assert int(host(ws).astype(np.int64).sum()) == 0
    assert int(host(ref.kv_lens).astype(np.int64).sum()) == int(inp["kv_lens"].astype(np.int64).sum()) + 2 * batch
