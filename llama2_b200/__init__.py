"""B200-native (sm_100a) Llama-2 layer kernels behind the pentatracy5/llama2
operator API.

    llama2_b200.capi      — ctypes binding of the C ABI (include/llama2_b200.h)
    llama2_b200.ops       — the reference's launch_* operators over torch tensors
    llama2_b200.chain     — the decode / prefill layer-kernel chain (CUDA graphs)
    llama2_b200.workloads — benchmark shapes and seeded synthetic inputs
    llama2_b200.build     — builds libllama2_b200.so in-tree for sm_100a
"""
from . import capi  # noqa: F401

__all__ = ["capi", "ops", "chain", "workloads", "build"]
