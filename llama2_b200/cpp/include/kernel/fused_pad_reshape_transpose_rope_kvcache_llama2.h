// launch_fused_pad_reshape_transpose_rope_kvcache_llama2 — the reference's
// include/kernel/fused_pad_reshape_transpose_rope_kvcache_llama2.h:6-13 signature.
#pragma once

template <typename T>
class Tensor;

// As launch_fused_pad_reshape_transpose_rope_kvcache with pairs (i, i + head_dim/2).
template <typename T>
void launch_fused_pad_reshape_transpose_rope_kvcache_llama2(const Tensor<T> &input,
                                                            const Tensor<unsigned int> &q_lens,
                                                            const Tensor<unsigned int> &kv_lens,
                                                            const Tensor<unsigned int> &unpad_to_pad_idx,
                                                            Tensor<T> &q,
                                                            Tensor<T> &k,
                                                            Tensor<T> &v);
