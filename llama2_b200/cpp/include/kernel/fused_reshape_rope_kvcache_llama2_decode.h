// launch_fused_reshape_rope_kvcache_llama2_decode — the reference's
// include/kernel/fused_reshape_rope_kvcache_llama2_decode.h:6-12 signature.
#pragma once

template <typename T>
class Tensor;

// As launch_fused_reshape_rope_kvcache_decode with pairs (i, i + head_dim/2).
template <typename T>
void launch_fused_reshape_rope_kvcache_llama2_decode(const Tensor<T> &input,
                                                     const Tensor<unsigned char> &is_done,
                                                     const Tensor<unsigned int> &kv_lens,
                                                     Tensor<T> &q,
                                                     Tensor<T> &k,
                                                     Tensor<T> &v);
