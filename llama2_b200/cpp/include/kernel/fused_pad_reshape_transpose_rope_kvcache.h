// launch_fused_pad_reshape_transpose_rope_kvcache — the reference's
// include/kernel/fused_pad_reshape_transpose_rope_kvcache.h:6-13 signature.
#pragma once

template <typename T>
class Tensor;

// Prefill: token t of sequence b (via unpad_to_pad_idx) at pos = kv_len - q_len + t;
// q padded to (batch, Hq, q_cache_len, head_dim); k, v appended at pos. Pairs (2i, 2i+1).
template <typename T>
void launch_fused_pad_reshape_transpose_rope_kvcache(const Tensor<T> &input,                       // (num_input_tokens, (Hq + 2 Hkv) * head_dim)
                                                     const Tensor<unsigned int> &q_lens,           // (batch)
                                                     const Tensor<unsigned int> &kv_lens,          // (batch), history + new
                                                     const Tensor<unsigned int> &unpad_to_pad_idx, // (num_input_tokens)
                                                     Tensor<T> &q,                                 // (batch, Hq, q_cache_len, head_dim)
                                                     Tensor<T> &k,                                 // (batch, Hkv, kv_cache_len, head_dim)
                                                     Tensor<T> &v);                                // (batch, Hkv, kv_cache_len, head_dim)
