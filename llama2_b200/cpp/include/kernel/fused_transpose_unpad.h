// launch_fused_transpose_unpad — the reference's
// include/kernel/fused_transpose_unpad.h:6-11 signature.
#pragma once

template <typename T>
class Tensor;

// unpad_qkv[t, h * head_size + d] = qkv[b, h, i, d], b * q_cache_len + i = unpad_to_pad_idx[t]
template <typename T>
void launch_fused_transpose_unpad(const unsigned int num_input_tokens,
                                  const Tensor<T> &qkv,                         // (batch_size, q_head_num, q_cache_len, head_size)
                                  const Tensor<unsigned int> &unpad_to_pad_idx, // (batch_size, q_cache_len)
                                  Tensor<T> &unpad_qkv);                        // (num_input_tokens, embed_dim)
