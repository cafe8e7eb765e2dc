// launch_compute_masked_attention_score — the reference's
// include/kernel/compute_masked_attention_score.h:6-12 signature.
#pragma once

template <typename T>
class Tensor;

// In place on qk for rows q < q_lens[b] and keys k < max_kv_len:
// qk = mask ? exp(qk / sqrt(head_dim) - max) / (sum + SOFTMAX_EPS) : 0.
template <typename T, typename MASK_T>
void launch_compute_masked_attention_score(const unsigned int head_dim, const unsigned int max_q_len,
                                           const unsigned int max_kv_len,
                                           const Tensor<unsigned int> &q_lens, // (batch)
                                           const Tensor<MASK_T> &mask,         // (batch, q_cache_len, kv_cache_len)
                                           Tensor<T> &qk);                     // (batch, Hq, q_cache_len, kv_cache_len)
