// launch_build_causal_mask — the reference's include/kernel/build_causal_mask.h:6-11 signature.
#pragma once

template <typename T>
class Tensor;

// mask[b, q, k] over [0, max_q_len) x [0, max_kv_len) with the reference's
// unsigned expression q < q_len && k < kv_len && q >= k - (kv_len - q_len).
template <typename T>
void launch_build_causal_mask(const unsigned int max_q_len,
                              const unsigned int max_kv_len,
                              const Tensor<unsigned int> &q_lens,  // (batch)
                              const Tensor<unsigned int> &kv_lens, // (batch)
                              Tensor<T> &mask);                    // (batch, q_cache_len, kv_cache_len)
