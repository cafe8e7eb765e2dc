// Fused attention-score operators of this library (no single counterpart in
// the reference, whose chain runs launch_linear for QK^T and then
// launch_compute_masked_attention_score on a materialized mask).
#pragma once

template <typename T>
class Tensor;

// One query row per sequence: q (batch, Hq, 1, hd), k (batch, Hkv, S, hd),
// qk (batch, Hq, 1, S); keys 0..kv_lens[b]-1 kept; max_kv_len is a 1-element
// device tensor (as written by launch_update_q_kv_lens into device tensors).
template <typename T>
void launch_decode_attention_scores(const Tensor<T> &q, const Tensor<T> &k, const Tensor<unsigned int> &kv_lens,
                                    const Tensor<unsigned int> &max_kv_len, Tensor<T> &qk);

// q_len rows per sequence, causal: row i keeps keys <= kv_len - q_len + i.
template <typename T>
void launch_prefill_attention_scores(const Tensor<T> &q, const Tensor<T> &k, const Tensor<unsigned int> &q_lens,
                                     const Tensor<unsigned int> &kv_lens, const unsigned int max_q_len,
                                     const unsigned int max_kv_len, Tensor<T> &qk);
