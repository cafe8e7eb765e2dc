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

// The scores of launch_decode_attention_scores (into qk) and the attention
// output qkv (batch, Hq, 1, hd) = P.V over keys 0..kv_lens[b]-1, in one pass
// over the K and V caches.
template <typename T>
void launch_decode_attention(const Tensor<T> &q, const Tensor<T> &k, const Tensor<T> &v,
                             const Tensor<unsigned int> &kv_lens, const Tensor<unsigned int> &max_kv_len, Tensor<T> &qk,
                             Tensor<T> &qkv);

// P.V at the qk x v launch_linear call site without pointer arrays:
// qkv[b, h, i, :] = sum_{j < N} qk[b, h, i, j] * v[b, h / (Hq/Hkv), j, :], i < M.
template <typename T>
void launch_attention_qkv(const Tensor<T> &qk, const Tensor<T> &v, Tensor<T> &qkv, const unsigned int M,
                          const unsigned int N);

// The whole decode chain of one layer step in one launch (no counterpart in
// the reference): kv_lens += q_lens and max_lens = (max q_len, max kv_len);
// x = embed_table[input_ids]; normed = RMSNorm(x) with norm_weight; RoPE of
// q and k at kv_len - 1 ((i, i + hd/2) pairs when llama2_pairs, (2i, 2i+1)
// otherwise) with the K/V rows appended to the caches (skipped for
// is_done); qk = softmax over keys 0..kv_len-1; ffn_out = silu(gate) * up.
// Same results as running those operators one after another. Uses the
// library's static scratch (l2k_decode_step_no_alloc): steps on one device
// must not overlap, which the legacy default stream guarantees.
template <typename T>
void launch_decode_step(const Tensor<unsigned int> &q_lens, Tensor<unsigned int> &kv_lens,
                        Tensor<unsigned int> &max_lens, const Tensor<unsigned int> &input_ids,
                        const Tensor<T> &embed_table, const Tensor<T> &norm_weight, Tensor<T> &x, Tensor<T> &normed,
                        const Tensor<T> &qkv, const Tensor<unsigned char> &is_done, Tensor<T> &q, Tensor<T> &k_cache,
                        Tensor<T> &v_cache, Tensor<T> &qk, const Tensor<T> &gate_up, Tensor<T> &ffn_out,
                        bool llama2_pairs);

// launch_decode_step with the attention output attn_out (batch, Hq, 1, hd) =
// P.V over the appended V cache, in the same launch (static scratch, as
// launch_decode_step).
template <typename T>
void launch_decode_step_attention(const Tensor<unsigned int> &q_lens, Tensor<unsigned int> &kv_lens,
                                  Tensor<unsigned int> &max_lens, const Tensor<unsigned int> &input_ids,
                                  const Tensor<T> &embed_table, const Tensor<T> &norm_weight, Tensor<T> &x,
                                  Tensor<T> &normed, const Tensor<T> &qkv, const Tensor<unsigned char> &is_done,
                                  Tensor<T> &q, Tensor<T> &k_cache, Tensor<T> &v_cache, Tensor<T> &qk,
                                  const Tensor<T> &gate_up, Tensor<T> &ffn_out, Tensor<T> &attn_out,
                                  bool llama2_pairs);
