// launch_fused_reshape_rope_kvcache_decode — the reference's
// include/kernel/fused_reshape_rope_kvcache_decode.h:6-12 signature.
#pragma once

template <typename T>
class Tensor;

// RoPE with pairs (2i, 2i+1) at pos = kv_lens[b] - 1; q written, k and v rows
// appended at pos; sequences with is_done[b] != 0 are skipped.
template <typename T>
void launch_fused_reshape_rope_kvcache_decode(const Tensor<T> &input,               // (batch, (Hq + 2 Hkv) * head_dim)
                                              const Tensor<unsigned char> &is_done, // (batch)
                                              const Tensor<unsigned int> &kv_lens,  // (batch), includes this token
                                              Tensor<T> &q,                         // (batch, Hq, 1, head_dim)
                                              Tensor<T> &k,                         // (batch, Hkv, kv_cache_len, head_dim)
                                              Tensor<T> &v);                        // (batch, Hkv, kv_cache_len, head_dim)
