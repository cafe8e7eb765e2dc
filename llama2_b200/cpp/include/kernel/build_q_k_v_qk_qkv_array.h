// launch_build_q_k_v_qk_qkv_array — the reference's include/kernel/build_q_k_v_qk_qkv_array.h:6-22 signature.
#pragma once

template <typename T>
class Tensor;

// Per (batch, q head) slice pointers; k and v slots point at the grouped kv head.
template <typename T>
void launch_build_q_k_v_qk_qkv_array(Tensor<T> &q, Tensor<T> &q_decode, Tensor<T> &k, Tensor<T> &v, Tensor<T> &qk,
                                     Tensor<T> &qk_decode, Tensor<T> &qkv, Tensor<T> &qkv_decode,
                                     Tensor<void *> &q_array, Tensor<void *> &q_decode_array,
                                     Tensor<void *> &k_array, Tensor<void *> &v_array, Tensor<void *> &qk_array,
                                     Tensor<void *> &qk_decode_array, Tensor<void *> &qkv_array,
                                     Tensor<void *> &qkv_decode_array);
