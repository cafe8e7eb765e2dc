// launch_build_padding_index_maps — the reference's include/kernel/build_padding_index_maps.h:6-10 signature.
#pragma once

template <typename T>
class Tensor;

void launch_build_padding_index_maps(const unsigned int num_input_tokens,
                                     const Tensor<unsigned int> &seq_lens,   // (batch)
                                     Tensor<unsigned int> &unpad_to_pad_idx, // (batch, q_cache_len); first num_input_tokens written
                                     Tensor<unsigned int> &seq_offsets);     // (batch)
