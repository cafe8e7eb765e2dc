// launch_embedding — the reference's include/kernel/embedding.h:6-9 signature.
#pragma once

template <typename T>
class Tensor;

// output[t, :] = embed_table[input_ids[t], :]; ids >= vocab give a zero row.
template <typename T>
void launch_embedding(const Tensor<unsigned int> &input_ids, // (num_input_tokens)
                      const Tensor<T> &embed_table,          // (vocab_size, embed_dim)
                      Tensor<T> &output);                    // (num_input_tokens, embed_dim)
