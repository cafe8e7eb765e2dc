// launch_swiglu — the reference's include/kernel/swiglu.h:6-8 signature.
#pragma once

template <typename T>
class Tensor;

// output[t, i] = silu(input[t, i]) * input[t, F + i]
template <typename T>
void launch_swiglu(const Tensor<T> &input, // (num_input_tokens, 2 * intermediate_size)
                   Tensor<T> &output);     // (num_input_tokens, intermediate_size)
