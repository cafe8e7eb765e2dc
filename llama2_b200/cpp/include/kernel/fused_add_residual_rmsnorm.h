// launch_fused_add_residual_rmsnorm — the reference's
// include/kernel/fused_add_residual_rmsnorm.h:16-19 signature.
#pragma once

template <typename T>
class Tensor;

// if add_residual: x = x + residual (written back to x)
// residual = x * weights / sqrt(mean(x^2) + RMSNORM_EPS)   (the result lands in `residual`)
template <typename T, bool add_residual>
void launch_fused_add_residual_rmsnorm(const Tensor<T> &weights, // (embed_dim)
                                       Tensor<T> &x,             // (num_input_tokens, embed_dim)
                                       Tensor<T> &residual);     // (num_input_tokens, embed_dim)
