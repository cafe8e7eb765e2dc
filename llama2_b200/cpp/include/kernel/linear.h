// launch_linear — the reference's include/kernel/linear.h:9-24 signature.
#pragma once

struct cublasContext;
typedef struct cublasContext *cublasHandle_t;

template <typename T>
class Tensor;

// Row-major C = op(A) op(B) (M x N), fp32 accumulation, by this library's own
// kernel on the legacy default stream; cublas_handle is accepted for source
// compatibility and not used. For C of rank > 2 the GEMMs are batched through
// the device pointer arrays; for rank 2 pass empty Tensor<void *>({}).
template <typename T>
void launch_linear(cublasHandle_t &cublas_handle, const bool trans_A, const bool trans_B, const unsigned int M,
                   const unsigned int N, const unsigned int K, const Tensor<T> &A, const Tensor<T> &B, Tensor<T> &C,
                   const Tensor<void *> &A_array, const Tensor<void *> &B_array, Tensor<void *> &C_array);
