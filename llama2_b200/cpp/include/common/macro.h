// Error-check macros of the C++ operator API: a failed CUDA call prints the
// error and exits, as the reference's include/common/macro.h:22-40 do.
#pragma once

#include <cstdio>
#include <cstdlib>
#include <cuda_runtime.h>

#define CUDA_CHECK(call)                                                                              \
    do                                                                                                \
    {                                                                                                 \
        cudaError_t err_ = (call);                                                                    \
        if (err_ != cudaSuccess)                                                                      \
        {                                                                                             \
            std::fprintf(stderr, "CUDA error: %s at %s:%d\n", cudaGetErrorString(err_), __FILE__, __LINE__); \
            std::exit(EXIT_FAILURE);                                                                  \
        }                                                                                             \
    } while (0)

#define CUDA_KERNEL_LAUNCH_CHECK()                                                                    \
    do                                                                                                \
    {                                                                                                 \
        cudaError_t err_ = cudaGetLastError();                                                        \
        if (err_ != cudaSuccess)                                                                      \
        {                                                                                             \
            std::fprintf(stderr, "CUDA kernel launch error: %s at %s:%d\n", cudaGetErrorString(err_), __FILE__, \
                         __LINE__);                                                                   \
            std::exit(EXIT_FAILURE);                                                                  \
        }                                                                                             \
    } while (0)

// For callers that hold a cuBLAS handle (the reference's include/common/macro.h:42-50 offers the same check);
// expands only where cublas_v2.h is included. The operators of this library do not call cuBLAS.
#define CUBLAS_CHECK(call)                                                                            \
    do                                                                                                \
    {                                                                                                 \
        cublasStatus_t st_ = (call);                                                                  \
        if (st_ != CUBLAS_STATUS_SUCCESS)                                                             \
        {                                                                                             \
            std::fprintf(stderr, "cuBLAS error: %s at %s:%d\n", cublasGetStatusString(st_), __FILE__, __LINE__); \
            std::exit(EXIT_FAILURE);                                                                  \
        }                                                                                             \
    } while (0)

#define MALLOC_CHECK(ptr)                                                                             \
    do                                                                                                \
    {                                                                                                 \
        if ((ptr) == nullptr)                                                                         \
        {                                                                                             \
            std::fprintf(stderr, "Host memory allocation failed at %s:%d\n", __FILE__, __LINE__);     \
            std::exit(EXIT_FAILURE);                                                                  \
        }                                                                                             \
    } while (0)
