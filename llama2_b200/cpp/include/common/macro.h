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
