// Shared device/host helpers of the sm_100a kernels: element types, 16-byte
// global memory access with cache hints, argument checking and error state.
#pragma once

#include <type_traits>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_fp8.h>
#include <stdint.h>

#include "llama2_b200.h"

namespace l2k
{

// ---------------------------------------------------------------------------
// Error reporting (status.cu). set_error returns its status so that
// entry points can write `return set_error(...)`.
// ---------------------------------------------------------------------------
int set_error(int status, const char *fmt, ...);
int check_launch(const char *what);

#define L2K_REQUIRE(cond, ...)                                               \
    do                                                                       \
    {                                                                        \
        if (!(cond))                                                         \
            return ::l2k::set_error(L2K_ERR_INVALID_ARGUMENT, __VA_ARGS__);  \
    } while (0)

#define L2K_REQUIRE_SHAPE(cond, ...)                                         \
    do                                                                       \
    {                                                                        \
        if (!(cond))                                                         \
            return ::l2k::set_error(L2K_ERR_UNSUPPORTED_SHAPE, __VA_ARGS__); \
    } while (0)

inline bool is_aligned(const void *p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }
inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t dtype_size(int dtype) { return dtype == L2K_F32 ? 4 : 2; }
inline bool dtype_ok(int dtype) { return dtype == L2K_F32 || dtype == L2K_F16 || dtype == L2K_BF16; }

constexpr int kNumSMs = 148; // B200
int num_sms();               // queried once per process (status.cu)

// ---------------------------------------------------------------------------
// Element types. All arithmetic is fp32; 16-bit types round to nearest-even.
// ---------------------------------------------------------------------------
template <typename T>
struct Elem;
template <>
struct Elem<float>
{
    static __device__ __forceinline__ float to_f(float v) { return v; }
    static __device__ __forceinline__ float from_f(float v) { return v; }
};
template <>
struct Elem<__half>
{
    static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
    static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};
template <>
struct Elem<__nv_bfloat16>
{
    static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
    static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

template <typename T>
__device__ __forceinline__ float to_f(T v) { return Elem<T>::to_f(v); }
template <typename T>
__device__ __forceinline__ T from_f(float v) { return Elem<T>::from_f(v); }

// 16 bytes of elements, viewed as N values of T.
template <typename T>
struct alignas(16) Vec16
{
    static constexpr int N = 16 / sizeof(T);
    T v[N];
};

// ---------------------------------------------------------------------------
// 16-byte global accesses.
//   ldg_stream: read-only, do not allocate in L1 (data read once).
//   ldg_keep:   read-only through the non-coherent path (reused data).
//   stg_stream: streaming store (evict-first).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_stream(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ldg_keep(const void *p)
{
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ldg_coherent(const void *p)
{
    uint4 r;
    asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ void stg_stream(void *p, uint4 v)
{
    asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}
__device__ __forceinline__ void stg(void *p, uint4 v)
{
    asm volatile("st.global.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
}

template <typename T>
__device__ __forceinline__ Vec16<T> as_vec(uint4 u)
{
    Vec16<T> r;
    static_assert(sizeof(r) == sizeof(u), "Vec16 size");
    __builtin_memcpy(&r, &u, 16);
    return r;
}
template <typename T>
__device__ __forceinline__ uint4 as_u4(const Vec16<T> &v)
{
    uint4 r;
    __builtin_memcpy(&r, &v, 16);
    return r;
}

// silu(g) * u as the reference's SwiGLU oracle evaluates it:
// (g * (1 / (1 + exp(-g)))) * u. fp32 data: IEEE reciprocal and
// full-precision expf. 16-bit data (whose result is rounded to 8 or 11
// mantissa bits): the fast exp and reciprocal intrinsics, a few ulp of fp32
// each, which halve the instructions of this otherwise issue-bound
// streaming step.
template <typename T>
__device__ __forceinline__ float silu_mul(float g, float u)
{
    if constexpr (std::is_same<T, float>::value)
    {
        const float sig = __frcp_rn(__fadd_rn(1.0f, expf(-g)));
        return __fmul_rn(__fmul_rn(g, sig), u);
    }
    else
    {
        const float sig = __fdividef(1.0f, __fadd_rn(1.0f, __expf(-g)));
        return __fmul_rn(__fmul_rn(g, sig), u);
    }
}

// ---------------------------------------------------------------------------
// Reductions.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}
__device__ __forceinline__ uint32_t warp_max_u32(uint32_t v)
{
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum/max of one value per thread; every thread gets the result.
// `scratch` holds at least 32 floats; the block size is a multiple of 32.
__device__ __forceinline__ float block_sum(float v, float *scratch)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0)
        scratch[warp] = v;
    __syncthreads();
    v = lane < nwarps ? scratch[lane] : 0.f;
    return warp_sum(v);
}
__device__ __forceinline__ float block_max(float v, float *scratch)
{
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    v = warp_max(v);
    __syncthreads();
    if (lane == 0)
        scratch[warp] = v;
    __syncthreads();
    v = lane < nwarps ? scratch[lane] : -INFINITY;
    return warp_max(v);
}

} // namespace l2k

// dtype dispatch: runs the body (variadic, so it may contain commas) with `T`
// bound to the element type.
#define L2K_DISPATCH(dtype, ...)                                                        \
    switch (dtype)                                                                      \
    {                                                                                   \
    case L2K_F32:                                                                       \
    {                                                                                   \
        using T = float;                                                                \
        __VA_ARGS__;                                                                    \
    }                                                                                   \
    break;                                                                              \
    case L2K_F16:                                                                       \
    {                                                                                   \
        using T = __half;                                                               \
        __VA_ARGS__;                                                                    \
    }                                                                                   \
    break;                                                                              \
    case L2K_BF16:                                                                      \
    {                                                                                   \
        using T = __nv_bfloat16;                                                        \
        __VA_ARGS__;                                                                    \
    }                                                                                   \
    break;                                                                              \
    default:                                                                            \
        return ::l2k::set_error(L2K_ERR_UNSUPPORTED_DTYPE, "unsupported dtype %d", (int)(dtype)); \
    }
