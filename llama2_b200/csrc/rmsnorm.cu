// Fused add-residual + RMSNorm.
//
//   if ADD: x = x + residual (written back to x, rounded to T)
//   residual = x * w * inv_rms,  inv_rms = 1 / sqrt(sum(x^2) / D + 1e-5)
//
// One CTA per row (rows strided by gridDim.x). The row is read from HBM
// exactly once and kept in registers (NV 16-byte chunks per thread); the
// sum of squares is a warp-shuffle + shared-memory block reduction in fp32;
// inv_rms is computed with IEEE division and square root (the reference
// oracle's 1/std::sqrt, not rsqrtf) and stays fp32 for the final products,
// which are evaluated as (x * w) * inv_rms like the oracle. For 16-bit types
// the sum of squares uses the stored (rounded) x.
//
// Reference: src/kernel/fused_add_residual_rmsnorm.cu:11-126 (reads the row
// twice, casts inv_var to T).
#include "common.cuh"

#include <algorithm>

namespace l2k
{
namespace
{

constexpr float kRmsEps = 1e-5f;
constexpr int kThreads = 256;

template <typename T, int NV, bool ADD>
__global__ void __launch_bounds__(kThreads) rmsnorm_vec_kernel(const T *__restrict__ w, T *__restrict__ x,
                                                               T *__restrict__ res, int64_t n_rows, int64_t dim)
{
    constexpr int N = Vec16<T>::N;
    __shared__ float scratch[32];
    const int64_t chunks = dim / N;
    const float fdim = (float)dim;
    for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x)
    {
        T *xr = x + row * dim;
        T *rr = res + row * dim;
        float v[NV][N];
        float sq = 0.f;
#pragma unroll
        for (int j = 0; j < NV; ++j)
        {
            const int64_t c = threadIdx.x + (int64_t)j * kThreads;
            if (c < chunks)
            {
                Vec16<T> xv = as_vec<T>(ldg_coherent(xr + c * N));
                if constexpr (ADD)
                {
                    const Vec16<T> rv = as_vec<T>(ldg_coherent(rr + c * N));
#pragma unroll
                    for (int e = 0; e < N; ++e)
                        xv.v[e] = from_f<T>(__fadd_rn(to_f(xv.v[e]), to_f(rv.v[e])));
                    stg(xr + c * N, as_u4(xv));
                }
#pragma unroll
                for (int e = 0; e < N; ++e)
                {
                    v[j][e] = to_f(xv.v[e]);
                    sq = fmaf(v[j][e], v[j][e], sq);
                }
            }
        }
        const float total = block_sum(sq, scratch);
        const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, fdim), kRmsEps)));
#pragma unroll
        for (int j = 0; j < NV; ++j)
        {
            const int64_t c = threadIdx.x + (int64_t)j * kThreads;
            if (c < chunks)
            {
                const Vec16<T> wv = as_vec<T>(ldg_keep(w + c * N));
                Vec16<T> o;
#pragma unroll
                for (int e = 0; e < N; ++e)
                    o.v[e] = from_f<T>(__fmul_rn(__fmul_rn(v[j][e], to_f(wv.v[e])), inv_rms));
                stg(rr + c * N, as_u4(o));
            }
        }
    }
}

// Any dim / alignment: two passes over the row (the second re-reads it,
// normally from L2).
template <typename T, bool ADD>
__global__ void __launch_bounds__(kThreads) rmsnorm_generic_kernel(const T *__restrict__ w, T *__restrict__ x,
                                                                   T *__restrict__ res, int64_t n_rows, int64_t dim)
{
    __shared__ float scratch[32];
    const float fdim = (float)dim;
    for (int64_t row = blockIdx.x; row < n_rows; row += gridDim.x)
    {
        T *xr = x + row * dim;
        T *rr = res + row * dim;
        float sq = 0.f;
        for (int64_t d = threadIdx.x; d < dim; d += blockDim.x)
        {
            float xv = to_f(xr[d]);
            if constexpr (ADD)
            {
                const T s = from_f<T>(__fadd_rn(xv, to_f(rr[d])));
                xr[d] = s;
                xv = to_f(s);
            }
            sq = fmaf(xv, xv, sq);
        }
        const float total = block_sum(sq, scratch);
        const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, fdim), kRmsEps)));
        for (int64_t d = threadIdx.x; d < dim; d += blockDim.x)
            rr[d] = from_f<T>(__fmul_rn(__fmul_rn(to_f(xr[d]), to_f(w[d])), inv_rms));
        __syncthreads();
    }
}

template <typename T, bool ADD>
int launch_rmsnorm(const void *w, void *x, void *res, int64_t n_rows, int64_t dim, cudaStream_t stream)
{
    constexpr int N = Vec16<T>::N;
    const int grid = (int)std::min<int64_t>(n_rows, (int64_t)num_sms() * 8);
    const bool vec = dim % N == 0 && is_aligned(w, 16) && is_aligned(x, 16) && is_aligned(res, 16);
    const int64_t chunks = dim / N;
    auto W = static_cast<const T *>(w);
    auto X = static_cast<T *>(x);
    auto R = static_cast<T *>(res);
    if (vec && chunks <= kThreads)
        rmsnorm_vec_kernel<T, 1, ADD><<<grid, kThreads, 0, stream>>>(W, X, R, n_rows, dim);
    else if (vec && chunks <= 2 * kThreads)
        rmsnorm_vec_kernel<T, 2, ADD><<<grid, kThreads, 0, stream>>>(W, X, R, n_rows, dim);
    else if (vec && chunks <= 4 * kThreads)
        rmsnorm_vec_kernel<T, 4, ADD><<<grid, kThreads, 0, stream>>>(W, X, R, n_rows, dim);
    else if (vec && chunks <= 8 * kThreads)
        rmsnorm_vec_kernel<T, 8, ADD><<<grid, kThreads, 0, stream>>>(W, X, R, n_rows, dim);
    else
        rmsnorm_generic_kernel<T, ADD><<<grid, kThreads, 0, stream>>>(W, X, R, n_rows, dim);
    return check_launch("l2k_fused_add_residual_rmsnorm");
}

} // namespace
} // namespace l2k

extern "C" int l2k_fused_add_residual_rmsnorm(const void *weights, void *x, void *residual, int64_t num_tokens,
                                              int64_t embed_dim, int add_residual, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(num_tokens >= 0 && embed_dim >= 0, "l2k_fused_add_residual_rmsnorm: negative size");
    L2K_REQUIRE(dtype_ok(dtype), "l2k_fused_add_residual_rmsnorm: unsupported dtype %d", dtype);
    if (num_tokens == 0 || embed_dim == 0)
        return L2K_OK;
    L2K_REQUIRE(weights && x && residual, "l2k_fused_add_residual_rmsnorm: null pointer");
    L2K_REQUIRE(x != residual, "l2k_fused_add_residual_rmsnorm: x and residual must be distinct buffers");
    L2K_DISPATCH(dtype, {
        return add_residual ? launch_rmsnorm<T, true>(weights, x, residual, num_tokens, embed_dim, stream)
                            : launch_rmsnorm<T, false>(weights, x, residual, num_tokens, embed_dim, stream);
    });
    return L2K_OK;
}
