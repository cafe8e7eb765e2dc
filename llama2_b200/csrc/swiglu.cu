// SwiGLU: out[t, i] = silu(g) * u, g = in[t, i], u = in[t, F + i].
//
// Pure streaming (read 2F, write F per row). gridDim.x tiles a row in
// 16-byte chunks, gridDim.y strides over rows; each thread handles one chunk
// of gate and one of up per row, loading four rows before computing them. silu(g) * u is evaluated as the reference
// oracle does, (g * (1 / (1 + exp(-g)))) * u (silu_mul: IEEE reciprocal and
// full-precision expf for fp32, the fast intrinsics for 16-bit data); rows
// whose size or alignment rules out 16-byte access take the scalar kernel.
//
// Reference: src/kernel/swiglu.cu:10-72 (one CTA per token, product in T).
#include "common.cuh"

#include <algorithm>

namespace l2k
{
namespace
{

// Rows per thread in flight: the loads of kRows rows are issued before any
// of them is computed, so a thread keeps 32 x kRows bytes in flight.
constexpr int kRows = 4;

template <typename T>
__global__ void __launch_bounds__(256) swiglu_vec_kernel(const T *__restrict__ in, T *__restrict__ out,
                                                         int64_t n_rows, int64_t inter)
{
    constexpr int N = Vec16<T>::N;
    const int64_t chunks = inter / N;
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= chunks)
        return;
    const int64_t stride = gridDim.y;
    for (int64_t row0 = blockIdx.y; row0 < n_rows; row0 += kRows * stride)
    {
        uint4 g[kRows], u[kRows];
#pragma unroll
        for (int r = 0; r < kRows; ++r)
        {
            const int64_t row = row0 + r * stride;
            if (row < n_rows)
            {
                const T *src = in + row * 2 * inter + c * N;
                g[r] = ldg_stream(src);
                u[r] = ldg_stream(src + inter);
            }
        }
#pragma unroll
        for (int r = 0; r < kRows; ++r)
        {
            const int64_t row = row0 + r * stride;
            if (row >= n_rows)
                break;
            const Vec16<T> gv = as_vec<T>(g[r]), uv = as_vec<T>(u[r]);
            Vec16<T> o;
#pragma unroll
            for (int e = 0; e < N; ++e)
                o.v[e] = from_f<T>(silu_mul<T>(to_f(gv.v[e]), to_f(uv.v[e])));
            stg(out + row * inter + c * N, as_u4(o));
        }
    }
}

template <typename T>
__global__ void __launch_bounds__(256) swiglu_scalar_kernel(const T *__restrict__ in, T *__restrict__ out,
                                                            int64_t n_rows, int64_t inter)
{
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= inter)
        return;
    for (int64_t row = blockIdx.y; row < n_rows; row += gridDim.y)
        out[row * inter + i] = from_f<T>(silu_mul<T>(to_f(in[row * 2 * inter + i]), to_f(in[row * 2 * inter + inter + i])));
}

template <typename T>
int launch_swiglu(const void *in, void *out, int64_t n_rows, int64_t inter, cudaStream_t stream)
{
    constexpr int N = Vec16<T>::N;
    const bool vec = inter % N == 0 && is_aligned(in, 16) && is_aligned(out, 16);
    const int64_t per_row = vec ? inter / N : inter;
    // The block size in [128, 256] (multiples of 32) that leaves the fewest
    // idle threads in a row's last CTA; shorter rows take one CTA.
    int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ceil_div(per_row, 32) * 32));
    if (per_row > 256)
        for (int b = 224; b >= 128; b -= 32)
            if (ceil_div(per_row, b) * b < ceil_div(per_row, block) * block)
                block = b;
    const int64_t gx = ceil_div(per_row, block);
    // Enough CTAs for ~16 per SM (each row span covered by gx of them); each
    // thread then walks rows in groups of kRows.
    const int64_t rows_per_cta = vec ? kRows : 1;
    const int64_t gy = std::max<int64_t>(
        1, std::min<int64_t>(ceil_div(n_rows, rows_per_cta),
                             std::min<int64_t>(65535, ceil_div((int64_t)num_sms() * 16, gx))));
    const dim3 grid((unsigned)gx, (unsigned)gy);
    if (vec)
        swiglu_vec_kernel<T><<<grid, block, 0, stream>>>(static_cast<const T *>(in), static_cast<T *>(out), n_rows, inter);
    else
        swiglu_scalar_kernel<T><<<grid, block, 0, stream>>>(static_cast<const T *>(in), static_cast<T *>(out), n_rows, inter);
    return check_launch("l2k_swiglu");
}

} // namespace
} // namespace l2k

extern "C" int l2k_swiglu(const void *input, void *output, int64_t num_tokens, int64_t intermediate_size, int dtype,
                          l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(num_tokens >= 0 && intermediate_size >= 0, "l2k_swiglu: negative size");
    L2K_REQUIRE(dtype_ok(dtype), "l2k_swiglu: unsupported dtype %d", dtype);
    if (num_tokens == 0 || intermediate_size == 0)
        return L2K_OK;
    L2K_REQUIRE(input && output, "l2k_swiglu: null pointer");
    L2K_REQUIRE_SHAPE(ceil_div(intermediate_size, 32) <= 65535LL * 256, "l2k_swiglu: intermediate_size too large");
    L2K_DISPATCH(dtype, { return launch_swiglu<T>(input, output, num_tokens, intermediate_size, stream); });
    return L2K_OK;
}
