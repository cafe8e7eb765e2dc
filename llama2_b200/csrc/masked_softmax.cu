// Scale + mask + softmax over attention-score rows, in place.
//
// One CTA per (seq, head, q) row with q < q_lens[seq]; keys k < max_kv.
// The row is read from HBM once into registers (NV 16-byte chunks per
// thread), the max and the sum of exponentials are block reductions, and the
// row is written once: 1 read + 1 write of qk (the reference makes three
// passes over qk and the mask on a grid capped at 256 x 2 x 2 CTAs:
// src/kernel/compute_masked_attention_score.cu:12-140).
//
// Mask sources:
//   MASK_TENSOR — a u8 mask (B, q_cache_len, kv_cache_len), nonzero = keep;
//                 the drop-in for launch_compute_masked_attention_score;
//   MASK_CAUSAL — keep k < kv_len && k <= kv_len - q_len + q, computed from
//                 the lengths (the unfused prefill score path).
// Entries with q >= q_len or k >= max_kv are never written. Masked entries
// become 0; a row with nothing kept becomes all 0.
// Per element: x = qk * scale (scale = 1/sqrtf(head_dim) computed on the
// host as the oracle does), p = expf(x - m) / (sum + 1e-6) with IEEE
// division, as the reference oracle evaluates it.
#include "common.cuh"

#include <algorithm>
#include <cmath>

namespace l2k
{
namespace
{

constexpr float kSoftmaxEps = 1e-6f;

enum MaskMode
{
    MASK_TENSOR = 0,
    MASK_CAUSAL = 1
};

struct SoftmaxArgs
{
    void *qk;
    const uint8_t *mask;
    const uint32_t *q_lens;
    const uint32_t *kv_lens; // MASK_CAUSAL only
    int64_t H;
    int64_t qc;
    int64_t S;
    int64_t max_kv;
    float scale;
};

template <int MODE>
__device__ __forceinline__ bool keep(const SoftmaxArgs &a, const uint8_t *mrow, int64_t k, int64_t causal_limit)
{
    if constexpr (MODE == MASK_TENSOR)
        return mrow[k] != 0;
    else
        return k <= causal_limit;
}

// Register-cached path: row fits in NV chunks of N elements per thread.
template <typename T, int MODE, int NV>
__global__ void __launch_bounds__(256) softmax_rows_vec(const SoftmaxArgs a)
{
    constexpr int N = Vec16<T>::N;
    __shared__ float scratch[32];
    const int64_t q = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const uint32_t q_len = a.q_lens[b];
    if (q >= q_len)
        return;
    T *row = static_cast<T *>(a.qk) + ((b * a.H + h) * a.qc + q) * a.S;
    const uint8_t *mrow = MODE == MASK_TENSOR ? a.mask + (b * a.qc + q) * a.S : nullptr;
    int64_t limit = -1; // last kept key for MASK_CAUSAL
    if constexpr (MODE == MASK_CAUSAL)
    {
        const int64_t kv_len = a.kv_lens[b];
        limit = min(kv_len - 1, kv_len - (int64_t)q_len + q);
    }
    const int64_t L = a.max_kv;
    float x[NV][N];
    bool kp[NV][N];
    float m = -INFINITY;
#pragma unroll
    for (int j = 0; j < NV; ++j)
    {
        const int64_t k0 = ((int64_t)threadIdx.x + (int64_t)j * blockDim.x) * N;
        if (k0 + N <= L)
        {
            const Vec16<T> v = as_vec<T>(ldg_coherent(row + k0));
#pragma unroll
            for (int e = 0; e < N; ++e)
            {
                x[j][e] = __fmul_rn(to_f(v.v[e]), a.scale);
                kp[j][e] = keep<MODE>(a, mrow, k0 + e, limit);
            }
        }
        else
        {
#pragma unroll
            for (int e = 0; e < N; ++e)
            {
                const bool in = k0 + e < L;
                x[j][e] = in ? __fmul_rn(to_f(row[k0 + e]), a.scale) : 0.f;
                kp[j][e] = in && keep<MODE>(a, mrow, k0 + e, limit);
            }
        }
#pragma unroll
        for (int e = 0; e < N; ++e)
            if (kp[j][e])
                m = fmaxf(m, x[j][e]);
    }
    m = block_max(m, scratch);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
#pragma unroll
        for (int e = 0; e < N; ++e)
        {
            x[j][e] = kp[j][e] ? expf(__fsub_rn(x[j][e], m)) : 0.f;
            sum += x[j][e];
        }
    sum = block_sum(sum, scratch);
    const float denom = __fadd_rn(sum, kSoftmaxEps);
#pragma unroll
    for (int j = 0; j < NV; ++j)
    {
        const int64_t k0 = ((int64_t)threadIdx.x + (int64_t)j * blockDim.x) * N;
        Vec16<T> o;
#pragma unroll
        for (int e = 0; e < N; ++e)
            o.v[e] = from_f<T>(kp[j][e] ? __fdiv_rn(x[j][e], denom) : 0.f);
        if (k0 + N <= L)
            stg(row + k0, as_u4(o));
        else
            for (int e = 0; e < N && k0 + e < L; ++e)
                row[k0 + e] = o.v[e];
    }
}

// Any length / alignment: three passes over the row (re-reads hit L2).
template <typename T, int MODE>
__global__ void __launch_bounds__(256) softmax_rows_generic(const SoftmaxArgs a)
{
    __shared__ float scratch[32];
    const int64_t q = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const uint32_t q_len = a.q_lens[b];
    if (q >= q_len)
        return;
    T *row = static_cast<T *>(a.qk) + ((b * a.H + h) * a.qc + q) * a.S;
    const uint8_t *mrow = MODE == MASK_TENSOR ? a.mask + (b * a.qc + q) * a.S : nullptr;
    int64_t limit = -1;
    if constexpr (MODE == MASK_CAUSAL)
    {
        const int64_t kv_len = a.kv_lens[b];
        limit = min(kv_len - 1, kv_len - (int64_t)q_len + q);
    }
    float m = -INFINITY;
    for (int64_t k = threadIdx.x; k < a.max_kv; k += blockDim.x)
        if (keep<MODE>(a, mrow, k, limit))
            m = fmaxf(m, __fmul_rn(to_f(row[k]), a.scale));
    m = block_max(m, scratch);
    float sum = 0.f;
    for (int64_t k = threadIdx.x; k < a.max_kv; k += blockDim.x)
        if (keep<MODE>(a, mrow, k, limit))
            sum += expf(__fsub_rn(__fmul_rn(to_f(row[k]), a.scale), m));
    sum = block_sum(sum, scratch);
    const float denom = __fadd_rn(sum, kSoftmaxEps);
    for (int64_t k = threadIdx.x; k < a.max_kv; k += blockDim.x)
    {
        const bool kp = keep<MODE>(a, mrow, k, limit);
        row[k] = from_f<T>(kp ? __fdiv_rn(expf(__fsub_rn(__fmul_rn(to_f(row[k]), a.scale), m)), denom) : 0.f);
    }
}

template <typename T, int MODE>
int launch_softmax(const SoftmaxArgs &a, int64_t batch, int64_t max_q, cudaStream_t stream)
{
    constexpr int N = Vec16<T>::N;
    const dim3 grid((unsigned)max_q, (unsigned)a.H, (unsigned)batch);
    const bool vec = (a.S * (int64_t)sizeof(T)) % 16 == 0 && is_aligned(a.qk, 16);
    const int64_t chunks = ceil_div(a.max_kv, N);
    int block = 256;
    if (chunks <= 128)
        block = (int)std::max<int64_t>(32, ceil_div(chunks, 32) * 32);
    if (vec && chunks <= block)
        softmax_rows_vec<T, MODE, 1><<<grid, block, 0, stream>>>(a);
    else if (vec && chunks <= 2 * block)
        softmax_rows_vec<T, MODE, 2><<<grid, block, 0, stream>>>(a);
    else if (vec && chunks <= 4 * block)
        softmax_rows_vec<T, MODE, 4><<<grid, block, 0, stream>>>(a);
    else if (vec && chunks <= 8 * block)
        softmax_rows_vec<T, MODE, 8><<<grid, block, 0, stream>>>(a);
    else
        softmax_rows_generic<T, MODE><<<grid, block, 0, stream>>>(a);
    return check_launch("l2k masked softmax");
}

} // namespace

// Also used by the unfused prefill score path (scores.cu).
int masked_softmax_causal(void *qk, const uint32_t *q_lens, const uint32_t *kv_lens, int64_t batch, int64_t H,
                          int64_t qc, int64_t S, int64_t max_q, int64_t max_kv, int64_t head_dim, int dtype,
                          cudaStream_t stream)
{
    const SoftmaxArgs a{qk, nullptr, q_lens, kv_lens, H, qc, S, max_kv, 1.f / sqrtf((float)head_dim)};
    L2K_DISPATCH(dtype, { return launch_softmax<T, MASK_CAUSAL>(a, batch, max_q, stream); });
    return L2K_OK;
}

} // namespace l2k

extern "C" int l2k_compute_masked_attention_score(int64_t head_dim, uint32_t max_q_len, uint32_t max_kv_len,
                                                  const uint32_t *q_lens, const uint8_t *mask, void *qk,
                                                  int64_t batch, int64_t q_head_num, int64_t q_cache_len,
                                                  int64_t kv_cache_len, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_compute_masked_attention_score: unsupported dtype %d", dtype);
    L2K_REQUIRE(head_dim > 0 && batch >= 0 && q_head_num >= 0 && q_cache_len >= 0 && kv_cache_len >= 0,
                "l2k_compute_masked_attention_score: bad size");
    L2K_REQUIRE(max_q_len <= q_cache_len && max_kv_len <= kv_cache_len,
                "l2k_compute_masked_attention_score: max_q_len/max_kv_len exceed the cache dims");
    if (batch == 0 || q_head_num == 0 || max_q_len == 0 || max_kv_len == 0)
        return L2K_OK;
    L2K_REQUIRE(q_lens && mask && qk, "l2k_compute_masked_attention_score: null pointer");
    L2K_REQUIRE_SHAPE(batch <= 65535 && q_head_num <= 65535, "l2k_compute_masked_attention_score: grid too large");
    // The reference's kernel walks q < q_lens[b] (not max_q_len); so does this one,
    // but rows beyond max_q_len are outside the grid, as in the reference launch.
    const SoftmaxArgs a{qk, mask, q_lens, nullptr, q_head_num, q_cache_len, kv_cache_len, (int64_t)max_kv_len,
                        1.f / sqrtf((float)head_dim)};
    L2K_DISPATCH(dtype, { return launch_softmax<T, MASK_TENSOR>(a, batch, max_q_len, stream); });
    return L2K_OK;
}
