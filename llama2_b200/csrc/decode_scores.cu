// Fused decode attention scores: QK^T + 1/sqrt(hd) + length mask + softmax
// in one pass over the K cache.
//
// Layout: one (seq, q head) score row is split over a thread-block cluster
// of C CTAs; CTA c owns keys [c*chunk, (c+1)*chunk). Each CTA
//   1. streams its K rows (contiguous in the (B, Hkv, S, hd) cache) with
//      16-byte read-once loads: a K row spans LPR = hd*sizeof(T)/16 lanes,
//      a warp issues R row-loads per iteration (4 KB in flight per warp) and
//      folds the R partial dot products with a transpose-reduce
//      (R - 1 + log2(LPR/R) shuffles for R rows instead of R*log2(LPR));
//   2. keeps the scaled logits of its keys in shared memory and reduces its
//      local max m_c and sum l_c = sum exp(s - m_c);
//   3. reads every peer's (m_c, l_c) through distributed shared memory after
//      one cluster barrier, forms the row max and denominator, and writes its
//      normalized probabilities once.
// HBM traffic is the K rows 0..kv_len-1, q, and the score row: no logits
// round trip, no mask tensor, no second kernel.
//
// Reference composition: QK^T via cuBLAS batched GEMM (src/kernel/linear.cu:96-128)
// + masked softmax (src/kernel/compute_masked_attention_score.cu:12-103)
// with the mask "positions 0..pos".
#include "common.cuh"

#include <algorithm>
#include <cmath>
#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace l2k
{
namespace
{

constexpr int kThreads = 256;
constexpr int kMaxChunk = 8192; // logits per CTA kept in shared memory (32 KB)
constexpr float kSoftmaxEps = 1e-6f;

// A score row is (seq b, q head h, query row i). Decode: Qc = 1, q_lens = NULL
// (one query per sequence at position kv_len - 1). Prefill: row i of a
// sequence with q_len new tokens sees keys j <= kv_len - q_len + i.
struct DecodeArgs
{
    const void *q;        // (B, Hq, Qc, hd)
    const void *k;        // (B, Hkv, S, hd)
    const uint32_t *q_lens; // NULL for decode
    const uint32_t *kv_lens;
    const uint32_t *max_kv; // device pointer, or NULL to use max_kv_host
    uint32_t max_kv_host;
    void *qk;             // (B, Hq, Qc, S)
    int64_t Hq;
    int64_t group; // Hq / Hkv
    int64_t Hkv;
    int64_t Qc;
    int64_t S;
    int64_t hd;
    int64_t chunk;
    float scale;
};

struct RowInfo
{
    int64_t b, h, i;
    int64_t limit; // last key kept (-1: none); the row is skipped when i >= q_len
    int64_t M;     // keys written: [0, M)
    bool active;
};

__device__ __forceinline__ RowInfo row_info(const DecodeArgs &a, int64_t row)
{
    RowInfo r;
    const int64_t bh = row / a.Qc;
    r.i = row - bh * a.Qc;
    r.b = bh / a.Hq;
    r.h = bh - r.b * a.Hq;
    const int64_t kv_len = min((int64_t)a.kv_lens[r.b], a.S);
    const int64_t q_len = a.q_lens ? (int64_t)a.q_lens[r.b] : 1;
    r.active = r.i < q_len;
    r.limit = min(kv_len - 1, kv_len - q_len + r.i);
    r.M = min((int64_t)(a.max_kv ? *a.max_kv : a.max_kv_host), a.S);
    return r;
}

// R partial sums per lane, each a sum over LPR consecutive lanes, reduced so
// that lane l ends with the full sum of value `idx`. R <= LPR, powers of 2.
template <int R, int LPR>
__device__ __forceinline__ float multi_reduce(float (&v)[R], int lane, int &idx)
{
    idx = 0;
#pragma unroll
    for (int n = R, off = LPR / 2; n > 1; n >>= 1, off >>= 1)
    {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; ++i)
        {
            const float send = upper ? v[i] : v[i + n / 2];
            const float keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
        if (upper)
            idx += n / 2;
    }
    float s = v[0];
#pragma unroll
    for (int off = LPR / (2 * R); off > 0; off >>= 1)
        s += __shfl_xor_sync(0xffffffffu, s, off);
    return s;
}

// Cluster-wide softmax over the logits in shared memory; writes the row.
template <typename T>
__device__ __forceinline__ void finish_row(cg::cluster_group &cluster, const float *logits, float2 *stats,
                                           float *scratch, int64_t j0, int64_t n_valid, int64_t n_write,
                                           T *out_row)
{
    float m = -INFINITY;
    for (int64_t i = threadIdx.x; i < n_valid; i += blockDim.x)
        m = fmaxf(m, logits[i]);
    m = block_max(m, scratch);
    float l = 0.f;
    for (int64_t i = threadIdx.x; i < n_valid; i += blockDim.x)
        l += expf(__fsub_rn(logits[i], m));
    l = block_sum(l, scratch);
    if (threadIdx.x == 0)
        stats[0] = make_float2(m, l);
    cluster.sync();
    // Warp 0 reads the C <= 32 peers' (m, l) over DSMEM, one peer per lane,
    // and publishes the row max and denominator through shared memory.
    if (threadIdx.x < 32)
    {
        const int C = (int)cluster.num_blocks();
        float2 sp = make_float2(-INFINITY, 0.f);
        if ((int)threadIdx.x < C)
            sp = *cluster.map_shared_rank(stats, (int)threadIdx.x);
        const float M = warp_max(sp.y > 0.f ? sp.x : -INFINITY);
        const float L = warp_sum(sp.y > 0.f ? sp.y * expf(__fsub_rn(sp.x, M)) : 0.f);
        if (threadIdx.x == 0)
            stats[1] = make_float2(M, __fadd_rn(L, kSoftmaxEps));
    }
    __syncthreads();
    const float M = stats[1].x;
    const float denom = stats[1].y;
    for (int64_t i = threadIdx.x; i < n_write; i += blockDim.x)
        out_row[j0 + i] = from_f<T>(i < n_valid ? __fdiv_rn(expf(__fsub_rn(logits[i], M)), denom) : 0.f);
    cluster.sync(); // peers may still be reading stats[0]
}

template <typename T, int LPR>
__global__ void __launch_bounds__(kThreads) decode_scores_kernel(const DecodeArgs a)
{
    constexpr int N = Vec16<T>::N;
    constexpr int R = LPR < 8 ? LPR : 8;
    constexpr int RPL = 32 / LPR; // K rows per warp-wide load
    constexpr int ROWS = R * RPL; // K rows per warp iteration
    extern __shared__ float logits[];
    __shared__ float2 stats[2];
    __shared__ float scratch[32];

    cg::cluster_group cluster = cg::this_cluster();
    const int C = (int)cluster.num_blocks();
    const int64_t c = cluster.block_rank();
    const int64_t row = blockIdx.x / C;
    const RowInfo ri = row_info(a, row);
    if (!ri.active)
        return; // the whole cluster shares the row and leaves together
    const int64_t kvh = ri.h / a.group;
    const int64_t S = a.S;
    const int64_t j0 = c * a.chunk;
    const int64_t n_valid = max((int64_t)0, min(j0 + a.chunk, ri.limit + 1) - j0);
    const int64_t n_write = max((int64_t)0, min(j0 + a.chunk, ri.M) - j0);

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
    if (n_valid > 0)
    {
        const int sub = lane % LPR; // 16-byte slice of the row this lane reads
        const T *qrow = static_cast<const T *>(a.q) + row * a.hd;
        const Vec16<T> qv = as_vec<T>(ldg_keep(qrow + sub * N));
        float qf[N];
#pragma unroll
        for (int e = 0; e < N; ++e)
            qf[e] = to_f(qv.v[e]);
        const T *kbase = static_cast<const T *>(a.k) + ((ri.b * a.Hkv + kvh) * S + j0) * a.hd + sub * N;
        for (int64_t base = (int64_t)warp * ROWS; base < n_valid; base += (int64_t)nwarps * ROWS)
        {
            float part[R];
            uint4 raw[R];
#pragma unroll
            for (int i = 0; i < R; ++i)
            {
                const int64_t r = base + i * RPL + lane / LPR;
                if (r < n_valid)
                    raw[i] = ldg_stream(kbase + r * a.hd);
                else
                    raw[i] = make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int i = 0; i < R; ++i)
            {
                const Vec16<T> kv = as_vec<T>(raw[i]);
                float s = 0.f;
#pragma unroll
                for (int e = 0; e < N; ++e)
                    s = fmaf(to_f(kv.v[e]), qf[e], s);
                part[i] = s;
            }
            int idx;
            const float dot = multi_reduce<R, LPR>(part, lane, idx);
            const int64_t r = base + idx * RPL + lane / LPR;
            if ((lane & (LPR / R - 1)) == 0 && r < n_valid)
                logits[r] = __fmul_rn(dot, a.scale);
        }
    }
    __syncthreads();
    T *out_row = static_cast<T *>(a.qk) + row * S;
    finish_row<T>(cluster, logits, stats, scratch, j0, n_valid, n_write, out_row);
}

// Any head_dim / alignment: one thread per key, q staged in shared memory.
template <typename T>
__global__ void __launch_bounds__(kThreads) decode_scores_generic_kernel(const DecodeArgs a)
{
    extern __shared__ float smem[];
    float *qs = smem;            // hd floats
    float *logits = smem + a.hd; // chunk floats
    __shared__ float2 stats[2];
    __shared__ float scratch[32];
    cg::cluster_group cluster = cg::this_cluster();
    const int C = (int)cluster.num_blocks();
    const int64_t c = cluster.block_rank();
    const int64_t row = blockIdx.x / C;
    const RowInfo ri = row_info(a, row);
    if (!ri.active)
        return;
    const int64_t kvh = ri.h / a.group;
    const int64_t S = a.S;
    const int64_t j0 = c * a.chunk;
    const int64_t n_valid = max((int64_t)0, min(j0 + a.chunk, ri.limit + 1) - j0);
    const int64_t n_write = max((int64_t)0, min(j0 + a.chunk, ri.M) - j0);
    const T *qrow = static_cast<const T *>(a.q) + row * a.hd;
    for (int64_t d = threadIdx.x; d < a.hd; d += blockDim.x)
        qs[d] = to_f(qrow[d]);
    __syncthreads();
    const T *kbase = static_cast<const T *>(a.k) + ((ri.b * a.Hkv + kvh) * S + j0) * a.hd;
    for (int64_t r = threadIdx.x; r < n_valid; r += blockDim.x)
    {
        const T *kr = kbase + r * a.hd;
        float s = 0.f;
        for (int64_t d = 0; d < a.hd; ++d)
            s = fmaf(to_f(kr[d]), qs[d], s);
        logits[r] = __fmul_rn(s, a.scale);
    }
    __syncthreads();
    T *out_row = static_cast<T *>(a.qk) + row * S;
    finish_row<T>(cluster, logits, stats, scratch, j0, n_valid, n_write, out_row);
}

template <typename K>
cudaError_t launch_clustered(K kernel, int C, int64_t rows, size_t smem, cudaStream_t stream, const DecodeArgs &a)
{
    if (smem > 48 * 1024)
    {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess)
            return e;
    }
    if (C > 8)
    {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess)
            return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(rows * C));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, a);
}

template <typename T>
int launch_score_rows(DecodeArgs a, int64_t batch, cudaStream_t stream)
{
    const int64_t rows = batch * a.Hq * a.Qc;
    // Cluster size: enough CTAs for two waves over the SMs, chunks <= kMaxChunk.
    int C = rows * 8 >= 2LL * num_sms() ? 8 : 16;
    C = (int)std::min<int64_t>(C, std::max<int64_t>(1, ceil_div(a.S, 64)));
    while (ceil_div(a.S, C) > kMaxChunk && C < 16)
        C *= 2;
    L2K_REQUIRE_SHAPE(ceil_div(a.S, C) <= kMaxChunk, "l2k_decode_attention_scores: kv_cache_len %lld > %d",
                      (long long)a.S, 16 * kMaxChunk);
    a.chunk = ceil_div(a.S, C);
    const int64_t row_bytes = a.hd * (int64_t)sizeof(T);
    const bool vec = row_bytes % 16 == 0 && is_aligned(a.q, 16) && is_aligned(a.k, 16);
    const int lpr = (int)(row_bytes / 16);
    cudaError_t e;
    const size_t smem = (size_t)a.chunk * sizeof(float);
    if (vec && lpr == 32)
        e = launch_clustered(decode_scores_kernel<T, 32>, C, rows, smem, stream, a);
    else if (vec && lpr == 16)
        e = launch_clustered(decode_scores_kernel<T, 16>, C, rows, smem, stream, a);
    else if (vec && lpr == 8)
        e = launch_clustered(decode_scores_kernel<T, 8>, C, rows, smem, stream, a);
    else if (vec && lpr == 4)
        e = launch_clustered(decode_scores_kernel<T, 4>, C, rows, smem, stream, a);
    else
        e = launch_clustered(decode_scores_generic_kernel<T>, C, rows, smem + (size_t)a.hd * sizeof(float), stream,
                             a);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_decode_attention_scores: %s", cudaGetErrorString(e));
    return check_launch("l2k_decode_attention_scores");
}

} // namespace

// Prefill score rows through the same cluster kernel (one cluster per query
// row): logits stay fp32 until the final store. Used by scores.cu for the
// shapes the tensor-core kernel does not take.
int prefill_score_rows(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens,
                       uint32_t max_kv, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc, int64_t S,
                       int64_t hd, int dtype, cudaStream_t stream)
{
    L2K_REQUIRE_SHAPE(batch * Hq * Qc * 16 < (int64_t(1) << 31), "prefill score rows: grid too large");
    DecodeArgs a{q, k, q_lens, kv_lens, nullptr, max_kv, qk, Hq, Hq / Hkv, Hkv, Qc, S, hd, 0,
                 1.f / sqrtf((float)hd)};
    L2K_DISPATCH(dtype, { return launch_score_rows<T>(a, batch, stream); });
    return L2K_OK;
}

} // namespace l2k

extern "C" int l2k_decode_attention_scores(const void *q, const void *k, const uint32_t *kv_lens,
                                           const uint32_t *max_kv_len, void *qk, int64_t batch, int64_t q_head_num,
                                           int64_t kv_head_num, int64_t kv_cache_len, int64_t head_dim, int dtype,
                                           l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_decode_attention_scores: unsupported dtype %d", dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && kv_cache_len >= 0 && head_dim > 0,
                "l2k_decode_attention_scores: bad size");
    if (batch == 0 || q_head_num == 0 || kv_cache_len == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_decode_attention_scores: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(q && k && kv_lens && max_kv_len && qk, "l2k_decode_attention_scores: null pointer");
    L2K_REQUIRE_SHAPE(head_dim <= 4096, "l2k_decode_attention_scores: head_dim > 4096");
    L2K_REQUIRE_SHAPE(batch * q_head_num * 16 < (int64_t(1) << 31), "l2k_decode_attention_scores: grid too large");
    DecodeArgs a{q, k, nullptr, kv_lens, max_kv_len, 0u, qk, q_head_num, q_head_num / kv_head_num, kv_head_num, 1,
                 kv_cache_len, head_dim, 0, 1.f / sqrtf((float)head_dim)};
    L2K_DISPATCH(dtype, { return launch_score_rows<T>(a, batch, stream); });
    return L2K_OK;
}
