// Attention score rows: QK^T + 1/sqrt(hd) + causal/length mask + softmax in
// one pass over the K cache — the fused decode operator, and the prefill
// operator for shapes the tensor-core kernel does not take.
//
// Rows whose K rows are 64, 128, 256 or 512 bytes run the streaming kernel
// (score_stream.cuh: 16 KB key blocks streamed by cp.async.bulk into a
// shared-memory ring, cluster-wide softmax over distributed shared memory);
// other head sizes run a generic one-thread-per-key kernel.
//
// Reference composition: QK^T via cuBLAS batched GEMM (src/kernel/linear.cu:96-128)
// + masked softmax (src/kernel/compute_masked_attention_score.cu:12-103)
// with the mask "positions 0..pos".
#include "common.cuh"
#include "score_stream.cuh"

#include <algorithm>
#include <cmath>
#include <cooperative_groups.h>

namespace l2k
{
namespace
{

constexpr int kThreads = 256;
constexpr int kMaxChunk = 8192; // logits per CTA kept in shared memory (32 KB)

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

__device__ int g_scores_error = 0; // first timeout code of this file's kernels

template <typename T, int LPR>
__global__ void __launch_bounds__(kStreamThreads) score_rows_stream_kernel(const DecodeArgs a)
{
    extern __shared__ __align__(128) uint8_t stream_smem[];
    __shared__ StreamShared sh;
    cg::cluster_group cluster = cg::this_cluster();
    const StepRowArgs none{};
    score_row_stream<T, LPR, false>(a, none, (int64_t)blockIdx.x / cluster.num_blocks(), cluster, stream_smem, sh,
                                    &g_scores_error);
}

// Attention rows: the score row and its P.V output in one streamed pass
// over the row's K and V blocks (score_row_stream with PV).
// TC: the cache element type (T, or fp8 e4m3 with 16-bit T).
template <typename T, int LPR, typename TC = T>
__global__ void __launch_bounds__(kStreamThreads) attention_rows_stream_kernel(const DecodeArgs a)
{
    extern __shared__ __align__(128) uint8_t stream_smem[];
    __shared__ StreamShared sh;
    cg::cluster_group cluster = cg::this_cluster();
    const StepRowArgs none{};
    score_row_stream<T, LPR, false, true, TC>(a, none, (int64_t)blockIdx.x / cluster.num_blocks(), cluster,
                                              stream_smem, sh, &g_scores_error);
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
cudaError_t launch_clustered(K kernel, int C, int64_t rows, size_t smem, cudaStream_t stream, const DecodeArgs &a,
                             int threads)
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
    cfg.blockDim = dim3(threads);
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

// Whether score rows of this shape run the streaming kernel (K rows of 64,
// 128, 256 or 512 bytes, 16-byte aligned operands; with P.V also V and qkv).
template <typename T>
bool stream_rows_ok(const DecodeArgs &a, bool pv)
{
    const int64_t row_bytes = a.hd * (int64_t)sizeof(T);
    const int lpr = (int)(row_bytes / 16);
    const bool vec = row_bytes % 16 == 0 && is_aligned(a.q, 16) && is_aligned(a.k, 16) &&
                     (!pv || (is_aligned(a.v, 16) && is_aligned(a.qkv, 16)));
    return vec && (lpr == 4 || lpr == 8 || lpr == 16 || lpr == 32);
}

template <typename T, typename TC = T>
int launch_attention_rows(const DecodeArgs &a, int64_t batch, cudaStream_t stream)
{
    const int64_t rows = batch * a.Hq * a.Qc;
    const int64_t row_bytes = a.hd * (int64_t)sizeof(TC);
    const int lpr = (int)(row_bytes / 16);
    const int64_t kb = kBlockBytes / row_bytes;
    const int64_t blocks_per_row = ceil_div(a.S, kb);
    int C = 1;
    while (C < 8 && rows * C < 3LL * num_sms() && C * 2 <= blocks_per_row)
        C *= 2;
    const size_t smem = stream_smem_bytes(a.S, row_bytes, C) + pv_smem_bytes(a.hd);
    L2K_REQUIRE_SHAPE(smem <= (size_t)kNS * kBlockBytes + 128 * 1024, "attention rows: kv_cache_len %lld too long",
                      (long long)a.S);
    cudaError_t e;
    if (lpr == 32)
        e = launch_clustered(attention_rows_stream_kernel<T, 32, TC>, C, rows, smem, stream, a, kStreamThreads);
    else if (lpr == 16)
        e = launch_clustered(attention_rows_stream_kernel<T, 16, TC>, C, rows, smem, stream, a, kStreamThreads);
    else if (lpr == 8)
        e = launch_clustered(attention_rows_stream_kernel<T, 8, TC>, C, rows, smem, stream, a, kStreamThreads);
    else
        e = launch_clustered(attention_rows_stream_kernel<T, 4, TC>, C, rows, smem, stream, a, kStreamThreads);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "attention rows: %s", cudaGetErrorString(e));
    return check_launch("attention rows");
}

template <typename T>
int launch_score_rows(DecodeArgs a, int64_t batch, cudaStream_t stream)
{
    const int64_t rows = batch * a.Hq * a.Qc;
    const int64_t row_bytes = a.hd * (int64_t)sizeof(T);
    const int lpr = (int)(row_bytes / 16);
    const bool stream_ok = stream_rows_ok<T>(a, false);
    a.bulk_out = (a.S * (int64_t)sizeof(T)) % 16 == 0 && is_aligned(a.qk, 16);
    cudaError_t e;
    if (stream_ok)
    {
        // Cluster size: enough CTAs for ~3 per SM, at most one block per CTA-rank.
        const int64_t kb = kBlockBytes / row_bytes;
        const int64_t blocks_per_row = ceil_div(a.S, kb);
        int C = 1;
        while (C < 8 && rows * C < 3LL * num_sms() && C * 2 <= blocks_per_row)
            C *= 2;
        const size_t smem = stream_smem_bytes(a.S, row_bytes, C);
        L2K_REQUIRE_SHAPE(smem <= (size_t)kNS * kBlockBytes + 128 * 1024, "score rows: kv_cache_len %lld too long",
                          (long long)a.S);
        if (lpr == 32)
            e = launch_clustered(score_rows_stream_kernel<T, 32>, C, rows, smem, stream, a, kStreamThreads);
        else if (lpr == 16)
            e = launch_clustered(score_rows_stream_kernel<T, 16>, C, rows, smem, stream, a, kStreamThreads);
        else if (lpr == 8)
            e = launch_clustered(score_rows_stream_kernel<T, 8>, C, rows, smem, stream, a, kStreamThreads);
        else
            e = launch_clustered(score_rows_stream_kernel<T, 4>, C, rows, smem, stream, a, kStreamThreads);
    }
    else
    {
        int C = rows * 8 >= 2LL * num_sms() ? 8 : 16;
        C = (int)std::min<int64_t>(C, std::max<int64_t>(1, ceil_div(a.S, 64)));
        while (ceil_div(a.S, C) > kMaxChunk && C < 16)
            C *= 2;
        L2K_REQUIRE_SHAPE(ceil_div(a.S, C) <= kMaxChunk, "score rows: kv_cache_len %lld > %d", (long long)a.S,
                          16 * kMaxChunk);
        a.chunk = ceil_div(a.S, C);
        const size_t smem = (size_t)a.chunk * sizeof(float) + (size_t)a.hd * sizeof(float);
        e = launch_clustered(decode_scores_generic_kernel<T>, C, rows, smem, stream, a, kThreads);
    }
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "attention score rows: %s", cudaGetErrorString(e));
    return check_launch("attention score rows");
}

} // namespace

int read_scores_error(bool clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_scores_error, sizeof(int)) != cudaSuccess)
        return -1;
    if (clear && v)
    {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_scores_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

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

int attention_qkv_cuda_cores(const void *qk, const void *v, void *qkv, int64_t batch, int64_t Hq, int64_t Hkv,
                             int64_t qc, int64_t S, int64_t hd, int64_t m, int64_t n, const uint32_t *n_dev,
                             int dtype, cudaStream_t stream);

} // namespace l2k

extern "C" int l2k_decode_attention(const void *q, const void *k, const void *v, const uint32_t *kv_lens,
                                    const uint32_t *max_kv_len, void *qk, void *qkv, int64_t batch,
                                    int64_t q_head_num, int64_t kv_head_num, int64_t kv_cache_len, int64_t head_dim,
                                    int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_decode_attention: unsupported dtype %d", dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && kv_cache_len >= 0 && head_dim > 0,
                "l2k_decode_attention: bad size");
    if (batch == 0 || q_head_num == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_decode_attention: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(q && k && v && kv_lens && max_kv_len && qk && qkv, "l2k_decode_attention: null pointer");
    L2K_REQUIRE(kv_cache_len > 0, "l2k_decode_attention: kv_cache_len must be positive");
    L2K_REQUIRE_SHAPE(head_dim <= 4096, "l2k_decode_attention: head_dim > 4096");
    L2K_REQUIRE_SHAPE(batch * q_head_num * 16 < (int64_t(1) << 31), "l2k_decode_attention: grid too large");
    DecodeArgs a{q, k, nullptr, kv_lens, max_kv_len, 0u, qk, q_head_num, q_head_num / kv_head_num, kv_head_num, 1,
                 kv_cache_len, head_dim, 0, 1.f / sqrtf((float)head_dim)};
    a.v = v;
    a.qkv = qkv;
    bool streamed = false;
    L2K_DISPATCH(dtype, { streamed = stream_rows_ok<T>(a, true); });
    if (streamed)
    {
        L2K_DISPATCH(dtype, { return launch_attention_rows<T>(a, batch, stream); });
    }
    // Other head sizes / alignments: the score rows, then P.V over the keys
    // j < *max_kv_len on the CUDA cores (the reference's call-site order).
    int st = L2K_OK;
    L2K_DISPATCH(dtype, { st = launch_score_rows<T>(a, batch, stream); });
    if (st != L2K_OK)
        return st;
    return attention_qkv_cuda_cores(qk, v, qkv, batch, q_head_num, kv_head_num, 1, kv_cache_len, head_dim, 1,
                                    kv_cache_len, max_kv_len, dtype, stream);
}

extern "C" int64_t l2k_paged_block_rows(int64_t head_dim, int dtype)
{
    using namespace l2k;
    if (!(dtype_ok(dtype) || dtype == L2K_E4M3) || head_dim <= 0)
        return 0;
    const int64_t row_bytes = head_dim * (dtype == L2K_E4M3 ? int64_t(1) : (int64_t)dtype_size(dtype));
    const int64_t lpr = row_bytes / 16;
    if (row_bytes % 16 != 0 || !(lpr == 4 || lpr == 8 || lpr == 16 || lpr == 32))
        return 0;
    return kBlockBytes / row_bytes;
}

extern "C" int l2k_decode_attention_paged(const void *q, const void *k_pages, const void *v_pages,
                                          const uint32_t *block_table, int64_t max_pages, int64_t num_pages,
                                          const uint32_t *kv_lens, const uint32_t *max_kv_len, void *qk, void *qkv,
                                          int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
                                          int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_decode_attention_paged: unsupported dtype %d", dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim > 0 && max_pages >= 0 &&
                    num_pages >= 0,
                "l2k_decode_attention_paged: bad size");
    if (batch == 0 || q_head_num == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_decode_attention_paged: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(max_pages > 0 && num_pages > 0, "l2k_decode_attention_paged: empty block table or page pool");
    L2K_REQUIRE(q && k_pages && v_pages && block_table && kv_lens && max_kv_len && qk && qkv,
                "l2k_decode_attention_paged: null pointer");
    const int64_t page_rows = l2k_paged_block_rows(head_dim, dtype);
    L2K_REQUIRE_SHAPE(page_rows > 0, "l2k_decode_attention_paged: head_dim * element size must be 64, 128, 256 or "
                                     "512 bytes");
    L2K_REQUIRE_SHAPE(batch * q_head_num * 16 < (int64_t(1) << 31), "l2k_decode_attention_paged: grid too large");
    const int64_t S = max_pages * page_rows;
    DecodeArgs a{q, k_pages, nullptr, kv_lens, max_kv_len, 0u, qk, q_head_num, q_head_num / kv_head_num,
                 kv_head_num, 1, S, head_dim, 0, 1.f / sqrtf((float)head_dim)};
    a.v = v_pages;
    a.qkv = qkv;
    a.block_table = block_table;
    a.max_pages = max_pages;
    a.num_pages = num_pages;
    bool streamed = false;
    L2K_DISPATCH(dtype, { streamed = stream_rows_ok<T>(a, true); });
    L2K_REQUIRE_SHAPE(streamed, "l2k_decode_attention_paged: q, the pages, qkv must be 16-byte aligned");
    L2K_DISPATCH(dtype, { return launch_attention_rows<T>(a, batch, stream); });
    return L2K_OK;
}

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

// ---------------------------------------------------------------------------
// Decode attention over fp8 (e4m3) K/V caches: the streaming attention rows
// with each 16 KB block holding 16384 / head_dim rows; q, the probabilities
// and the output in `dtype` (16-bit); the logits are (q . k8) * (k_scale /
// sqrt(hd)) and the output v_scale * sum_j p_j v8_j, fp32 throughout.
// block_table == NULL: contiguous caches (B, Hkv, S, hd) of bytes; else pools
// (num_pages, Hkv, 16384 / hd, hd) with S = max_pages * 16384 / hd.
// ---------------------------------------------------------------------------
namespace l2k
{
namespace
{
int decode_attention_fp8(const char *name, const void *q, const void *k, const void *v, float k_scale, float v_scale,
                         const uint32_t *block_table, int64_t max_pages, int64_t num_pages, const uint32_t *kv_lens,
                         const uint32_t *max_kv_len, void *qk, void *qkv, int64_t batch, int64_t q_head_num,
                         int64_t kv_head_num, int64_t kv_cache_len, int64_t head_dim, int dtype, cudaStream_t stream)
{
    L2K_REQUIRE(dtype == L2K_BF16 || dtype == L2K_F16, "%s: q/qk/qkv must be bf16 or f16 (dtype %d)", name, dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && kv_cache_len >= 0 && head_dim > 0,
                "%s: bad size", name);
    L2K_REQUIRE(k_scale > 0.f && v_scale > 0.f && std::isfinite(k_scale) && std::isfinite(v_scale),
                "%s: the cache scales must be positive and finite", name);
    if (batch == 0 || q_head_num == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0, "%s: q_head_num must be a multiple of kv_head_num",
                name);
    L2K_REQUIRE(q && k && v && kv_lens && max_kv_len && qk && qkv, "%s: null pointer", name);
    L2K_REQUIRE(kv_cache_len > 0, "%s: kv_cache_len must be positive", name);
    L2K_REQUIRE_SHAPE(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512,
                      "%s: head_dim must be 64, 128, 256 or 512 (16-byte slices of 1-byte elements)", name);
    L2K_REQUIRE_SHAPE(is_aligned(q, 16) && is_aligned(k, 16) && is_aligned(v, 16) && is_aligned(qkv, 16),
                      "%s: q, the caches and qkv must be 16-byte aligned", name);
    L2K_REQUIRE_SHAPE(batch * q_head_num * 16 < (int64_t(1) << 31), "%s: grid too large", name);
    DecodeArgs a{q, k, nullptr, kv_lens, max_kv_len, 0u, qk, q_head_num, q_head_num / kv_head_num, kv_head_num, 1,
                 kv_cache_len, head_dim, 0, (1.f / sqrtf((float)head_dim)) * k_scale};
    a.v = v;
    a.qkv = qkv;
    a.v_scale = v_scale;
    a.block_table = block_table;
    a.max_pages = max_pages;
    a.num_pages = num_pages;
    if (dtype == L2K_BF16)
        return launch_attention_rows<__nv_bfloat16, __nv_fp8_e4m3>(a, batch, stream);
    return launch_attention_rows<__half, __nv_fp8_e4m3>(a, batch, stream);
}
} // namespace
} // namespace l2k

extern "C" int l2k_decode_attention_fp8(const void *q, const void *k_cache, const void *v_cache, float k_scale,
                                        float v_scale, const uint32_t *kv_lens, const uint32_t *max_kv_len, void *qk,
                                        void *qkv, int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                        int64_t kv_cache_len, int64_t head_dim, int dtype, l2k_stream_t stream)
{
    return l2k::decode_attention_fp8("l2k_decode_attention_fp8", q, k_cache, v_cache, k_scale, v_scale, nullptr, 0, 0,
                                     kv_lens, max_kv_len, qk, qkv, batch, q_head_num, kv_head_num, kv_cache_len,
                                     head_dim, dtype, stream);
}

extern "C" int l2k_decode_attention_fp8_paged(const void *q, const void *k_pages, const void *v_pages, float k_scale,
                                              float v_scale, const uint32_t *block_table, int64_t max_pages,
                                              int64_t num_pages, const uint32_t *kv_lens, const uint32_t *max_kv_len,
                                              void *qk, void *qkv, int64_t batch, int64_t q_head_num,
                                              int64_t kv_head_num, int64_t head_dim, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(max_pages > 0 && num_pages > 0 && block_table, "l2k_decode_attention_fp8_paged: empty block table "
                                                               "or page pool");
    L2K_REQUIRE_SHAPE(head_dim > 0 && 16384 % head_dim == 0, "l2k_decode_attention_fp8_paged: bad head_dim");
    return l2k::decode_attention_fp8("l2k_decode_attention_fp8_paged", q, k_pages, v_pages, k_scale, v_scale,
                                     block_table, max_pages, num_pages, kv_lens, max_kv_len, qk, qkv, batch,
                                     q_head_num, kv_head_num, max_pages * (16384 / head_dim), head_dim, dtype, stream);
}
