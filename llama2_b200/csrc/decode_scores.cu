// Attention score rows: QK^T + 1/sqrt(hd) + causal/length mask + softmax in
// one pass over the K cache — the fused decode operator, and the prefill
// operator for shapes the tensor-core kernel does not take.
//
// A score row is (seq, q head, query row). Its keys are cut into 16 KB
// blocks of whole K rows (contiguous in the (B, Hkv, S, hd) cache) and spread
// over a thread-block cluster of C CTAs (block g -> rank g % C). Each CTA
// streams its blocks with cp.async.bulk (TMA) into a 4-stage shared-memory
// ring, computes the logits of its keys from shared memory, reduces its
// local max and sum of exponentials, exchanges them with its peers through
// distributed shared memory after one cluster barrier, and writes its
// normalized probabilities once. HBM traffic: the visible K rows, q, and
// the score row — no logits round trip, no mask tensor, no second kernel.
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

// ---------------------------------------------------------------------------
// Streaming kernel (head_dim * sizeof(T) in {64, 128, 256, 512} bytes).
// Keys are cut into 16 KB blocks of whole K rows (contiguous in the cache);
// global block g belongs to cluster rank g % C, so every CTA of the cluster
// has work whatever kv_len is. Per CTA, warp 4 is the producer: one lane
// issues cp.async.bulk copies of the CTA's blocks into a 4-stage shared
// ring (mbarrier full/empty pairs, bounded waits); warps 0..3 consume stage
// w: each lane holds a 16-byte slice of q, reads the matching slice of R K
// rows from shared memory per step and folds the R partial dot products with
// multi_reduce. Logits stay in shared memory for the cluster softmax.
// ---------------------------------------------------------------------------
constexpr int kNS = 4;                 // ring stages
constexpr int kCW = 8;                 // consumer warps (two per stage, one half-block each)
constexpr int kBlockBytes = 16384;     // one key block
constexpr int kStreamThreads = 32 * (kCW + 1);
constexpr long long kWaitCycles = 4000000000LL; // ~2 s

__device__ int g_scores_error = 0;     // first timeout code of this file's kernels

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity)
{
    const long long t0 = clock64();
    while (true)
    {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\t"
                     "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
                     "selp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done)
                     : "r"(bar), "r"(parity)
                     : "memory");
        if (done)
            return true;
        if (clock64() - t0 > kWaitCycles)
            return false;
    }
}

template <typename T, int LPR>
__global__ void __launch_bounds__(kStreamThreads) score_rows_stream_kernel(const DecodeArgs a)
{
    constexpr int N = Vec16<T>::N;
    constexpr int ROW_BYTES = LPR * 16;
    constexpr int KB = kBlockBytes / ROW_BYTES; // K rows per block
    constexpr int HALF = KB / 2;                // rows per consumer warp per block
    constexpr int R = LPR < 8 ? LPR : 8;
    constexpr int RPL = 32 / LPR;               // K rows per warp-wide read
    constexpr int ROWS = R * RPL;               // K rows per multi_reduce step
    static_assert(HALF % ROWS == 0, "half block must hold whole steps");
    extern __shared__ __align__(128) uint8_t stream_smem[];
    uint8_t *smem = stream_smem;
    float *logits = reinterpret_cast<float *>(smem + kNS * kBlockBytes);
    __shared__ __align__(8) uint64_t full[kNS], empty[kNS];
    __shared__ float2 stats[2];
    __shared__ float scratch[32];
    __shared__ int abort_flag;

    cg::cluster_group cluster = cg::this_cluster();
    const int C = (int)cluster.num_blocks();
    const int c = (int)cluster.block_rank();
    const int64_t row = blockIdx.x / C;
    const RowInfo ri = row_info(a, row);
    if (!ri.active)
        return; // the whole cluster shares the row and leaves together
    const int64_t kvh = ri.h / a.group;
    const int64_t n_keys = max((int64_t)0, ri.limit + 1);
    const int64_t n_blk = (n_keys + KB - 1) / KB;                 // blocks holding valid keys
    const int n_mine = n_blk > c ? (int)((n_blk - c + C - 1) / C) : 0;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    if (tid == 0)
    {
        for (int i = 0; i < kNS; ++i)
        {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&full[i])) : "memory");
            asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&empty[i])), "r"(kCW / kNS)
                         : "memory");
        }
        abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();

    const char *kbase = static_cast<const char *>(a.k) + (ri.b * a.Hkv + kvh) * a.S * (int64_t)ROW_BYTES;
    int n_issued = 0; // producer lane only
    if (warp == kCW)
    {
        if (lane == 0)
        {
            for (int i = 0; i < n_mine && !abort_flag; ++i)
            {
                const int st = i % kNS;
                if (i >= kNS && !bar_wait(smem_addr(&empty[st]), ((i / kNS) - 1) & 1))
                {
                    atomicCAS(&g_scores_error, 0, 0x201);
                    abort_flag = 1;
                    break;
                }
                // Whole blocks (up to the cache end): rows past kv_len are computed and masked,
                // which keeps the consumers' inner loop free of bounds checks.
                const int64_t g = c + (int64_t)C * i;
                const uint32_t bytes = (uint32_t)(min((int64_t)KB, a.S - g * KB) * ROW_BYTES);
                const uint32_t bar = smem_addr(&full[st]);
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
                asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                                 smem_addr(smem + st * kBlockBytes)),
                             "l"(kbase + g * KB * ROW_BYTES), "r"(bytes), "r"(bar)
                             : "memory");
                n_issued = i + 1;
            }
        }
    }
    else
    {
        const int st = warp % kNS, hf = warp / kNS; // ring stage, half of the block
        const int sub = lane % LPR;
        const T *qrow = static_cast<const T *>(a.q) + row * a.hd;
        const Vec16<T> qv = as_vec<T>(ldg_keep(qrow + sub * N));
        float qf[N];
#pragma unroll
        for (int e = 0; e < N; ++e)
            qf[e] = to_f(qv.v[e]);
        const uint8_t *stage = smem + st * kBlockBytes + (hf * HALF + lane / LPR) * ROW_BYTES + sub * 16;
        for (int i = st; i < n_mine; i += kNS)
        {
            if (!bar_wait(smem_addr(&full[st]), (i / kNS) & 1))
            {
                atomicCAS(&g_scores_error, 0, 0x202);
                abort_flag = 1;
                break;
            }
            const int64_t g = c + (int64_t)C * i;
            const int64_t valid = n_keys - g * KB - hf * HALF; // rows of this half below kv_len
#pragma unroll
            for (int base = 0; base < HALF; base += ROWS)
            {
                float part[R];
#pragma unroll
                for (int j = 0; j < R; ++j)
                {
                    const Vec16<T> kv =
                        as_vec<T>(*reinterpret_cast<const uint4 *>(stage + (base + j * RPL) * ROW_BYTES));
                    float sacc = 0.f;
#pragma unroll
                    for (int e = 0; e < N; ++e)
                        sacc = fmaf(to_f(kv.v[e]), qf[e], sacc);
                    part[j] = sacc;
                }
                int idx;
                const float dot = multi_reduce<R, LPR>(part, lane, idx);
                const int rr = base + idx * RPL + lane / LPR;
                if ((lane & (LPR / R - 1)) == 0)
                    logits[i * KB + hf * HALF + rr] = rr < valid ? __fmul_rn(dot, a.scale) : -INFINITY;
            }
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&empty[st])) : "memory");
        }
    }
    __syncthreads();
    if (abort_flag && warp == kCW && lane == 0)
    {
        // A wait expired: let this CTA's copies still in flight land before it
        // leaves (each wait bounded again).
        for (int i = max(0, n_issued - kNS); i < n_issued; ++i)
            bar_wait(smem_addr(&full[i % kNS]), (i / kNS) & 1);
    }

    // CTA statistics over its logits (one expf per logit, kept in place),
    // cluster-wide combination, normalized store.
    const int64_t n_log = (int64_t)n_mine * KB;
    float m = -INFINITY;
    for (int64_t i = tid; i < n_log; i += blockDim.x)
        m = fmaxf(m, logits[i]);
    m = block_max(m, scratch); // (its barriers also order the abort drain above)
    float l = 0.f;
    for (int64_t i = tid; i < n_log; i += blockDim.x)
    {
        const float x = logits[i];
        const float e = x == -INFINITY ? 0.f : expf(__fsub_rn(x, m));
        logits[i] = e;
        l += e;
    }
    l = block_sum(l, scratch);
    // p = e * exp(m - M) / (L + eps), M, L over the whole row
    float factor = 1.f, denom = __fadd_rn(l, kSoftmaxEps);
    if (C > 1)
    {
        if (tid == 0)
            stats[0] = make_float2(m, l);
        cluster.sync();
        if (tid < 32)
        {
            float2 sp = make_float2(-INFINITY, 0.f);
            if (tid < C)
                sp = *cluster.map_shared_rank(stats, tid);
            const float Mx = warp_max(sp.y > 0.f ? sp.x : -INFINITY);
            const float L = warp_sum(sp.y > 0.f ? sp.y * expf(__fsub_rn(sp.x, Mx)) : 0.f);
            if (tid == 0)
                stats[1] = make_float2(Mx, __fadd_rn(L, kSoftmaxEps));
        }
        __syncthreads();
        denom = stats[1].y;
        factor = l > 0.f ? expf(__fsub_rn(m, stats[1].x)) : 0.f;
    }
    const float scale_out = __fdiv_rn(factor, denom);
    T *out_row = static_cast<T *>(a.qk) + row * a.S;
    const int64_t n_wblk = (ri.M + KB - 1) / KB; // blocks with keys < M
    for (int64_t g = c; g < n_wblk; g += C)
    {
        const int64_t i = (g - c) / C;
        for (int r = tid; r < KB; r += blockDim.x)
        {
            const int64_t j = g * KB + r;
            if (j >= ri.M)
                break;
            const float p = (i < n_mine && j < n_keys) ? __fmul_rn(logits[i * KB + r], scale_out) : 0.f;
            out_row[j] = from_f<T>(p);
        }
    }
    if (C > 1)
        cluster.sync(); // peers may still be reading stats[0]
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

template <typename T>
int launch_score_rows(DecodeArgs a, int64_t batch, cudaStream_t stream)
{
    const int64_t rows = batch * a.Hq * a.Qc;
    const int64_t row_bytes = a.hd * (int64_t)sizeof(T);
    const bool vec = row_bytes % 16 == 0 && is_aligned(a.q, 16) && is_aligned(a.k, 16);
    const int lpr = (int)(row_bytes / 16);
    const bool stream_ok = vec && (lpr == 4 || lpr == 8 || lpr == 16 || lpr == 32);
    cudaError_t e;
    if (stream_ok)
    {
        // Cluster size: enough CTAs for ~3 per SM, at most one block per CTA-rank.
        const int64_t kb = kBlockBytes / row_bytes;
        const int64_t blocks_per_row = ceil_div(a.S, kb);
        int C = 1;
        while (C < 8 && rows * C < 3LL * num_sms() && C * 2 <= blocks_per_row)
            C *= 2;
        const int64_t logit_bytes = ceil_div(blocks_per_row, C) * kb * (int64_t)sizeof(float);
        L2K_REQUIRE_SHAPE(logit_bytes <= 128 * 1024, "score rows: kv_cache_len %lld too long", (long long)a.S);
        const size_t smem = (size_t)kNS * kBlockBytes + (size_t)logit_bytes;
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
