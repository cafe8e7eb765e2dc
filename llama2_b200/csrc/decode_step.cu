// One decode step of the layer-kernel chain in ONE launch:
//
//   kv_lens += q_lens, max_lens = (max q_len, max kv_len)      (update_q_kv_lens)
//   x = embed_table[ids], normed = RMSNorm(x)                   (embedding, RMSNorm)
//   q, k_cache[pos], v_cache[pos] = RoPE(qkv), pos = kv_len - 1 (fused RoPE + KV append)
//   qk = softmax(q K^T / sqrt(hd), keys 0..pos)                 (QK^T + masked softmax)
//   ffn_out = silu(gate) * up                                   (SwiGLU)
//   [attn_out = qk V over keys 0..pos                           (l2k_decode_step_attention)]
//
// with exactly the results of those operators run one after another
// (l2k_update_q_kv_lens, l2k_embedding, l2k_fused_add_residual_rmsnorm
// without add, l2k_fused_reshape_rope_kvcache[_llama2]_decode,
// l2k_decode_attention_scores — l2k_decode_attention with the attention
// output — , l2k_swiglu).
//
// At small batch every one of those kernels is latency-bound (a 7B batch-1
// step moves ~9-35 MB, a few microseconds of HBM time, while each launch and
// its dependent loads cost about as much), so the step is one grid of three
// CTA roles that run concurrently:
//   * score rows, one thread-block cluster per (seq, q head) — the streaming
//     kernel of score_stream.cuh with the RoPE of q and of the new K row done
//     in place (the rotated K row replaces the stale cache row in shared
//     memory; the owning CTA appends K and V to the cache);
//   * embedding + RMSNorm, one CTA per token (the row is read once from the
//     table, written to x, reduced, normalized);
//   * SwiGLU over contiguous ranges of 16-byte vectors.
// The length update is done by the CTA that takes the last ticket: every
// CTA takes one ticket from a counter in caller-provided workspace after its
// last read of the old lengths; the holder of the last ticket writes kv_lens
// and the maxima and returns the counter to zero. Nothing waits on the
// counter.
//
// Reference: the operators above — src/kernel/update_q_kv_lens.cu:9-61,
// src/kernel/embedding.cu:10-49, src/kernel/fused_add_residual_rmsnorm.cu:11-126,
// src/kernel/fused_reshape_rope_kvcache_decode.cu:11-125,
// src/kernel/fused_reshape_rope_kvcache_llama2_decode.cu:11-114,
// src/kernel/linear.cu:96-128 + src/kernel/compute_masked_attention_score.cu:12-103,
// src/kernel/swiglu.cu:10-72. The reference has no fused step.
#include "common.cuh"
#include "score_stream.cuh"

#include <algorithm>
#include <cmath>
#include <mutex>

namespace l2k
{
namespace
{

constexpr float kRmsEps = 1e-5f;
constexpr int kSwigluVecsPerThread = 4;

__device__ int g_step_error = 0; // first timeout code of the step kernel

struct StepArgs
{
    DecodeArgs d;   // score rows (q = the q buffer, k = the K cache, qk)
    StepRowArgs r;  // RoPE inputs and cache outputs of the score rows
    // embedding + RMSNorm
    const uint32_t *ids;
    const void *embed;
    const void *norm_w;
    void *x;
    void *normed;
    int64_t vocab;
    int64_t dim;
    // SwiGLU
    const void *gate_up;
    void *ffn_out;
    int64_t hidden;
    // CTA roles: [0, score_ctas) score rows, then norm_ctas, then sw_ctas
    int64_t score_ctas;
    int64_t norm_ctas;
    int64_t sw_ctas;
    int64_t sw_per_cta; // 16-byte vectors of SwiGLU output per CTA
};

// x[t] = table[ids[t]] (zero row for ids >= vocab), normed[t] = x w / rms(x).
// Same arithmetic as rmsnorm.cu: fp32 sum of squares of the stored x,
// inv_rms = 1 / sqrt(sum / D + eps) with IEEE division and square root,
// normed = (x * w) * inv_rms.
template <typename T>
__device__ __forceinline__ void embed_norm_row(const StepArgs &a, int64_t t, float *scratch)
{
    constexpr int N = Vec16<T>::N;
    const int64_t nv = a.dim / N;
    const uint32_t id = a.ids[t];
    const bool ok = id < a.vocab;
    const T *src = static_cast<const T *>(a.embed) + (int64_t)id * a.dim;
    T *x = static_cast<T *>(a.x) + t * a.dim;
    T *out = static_cast<T *>(a.normed) + t * a.dim;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    float sq = 0.f;
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x)
    {
        const uint4 raw = ok ? ldg_keep(src + v * N) : zero;
        stg(x + v * N, raw);
        const Vec16<T> xv = as_vec<T>(raw);
#pragma unroll
        for (int e = 0; e < N; ++e)
        {
            const float f = to_f(xv.v[e]);
            sq = fmaf(f, f, sq);
        }
    }
    const float total = block_sum(sq, scratch);
    const float inv_rms = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)a.dim), kRmsEps)));
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x)
    {
        const Vec16<T> xv = as_vec<T>(ok ? ldg_keep(src + v * N) : zero);
        const Vec16<T> wv = as_vec<T>(ldg_keep(static_cast<const T *>(a.norm_w) + v * N));
        Vec16<T> o;
#pragma unroll
        for (int e = 0; e < N; ++e)
            o.v[e] = from_f<T>(__fmul_rn(__fmul_rn(to_f(xv.v[e]), to_f(wv.v[e])), inv_rms));
        stg(out + v * N, as_u4(o));
    }
}

// SwiGLU over output vectors [n * per, (n + 1) * per) of the [batch, hidden]
// output (16-byte vectors; hidden is a multiple of the vector width).
template <typename T>
__device__ __forceinline__ void swiglu_range(const StepArgs &a, int64_t n)
{
    constexpr int N = Vec16<T>::N;
    const int64_t fv = a.hidden / N;
    const int64_t end = min((n + 1) * a.sw_per_cta, a.r.batch * fv);
    const T *in = static_cast<const T *>(a.gate_up);
    T *out = static_cast<T *>(a.ffn_out);
    for (int64_t e = n * a.sw_per_cta + threadIdx.x; e < end; e += blockDim.x)
    {
        const int64_t t = e / fv;
        const int64_t c = e - t * fv;
        const T *g = in + t * 2 * a.hidden + c * N;
        const Vec16<T> gv = as_vec<T>(ldg_stream(g));
        const Vec16<T> uv = as_vec<T>(ldg_stream(g + a.hidden));
        Vec16<T> o;
#pragma unroll
        for (int k = 0; k < N; ++k)
            o.v[k] = from_f<T>(silu_mul<T>(to_f(gv.v[k]), to_f(uv.v[k])));
        stg(out + t * a.hidden + c * N, as_u4(o));
    }
}

// PV: the score rows also produce the attention output P.V (the V blocks
// stream after the K blocks; this step's V row is patched in like the K row).
// DEV_ANGLES: some position of the launch may lie outside the host cos/sin
// table (see score_row_stream). Three CTAs per SM: the streaming rows need
// three 64 KB rings per SM, so registers are capped at what three CTAs leave
// (80 per thread at 7 warps).
template <typename T, int LPR, bool PV, bool DEV_ANGLES>
__global__ void __launch_bounds__(kStreamThreads, 3) decode_step_kernel(const StepArgs a)
{
    extern __shared__ __align__(128) uint8_t step_smem[];
    __shared__ StreamShared sh;
    const int64_t bid = blockIdx.x;
    if (bid < a.score_ctas)
    {
        // (takes its ticket for the length update inside)
        cg::cluster_group cluster = cg::this_cluster();
        score_row_stream<T, LPR, true, PV, T, DEV_ANGLES>(a.d, a.r, bid / (int64_t)cluster.num_blocks(), cluster,
                                                          step_smem, sh, &g_step_error);
        return;
    }
    // Other roles read no lengths: their ticket comes first.
    if (threadIdx.x < 32)
        step_ticket(a.r, threadIdx.x, false, 0u, 0u);
    if (bid < a.score_ctas + a.norm_ctas)
        embed_norm_row<T>(a, bid - a.score_ctas, sh.scratch);
    else if (bid < a.score_ctas + a.norm_ctas + a.sw_ctas)
        swiglu_range<T>(a, bid - a.score_ctas - a.norm_ctas);
}

// Paged K/V caches of a step: pools (num_pages, Hkv, page_rows, head_dim)
// with page_rows = l2k_paged_block_rows (one streamed key block per page);
// positions [j page_rows, (j + 1) page_rows) of sequence b live in page
// block_table[b * max_pages + j].
struct PagedCaches
{
    const uint32_t *block_table;
    int64_t max_pages;
    int64_t num_pages;
};

struct Plan
{
    int lpr;
    int C;
    bool pv;
    bool dev_angles; // some appended position may lie outside the host cos/sin table
    size_t smem;
    StepArgs k;
};

// Validates the arguments and lays out the grid; L2K_OK or a status.
template <typename T>
int plan_step(const l2k_decode_step_args &p, void *attn_out, uint32_t *workspace, const PagedCaches *paged,
              Plan &plan)
{
    constexpr int N = Vec16<T>::N;
    const int64_t row_bytes = p.head_dim * (int64_t)sizeof(T);
    const int lpr = (int)(row_bytes / 16);
    L2K_REQUIRE_SHAPE(row_bytes % 16 == 0 && (lpr == 4 || lpr == 8 || lpr == 16 || lpr == 32),
                      "l2k_decode_step: head_dim * element size must be 64, 128, 256 or 512 bytes (got %lld)",
                      (long long)row_bytes);
    L2K_REQUIRE_SHAPE(p.pairing == L2K_ROPE_INTERLEAVED || (p.head_dim / 2) % N == 0,
                      "l2k_decode_step: head_dim / 2 must be a multiple of %d for the half pairing", N);
    L2K_REQUIRE_SHAPE(p.dim % N == 0 && p.hidden % N == 0,
                      "l2k_decode_step: dim and hidden must be multiples of %d", N);
    const void *vec_ptrs[] = {p.qkv, p.q, p.k_cache, p.v_cache, p.embed_table, p.norm_weight, p.x, p.normed};
    for (const void *ptr : vec_ptrs)
        L2K_REQUIRE_SHAPE(is_aligned(ptr, 16), "l2k_decode_step: tensors must be 16-byte aligned");
    if (p.hidden > 0)
        L2K_REQUIRE_SHAPE(is_aligned(p.gate_up, 16) && is_aligned(p.ffn_out, 16),
                          "l2k_decode_step: gate_up / ffn_out must be 16-byte aligned");
    L2K_REQUIRE(p.rope_table == nullptr || is_aligned(p.rope_table, 8),
                "l2k_decode_step: rope_table must be 8-byte aligned");

    const int64_t rows = p.batch * p.q_head_num;
    const int64_t kb = kBlockBytes / row_bytes;
    const int64_t blocks_per_row = ceil_div(p.kv_cache_len, kb);
    int C = 1;
    while (C < 8 && rows * C < 3LL * num_sms() && C * 2 <= blocks_per_row)
        C *= 2;
    const size_t smem = stream_smem_bytes(p.kv_cache_len, row_bytes, C) + (attn_out ? pv_smem_bytes(p.head_dim) : 0);
    L2K_REQUIRE_SHAPE(smem <= (size_t)kNS * kBlockBytes + 128 * 1024, "l2k_decode_step: kv_cache_len %lld too long",
                      (long long)p.kv_cache_len);
    L2K_REQUIRE_SHAPE(attn_out == nullptr || is_aligned(attn_out, 16),
                      "l2k_decode_step_attention: attn_out must be 16-byte aligned");

    StepArgs &k = plan.k;
    k = StepArgs{};
    k.d = DecodeArgs{p.q, p.k_cache, nullptr, p.kv_lens, nullptr, 0u, p.qk, p.q_head_num,
                     p.q_head_num / p.kv_head_num, p.kv_head_num, 1, p.kv_cache_len, p.head_dim, 0,
                     1.f / sqrtf((float)p.head_dim),
                     (p.kv_cache_len * (int64_t)sizeof(T)) % 16 == 0 && is_aligned(p.qk, 16)};
    k.d.v = p.v_cache;
    k.d.qkv = attn_out; // (B, Hq, 1, hd); null without the attention output
    if (paged)
    {
        // k_cache / v_cache are page pools; kv_cache_len is the logical length
        L2K_REQUIRE_SHAPE(p.kv_cache_len == paged->max_pages * kb,
                          "l2k_decode_step_paged: kv_cache_len (%lld) must be max_pages * page_rows (%lld * %lld)",
                          (long long)p.kv_cache_len, (long long)paged->max_pages, (long long)kb);
        k.d.block_table = paged->block_table;
        k.d.max_pages = paged->max_pages;
        k.d.num_pages = paged->num_pages;
    }
    k.r = StepRowArgs{p.qkv, p.is_done, p.q_lens, p.kv_lens, p.max_lens, workspace, p.q, p.k_cache, p.v_cache,
                      reinterpret_cast<const float2 *>(p.rope_table), p.rope_table ? p.rope_table_positions : 0,
                      p.batch, (p.q_head_num + 2 * p.kv_head_num) * p.head_dim, p.pairing};
    k.ids = p.input_ids;
    k.embed = p.embed_table;
    k.norm_w = p.norm_weight;
    k.x = p.x;
    k.normed = p.normed;
    k.vocab = p.vocab_size;
    k.dim = p.dim;
    k.gate_up = p.gate_up;
    k.ffn_out = p.ffn_out;
    k.hidden = p.hidden;
    k.score_ctas = rows * C;
    k.norm_ctas = p.batch;
    const int64_t sw_vecs = p.batch * (p.hidden / N);
    k.sw_per_cta = (int64_t)kStreamThreads * kSwigluVecsPerThread;
    k.sw_ctas = ceil_div(sw_vecs, k.sw_per_cta);
    const int64_t aux = ceil_div(k.norm_ctas + k.sw_ctas, C) * C;
    L2K_REQUIRE_SHAPE(k.score_ctas + aux < (int64_t(1) << 31), "l2k_decode_step: grid too large");
    plan.lpr = lpr;
    plan.C = C;
    plan.pv = attn_out != nullptr;
    // Appended positions are < kv_cache_len, and the table row is used when the
    // updated length is at most 4096 and the position is in the table.
    plan.dev_angles = !(p.rope_table && p.kv_cache_len <= 4096 && p.kv_cache_len <= p.rope_table_positions);
    plan.smem = smem;
    return L2K_OK;
}

template <typename T, int LPR, bool PV>
cudaError_t launch_step_kernel(const Plan &plan, cudaStream_t stream)
{
    auto kernel = plan.dev_angles ? decode_step_kernel<T, LPR, PV, true> : decode_step_kernel<T, LPR, PV, false>;
    if (plan.smem > 48 * 1024)
    {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)plan.smem);
        if (e != cudaSuccess)
            return e;
    }
    const int64_t aux = ceil_div(plan.k.norm_ctas + plan.k.sw_ctas, plan.C) * plan.C;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(plan.k.score_ctas + aux));
    cfg.blockDim = dim3(kStreamThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)plan.C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kernel, plan.k);
}

template <typename T, bool PV>
cudaError_t launch_step_lpr(const Plan &plan, cudaStream_t stream)
{
    switch (plan.lpr)
    {
    case 32:
        return launch_step_kernel<T, 32, PV>(plan, stream);
    case 16:
        return launch_step_kernel<T, 16, PV>(plan, stream);
    case 8:
        return launch_step_kernel<T, 8, PV>(plan, stream);
    default:
        return launch_step_kernel<T, 4, PV>(plan, stream);
    }
}

template <typename T>
int run_step(const l2k_decode_step_args &p, void *attn_out, uint32_t *workspace, const PagedCaches *paged,
             cudaStream_t stream, bool launch)
{
    Plan plan;
    if (int st = plan_step<T>(p, attn_out, workspace, paged, plan))
        return st;
    if (!launch)
        return L2K_OK;
    const cudaError_t e = plan.pv ? launch_step_lpr<T, true>(plan, stream) : launch_step_lpr<T, false>(plan, stream);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_decode_step: %s", cudaGetErrorString(e));
    return check_launch("l2k_decode_step");
}

int step_entry(const l2k_decode_step_args *pp, void *attn_out, uint32_t *workspace, cudaStream_t stream, bool launch,
               const PagedCaches *paged = nullptr)
{
    L2K_REQUIRE(pp != nullptr, "l2k_decode_step: null args");
    const l2k_decode_step_args &p = *pp;
    L2K_REQUIRE(dtype_ok(p.dtype), "l2k_decode_step: unsupported dtype %d", p.dtype);
    L2K_REQUIRE(p.pairing == L2K_ROPE_INTERLEAVED || p.pairing == L2K_ROPE_HALF,
                "l2k_decode_step: bad pairing %d", p.pairing);
    L2K_REQUIRE(p.batch >= 0 && p.vocab_size >= 0 && p.dim > 0 && p.q_head_num > 0 && p.kv_head_num > 0 &&
                    p.head_dim > 0 && p.kv_cache_len > 0 && p.hidden >= 0 && p.rope_table_positions >= 0,
                "l2k_decode_step: bad size");
    L2K_REQUIRE(p.head_dim % 2 == 0, "l2k_decode_step: head_dim must be even (got %lld)", (long long)p.head_dim);
    L2K_REQUIRE(p.q_head_num % p.kv_head_num == 0, "l2k_decode_step: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(workspace != nullptr && is_aligned(workspace, 4), "l2k_decode_step: null or misaligned workspace");
    if (p.batch == 0)
        return L2K_OK;
    L2K_REQUIRE(p.q_lens && p.kv_lens && p.max_lens && p.input_ids && p.embed_table && p.norm_weight && p.x &&
                    p.normed && p.qkv && p.is_done && p.q && p.k_cache && p.v_cache && p.qk,
                "l2k_decode_step: null pointer");
    L2K_REQUIRE(p.hidden == 0 || (p.gate_up && p.ffn_out), "l2k_decode_step: null gate_up / ffn_out");
    L2K_REQUIRE(p.x != p.normed, "l2k_decode_step: x and normed must be distinct buffers");
    if (paged)
        L2K_REQUIRE(paged->block_table && paged->max_pages > 0 && paged->num_pages > 0,
                    "l2k_decode_step_paged: null block table or empty page pool");
    L2K_DISPATCH(p.dtype, { return run_step<T>(p, attn_out, workspace, paged, stream, launch); });
    return L2K_OK;
}

} // namespace

int read_step_error(bool clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_step_error, sizeof(int)) != cudaSuccess)
        return -1;
    if (clear && v)
    {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_step_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

} // namespace l2k

extern "C" int64_t l2k_decode_step_workspace_bytes(void) { return 16; }

extern "C" int l2k_decode_step_supported(const l2k_decode_step_args *args)
{
    uint32_t dummy = 0; // never dereferenced: nothing is launched
    return l2k::step_entry(args, nullptr, &dummy, nullptr, false);
}

extern "C" int l2k_decode_step(const l2k_decode_step_args *args, uint32_t *workspace, l2k_stream_t stream)
{
    return l2k::step_entry(args, nullptr, workspace, stream, true);
}

extern "C" int l2k_decode_step_attention(const l2k_decode_step_args *args, void *attn_out, uint32_t *workspace,
                                         l2k_stream_t stream)
{
    L2K_REQUIRE(attn_out != nullptr, "l2k_decode_step_attention: null attn_out");
    return l2k::step_entry(args, attn_out, workspace, stream, true);
}

extern "C" int l2k_decode_step_paged(const l2k_decode_step_args *args, const uint32_t *block_table, int64_t max_pages,
                                     int64_t num_pages, uint32_t *workspace, l2k_stream_t stream)
{
    const l2k::PagedCaches paged{block_table, max_pages, num_pages};
    return l2k::step_entry(args, nullptr, workspace, stream, true, &paged);
}

extern "C" int l2k_decode_step_attention_paged(const l2k_decode_step_args *args, const uint32_t *block_table,
                                               int64_t max_pages, int64_t num_pages, void *attn_out,
                                               uint32_t *workspace, l2k_stream_t stream)
{
    L2K_REQUIRE(attn_out != nullptr, "l2k_decode_step_attention_paged: null attn_out");
    const l2k::PagedCaches paged{block_table, max_pages, num_pages};
    return l2k::step_entry(args, attn_out, workspace, stream, true, &paged);
}

// ---------------------------------------------------------------------------
// l2k_decode_step_no_alloc: the same launch with its workspace in a
// file-scope device array instead of caller memory. The array is 256 bytes
// (the step needs l2k_decode_step_workspace_bytes() of them); each device
// has its own copy, zero when the module loads, and every step that runs to
// its end (including one whose bounded waits expired) leaves it zero again.
// Its address is looked up with cudaGetSymbolAddress on the first call on a
// device, with that device current, and cached together with the device's
// current driver context; a call that finds another context current (after
// cudaDeviceReset, or under a driver context the caller made current) looks
// it up again, so the cached address never outlives the context it belongs
// to. Nothing is allocated.
// ---------------------------------------------------------------------------
namespace l2k
{
constexpr int kStepScratchBytes = 256;
constexpr int kMaxScratchDevices = 64;
static __device__ __align__(256) uint32_t g_step_scratch[kStepScratchBytes / 4];

namespace
{
struct ScratchSlot
{
    void *ctx = nullptr;     // the driver context the address was looked up in
    uint32_t *ptr = nullptr; // g_step_scratch's device address in that context
};
std::mutex g_scratch_mutex;
ScratchSlot g_scratch[kMaxScratchDevices];

// cuCtxGetCurrent from the driver, found at run time (the library links the
// CUDA runtime statically and does not link the driver library itself).
using CtxGetCurrentFn = int (*)(void **);
CtxGetCurrentFn ctx_get_current()
{
    static CtxGetCurrentFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    return fn;
}

// The static scratch of the device `stream` belongs to, which must be the
// current device (cudaGetSymbolAddress answers for the current context).
int static_scratch(const char *who, cudaStream_t stream, uint32_t **out)
{
    if (l2k_decode_step_workspace_bytes() > kStepScratchBytes)
        return set_error(L2K_ERR_UNSUPPORTED_SHAPE, "%s: the step needs %lld bytes of scratch, the static scratch "
                         "holds %d", who, (long long)l2k_decode_step_workspace_bytes(), kStepScratchBytes);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "%s: cudaGetDevice: %s", who, cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxScratchDevices)
        return set_error(L2K_ERR_UNSUPPORTED_SHAPE, "%s: device %d >= %d", who, dev, kMaxScratchDevices);
    if (stream != nullptr && stream != cudaStreamLegacy && stream != cudaStreamPerThread)
    {
        int sdev = -1;
        e = cudaStreamGetDevice(stream, &sdev);
        if (e != cudaSuccess)
            return set_error(L2K_ERR_CUDA, "%s: cudaStreamGetDevice: %s", who, cudaGetErrorString(e));
        if (sdev != dev)
            return set_error(L2K_ERR_INVALID_ARGUMENT, "%s: the stream belongs to device %d but device %d is "
                             "current; make the stream's device current first", who, sdev, dev);
    }
    // The context the lookup is valid for: the current one. A null context
    // means the runtime has not made one current yet; the lookup below does.
    void *ctx = nullptr;
    if (CtxGetCurrentFn get = ctx_get_current())
        get(&ctx);
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    ScratchSlot &slot = g_scratch[dev];
    if (!slot.ptr || !ctx || slot.ctx != ctx)
    {
        void *p = nullptr;
        e = cudaGetSymbolAddress(&p, g_step_scratch);
        if (e != cudaSuccess)
            return set_error(L2K_ERR_CUDA, "%s: cudaGetSymbolAddress: %s", who, cudaGetErrorString(e));
        if (!ctx)
            if (CtxGetCurrentFn get = ctx_get_current())
                get(&ctx); // the lookup made the primary context current
        slot.ptr = static_cast<uint32_t *>(p);
        slot.ctx = ctx;
    }
    *out = slot.ptr;
    return L2K_OK;
}
} // namespace
} // namespace l2k

extern "C" int l2k_decode_step_no_alloc(const l2k_decode_step_args *args, l2k_stream_t stream)
{
    uint32_t *scratch = nullptr;
    if (int st = l2k::static_scratch("l2k_decode_step_no_alloc", (cudaStream_t)stream, &scratch))
        return st;
    return l2k::step_entry(args, nullptr, scratch, stream, true);
}

extern "C" int l2k_decode_step_attention_no_alloc(const l2k_decode_step_args *args, void *attn_out,
                                                  l2k_stream_t stream)
{
    L2K_REQUIRE(attn_out != nullptr, "l2k_decode_step_attention_no_alloc: null attn_out");
    uint32_t *scratch = nullptr;
    if (int st = l2k::static_scratch("l2k_decode_step_attention_no_alloc", (cudaStream_t)stream, &scratch))
        return st;
    return l2k::step_entry(args, attn_out, scratch, stream, true);
}
