// Row-major GEMM on the CUDA cores with fp32 accumulation: the drop-in for
// the reference's launch_linear (src/kernel/linear.cu:42-155, a cuBLAS call)
// wherever the tensor-core kernel (gemm_tc.cu: plain 16-bit GEMMs with A
// not transposed) does not take it, and the fp32 QK^T path. 64x64 output tile per CTA, 16-deep K slices staged
// in shared memory, 4x4 outputs per thread. Three batch addressings:
// plain (one GEMM), pointer arrays (the reference's batched form), and the
// attention call sites computed from (seq, head) with grouped KV heads:
// QK^T (trans_B) and P.V.
#include "common.cuh"

#include <algorithm>

namespace l2k
{
namespace
{

constexpr int BM = 64, BN = 64, BK = 16;

enum BatchMode
{
    PLAIN = 0,
    PTR_ARRAYS = 1,
    QK_HEADS = 2 // (seq, head) slices; also the P.V call site
};

struct GemmArgs
{
    int trans_a, trans_b;
    int64_t m, n, k;
    const void *a;
    int64_t lda;
    const void *b;
    int64_t ldb;
    void *c;
    int64_t ldc;
    int64_t batch;
    const void *const *a_array;
    const void *const *b_array;
    void *const *c_array;
    // QK_HEADS
    int64_t Hq, group, Hkv, qc, S;
    const uint32_t *row_lens; // optional: rows i >= row_lens[seq] are skipped
    const uint32_t *k_dev;    // optional: the contraction length is min(k, *k_dev)
};

template <typename T, int MODE>
__global__ void __launch_bounds__(256) gemm_kernel(const GemmArgs g)
{
    __shared__ float As[BK][BM + 1];
    __shared__ float Bs[BK][BN + 1];
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    const int64_t i0 = (int64_t)blockIdx.y * BM, j0 = (int64_t)blockIdx.x * BN;
    for (int64_t z = blockIdx.z; z < g.batch; z += gridDim.z)
    {
        const T *A;
        const T *B;
        T *C;
        int64_t m = g.m;
        if constexpr (MODE == PLAIN)
        {
            A = static_cast<const T *>(g.a);
            B = static_cast<const T *>(g.b);
            C = static_cast<T *>(g.c);
        }
        else if constexpr (MODE == PTR_ARRAYS)
        {
            A = static_cast<const T *>(g.a_array[z]);
            B = static_cast<const T *>(g.b_array[z]);
            C = static_cast<T *>(g.c_array[z]);
        }
        else
        {
            const int64_t bb = z / g.Hq, h = z - bb * g.Hq;
            A = static_cast<const T *>(g.a) + (bb * g.Hq + h) * g.qc * g.lda;
            B = static_cast<const T *>(g.b) + (bb * g.Hkv + h / g.group) * g.S * g.ldb;
            C = static_cast<T *>(g.c) + (bb * g.Hq + h) * g.qc * g.ldc;
            if (g.row_lens)
                m = min(m, (int64_t)g.row_lens[bb]);
        }
        if (i0 >= m)
            continue;
        const int64_t kl = g.k_dev ? min(g.k, (int64_t)*g.k_dev) : g.k;
        float acc[4][4] = {};
        for (int64_t k0 = 0; k0 < kl; k0 += BK)
        {
            for (int e = threadIdx.x; e < BM * BK; e += blockDim.x)
            {
                const int r = e / BK, kk = e % BK;
                const int64_t gi = i0 + r, gk = k0 + kk;
                float v = 0.f;
                if (gi < m && gk < kl)
                    v = to_f(g.trans_a ? A[gk * g.lda + gi] : A[gi * g.lda + gk]);
                As[kk][r] = v;
            }
            for (int e = threadIdx.x; e < BN * BK; e += blockDim.x)
            {
                const int cidx = e / BK, kk = e % BK;
                const int64_t gj = j0 + cidx, gk = k0 + kk;
                float v = 0.f;
                if (gj < g.n && gk < kl)
                    v = to_f(g.trans_b ? B[gj * g.ldb + gk] : B[gk * g.ldb + gj]);
                Bs[kk][cidx] = v;
            }
            __syncthreads();
#pragma unroll
            for (int kk = 0; kk < BK; ++kk)
            {
                float av[4], bv[4];
#pragma unroll
                for (int u = 0; u < 4; ++u)
                {
                    av[u] = As[kk][ty * 4 + u];
                    bv[u] = Bs[kk][tx * 4 + u];
                }
#pragma unroll
                for (int u = 0; u < 4; ++u)
#pragma unroll
                    for (int w = 0; w < 4; ++w)
                        acc[u][w] = fmaf(av[u], bv[w], acc[u][w]);
            }
            __syncthreads();
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int w = 0; w < 4; ++w)
            {
                const int64_t gi = i0 + ty * 4 + u, gj = j0 + tx * 4 + w;
                if (gi < m && gj < g.n)
                    C[gi * g.ldc + gj] = from_f<T>(acc[u][w]);
            }
    }
}

template <typename T, int MODE>
int launch_gemm(const GemmArgs &g, cudaStream_t stream)
{
    const dim3 grid((unsigned)ceil_div(g.n, BN), (unsigned)ceil_div(g.m, BM),
                    (unsigned)std::max<int64_t>(1, std::min<int64_t>(g.batch, 65535)));
    gemm_kernel<T, MODE><<<grid, 256, 0, stream>>>(g);
    return check_launch("l2k gemm");
}

} // namespace

// Shared with scores.cu: QK^T per (seq, head) on the CUDA cores.
int qk_scores_cuda_cores(const void *q, const void *k, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t qc,
                         int64_t S, int64_t hd, int64_t m, int64_t n, const uint32_t *row_lens, int dtype,
                         cudaStream_t stream)
{
    GemmArgs g{};
    g.trans_a = 0;
    g.trans_b = 1;
    g.m = m;
    g.n = n;
    g.k = hd;
    g.a = q;
    g.lda = hd;
    g.b = k;
    g.ldb = hd;
    g.c = qk;
    g.ldc = S;
    g.batch = batch * Hq;
    g.Hq = Hq;
    g.group = Hq / Hkv;
    g.Hkv = Hkv;
    g.qc = qc;
    g.S = S;
    g.row_lens = row_lens;
    L2K_DISPATCH(dtype, { return launch_gemm<T, QK_HEADS>(g, stream); });
    return L2K_OK;
}

// P.V per (seq, head) on the CUDA cores: qkv[b,h,i,:] = sum_{j<n} qk[b,h,i,j] v[b,h/g,j,:]
// for i < m (n further capped by *n_dev when given).
int attention_qkv_cuda_cores(const void *qk, const void *v, void *qkv, int64_t batch, int64_t Hq, int64_t Hkv,
                             int64_t qc, int64_t S, int64_t hd, int64_t m, int64_t n, const uint32_t *n_dev,
                             int dtype, cudaStream_t stream)
{
    GemmArgs g{};
    g.trans_a = 0;
    g.trans_b = 0;
    g.m = m;
    g.n = hd;
    g.k = n;
    g.a = qk;
    g.lda = S;
    g.b = v;
    g.ldb = hd;
    g.c = qkv;
    g.ldc = hd;
    g.batch = batch * Hq;
    g.Hq = Hq;
    g.group = Hq / Hkv;
    g.Hkv = Hkv;
    g.qc = qc;
    g.S = S;
    g.k_dev = n_dev;
    L2K_DISPATCH(dtype, { return launch_gemm<T, QK_HEADS>(g, stream); });
    return L2K_OK;
}

bool gemv_supported(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const void *b,
                    int64_t ldb); // gemv.cu
int gemv(int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda, const void *b, int64_t ldb,
         void *c, int64_t ldc, int dtype, cudaStream_t stream);
bool gemm_tc_supported(int dtype, int trans_a, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda,
                       const void *b, int64_t ldb, const void *c); // gemm_tc.cu
int gemm_tc(int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda, const void *b, int64_t ldb,
            void *c, int64_t ldc, int dtype, cudaStream_t stream);
bool attention_qkv_tc_supported(int dtype, int64_t head_dim, int64_t S, int64_t n, const void *qk, const void *v,
                                const void *qkv, int64_t grid); // attention_qkv_tc.cu
int attention_qkv_tc(const void *qk, const void *v, void *qkv, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc,
                     int64_t S, int64_t m, int64_t n, int dtype, cudaStream_t stream,
                     const uint32_t *block_table = nullptr, const uint32_t *kv_lens = nullptr, int64_t max_pages = 0,
                     int64_t num_pages = 0);

} // namespace l2k

extern "C" int l2k_linear(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda,
                          const void *b, int64_t ldb, void *c, int64_t ldc, int64_t batch_count,
                          const void *const *a_array, const void *const *b_array, void *const *c_array, int dtype,
                          l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_linear: unsupported dtype %d", dtype);
    L2K_REQUIRE(m >= 0 && n >= 0 && k >= 0 && batch_count >= 0, "l2k_linear: negative size");
    L2K_REQUIRE(ldc >= n && lda >= (trans_a ? m : k) && ldb >= (trans_b ? k : n), "l2k_linear: leading dimension too small");
    if (m == 0 || n == 0)
        return L2K_OK;
    L2K_REQUIRE_SHAPE(ceil_div(m, BM) <= 65535, "l2k_linear: m too large");
    GemmArgs g{};
    g.trans_a = trans_a ? 1 : 0;
    g.trans_b = trans_b ? 1 : 0;
    g.m = m;
    g.n = n;
    g.k = k;
    g.a = a;
    g.lda = lda;
    g.b = b;
    g.ldb = ldb;
    g.c = c;
    g.ldc = ldc;
    g.a_array = a_array;
    g.b_array = b_array;
    g.c_array = c_array;
    if (batch_count == 0)
    {
        L2K_REQUIRE(a && b && c, "l2k_linear: null pointer");
        // 16-bit with A not transposed: up to 8 rows stream B on the CUDA cores,
        // more on tcgen05 (A and B tiles by TMA, fp32 accumulator in tensor memory)
        if (gemv_supported(dtype, trans_a, trans_b, m, n, k, b, ldb))
            return gemv(trans_b, m, n, k, a, lda, b, ldb, c, ldc, dtype, stream);
        if (gemm_tc_supported(dtype, trans_a, m, n, k, a, lda, b, ldb, c))
            return gemm_tc(trans_b, m, n, k, a, lda, b, ldb, c, ldc, dtype, stream);
        g.batch = 1;
        L2K_DISPATCH(dtype, { return launch_gemm<T, PLAIN>(g, stream); });
    }
    else
    {
        L2K_REQUIRE(a_array && b_array && c_array, "l2k_linear: null pointer array");
        g.batch = batch_count;
        L2K_DISPATCH(dtype, { return launch_gemm<T, PTR_ARRAYS>(g, stream); });
    }
    return L2K_OK;
}

extern "C" int l2k_qk_scores(const void *q, const void *k, void *qk, int64_t batch, int64_t q_head_num,
                             int64_t kv_head_num, int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim,
                             int64_t m, int64_t n, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_qk_scores: unsupported dtype %d", dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim >= 0 && m >= 0 && n >= 0,
                "l2k_qk_scores: negative size");
    L2K_REQUIRE(m <= q_cache_len && n <= kv_cache_len, "l2k_qk_scores: m/n exceed the cache dims");
    if (batch == 0 || q_head_num == 0 || m == 0 || n == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_qk_scores: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(q && k && qk, "l2k_qk_scores: null pointer");
    return qk_scores_cuda_cores(q, k, qk, batch, q_head_num, kv_head_num, q_cache_len, kv_cache_len, head_dim, m, n,
                                nullptr, dtype, stream);
}

extern "C" int l2k_attention_qkv(const void *qk, const void *v, void *qkv, int64_t batch, int64_t q_head_num,
                                 int64_t kv_head_num, int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim,
                                 int64_t m, int64_t n, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_attention_qkv: unsupported dtype %d", dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim >= 0 && m >= 0 && n >= 0,
                "l2k_attention_qkv: negative size");
    L2K_REQUIRE(m <= q_cache_len && n <= kv_cache_len, "l2k_attention_qkv: m/n exceed the cache dims");
    if (batch == 0 || q_head_num == 0 || m == 0 || head_dim == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_attention_qkv: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(qk && v && qkv, "l2k_attention_qkv: null pointer");
    // 16-bit, head_dim 128: tcgen05 (P tiles by TMA, fp32 accumulator in tensor memory)
    if (attention_qkv_tc_supported(dtype, head_dim, kv_cache_len, n, qk, v, qkv, ceil_div(m, 128) * batch * q_head_num))
        return attention_qkv_tc(qk, v, qkv, batch, q_head_num, kv_head_num, q_cache_len, kv_cache_len, m, n, dtype,
                                stream);
    L2K_REQUIRE_SHAPE(ceil_div(m, BM) <= 65535, "l2k_attention_qkv: m too large");
    return attention_qkv_cuda_cores(qk, v, qkv, batch, q_head_num, kv_head_num, q_cache_len, kv_cache_len, head_dim,
                                    m, n, nullptr, dtype, stream);
}

// P.V over a paged V cache (16-bit, head_dim 128: one page is one 64-key
// block of the tcgen05 kernel). qk is (batch, Hq, q_cache_len, max_pages * 64).
extern "C" int l2k_attention_qkv_paged(const void *qk, const void *v_pages, const uint32_t *block_table,
                                       int64_t max_pages, int64_t num_pages, const uint32_t *kv_lens, void *qkv,
                                       int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t q_cache_len,
                                       int64_t head_dim, int64_t m, int64_t n, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    const char *name = "l2k_attention_qkv_paged";
    L2K_REQUIRE(dtype_ok(dtype), "%s: unsupported dtype %d", name, dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim >= 0 && m >= 0 && n >= 0 &&
                    max_pages >= 0 && num_pages >= 0,
                "%s: negative size", name);
    const int64_t S = max_pages * 64;
    L2K_REQUIRE(m <= q_cache_len && n <= S, "%s: m/n exceed the cache dims", name);
    if (batch == 0 || q_head_num == 0 || m == 0 || head_dim == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0, "%s: q_head_num must be a multiple of kv_head_num",
                name);
    L2K_REQUIRE(qk && v_pages && qkv && block_table && kv_lens && num_pages > 0, "%s: null pointer or no pages", name);
    L2K_REQUIRE_SHAPE(num_pages * kv_head_num < (int64_t(1) << 31), "%s: page pool too large", name);
    L2K_REQUIRE_SHAPE(attention_qkv_tc_supported(dtype, head_dim, S, n, qk, v_pages, qkv,
                                                 ceil_div(m, 128) * batch * q_head_num),
                      "%s: the paged path takes 16-bit data with head_dim 128, 16-byte aligned, n >= 1", name);
    return attention_qkv_tc(qk, v_pages, qkv, batch, q_head_num, kv_head_num, q_cache_len, S, m, n, dtype, stream,
                            block_table, kv_lens, max_pages, num_pages);
}
