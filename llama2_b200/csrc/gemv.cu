// Few-row products C = A op(B) for plain 16-bit launch_linear calls with at
// most 8 rows in A (decode at small batch): bound by reading B once, which
// the CUDA cores keep up with (at most 8 FMAs per 2-byte element of B).
//
//   * B stored K x N (trans_B = false, a weight [in, out]): a CTA owns 256
//     columns (each of its 8 warps' lanes 8 consecutive columns = one 16-byte
//     load of a B row) and a range of k rows; warp w takes every 8th row of
//     the range, four rows in flight per lane; the warps' partial sums meet
//     in shared memory. The k range is split over a thread-block cluster of
//     up to 8 CTAs (enough CTAs to fill the GPU); ranks 1.. push their partial
//     sums into rank 0 over distributed shared memory (st.async), and rank 0
//     adds them in rank order and stores.
//   * B stored N x K (trans_B = true): one warp per column n, lanes striding
//     the row in 16-byte units, a warp-shuffle reduction per A row.
// A's rows are staged in shared memory as fp32. Accumulation is fp32 in a
// fixed order (results do not depend on timing).
//
// Reference: src/kernel/linear.cu:42-155 (cublasGemmEx).
#include "common.cuh"

#include <algorithm>

namespace l2k
{

__device__ int g_gemv_error = 0; // first timeout code of the kernels of this file

namespace
{

constexpr int kMaxRows = 8;
constexpr int kThreads = 256;
constexpr int kCols = 256;                 // columns per CTA (K x N layout)
constexpr long long kGemvWaitCycles = 4000000000LL;

struct GemvArgs
{
    const void *a;
    int64_t lda;
    const void *b;
    int64_t ldb;
    void *c;
    int64_t ldc;
    int m, n, k;
    int split; // CTAs of a cluster sharing one column block (K x N layout)
};

__device__ __forceinline__ uint32_t sm_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Floats reserved for A's rows in the K x N kernel: M rows of the longest
// k range, rounded up to 4 floats (16 bytes).
__host__ __device__ constexpr int64_t a_floats(int64_t m_rows, int64_t k, int64_t split)
{
    return (m_rows * ((k + split - 1) / split) + 3) / 4 * 4;
}

// Cluster size and dynamic shared memory of the K x N kernel.
inline void kn_plan(int64_t m_rows, int64_t n, int64_t k, int *split_out, size_t *smem_out)
{
    const int64_t col_blocks = ceil_div(n, kCols);
    int split = 1;
    while (split < 8 && col_blocks * split * 2 <= 4LL * num_sms() && split * 2 * 64 <= k)
        split *= 2;
    *split_out = split;
    *smem_out = (size_t)(a_floats(m_rows, k, split) + (int64_t)(8 + 1 + split - 1) * m_rows * kCols) * sizeof(float);
}

// Rows of A as fp32 in shared memory: s_a[r * k_len + i] = A[r, k0 + i].
template <typename T>
__device__ __forceinline__ void stage_a(const GemvArgs &g, int k0, int k_len, float *s_a)
{
    const T *A = static_cast<const T *>(g.a);
    for (int idx = threadIdx.x; idx < g.m * k_len; idx += blockDim.x)
    {
        const int r = idx / k_len, i = idx - r * k_len;
        s_a[idx] = to_f(A[(int64_t)r * g.lda + k0 + i]);
    }
}

template <typename T, int M>
__global__ void __launch_bounds__(kThreads) gemv_kn_kernel(const GemvArgs g)
{
    extern __shared__ __align__(16) float s_dyn[];
    __shared__ uint64_t bar; // rank 0: the peers' partial sums have landed
    constexpr int N = Vec16<T>::N; // 8 columns per lane
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = g.split;
    const int rank = (int)(blockIdx.x % split);
    const int col_block = (int)(blockIdx.x / split);
    const int k0 = (int)((int64_t)rank * g.k / split), k1 = (int)((int64_t)(rank + 1) * g.k / split);
    const int k_len = k1 - k0;
    // The same layout in every rank (the peers address rank 0's slots by it):
    // A's rows for up to a_floats(M, k, split) floats, 16-byte aligned parts.
    float *s_a = s_dyn;                                   // [M][k_len]
    float *s_part = s_dyn + a_floats(M, g.k, split);      // [8 warps][M][256] (then rank 0's receive slots)
    if (split > 1 && tid == 0)
    {
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sm_addr(&bar)) : "memory");
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    stage_a<T>(g, k0, k_len, s_a);
    __syncthreads();

    const int64_t col = (int64_t)col_block * kCols + lane * N; // this lane's 8 columns (the same in every warp)
    const bool col_ok = col < g.n;
    float acc[M][N];
#pragma unroll
    for (int r = 0; r < M; ++r)
#pragma unroll
        for (int e = 0; e < N; ++e)
            acc[r][e] = 0.f;
    if (col_ok)
    {
        const T *B = static_cast<const T *>(g.b) + col;
        const bool full = col + N <= g.n;
        // rows k0 + warp, + 8, ...: four in flight per lane
        int i = warp;
        for (; i + 24 < k_len; i += 32)
        {
            uint4 w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                w[u] = full ? ldg_stream(B + (int64_t)(k0 + i + 8 * u) * g.ldb) : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
            for (int u = 0; u < 4; ++u)
            {
                const Vec16<T> wv = as_vec<T>(w[u]);
#pragma unroll
                for (int r = 0; r < M; ++r)
                {
                    const float av = s_a[r * k_len + i + 8 * u];
#pragma unroll
                    for (int e = 0; e < N; ++e)
                        acc[r][e] = fmaf(av, to_f(wv.v[e]), acc[r][e]);
                }
            }
        }
        for (; i < k_len; i += 8)
        {
            Vec16<T> wv;
            const T *row = B + (int64_t)(k0 + i) * g.ldb;
#pragma unroll
            for (int e = 0; e < N; ++e)
                wv.v[e] = col + e < g.n ? row[e] : from_f<T>(0.f);
#pragma unroll
            for (int r = 0; r < M; ++r)
            {
                const float av = s_a[r * k_len + i];
#pragma unroll
                for (int e = 0; e < N; ++e)
                    acc[r][e] = fmaf(av, to_f(wv.v[e]), acc[r][e]);
            }
        }
        if (!full)
        {
            // (a ragged last column block: the 16-byte loop above read nothing)
#pragma unroll
            for (int r = 0; r < M; ++r)
#pragma unroll
                for (int e = 0; e < N; ++e)
                    acc[r][e] = 0.f;
            for (int ii = warp; ii < k_len; ii += 8)
            {
                const T *row = B + (int64_t)(k0 + ii) * g.ldb;
#pragma unroll
                for (int r = 0; r < M; ++r)
                {
                    const float av = s_a[r * k_len + ii];
#pragma unroll
                    for (int e = 0; e < N; ++e)
                        if (col + e < g.n)
                            acc[r][e] = fmaf(av, to_f(row[e]), acc[r][e]);
                }
            }
        }
    }
    // warps -> CTA partial sums (fixed order)
#pragma unroll
    for (int r = 0; r < M; ++r)
#pragma unroll
        for (int e = 0; e < N; e += 4)
            *reinterpret_cast<float4 *>(s_part + ((int64_t)warp * M + r) * kCols + lane * N + e) =
                make_float4(acc[r][e], acc[r][e + 1], acc[r][e + 2], acc[r][e + 3]);
    __syncthreads();
    float *cta = s_part + (int64_t)8 * M * kCols; // [M][256] this CTA's sums, then rank 0's receive slots
    for (int idx = tid; idx < M * kCols; idx += kThreads)
    {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < 8; ++w)
            s += s_part[(int64_t)w * M * kCols + idx];
        cta[idx] = s;
    }
    __syncthreads();
    if (split > 1)
    {
        // every rank's sums are ready; ranks 1.. push theirs into rank 0's slots
        asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
        asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
        float *slots = cta + M * kCols; // rank 0: [split - 1][M][256]
        if (rank != 0)
        {
            for (int idx = tid * 4; idx < M * kCols; idx += kThreads * 4)
            {
                uint32_t dst, bar0;
                asm volatile("mapa.shared::cluster.u32 %0, %1, 0;"
                             : "=r"(dst)
                             : "r"(sm_addr(slots + (int64_t)(rank - 1) * M * kCols + idx)));
                asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(bar0) : "r"(sm_addr(&bar)));
                const float4 v = *reinterpret_cast<const float4 *>(cta + idx);
                asm volatile(
                    "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                        dst),
                    "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar0)
                    : "memory");
            }
            return;
        }
        if (tid == 0)
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sm_addr(&bar)),
                         "r"((uint32_t)((split - 1) * M * kCols * (int)sizeof(float)))
                         : "memory");
        const long long t0 = clock64();
        while (true)
        {
            uint32_t done;
            asm volatile("{\n\t.reg .pred p;\n\t"
                         "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], 0;\n\t"
                         "selp.u32 %0, 1, 0, p;\n\t}"
                         : "=r"(done)
                         : "r"(sm_addr(&bar))
                         : "memory");
            if (done)
                break;
            if (clock64() - t0 > kGemvWaitCycles)
            {
                atomicCAS(&g_gemv_error, 0, 0x501);
                return;
            }
        }
        for (int idx = tid; idx < M * kCols; idx += kThreads)
        {
            float s = cta[idx];
            for (int p = 1; p < split; ++p)
                s += slots[(int64_t)(p - 1) * M * kCols + idx];
            cta[idx] = s;
        }
        __syncthreads();
    }
    // store C[r, col_block * 256 + j]
    T *C = static_cast<T *>(g.c);
    for (int idx = tid; idx < M * kCols; idx += kThreads)
    {
        const int r = idx / kCols, j = idx - r * kCols;
        const int64_t cc = (int64_t)col_block * kCols + j;
        if (r < g.m && cc < g.n)
            C[(int64_t)r * g.ldc + cc] = from_f<T>(cta[idx]);
    }
}

// B stored N x K: one warp per column.
template <typename T, int M>
__global__ void __launch_bounds__(kThreads) gemv_nk_kernel(const GemvArgs g)
{
    extern __shared__ __align__(16) float s_dyn[];
    constexpr int N = Vec16<T>::N;
    float *s_a = s_dyn; // [M][k]
    stage_a<T>(g, 0, g.k, s_a);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t n = (int64_t)blockIdx.x * (kThreads / 32) + warp;
    if (n >= g.n)
        return;
    const T *row = static_cast<const T *>(g.b) + n * g.ldb;
    float acc[M];
#pragma unroll
    for (int r = 0; r < M; ++r)
        acc[r] = 0.f;
    const bool vec = (g.k % N) == 0;
    if (vec)
    {
        for (int u = lane; u < g.k / N; u += 32)
        {
            const Vec16<T> wv = as_vec<T>(ldg_stream(row + (int64_t)u * N));
#pragma unroll
            for (int r = 0; r < M; ++r)
#pragma unroll
                for (int e = 0; e < N; ++e)
                    acc[r] = fmaf(s_a[r * g.k + u * N + e], to_f(wv.v[e]), acc[r]);
        }
    }
    else
    {
        for (int i = lane; i < g.k; i += 32)
        {
            const float wv = to_f(row[i]);
#pragma unroll
            for (int r = 0; r < M; ++r)
                acc[r] = fmaf(s_a[r * g.k + i], wv, acc[r]);
        }
    }
#pragma unroll
    for (int r = 0; r < M; ++r)
    {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
    }
    if (lane == 0)
    {
        T *C = static_cast<T *>(g.c);
        for (int r = 0; r < g.m; ++r)
            C[(int64_t)r * g.ldc + n] = from_f<T>(acc[r]);
    }
}

template <typename T, int M>
int launch_m(const GemvArgs &g0, int trans_b, cudaStream_t stream)
{
    GemvArgs g = g0;
    if (trans_b)
    {
        const size_t smem = (size_t)M * g.k * sizeof(float);
        auto kernel = gemv_nk_kernel<T, M>;
        if (smem > 48 * 1024)
        {
            cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
            if (e != cudaSuccess)
                return set_error(L2K_ERR_CUDA, "l2k_linear (gemv): %s", cudaGetErrorString(e));
        }
        const int64_t grid = ceil_div(g.n, kThreads / 32);
        kernel<<<(unsigned)grid, kThreads, smem, stream>>>(g);
        return check_launch("l2k_linear (gemv)");
    }
    const int64_t col_blocks = ceil_div(g.n, kCols);
    int split;
    size_t smem;
    kn_plan(M, g.n, g.k, &split, &smem);
    g.split = split;
    auto kernel = gemv_kn_kernel<T, M>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear (gemv): %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(col_blocks * split));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, g);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear (gemv): %s", cudaGetErrorString(e));
    return check_launch("l2k_linear (gemv)");
}

template <typename T>
int launch_gemv_t(const GemvArgs &g, int trans_b, cudaStream_t stream)
{
    switch (g.m)
    {
    case 1:
        return launch_m<T, 1>(g, trans_b, stream);
    case 2:
        return launch_m<T, 2>(g, trans_b, stream);
    case 3:
    case 4:
        return launch_m<T, 4>(g, trans_b, stream);
    default:
        return launch_m<T, 8>(g, trans_b, stream);
    }
}

} // namespace

// Whether the few-row path takes this plain GEMM: 16-bit, trans_A false,
// 1..8 rows, B rows 16-byte aligned (K x N layout: ldb and the base; N x K:
// the base), A's rows fit shared memory.
bool gemv_supported(int dtype, int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const void *b,
                    int64_t ldb)
{
    if (!(dtype == L2K_BF16 || dtype == L2K_F16) || trans_a || m < 1 || m > kMaxRows || n < 1 || k < 1)
        return false;
    if (!is_aligned(b, 16) || (ldb * 2) % 16 != 0)
        return false;
    const int64_t rows = m <= 2 ? m : (m <= 4 ? 4 : 8);
    if (trans_b)
        return rows * k * 4 <= 200 * 1024 && n < (int64_t(1) << 31) && k < (int64_t(1) << 31);
    int split;
    size_t smem;
    kn_plan(rows, n, k, &split, &smem);
    return smem <= 200 * 1024 && k < (int64_t(1) << 31) && n < (int64_t(1) << 31);
}

int gemv(int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda, const void *b, int64_t ldb,
         void *c, int64_t ldc, int dtype, cudaStream_t stream)
{
    GemvArgs g{a, lda, b, ldb, c, ldc, (int)m, (int)n, (int)k, 1};
    if (dtype == L2K_BF16)
        return launch_gemv_t<__nv_bfloat16>(g, trans_b, stream);
    return launch_gemv_t<__half>(g, trans_b, stream);
}

int read_gemv_error(bool clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemv_error, sizeof(int)) != cudaSuccess)
        return -1;
    if (clear && v)
    {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_gemv_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

} // namespace l2k
