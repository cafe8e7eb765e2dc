// Row-major GEMM C = A op(B) on the 5th-generation tensor cores, for the
// plain (2-D) launch_linear with 16-bit data and trans_A = false:
//   C[m, n] = sum_k A[m, k] * B'[k, n],  B' = B (K x N) or B^T (B stored N x K),
// fp32 accumulation in tensor memory, one rounding to bf16/f16 at the end.
//
// One CTA computes a 128 x BN tile of C (BN = 256, or 128 for products of at
// most 128 rows), walking K in blocks of 64. Per block TMA brings (128-byte
// swizzle)
//   * the A tile, 128 rows x 64 k: the K-major A operand;
//   * the B tile: with trans_B (B stored N x K) BN rows x 64 k, the K-major
//     B operand; without it (B stored K x N, e.g. a weight [in, out]) 64 k
//     rows x BN columns as 64-column boxes, the MN-major B operand (SBO 1024
//     bytes between 8-row k groups, LBO 8 KB between the 64-column chunks);
// through a ring (2 stages of 48 KB at BN = 256, two CTAs per SM so one
// CTA's epilogue overlaps the other's main loop; 4 stages of 32 KB at
// BN = 128). One thread issues the loads, refilling a stage as soon as the
// MMAs that read it complete; another issues four 128 x BN x 16 MMAs per
// block. The tensor maps bound rows at M, columns at N and k at K, so partial
// tiles read zeros. The four warps then read their 32 TMEM lanes (rows) and
// store the rows' BN columns. Products of one row tile (M <= 128: decode
// batches, bound by reading B) split K over a thread-block cluster of up to
// 8 CTAs that reduce their fp32 rows into rank 0 over distributed shared
// memory.
// Every mbarrier wait is bounded; on expiry the kernel records an error code
// (l2k_device_error) and leaves after its copies and MMAs have drained.
//
// Reference: src/kernel/linear.cu:42-155 (cublasGemmEx with op_A/op_B from
// trans_B/trans_A on the swapped operands; 16-bit data accumulates in 16
// bits there).
#include "common.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <type_traits>

namespace l2k
{

__device__ int g_gemm_error = 0; // first error code recorded by the kernel of this file

namespace
{

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 128;
constexpr uint32_t kABox = BM * 128; // 128 rows x 64 k

// Tile configuration: BN columns of C per CTA, STAGES-deep ring.
template <int BN, int STAGES>
struct Cfg
{
    static constexpr uint32_t kBTile = BN * 128; // BN n x 64 k (either layout)
    static constexpr uint32_t kStageBytes = kABox + kBTile;
    static constexpr uint32_t kOffBar = STAGES * kStageBytes;
    static constexpr uint32_t kOffMisc = kOffBar + 128;
    static constexpr uint32_t kSmemBytes = kOffMisc + 64; // the dynamic base is 1024-aligned (checked)
    static constexpr uint32_t kTmemCols = BN;
    static constexpr int kMinBlocks = (2 * (kSmemBytes + 1024) <= 228 * 1024) ? 2 : 1;
};

enum GemmError
{
    ERR_GEMM_WAIT_LOAD = 0x401,
    ERR_GEMM_WAIT_MMA = 0x402,
    ERR_GEMM_WAIT_DONE = 0x403,
    ERR_GEMM_SMEM_ALIGN = 0x404
};

struct GemmTcArgs
{
    void *c;
    int64_t ldc;
    int64_t m, n;
    int n_kb;   // k blocks
    int n_nt;   // column tiles
    int wide;   // C rows are 16-byte aligned: 16-byte stores
    int split;  // SPLIT: CTAs per cluster sharing one C tile, each a K range
};

// Pushes 4 floats into cluster rank 0's copy of *local_slot (16-byte
// aligned) and signals 16 bytes on rank 0's copy of *local_bar.
__device__ __forceinline__ void push_rank0(const float4 *local_slot, uint32_t local_bar, float4 v)
{
    uint32_t slot, bar;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(slot) : "r"(smem_u32(local_slot)));
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(bar) : "r"(local_bar));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     slot),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
                 : "memory");
}

// MN-major operand, 128-byte swizzle: LBO = 8 KB between the two 64-column
// halves, SBO = 1024 bytes between 8-row k groups.
__device__ __forceinline__ uint64_t desc_mn(uint32_t addr)
{
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((BK * 128) >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, D f32, A and B bf16 (1) or f16 (0), A K-major, B K-major (0) or MN-major (1), M = 128, N = n.
__host__ __device__ constexpr uint32_t gemm_instr_desc(uint32_t ab_format, uint32_t b_mn, uint32_t n)
{
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (b_mn << 16) | ((n >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void gemm_fail(int code, volatile int *abort_flag)
{
    atomicCAS(&g_gemm_error, 0, code);
    *abort_flag = 1;
}

// SPLIT: a cluster of a.split CTAs shares one C tile, each CTA summing a
// contiguous range of the k blocks; once every rank's MMAs are done (cluster
// barrier) ranks 1.. push their fp32 rows into rank 0's idle ring with
// st.async, and rank 0 adds them to its own in rank order and stores.
template <typename T, bool B_MN, int BN, int STAGES, bool SPLIT>
__global__ void __launch_bounds__(kThreads, (Cfg<BN, STAGES>::kMinBlocks))
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const GemmTcArgs a)
{
    using C = Cfg<BN, STAGES>;
    constexpr int kStages = STAGES;
    constexpr uint32_t kStageBytes = C::kStageBytes, kOffBar = C::kOffBar, kOffMisc = C::kOffMisc;
    constexpr uint32_t kTmemCols = C::kTmemCols;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u)
    {
        if (threadIdx.x == 0)
            atomicCAS(&g_gemm_error, 0, ERR_GEMM_SMEM_ALIGN);
        return;
    }
    const uint32_t bar_full = sbase + kOffBar;            // + 8 * stage: the stage's tiles landed
    const uint32_t bar_freed = bar_full + 8 * kStages;    // + 8 * stage: the MMAs reading it completed
    const uint32_t bar_done = bar_freed + 8 * kStages;    // every MMA completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kOffMisc + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = SPLIT ? a.split : 1;
    const int rank = SPLIT ? (int)(blockIdx.x % split) : 0;
    const int tile = (int)(blockIdx.x / split);
    const int mt = tile / a.n_nt, nt = tile % a.n_nt;
    const int row0 = mt * BM, col0 = nt * BN;
    // this CTA's k blocks: [kb0, kb0 + n_kb)
    const int kb0 = (int)((int64_t)rank * a.n_kb / split);
    const int n_kb = (int)((int64_t)(rank + 1) * a.n_kb / split) - kb0;
    const uint32_t bar_red = bar_done + 8; // SPLIT, rank 0: the peers' rows have landed

    if (tid == 0)
    {
        for (int i = 0; i < kStages; ++i)
        {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_freed + 8 * i, 1);
        }
        mbar_init(bar_done, 1);
        if (SPLIT)
            mbar_init(bar_red, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 0)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int issued = 0; // producer thread: k blocks whose loads were issued
    if (n_kb > 0 && tid == 0)
    {
        // ---- producer (warp 0, lane 0) ----
        for (int kb = 0; kb < n_kb && !*abort_flag; ++kb)
        {
            const int st = kb % kStages;
            if (kb >= kStages && !mbar_wait(bar_freed + 8 * st, ((kb / kStages) - 1) & 1, abort_flag))
            {
                gemm_fail(ERR_GEMM_WAIT_MMA, abort_flag);
                break;
            }
            const uint32_t dst = sbase + st * kStageBytes;
            const uint32_t bar = bar_full + 8 * st;
            mbar_expect_tx(bar, kStageBytes);
            const int kx = (kb0 + kb) * BK;
            tma_load_3d(dst, &tm_a, kx, row0, 0, bar);
            if constexpr (B_MN)
            {
#pragma unroll
                for (int h = 0; h < BN / 64; ++h)
                    tma_load_3d(dst + kABox + h * BK * 128, &tm_b, col0 + 64 * h, kx, 0, bar);
            }
            else
                tma_load_3d(dst + kABox, &tm_b, kx, col0, 0, bar);
            issued = kb + 1;
        }
    }
    else if (n_kb > 0 && tid == 32)
    {
        // ---- MMA issuer (warp 1, lane 0) ----
        const uint32_t idesc =
            gemm_instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, B_MN ? 1u : 0u, (uint32_t)BN);
        for (int kb = 0; kb < n_kb && !*abort_flag; ++kb)
        {
            const int st = kb % kStages;
            if (!mbar_wait(bar_full + 8 * st, (kb / kStages) & 1, abort_flag))
            {
                gemm_fail(ERR_GEMM_WAIT_LOAD, abort_flag);
                break;
            }
            tc_fence_after();
            const uint32_t pa = sbase + st * kStageBytes, pb = pa + kABox;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
            {
                // 16 k: 32 bytes along the K-major rows, or 2 x 1024 bytes of MN-major k rows
                const uint64_t bd = B_MN ? desc_mn(pb + 2048u * k) : smem_desc(pb + 32u * k);
                mma_f16(tmem, smem_desc(pa + 32u * k), bd, idesc, (kb | k) ? 1u : 0u);
            }
            mma_commit(bar_freed + 8 * st); // the stage is free once these MMAs have read it
        }
        mma_commit(bar_done);
    }
    __syncwarp();

    // -------- epilogue: warp w holds rows row0 + 32 w + lane --------
    const int64_t row = row0 + 32 * warp + lane;
    T *out = static_cast<T *>(a.c) + row * a.ldc;
    const bool store = row < a.m;
    const bool wide = a.wide != 0;
    const int lrow = 32 * warp + lane;          // row within the tile
    float *red = reinterpret_cast<float *>(smem); // SPLIT, rank 0: [split - 1][m][BN] peer rows (in the idle ring)
    const int m_tile = (int)min((int64_t)BM, a.m - row0);
    if (n_kb > 0)
    {
        if (!mbar_wait(bar_done, 0, abort_flag))
            gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
        tc_fence_after();
        __syncwarp();
        if constexpr (SPLIT)
        {
            // every rank's MMAs are done: rank 0's ring may take the peers' rows
            asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
            asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
            if (rank == 0 && tid == 0)
                mbar_expect_tx(bar_red, (uint32_t)((split - 1) * m_tile * BN * (int)sizeof(float)));
            if (rank != 0)
            {
#pragma unroll 1
                for (int c0 = 0; c0 < BN; c0 += 32)
                {
                    uint32_t r[32];
                    tmem_ld32_async(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, r);
                    tmem_wait_ld();
                    if (lrow < m_tile && !*abort_flag)
                    {
                        const float4 *dst =
                            reinterpret_cast<const float4 *>(red + ((int64_t)(rank - 1) * m_tile + lrow) * BN + c0);
#pragma unroll
                        for (int v = 0; v < 8; ++v)
                            push_rank0(dst + v, bar_red,
                                       make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                   __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3])));
                    }
                }
            }
            else
            {
                // (also after a failure: the peers' rows land before this CTA leaves)
                if (!mbar_wait(bar_red, 0, abort_flag))
                    gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
            }
        }
        if (!*abort_flag && (!SPLIT || rank == 0))
        {
#pragma unroll 1
            for (int c0 = 0; c0 < BN; c0 += 32)
            {
                uint32_t r[32];
                tmem_ld32_async(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, r);
                tmem_wait_ld();
                if (!store)
                    continue;
                if constexpr (SPLIT)
                {
                    for (int p = 1; p < split; ++p)
                    {
                        const float *src = red + ((int64_t)(p - 1) * m_tile + lrow) * BN + c0;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            r[j] = __float_as_uint(__uint_as_float(r[j]) + src[j]);
                    }
                }
#pragma unroll
                for (int v = 0; v < 4; ++v)
                {
                    const int64_t col = (int64_t)col0 + c0 + 8 * v;
                    if (col >= a.n)
                        break;
                    uint4 w;
                    w.x = pack2<T>(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
                    w.y = pack2<T>(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
                    w.z = pack2<T>(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
                    w.w = pack2<T>(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
                    if (wide && col + 8 <= a.n)
                        stg(out + col, w);
                    else
                    {
                        const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
                        for (int e = 0; e < 8 && col + e < a.n; ++e)
                        {
                            const uint16_t bits = (uint16_t)(e & 1 ? (w4[e / 2] >> 16) : (w4[e / 2] & 0xFFFF));
                            reinterpret_cast<uint16_t *>(out)[col + e] = bits;
                        }
                    }
                }
            }
        }
    }
    else if (store)
    {
        for (int64_t col = col0; col < min((int64_t)col0 + BN, a.n); ++col)
            out[col] = from_f<T>(0.f); // K = 0: a zero tile
    }

    // -------- teardown --------
    if (tid == 0 && *abort_flag)
    {
        const int quiet = 0;
        for (int kb = std::max(0, issued - kStages); kb < issued; ++kb)
            mbar_wait(bar_full + 8 * (kb % kStages), (kb / kStages) & 1, &quiet);
        if (n_kb > 0)
            mbar_wait(bar_done, 0, &quiet);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

template <typename T, bool B_MN, int BN, int STAGES, bool SPLIT = false>
int launch_gemm_tc(const void *A, int64_t lda, const void *B, int64_t ldb, void *C, int64_t ldc, int64_t m,
                   int64_t n, int64_t k, cudaStream_t stream, int split = 1)
{
    constexpr uint32_t kSmemBytes = Cfg<BN, STAGES>::kSmemBytes;
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap ma, mb;
    bool ok = make_map(&ma, dt, A, (uint64_t)k, (uint64_t)m, 1, (uint64_t)lda * 2, (uint64_t)(lda * 2 * m), BM, BK);
    if (B_MN) // B stored K x N: boxes of 64 k rows x 64 columns
        ok = ok && make_map(&mb, dt, B, (uint64_t)n, (uint64_t)k, 1, (uint64_t)ldb * 2, (uint64_t)(ldb * 2 * k), BK,
                            64);
    else // B stored N x K: boxes of BN n rows x 64 k
        ok = ok && make_map(&mb, dt, B, (uint64_t)k, (uint64_t)n, 1, (uint64_t)ldb * 2, (uint64_t)(ldb * 2 * n), BN,
                            BK);
    if (!ok)
        return set_error(L2K_ERR_CUDA, "l2k_linear: tensor map encoding failed");
    GemmTcArgs a{C, ldc, m, n, (int)ceil_div(k, BK), (int)ceil_div(n, BN),
                 (ldc * 2) % 16 == 0 && is_aligned(C, 16) ? 1 : 0, split};
    auto kernel = gemm_tc_kernel<T, B_MN, BN, STAGES, SPLIT>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e == cudaSuccess) // two CTAs per SM need the whole shared-memory carveout
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear: %s", cudaGetErrorString(e));
    const int64_t grid = ceil_div(m, BM) * a.n_nt * split;
    if (!SPLIT)
    {
        kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(ma, mb, a);
        return check_launch("l2k_linear (tcgen05)");
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)split;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, a);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear (split k): %s", cudaGetErrorString(e));
    return check_launch("l2k_linear (tcgen05, split k)");
}

} // namespace

// Whether the tensor-core path takes this plain GEMM: 16-bit, trans_A false,
// 16-byte aligned bases and row strides (the tensor maps), sizes in range.
bool gemm_tc_supported(int dtype, int trans_a, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda,
                       const void *b, int64_t ldb, const void *c)
{
    return (dtype == L2K_BF16 || dtype == L2K_F16) && !trans_a && m >= 1 && n >= 1 && k >= 1 && is_aligned(a, 16) &&
           is_aligned(b, 16) && is_aligned(c, 2) && (lda * 2) % 16 == 0 && (ldb * 2) % 16 == 0 &&
           ceil_div(m, BM) * ceil_div(n, 128) < (int64_t(1) << 31) && m < (int64_t(1) << 31) &&
           n < (int64_t(1) << 31) && k < (int64_t(1) << 31) && encode_fn() != nullptr;
}

// Tile shape by M: above 128 rows, 128 x 256 tiles (N = 256 MMAs read half
// the A operand per FLOP from shared memory) in a 2-stage ring, two CTAs per
// SM; up to 128 rows (decode-sized products, bound by reading B), 128 x 128
// tiles for twice the CTAs, in a 4-stage ring.
template <typename T, bool B_MN>
int launch_tiles(const void *a, int64_t lda, const void *b, int64_t ldb, void *c, int64_t ldc, int64_t m, int64_t n,
                 int64_t k, cudaStream_t stream)
{
    if (m > BM)
        return launch_gemm_tc<T, B_MN, 256, 2>(a, lda, b, ldb, c, ldc, m, n, k, stream);
    // One row tile: too few CTAs to stream B at full bandwidth unless K is
    // split across a cluster (the peers' fp32 rows must fit rank 0's ring).
    constexpr int kSplitStages = 3;
    const int64_t tiles = ceil_div(n, 128), n_kb = ceil_div(k, BK);
    const int64_t ring = (int64_t)kSplitStages * Cfg<128, kSplitStages>::kStageBytes;
    int split = 1;
    while (split < 8 && tiles * split * 2 <= 2LL * num_sms() && split * 2 <= n_kb &&
           (int64_t)(split * 2 - 1) * m * 128 * 4 <= ring)
        split *= 2;
    if (split > 1)
        return launch_gemm_tc<T, B_MN, 128, kSplitStages, true>(a, lda, b, ldb, c, ldc, m, n, k, stream, split);
    return launch_gemm_tc<T, B_MN, 128, 4>(a, lda, b, ldb, c, ldc, m, n, k, stream);
}

int gemm_tc(int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda, const void *b, int64_t ldb,
            void *c, int64_t ldc, int dtype, cudaStream_t stream)
{
    if (dtype == L2K_BF16)
        return trans_b ? launch_tiles<__nv_bfloat16, false>(a, lda, b, ldb, c, ldc, m, n, k, stream)
                       : launch_tiles<__nv_bfloat16, true>(a, lda, b, ldb, c, ldc, m, n, k, stream);
    return trans_b ? launch_tiles<__half, false>(a, lda, b, ldb, c, ldc, m, n, k, stream)
                   : launch_tiles<__half, true>(a, lda, b, ldb, c, ldc, m, n, k, stream);
}

int read_gemm_error(bool clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_gemm_error, sizeof(int)) != cudaSuccess)
        return -1;
    if (clear && v)
    {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_gemm_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

} // namespace l2k
