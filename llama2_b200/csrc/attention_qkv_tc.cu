// P.V on the 5th-generation tensor cores (the qk x v call site of the
// reference's launch_linear, 16-bit I/O, head_dim 128):
//   qkv[b, h, i, :] = sum_{j < n} qk[b, h, i, j] * v[b, h / (Hq/Hkv), j, :],  i < m,
// fp32 accumulation in tensor memory, one rounding to bf16/f16 at the end.
//
// One CTA owns 128 query rows of one (seq, head) and walks the n keys in
// blocks of 64. Per block, TMA brings
//   * the P tile, 128 rows x 64 keys (128-byte rows, 128-byte swizzle): the
//     K-major A operand;
//   * the V tile, 64 keys x 128 head columns as two 64-column boxes: each key
//     row is 128 bytes of head columns, so the tile is the MN-major B operand
//     (swizzle atoms of 8 keys x 128 bytes; SBO = 1024 bytes between 8-key
//     groups, LBO = 8 KB between the two 64-column halves);
// into two rings: P through 5 stages (the HBM stream), V through 2 (its
// tiles are re-read from L2 by the head's other row tiles); 112 KB, two CTAs
// per SM. Two producer threads refill a stage as soon as the MMAs that read
// it complete (tcgen05.commit onto the stage's mbarrier); a third issues
// four 128 x 128 x 16 MMAs per block into a 128-column fp32 accumulator. The tensor maps bound the keys at n and the rows at
// q_cache_len, so keys >= n and rows past the cache read as zeros and are
// never fetched. After the last block the four warps read their 32 TMEM
// lanes (rows) and store rows i < m.
// The kernel is bound by reading P (2 bytes per (row, key)); the MMAs take a
// small share of the tensor pipe (128 x 128 x 64 per 16 KB of P).
// Every mbarrier wait is bounded; on expiry the kernel records an error code
// (l2k_device_error) and leaves after its own copies and MMAs have drained.
//
// Reference: src/kernel/linear.cu:96-128 (cublasGemmBatchedEx over the qk, v
// and qkv pointer arrays of include/kernel/build_q_k_v_qk_qkv_array.h:6-22).
#include "common.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <type_traits>

namespace l2k
{

__device__ int g_pv_error = 0; // first error code recorded by the kernel of this file

namespace
{

constexpr int BM = 128, HD = 128, BK = 64;
constexpr int kThreads = 128;
constexpr int kPStages = 4;                     // P ring: the HBM stream
constexpr int kVStages = 3;                     // V ring: tiles re-read from L2 by the head's row tiles
constexpr uint32_t kPBox = BM * 128;             // 128 rows x 64 keys
constexpr uint32_t kVBox = BK * 128;             // 64 keys x 64 head columns
constexpr uint32_t kVStage = 2 * kVBox;
constexpr uint32_t kOffV = kPStages * kPBox;
constexpr uint32_t kOffBar = kOffV + kVStages * kVStage;
constexpr uint32_t kOffMisc = kOffBar + 128;
constexpr uint32_t kSmemBytes = kOffMisc + 64;   // the dynamic base is 1024-aligned (checked)
constexpr uint32_t kTmemCols = HD;

enum PvError
{
    ERR_PV_WAIT_LOAD = 0x301,
    ERR_PV_WAIT_MMA = 0x302,
    ERR_PV_WAIT_DONE = 0x303,
    ERR_PV_SMEM_ALIGN = 0x304,
    ERR_PV_PAGE = 0x305 // a block-table entry past the page pool (page 0 was read instead)
};

struct PvArgs
{
    void *qkv;
    int64_t Hq, group, Hkv, Qc;
    int64_t m;  // rows written per (seq, head)
    int n_kb;   // key blocks covering [0, n)
    int n_mt;   // row tiles per (seq, head)
    // Paged V cache (null block_table: contiguous): V is (num_pages, Hkv, 64, 128);
    // key block kb of sequence b is page block_table[b * max_pages + kb].
    const uint32_t *block_table;
    const uint32_t *kv_lens;
    int64_t max_pages, num_pages;
};

// MN-major operand, 128-byte swizzle (version 1): LBO = 8 KB between the two
// 64-column halves, SBO = 1024 bytes between 8-key groups.
__device__ __forceinline__ uint64_t smem_desc_mn(uint32_t addr)
{
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)(kVBox >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16, D f32, A and B bf16 (1) or f16 (0), A K-major, B MN-major, M = 128, N = 128.
__host__ __device__ constexpr uint32_t pv_instr_desc(uint32_t ab_format)
{
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (1u << 16) | ((uint32_t)(HD >> 3) << 17) |
           ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void pv_fail(int code, volatile int *abort_flag)
{
    atomicCAS(&g_pv_error, 0, code);
    *abort_flag = 1;
}

template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    attention_qkv_tc_kernel(const __grid_constant__ CUtensorMap tm_p, const __grid_constant__ CUtensorMap tm_v,
                            const PvArgs a)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u)
    {
        if (threadIdx.x == 0)
            atomicCAS(&g_pv_error, 0, ERR_PV_SMEM_ALIGN);
        return;
    }
    const uint32_t bar_pfull = sbase + kOffBar;         // + 8 * P stage: the P tile landed
    const uint32_t bar_pfreed = bar_pfull + 8 * kPStages; // + 8 * P stage: the MMAs reading it completed
    const uint32_t bar_vfull = bar_pfreed + 8 * kPStages; // + 8 * V stage
    const uint32_t bar_vfreed = bar_vfull + 8 * kVStages; // + 8 * V stage
    const uint32_t bar_done = bar_vfreed + 8 * kVStages;  // every MMA completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kOffMisc + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t bh = blockIdx.x / a.n_mt;
    const int mt = (int)(blockIdx.x % a.n_mt);
    const int64_t b = bh / a.Hq, h = bh - b * a.Hq;
    const int64_t row0 = (int64_t)mt * BM;
    const int n_kb = a.n_kb;

    if (tid == 0)
    {
        for (int i = 0; i < kPStages; ++i)
        {
            mbar_init(bar_pfull + 8 * i, 1);
            mbar_init(bar_pfreed + 8 * i, 1);
        }
        for (int i = 0; i < kVStages; ++i)
        {
            mbar_init(bar_vfull + 8 * i, 1);
            mbar_init(bar_vfreed + 8 * i, 1);
        }
        mbar_init(bar_done, 1);
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

    // Producers refill a stage as soon as the MMAs that read it completed.
    int issued = 0; // the calling producer thread's issued blocks
    auto produce = [&](int n_st, uint32_t full, uint32_t freed, uint32_t bytes, auto &&load) {
        for (int kb = 0; kb < n_kb && !*abort_flag; ++kb)
        {
            const int st = kb % n_st;
            if (kb >= n_st && !mbar_wait(freed + 8 * st, ((kb / n_st) - 1) & 1, abort_flag))
            {
                pv_fail(ERR_PV_WAIT_MMA, abort_flag);
                break;
            }
            mbar_expect_tx(full + 8 * st, bytes);
            load(kb, st, full + 8 * st);
            issued = kb + 1;
        }
    };
    if (n_kb > 0 && tid == 0)
    {
        // ---- P producer (warp 0, lane 0): the HBM stream ----
        produce(kPStages, bar_pfull, bar_pfreed, kPBox, [&](int kb, int st, uint32_t bar) {
            tma_load_3d(sbase + st * kPBox, &tm_p, kb * BK, (int)row0, (int)bh, bar);
        });
    }
    else if (n_kb > 0 && tid == 64)
    {
        // ---- V producer (warp 2, lane 0) ----
        const int64_t kvh = h / a.group;
        const int vz = (int)(b * a.Hkv + kvh);
        // Paged: a block wholly past the sequence's length (its table entry may
        // be unset; its probabilities are zero) reads pool page 0 instead.
        const int64_t kvl = a.block_table ? (int64_t)a.kv_lens[b] : 0;
        produce(kVStages, bar_vfull, bar_vfreed, kVStage, [&](int kb, int st, uint32_t bar) {
            const uint32_t dst = sbase + kOffV + st * kVStage;
            if (a.block_table)
            {
                int64_t page = ((int64_t)kb * BK < kvl && kb < a.max_pages) ? a.block_table[b * a.max_pages + kb] : 0;
                if (page >= a.num_pages)
                {
                    atomicCAS(&g_pv_error, 0, ERR_PV_PAGE);
                    page = 0;
                }
                const int pz = (int)(page * a.Hkv + kvh);
                tma_load_3d(dst, &tm_v, 0, 0, pz, bar);
                tma_load_3d(dst + kVBox, &tm_v, BK, 0, pz, bar);
                return;
            }
            tma_load_3d(dst, &tm_v, 0, kb * BK, vz, bar);
            tma_load_3d(dst + kVBox, &tm_v, BK, kb * BK, vz, bar);
        });
    }
    else if (n_kb > 0 && tid == 32)
    {
        // ---- MMA issuer (warp 1, lane 0) ----
        const uint32_t idesc = pv_instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u);
        for (int kb = 0; kb < n_kb && !*abort_flag; ++kb)
        {
            const int ps = kb % kPStages, vs = kb % kVStages;
            if (!mbar_wait(bar_pfull + 8 * ps, (kb / kPStages) & 1, abort_flag) ||
                !mbar_wait(bar_vfull + 8 * vs, (kb / kVStages) & 1, abort_flag))
            {
                pv_fail(ERR_PV_WAIT_LOAD, abort_flag);
                break;
            }
            tc_fence_after();
            const uint32_t pa = sbase + ps * kPBox, vb = sbase + kOffV + vs * kVStage;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) // 16 keys: 32 bytes along the P rows, 2 x 1024 bytes of V key rows
                mma_f16(tmem, smem_desc(pa + 32u * k), smem_desc_mn(vb + 2048u * k), idesc, (kb | k) ? 1u : 0u);
            mma_commit(bar_pfreed + 8 * ps); // the stages are free once these MMAs have read them
            mma_commit(bar_vfreed + 8 * vs);
        }
        mma_commit(bar_done);
    }
    __syncwarp();

    // -------- epilogue: warp w holds rows row0 + 32 w + lane --------
    const int64_t row = row0 + 32 * warp + lane;
    T *out = static_cast<T *>(a.qkv) + (bh * a.Qc + row) * HD;
    const bool store = row < a.m;
    if (n_kb > 0)
    {
        if (!mbar_wait(bar_done, 0, abort_flag))
            pv_fail(ERR_PV_WAIT_DONE, abort_flag);
        tc_fence_after();
        __syncwarp();
        if (!*abort_flag)
        {
#pragma unroll 1
            for (int c0 = 0; c0 < HD; c0 += 32)
            {
                uint32_t r[32];
                tmem_ld32_async(tmem + ((uint32_t)(32 * warp) << 16) + (uint32_t)c0, r);
                tmem_wait_ld();
                if (store)
                {
#pragma unroll
                    for (int v = 0; v < 4; ++v)
                    {
                        uint4 w;
                        w.x = pack2<T>(__uint_as_float(r[8 * v + 0]), __uint_as_float(r[8 * v + 1]));
                        w.y = pack2<T>(__uint_as_float(r[8 * v + 2]), __uint_as_float(r[8 * v + 3]));
                        w.z = pack2<T>(__uint_as_float(r[8 * v + 4]), __uint_as_float(r[8 * v + 5]));
                        w.w = pack2<T>(__uint_as_float(r[8 * v + 6]), __uint_as_float(r[8 * v + 7]));
                        stg(out + c0 + 8 * v, w);
                    }
                }
            }
        }
    }
    else if (store)
    {
        for (int c0 = 0; c0 < HD; c0 += 8)
            stg(out + c0, make_uint4(0u, 0u, 0u, 0u)); // no keys: a zero row
    }

    // -------- teardown --------
    if ((tid == 0 || tid == 64) && *abort_flag)
    {
        // Each producer drains its loads still in flight; thread 0 also the MMAs (each wait bounded).
        const int quiet = 0;
        const int n_st = tid == 0 ? kPStages : kVStages;
        const uint32_t full = tid == 0 ? bar_pfull : bar_vfull;
        for (int kb = std::max(0, issued - n_st); kb < issued; ++kb)
            mbar_wait(full + 8 * (kb % n_st), (kb / n_st) & 1, &quiet);
        if (tid == 0 && n_kb > 0)
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

template <typename T>
int launch_pv_tc(const void *qk, const void *v, void *qkv, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc,
                 int64_t S, int64_t m, int64_t n, const uint32_t *block_table, const uint32_t *kv_lens,
                 int64_t max_pages, int64_t num_pages, cudaStream_t stream)
{
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUtensorMap mp, mv;
    if (!make_map(&mp, dt, qk, (uint64_t)n, (uint64_t)Qc, (uint64_t)(batch * Hq), (uint64_t)S * 2,
                  (uint64_t)(Qc * S * 2), BM, BK) ||
        !(block_table ? make_map(&mv, dt, v, HD, BK, (uint64_t)(num_pages * Hkv), HD * 2, (uint64_t)(BK * HD * 2), BK,
                                 BK)
                      : make_map(&mv, dt, v, HD, (uint64_t)n, (uint64_t)(batch * Hkv), HD * 2,
                                 (uint64_t)(S * HD * 2), BK, BK)))
        return set_error(L2K_ERR_CUDA, "l2k_attention_qkv: tensor map encoding failed");
    PvArgs a{qkv,        Hq,      Hq / Hkv, Hkv,      Qc,       m, (int)ceil_div(n, BK), (int)ceil_div(m, BM),
             block_table, kv_lens, max_pages, num_pages};
    auto kernel = attention_qkv_tc_kernel<T>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e == cudaSuccess) // two CTAs per SM need the whole shared-memory carveout
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_attention_qkv: %s", cudaGetErrorString(e));
    const int64_t grid = (int64_t)a.n_mt * batch * Hq;
    kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(mp, mv, a);
    return check_launch("l2k_attention_qkv (tcgen05)");
}

} // namespace

// Whether the tensor-core path takes this P.V call: 16-bit, head_dim 128,
// 16-byte aligned operands and qk rows (the tensor maps' strides), n >= 1.
bool attention_qkv_tc_supported(int dtype, int64_t head_dim, int64_t S, int64_t n, const void *qk, const void *v,
                                const void *qkv, int64_t grid)
{
    return (dtype == L2K_BF16 || dtype == L2K_F16) && head_dim == HD && S % 8 == 0 && n >= 1 && is_aligned(qk, 16) &&
           is_aligned(v, 16) && is_aligned(qkv, 16) && grid < (int64_t(1) << 31) && S < (int64_t(1) << 31) &&
           encode_fn() != nullptr;
}

int attention_qkv_tc(const void *qk, const void *v, void *qkv, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc,
                     int64_t S, int64_t m, int64_t n, int dtype, cudaStream_t stream, const uint32_t *block_table,
                     const uint32_t *kv_lens, int64_t max_pages, int64_t num_pages)
{
    if (dtype == L2K_BF16)
        return launch_pv_tc<__nv_bfloat16>(qk, v, qkv, batch, Hq, Hkv, Qc, S, m, n, block_table, kv_lens, max_pages,
                                           num_pages, stream);
    return launch_pv_tc<__half>(qk, v, qkv, batch, Hq, Hkv, Qc, S, m, n, block_table, kv_lens, max_pages, num_pages,
                                stream);
}

int read_pv_error(bool clear)
{
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_pv_error, sizeof(int)) != cudaSuccess)
        return -1;
    if (clear && v)
    {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_pv_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    return v;
}

} // namespace l2k
