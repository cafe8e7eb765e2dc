// Fused prefill attention scores on the 5th-generation tensor cores:
//   P = softmax_causal(Q K^T / sqrt(128)),  bf16/f16 in, fp32 accumulate, bf16/f16 out.
//
// One CTA owns 128 query rows of one (seq, head); key tiles are 128 wide, so
// each tcgen05.mma is 128 x 128 x 16 (wide enough to keep the tensor pipe
// efficient; two CTAs per SM still fit: 112 KB of shared memory, 256 TMEM
// columns each).
// Warp roles (320 threads):
//   * warp 9 (producer): TMA (cp.async.bulk.tensor, 128-byte swizzle) of the
//     Q tile once and of K tiles (2 x 16 KB boxes) through a 2-stage ring,
//     each stage refilled as soon as the MMAs that read it have completed
//     (tcgen05.commit onto the stage's "empty" mbarrier);
//   * warp 8 (MMA): tcgen05.mma with both operands in shared memory and the
//     fp32 accumulator in tensor memory (2 x 128 columns, double buffered),
//     issued back to back as K stages and TMEM buffers become available;
//     tcgen05.commit signals "tile ready" on an mbarrier.
//   * warps 0-7 (epilogue): warp w reads TMEM lanes 32*(w%4).. (its rows) and
//     columns 64*(w/4).. of each tile (two tcgen05.ld of 32 columns).
//     Phase A walks the causally visible key tiles keeping an online row max
//     and sum of exponentials (log2 units, ex2); phase B re-runs the MMAs
//     and writes P = 2^(s*c - m - log2(sum + 1e-6)) once: each warp transposes
//     its 32 x 32 blocks through 2 KB of shared memory (64-byte swizzle) and
//     writes them with coalesced 16-byte stores (64 contiguous bytes per row).
//     Each tile frees its TMEM buffer through an mbarrier as soon as it is in
//     registers, so the MMA of the next tile overlaps.
//   * Key columns beyond the causal limit are TMA-stored (128 x 64 boxes)
//     from the zeroed staging region at the start, overlapping phase A. Keys
//     >= max_kv are never written (the store map's extent; its 16-byte-rounded
//     tail is written directly); tiles whose rows straddle q_len write only
//     their valid rows.
// CTA order is (seq, head)-major so the query tiles of one head run together
// and share its K tiles in L2.
// Every mbarrier wait is bounded (~2 s of clock cycles); on expiry the kernel
// records an error code (l2k_device_error) and leaves after draining its own
// copies, so a defect shows up as an error, not a hung GPU.
//
// Reference composition: cuBLAS QK^T (src/kernel/linear.cu:96-128) + masked
// softmax (src/kernel/compute_masked_attention_score.cu:12-103) with the mask
// k <= kv_len - q_len + q.
#include "common.cuh"
#include "tcgen05.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <type_traits>

namespace l2k
{

__device__ int g_device_error = 0; // first error code recorded by a kernel of this file

namespace
{

constexpr int BM = 128, BN = 128, HD = 128, KH = 64; // KH: elements per 128-byte swizzle row
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (kEpiWarps + 2);
constexpr int kCtl = kEpiWarps;                        // MMA warp index
constexpr int kProd = kEpiWarps + 1;                   // producer warp index
constexpr int kColGroups = kEpiWarps / 4;              // epilogue warps per TMEM lane quadrant
constexpr int kColsPerWarp = BN / kColGroups;          // 64
constexpr uint32_t kQBox = 128 * 128;                  // 128 rows x 128 B
constexpr uint32_t kKBox = BN * 128;                   // 128 rows x 128 B
constexpr int kKStages = 2;                            // K ring depth (32 KB per stage)
constexpr uint32_t kWarpStage = 32 * 64;               // one warp's 32 x 32 block of P (64-byte rows)
constexpr uint32_t kOffQ = 0;                          // 2 boxes (hd halves)
constexpr uint32_t kOffK = kOffQ + 2 * kQBox;          // kKStages stages x 2 boxes
constexpr uint32_t kOffP = kOffK + kKStages * 2 * kKBox; // 8 warp blocks; the zeroed 128 x 64 box at the start;
                                                       // the phase-A statistics at its end
constexpr uint32_t kOffBar = kOffP + kEpiWarps * kWarpStage; // mbarriers
constexpr uint32_t kOffMisc = kOffBar + 128;           // tmem slot, abort flag
constexpr uint32_t kSmemBytes = kOffMisc + 64;         // the dynamic base is 1024-aligned (checked)
constexpr uint32_t kTmemCols = 2 * BN;
static_assert(kColGroups * 128 * 8 <= kEpiWarps * kWarpStage, "statistics fit the staging region");
constexpr float kNegBig = -1e30f;

enum DevError
{
    ERR_WAIT_Q = 0x101,
    ERR_WAIT_K = 0x102,
    ERR_WAIT_MMA = 0x103,
    ERR_WAIT_TMEM = 0x104,
    ERR_SMEM_ALIGN = 0x105,
    ERR_PAGE = 0x106 // a block-table entry past the page pool (page 0 was read instead)
};

constexpr int kPageRows = 64; // rows of one page of a paged K cache: 16 KB of 128 x 16-bit rows

struct TcArgs
{
    const uint32_t *q_lens;
    const uint32_t *kv_lens;
    void *qk;
    int64_t Hq, group, Hkv, Qc, S;
    int64_t M;     // keys written per row: min(max_kv, S)
    int64_t M8;    // keys written by TMA stores: M rounded down to 8 (16 bytes)
    int n_qt;      // query tiles per (seq, head)
    int n_kt;      // key tiles covering [0, M)
    float c;       // scale * log2(e)
    // Paged K cache (null block_table: contiguous): K is (num_pages, Hkv, 64, 128);
    // keys [64 j, 64 j + 64) of sequence b are page block_table[b * max_pages + j].
    const uint32_t *block_table;
    int64_t max_pages, num_pages;
};

// ---------------------------------------------------------------------------
// Kernel-local helpers (the shared tcgen05 / TMA wrappers are in tcgen05.cuh)
// ---------------------------------------------------------------------------
// Named barrier among the epilogue warps only.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory"); }

// kind::f16 instruction descriptor: D f32, A/B bf16 (1) or f16 (0), both K-major, M=128, N=n.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t ab_format, uint32_t n)
{
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((n >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ uint16_t half_of(uint32_t w, int hi) { return (uint16_t)(hi ? (w >> 16) : (w & 0xFFFF)); }

__device__ __forceinline__ void fail(int code, volatile int *abort_flag)
{
    atomicCAS(&g_device_error, 0, code);
    *abort_flag = 1;
}

// ---------------------------------------------------------------------------
// The kernel
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(kThreads, 2)
    prefill_scores_tc_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                             const __grid_constant__ CUtensorMap tm_p, const TcArgs a)
{
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u)
    {
        // the 128-byte-swizzled TMA boxes need a 1024-byte aligned base
        if (threadIdx.x == 0)
            atomicCAS(&g_device_error, 0, ERR_SMEM_ALIGN);
        return;
    }
    const uint32_t bar_q = sbase + kOffBar;
    const uint32_t bar_kfull = bar_q + 8;    // + 8 * stage (kKStages)
    const uint32_t bar_mma = bar_q + 32;     // + 8 * buffer: tile in TMEM buffer is ready
    const uint32_t bar_tfree = bar_q + 48;   // + 8 * buffer: epilogue finished with TMEM buffer
    const uint32_t bar_kempty = bar_q + 64;  // + 8 * stage: the MMAs reading the K stage completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kOffMisc + 8);
    float2 *stats = reinterpret_cast<float2 *>(smem + kOffP); // [kColGroups][128], after the zero stores

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t bh = blockIdx.x / a.n_qt;
    const int qt = a.n_qt - 1 - (int)(blockIdx.x % a.n_qt);
    const int64_t b = bh / a.Hq, h = bh - b * a.Hq;
    const int64_t kvh = h / a.group;
    const int64_t q_len = a.q_lens[b];
    const int64_t kv_len = min((int64_t)a.kv_lens[b], a.S);
    const int64_t hist = kv_len - q_len;
    const int64_t row0 = (int64_t)qt * BM;
    if (row0 >= q_len)
        return; // no output rows in this tile (uniform over the CTA)
    const int rows_valid = (int)min((int64_t)BM, q_len - row0);
    // Zero columns go out as TMA stores of whole 128-row boxes; that map covers keys [0, M8).
    const bool full_rows = rows_valid == BM && a.M8 > 0;
    const int64_t max_lim = min(kv_len - 1, hist + row0 + rows_valid - 1);
    const int64_t min_lim = min(kv_len - 1, hist + row0);
    const int n_a = max_lim >= 0 ? (int)min((int64_t)a.n_kt, max_lim / BN + 1) : 0;
    const int n_steps = 2 * n_a;

    // -------- setup --------
    if (tid == 0)
    {
        mbar_init(bar_q, 1);
        for (int i = 0; i < kKStages; ++i)
            mbar_init(bar_kfull + 8 * i, 1);
        for (int i = 0; i < 2; ++i)
        {
            mbar_init(bar_mma + 8 * i, 1);
            mbar_init(bar_tfree + 8 * i, kEpiWarps);
        }
        for (int i = 0; i < kKStages; ++i)
            mbar_init(bar_kempty + 8 * i, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == kCtl)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    {
        // the staging region starts zeroed: the source of the zero-column stores
        uint4 *z = reinterpret_cast<uint4 *>(smem + kOffP);
        for (int i = tid; i < (int)(kEpiWarps * kWarpStage / 16); i += kThreads)
            z[i] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kProd)
    {
        // ================= producer warp =================
        if (lane == 0 && n_steps > 0)
        {
            const int kz = (int)(b * a.Hkv + kvh);
            // Paged: the tile's two 64-key pages. A page wholly past the
            // sequence's length (its table entry may be unset) is replaced by
            // the tile's first page: those keys are masked for every row.
            auto page_z = [&](int kt, int half) -> int {
                int64_t j = 2 * (int64_t)kt + half;
                if (j * kPageRows >= kv_len || j >= a.max_pages)
                    j = 2 * (int64_t)kt;
                int64_t page = a.block_table[b * a.max_pages + j];
                if (page >= a.num_pages)
                {
                    atomicCAS(&g_device_error, 0, ERR_PAGE);
                    page = 0;
                }
                return (int)(page * a.Hkv + kvh);
            };
            auto issue_k = [&](int t) {
                const int kt = t % n_a, st = t % kKStages;
                const uint32_t dst = sbase + kOffK + st * 2 * kKBox;
                mbar_expect_tx(bar_kfull + 8 * st, 2 * kKBox);
                if (a.block_table)
                {
                    const int z0 = page_z(kt, 0), z1 = page_z(kt, 1);
                    for (int hf = 0; hf < 2; ++hf)
                    {
                        tma_load_3d(dst + hf * kKBox, &tm_k, hf * KH, 0, z0, bar_kfull + 8 * st);
                        tma_load_3d(dst + hf * kKBox + kKBox / 2, &tm_k, hf * KH, 0, z1, bar_kfull + 8 * st);
                    }
                    return;
                }
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_3d(dst + hf * kKBox, &tm_k, hf * KH, kt * BN, kz, bar_kfull + 8 * st);
            };
            mbar_expect_tx(bar_q, 2 * kQBox);
            for (int hf = 0; hf < 2; ++hf)
                tma_load_3d(sbase + kOffQ + hf * kQBox, &tm_q, hf * KH, (int)row0, (int)bh, bar_q);
            for (int t = 0; t < n_steps && !*abort_flag; ++t)
            {
                const int ks = t % kKStages;
                if (t >= kKStages && !mbar_wait(bar_kempty + 8 * ks, ((t / kKStages) - 1) & 1, abort_flag))
                {
                    fail(ERR_WAIT_MMA, abort_flag);
                    break;
                }
                issue_k(t);
            }
        }
    }
    else if (warp == kCtl)
    {
        // ================= MMA warp =================
        if (lane == 0 && n_steps > 0)
        {
            const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
            const uint32_t idesc_full = instr_desc(fmt, BN), idesc_half = instr_desc(fmt, BN / 2);
            if (!mbar_wait(bar_q, 0, abort_flag))
                fail(ERR_WAIT_Q, abort_flag);
            for (int t = 0; t < n_steps && !*abort_flag; ++t)
            {
                const int st = t & 1, ks = t % kKStages; // TMEM buffer, K stage
                const int kt = t % n_a;
                if (!mbar_wait(bar_kfull + 8 * ks, (t / kKStages) & 1, abort_flag))
                {
                    fail(ERR_WAIT_K, abort_flag);
                    break;
                }
                if (t >= 2 && !mbar_wait(bar_tfree + 8 * st, ((t >> 1) - 1) & 1, abort_flag))
                {
                    fail(ERR_WAIT_TMEM, abort_flag);
                    break;
                }
                tc_fence_after();
                const uint32_t kb = sbase + kOffK + ks * 2 * kKBox;
                const uint32_t d = tmem + (uint32_t)(st * BN);
                // keys [BN/2, BN) of the tile masked for every row: half-width MMAs
                const uint32_t idesc = max_lim < (int64_t)kt * BN + BN / 2 ? idesc_half : idesc_full;
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                {
                    const uint32_t offa = (uint32_t)((k & 3) * 32) + (uint32_t)(k >> 2) * kQBox;
                    const uint32_t offb = (uint32_t)((k & 3) * 32) + (uint32_t)(k >> 2) * kKBox;
                    mma_f16(d, smem_desc(sbase + kOffQ + offa), smem_desc(kb + offb), idesc, k > 0 ? 1u : 0u);
                }
                mma_commit(bar_mma + 8 * st);    // the tile is in TMEM
                mma_commit(bar_kempty + 8 * ks); // the K stage may be refilled
            }
        }
    }
    else
    {
        // ================= epilogue warps =================
        const int quad = warp & 3, cg = warp >> 2; // TMEM lanes 32*quad.., columns 64*cg..
        const int r = quad * 32 + lane;            // row within the tile
        const int64_t lim_r = min(kv_len - 1, hist + row0 + r);
        float m = kNegBig, l = 0.f;                // log2-domain running max / sum
        uint16_t *qk16 = static_cast<uint16_t *>(a.qk);
        const int64_t row_off = (bh * a.Qc + row0 + r) * a.S;
        uint8_t *wst = smem + kOffP + (uint32_t)warp * kWarpStage; // this warp's transpose buffer

        if (tid == 0 && full_rows)
        {
            // zero columns beyond the causal limit, 128 x 64 boxes from the zeroed region
            for (int64_t x = (int64_t)n_a * BN; x < a.M; x += KH)
                tma_store_3d(&tm_p, sbase + kOffP, (int)x, (int)row0, (int)bh);
            bulk_commit();
        }

        for (int t = 0; t < n_steps; ++t)
        {
            const int st = t & 1;
            // After a failure the remaining steps run on whatever TMEM holds (the
            // error is recorded); no warp leaves early, so the named barrier below
            // is met by all epilogue warps.
            if (!mbar_wait(bar_mma + 8 * st, (t >> 1) & 1, abort_flag))
                fail(ERR_WAIT_MMA, abort_flag);
            tc_fence_after();
            const bool phase_b = t >= n_a;
            const int kt = phase_b ? t - n_a : t;
            const int64_t key0 = (int64_t)kt * BN + cg * kColsPerWarp;
            uint32_t raw0[32], raw1[32];
            const uint32_t taddr = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(st * BN + cg * kColsPerWarp);
            tmem_ld32_async(taddr, raw0);
            tmem_ld32_async(taddr + 32, raw1);
            tmem_wait_ld();
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(bar_tfree + 8 * st); // the TMEM buffer may take the next tile
            float v[64];
#pragma unroll
            for (int j = 0; j < 32; ++j)
            {
                v[j] = __uint_as_float(raw0[j]);
                v[32 + j] = __uint_as_float(raw1[j]);
            }
            // live[hh]: some row of this warp sees a key of columns [32 hh, 32 hh + 32);
            // a half no row sees is all -inf and adds nothing to the statistics.
            bool live[2] = {true, true};
            if ((int64_t)kt * BN + BN - 1 > min_lim)
            {
                // keys past this row's limit (tile-uniform test, 32-bit compares)
                const int64_t vis64 = lim_r - key0 + 1;
                const int vis = (int)max((int64_t)0, min((int64_t)64, vis64));
#pragma unroll
                for (int j = 0; j < 64; ++j)
                    v[j] = j < vis ? v[j] : -INFINITY;
                live[0] = __any_sync(0xffffffffu, vis > 0);
                live[1] = __any_sync(0xffffffffu, vis > 32);
            }
            if (!phase_b)
            {
                float tmax = -INFINITY;
#pragma unroll
                for (int j = 0; j < 64; ++j)
                    tmax = fmaxf(tmax, v[j]);
                const float m_new = fmaxf(m, tmax * a.c);
                float sum0 = 0.f, sum1 = 0.f;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh)
                {
                    if (!live[hh])
                        continue; // (its terms are exact zeros: the sums do not change)
#pragma unroll
                    for (int j = 32 * hh; j < 32 * hh + 32; j += 2)
                    {
                        sum0 += ex2(fmaf(v[j], a.c, -m_new));
                        sum1 += ex2(fmaf(v[j + 1], a.c, -m_new));
                    }
                }
                l = l * ex2(m - m_new) + (sum0 + sum1);
                m = m_new;
                if (t == n_a - 1)
                {
                    // The statistics go to the staging region once the zero-column
                    // stores have read it.
                    if (tid == 0)
                        bulk_wait_read_0();
                    epi_sync();
                    stats[cg * 128 + r] = make_float2(m, l);
                    epi_sync();
                    float Mx = stats[r].x;
#pragma unroll
                    for (int g = 1; g < kColGroups; ++g)
                        Mx = fmaxf(Mx, stats[g * 128 + r].x);
                    float L = 0.f;
#pragma unroll
                    for (int g = 0; g < kColGroups; ++g)
                    {
                        const float2 sg = stats[g * 128 + r];
                        L += sg.y * ex2(sg.x - Mx);
                    }
                    // phase B: p = 2^(s*c - m) / (L + eps) = 2^(s*c - (m + log2(L + eps)))
                    m = __fadd_rn(Mx, log2f(__fadd_rn(L, 1e-6f)));
                    epi_sync(); // every row's statistics read before the region becomes staging again
                }
                continue;
            }
#pragma unroll
            for (int hh = 0; hh < 2; ++hh)
            {
                uint32_t packed[16];
#pragma unroll
                for (int j = 0; j < 32; j += 2)
                    packed[j / 2] = pack2<T>(ex2(fmaf(v[hh * 32 + j], a.c, -m)), ex2(fmaf(v[hh * 32 + j + 1], a.c, -m)));
                // Transpose this 32 x 32 block through shared memory: lane = row,
                // 16-byte chunk c of a row at c ^ ((row / 2) % 4) (conflict-free both ways),
                // then each store instruction writes 8 rows x 64 contiguous bytes.
                __syncwarp(); // the previous block has been read back
                uint8_t *mine = wst + (uint32_t)lane * 64;
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
                    *reinterpret_cast<uint4 *>(mine + ((c4 ^ ((lane >> 1) & 3)) * 16)) =
                        make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2], packed[4 * c4 + 3]);
                __syncwarp();
                const int64_t col0 = key0 + hh * 32;
#pragma unroll
                for (int i = 0; i < 4; ++i)
                {
                    const int rr = i * 8 + (lane >> 2), c = lane & 3;
                    const uint4 val = *reinterpret_cast<const uint4 *>(wst + rr * 64 + ((c ^ ((rr >> 1) & 3)) * 16));
                    const int row = quad * 32 + rr;
                    const int64_t col = col0 + c * 8;
                    if (row < rows_valid && col < a.M)
                    {
                        uint16_t *dst = qk16 + (bh * a.Qc + row0 + row) * a.S + col;
                        if (col + 8 <= a.M)
                            *reinterpret_cast<uint4 *>(dst) = val;
                        else
                        {
                            const uint32_t w4[4] = {val.x, val.y, val.z, val.w};
#pragma unroll
                            for (int e = 0; e < 8; ++e)
                                if (col + e < a.M)
                                    dst[e] = half_of(w4[e / 2], e & 1);
                        }
                    }
                }
            }
        }

        // Zero tails: keys [M8, M) beyond the zero-column stores' map, and every
        // zero key of tiles whose rows straddle q_len.
        if (full_rows && a.M8 < a.M && (int64_t)n_a * BN < a.M)
        {
            for (int64_t j = max(a.M8, (int64_t)n_a * BN) + cg; j < a.M; j += kColGroups)
                qk16[row_off + j] = 0;
        }
        if (!full_rows && r < rows_valid)
        {
            for (int64_t j = (int64_t)n_a * BN + cg; j < a.M; j += kColGroups)
                qk16[row_off + j] = 0;
        }
        if (tid == 0)
            bulk_wait_all(); // the zero-column stores
    }

    // -------- teardown --------
    if (warp == kCtl && lane == 0 && *abort_flag)
    {
        // Drain whatever this CTA may still have in flight, each wait bounded.
        const int quiet = 0; // these waits must not stop early on the abort flag
        for (int i = 0; i < kKStages; ++i)
            mbar_wait(bar_kfull + 8 * i, 0, &quiet);
        for (int i = 0; i < 2; ++i)
            mbar_wait(bar_mma + 8 * i, 0, &quiet);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == kCtl)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
    }
}

// ---------------------------------------------------------------------------
// Host side: launch
// ---------------------------------------------------------------------------
template <typename T>
int launch_tc(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens, uint32_t max_q,
              uint32_t max_kv, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc, int64_t S,
              const uint32_t *block_table, int64_t max_pages, int64_t num_pages, cudaStream_t stream)
{
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int64_t M = std::min<int64_t>(max_kv, S);
    CUtensorMap mq, mk, mp;
    const int64_t m8 = std::max<int64_t>(M & ~int64_t(7), 8);
    const bool kmap = block_table ? make_map(&mk, dt, k, HD, kPageRows, num_pages * Hkv, HD * 2,
                                             kPageRows * HD * 2, kPageRows)
                                  : make_map(&mk, dt, k, HD, S, batch * Hkv, HD * 2, S * HD * 2, BN);
    if (!make_map(&mq, dt, q, HD, Qc, batch * Hq, HD * 2, Qc * HD * 2, BM) || !kmap ||
        !make_map(&mp, dt, qk, m8, Qc, batch * Hq, S * 2, Qc * S * 2, BM))
        return set_error(L2K_ERR_CUDA, "l2k_prefill_attention_scores: tensor map encoding failed");
    // c = (1/sqrtf(128)) * log2(e): the oracle's fp32 scale, moved to base 2 for ex2.
    TcArgs a{q_lens, kv_lens, qk, Hq, Hq / Hkv, Hkv, Qc, S, M, M & ~int64_t(7), (int)ceil_div(max_q, BM),
             (int)ceil_div(M, BN), (1.f / sqrtf((float)HD)) * 1.44269504088896340736f, block_table, max_pages,
             num_pages};
    auto kernel = prefill_scores_tc_kernel<T>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_prefill_attention_scores: %s", cudaGetErrorString(e));
    const int64_t grid = (int64_t)a.n_qt * batch * Hq;
    kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(mq, mk, mp, a);
    return check_launch("l2k_prefill_attention_scores (tcgen05)");
}

} // namespace

// Whether the tensor-core path takes this call.
bool prefill_tc_supported(int dtype, int64_t head_dim, int64_t S, int64_t Qc, const void *q, const void *k,
                          const void *qk, int64_t grid)
{
    return (dtype == L2K_BF16 || dtype == L2K_F16) && head_dim == HD && S % 8 == 0 && is_aligned(q, 16) &&
           is_aligned(k, 16) && is_aligned(qk, 16) && grid < (int64_t(1) << 31) && encode_fn() != nullptr &&
           Qc < (int64_t(1) << 31) && S < (int64_t(1) << 31);
}

int prefill_scores_tc(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens, uint32_t max_q,
                      uint32_t max_kv, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc, int64_t S,
                      int dtype, cudaStream_t stream, const uint32_t *block_table, int64_t max_pages,
                      int64_t num_pages)
{
    if (dtype == L2K_BF16)
        return launch_tc<__nv_bfloat16>(q, k, q_lens, kv_lens, max_q, max_kv, qk, batch, Hq, Hkv, Qc, S, block_table,
                                        max_pages, num_pages, stream);
    return launch_tc<__half>(q, k, q_lens, kv_lens, max_q, max_kv, qk, batch, Hq, Hkv, Qc, S, block_table, max_pages,
                             num_pages, stream);
}

int read_scores_error(bool clear); // decode_scores.cu
int read_step_error(bool clear);   // decode_step.cu
int read_pv_error(bool clear);     // attention_qkv_tc.cu
int read_gemm_error(bool clear);   // gemm_tc.cu
int read_gemv_error(bool clear);   // gemv.cu

} // namespace l2k

extern "C" int l2k_device_error(int clear)
{
    int v = 0;
    cudaError_t e = cudaMemcpyFromSymbol(&v, l2k::g_device_error, sizeof(int));
    if (e != cudaSuccess)
        return -1;
    if (clear && v)
    {
        const int zero = 0;
        if (cudaMemcpyToSymbol(l2k::g_device_error, &zero, sizeof(int)) != cudaSuccess)
            return -1;
    }
    const int v2 = l2k::read_scores_error(clear != 0);
    const int v3 = l2k::read_step_error(clear != 0);
    const int v4 = l2k::read_pv_error(clear != 0);
    const int v5 = l2k::read_gemm_error(clear != 0);
    const int v6 = l2k::read_gemv_error(clear != 0);
    if (v2 < 0 || v3 < 0 || v4 < 0 || v5 < 0 || v6 < 0)
        return -1;
    const int others[] = {v2, v3, v4, v5, v6};
    for (int o : others)
        if (!v && o)
            v = o;
    return v;
}
