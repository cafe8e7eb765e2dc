// Fused prefill attention scores on the 5th-generation tensor cores:
//   P = softmax_causal(Q K^T / sqrt(128)),  bf16/f16 in, fp32 accumulate, bf16/f16 out.
//
// One CTA owns 128 query rows of one (seq, head); key tiles are 64 wide.
// Warp roles (288 threads, two CTAs per SM):
//   * warp 8 (control): TMA (cp.async.bulk.tensor, 128-byte swizzle) of the
//     Q tile once and of K tiles through a 3-stage ring; tcgen05.mma
//     (M=128, N=64, K=16 x 8) with both operands in shared memory and the
//     fp32 accumulator in tensor memory (2 x 64 columns, double buffered);
//     tcgen05.commit signals "tile ready" on an mbarrier.
//   * warps 0-7 (epilogue): warp w reads TMEM lanes 32*(w%4).. (its rows) and
//     columns 32*(w/4).. of each tile with tcgen05.ld.
//     Phase A walks the causally visible key tiles keeping an online row max
//     and sum of exponentials (log2 units, ex2); phase B re-runs the MMAs
//     and writes P = 2^(s*c - m) / (sum + 1e-6) once: each warp stages its
//     32 x 32 block (64-byte swizzle) and TMA-stores it itself, so phase B
//     has no CTA-wide barrier. Each finished tile frees its TMEM buffer
//     through an mbarrier, so the MMA of the next tile overlaps.
//   * Key tiles beyond the causal limit are TMA-stored from the zeroed staging
//     region at the start (overlapping phase A). Keys >= max_kv are never
//     written (the store map's extent; its 16-byte-rounded tail is written
//     directly); tiles whose rows straddle q_len are written directly.
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

constexpr int BM = 128, BN = 64, HD = 128, KH = 64; // KH: elements per 128-byte swizzle row
constexpr int kEpiWarps = 8;
constexpr int kThreads = 32 * (kEpiWarps + 1);
constexpr int kCtl = kEpiWarps;                        // control warp index
constexpr uint32_t kQBox = 128 * 128;                  // 128 rows x 128 B
constexpr uint32_t kKBox = 64 * 128;                   // 64 rows x 128 B
constexpr int kKStages = 3;                            // K ring depth
constexpr uint32_t kWarpStage = 32 * 64;               // one warp's 32 x 32 block of P (64-byte rows)
constexpr uint32_t kOffQ = 0;                          // 2 boxes (hd halves)
constexpr uint32_t kOffK = kOffQ + 2 * kQBox;          // kKStages stages x 2 boxes
constexpr uint32_t kOffP = kOffK + kKStages * 2 * kKBox; // 8 warp blocks = one zeroed 128 x 64 box at the start
constexpr uint32_t kOffBar = kOffP + kEpiWarps * kWarpStage; // mbarriers
constexpr uint32_t kOffMisc = kOffBar + 128;           // tmem slot, abort flag
constexpr uint32_t kOffStats = kOffMisc + 64;          // 2 x 128 float2
constexpr uint32_t kSmemBytes = kOffStats + 2 * 128 * 8 + 1024; // + alignment slack
constexpr uint32_t kTmemCols = 2 * BN;
constexpr long long kWaitCycles = 4000000000LL;        // ~2 s at 2 GHz
constexpr float kNegBig = -1e30f;

enum DevError
{
    ERR_WAIT_Q = 0x101,
    ERR_WAIT_K = 0x102,
    ERR_WAIT_MMA = 0x103,
    ERR_WAIT_TMEM = 0x104
};

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
};

// ---------------------------------------------------------------------------
// PTX wrappers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Bounded wait on phase `parity`; false when the time limit expired or when
// another thread of the CTA has already given up (abort), so that after a
// failure every warp runs through its remaining steps quickly and still meets
// every barrier it shares with the others.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, const volatile int *abort_flag)
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
        if (*abort_flag || clock64() - t0 > kWaitCycles)
            return false;
    }
}

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap *map, int x, int y, int z, uint32_t bar)
{
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
                 "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, uint32_t src, int x, int y, int z)
{
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(map),
                 "r"(src), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read_0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// Named barrier among the epilogue warps only.
__device__ __forceinline__ void epi_sync() { asm volatile("bar.sync 1, %0;" ::"n"(32 * kEpiWarps) : "memory"); }

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// K-major operand, 128-byte swizzle: 8-row atoms of 1024 bytes (SBO), version 1.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr)
{
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// kind::f16 instruction descriptor: D f32, A/B bf16 (1) or f16 (0), both K-major, M=128, N=BN.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t ab_format)
{
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
                 "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
                 : "memory");
}
__device__ __forceinline__ void mma_commit(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32])
{
    uint32_t r[32];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
                 "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                   "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
                   "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
                   "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
                   "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
                 : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i)
        v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float a, float b);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float a, float b)
{
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float a, float b)
{
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
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
                             const __grid_constant__ CUtensorMap tm_p, const __grid_constant__ CUtensorMap tm_pw,
                             const TcArgs a)
{
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const uint32_t sbase = smem_u32(smem);
    const uint32_t bar_q = sbase + kOffBar;
    const uint32_t bar_kfull = bar_q + 8;    // + 8 * stage (kKStages)
    const uint32_t bar_mma = bar_q + 32;     // + 8 * buffer: tile in TMEM buffer is ready
    const uint32_t bar_tfree = bar_q + 48;   // + 8 * buffer: epilogue finished with TMEM buffer
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kOffMisc + 8);
    float2 *stats = reinterpret_cast<float2 *>(smem + kOffStats); // [2][128]

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
    // TMA stores need whole 128-row tiles; their map covers keys [0, M8).
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
        // the staging region starts as the zero 128 x 64 tile
        uint4 *z = reinterpret_cast<uint4 *>(smem + kOffP);
        for (int i = tid; i < (int)(kEpiWarps * kWarpStage / 16); i += kThreads)
            z[i] = make_uint4(0, 0, 0, 0);
    }
    fence_proxy_async();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == kCtl)
    {
        // ================= control warp =================
        if (lane == 0 && n_steps > 0)
        {
            const uint32_t idesc = instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u);
            const int kz = (int)(b * a.Hkv + kvh);
            auto issue_k = [&](int t) {
                const int kt = t % n_a, st = t % kKStages;
                const uint32_t dst = sbase + kOffK + st * 2 * kKBox;
                mbar_expect_tx(bar_kfull + 8 * st, 2 * kKBox);
                for (int hf = 0; hf < 2; ++hf)
                    tma_load_3d(dst + hf * kKBox, &tm_k, hf * KH, kt * BN, kz, bar_kfull + 8 * st);
            };
            mbar_expect_tx(bar_q, 2 * kQBox);
            for (int hf = 0; hf < 2; ++hf)
                tma_load_3d(sbase + kOffQ + hf * kQBox, &tm_q, hf * KH, (int)row0, (int)bh, bar_q);
            for (int t = 0; t < kKStages && t < n_steps; ++t)
                issue_k(t);
            if (!mbar_wait(bar_q, 0, abort_flag))
                fail(ERR_WAIT_Q, abort_flag);
            for (int t = 0; t < n_steps && !*abort_flag; ++t)
            {
                const int st = t & 1, ks = t % kKStages; // TMEM buffer, K stage
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
#pragma unroll
                for (int k = 0; k < HD / 16; ++k)
                {
                    const uint32_t offa = (uint32_t)((k & 3) * 32) + (uint32_t)(k >> 2) * kQBox;
                    const uint32_t offb = (uint32_t)((k & 3) * 32) + (uint32_t)(k >> 2) * kKBox;
                    mma_f16(d, smem_desc(sbase + kOffQ + offa), smem_desc(kb + offb), idesc, k > 0 ? 1u : 0u);
                }
                mma_commit(bar_mma + 8 * st);
                if (t >= 1 && t + 2 < n_steps)
                {
                    // K stage (t - 1) % kKStages = (t + 2) % kKStages is free once
                    // the previous tile's MMAs (long done) have read it
                    if (!mbar_wait(bar_mma + 8 * ((t - 1) & 1), ((t - 1) >> 1) & 1, abort_flag))
                    {
                        fail(ERR_WAIT_MMA, abort_flag);
                        break;
                    }
                    issue_k(t + 2);
                }

            }
        }
    }
    else
    {
        // ================= epilogue warps =================
        const int quad = warp & 3, ch = warp >> 2; // TMEM lanes 32*quad.., columns 32*ch..
        const int r = quad * 32 + lane;            // row within the tile
        const int64_t lim_r = min(kv_len - 1, hist + row0 + r);
        float m = kNegBig, l = 0.f, inv = 0.f;     // log2-domain running max / sum
        uint16_t *qk16 = static_cast<uint16_t *>(a.qk);
        const int64_t row_off = (bh * a.Qc + row0 + r) * a.S;

        if (tid == 0 && full_rows)
        {
            // zero key tiles beyond the causal limit, from staging buffer 0
            for (int kt = n_a; kt < a.n_kt; ++kt)
                tma_store_3d(&tm_p, sbase + kOffP, kt * BN, (int)row0, (int)bh);
            bulk_commit();
        }

        for (int t = 0; t < n_steps; ++t)
        {
            const int st = t & 1;
            // After a failure the remaining steps run on whatever TMEM holds (the
            // error is recorded); no warp leaves early, so the named barriers below
            // are met by all epilogue warps.
            if (!mbar_wait(bar_mma + 8 * st, (t >> 1) & 1, abort_flag))
                fail(ERR_WAIT_MMA, abort_flag);
            tc_fence_after();
            const bool phase_b = t >= n_a;
            const int kt = phase_b ? t - n_a : t;
            const int64_t key0 = (int64_t)kt * BN + ch * 32;
            const bool masked = (int64_t)kt * BN + BN - 1 > min_lim;
            float v[32];
            tmem_ld32(tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(st * BN + ch * 32), v);
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(bar_tfree + 8 * st); // the TMEM buffer may take the next tile
            if (masked)
            {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    v[j] = key0 + j <= lim_r ? v[j] : -INFINITY;
            }
            if (!phase_b)
            {
                float tmax = -INFINITY;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    tmax = fmaxf(tmax, v[j]);
                const float m_new = fmaxf(m, tmax * a.c);
                float sum = 0.f;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    sum += ex2(fmaf(v[j], a.c, -m_new));
                l = l * ex2(m - m_new) + sum;
                m = m_new;
                if (t == n_a - 1)
                {
                    stats[ch * 128 + r] = make_float2(m, l);
                    if (tid == 0)
                        bulk_wait_read_0(); // the zero-tile stores are done with staging buffer 0
                    epi_sync();
                    const float2 s0 = stats[r], s1 = stats[128 + r];
                    const float Mx = fmaxf(s0.x, s1.x);
                    const float L = s0.y * ex2(s0.x - Mx) + s1.y * ex2(s1.x - Mx);
                    m = Mx;
                    inv = __frcp_rn(__fadd_rn(L, 1e-6f));
                }
                continue;
            }
            uint32_t packed[16];
#pragma unroll
            for (int j = 0; j < 32; j += 2)
                packed[j / 2] = pack2<T>(ex2(fmaf(v[j], a.c, -m)) * inv, ex2(fmaf(v[j + 1], a.c, -m)) * inv);
            if (full_rows)
            {
                // This warp's 32 x 32 block (rows quad*32.., keys key0..) staged with
                // the 64-byte swizzle (16-byte chunk c of row r at c ^ ((r / 2) % 4))
                // and stored by the warp itself.
                uint8_t *wst = smem + kOffP + (uint32_t)warp * kWarpStage;
                if (lane == 0)
                    bulk_wait_read_0(); // this warp's previous store has read the block
                __syncwarp();
                uint8_t *dst = wst + (uint32_t)lane * 64;
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
                    *reinterpret_cast<uint4 *>(dst + ((c4 ^ ((lane >> 1) & 3)) * 16)) =
                        make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2], packed[4 * c4 + 3]);
                if (key0 + 32 > a.M8 && key0 < a.M)
                {
                    // keys [M8, M) are beyond the store map: written directly
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        if (key0 + e >= a.M8 && key0 + e < a.M)
                            qk16[row_off + key0 + e] = half_of(packed[e / 2], e & 1);
                }
                fence_proxy_async();
                __syncwarp();
                if (lane == 0)
                {
                    tma_store_3d(&tm_pw, smem_u32(wst), (int)key0, (int)(row0 + quad * 32), (int)bh);
                    bulk_commit();
                }
            }
            else if (r < rows_valid)
            {
#pragma unroll
                for (int c4 = 0; c4 < 4; ++c4)
                {
                    const int64_t col = key0 + c4 * 8;
                    if (col + 8 <= a.M)
                        *reinterpret_cast<uint4 *>(qk16 + row_off + col) =
                            make_uint4(packed[4 * c4], packed[4 * c4 + 1], packed[4 * c4 + 2], packed[4 * c4 + 3]);
                    else
                    {
#pragma unroll
                        for (int e = 0; e < 8; ++e)
                            if (col + e < a.M)
                                qk16[row_off + col + e] = half_of(packed[4 * c4 + e / 2], e & 1);
                    }
                }
            }
        }

        // Zero tails: keys [M8, M) of the zero tiles of full-row tiles, and
        // every zero key of tiles whose rows straddle q_len.
        if (full_rows && a.M8 < a.M && (int64_t)n_a * BN < a.M)
        {
            for (int64_t j = max(a.M8, (int64_t)n_a * BN) + ch; j < a.M; j += 2)
                qk16[row_off + j] = 0;
        }
        if (!full_rows && r < rows_valid)
        {
            for (int64_t j = (int64_t)n_a * BN + ch; j < a.M; j += 2)
                qk16[row_off + j] = 0;
        }
        if (lane == 0)
            bulk_wait_all(); // this warp's stores (and, for warp 0, the zero tiles)
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
// Host side: tensor maps and launch
// ---------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        else
            cudaGetLastError();
    });
    return fn;
}

bool make_map(CUtensorMap *map, CUtensorMapDataType dt, const void *base, uint64_t d0, uint64_t d1, uint64_t d2,
              uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box_rows, uint32_t box_cols = KH,
              CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B)
{
    auto fn = encode_fn();
    if (!fn)
        return false;
    const cuuint64_t dims[3] = {d0, d1, d2};
    const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
    const cuuint32_t box[3] = {box_cols, box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, dt, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
              CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
int launch_tc(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens, uint32_t max_q,
              uint32_t max_kv, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc, int64_t S,
              cudaStream_t stream)
{
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const int64_t M = std::min<int64_t>(max_kv, S);
    CUtensorMap mq, mk, mp, mpw;
    const int64_t m8 = std::max<int64_t>(M & ~int64_t(7), 8);
    if (!make_map(&mq, dt, q, HD, Qc, batch * Hq, HD * 2, Qc * HD * 2, BM) ||
        !make_map(&mk, dt, k, HD, S, batch * Hkv, HD * 2, S * HD * 2, BN) ||
        !make_map(&mp, dt, qk, m8, Qc, batch * Hq, S * 2, Qc * S * 2, BM) ||
        !make_map(&mpw, dt, qk, m8, Qc, batch * Hq, S * 2, Qc * S * 2, 32, 32, CU_TENSOR_MAP_SWIZZLE_64B))
        return set_error(L2K_ERR_CUDA, "l2k_prefill_attention_scores: tensor map encoding failed");
    // c = (1/sqrtf(128)) * log2(e): the oracle's fp32 scale, moved to base 2 for ex2.
    TcArgs a{q_lens, kv_lens, qk, Hq, Hq / Hkv, Hkv, Qc, S, M, M & ~int64_t(7), (int)ceil_div(max_q, BM),
             (int)ceil_div(M, BN), (1.f / sqrtf((float)HD)) * 1.44269504088896340736f};
    auto kernel = prefill_scores_tc_kernel<T>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_prefill_attention_scores: %s", cudaGetErrorString(e));
    const int64_t grid = (int64_t)a.n_qt * batch * Hq;
    kernel<<<(unsigned)grid, kThreads, kSmemBytes, stream>>>(mq, mk, mp, mpw, a);
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
                      int dtype, cudaStream_t stream)
{
    if (dtype == L2K_BF16)
        return launch_tc<__nv_bfloat16>(q, k, q_lens, kv_lens, max_q, max_kv, qk, batch, Hq, Hkv, Qc, S, stream);
    return launch_tc<__half>(q, k, q_lens, kv_lens, max_q, max_kv, qk, batch, Hq, Hkv, Qc, S, stream);
}

int read_scores_error(bool clear); // decode_scores.cu
int read_step_error(bool clear);   // decode_step.cu

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
    if (v2 < 0 || v3 < 0)
        return -1;
    return v ? v : (v2 ? v2 : v3);
}
