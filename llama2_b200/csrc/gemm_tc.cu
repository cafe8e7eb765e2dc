// Row-major GEMM C = A op(B) on the 5th-generation tensor cores, for the
// plain (2-D) launch_linear with 16-bit data and trans_A = false:
//   C[m, n] = sum_k A[m, k] * B'[k, n],  B' = B (K x N) or B^T (B stored N x K),
// fp32 accumulation in tensor memory, one rounding to bf16/f16 at the end.
//
// A CTA computes 128 x BN tiles of C, walking K in blocks of 64. Per block
// TMA brings (128-byte swizzle)
//   * the A tile, 128 rows x 64 k: the K-major A operand;
//   * the B tile: with trans_B (B stored N x K) BN rows x 64 k, the K-major
//     B operand; without it (B stored K x N, e.g. a weight [in, out]) 64 k
//     rows x BN columns as 64-column boxes, the MN-major B operand (SBO 1024
//     bytes between 8-row k groups, LBO 8 KB between the 64-column chunks).
// One thread issues the loads into a ring, refilling a stage as soon as the
// MMAs that read it complete; another issues four 128 x BN x 16 MMAs per
// block into TMEM. The tensor maps bound rows at M, columns at N and k at K,
// so partial tiles read zeros. Two warps per TMEM lane quadrant (32 rows)
// read the accumulator, each taking half of the rows' 32-column chunks.
// Five shapes:
//   * at least 256 rows (prefill): the two-SM kernel below, clusters of two
//     CTAs computing 256 x 256 tiles with tcgen05.mma.cta_group::2, each SM
//     holding half of the A and half of the B tile (32 KB per 64-k step in a
//     6-stage ring), two TMEM accumulators per CTA;
//   * 129 to 255 rows: the persistent kernel below, one CTA per SM over
//     128 x 256 tiles, a 4-stage ring of 48 KB, two TMEM accumulators so the
//     epilogue warps drain one tile while the next one's MMAs run;
//   * at most 64 rows (decode batches, bound by streaming B once): the decode
//     kernel below, M = 64 MMAs over 64 x 128 or 64 x 256 tiles with an 8- or
//     5-stage ring, K split over a cluster whose ranks share the reduction
//     and the epilogue (plan: dec_plan);
//   * 65 to 128 rows with at most one 128-column tile per SM: 128 x 128
//     tiles with K split over a thread-block cluster of up to 8 CTAs that
//     reduce their fp32 rows into rank 0 over distributed shared memory
//     (3 stages of 32 KB, two CTAs per SM), or a 4-stage ring without the
//     split;
//   * 65 to 128 rows with more 128-column tiles than SMs: 128 x 256 tiles in
//     a 4-stage ring of 48 KB, one CTA per SM, one wave.
// Every mbarrier wait is bounded; on expiry the kernel records an error code
// (l2k_device_error) and leaves after its copies and MMAs have drained.
//
// Two epilogues replace the store with the operator that follows the
// product in a Llama-2 layer, so the product never goes to HBM:
//   * SwiGLU (gate/up projection): a tile takes BN/2 gate columns and the
//     BN/2 up columns F apart (two B loads per k block) and stores
//     silu(g) * u for its BN/2 output columns;
//   * RoPE + K/V append (QKV projection): a tile covers whole heads of a
//     token row; q and k heads are rotated at the token's position (decode:
//     kv_len - 1; prefill: kv_len - q_len + slot through the unpad -> pad
//     map) and written to the q buffer and the K cache row, v heads to the V
//     cache row.
// Both round the fp32 accumulator to the 16-bit type first (where the
// separate launches read the stored product), then evaluate the separate
// operator's arithmetic, so results are those of launch_linear followed by
// launch_swiglu / the fused RoPE operator for the same tile configuration.
//
// Reference: src/kernel/linear.cu:42-155 (cublasGemmEx with op_A/op_B from
// trans_B/trans_A on the swapped operands; 16-bit data accumulates in 16
// bits there); the epilogues follow src/kernel/swiglu.cu:10-72 and
// src/kernel/fused_reshape_rope_kvcache[_llama2]_decode.cu,
// src/kernel/fused_pad_reshape_transpose_rope_kvcache[_llama2].cu.
#include "common.cuh"
#include "rope_math.cuh"
#include "tcgen05.cuh"

#include <algorithm>
#include <type_traits>

namespace l2k
{

__device__ int g_gemm_error = 0; // first error code recorded by the kernel of this file

bool gemm_tc_supported(int dtype, int trans_a, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda,
                       const void *b, int64_t ldb, const void *c);

namespace
{

constexpr int BM = 128, BK = 64;
constexpr int kEpiParts = 2;             // warps per TMEM lane quadrant in the epilogue
constexpr int kThreads = 128 * kEpiParts;
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

enum Epilogue
{
    EPI_STORE = 0,  // C = A op(B)
    EPI_SWIGLU = 1, // C[:, j] = silu(P[:, j]) * P[:, up_col + j], P = A op(B)
    EPI_ROPE = 2    // P's token rows rotated and written to q / the K and V caches
};

// EPI_ROPE: where a token row's heads go (the fused RoPE operators' arguments).
struct RopeEpi
{
    void *q, *k, *v;
    const uint8_t *is_done;        // decode
    const uint32_t *q_lens;        // prefill
    const uint32_t *kv_lens;
    const uint32_t *unpad_to_pad;  // prefill
    int64_t batch, hq, hkv, hd, qc, S;
    const float2 *table;           // cos/sin table (16-byte aligned) or null
    int64_t table_pos;
    int pairing;
    int prefill;
};

struct GemmTcArgs
{
    void *c;
    int64_t ldc;
    int64_t m, n;   // n: columns of C (EPI_SWIGLU: output columns F; EPI_ROPE: q/k/v columns)
    int n_kb;       // k blocks
    int n_nt;       // column tiles
    int wide;       // C rows are 16-byte aligned: 16-byte stores
    int split;      // SPLIT: CTAs per cluster sharing one C tile, each a K range
    int64_t up_col; // EPI_SWIGLU: column of op(B) where the up half starts
    RopeEpi rope;
};

// Rounds an fp32 accumulator to T and back (the value a separate launch reads).
template <typename T>
__device__ __forceinline__ float round_t(uint32_t bits)
{
    return to_f(from_f<T>(__uint_as_float(bits)));
}

template <typename T>
__device__ __forceinline__ uint4 pack8(const float *o)
{
    uint4 w;
    w.x = pack2<T>(o[0], o[1]);
    w.y = pack2<T>(o[2], o[3]);
    w.z = pack2<T>(o[4], o[5]);
    w.w = pack2<T>(o[6], o[7]);
    return w;
}

// 32 consecutive values to a 16-byte aligned run of T.
template <typename T>
__device__ __forceinline__ void store32(T *dst, const float (&o)[32])
{
#pragma unroll
    for (int v = 0; v < 4; ++v)
        stg(dst + 8 * v, pack8<T>(o + 8 * v));
}

// Columns [col, col + 32) of a row, bounded at n: 16-byte stores when wide,
// element stores at a ragged end.
template <typename T>
__device__ __forceinline__ void store_run(T *out, int64_t col, int64_t n, bool wide, const float (&o)[32])
{
#pragma unroll
    for (int v = 0; v < 4; ++v)
    {
        const int64_t cv = col + 8 * v;
        if (cv >= n)
            break;
        const uint4 w = pack8<T>(o + 8 * v);
        if (wide && cv + 8 <= n)
            stg(out + cv, w);
        else
        {
            const uint32_t w4[4] = {w.x, w.y, w.z, w.w};
            for (int e = 0; e < 8 && cv + e < n; ++e)
            {
                const uint16_t bits = (uint16_t)(e & 1 ? (w4[e / 2] >> 16) : (w4[e / 2] & 0xFFFF));
                reinterpret_cast<uint16_t *>(out)[cv + e] = bits;
            }
        }
    }
}

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

// EPI_ROPE: where this thread's token row goes. Tokens of finished
// sequences, padding slots past the batch and positions outside the cache
// are not written (as in the separate RoPE operators).
struct RopeTok
{
    bool live;
    int64_t seq, slot;
    uint32_t kv_len, pos;
};

__device__ __forceinline__ RopeTok rope_token(const RopeEpi &R, int64_t row, bool store)
{
    RopeTok t{false, 0, 0, 0u, 0u};
    if (!store)
        return t;
    if (R.prefill)
    {
        const int64_t padded = R.unpad_to_pad[row];
        t.seq = padded / R.qc;
        t.slot = padded - t.seq * R.qc;
        if (t.seq < R.batch)
        {
            t.kv_len = R.kv_lens[t.seq];
            t.pos = t.kv_len - R.q_lens[t.seq] + (uint32_t)t.slot;
            t.live = true;
        }
    }
    else
    {
        t.seq = row;
        t.kv_len = R.kv_lens[t.seq];
        t.pos = t.kv_len - 1u;
        t.live = R.is_done[t.seq] == 0;
    }
    t.live = t.live && (int64_t)t.pos < R.S;
    return t;
}

// TMEM columns [c0, c0 + 32) of this thread's row at taddr (every lane of
// the warp: the load is warp-wide), plus, for SPLIT, the peers' partial rows
// (peer p's at red + (p - 1) * red_stride) in rank order.
template <bool SPLIT>
__device__ __forceinline__ void acc32(uint32_t taddr, int c0, uint32_t (&r)[32], bool store, const float *red,
                                      int64_t red_stride, int split)
{
    tmem_ld32_async(taddr + (uint32_t)c0, r);
    tmem_wait_ld();
    if constexpr (SPLIT)
    {
        if (store)
            for (int p = 1; p < split; ++p)
            {
                const float *src = red + (int64_t)(p - 1) * red_stride + c0;
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    r[j] = __float_as_uint(__uint_as_float(r[j]) + src[j]);
            }
    }
}

// The epilogue of one tile for this thread's row: load(c, r) fills r with
// the row's fp32 sums of accumulator columns [c, c + 32) (called by every
// lane of the warp: a TMEM load is warp-wide); col0 = the tile's first
// column of op(B) (EPI_SWIGLU: of the gate half, also the first output
// column). The row's 32-column chunks are dealt to nparts warps: this warp
// takes chunks part, part + nparts, ...
template <typename T, int BN, int EPI, typename Load>
__device__ __forceinline__ void tile_epilogue(const GemmTcArgs &a, Load &&load, int64_t row, bool store, bool wide,
                                              int64_t col0, const RopeTok &tok, int part, int nparts)
{
    if constexpr (EPI == EPI_STORE)
    {
        T *out = static_cast<T *>(a.c) + row * a.ldc;
#pragma unroll 1
        for (int c0 = 32 * part; c0 < BN; c0 += 32 * nparts)
        {
            uint32_t r[32];
            load(c0, r);
            if (!store)
                continue;
            float o[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
                o[j] = __uint_as_float(r[j]);
            store_run<T>(out, col0 + c0, a.n, wide, o);
        }
    }
    else if constexpr (EPI == EPI_SWIGLU)
    {
        // accumulator columns [0, BN/2): gate; [BN/2, BN): up
        T *out = static_cast<T *>(a.c) + row * a.ldc;
#pragma unroll 1
        for (int c0 = 32 * part; c0 < BN / 2; c0 += 32 * nparts)
        {
            uint32_t g[32], u[32];
            load(c0, g);
            load(BN / 2 + c0, u);
            if (!store)
                continue;
            float o[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
                o[j] = silu_mul<T>(round_t<T>(g[j]), round_t<T>(u[j]));
            store_run<T>(out, col0 + c0, a.n, wide, o);
        }
    }
    else
    {
        // whole heads: accumulator columns [j hd, (j + 1) hd) hold head col0 / hd + j;
        // item counts the chunks (or chunk pairs) of the tile in order
        int item = 0;
        const RopeEpi &R = a.rope;
        const int hd = (int)R.hd, half = hd / 2;
        const int64_t total_heads = R.hq + 2 * R.hkv;
        const bool use_table = R.table && tok.kv_len <= 4096u && (int64_t)tok.pos < R.table_pos;
        const float2 *trow = use_table ? R.table + (int64_t)tok.pos * half : nullptr;
        // cos/sin of pairs i and i + 1 (i even: one 16-byte table load)
        auto cs2 = [&](int i, float(&c)[2], float(&s)[2]) {
            if (use_table)
            {
                const float4 cs = __ldg(reinterpret_cast<const float4 *>(trow + i));
                c[0] = cs.x;
                s[0] = cs.y;
                c[1] = cs.z;
                s[1] = cs.w;
            }
            else
            {
                rope_cos_sin_device(i, hd, tok.pos, tok.kv_len, c[0], s[0]);
                rope_cos_sin_device(i + 1, hd, tok.pos, tok.kv_len, c[1], s[1]);
            }
        };
#pragma unroll 1
        for (int j = 0; j < BN / hd; ++j)
        {
            const int64_t head = col0 / hd + j;
            if (head >= total_heads)
                break;
            const int hc = j * hd;
            T *dst = nullptr;
            if (tok.live)
            {
                if (head < R.hq)
                    dst = static_cast<T *>(R.q) + ((tok.seq * R.hq + head) * R.qc + tok.slot) * hd;
                else if (head < R.hq + R.hkv)
                    dst = static_cast<T *>(R.k) + ((tok.seq * R.hkv + head - R.hq) * R.S + tok.pos) * hd;
                else
                    dst = static_cast<T *>(R.v) + ((tok.seq * R.hkv + head - R.hq - R.hkv) * R.S + tok.pos) * hd;
            }
            if (head >= R.hq + R.hkv)
            {
                // v: copied unrotated
#pragma unroll 1
                for (int c0 = 0; c0 < hd; c0 += 32)
                {
                    if (item++ % nparts != part)
                        continue;
                    uint32_t r[32];
                    load(hc + c0, r);
                    if (!dst)
                        continue;
                    float o[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e)
                        o[e] = round_t<T>(r[e]);
                    store32<T>(dst + c0, o);
                }
            }
            else if (R.pairing == L2K_ROPE_INTERLEAVED)
            {
                // pairs (2i, 2i + 1): chunk c0 holds pairs c0/2 .. c0/2 + 15
#pragma unroll 1
                for (int c0 = 0; c0 < hd; c0 += 32)
                {
                    if (item++ % nparts != part)
                        continue;
                    uint32_t r[32];
                    load(hc + c0, r);
                    if (!dst)
                        continue;
                    float o[32];
#pragma unroll
                    for (int e = 0; e < 16; e += 2)
                    {
                        float c[2], s[2];
                        cs2(c0 / 2 + e, c, s);
#pragma unroll
                        for (int f = 0; f < 2; ++f)
                        {
                            const float x0 = round_t<T>(r[2 * (e + f)]), x1 = round_t<T>(r[2 * (e + f) + 1]);
                            o[2 * (e + f)] = rope_o0(c[f], s[f], x0, x1);
                            o[2 * (e + f) + 1] = rope_o1(c[f], s[f], x0, x1);
                        }
                    }
                    store32<T>(dst + c0, o);
                }
            }
            else
            {
                // pairs (i, i + hd/2): chunk c0 of each half
#pragma unroll 1
                for (int c0 = 0; c0 < half; c0 += 32)
                {
                    if (item++ % nparts != part)
                        continue;
                    uint32_t r0[32], r1[32];
                    load(hc + c0, r0);
                    load(hc + half + c0, r1);
                    if (!dst)
                        continue;
                    float o0[32], o1[32];
#pragma unroll
                    for (int e = 0; e < 32; e += 2)
                    {
                        float c[2], s[2];
                        cs2(c0 + e, c, s);
#pragma unroll
                        for (int f = 0; f < 2; ++f)
                        {
                            const float x0 = round_t<T>(r0[e + f]), x1 = round_t<T>(r1[e + f]);
                            o0[e + f] = rope_o0(c[f], s[f], x0, x1);
                            o1[e + f] = rope_o1(c[f], s[f], x0, x1);
                        }
                    }
                    store32<T>(dst + c0, o0);
                    store32<T>(dst + half + c0, o1);
                }
            }
        }
    }
}

// SPLIT: a cluster of a.split CTAs shares one C tile, each CTA summing a
// contiguous range of the k blocks; once every rank's MMAs are done (cluster
// barrier) ranks 1.. push their fp32 rows into rank 0's idle ring with
// st.async, and rank 0 adds them to its own in rank order and stores.
template <typename T, bool B_MN, int BN, int STAGES, bool SPLIT, int EPI>
__global__ void __launch_bounds__(kThreads, (Cfg<BN, STAGES>::kMinBlocks))
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                   const __grid_constant__ GemmTcArgs a)
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
    const int row0 = mt * BM;
    // first column of the tile in op(B) (EPI_SWIGLU: of the gate half, the up
    // half starts at up_col + col0; also the first output column)
    const int64_t col0 = EPI == EPI_SWIGLU ? (int64_t)nt * (BN / 2) : (int64_t)nt * BN;
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
                {
                    // EPI_SWIGLU: the second half of the boxes comes from the up columns
                    const int64_t cx = EPI == EPI_SWIGLU && h >= BN / 128 ? a.up_col + col0 + 64 * (h - BN / 128)
                                                                          : col0 + 64 * h;
                    tma_load_3d(dst + kABox + h * BK * 128, &tm_b, (int)cx, kx, 0, bar);
                }
            }
            else if constexpr (EPI == EPI_SWIGLU)
            {
                // two boxes of BN/2 rows, gate then up (whole 8-row swizzle groups)
                tma_load_3d(dst + kABox, &tm_b, kx, (int)col0, 0, bar);
                tma_load_3d(dst + kABox + (BN / 2) * 128, &tm_b, kx, (int)(a.up_col + col0), 0, bar);
            }
            else
                tma_load_3d(dst + kABox, &tm_b, kx, (int)col0, 0, bar);
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

    // -------- epilogue: warps w and w + 4 hold rows row0 + 32 w + lane (TMEM
    // lane quadrant w), each half of the row's column chunks --------
    const int quad = warp & 3, part = warp >> 2;
    const int64_t row = row0 + 32 * quad + lane;
    const bool store = row < a.m;
    const bool wide = a.wide != 0;
    const int lrow = 32 * quad + lane;          // row within the tile
    float *red = reinterpret_cast<float *>(smem); // SPLIT, rank 0: [split - 1][m][BN] peer rows (in the idle ring)
    const int m_tile = (int)min((int64_t)BM, a.m - row0);
    // EPI_ROPE: this row's token, read before the MMAs are waited for
    RopeTok tok{false, 0, 0, 0u, 0u};
    if constexpr (EPI == EPI_ROPE)
        tok = rope_token(a.rope, row, store);

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
                for (int c0 = 32 * part; c0 < BN; c0 += 32 * kEpiParts)
                {
                    uint32_t r[32];
                    tmem_ld32_async(tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)c0, r);
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
            const uint32_t taddr = tmem + ((uint32_t)(32 * quad) << 16);
            const float *rrow = red + (int64_t)lrow * BN;
            const int64_t rstride = (int64_t)m_tile * BN;
            tile_epilogue<T, BN, EPI>(
                a, [&](int c0, uint32_t(&r)[32]) { acc32<SPLIT>(taddr, c0, r, store, rrow, rstride, split); }, row,
                store, wide, col0, tok, part, kEpiParts);
        }
    }
    else if (EPI == EPI_STORE && store && part == 0)
    {
        T *out = static_cast<T *>(a.c) + row * a.ldc;
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

// Decode-sized products (at most 64 rows of A), bound by streaming B once:
// M = 64 MMAs (row r of the accumulator in TMEM lane (r % 16) + 32 (r / 16)),
// so a stage holds 8 KB of A and a deep ring of B tiles (8 stages of 16 KB
// at 128 columns, 5 of 32 KB at 256), one CTA per SM. Thread 0 initialises
// the barriers and issues the first stages' loads before TMEM is allocated,
// so the first tiles are in flight during the set-up. K is split over a
// thread-block cluster of `split` CTAs; the reduction is spread over the
// cluster: every rank writes its fp32 partial tile to its own shared memory
// (the drained ring), and after a cluster barrier each rank sums the column
// chunks dealt to it from all ranks' copies (distributed shared memory
// loads, rank 0's partial first, then ranks 1.. in order: the order of the
// single-rank reduction) and runs the epilogue on them; a second cluster
// barrier keeps every copy alive until its readers are done.
constexpr int kDM = 64;                  // rows of the MMA and of the A box
constexpr uint32_t kDABox = kDM * 128;   // 64 rows x 64 k
constexpr int kDThreads = 256;

template <int BN>
struct DecCfg
{
    static constexpr uint32_t kStageBytes = kDABox + BN * 128;
    static constexpr int kStages = BN == 128 ? 8 : 5;
    static constexpr uint32_t kOffBar = kStages * kStageBytes;
    static constexpr uint32_t kOffMisc = kOffBar + 8 * (2 * kStages + 1);
    static constexpr uint32_t kSmemBytes = kOffMisc + 16;
    static constexpr int kStride = BN + 4; // floats per staged partial row (16-byte shift per row: no bank conflicts)
    static_assert(2u * kDM * kStride * 4 <= kOffBar, "the staged and the reduced tile must fit the ring");
};

// kind::f16, D f32, A and B bf16 (1) or f16 (0), A K-major, B K-major (0) or MN-major (1), M = 64, N = n.
__host__ __device__ constexpr uint32_t dec_instr_desc(uint32_t ab_format, uint32_t b_mn, uint32_t n)
{
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (b_mn << 16) | ((n >> 3) << 17) |
           ((uint32_t)(kDM >> 4) << 24);
}

__device__ __forceinline__ void cluster_barrier()
{
    asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ float4 ld_cluster_f4(uint32_t addr)
{
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// Index of the k-th set bit of m (k < popcount(m)).
__device__ __forceinline__ int nth_set_bit(uint32_t m, int k)
{
    for (int i = 0; i < k; ++i)
        m &= m - 1;
    return __ffs((int)m) - 1;
}

// Bit c: the epilogue items of a tile that tile_epilogue deals to `rank`
// (items i with i % split == rank, counted in tile_epilogue's order) read
// accumulator columns [32 c, 32 c + 32).
template <int BN, int EPI>
__device__ __forceinline__ uint32_t owned_chunks(const GemmTcArgs &a, int64_t col0, int rank, int split)
{
    uint32_t mask = 0;
    if constexpr (EPI == EPI_STORE)
    {
        for (int c = 0; c < BN / 32; ++c)
            if (c % split == rank)
                mask |= 1u << c;
    }
    else if constexpr (EPI == EPI_SWIGLU)
    {
        for (int i = 0; i < BN / 64; ++i)
            if (i % split == rank)
                mask |= (1u << i) | (1u << (BN / 64 + i));
    }
    else
    {
        const RopeEpi &R = a.rope;
        const int hd = (int)R.hd, half = hd / 2;
        const int64_t total_heads = R.hq + 2 * R.hkv;
        int item = 0;
        for (int j = 0; j < BN / hd; ++j)
        {
            const int64_t head = col0 / hd + j;
            if (head >= total_heads)
                break;
            const int hc = j * hd;
            if (head >= R.hq + R.hkv || R.pairing == L2K_ROPE_INTERLEAVED)
            {
                for (int c0 = 0; c0 < hd; c0 += 32)
                    if (item++ % split == rank)
                        mask |= 1u << ((hc + c0) / 32);
            }
            else
            {
                for (int c0 = 0; c0 < half; c0 += 32)
                    if (item++ % split == rank)
                        mask |= (1u << ((hc + c0) / 32)) | (1u << ((hc + half + c0) / 32));
            }
        }
    }
    return mask;
}

template <typename T, bool B_MN, int BN, int EPI>
__global__ void __launch_bounds__(kDThreads, 1)
    gemm_dec_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                    const __grid_constant__ GemmTcArgs a)
{
    using C = DecCfg<BN>;
    constexpr int kStages = C::kStages;
    constexpr uint32_t kStageBytes = C::kStageBytes;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u) // (the same in every CTA: the whole cluster leaves)
    {
        if (threadIdx.x == 0)
            atomicCAS(&g_gemm_error, 0, ERR_GEMM_SMEM_ALIGN);
        return;
    }
    const uint32_t bar_full = sbase + C::kOffBar;      // + 8 * stage: the stage's tiles landed
    const uint32_t bar_freed = bar_full + 8 * kStages; // + 8 * stage: the MMAs reading it completed
    const uint32_t bar_done = bar_freed + 8 * kStages; // every MMA completed
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + C::kOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + C::kOffMisc + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = a.split;
    const int rank = (int)(blockIdx.x % split);
    const int nt = (int)(blockIdx.x / split);
    const int64_t col0 = EPI == EPI_SWIGLU ? (int64_t)nt * (BN / 2) : (int64_t)nt * BN;
    const int kb0 = (int)((int64_t)rank * a.n_kb / split);
    const int n_kb = (int)((int64_t)(rank + 1) * a.n_kb / split) - kb0;

    // the loads of k block kb (relative to kb0) into its stage
    auto issue = [&](int kb) {
        const int st = kb % kStages;
        const uint32_t dst = sbase + st * kStageBytes;
        const uint32_t bar = bar_full + 8 * st;
        mbar_expect_tx(bar, kStageBytes);
        const int kx = (kb0 + kb) * BK;
        tma_load_3d(dst, &tm_a, kx, 0, 0, bar);
        if constexpr (B_MN)
        {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h)
            {
                const int64_t cx =
                    EPI == EPI_SWIGLU && h >= BN / 128 ? a.up_col + col0 + 64 * (h - BN / 128) : col0 + 64 * h;
                tma_load_3d(dst + kDABox + h * BK * 128, &tm_b, (int)cx, kx, 0, bar);
            }
        }
        else if constexpr (EPI == EPI_SWIGLU)
        {
            tma_load_3d(dst + kDABox, &tm_b, kx, (int)col0, 0, bar);
            tma_load_3d(dst + kDABox + (BN / 2) * 128, &tm_b, kx, (int)(a.up_col + col0), 0, bar);
        }
        else
            tma_load_3d(dst + kDABox, &tm_b, kx, (int)col0, 0, bar);
    };

    int issued = 0; // producer thread: k blocks whose loads were issued
    if (tid == 0)
    {
        for (int i = 0; i < kStages; ++i)
        {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_freed + 8 * i, 1);
        }
        mbar_init(bar_done, 1);
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_a) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(&tm_b) : "memory");
        for (; issued < n_kb && issued < kStages; ++issued)
            issue(issued);
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (tid == 0)
    {
        // ---- producer: the rest of the ring ----
        for (int kb = issued; kb < n_kb && !*abort_flag; ++kb)
        {
            const int st = kb % kStages;
            if (!mbar_wait(bar_freed + 8 * st, ((kb / kStages) - 1) & 1, abort_flag))
            {
                gemm_fail(ERR_GEMM_WAIT_MMA, abort_flag);
                break;
            }
            issue(kb);
            issued = kb + 1;
        }
    }
    else if (tid == 32 && n_kb > 0)
    {
        // ---- MMA issuer ----
        const uint32_t idesc =
            dec_instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, B_MN ? 1u : 0u, (uint32_t)BN);
        for (int kb = 0; kb < n_kb && !*abort_flag; ++kb)
        {
            const int st = kb % kStages;
            if (!mbar_wait(bar_full + 8 * st, (kb / kStages) & 1, abort_flag))
            {
                gemm_fail(ERR_GEMM_WAIT_LOAD, abort_flag);
                break;
            }
            tc_fence_after();
            const uint32_t pa = sbase + st * kStageBytes, pb = pa + kDABox;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
            {
                const uint64_t bd = B_MN ? desc_mn(pb + 2048u * k) : smem_desc(pb + 32u * k);
                mma_f16(tmem, smem_desc(pa + 32u * k), bd, idesc, (kb | k) ? 1u : 0u);
            }
            mma_commit(bar_freed + 8 * st);
        }
        mma_commit(bar_done);
    }
    __syncwarp();

    if (n_kb > 0 && !mbar_wait(bar_done, 0, abort_flag))
        gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
    if (tid == 0 && *abort_flag)
    {
        // after a failure the copies and MMAs in flight land before the ring is reused
        const int quiet = 0;
        for (int kb = std::max(0, issued - kStages); kb < issued; ++kb)
            mbar_wait(bar_full + 8 * (kb % kStages), (kb / kStages) & 1, &quiet);
        if (n_kb > 0)
            mbar_wait(bar_done, 0, &quiet);
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();

    // -------- this CTA's partial tile to its shared memory: warps w and w + 4
    // read TMEM lane quadrant w (rows 16 w .. 16 w + 15 in lanes 0-15), each
    // half of the 32-column chunks --------
    float *stage = reinterpret_cast<float *>(smem); // [kDM][kStride] (the ring is drained)
    {
        const int quad = warp & 3, half = warp >> 2;
        const int srow = 16 * quad + lane;
#pragma unroll 1
        for (int c0 = 32 * half; c0 < BN; c0 += 64)
        {
            uint32_t r[32];
            tmem_ld32_async(tmem + ((uint32_t)(32 * quad) << 16) + (uint32_t)c0, r);
            tmem_wait_ld();
            if (lane < 16)
            {
                float4 *dst = reinterpret_cast<float4 *>(stage + srow * C::kStride + c0);
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    dst[v] = n_kb > 0 ? make_float4(__uint_as_float(r[4 * v]), __uint_as_float(r[4 * v + 1]),
                                                    __uint_as_float(r[4 * v + 2]), __uint_as_float(r[4 * v + 3]))
                                      : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            __syncwarp();
        }
    }
    cluster_barrier(); // every rank's partial is in its shared memory

    // -------- reduction (split > 1): the chunks that this rank's epilogue
    // items read, summed over the ranks' copies in rank order into `reduced`;
    // thread t takes float4 positions t, t + 256, ... two at a time, with all
    // ranks' loads of both in flight before the adds --------
    float *reduced = stage + kDM * C::kStride;
    if (split > 1)
    {
        const uint32_t own = owned_chunks<BN, EPI>(a, col0, rank, split);
        const int n_pos = __popc(own) * kDM * 8;
        const uint32_t stage_u32 = smem_u32(stage);
        uint32_t peer[8];
#pragma unroll
        for (int q = 0; q < 8; ++q)
        {
            uint32_t v = 0;
            if (q < split)
                asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(v) : "r"(stage_u32), "r"(q));
            peer[q] = v;
        }
#pragma unroll 1
        for (int pos0 = tid; pos0 < n_pos; pos0 += 2 * kDThreads)
        {
            float4 x[2][8];
            uint32_t off[2];
#pragma unroll
            for (int b = 0; b < 2; ++b)
            {
                const int pos = pos0 + b * kDThreads;
                off[b] = 0;
                if (pos < n_pos)
                {
                    const int k = pos / (kDM * 8), rem = pos - k * (kDM * 8);
                    off[b] = (uint32_t)(((rem >> 3) * C::kStride + 32 * nth_set_bit(own, k) + 4 * (rem & 7)) * 4);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        if (q < split)
                            x[b][q] = ld_cluster_f4(peer[q] + off[b]);
                }
            }
#pragma unroll
            for (int b = 0; b < 2; ++b)
            {
                if (pos0 + b * kDThreads >= n_pos)
                    continue;
                float4 sum = x[b][0];
#pragma unroll
                for (int q = 1; q < 8; ++q)
                    if (q < split)
                    {
                        sum.x += x[b][q].x;
                        sum.y += x[b][q].y;
                        sum.z += x[b][q].z;
                        sum.w += x[b][q].w;
                    }
                *reinterpret_cast<float4 *>(reinterpret_cast<uint8_t *>(reduced) + off[b]) = sum;
            }
        }
    }
    __syncthreads();

    // -------- epilogue: warps 2p and 2p + 1 take rows 0-31 and 32-63 of part
    // p; items are dealt over (part, rank) as owned_chunks assumes --------
    {
        const int64_t row = 32 * (warp & 1) + lane;
        const int part = (warp >> 1) * split + rank, nparts = (kDThreads / 64) * split;
        const bool store = row < a.m;
        RopeTok tok{false, 0, 0, 0u, 0u};
        if constexpr (EPI == EPI_ROPE)
            tok = rope_token(a.rope, row, store);
        const float *mine = (split > 1 ? reduced : stage) + row * C::kStride;
        auto load = [&](int c0, uint32_t(&r)[32]) {
#pragma unroll
            for (int v = 0; v < 8; ++v)
            {
                const float4 x = *reinterpret_cast<const float4 *>(mine + c0 + 4 * v);
                r[4 * v] = __float_as_uint(x.x);
                r[4 * v + 1] = __float_as_uint(x.y);
                r[4 * v + 2] = __float_as_uint(x.z);
                r[4 * v + 3] = __float_as_uint(x.w);
            }
        };
        if (!*abort_flag)
            tile_epilogue<T, BN, EPI>(a, load, row, store, a.wide != 0, col0, tok, part, nparts);
    }
    __syncwarp();
    cluster_barrier(); // no rank leaves while another may still read its partial

    // -------- teardown --------
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
    }
}

// Persistent variant for products of more than one row tile (prefill-sized):
// one CTA per SM walks the 128 x 256 tiles blockIdx.x, blockIdx.x +
// gridDim.x, ...; warp 0 streams A and B tiles through a 4-stage ring of
// 48 KB across tile boundaries, warp 1 issues the MMAs of a tile into one of
// two 256-column TMEM accumulators, and warps 2-9 (two per TMEM lane
// quadrant) run the epilogue of the previous tile from the other
// accumulator, so the epilogue (a store, SwiGLU or RoPE) overlaps the next
// tile's main loop. Accumulator hand-over: acc_full[b] (the tile's MMAs
// completed, tcgen05.commit) and acc_empty[b] (the eight epilogue warps
// have read it).
constexpr int kPThreads = 64 + 128 * kEpiParts; // producer warp, MMA warp, epilogue warps
constexpr int kPStages = 4;
constexpr int kPBN = 256;
constexpr uint32_t kPStageBytes = kABox + kPBN * 128;
constexpr uint32_t kPOffBar = kPStages * kPStageBytes;
constexpr uint32_t kPOffMisc = kPOffBar + 128;
constexpr uint32_t kPSmemBytes = kPOffMisc + 64;

template <typename T, bool B_MN, int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_tc_persistent_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                              const __grid_constant__ GemmTcArgs a)
{
    constexpr int BN = kPBN;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    if (sbase & 1023u)
    {
        if (threadIdx.x == 0)
            atomicCAS(&g_gemm_error, 0, ERR_GEMM_SMEM_ALIGN);
        return;
    }
    const uint32_t bar_full = sbase + kPOffBar;             // + 8 * stage
    const uint32_t bar_freed = bar_full + 8 * kPStages;     // + 8 * stage
    const uint32_t bar_acc_full = bar_freed + 8 * kPStages; // + 8 * accumulator
    const uint32_t bar_acc_empty = bar_acc_full + 16;       // + 8 * accumulator
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kPOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kPOffMisc + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n_tiles = (int64_t)((a.m + BM - 1) / BM) * a.n_nt;
    const int n_kb = a.n_kb;

    if (tid == 0)
    {
        for (int i = 0; i < kPStages; ++i)
        {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_freed + 8 * i, 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(bar_acc_full + 8 * b, 1);
            mbar_init(bar_acc_empty + 8 * b, 4 * kEpiParts);
        }
        *abort_flag = 0;
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    int64_t issued = 0;     // producer: k blocks whose loads were issued (over all tiles)
    int64_t mma_done = -1;  // MMA thread: the last k block whose MMAs were committed
    if (warp == 0)
    {
        if (lane == 0)
        {
            int64_t it = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x)
            {
                const int row0 = (int)(tile / a.n_nt) * BM;
                const int col0 = (int)(tile % a.n_nt) * BN;
                for (int kb = 0; kb < n_kb; ++kb, ++it)
                {
                    const int st = (int)(it % kPStages);
                    if (it >= kPStages && !mbar_wait(bar_freed + 8 * st, (uint32_t)((it / kPStages) - 1) & 1u,
                                                     abort_flag))
                    {
                        gemm_fail(ERR_GEMM_WAIT_MMA, abort_flag);
                        break;
                    }
                    const uint32_t dst = sbase + st * kPStageBytes;
                    const uint32_t bar = bar_full + 8 * st;
                    mbar_expect_tx(bar, kPStageBytes);
                    const int kx = kb * BK;
                    tma_load_3d(dst, &tm_a, kx, row0, 0, bar);
                    if constexpr (B_MN)
                    {
#pragma unroll
                        for (int h = 0; h < BN / 64; ++h)
                        {
                            const int64_t cx = EPI == EPI_SWIGLU && h >= BN / 128
                                                   ? a.up_col + col0 / 2 + 64 * (h - BN / 128)
                                                   : (EPI == EPI_SWIGLU ? col0 / 2 : col0) + 64 * h;
                            tma_load_3d(dst + kABox + h * BK * 128, &tm_b, (int)cx, kx, 0, bar);
                        }
                    }
                    else if constexpr (EPI == EPI_SWIGLU)
                    {
                        tma_load_3d(dst + kABox, &tm_b, kx, col0 / 2, 0, bar);
                        tma_load_3d(dst + kABox + (BN / 2) * 128, &tm_b, kx, (int)(a.up_col + col0 / 2), 0, bar);
                    }
                    else
                        tma_load_3d(dst + kABox, &tm_b, kx, col0, 0, bar);
                    issued = it + 1;
                }
            }
        }
    }
    else if (warp == 1)
    {
        if (lane == 0)
        {
            const uint32_t idesc =
                gemm_instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, B_MN ? 1u : 0u, (uint32_t)BN);
            int64_t it = 0, lt = 0;
            for (int64_t tile = blockIdx.x; tile < n_tiles && !*abort_flag; tile += gridDim.x, ++lt)
            {
                const int buf = (int)(lt & 1);
                if (lt >= 2 && !mbar_wait(bar_acc_empty + 8 * buf, (uint32_t)((lt >> 1) - 1) & 1u, abort_flag))
                {
                    gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * BN);
                for (int kb = 0; kb < n_kb; ++kb, ++it)
                {
                    const int st = (int)(it % kPStages);
                    if (!mbar_wait(bar_full + 8 * st, (uint32_t)(it / kPStages) & 1u, abort_flag))
                    {
                        gemm_fail(ERR_GEMM_WAIT_LOAD, abort_flag);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t pa = sbase + st * kPStageBytes, pb = pa + kABox;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                    {
                        const uint64_t bd = B_MN ? desc_mn(pb + 2048u * k) : smem_desc(pb + 32u * k);
                        mma_f16(acc, smem_desc(pa + 32u * k), bd, idesc, (kb | k) ? 1u : 0u);
                    }
                    mma_commit(bar_freed + 8 * st);
                    mma_done = it;
                }
                if (*abort_flag)
                    break;
                mma_commit(bar_acc_full + 8 * buf);
            }
        }
    }
    else
    {
        // epilogue warps 2..: TMEM lane quadrant warp % 4 holds rows 32 (warp % 4) + lane of a tile;
        // the kEpiParts warps of a quadrant share its column chunks
        const int quad = warp & 3, part = (warp - 2) >> 2;
        const bool wide = a.wide != 0;
        int64_t lt = 0;
        for (int64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x, ++lt)
        {
            const int buf = (int)(lt & 1);
            const int64_t row = (tile / a.n_nt) * BM + 32 * quad + lane;
            const int64_t ocol0 = (tile % a.n_nt) * (int64_t)(EPI == EPI_SWIGLU ? BN / 2 : BN);
            const bool store = row < a.m;
            RopeTok tok{false, 0, 0, 0u, 0u};
            if constexpr (EPI == EPI_ROPE)
                tok = rope_token(a.rope, row, store);
            if (!mbar_wait(bar_acc_full + 8 * buf, (uint32_t)(lt >> 1) & 1u, abort_flag))
            {
                gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
                break;
            }
            tc_fence_after();
            __syncwarp();
            const uint32_t taddr = tmem + (uint32_t)(buf * BN) + ((uint32_t)(32 * quad) << 16);
            tile_epilogue<T, BN, EPI>(
                a, [&](int c0, uint32_t(&r)[32]) { acc32<false>(taddr, c0, r, store, nullptr, 0, 1); }, row, store,
                wide, ocol0, tok, part, kEpiParts);
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive(bar_acc_empty + 8 * buf);
        }
    }

    // -------- teardown: after a failure, copies and MMAs in flight land first --------
    if (*abort_flag)
    {
        const int quiet = 0;
        if (tid == 0)
            for (int64_t it = std::max<int64_t>(0, issued - kPStages); it < issued; ++it)
                mbar_wait(bar_full + 8 * (int)(it % kPStages), (uint32_t)(it / kPStages) & 1u, &quiet);
        if (tid == 32 && mma_done >= 0)
            mbar_wait(bar_freed + 8 * (int)(mma_done % kPStages), (uint32_t)(mma_done / kPStages) & 1u, &quiet);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
    }
}

// Two-SM variant for products of at least 256 rows: a cluster of two CTAs
// (one per SM) computes 256 x 256 tiles with tcgen05.mma.cta_group::2
// (M = 256, N = 256): CTA rank r holds rows [128 r, 128 r + 128) of the A
// tile and op(B) columns [128 r, 128 r + 128) of the B tile in its shared
// memory, at the same offsets, and receives rows [128 r, 128 r + 128) of the
// 256 x 256 accumulator in its tensor memory. Per 64-k step each SM loads
// 16 KB of A and 16 KB of B (the one-SM 128 x 256 tile loads 16 + 32 KB for
// the same work per SM). Roles: warp 0 of each CTA streams its halves
// through a 6-stage ring, the loads completing on rank 0's "full" barrier;
// warp 1 of rank 0 issues the MMAs and commits to both CTAs' "empty" and
// "accumulator full" barriers (tcgen05.commit multicast); warps 2-9 of each
// CTA run the epilogue of their 128 rows and release the accumulator on
// rank 0's "accumulator empty" barrier. The cluster walks the tiles
// persistently; the two accumulators double-buffer the epilogue.
constexpr int kQStages = 6;
constexpr int kQBN = 256;                          // N of the pair's MMA (B columns per tile)
constexpr uint32_t kQBHalf = 128 * 128;            // one CTA's B half: 128 columns x 64 k
constexpr uint32_t kQStageBytes = kABox + kQBHalf; // 32 KB
constexpr uint32_t kQOffBar = kQStages * kQStageBytes;
constexpr uint32_t kQOffMisc = kQOffBar + 256;
constexpr uint32_t kQSmemBytes = kQOffMisc + 64;

__device__ __forceinline__ uint32_t cluster_rank0_addr(uint32_t local)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(r) : "r"(local));
    return r;
}
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap *map, int x, int y, int z,
                                                 uint32_t bar_cluster)
{
    asm volatile("cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, "
                 "{%2, %3, %4}], [%5];" ::"r"(dst),
                 "l"(map), "r"(x), "r"(y), "r"(z), "r"(bar_cluster)
                 : "memory");
}
__device__ __forceinline__ void mma_f16_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc,
                                             uint32_t accumulate)
{
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
                 "l"(a), "l"(b), "r"(idesc), "r"(accumulate)
                 : "memory");
}
// Arrives on the mbarrier at `bar` (same offset) in both CTAs of the pair once
// the MMAs issued so far have completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar)
{
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                     "r"(bar),
                 "h"((uint16_t)3)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}
__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// kind::f16 for the pair: D f32, A K-major, B K-major (0) or MN-major (1), M = 256, N = 256.
__host__ __device__ constexpr uint32_t pair_instr_desc(uint32_t ab_format, uint32_t b_mn)
{
    return (1u << 4) | (ab_format << 7) | (ab_format << 10) | (b_mn << 16) | ((uint32_t)(kQBN >> 3) << 17) |
           ((uint32_t)(256 >> 4) << 24);
}

template <typename T, bool B_MN, int EPI>
__global__ void __launch_bounds__(kPThreads, 1)
    gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                        const __grid_constant__ GemmTcArgs a)
{
    constexpr int BN = kQBN;
    extern __shared__ __align__(1024) uint8_t smem[];
    const uint32_t sbase = smem_u32(smem);
    uint32_t rank;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(rank));
    const bool leader = rank == 0;
    const uint32_t bar_full = sbase + kQOffBar;             // + 8 * stage (rank 0's are the live ones)
    const uint32_t bar_empty = bar_full + 8 * kQStages;     // + 8 * stage
    const uint32_t bar_acc_full = bar_empty + 8 * kQStages; // + 8 * accumulator
    const uint32_t bar_acc_empty = bar_acc_full + 16;       // + 8 * accumulator (rank 0's are the live ones)
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + kQOffMisc);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kQOffMisc + 8);

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t n_tiles = (int64_t)((a.m + 255) / 256) * a.n_nt;
    const int64_t cluster_id = blockIdx.x >> 1, n_clusters = gridDim.x >> 1;
    const int n_kb = a.n_kb;
    const bool misaligned = (sbase & 1023u) != 0; // uniform over the cluster (same layout); checked after the sync

    if (tid == 0)
    {
        for (int i = 0; i < kQStages; ++i)
        {
            mbar_init(bar_full + 8 * i, 1);
            mbar_init(bar_empty + 8 * i, 1);
        }
        for (int b = 0; b < 2; ++b)
        {
            mbar_init(bar_acc_full + 8 * b, 1);
            mbar_init(bar_acc_empty + 8 * b, 2 * 4 * kEpiParts); // both CTAs' epilogue warps
        }
        *abort_flag = misaligned ? 1 : 0;
        if (misaligned)
            atomicCAS(&g_gemm_error, 0, ERR_GEMM_SMEM_ALIGN);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1)
    {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(2 * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    }
    tc_fence_before();
    cluster_sync_all(); // both CTAs' barriers are initialized and the tensor memory allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t full0 = cluster_rank0_addr(bar_full);          // rank 0's full barriers
    const uint32_t acc_empty0 = cluster_rank0_addr(bar_acc_empty); // rank 0's accumulator-empty barriers

    int64_t issued = 0;    // producer: k blocks whose loads were issued
    int64_t mma_done = -1; // rank 0's MMA thread: the last k block whose MMAs were committed
    if (warp == 0)
    {
        if (lane == 0 && !*abort_flag)
        {
            int64_t it = 0;
            for (int64_t tile = cluster_id; tile < n_tiles && !*abort_flag; tile += n_clusters)
            {
                const int row0 = (int)(tile / a.n_nt) * 256 + 128 * (int)rank;
                const int col0 = (int)(tile % a.n_nt) * BN;
                for (int kb = 0; kb < n_kb; ++kb, ++it)
                {
                    const int st = (int)(it % kQStages);
                    if (it >= kQStages && !mbar_wait(bar_empty + 8 * st, (uint32_t)((it / kQStages) - 1) & 1u,
                                                     abort_flag))
                    {
                        gemm_fail(ERR_GEMM_WAIT_MMA, abort_flag);
                        break;
                    }
                    const uint32_t dst = sbase + st * kQStageBytes;
                    const uint32_t bar = full0 + 8 * st;
                    if (leader)
                        mbar_expect_tx(bar_full + 8 * st, 2 * kQStageBytes); // both CTAs' halves
                    const int kx = kb * BK;
                    tma_load_3d_pair(dst, &tm_a, kx, row0, 0, bar);
                    if constexpr (B_MN)
                    {
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh)
                        {
                            const int h = 2 * (int)rank + hh; // 64-column chunk of the 256-column tile
                            const int64_t cx = EPI == EPI_SWIGLU && h >= 2 ? a.up_col + col0 / 2 + 64 * (h - 2)
                                                                           : (EPI == EPI_SWIGLU ? col0 / 2 : col0) + 64 * h;
                            tma_load_3d_pair(dst + kABox + hh * BK * 128, &tm_b, (int)cx, kx, 0, bar);
                        }
                    }
                    else
                    {
                        const int64_t cy = EPI == EPI_SWIGLU ? (rank ? a.up_col + col0 / 2 : col0 / 2)
                                                             : col0 + 128 * (int64_t)rank;
                        tma_load_3d_pair(dst + kABox, &tm_b, kx, (int)cy, 0, bar);
                    }
                    issued = it + 1;
                }
            }
        }
    }
    else if (warp == 1)
    {
        if (leader && lane == 0 && !*abort_flag)
        {
            const uint32_t idesc =
                pair_instr_desc(std::is_same<T, __nv_bfloat16>::value ? 1u : 0u, B_MN ? 1u : 0u);
            int64_t it = 0, lt = 0;
            for (int64_t tile = cluster_id; tile < n_tiles && !*abort_flag; tile += n_clusters, ++lt)
            {
                const int buf = (int)(lt & 1);
                if (lt >= 2 && !mbar_wait(bar_acc_empty + 8 * buf, (uint32_t)((lt >> 1) - 1) & 1u, abort_flag))
                {
                    gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
                    break;
                }
                tc_fence_after();
                const uint32_t acc = tmem + (uint32_t)(buf * BN);
                for (int kb = 0; kb < n_kb; ++kb, ++it)
                {
                    const int st = (int)(it % kQStages);
                    if (!mbar_wait(bar_full + 8 * st, (uint32_t)(it / kQStages) & 1u, abort_flag))
                    {
                        gemm_fail(ERR_GEMM_WAIT_LOAD, abort_flag);
                        break;
                    }
                    tc_fence_after();
                    const uint32_t pa = sbase + st * kQStageBytes, pb = pa + kABox;
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k)
                    {
                        const uint64_t bd = B_MN ? desc_mn(pb + 2048u * k) : smem_desc(pb + 32u * k);
                        mma_f16_pair(acc, smem_desc(pa + 32u * k), bd, idesc, (kb | k) ? 1u : 0u);
                    }
                    mma_commit_pair(bar_empty + 8 * st); // both CTAs may refill the stage
                    mma_done = it;
                }
                if (*abort_flag)
                    break;
                mma_commit_pair(bar_acc_full + 8 * buf);
            }
        }
    }
    else
    {
        // epilogue warps 2..: TMEM lane quadrant warp % 4 holds rows 32 (warp % 4) + lane of this CTA's half
        const int quad = warp & 3, part = (warp - 2) >> 2;
        const bool wide = a.wide != 0;
        int64_t lt = 0;
        for (int64_t tile = cluster_id; tile < n_tiles && !*abort_flag; tile += n_clusters, ++lt)
        {
            const int buf = (int)(lt & 1);
            const int64_t row = (tile / a.n_nt) * 256 + 128 * (int64_t)rank + 32 * quad + lane;
            const int64_t ocol0 = (tile % a.n_nt) * (int64_t)(EPI == EPI_SWIGLU ? BN / 2 : BN);
            const bool store = row < a.m;
            RopeTok tok{false, 0, 0, 0u, 0u};
            if constexpr (EPI == EPI_ROPE)
                tok = rope_token(a.rope, row, store);
            if (!mbar_wait(bar_acc_full + 8 * buf, (uint32_t)(lt >> 1) & 1u, abort_flag))
            {
                gemm_fail(ERR_GEMM_WAIT_DONE, abort_flag);
                break;
            }
            tc_fence_after();
            __syncwarp();
            const uint32_t taddr = tmem + (uint32_t)(buf * BN) + ((uint32_t)(32 * quad) << 16);
            tile_epilogue<T, BN, EPI>(
                a, [&](int c0, uint32_t(&r)[32]) { acc32<false>(taddr, c0, r, store, nullptr, 0, 1); }, row, store,
                wide, ocol0, tok, part, kEpiParts);
            tc_fence_before();
            __syncwarp();
            if (lane == 0)
                mbar_arrive_cluster(acc_empty0 + 8 * buf);
        }
    }

    // -------- teardown: after a failure, copies and MMAs in flight land first --------
    if (*abort_flag)
    {
        const int quiet = 0;
        if (tid == 32 && leader && mma_done >= 0)
            mbar_wait(bar_empty + 8 * (int)(mma_done % kQStages), (uint32_t)(mma_done / kQStages) & 1u, &quiet);
        if (tid == 0 && leader)
            for (int64_t it = std::max<int64_t>(0, issued - kQStages); it < issued; ++it)
                mbar_wait(bar_full + 8 * (int)(it % kQStages), (uint32_t)(it / kQStages) & 1u, &quiet);
    }
    __syncwarp();
    tc_fence_before();
    cluster_sync_all(); // no CTA leaves while its peer may still signal its barriers or read its tensor memory
    if (warp == 1)
    {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
    }
}

// One GEMM and its epilogue: A (m x k, row stride lda), B (row stride ldb)
// whose op(B) has nb columns, and the kernel arguments the caller fills (c,
// ldc, n, up_col, rope).
struct GemmProblem
{
    const void *a;
    int64_t lda;
    const void *b;
    int64_t ldb;
    int64_t m, nb, k;
    GemmTcArgs args;
};

// The A and B tensor maps and the kernel arguments of a problem run in
// BN-column tiles.
template <typename T, bool B_MN, int BN, int EPI>
bool prepare(const GemmProblem &p, int split, CUtensorMap *ma, CUtensorMap *mb, GemmTcArgs *a)
{
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t m = (uint64_t)p.m, nb = (uint64_t)p.nb, k = (uint64_t)p.k;
    const uint64_t lda = (uint64_t)p.lda, ldb = (uint64_t)p.ldb;
    bool ok = make_map(ma, dt, p.a, k, m, 1, lda * 2, lda * 2 * m, BM, BK);
    if (B_MN) // B stored K x N: boxes of 64 k rows x 64 columns
        ok = ok && make_map(mb, dt, p.b, nb, k, 1, ldb * 2, ldb * 2 * k, BK, 64);
    else // B stored N x K: boxes of BN n rows x 64 k (EPI_SWIGLU: two boxes of BN/2 rows)
        ok = ok && make_map(mb, dt, p.b, k, nb, 1, ldb * 2, ldb * 2 * nb, EPI == EPI_SWIGLU ? BN / 2 : BN, BK);
    *a = p.args;
    a->m = p.m;
    a->n_kb = (int)ceil_div(p.k, BK);
    a->n_nt = (int)ceil_div(a->n, EPI == EPI_SWIGLU ? BN / 2 : BN);
    a->wide = EPI != EPI_ROPE && (a->ldc * 2) % 16 == 0 && is_aligned(a->c, 16) ? 1 : 0;
    a->split = split;
    return ok;
}

template <typename T, bool B_MN, int EPI>
int launch_gemm_persistent(const GemmProblem &p, cudaStream_t stream)
{
    CUtensorMap ma, mb;
    GemmTcArgs a;
    if (!prepare<T, B_MN, kPBN, EPI>(p, 1, &ma, &mb, &a))
        return set_error(L2K_ERR_CUDA, "l2k_linear: tensor map encoding failed");
    auto kernel = gemm_tc_persistent_kernel<T, B_MN, EPI>;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPSmemBytes);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear: %s", cudaGetErrorString(e));
    const int64_t tiles = ceil_div(p.m, BM) * a.n_nt;
    kernel<<<(unsigned)std::min<int64_t>(tiles, num_sms()), kPThreads, kPSmemBytes, stream>>>(ma, mb, a);
    return check_launch("l2k_linear (tcgen05, persistent)");
}

// The two-SM kernel: 256 x 256 tiles over clusters of two CTAs.
template <typename T, bool B_MN, int EPI>
int launch_gemm_pair(const GemmProblem &p, cudaStream_t stream)
{
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t m = (uint64_t)p.m, nb = (uint64_t)p.nb, k = (uint64_t)p.k;
    const uint64_t lda = (uint64_t)p.lda, ldb = (uint64_t)p.ldb;
    CUtensorMap ma, mb;
    bool ok = make_map(&ma, dt, p.a, k, m, 1, lda * 2, lda * 2 * m, BM, BK);
    if (B_MN) // B stored K x N: boxes of 64 k rows x 64 columns
        ok = ok && make_map(&mb, dt, p.b, nb, k, 1, ldb * 2, ldb * 2 * k, BK, 64);
    else // B stored N x K: each CTA's half, 128 n rows x 64 k
        ok = ok && make_map(&mb, dt, p.b, k, nb, 1, ldb * 2, ldb * 2 * nb, 128, BK);
    if (!ok)
        return set_error(L2K_ERR_CUDA, "l2k_linear: tensor map encoding failed");
    GemmTcArgs a = p.args;
    a.m = p.m;
    a.n_kb = (int)ceil_div(p.k, BK);
    a.n_nt = (int)ceil_div(a.n, EPI == EPI_SWIGLU ? kQBN / 2 : kQBN);
    a.wide = EPI != EPI_ROPE && (a.ldc * 2) % 16 == 0 && is_aligned(a.c, 16) ? 1 : 0;
    a.split = 1;
    auto kernel = gemm_tc_pair_kernel<T, B_MN, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQSmemBytes);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear: %s", cudaGetErrorString(e));
    const int64_t tiles = ceil_div(p.m, 256) * a.n_nt;
    const int64_t clusters = std::min<int64_t>(tiles, num_sms() / 2);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(2 * clusters));
    cfg.blockDim = dim3(kPThreads);
    cfg.dynamicSmemBytes = kQSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, kernel, ma, mb, a);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear (two-SM tiles): %s", cudaGetErrorString(e));
    return check_launch("l2k_linear (tcgen05, two-SM tiles)");
}

template <typename T, bool B_MN, int BN, int STAGES, bool SPLIT, int EPI>
int launch_gemm_tc(const GemmProblem &p, cudaStream_t stream, int split)
{
    constexpr uint32_t kSmemBytes = Cfg<BN, STAGES>::kSmemBytes;
    CUtensorMap ma, mb;
    GemmTcArgs a;
    if (!prepare<T, B_MN, BN, EPI>(p, split, &ma, &mb, &a))
        return set_error(L2K_ERR_CUDA, "l2k_linear: tensor map encoding failed");
    auto kernel = gemm_tc_kernel<T, B_MN, BN, STAGES, SPLIT, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e == cudaSuccess) // two CTAs per SM need the whole shared-memory carveout
        e = cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear: %s", cudaGetErrorString(e));
    const int64_t grid = ceil_div(p.m, BM) * a.n_nt * split;
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

// The decode kernel: BN-column tiles, K split over clusters of `split` CTAs.
template <typename T, bool B_MN, int BN, int EPI>
int launch_gemm_dec(const GemmProblem &p, cudaStream_t stream, int split)
{
    constexpr uint32_t kSmemBytes = DecCfg<BN>::kSmemBytes;
    const CUtensorMapDataType dt =
        std::is_same<T, __nv_bfloat16>::value ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    const uint64_t m = (uint64_t)p.m, nb = (uint64_t)p.nb, k = (uint64_t)p.k;
    const uint64_t lda = (uint64_t)p.lda, ldb = (uint64_t)p.ldb;
    CUtensorMap ma, mb;
    bool ok = make_map(&ma, dt, p.a, k, m, 1, lda * 2, lda * 2 * m, kDM, BK);
    if (B_MN) // B stored K x N: boxes of 64 k rows x 64 columns
        ok = ok && make_map(&mb, dt, p.b, nb, k, 1, ldb * 2, ldb * 2 * k, BK, 64);
    else // B stored N x K: boxes of BN n rows x 64 k (EPI_SWIGLU: two boxes of BN/2 rows)
        ok = ok && make_map(&mb, dt, p.b, k, nb, 1, ldb * 2, ldb * 2 * nb, EPI == EPI_SWIGLU ? BN / 2 : BN, BK);
    if (!ok)
        return set_error(L2K_ERR_CUDA, "l2k_linear: tensor map encoding failed");
    GemmTcArgs a = p.args;
    a.m = p.m;
    a.n_kb = (int)ceil_div(p.k, BK);
    a.n_nt = (int)ceil_div(a.n, EPI == EPI_SWIGLU ? BN / 2 : BN);
    a.wide = EPI != EPI_ROPE && (a.ldc * 2) % 16 == 0 && is_aligned(a.c, 16) ? 1 : 0;
    a.split = split;
    auto kernel = gemm_dec_kernel<T, B_MN, BN, EPI>;
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes);
    if (e != cudaSuccess)
        return set_error(L2K_ERR_CUDA, "l2k_linear: %s", cudaGetErrorString(e));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)((int64_t)a.n_nt * split));
    cfg.blockDim = dim3(kDThreads);
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
        return set_error(L2K_ERR_CUDA, "l2k_linear (decode tiles): %s", cudaGetErrorString(e));
    return check_launch("l2k_linear (tcgen05, decode tiles)");
}

// Clusters of `split` CTAs of the decode kernel with BN-column tiles that
// the device runs at once (cached per device; 0 when the query fails).
template <int BN>
int dec_max_clusters(int split)
{
    static std::mutex mu;
    static int cache[64][9] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64 || split < 1 || split > 8)
        return 0;
    std::lock_guard<std::mutex> lock(mu);
    int &c = cache[dev][split];
    if (c == 0)
    {
        auto kernel = gemm_dec_kernel<__nv_bfloat16, true, BN, EPI_STORE>;
        constexpr uint32_t kSmemBytes = DecCfg<BN>::kSmemBytes;
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
            return 0;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)split);
        cfg.blockDim = dim3(kDThreads);
        cfg.dynamicSmemBytes = kSmemBytes;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = (unsigned)split;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess)
        {
            (void)cudaGetLastError();
            return 0;
        }
        c = n > 0 ? n : -1;
    }
    return c > 0 ? c : 0;
}

// Decode-kernel plan for a product of at most 64 rows. The k-block rate of
// one CTA, not its bytes in flight, paces the stream: measured on B200 with
// these rings, about 40 GB/s of B per CTA with 128-column tiles and 76 GB/s
// with 256-column tiles. A plan (tile width, cluster size; every cluster
// resident at once, at least two k blocks per rank) streams at about
// min(CTAs x rate, 6.5 TB/s); the plan is the fastest, and among plans
// within 3 % of it, the smallest cluster (the least reduction), then 256
// columns. False when no tile width fits one wave.
template <int EPI>
bool dec_plan(int64_t n_out, int64_t n_kb, int *bn_out, int *split_out)
{
    struct Cand
    {
        int bn, split;
        double rate;
    } cand[16];
    int nc = 0;
    double best = 0.0;
    for (int bn : {256, 128})
    {
        const int64_t tiles = ceil_div(n_out, EPI == EPI_SWIGLU ? bn / 2 : bn);
        for (int s = 1; s <= 8 && (s == 1 || 2LL * s <= n_kb); ++s)
        {
            const int cap = bn == 128 ? dec_max_clusters<128>(s) : dec_max_clusters<256>(s);
            if (tiles > cap)
                continue;
            const double rate = std::min(6500.0, (double)(tiles * s) * (bn == 256 ? 76.0 : 40.0));
            cand[nc++] = Cand{bn, s, rate};
            best = std::max(best, rate);
        }
    }
    int pick = -1;
    for (int i = 0; i < nc; ++i)
        if (cand[i].rate >= 0.97 * best && (pick < 0 || cand[i].split < cand[pick].split))
            pick = i;
    if (pick < 0)
        return false;
    *bn_out = cand[pick].bn;
    *split_out = cand[pick].split;
    return true;
}

// Tile shape by M: above 128 rows, 128 x 256 tiles (N = 256 MMAs read half
// the A operand per FLOP from shared memory) in a 2-stage ring, two CTAs per
// SM; up to 128 rows (decode-sized products, bound by reading B), 128 x 128
// tiles for twice the CTAs, in a 4-stage ring. The choice depends on m, the
// columns of op(B) and k only, so an epilogue variant runs the same tiles
// (and accumulates the same sums) as the plain product.
template <typename T, bool B_MN, int EPI>
int launch_tiles(const GemmProblem &p, cudaStream_t stream)
{
    if (p.m >= 2 * BM)
        return launch_gemm_pair<T, B_MN, EPI>(p, stream);
    if (p.m > BM)
        return launch_gemm_persistent<T, B_MN, EPI>(p, stream);
    const int64_t tiles = ceil_div(p.nb, 128), n_kb = ceil_div(p.k, BK);
    int dec_bn = 0, dec_split = 0;
    if (p.m <= kDM && dec_plan<EPI>(p.args.n, n_kb, &dec_bn, &dec_split))
        return dec_bn == 128 ? launch_gemm_dec<T, B_MN, 128, EPI>(p, stream, dec_split)
                             : launch_gemm_dec<T, B_MN, 256, EPI>(p, stream, dec_split);
    // One row tile, more 128-column tiles than SMs (a gate/up projection):
    // 256-column tiles with a 4-stage ring (128 KB of B in flight per SM) in
    // one wave. Measured at 64 x 22016 x 4096: 39 us, against 66 us for
    // 128-column tiles at one CTA per SM (two waves) and 43 us at two.
    if (tiles > num_sms())
        return launch_gemm_tc<T, B_MN, 256, 4, false, EPI>(p, stream, 1);
    // Otherwise too few CTAs to stream B at full bandwidth unless K is split
    // across a cluster (the peers' fp32 rows must fit rank 0's ring).
    constexpr int kSplitStages = 3;
    const int64_t ring = (int64_t)kSplitStages * Cfg<128, kSplitStages>::kStageBytes;
    int split = 1;
    while (split < 8 && tiles * split * 2 <= 2LL * num_sms() && split * 2 <= n_kb &&
           (int64_t)(split * 2 - 1) * p.m * 128 * 4 <= ring)
        split *= 2;
    if (split > 1)
        return launch_gemm_tc<T, B_MN, 128, kSplitStages, true, EPI>(p, stream, split);
    return launch_gemm_tc<T, B_MN, 128, 4, false, EPI>(p, stream, 1);
}

template <int EPI>
int dispatch_tc(int trans_b, int dtype, const GemmProblem &p, cudaStream_t stream)
{
    if (dtype == L2K_BF16)
        return trans_b ? launch_tiles<__nv_bfloat16, false, EPI>(p, stream)
                       : launch_tiles<__nv_bfloat16, true, EPI>(p, stream);
    return trans_b ? launch_tiles<__half, false, EPI>(p, stream) : launch_tiles<__half, true, EPI>(p, stream);
}

// Checks and launch of the RoPE epilogue (m token rows of A).
int rope_gemm_entry(int trans_b, const void *a, int64_t lda, const void *b, int64_t ldb, int64_t dim,
                    const RopeEpi &r, int64_t m, int dtype, cudaStream_t stream, const char *name)
{
    L2K_REQUIRE(dtype_ok(dtype), "%s: unsupported dtype %d", name, dtype);
    L2K_REQUIRE(r.pairing == L2K_ROPE_INTERLEAVED || r.pairing == L2K_ROPE_HALF, "%s: bad pairing %d", name,
                r.pairing);
    L2K_REQUIRE(m >= 0 && dim >= 0 && r.batch >= 0 && r.hq >= 0 && r.hkv >= 0 && r.hd >= 0 && r.S >= 0 &&
                    r.qc >= 0 && r.table_pos >= 0,
                "%s: negative size", name);
    const int64_t n = (r.hq + 2 * r.hkv) * r.hd;
    L2K_REQUIRE(lda >= dim && ldb >= (trans_b ? dim : n), "%s: leading dimension too small", name);
    if (m == 0 || n == 0)
        return L2K_OK;
    L2K_REQUIRE(a && b && r.kv_lens && r.q && (r.hkv == 0 || (r.k && r.v)), "%s: null pointer", name);
    if (r.prefill)
        L2K_REQUIRE(r.q_lens && r.unpad_to_pad && r.qc > 0, "%s: null q_lens/unpad_to_pad or q_cache_len 0", name);
    else
        L2K_REQUIRE(r.is_done, "%s: null is_done", name);
    if (dtype == L2K_F32)
        return set_error(L2K_ERR_UNSUPPORTED_DTYPE, "%s: tensor cores take 16-bit data only", name);
    L2K_REQUIRE_SHAPE((r.hd == 64 || r.hd == 128) && is_aligned(r.q, 16) &&
                          (r.hkv == 0 || (is_aligned(r.k, 16) && is_aligned(r.v, 16))) &&
                          (r.table == nullptr || is_aligned(r.table, 16)) &&
                          gemm_tc_supported(dtype, 0, m, n, dim, a, lda, b, ldb, r.q),
                      "%s: needs head_dim 64 or 128, 16-byte aligned q/k/v/table and operands, k >= 1 "
                      "(run l2k_linear and the RoPE operator instead)",
                      name);
    GemmProblem p{a, lda, b, ldb, m, n, dim, GemmTcArgs{}};
    p.args.n = n;
    p.args.rope = r;
    return dispatch_tc<EPI_ROPE>(trans_b ? 1 : 0, dtype, p, stream);
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

int gemm_tc(int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda, const void *b, int64_t ldb,
            void *c, int64_t ldc, int dtype, cudaStream_t stream)
{
    GemmProblem p{a, lda, b, ldb, m, n, k, GemmTcArgs{}};
    p.args.c = c;
    p.args.ldc = ldc;
    p.args.n = n;
    return dispatch_tc<EPI_STORE>(trans_b, dtype, p, stream);
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

extern "C" int l2k_linear_swiglu(int trans_b, int64_t m, int64_t inter, int64_t k, const void *a, int64_t lda,
                                 const void *b, int64_t ldb, void *out, int64_t ldo, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_linear_swiglu: unsupported dtype %d", dtype);
    L2K_REQUIRE(m >= 0 && inter >= 0 && k >= 0, "l2k_linear_swiglu: negative size");
    L2K_REQUIRE(ldo >= inter && lda >= k && ldb >= (trans_b ? k : 2 * inter),
                "l2k_linear_swiglu: leading dimension too small");
    if (m == 0 || inter == 0)
        return L2K_OK;
    L2K_REQUIRE(a && b && out, "l2k_linear_swiglu: null pointer");
    if (dtype == L2K_F32)
        return set_error(L2K_ERR_UNSUPPORTED_DTYPE, "l2k_linear_swiglu: tensor cores take 16-bit data only");
    L2K_REQUIRE_SHAPE(inter % 8 == 0 && gemm_tc_supported(dtype, 0, m, 2 * inter, k, a, lda, b, ldb, out),
                      "l2k_linear_swiglu: needs inter %% 8 == 0, 16-byte aligned operands and k >= 1 "
                      "(run l2k_linear and l2k_swiglu instead)");
    GemmProblem p{a, lda, b, ldb, m, 2 * inter, k, GemmTcArgs{}};
    p.args.c = out;
    p.args.ldc = ldo;
    p.args.n = inter;
    p.args.up_col = inter;
    return dispatch_tc<EPI_SWIGLU>(trans_b ? 1 : 0, dtype, p, stream);
}

extern "C" int l2k_linear_rope_kvcache_decode(int trans_b, const void *a, int64_t lda, const void *b, int64_t ldb,
                                              int64_t dim, const uint8_t *is_done, const uint32_t *kv_lens, void *q,
                                              void *k, void *v, int64_t batch, int64_t q_head_num,
                                              int64_t kv_head_num, int64_t head_dim, int64_t kv_cache_len,
                                              const float *rope_table, int64_t rope_table_positions, int pairing,
                                              int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    const RopeEpi r{q,         k,           v,        is_done,     nullptr, kv_lens, nullptr,
                    batch,     q_head_num,  kv_head_num, head_dim, 1,       kv_cache_len,
                    reinterpret_cast<const float2 *>(rope_table), rope_table ? rope_table_positions : 0,
                    pairing,   0};
    return rope_gemm_entry(trans_b, a, lda, b, ldb, dim, r, batch, dtype, stream, "l2k_linear_rope_kvcache_decode");
}

extern "C" int l2k_linear_pad_rope_kvcache_prefill(int trans_b, const void *a, int64_t lda, const void *b,
                                                   int64_t ldb, int64_t dim, const uint32_t *q_lens,
                                                   const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx, void *q,
                                                   void *k, void *v, int64_t num_tokens, int64_t batch,
                                                   int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
                                                   int64_t q_cache_len, int64_t kv_cache_len,
                                                   const float *rope_table, int64_t rope_table_positions, int pairing,
                                                   int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    const RopeEpi r{q,           k,          v,           nullptr,  q_lens,      kv_lens, unpad_to_pad_idx,
                    batch,       q_head_num, kv_head_num, head_dim, q_cache_len, kv_cache_len,
                    reinterpret_cast<const float2 *>(rope_table), rope_table ? rope_table_positions : 0,
                    pairing,     1};
    return rope_gemm_entry(trans_b, a, lda, b, ldb, dim, r, num_tokens, dtype, stream,
                           "l2k_linear_pad_rope_kvcache_prefill");
}
