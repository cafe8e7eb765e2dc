// Streaming score rows: QK^T + scale + length mask + softmax for one score
// row per thread-block cluster, shared by the fused decode-scores operator
// (decode_scores.cu) and the one-launch decode step (decode_step.cu).
//
// A score row is (seq b, q head h, query row i). Its keys are cut into 16 KB
// blocks of whole K rows (one (b, kv head) plane of the (B, Hkv, S, hd) cache
// is contiguous, so a block is one linear range); global block g belongs to
// cluster rank g % C, so every CTA of the cluster has work whatever kv_len
// is. Per CTA, warp kCW is the producer: one lane issues cp.async.bulk copies
// of the CTA's blocks into a kNS-stage shared-memory ring (mbarrier full /
// empty pairs, every wait bounded); warps 0..kCW-1 consume: warp w takes ring
// stage w % kNS and half w / kNS of each block; each lane holds a 16-byte
// slice of q, reads the matching slice of R K rows from shared memory per
// step and folds the R partial dot products with multi_reduce. Logits stay in
// shared memory; the CTA reduces its max and sum of exponentials (one expf
// per logit, kept in place), the cluster combines them over distributed
// shared memory, and each CTA writes its normalized probabilities once.
//
// In the fused decode step (STEP = true) the row also does the RoPE of its
// q head and of the new K row: q is rotated from the packed qkv input instead
// of being read back, and the rotated K row replaces the stale cache row in
// shared memory before the logits are computed; the CTA that owns that block
// also writes the K and V rows into the cache.
//
// Reference composition: QK^T via cuBLAS batched GEMM (src/kernel/linear.cu:96-128)
// + masked softmax (src/kernel/compute_masked_attention_score.cu:12-103)
// with the mask "positions 0..pos"; RoPE + KV append as in
// src/kernel/fused_reshape_rope_kvcache_decode.cu:11-84 and
// src/kernel/fused_reshape_rope_kvcache_llama2_decode.cu:11-74.
#pragma once

#include "common.cuh"
#include "rope_math.cuh"

#include <cooperative_groups.h>

namespace l2k
{
namespace
{
namespace cg = cooperative_groups;

constexpr float kSoftmaxEps = 1e-6f;
constexpr int kNS = 3;                 // ring stages (3 CTAs of 64 KB fit one SM)
constexpr int kCW = 2 * kNS;            // consumer warps (two per stage, one half-block each)
constexpr int kBlockBytes = 16384;     // one key block
constexpr int kStreamThreads = 32 * (kCW + 1);
constexpr long long kWaitCycles = 4000000000LL; // ~2 s

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
    int bulk_out; // score rows start 16-byte aligned: stored with cp.async.bulk
    // PV rows only: the V cache and the attention output P.V
    const void *v;        // (B, Hkv, S, hd)
    void *qkv;            // (B, Hq, Qc, hd)
    // Paged caches (decode only): k and v are (num_pages, Hkv, KB, hd), one
    // key block per page; block g of sequence b is page block_table[b][g]
    // (max_pages entries per sequence; S = max_pages * KB).
    const uint32_t *block_table;
    int64_t max_pages;
    int64_t num_pages;
    // fp8 (e4m3) caches only: V values are v_scale * e4m3 (K's scale is
    // folded into `scale`).
    float v_scale;
};

// Extra inputs of a score row inside the fused decode step. kv_lens and
// q_lens are the lengths before this step's update (the step's length update
// is written by its last CTA).
struct StepRowArgs
{
    const void *qkv;          // [B, (Hq + 2 Hkv) * hd]
    const uint8_t *is_done;
    const uint32_t *q_lens;
    uint32_t *kv_lens;        // read at the start, updated by the last CTA
    uint32_t *max_lens;       // [2]: max q_len, max kv_len (written by the last CTA)
    uint32_t *counter;        // ticket counter, zero before and after the launch
    void *q_out;              // (B, Hq, 1, hd)
    void *k_cache;
    void *v_cache;
    const float2 *table;
    int64_t table_pos;
    int64_t batch;
    int64_t qkv_stride;       // (Hq + 2 Hkv) * hd
    int pairing;
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

// Dot product of 16 bytes of a K row with this lane's slice of q, as the
// chain sacc = fma(k_e, q_e, sacc), e = 0..N-1, from sacc = 0. For 16-bit
// elements each step is the sm_100 mixed-precision fma (16-bit a and b,
// fp32 c and d): it rounds a*b+c once, exactly as fmaf does on the widened
// (exact) operands, and saves the two widening instructions per element.
template <typename T>
__device__ __forceinline__ float dot16(uint4 k, uint4 q, const float *qf)
{
    const Vec16<T> kv = as_vec<T>(k);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < Vec16<T>::N; ++e)
        s = fmaf(to_f(kv.v[e]), qf[e], s);
    return s;
}
#define L2K_DOT16_MIXED(TYPE, PTXTYPE)                                                                       \
    template <>                                                                                              \
    __device__ __forceinline__ float dot16<TYPE>(uint4 k, uint4 q, const float *)                           \
    {                                                                                                        \
        float s;                                                                                             \
        asm("{\n\t.reg .b16 k0, k1, k2, k3, k4, k5, k6, k7, q0, q1, q2, q3, q4, q5, q6, q7;\n\t"             \
            "mov.b32 {k0, k1}, %1;\n\tmov.b32 {k2, k3}, %2;\n\tmov.b32 {k4, k5}, %3;\n\tmov.b32 {k6, k7}, %4;\n\t" \
            "mov.b32 {q0, q1}, %5;\n\tmov.b32 {q2, q3}, %6;\n\tmov.b32 {q4, q5}, %7;\n\tmov.b32 {q6, q7}, %8;\n\t" \
            "fma.rn.f32." PTXTYPE " %0, k0, q0, 0f00000000;\n\t"                                             \
            "fma.rn.f32." PTXTYPE " %0, k1, q1, %0;\n\t"                                                     \
            "fma.rn.f32." PTXTYPE " %0, k2, q2, %0;\n\t"                                                     \
            "fma.rn.f32." PTXTYPE " %0, k3, q3, %0;\n\t"                                                     \
            "fma.rn.f32." PTXTYPE " %0, k4, q4, %0;\n\t"                                                     \
            "fma.rn.f32." PTXTYPE " %0, k5, q5, %0;\n\t"                                                     \
            "fma.rn.f32." PTXTYPE " %0, k6, q6, %0;\n\t"                                                     \
            "fma.rn.f32." PTXTYPE " %0, k7, q7, %0;\n\t}"                                                    \
            : "=f"(s)                                                                                        \
            : "r"(k.x), "r"(k.y), "r"(k.z), "r"(k.w), "r"(q.x), "r"(q.y), "r"(q.z), "r"(q.w));              \
        return s;                                                                                            \
    }
L2K_DOT16_MIXED(__nv_bfloat16, "bf16")
L2K_DOT16_MIXED(__half, "f16")
#undef L2K_DOT16_MIXED

// 16 e4m3 cache elements as fp32: e4m3 -> f16 pairs (exact), f16 -> fp32 (exact).
__device__ __forceinline__ void e4m3x16_to_f32(uint4 k, float (&f)[16])
{
    const uint32_t w[4] = {k.x, k.y, k.z, k.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xFFFFu), __NV_E4M3);
        const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&lo));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&hi));
        f[4 * i] = a.x;
        f[4 * i + 1] = a.y;
        f[4 * i + 2] = b.x;
        f[4 * i + 3] = b.y;
    }
}
// Dot product of 16 e4m3 elements of a K row with this lane's 16 q values
// (fp32), as the chain sacc = fma(k_e, q_e, sacc) from 0.
__device__ __forceinline__ float dot16_e4m3(uint4 k, const float *qf)
{
    float kf[16];
    e4m3x16_to_f32(k, kf);
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e)
        s = fmaf(kf[e], qf[e], s);
    return s;
}

// The same dot product with q held as 8 f16 pairs (exact conversions of the
// q values, see score_row_stream): each e4m3 pair widens to an f16 pair and
// each element is the sm_100 mixed-precision fma (f16 operands, fp32
// accumulate), which rounds k*q+s once as fmaf does on the widened values —
// so the result equals dot16_e4m3's bit for bit, at fewer instructions.
__device__ __forceinline__ float dot16_e4m3_h(uint4 k, const uint32_t (&qh)[8])
{
    const uint32_t w[4] = {k.x, k.y, k.z, k.w};
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i)
    {
        const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] & 0xFFFFu), __NV_E4M3);
        const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[i] >> 16), __NV_E4M3);
        const uint32_t k0 = (uint32_t)lo.x | ((uint32_t)lo.y << 16), k1 = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
        asm("{\n\t.reg .b16 a0, a1, b0, b1, c0, c1, d0, d1;\n\t"
            "mov.b32 {a0, a1}, %1;\n\tmov.b32 {b0, b1}, %2;\n\tmov.b32 {c0, c1}, %3;\n\tmov.b32 {d0, d1}, %4;\n\t"
            "fma.rn.f32.f16 %0, a0, b0, %0;\n\tfma.rn.f32.f16 %0, a1, b1, %0;\n\t"
            "fma.rn.f32.f16 %0, c0, d0, %0;\n\tfma.rn.f32.f16 %0, c1, d1, %0;\n\t}"
            : "+f"(s)
            : "r"(k0), "r"(qh[2 * i]), "r"(k1), "r"(qh[2 * i + 1]));
    }
    return s;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }

// Bounded wait on an mbarrier phase: false after ~2 s.
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

// Static shared state of one streaming score row.
struct StreamShared
{
    uint64_t full[kNS];
    uint64_t empty[kNS];
    float2 wstat[kCW];  // per consumer warp: (max, sum of exp) of its logits
    float2 cstat[8];    // per cluster rank: (max, sum of exp), pushed by every rank
    uint64_t xbar;      // completes when the C - 1 peers' pairs have landed in cstat
    uint64_t pvbar;     // PV, rank 0: completes when the C - 1 peers' partial P.V rows have landed
    uint32_t wkv[kCW];  // STEP: per consumer warp, max of the updated lengths
    uint4 knew[32];     // STEP and fresh: the rotated new K row, one 16-byte slice per lane of a row
    float scratch[32];  // (block reductions of the step kernel's other roles)
    int abort_flag;
};

// Dynamic shared memory of one streaming score row: the ring and the logits,
// and for PV rows the per-warp partial P.V rows and rank 0's receive slots
// of the cluster's partial rows (kCW + 8 rows of head_dim floats).
inline size_t stream_smem_bytes(int64_t S, int64_t row_bytes, int C)
{
    const int64_t kb = kBlockBytes / row_bytes;
    const int64_t logit_bytes = ceil_div(ceil_div(S, kb), C) * kb * (int64_t)sizeof(float);
    return (size_t)kNS * kBlockBytes + (size_t)logit_bytes;
}
inline size_t pv_smem_bytes(int64_t head_dim) { return (size_t)(kCW + 8) * (size_t)head_dim * sizeof(float); }

// (max, sum of exp) pairs: the pair of the union of both sets.
__device__ __forceinline__ float2 stat_merge(float2 a, float2 b)
{
    const float m = fmaxf(a.x, b.x);
    if (m == -INFINITY)
        return make_float2(-INFINITY, 0.f);
    const float la = a.x == -INFINITY ? 0.f : a.y * expf(__fsub_rn(a.x, m));
    const float lb = b.x == -INFINITY ? 0.f : b.y * expf(__fsub_rn(b.x, m));
    return make_float2(m, la + lb);
}

__device__ __forceinline__ float2 shfl_xor_stat(float2 v, int off)
{
    return make_float2(__shfl_xor_sync(0xffffffffu, v.x, off), __shfl_xor_sync(0xffffffffu, v.y, off));
}

__device__ __forceinline__ void named_sync_consumers()
{
    asm volatile("bar.sync 1, %0;" ::"n"(kCW * 32) : "memory");
}
// Barrier of the consumer warps that also ORs a per-thread flag: every
// consumer thread gets the same answer, so a decision to leave (on an abort
// flag that another thread may be setting meanwhile) is taken by all of them
// or by none, and no consumer is left waiting at a later named barrier.
__device__ __forceinline__ bool consumers_any(bool v)
{
    uint32_t r;
    asm volatile("{\n\t.reg .pred p, q;\n\t"
                 "setp.ne.u32 p, %1, 0;\n\t"
                 "bar.red.or.pred q, 1, %2, p;\n\t"
                 "selp.u32 %0, 1, 0, q;\n\t}"
                 : "=r"(r)
                 : "r"((uint32_t)v), "n"(kCW * 32)
                 : "memory");
    return r != 0;
}
__device__ __forceinline__ void cluster_arrive_relaxed()
{
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire()
{
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Pushes v into rank `rank`'s copy of *local_slot and signals 8 bytes on
// that rank's copy of *local_bar (st.async with mbarrier complete_tx).
__device__ __forceinline__ void push_stat(float2 *local_slot, uint64_t *local_bar, int rank, float2 v)
{
    uint32_t slot, bar;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(slot) : "r"(smem_addr(local_slot)), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(smem_addr(local_bar)), "r"(rank));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(slot),
                 "f"(v.x), "f"(v.y), "r"(bar)
                 : "memory");
}
// Pushes 4 floats into rank `rank`'s copy of *local_slot (16-byte aligned)
// and signals 16 bytes on that rank's copy of *local_bar.
__device__ __forceinline__ void push_f4(float4 *local_slot, uint64_t *local_bar, int rank, float4 v)
{
    uint32_t slot, bar;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(slot) : "r"(smem_addr(local_slot)), "r"(rank));
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(bar) : "r"(smem_addr(local_bar)), "r"(rank));
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(
                     slot),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
                 : "memory");
}
__device__ __forceinline__ void bulk_store(void *gdst, const void *ssrc, uint32_t bytes)
{
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem_addr(ssrc)),
                 "r"(bytes)
                 : "memory");
}

// Length update of the fused decode step, by the warp that took the last
// ticket (every other CTA has finished reading the old lengths):
// kv_lens += q_lens, max_lens = (max q_len, max kv_len), counter back to 0.
// With `have` (batch <= 32) lane b already holds q_lens[b] / kv_lens[b].
__device__ __forceinline__ void step_update_lens(const StepRowArgs &sa, int lane, bool have, uint32_t pq,
                                                 uint32_t pkv)
{
    uint32_t mq = 0, mkv = 0;
    if (have)
    {
        if (lane < sa.batch)
        {
            sa.kv_lens[lane] = pkv + pq;
            mq = pq;
            mkv = pkv + pq;
        }
    }
    else
    {
        for (int64_t b = lane; b < sa.batch; b += 32)
        {
            const uint32_t q = sa.q_lens[b];
            const uint32_t kv = sa.kv_lens[b] + q;
            sa.kv_lens[b] = kv;
            mq = max(mq, q);
            mkv = max(mkv, kv);
        }
    }
    mq = warp_max_u32(mq);
    mkv = warp_max_u32(mkv);
    if (lane == 0)
    {
        sa.max_lens[0] = mq;
        sa.max_lens[1] = mkv;
        *sa.counter = 0u;
    }
}

// Takes this CTA's ticket (lane 0 of the calling warp) and, if it is the
// last one, performs the length update with this warp. Called after a
// barrier that follows every read of the old lengths in this CTA; the
// acq_rel ticket orders those reads before the last CTA's writes.
__device__ __forceinline__ void step_ticket(const StepRowArgs &sa, int lane, bool have, uint32_t pq, uint32_t pkv)
{
    __syncwarp();
    uint32_t t = 0;
    if (lane == 0)
        asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], 1;" : "=r"(t) : "l"(sa.counter) : "memory");
    __syncwarp();
    t = __shfl_sync(0xffffffffu, t, 0);
    if (t == gridDim.x - 1u)
        step_update_lens(sa, lane, have, pq, pkv);
}

// Start of key block g of the (b, kv head) plane: in the contiguous cache
// (B, Hkv, S, hd), or page block_table[b][g] of a paged one (a page id past
// the pool is recorded as an error and read as page 0, so nothing outside
// the pool is touched).
template <int KB, int ROW_BYTES>
__device__ __forceinline__ const char *block_ptr(const DecodeArgs &a, const void *cache, int64_t b, int64_t kvh,
                                                 int64_t g, int *err)
{
    const char *base = static_cast<const char *>(cache);
    if (a.block_table)
    {
        int64_t page = a.block_table[b * a.max_pages + g];
        if (page >= a.num_pages)
        {
            atomicCAS(err, 0, 0x206);
            page = 0;
        }
        return base + (page * a.Hkv + kvh) * (int64_t)KB * ROW_BYTES;
    }
    return base + ((b * a.Hkv + kvh) * a.S + g * KB) * (int64_t)ROW_BYTES;
}

// L2 prefetch of this rank's first two key blocks of the (b, kv head) plane,
// issued before the lengths are known (they are needed to know how many
// blocks there are): the blocks exist whatever the length, and the copies
// that follow find them in L2 instead of waiting a DRAM round trip.
template <int KB, int ROW_BYTES>
__device__ __forceinline__ void prefetch_first_blocks(const DecodeArgs &a, int64_t b, int64_t kvh, int c, int C,
                                                      int *err)
{
    for (int i = 0; i < 2; ++i)
    {
        const int64_t g = c + (int64_t)C * i;
        if (g * KB >= a.S)
            break;
        const uint32_t bytes = (uint32_t)(min((int64_t)KB, a.S - g * KB) * ROW_BYTES);
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(block_ptr<KB, ROW_BYTES>(a, a.k, b, kvh, g,
                                                                                                   err)),
                     "r"(bytes)
                     : "memory");
    }
}

// The P.V part of a PV row, run by the consumer warps after the row's
// (max, sum of exp) is known: probabilities in place of this CTA's logits,
// their store (keys in [n_keys, M) as 0), the fold of p_j * V_j over this
// CTA's V blocks (ring sequences n_mine + i, i < n_mine), and the reduction
// lanes -> warps -> cluster ranks, the ranks' rows summed by rank 0 in rank
// order and written to qkv[row].
//
// In the fused decode step the V row at this step's position is still being
// written to the cache (by the CTA that owns its block), so the warp that
// folds that block replaces the row in shared memory with the new V row
// (vnew_src, this lane's 16-byte slice read at the start) before folding;
// patch_pos < 0 when there is nothing to patch.
template <typename T, int LPR, typename TC = T>
__device__ __forceinline__ void pv_row(const DecodeArgs &a, const int64_t row, const RowInfo &ri,
                                       const int64_t n_keys, const int n_mine, const int c, const int C,
                                       const float2 row_stat, uint8_t *smem, StreamShared &sh, int *err,
                                       const int64_t patch_pos = -1, const T *vnew_src = nullptr)
{
    constexpr bool F8 = std::is_same<TC, __nv_fp8_e4m3>::value;
    constexpr int N = F8 ? 16 : Vec16<T>::N; // V elements per lane slice (16 bytes of a V row)
    constexpr int ROW_BYTES = LPR * 16;
    constexpr int KB = kBlockBytes / ROW_BYTES;
    constexpr int HALF = KB / 2;
    constexpr int RPL = 32 / LPR;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    float *logits = reinterpret_cast<float *>(smem + kNS * kBlockBytes);
    const int64_t n_logits = ((a.S + KB - 1) / KB + C - 1) / C * KB;
    float *pv_w = logits + n_logits;   // kCW partial rows of this CTA's warps
    float *pv_r = pv_w + kCW * a.hd;   // rank 0: slot r receives rank r's partial row
    const bool gather = C > 1 && c == 0;
    if (gather && tid == 0)
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&sh.pvbar)),
                     "r"((uint32_t)((C - 1) * a.hd * (int64_t)sizeof(float)))
                     : "memory");
    auto leave = [&]() {
        // Rank 0 lets peer rows still on their way land before it leaves.
        if (gather)
            bar_wait(smem_addr(&sh.pvbar), 0);
    };
    // The warp (stage, half) that will fold the V block holding patch_pos
    // reads its slice of the new V row now, ahead of need.
    int patch_i = -1, patch_r = -1;
    uint4 vnew = make_uint4(0u, 0u, 0u, 0u);
    if (patch_pos >= 0)
    {
        const int64_t g = patch_pos / KB;
        const int rib = (int)(patch_pos - g * KB);
        if (g % C == c && (g - c) / C < n_mine && (int)((n_mine + (g - c) / C) % kNS) == warp % kNS &&
            rib / HALF == warp / kNS)
        {
            patch_i = (int)((g - c) / C);
            patch_r = rib - (warp / kNS) * HALF;
            if (lane < LPR)
                vnew = ldg_keep(vnew_src + lane * (16 / (int)sizeof(T)));
        }
    }
    if (consumers_any(sh.abort_flag != 0))
        return leave();

    const float Mx = row_stat.x;
    const float inv = __fdiv_rn(1.f, __fadd_rn(row_stat.y, kSoftmaxEps));
    for (int e = tid; e < n_mine * KB; e += kCW * 32)
    {
        const int64_t j = (c + (int64_t)C * (e / KB)) * KB + e % KB;
        logits[e] = j < n_keys ? __fmul_rn(expf(__fsub_rn(logits[e], Mx)), inv) : 0.f;
    }
    named_sync_consumers();
    {
        T *out_row = static_cast<T *>(a.qk) + row * a.S;
        const int64_t n_wblk = (ri.M + KB - 1) / KB; // blocks with keys < M
        const int n_wmine = n_wblk > c ? (int)((n_wblk - c + C - 1) / C) : 0;
        for (int e = tid; e < n_wmine * KB; e += kCW * 32)
        {
            const int ib = e / KB;
            const int64_t j = (c + (int64_t)C * ib) * KB + e % KB;
            if (j < ri.M)
                out_row[j] = from_f<T>(ib < n_mine ? logits[e] : 0.f);
        }
    }

    float acc[N];
#pragma unroll
    for (int e = 0; e < N; ++e)
        acc[e] = 0.f;
    {
        const int st = warp % kNS, hf = warp / kNS, sub = lane % LPR;
        const uint8_t *stage = smem + st * kBlockBytes + hf * HALF * ROW_BYTES + sub * 16;
        for (int i = ((st - n_mine) % kNS + kNS) % kNS; i < n_mine; i += kNS)
        {
            const int n = n_mine + i; // ring sequence: n % kNS == st
            if (!bar_wait(smem_addr(&sh.full[st]), (n / kNS) & 1))
            {
                atomicCAS(err, 0, 0x204);
                sh.abort_flag = 1;
                break;
            }
            if (i == patch_i)
            {
                // this step's V row: stale in the cache copy, replaced by the new row
                if (lane < LPR)
                {
                    *reinterpret_cast<uint4 *>(const_cast<uint8_t *>(stage) + patch_r * ROW_BYTES) = vnew;
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); // before the stage is refilled
                }
                __syncwarp();
            }
            const int64_t valid = n_keys - (c + (int64_t)C * i) * KB - hf * HALF; // rows of this half with keys
            const float *pr = logits + i * KB + hf * HALF;
            auto fold = [&](int r) {
                const float p = pr[r];
                if constexpr (F8)
                {
                    float vf[16];
                    e4m3x16_to_f32(*reinterpret_cast<const uint4 *>(stage + r * ROW_BYTES), vf);
#pragma unroll
                    for (int e = 0; e < N; ++e)
                        acc[e] = fmaf(p, vf[e], acc[e]);
                }
                else
                {
                    const Vec16<T> vv = as_vec<T>(*reinterpret_cast<const uint4 *>(stage + r * ROW_BYTES));
#pragma unroll
                    for (int e = 0; e < N; ++e)
                        acc[e] = fmaf(p, to_f(vv.v[e]), acc[e]);
                }
            };
            if (valid >= HALF)
            {
#pragma unroll 4
                for (int r = lane / LPR; r < HALF; r += RPL)
                    fold(r);
            }
            else
            {
                for (int r = lane / LPR; r < valid; r += RPL)
                    fold(r);
            }
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&sh.empty[st])) : "memory");
        }
    }
#pragma unroll
    for (int off = LPR; off < 32; off <<= 1)
#pragma unroll
        for (int e = 0; e < N; ++e)
            acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], off);
    if (lane < LPR)
    {
#pragma unroll
        for (int e = 0; e < N; e += 4)
            *reinterpret_cast<float4 *>(pv_w + warp * a.hd + lane * N + e) =
                make_float4(acc[e], acc[e + 1], acc[e + 2], acc[e + 3]);
    }
    if (consumers_any(sh.abort_flag != 0)) // (also the barrier after the partial rows)
        return leave();

    const int nq = (int)(a.hd / 4);
    if (tid < nq)
    {
        float4 sum = reinterpret_cast<const float4 *>(pv_w)[tid];
#pragma unroll
        for (int w = 1; w < kCW; ++w)
        {
            const float4 x = reinterpret_cast<const float4 *>(pv_w + w * a.hd)[tid];
            sum = make_float4(sum.x + x.x, sum.y + x.y, sum.z + x.z, sum.w + x.w);
        }
        if (C > 1 && c != 0)
        {
            push_f4(reinterpret_cast<float4 *>(pv_r + c * a.hd) + tid, &sh.pvbar, 0, sum);
            return;
        }
        if (gather)
        {
            if (!bar_wait(smem_addr(&sh.pvbar), 0))
            {
                atomicCAS(err, 0, 0x205);
                return;
            }
            for (int r = 1; r < C; ++r)
            {
                const float4 x = reinterpret_cast<const float4 *>(pv_r + r * a.hd)[tid];
                sum = make_float4(sum.x + x.x, sum.y + x.y, sum.z + x.z, sum.w + x.w);
            }
        }
        if constexpr (F8)
            sum = make_float4(__fmul_rn(sum.x, a.v_scale), __fmul_rn(sum.y, a.v_scale), __fmul_rn(sum.z, a.v_scale),
                              __fmul_rn(sum.w, a.v_scale));
        T *o = static_cast<T *>(a.qkv) + row * a.hd + 4 * tid;
        o[0] = from_f<T>(sum.x);
        o[1] = from_f<T>(sum.y);
        o[2] = from_f<T>(sum.z);
        o[3] = from_f<T>(sum.w);
    }
}

// One score row on this CTA's share of its keys (see the file comment).
// head_dim * sizeof(T) = LPR * 16 bytes, LPR in {4, 8, 16, 32}. Every CTA of
// the cluster calls it for the same row. `err` receives the first timeout
// code.
//
// Latency structure (what a small batch waits for): every independent load
// is issued first (lengths, the q/k slices, the batch's lengths for the row
// width); the producer lane initializes the ring and issues the first kNS
// copies without waiting for the other warps; the consumers keep an online
// (max, sum of exp) per lane while they compute logits, so the CTA's
// statistics need one barrier; cluster peers push their statistics into
// each other's shared memory before a single cluster barrier; probabilities
// are staged in the (now idle) ring and written with cp.async.bulk stores.
//
// PV rows (attention output, flash-decode style; also in the fused decode
// step) also stream the V rows of the same blocks: once its K blocks are issued the producer lane continues
// with the V blocks into the same ring (the first kNS while the consumers
// still finish the keys), and after the cluster's statistics are known the
// consumers turn their logits into probabilities in place, store them, and
// fold p_j * V_j over their V blocks from shared memory (each lane a 16-byte
// slice of head_dim). Lanes, warps and then the cluster's CTAs are summed in
// a fixed order (peers push their partial rows into rank 0's shared memory
// with st.async), so the output does not depend on timing.
// DEV_ANGLES (STEP): whether cos/sin may be evaluated on the device for
// positions the host table does not cover. A launch whose every position is in
// the table passes false: the device formula (powf, cosf, sinf, whose slow
// paths are calls) is then not compiled into the kernel, which lets the
// register allocator keep the key loop free of spills.
template <typename T, int LPR, bool STEP, bool PV = false, typename TC = T, bool DEV_ANGLES = true>
__device__ __forceinline__ void score_row_stream(const DecodeArgs &a, const StepRowArgs &sa, const int64_t row,
                                                 cg::cluster_group &cluster, uint8_t *smem, StreamShared &sh,
                                                 int *err)
{
    // TC: the cache element type. fp8 (e4m3) caches hold 16 elements per
    // 16-byte lane slice; the logits scale includes K's dequantization scale.
    constexpr bool F8 = std::is_same<TC, __nv_fp8_e4m3>::value;
    static_assert(!(F8 && STEP), "the fused decode step keeps 16-bit or fp32 caches");
    constexpr int N = F8 ? 16 : Vec16<T>::N;
    constexpr int ROW_BYTES = LPR * 16;
    constexpr int KB = kBlockBytes / ROW_BYTES; // K rows per block
    constexpr int HALF = KB / 2;                // rows per consumer warp per block
    constexpr int R = LPR < 8 ? LPR : 8;
    constexpr int RPL = 32 / LPR;               // K rows per warp-wide read
    constexpr int ROWS = R * RPL;               // K rows per multi_reduce step
    static_assert(HALF % ROWS == 0, "half block must hold whole steps");
    float *logits = reinterpret_cast<float *>(smem + kNS * kBlockBytes);

    const int C = (int)cluster.num_blocks();
    const int c = (int)cluster.block_rank();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sub = lane % LPR;
    const int64_t i0 = (int64_t)sub * N; // this lane's 16-byte slice of a head
    // Cluster barrier phase 0 (arrive now, wait before the first remote
    // write): every peer has started and initialized its barriers. The
    // producer warp arrives after initializing this CTA's barriers.
    if (C > 1 && warp < kCW)
        cluster_arrive_relaxed();

    // ---- every independent load first ----
    RowInfo ri;
    bool fresh = false;          // STEP: this step's q and K row are rotated here
    uint32_t pos = 0, kv_new = 0;
    uint32_t mx_kv = 0;          // STEP: max updated length over this thread's sequences
    uint32_t pq = 0, pkv = 0;    // STEP, producer warp, batch <= 32: lengths of sequence `lane`
    uint4 qa = make_uint4(0u, 0u, 0u, 0u), qb = qa, ka = qa, kb = qa; // STEP: q / k slices and rotation partners
    uint4 va = qa; // STEP, the lanes that append: this lane's slice of the new V row
    const bool half_pair = sa.pairing != L2K_ROPE_INTERLEAVED;
    const int64_t hh = a.hd / 2;
    const int64_t j0 = half_pair ? (i0 < hh ? i0 : i0 - hh) : i0;
    if constexpr (STEP)
    {
        ri.i = 0;
        ri.b = row / a.Hq;
        ri.h = row - ri.b * a.Hq;
        const uint32_t kvl = sa.kv_lens[ri.b], ql = sa.q_lens[ri.b];
        const uint8_t done = sa.is_done[ri.b];
        if (warp < kCW)
        {
            const T *src = static_cast<const T *>(sa.qkv) + ri.b * sa.qkv_stride;
            const T *qh = src + ri.h * a.hd, *kh = src + (a.Hq + ri.h / a.group) * a.hd;
            qa = ldg_keep(qh + j0);
            ka = ldg_keep(kh + j0);
            if (half_pair)
            {
                qb = ldg_keep(qh + j0 + hh);
                kb = ldg_keep(kh + j0 + hh);
            }
            if (c == 0 && warp == 0 && lane < LPR && ri.h % a.group == 0)
                va = ldg_keep(src + (a.Hq + a.Hkv + ri.h / a.group) * a.hd + i0);
            for (int64_t b = tid; b < sa.batch; b += kCW * 32)
                mx_kv = max(mx_kv, sa.kv_lens[b] + sa.q_lens[b]);
        }
        else
        {
            if (sa.batch <= 32 && lane < sa.batch)
            {
                pq = sa.q_lens[lane];
                pkv = sa.kv_lens[lane];
            }
            if (lane == 0)
                prefetch_first_blocks<KB, ROW_BYTES>(a, ri.b, ri.h / a.group, c, C, err);
        }
        kv_new = kvl + ql;
        pos = kv_new - 1u;
        fresh = !done && (int64_t)pos < a.S;
        ri.limit = min((int64_t)kv_new, a.S) - 1;
        ri.active = true;
        ri.M = 0; // the largest updated length, after the key loop
    }
    else
    {
        if (warp == kCW && lane == 0)
        {
            const int64_t bh = row / a.Qc, b = bh / a.Hq;
            prefetch_first_blocks<KB, ROW_BYTES>(a, b, (bh - b * a.Hq) / a.group, c, C, err);
        }
        ri = row_info(a, row);
        if (!ri.active)
        {
            if (C > 1)
            {
                if (warp == kCW)
                    cluster_arrive_relaxed();
                cluster_wait_acquire(); // (the whole cluster shares the row and leaves together)
            }
            return;
        }
    }
    const int64_t kvh = ri.h / a.group;
    const int64_t n_keys = max((int64_t)0, ri.limit + 1);
    const int64_t n_blk = (n_keys + KB - 1) / KB; // blocks holding valid keys
    const int n_mine = n_blk > c ? (int)((n_blk - c + C - 1) / C) : 0;

    // Ring sequence number i: K block i for i < n_mine, V block i - n_mine
    // after (PV rows); sequence i lands in stage i % kNS.
    auto issue = [&](int i) {
        const int st = i % kNS;
        const bool is_v = PV && i >= n_mine;
        // Whole blocks (up to the cache end): rows past kv_len are computed and
        // masked, which keeps the consumers' inner loop free of bounds checks.
        const int64_t g = c + (int64_t)C * (is_v ? i - n_mine : i);
        const uint32_t bytes = (uint32_t)(min((int64_t)KB, a.S - g * KB) * ROW_BYTES);
        const uint32_t bar = smem_addr(&sh.full[st]);
        const char *src = block_ptr<KB, ROW_BYTES>(a, is_v ? a.v : a.k, ri.b, kvh, g, err);
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
        asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                         smem_addr(smem + st * kBlockBytes)),
                     "l"(src), "r"(bytes), "r"(bar)
                     : "memory");
    };
    // Producer lane: issues sequences up to `end`, each after its stage's
    // previous contents were consumed (bounded waits; stops on abort).
    auto issue_until = [&](int &n_iss, int end) {
        for (; n_iss < end && !sh.abort_flag; ++n_iss)
        {
            const int st = n_iss % kNS;
            if (n_iss >= kNS && !bar_wait(smem_addr(&sh.empty[st]), ((n_iss / kNS) - 1) & 1))
            {
                atomicCAS(err, 0, 0x201);
                sh.abort_flag = 1;
                break;
            }
            issue(n_iss);
        }
    };

    int n_issued = 0; // producer lane only
    float qf[N];
    uint32_t qh[8] = {};  // F8: this lane's q slice as f16 pairs (when q_f16)
    bool q_f16 = false;
    uint4 qraw;                              // the same slice as stored (16-bit types: the mixed fma's operand)
    if (warp == kCW)
    {
        if (lane == 0)
        {
            for (int i = 0; i < kNS; ++i)
            {
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sh.full[i])) : "memory");
                asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(&sh.empty[i])), "r"(kCW / kNS)
                             : "memory");
            }
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sh.xbar)) : "memory");
            if constexpr (PV)
                asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(&sh.pvbar)) : "memory");
            sh.abort_flag = 0;
            asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
            for (; n_issued < n_mine && n_issued < kNS; ++n_issued)
                issue(n_issued);
        }
        __syncwarp();
        if (C > 1)
            cluster_arrive_relaxed();
    }
    else
    {
        bool q_done = false;
        if constexpr (STEP)
        {
            if (fresh)
            {
                // RoPE at pos of this lane's q and k slices; cos/sin shared by both,
                // from the table (16-byte loads) when it covers the position.
                constexpr int NPMAX = N;                  // pairs per lane: N (half) or N / 2 (interleaved)
                const int np = half_pair ? N : N / 2;
                const int64_t p0 = half_pair ? j0 : i0 / 2; // first pair index
                float cs[2 * NPMAX];
                if (sa.table && kv_new <= 4096u && (int64_t)pos < sa.table_pos)
                {
                    const float4 *t4 = reinterpret_cast<const float4 *>(sa.table + (int64_t)pos * hh + p0);
#pragma unroll
                    for (int v = 0; v < NPMAX / 2; ++v)
                        if (v < np / 2)
                        {
                            const float4 t = __ldg(t4 + v);
                            cs[4 * v] = t.x;
                            cs[4 * v + 1] = t.y;
                            cs[4 * v + 2] = t.z;
                            cs[4 * v + 3] = t.w;
                        }
                }
                else if constexpr (DEV_ANGLES)
                {
#pragma unroll
                    for (int e = 0; e < NPMAX; ++e)
                        if (e < np)
                            rope_cos_sin_device(p0 + e, a.hd, pos, kv_new, cs[2 * e], cs[2 * e + 1]);
                }
                else
                {
                    // unreachable when the host's coverage check holds: recorded, not guessed
                    if (lane == 0)
                        atomicCAS(err, 0, 0x204);
#pragma unroll
                    for (int e = 0; e < 2 * NPMAX; ++e)
                        cs[e] = 0.f;
                }
                Vec16<T> qo, ko;
                if (!half_pair)
                {
                    const Vec16<T> xq = as_vec<T>(qa), xk = as_vec<T>(ka);
#pragma unroll
                    for (int e = 0; e < N / 2; ++e)
                    {
                        const float cc = cs[2 * e], ss = cs[2 * e + 1];
                        qo.v[2 * e] = from_f<T>(rope_o0(cc, ss, to_f(xq.v[2 * e]), to_f(xq.v[2 * e + 1])));
                        qo.v[2 * e + 1] = from_f<T>(rope_o1(cc, ss, to_f(xq.v[2 * e]), to_f(xq.v[2 * e + 1])));
                        ko.v[2 * e] = from_f<T>(rope_o0(cc, ss, to_f(xk.v[2 * e]), to_f(xk.v[2 * e + 1])));
                        ko.v[2 * e + 1] = from_f<T>(rope_o1(cc, ss, to_f(xk.v[2 * e]), to_f(xk.v[2 * e + 1])));
                    }
                }
                else
                {
                    const bool lo = i0 < hh;
                    const Vec16<T> q0 = as_vec<T>(qa), q1 = as_vec<T>(qb), k0 = as_vec<T>(ka), k1 = as_vec<T>(kb);
#pragma unroll
                    for (int e = 0; e < N; ++e)
                    {
                        const float cc = cs[2 * e], ss = cs[2 * e + 1];
                        const float qx0 = to_f(q0.v[e]), qx1 = to_f(q1.v[e]), kx0 = to_f(k0.v[e]), kx1 = to_f(k1.v[e]);
                        qo.v[e] = from_f<T>(lo ? rope_o0(cc, ss, qx0, qx1) : rope_o1(cc, ss, qx0, qx1));
                        ko.v[e] = from_f<T>(lo ? rope_o0(cc, ss, kx0, kx1) : rope_o1(cc, ss, kx0, kx1));
                    }
                }
#pragma unroll
                for (int e = 0; e < N; ++e)
                    qf[e] = to_f(qo.v[e]);
                qraw = as_u4(qo);
                if (warp == 0 && lane < LPR)
                    sh.knew[sub] = as_u4(ko); // (read in the key loop: not held in registers across it)
                if (c == 0 && warp == 0 && lane < LPR)
                {
                    stg(static_cast<T *>(sa.q_out) + row * a.hd + i0, as_u4(qo));
                    // Append K and V at pos (one CTA per kv head). A copy of the
                    // block holding pos may read the row before or after this
                    // store: every reader overwrites the row in its shared-memory
                    // copy with the rotated row (the key loop below).
                    if (ri.h % a.group == 0)
                    {
                        // contiguous (B, Hkv, S, hd), or the page holding pos (a page past
                        // the pool is not written; its streamed copy records the error)
                        const int64_t kvh0 = ri.h / a.group;
                        int64_t crow = ((ri.b * a.Hkv + kvh0) * a.S + pos) * a.hd + i0;
                        if (a.block_table)
                        {
                            const int64_t page = a.block_table[ri.b * a.max_pages + (int64_t)pos / KB];
                            crow = page < a.num_pages ? ((page * a.Hkv + kvh0) * KB + (int64_t)pos % KB) * a.hd + i0
                                                      : -1;
                        }
                        if (crow >= 0)
                        {
                            stg(static_cast<T *>(sa.k_cache) + crow, as_u4(ko));
                            stg(static_cast<T *>(sa.v_cache) + crow, va);
                        }
                    }
                }
                q_done = true;
            }
        }
        if (!q_done)
        {
            const T *qrow = static_cast<const T *>(a.q) + row * a.hd;
            if constexpr (F8)
            {
                // 16 q values (the lane's slice of the row) as fp32
                constexpr int QN = Vec16<T>::N;
#pragma unroll
                for (int part = 0; part < N / QN; ++part)
                {
                    const Vec16<T> qv = as_vec<T>(ldg_keep(qrow + i0 + part * QN));
#pragma unroll
                    for (int e = 0; e < QN; ++e)
                        qf[part * QN + e] = to_f(qv.v[e]);
                }
                qraw = make_uint4(0u, 0u, 0u, 0u);
                if constexpr (F8)
                {
                    // q as f16 pairs when every value of the slice converts exactly
                    // (zero, or a normal f16 magnitude and no more than 11
                    // significant bits, which 16-bit q always has); otherwise the
                    // fp32 dot product is used.
                    bool exact = true;
#pragma unroll
                    for (int e = 0; e < 16; e += 2)
                    {
                        const __half2 h = __floats2half2_rn(qf[e], qf[e + 1]);
                        const float2 back = __half22float2(h);
                        exact = exact && back.x == qf[e] && back.y == qf[e + 1] &&
                                (qf[e] == 0.f || fabsf(qf[e]) >= 6.103515625e-05f) &&
                                (qf[e + 1] == 0.f || fabsf(qf[e + 1]) >= 6.103515625e-05f);
                        qh[e / 2] = *reinterpret_cast<const uint32_t *>(&h);
                    }
                    q_f16 = exact;
                }
            }
            else
            {
                qraw = STEP ? ldg_coherent(qrow + i0) : ldg_keep(qrow + i0);
                const Vec16<T> qv = as_vec<T>(qraw);
#pragma unroll
                for (int e = 0; e < N; ++e)
                    qf[e] = to_f(qv.v[e]);
            }
        }
    }
    if constexpr (STEP)
    {
        // the largest updated length, reduced now (not held in registers across the key loop)
        if (warp < kCW)
        {
            const uint32_t wm = warp_max_u32(mx_kv);
            if (lane == 0)
                sh.wkv[warp] = wm;
        }
    }
    __syncthreads(); // the ring is initialized; q is ready

    float2 st_l = make_float2(-INFINITY, 0.f); // online (max, sum of exp) of this lane's logits
    if (warp == kCW)
    {
        if (lane == 0)
        {
            for (; n_issued < n_mine && !sh.abort_flag; ++n_issued)
            {
                const int st = n_issued % kNS;
                if (!bar_wait(smem_addr(&sh.empty[st]), ((n_issued / kNS) - 1) & 1))
                {
                    atomicCAS(err, 0, 0x201);
                    sh.abort_flag = 1;
                    break;
                }
                issue(n_issued);
            }
            if constexpr (PV) // the first V blocks, into stages the keys free
                issue_until(n_issued, n_mine + min(n_mine, kNS));
        }
        if (C > 1)
        {
            __syncwarp();
            cluster_wait_acquire(); // (phase 0)
        }
    }
    else
    {
        if (C > 1)
            cluster_wait_acquire(); // phase 0: every peer has started (waited while the first blocks land)
        const int st = warp % kNS, hf = warp / kNS; // ring stage, half of the block
        // STEP: the ring sequence number and stage row of this step's key when
        // it falls in this warp's half of one of this rank's blocks (else -1).
        int patch_i = -1, patch_row = 0;
        if constexpr (STEP)
        {
            if (fresh)
            {
                const int64_t gp = (int64_t)pos / KB;
                const int r = (int)((int64_t)pos - gp * KB);
                if (gp % C == c && r / HALF == hf)
                {
                    patch_i = (int)(gp / C);
                    patch_row = r;
                }
            }
        }
        const uint8_t *stage = smem + st * kBlockBytes + (hf * HALF + lane / LPR) * ROW_BYTES + sub * 16;
        for (int i = st; i < n_mine; i += kNS)
        {
            if (!bar_wait(smem_addr(&sh.full[st]), (i / kNS) & 1))
            {
                atomicCAS(err, 0, 0x202);
                sh.abort_flag = 1;
                break;
            }
            const int64_t g = c + (int64_t)C * i;
            if constexpr (STEP)
            {
                // The block holding this step's key: its cache row is stale (or
                // being written) — use the rotated row instead.
                if (i == patch_i)
                {
                    if (lane < LPR)
                    {
                        *reinterpret_cast<uint4 *>(smem + st * kBlockBytes + patch_row * ROW_BYTES + sub * 16) =
                            sh.knew[sub];
                        // the next bulk copy into this stage must see the generic writes ordered
                        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    }
                    __syncwarp();
                }
            }
            const int64_t valid = n_keys - g * KB - hf * HALF; // rows of this half below kv_len
#pragma unroll
            for (int base = 0; base < HALF; base += ROWS)
            {
                float part[R];
#pragma unroll
                for (int j = 0; j < R; ++j)
                {
                    const uint4 kraw = *reinterpret_cast<const uint4 *>(stage + (base + j * RPL) * ROW_BYTES);
                    if constexpr (F8)
                        part[j] = q_f16 ? dot16_e4m3_h(kraw, qh) : dot16_e4m3(kraw, qf);
                    else
                        part[j] = dot16<T>(kraw, qraw, qf);
                }
                int idx;
                const float dot = multi_reduce<R, LPR>(part, lane, idx);
                const int rr = base + idx * RPL + lane / LPR;
                if ((lane & (LPR / R - 1)) == 0)
                {
                    const float x = __fmul_rn(dot, a.scale);
                    const bool ok = rr < valid;
                    logits[i * KB + hf * HALF + rr] = ok ? x : -INFINITY;
                    if (ok)
                    {
                        if (x > st_l.x)
                        {
                            st_l.y = st_l.y * expf(__fsub_rn(st_l.x, x)) + 1.f;
                            st_l.x = x;
                        }
                        else
                            st_l.y += expf(__fsub_rn(x, st_l.x));
                    }
                }
            }
            __syncwarp();
            if (lane == 0)
                asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(&sh.empty[st])) : "memory");
        }
        // warp statistics
#pragma unroll
        for (int off = 16; off > 0; off >>= 1)
            st_l = stat_merge(st_l, shfl_xor_stat(st_l, off));
        if (lane == 0)
            sh.wstat[warp] = st_l;
    }
    __syncthreads(); // logits and warp statistics are complete
    if (sh.abort_flag && warp == kCW && lane == 0)
    {
        // A wait expired: let this CTA's copies still in flight land before it
        // leaves (each wait bounded again).
        for (int i = max(0, n_issued - kNS); i < n_issued; ++i)
            bar_wait(smem_addr(&sh.full[i % kNS]), (i / kNS) & 1);
    }

    // CTA statistics (every thread, from the 8 warp pairs), then the cluster's.
    float2 cta = sh.wstat[0];
#pragma unroll
    for (int w = 1; w < kCW; ++w)
        cta = stat_merge(cta, sh.wstat[w]);
    if constexpr (STEP)
    {
        uint32_t m = sh.wkv[0];
#pragma unroll
        for (int w = 1; w < kCW; ++w)
            m = max(m, sh.wkv[w]);
        ri.M = min((int64_t)m, a.S);
    }
    if (warp == kCW)
    {
        if (STEP)
            step_ticket(sa, lane, sa.batch <= 32, pq, pkv);
        if constexpr (PV)
        {
            if (lane == 0)
            {
                // The remaining V blocks, as the consumers free stages; then every
                // copy this CTA issued has landed before it can leave (on the
                // normal path the consumers have waited for each of them too).
                issue_until(n_issued, 2 * n_mine);
                for (int i = max(0, n_issued - kNS); i < n_issued; ++i)
                    bar_wait(smem_addr(&sh.full[i % kNS]), (i / kNS) & 1);
            }
        }
        return;
    }
    float2 row_stat = cta;
    if (C > 1)
    {
        // Each rank pushes its pair into every peer's cstat[c] with st.async,
        // which completes 8 bytes of transaction on the peer's xbar; a rank's
        // xbar completes when its C - 1 peers' pairs have landed.
        if (warp == 0)
        {
            if (lane < C && lane != c)
                push_stat(&sh.cstat[c], &sh.xbar, lane, cta);
            if (lane == 0)
            {
                sh.cstat[c] = cta;
                asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(&sh.xbar)),
                             "r"((uint32_t)(8 * (C - 1)))
                             : "memory");
            }
        }
        if (!bar_wait(smem_addr(&sh.xbar), 0))
        {
            atomicCAS(err, 0, 0x203);
            sh.abort_flag = 1;
        }
        row_stat = sh.cstat[0];
        for (int r = 1; r < C; ++r)
            row_stat = stat_merge(row_stat, sh.cstat[r]);
    }
    if constexpr (PV)
    {
        if constexpr (STEP)
        {
            const T *vsrc = static_cast<const T *>(sa.qkv) + ri.b * sa.qkv_stride + (a.Hq + a.Hkv + kvh) * a.hd;
            pv_row<T, LPR>(a, row, ri, n_keys, n_mine, c, C, row_stat, smem, sh, err, fresh ? (int64_t)pos : -1,
                           vsrc);
        }
        else
            pv_row<T, LPR, TC>(a, row, ri, n_keys, n_mine, c, C, row_stat, smem, sh, err);
        return;
    }
    if (consumers_any(sh.abort_flag != 0))
        return;

    // Probabilities p = exp(x - M) / (L + eps); keys in [n_keys, M) are
    // written as 0. Long rows are staged in the ring (idle now) and stored
    // with cp.async.bulk; short ones directly.
    const float Mx = row_stat.x;
    const float inv = __fdiv_rn(1.f, __fadd_rn(row_stat.y, kSoftmaxEps));
    T *out_row = static_cast<T *>(a.qk) + row * a.S;
    T *stage_out = reinterpret_cast<T *>(smem);
    constexpr int kChunkBlocks = kNS * kBlockBytes / (KB * (int)sizeof(T));
    const int64_t n_wblk = (ri.M + KB - 1) / KB; // blocks with keys < M
    const int n_wmine = n_wblk > c ? (int)((n_wblk - c + C - 1) / C) : 0;
    if (!a.bulk_out || (int64_t)n_wmine * KB <= 4 * kCW * 32)
    {
        // Few probabilities per thread (or an unaligned row): direct stores,
        // coalesced within each block, no staging.
        for (int e = tid; e < n_wmine * KB; e += kCW * 32)
        {
            const int ib = e / KB, r = e % KB;
            const int64_t j = (c + (int64_t)C * ib) * KB + r;
            if (j >= ri.M)
                continue;
            float p = 0.f;
            if (ib < n_mine && j < n_keys)
                p = __fmul_rn(expf(__fsub_rn(logits[ib * KB + r], Mx)), inv);
            out_row[j] = from_f<T>(p);
        }
        return;
    }
    for (int b0 = 0; b0 < n_wmine; b0 += kChunkBlocks)
    {
        const int nb = min(kChunkBlocks, n_wmine - b0);
        if (b0 > 0)
        {
            if (tid == 0)
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            named_sync_consumers();
        }
        for (int e = tid; e < nb * KB; e += kCW * 32)
        {
            const int ib = b0 + e / KB, r = e % KB;
            const int64_t j = (c + (int64_t)C * ib) * KB + r;
            float p = 0.f;
            if (ib < n_mine && j < n_keys)
                p = __fmul_rn(expf(__fsub_rn(logits[ib * KB + r], Mx)), inv);
            stage_out[e] = from_f<T>(p);
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        named_sync_consumers();
        if (tid == 0)
        {
            // C == 1: the chunk is one contiguous range of the row; else one store per block
            const int runs = C == 1 ? 1 : nb;
            for (int u = 0; u < runs; ++u)
            {
                const int64_t g = c + (int64_t)C * (b0 + u);
                const int64_t n = min((int64_t)(C == 1 ? nb * KB : KB), ri.M - g * KB);
                const uint32_t bytes = (uint32_t)(n * (int64_t)sizeof(T)) & ~15u;
                const T *s0 = stage_out + (int64_t)u * KB;
                if (bytes)
                    bulk_store(out_row + g * KB, s0, bytes);
                for (int64_t k = bytes / sizeof(T); k < n; ++k)
                    out_row[g * KB + k] = s0[k];
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
    if (tid == 0)
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); // the stage must outlive the reads
}

} // namespace
} // namespace l2k
