// RoPE fused with the KV-cache append, for decode and prefill, in both pair
// layouts (interleaved (2i, 2i+1) and half (i, i + hd/2)).
//
// Work item = VP rotation pairs of one q or k head, or 2*VP elements of one
// v head. gridDim.x covers the items of a token, gridDim.y strides over
// tokens (runs of 8 consecutive tokens for prefill, whose q and cache rows
// of one head are then written back to back: 256-byte rows of one head lie
// 512 KB apart otherwise), so a single decode token already spreads over
// several SMs. VP is
// chosen so that every access is 16 bytes: one load + store of 2 VP
// elements (interleaved pairs) or one in each half of the head (half pairs),
// with the cos/sin pairs read two per 16-byte load — no warp shuffles.
//
// Angles come from the host-built cos/sin table (rope_table.cpp) when the
// reference's length-scaling factor is exactly 1 (sequence length <= 4096),
// which makes the rotation bit-identical to the reference's CPU oracle: the
// products are evaluated as c*x0 - s*x1 and s*x0 + c*x1 with round-to-nearest
// intrinsics (no FMA contraction), exactly as the oracle's C++ does. Other
// positions evaluate the reference formula on the device
// (include/kernel/rope.cuh:14-17).
//
// Tokens whose cache position falls outside [0, kv_cache_len) are skipped
// (the reference writes out of bounds there).
//
// Reference: src/kernel/fused_reshape_rope_kvcache_decode.cu:11-84,
// src/kernel/fused_reshape_rope_kvcache_llama2_decode.cu:11-74,
// src/kernel/fused_pad_reshape_transpose_rope_kvcache.cu:11-83,
// src/kernel/fused_pad_reshape_transpose_rope_kvcache_llama2.cu:11-75.
#include "common.cuh"
#include "rope_math.cuh"

#include <algorithm>
#include <cmath>

namespace l2k
{
namespace
{

// Prefill: consecutive tokens per CTA row (decode keeps one token per row
// for parallelism: its few tokens are latency-bound).
constexpr int kTokRun = 8;

struct RopeArgs
{
    const void *input;
    const uint8_t *is_done;       // decode only
    const uint32_t *q_lens;       // prefill only
    const uint32_t *kv_lens;
    const uint32_t *unpad_to_pad; // prefill only
    void *q;
    void *k;
    void *v;
    int64_t n_tokens;
    int64_t batch;
    int64_t hq;
    int64_t hkv;
    int64_t hd;
    int64_t qc; // q rows per sequence in q (1 for decode)
    int64_t S;
    const float2 *table;
    int64_t table_pos;
    // Paged caches: k and v are (num_pages, Hkv, page_rows, hd); position pos
    // of sequence b lives in page block_table[b][pos / page_rows].
    const uint32_t *block_table;
    int64_t max_pages;
    int64_t num_pages;
    int64_t page_rows;
};

// Start of cache row pos of (seq, kv head h): contiguous (B, Hkv, S, hd) or
// paged; null when the page id is past the pool (nothing is written then).
template <typename T>
__device__ __forceinline__ T *cache_row(const RopeArgs &a, void *cache, int64_t seq, int64_t h, uint32_t pos)
{
    if (a.block_table)
    {
        const int64_t page = a.block_table[seq * a.max_pages + pos / a.page_rows];
        if (page >= a.num_pages)
            return nullptr;
        return static_cast<T *>(cache) + ((page * a.hkv + h) * a.page_rows + pos % a.page_rows) * a.hd;
    }
    return static_cast<T *>(cache) + ((seq * a.hkv + h) * a.S + pos) * a.hd;
}

template <int BYTES>
struct RawT;
template <>
struct RawT<16>
{
    using type = uint4;
};
template <>
struct RawT<8>
{
    using type = uint2;
};
template <>
struct RawT<4>
{
    using type = uint32_t;
};
template <>
struct RawT<2>
{
    using type = uint16_t;
};

// CNT elements at p: one vector access when WIDE (alignment checked by the
// launcher), element by element otherwise.
template <typename T, int CNT, bool WIDE>
__device__ __forceinline__ void load_elems(const T *p, float (&out)[CNT])
{
    if constexpr (WIDE)
    {
        using R = typename RawT<CNT * sizeof(T)>::type;
        const R raw = *reinterpret_cast<const R *>(p);
        T tmp[CNT];
        __builtin_memcpy(tmp, &raw, sizeof(R));
#pragma unroll
        for (int e = 0; e < CNT; ++e)
            out[e] = to_f(tmp[e]);
    }
    else
    {
#pragma unroll
        for (int e = 0; e < CNT; ++e)
            out[e] = to_f(p[e]);
    }
}

template <typename T, int CNT, bool WIDE>
__device__ __forceinline__ void store_elems(T *p, const float (&in)[CNT])
{
    T tmp[CNT];
#pragma unroll
    for (int e = 0; e < CNT; ++e)
        tmp[e] = from_f<T>(in[e]);
    if constexpr (WIDE)
    {
        using R = typename RawT<CNT * sizeof(T)>::type;
        R raw;
        __builtin_memcpy(&raw, tmp, sizeof(R));
        *reinterpret_cast<R *>(p) = raw;
    }
    else
    {
#pragma unroll
        for (int e = 0; e < CNT; ++e)
            p[e] = tmp[e];
    }
}

template <typename T, int PAIRING, int VP, bool PREFILL>
__global__ void __launch_bounds__(256) rope_kvcache_kernel(const RopeArgs a)
{
    const int64_t half = a.hd / 2;
    const int pc = (int)(half / VP); // items per rotated head (and per v head)
    const int items = (int)((a.hq + 2 * a.hkv) * pc);
    const int it = blockIdx.x * blockDim.x + threadIdx.x;
    if (it >= items)
        return;
    const int head = it / pc;
    const int64_t i0 = (int64_t)(it - head * pc) * VP;
    const int64_t total_heads = a.hq + 2 * a.hkv;

    // Each CTA row takes RUN consecutive tokens (then strides by the grid), so
    // a thread writes the consecutive cache / q rows of its head back to back.
    constexpr int RUN = PREFILL ? kTokRun : 1;
    for (int64_t tok0 = (int64_t)blockIdx.y * RUN; tok0 < a.n_tokens; tok0 += (int64_t)gridDim.y * RUN)
#pragma unroll 1
    for (int64_t tok = tok0; tok < tok0 + RUN && tok < a.n_tokens; ++tok)
    {
        int64_t seq, t;
        uint32_t kv_len, pos;
        if constexpr (PREFILL)
        {
            const int64_t padded = a.unpad_to_pad[tok];
            seq = padded / a.qc;
            t = padded - seq * a.qc;
            if (seq >= a.batch)
                continue;
            kv_len = a.kv_lens[seq];
            pos = kv_len - a.q_lens[seq] + (uint32_t)t;
        }
        else
        {
            seq = tok;
            t = 0;
            if (a.is_done[seq])
                continue;
            kv_len = a.kv_lens[seq];
            pos = kv_len - 1u;
        }
        if ((int64_t)pos >= a.S)
            continue;
        const T *src = static_cast<const T *>(a.input) + (tok * total_heads + head) * a.hd;
        if (head >= a.hq + a.hkv)
        {
            // v: copy 2*VP elements into cache row pos.
            const int64_t h = head - a.hq - a.hkv;
            T *dst = cache_row<T>(a, a.v, seq, h, pos);
            if (!dst)
                continue;
            if constexpr (2 * VP * sizeof(T) == 32)
            {
                const uint4 *s4 = reinterpret_cast<const uint4 *>(src + 2 * i0);
                uint4 *d4 = reinterpret_cast<uint4 *>(dst + 2 * i0);
                const uint4 lo = s4[0], hi = s4[1];
                d4[0] = lo;
                d4[1] = hi;
            }
            else if constexpr (VP > 1)
            {
                using R = typename RawT<2 * VP * sizeof(T)>::type;
                *reinterpret_cast<R *>(dst + 2 * i0) = *reinterpret_cast<const R *>(src + 2 * i0);
            }
            else
            {
                dst[2 * i0] = src[2 * i0];
                dst[2 * i0 + 1] = src[2 * i0 + 1];
            }
            continue;
        }
        float x0[VP], x1[VP];
        if constexpr (PAIRING == L2K_ROPE_INTERLEAVED)
        {
            float xx[2 * VP];
            load_elems<T, 2 * VP, (VP > 1)>(src + 2 * i0, xx);
#pragma unroll
            for (int e = 0; e < VP; ++e)
            {
                x0[e] = xx[2 * e];
                x1[e] = xx[2 * e + 1];
            }
        }
        else
        {
            load_elems<T, VP, (VP > 1)>(src + i0, x0);
            load_elems<T, VP, (VP > 1)>(src + half + i0, x1);
        }
        float c[VP], s[VP];
        if (a.table && kv_len <= 4096u && (int64_t)pos < a.table_pos)
        {
            const float2 *row = a.table + (int64_t)pos * half + i0;
            if constexpr (VP % 2 == 0)
            {
                // two pairs per 16-byte load (the launcher checked the table's alignment)
#pragma unroll
                for (int e = 0; e < VP; e += 2)
                {
                    const float4 cs = __ldg(reinterpret_cast<const float4 *>(row + e));
                    c[e] = cs.x;
                    s[e] = cs.y;
                    c[e + 1] = cs.z;
                    s[e + 1] = cs.w;
                }
            }
            else
            {
#pragma unroll
                for (int e = 0; e < VP; ++e)
                {
                    const float2 cs = __ldg(row + e);
                    c[e] = cs.x;
                    s[e] = cs.y;
                }
            }
        }
        else
        {
#pragma unroll
            for (int e = 0; e < VP; ++e)
                rope_cos_sin_device(i0 + e, a.hd, pos, kv_len, c[e], s[e]);
        }
        float o0[VP], o1[VP];
#pragma unroll
        for (int e = 0; e < VP; ++e)
        {
            o0[e] = __fsub_rn(__fmul_rn(c[e], x0[e]), __fmul_rn(s[e], x1[e]));
            o1[e] = __fadd_rn(__fmul_rn(s[e], x0[e]), __fmul_rn(c[e], x1[e]));
        }
        T *dst;
        if (head < a.hq)
            dst = static_cast<T *>(a.q) + ((seq * a.hq + head) * a.qc + t) * a.hd;
        else
            dst = cache_row<T>(a, a.k, seq, head - a.hq, pos);
        if (!dst)
            continue;
        if constexpr (PAIRING == L2K_ROPE_INTERLEAVED)
        {
            float oo[2 * VP];
#pragma unroll
            for (int e = 0; e < VP; ++e)
            {
                oo[2 * e] = o0[e];
                oo[2 * e + 1] = o1[e];
            }
            store_elems<T, 2 * VP, (VP > 1)>(dst + 2 * i0, oo);
        }
        else
        {
            store_elems<T, VP, (VP > 1)>(dst + i0, o0);
            store_elems<T, VP, (VP > 1)>(dst + half + i0, o1);
        }
    }
}

template <typename T, int PAIRING, int VP, bool PREFILL>
int launch_rope_vp(const RopeArgs &a, cudaStream_t stream)
{
    const int64_t pc = a.hd / 2 / VP;
    const int64_t items = (a.hq + 2 * a.hkv) * pc;
    const int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ceil_div(items, 32) * 32));
    const int64_t gx = ceil_div(items, block);
    const int64_t gy = std::min<int64_t>(ceil_div(a.n_tokens, PREFILL ? kTokRun : 1), 65535);
    rope_kvcache_kernel<T, PAIRING, VP, PREFILL><<<dim3((unsigned)gx, (unsigned)gy), block, 0, stream>>>(a);
    return check_launch(PREFILL ? "l2k prefill rope" : "l2k decode rope");
}

template <typename T, int PAIRING, bool PREFILL>
int launch_rope(const RopeArgs &a, cudaStream_t stream)
{
    // 16-byte accesses: interleaved pairs 2 VP contiguous elements, half pairs
    // VP contiguous elements in each half.
    constexpr int VPMAX = PAIRING == L2K_ROPE_INTERLEAVED ? 16 / (2 * sizeof(T)) : 16 / sizeof(T);
    const int64_t half = a.hd / 2;
    const bool vec = half % VPMAX == 0 && (a.hd * (int64_t)sizeof(T)) % 16 == 0 && is_aligned(a.input, 16) &&
                     is_aligned(a.q, 16) && is_aligned(a.k, 16) && is_aligned(a.v, 16) &&
                     (a.table == nullptr || is_aligned(a.table, 16));
    if (vec)
        return launch_rope_vp<T, PAIRING, VPMAX, PREFILL>(a, stream);
    return launch_rope_vp<T, PAIRING, 1, PREFILL>(a, stream);
}

int check_common(const RopeArgs &a, const char *name, int dtype)
{
    L2K_REQUIRE(dtype_ok(dtype), "%s: unsupported dtype %d", name, dtype);
    L2K_REQUIRE(a.n_tokens >= 0 && a.batch >= 0 && a.hq >= 0 && a.hkv >= 0 && a.hd >= 0 && a.S >= 0 && a.qc >= 0,
                "%s: negative size", name);
    L2K_REQUIRE(a.hd % 2 == 0, "%s: head_dim must be even (got %lld)", name, (long long)a.hd);
    L2K_REQUIRE(a.table_pos >= 0, "%s: negative rope_table_positions", name);
    L2K_REQUIRE(a.table == nullptr || is_aligned(a.table, 8), "%s: rope_table must be 8-byte aligned", name);
    L2K_REQUIRE_SHAPE((a.hq + 2 * a.hkv) * a.hd < (int64_t(1) << 30), "%s: too many heads", name);
    return L2K_OK;
}

int rope_entry(const RopeArgs &a, int pairing, bool prefill, int dtype, cudaStream_t stream, const char *name)
{
    if (int st = check_common(a, name, dtype))
        return st;
    if (a.n_tokens == 0 || a.hd == 0 || a.hq + a.hkv == 0)
        return L2K_OK;
    L2K_REQUIRE(a.input && a.kv_lens && a.q && (a.hkv == 0 || (a.k && a.v)), "%s: null pointer", name);
    if (prefill)
        L2K_REQUIRE(a.q_lens && a.unpad_to_pad && a.qc > 0, "%s: null q_lens/unpad_to_pad or q_cache_len 0", name);
    else
        L2K_REQUIRE(a.is_done, "%s: null is_done", name);
    L2K_DISPATCH(dtype, {
        if (pairing == L2K_ROPE_INTERLEAVED)
            return prefill ? launch_rope<T, L2K_ROPE_INTERLEAVED, true>(a, stream)
                           : launch_rope<T, L2K_ROPE_INTERLEAVED, false>(a, stream);
        return prefill ? launch_rope<T, L2K_ROPE_HALF, true>(a, stream)
                       : launch_rope<T, L2K_ROPE_HALF, false>(a, stream);
    });
    return L2K_OK;
}

RopeArgs decode_args(const void *input, const uint8_t *is_done, const uint32_t *kv_lens, void *q, void *k, void *v,
                     int64_t batch, int64_t hq, int64_t hkv, int64_t hd, int64_t S, const float *table,
                     int64_t table_pos)
{
    return RopeArgs{input, is_done, nullptr, kv_lens, nullptr, q, k, v, batch, batch, hq, hkv, hd, 1, S,
                    reinterpret_cast<const float2 *>(table), table ? table_pos : 0};
}

RopeArgs prefill_args(const void *input, const uint32_t *q_lens, const uint32_t *kv_lens, const uint32_t *unpad,
                      void *q, void *k, void *v, int64_t n_tokens, int64_t batch, int64_t hq, int64_t hkv, int64_t hd,
                      int64_t qc, int64_t S, const float *table, int64_t table_pos)
{
    return RopeArgs{input, nullptr, q_lens, kv_lens, unpad, q, k, v, n_tokens, batch, hq, hkv, hd, qc, S,
                    reinterpret_cast<const float2 *>(table), table ? table_pos : 0};
}

} // namespace
} // namespace l2k

extern "C" int l2k_fused_reshape_rope_kvcache_decode(const void *input, const uint8_t *is_done,
                                                     const uint32_t *kv_lens, void *q, void *k, void *v,
                                                     int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                     int64_t head_dim, int64_t kv_cache_len, const float *rope_table,
                                                     int64_t rope_table_positions, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    return rope_entry(decode_args(input, is_done, kv_lens, q, k, v, batch, q_head_num, kv_head_num, head_dim,
                                  kv_cache_len, rope_table, rope_table_positions),
                      L2K_ROPE_INTERLEAVED, false, dtype, stream, "l2k_fused_reshape_rope_kvcache_decode");
}

extern "C" int l2k_fused_reshape_rope_kvcache_llama2_decode(const void *input, const uint8_t *is_done,
                                                            const uint32_t *kv_lens, void *q, void *k, void *v,
                                                            int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                            int64_t head_dim, int64_t kv_cache_len,
                                                            const float *rope_table, int64_t rope_table_positions,
                                                            int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    return rope_entry(decode_args(input, is_done, kv_lens, q, k, v, batch, q_head_num, kv_head_num, head_dim,
                                  kv_cache_len, rope_table, rope_table_positions),
                      L2K_ROPE_HALF, false, dtype, stream, "l2k_fused_reshape_rope_kvcache_llama2_decode");
}

extern "C" int l2k_fused_pad_reshape_transpose_rope_kvcache(const void *input, const uint32_t *q_lens,
                                                            const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx,
                                                            void *q, void *k, void *v, int64_t num_tokens,
                                                            int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                            int64_t head_dim, int64_t q_cache_len,
                                                            int64_t kv_cache_len, const float *rope_table,
                                                            int64_t rope_table_positions, int dtype,
                                                            l2k_stream_t stream)
{
    using namespace l2k;
    return rope_entry(prefill_args(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v, num_tokens, batch, q_head_num,
                                   kv_head_num, head_dim, q_cache_len, kv_cache_len, rope_table,
                                   rope_table_positions),
                      L2K_ROPE_INTERLEAVED, true, dtype, stream, "l2k_fused_pad_reshape_transpose_rope_kvcache");
}

extern "C" int l2k_fused_pad_reshape_transpose_rope_kvcache_llama2(
    const void *input, const uint32_t *q_lens, const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx, void *q,
    void *k, void *v, int64_t num_tokens, int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
    int64_t q_cache_len, int64_t kv_cache_len, const float *rope_table, int64_t rope_table_positions, int dtype,
    l2k_stream_t stream)
{
    using namespace l2k;
    return rope_entry(prefill_args(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v, num_tokens, batch, q_head_num,
                                   kv_head_num, head_dim, q_cache_len, kv_cache_len, rope_table,
                                   rope_table_positions),
                      L2K_ROPE_HALF, true, dtype, stream, "l2k_fused_pad_reshape_transpose_rope_kvcache_llama2");
}

extern "C" int l2k_fused_reshape_rope_kvcache_paged_decode(const void *input, const uint8_t *is_done,
                                                           const uint32_t *kv_lens, void *q, void *k_pages,
                                                           void *v_pages, const uint32_t *block_table,
                                                           int64_t max_pages, int64_t num_pages, int64_t page_rows,
                                                           int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                           int64_t head_dim, const float *rope_table,
                                                           int64_t rope_table_positions, int pairing, int dtype,
                                                           l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(pairing == L2K_ROPE_INTERLEAVED || pairing == L2K_ROPE_HALF,
                "l2k_fused_reshape_rope_kvcache_paged_decode: bad pairing %d", pairing);
    L2K_REQUIRE(max_pages >= 0 && num_pages >= 0 && page_rows > 0,
                "l2k_fused_reshape_rope_kvcache_paged_decode: bad page geometry");
    L2K_REQUIRE(batch == 0 || (block_table && max_pages > 0 && num_pages > 0),
                "l2k_fused_reshape_rope_kvcache_paged_decode: null or empty block table");
    RopeArgs a = decode_args(input, is_done, kv_lens, q, k_pages, v_pages, batch, q_head_num, kv_head_num, head_dim,
                             max_pages * page_rows, rope_table, rope_table_positions);
    a.block_table = block_table;
    a.max_pages = max_pages;
    a.num_pages = num_pages;
    a.page_rows = page_rows;
    return rope_entry(a, pairing, false, dtype, stream, "l2k_fused_reshape_rope_kvcache_paged_decode");
}

extern "C" int l2k_fused_pad_reshape_transpose_rope_kvcache_paged(
    const void *input, const uint32_t *q_lens, const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx, void *q,
    void *k_pages, void *v_pages, const uint32_t *block_table, int64_t max_pages, int64_t num_pages, int64_t page_rows,
    int64_t num_tokens, int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t head_dim, int64_t q_cache_len,
    const float *rope_table, int64_t rope_table_positions, int pairing, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(pairing == L2K_ROPE_INTERLEAVED || pairing == L2K_ROPE_HALF,
                "l2k_fused_pad_reshape_transpose_rope_kvcache_paged: bad pairing %d", pairing);
    L2K_REQUIRE(max_pages >= 0 && num_pages >= 0 && page_rows > 0,
                "l2k_fused_pad_reshape_transpose_rope_kvcache_paged: bad page geometry");
    L2K_REQUIRE(batch == 0 || num_tokens == 0 || (block_table && max_pages > 0 && num_pages > 0),
                "l2k_fused_pad_reshape_transpose_rope_kvcache_paged: null or empty block table");
    RopeArgs a = prefill_args(input, q_lens, kv_lens, unpad_to_pad_idx, q, k_pages, v_pages, num_tokens, batch,
                              q_head_num, kv_head_num, head_dim, q_cache_len, max_pages * page_rows, rope_table,
                              rope_table_positions);
    a.block_table = block_table;
    a.max_pages = max_pages;
    a.num_pages = num_pages;
    a.page_rows = page_rows;
    return rope_entry(a, pairing, true, dtype, stream, "l2k_fused_pad_reshape_transpose_rope_kvcache_paged");
}

// ---------------------------------------------------------------------------
// Decode RoPE + K/V append into fp8 (e4m3) caches. q is rotated and stored in
// the activation type; the rotated k and the v row are scaled by the inverse
// of their cache's scale and rounded once to e4m3 (round to nearest even,
// saturating at +-448), straight from fp32 — no 16-bit rounding in between.
// One CTA per (sequence, head), one thread per rotation pair (a v head: two
// elements per thread).
// ---------------------------------------------------------------------------
namespace l2k
{
namespace
{
struct RopeFp8Args
{
    const void *input;
    const uint8_t *is_done;
    const uint32_t *kv_lens;
    void *q;
    uint8_t *k;
    uint8_t *v;
    int64_t batch, hq, hkv, hd, S;
    const float2 *table;
    int64_t table_pos;
    float inv_k_scale, inv_v_scale;
};

__device__ __forceinline__ uint8_t to_e4m3(float x)
{
    return (uint8_t)__nv_cvt_float_to_fp8(x, __NV_SATFINITE, __NV_E4M3);
}

template <typename T, int PAIRING>
__global__ void __launch_bounds__(256) rope_kvcache_fp8_decode_kernel(const RopeFp8Args a)
{
    const int64_t seq = blockIdx.x / (a.hq + 2 * a.hkv);
    const int64_t head = blockIdx.x - seq * (a.hq + 2 * a.hkv);
    if (a.is_done[seq])
        return;
    const uint32_t kv_len = a.kv_lens[seq];
    const uint32_t pos = kv_len - 1u;
    if ((int64_t)pos >= a.S)
        return;
    const int64_t half = a.hd / 2;
    const T *src = static_cast<const T *>(a.input) + (seq * (a.hq + 2 * a.hkv) + head) * a.hd;
    for (int64_t i = threadIdx.x; i < half; i += blockDim.x)
    {
        const int64_t i0 = PAIRING == L2K_ROPE_INTERLEAVED ? 2 * i : i;
        const int64_t i1 = PAIRING == L2K_ROPE_INTERLEAVED ? 2 * i + 1 : i + half;
        if (head >= a.hq + a.hkv)
        {
            const int64_t h = head - a.hq - a.hkv;
            uint8_t *dst = a.v + ((seq * a.hkv + h) * a.S + pos) * a.hd;
            dst[i0] = to_e4m3(__fmul_rn(to_f(src[i0]), a.inv_v_scale));
            dst[i1] = to_e4m3(__fmul_rn(to_f(src[i1]), a.inv_v_scale));
            continue;
        }
        float c, s;
        rope_cos_sin(a.table, a.table_pos, i, a.hd, pos, kv_len, c, s);
        const float x0 = to_f(src[i0]), x1 = to_f(src[i1]);
        const float o0 = rope_o0(c, s, x0, x1), o1 = rope_o1(c, s, x0, x1);
        if (head < a.hq)
        {
            T *dst = static_cast<T *>(a.q) + (seq * a.hq + head) * a.hd;
            dst[i0] = from_f<T>(o0);
            dst[i1] = from_f<T>(o1);
        }
        else
        {
            uint8_t *dst = a.k + ((seq * a.hkv + (head - a.hq)) * a.S + pos) * a.hd;
            dst[i0] = to_e4m3(__fmul_rn(o0, a.inv_k_scale));
            dst[i1] = to_e4m3(__fmul_rn(o1, a.inv_k_scale));
        }
    }
}
} // namespace
} // namespace l2k

extern "C" int l2k_fused_reshape_rope_kvcache_fp8_decode(const void *input, const uint8_t *is_done,
                                                         const uint32_t *kv_lens, void *q, void *k_cache,
                                                         void *v_cache, float k_scale, float v_scale, int64_t batch,
                                                         int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
                                                         int64_t kv_cache_len, const float *rope_table,
                                                         int64_t rope_table_positions, int pairing, int dtype,
                                                         l2k_stream_t stream)
{
    using namespace l2k;
    const char *name = "l2k_fused_reshape_rope_kvcache_fp8_decode";
    L2K_REQUIRE(dtype_ok(dtype), "%s: unsupported dtype %d", name, dtype);
    L2K_REQUIRE(pairing == L2K_ROPE_INTERLEAVED || pairing == L2K_ROPE_HALF, "%s: bad pairing %d", name, pairing);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim >= 0 && kv_cache_len >= 0,
                "%s: negative size", name);
    L2K_REQUIRE(head_dim % 2 == 0, "%s: head_dim must be even (got %lld)", name, (long long)head_dim);
    L2K_REQUIRE(k_scale > 0.f && v_scale > 0.f && std::isfinite(k_scale) && std::isfinite(v_scale),
                "%s: the cache scales must be positive and finite", name);
    L2K_REQUIRE(rope_table_positions >= 0, "%s: negative rope_table_positions", name);
    if (batch == 0 || head_dim == 0 || q_head_num + kv_head_num == 0)
        return L2K_OK;
    L2K_REQUIRE(input && is_done && kv_lens && q && (kv_head_num == 0 || (k_cache && v_cache)), "%s: null pointer",
                name);
    L2K_REQUIRE_SHAPE(batch * (q_head_num + 2 * kv_head_num) < (int64_t(1) << 31), "%s: grid too large", name);
    RopeFp8Args a{input, is_done, kv_lens, q, static_cast<uint8_t *>(k_cache), static_cast<uint8_t *>(v_cache),
                  batch, q_head_num, kv_head_num, head_dim, kv_cache_len,
                  reinterpret_cast<const float2 *>(rope_table), rope_table ? rope_table_positions : 0,
                  1.f / k_scale, 1.f / v_scale};
    const int threads = (int)std::min<int64_t>(256, std::max<int64_t>(32, (head_dim / 2 + 31) / 32 * 32));
    const unsigned grid = (unsigned)(batch * (q_head_num + 2 * kv_head_num));
    L2K_DISPATCH(dtype, {
        if (pairing == L2K_ROPE_INTERLEAVED)
            rope_kvcache_fp8_decode_kernel<T, L2K_ROPE_INTERLEAVED><<<grid, threads, 0, (cudaStream_t)stream>>>(a);
        else
            rope_kvcache_fp8_decode_kernel<T, L2K_ROPE_HALF><<<grid, threads, 0, (cudaStream_t)stream>>>(a);
        return check_launch(name);
    });
    return L2K_OK;
}
