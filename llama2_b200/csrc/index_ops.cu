// Integer kernels of the path: length update, causal mask, unpad->pad index
// map and the batched-GEMM pointer arrays. All are bit-exact restatements
// of the reference's semantics.
#include "common.cuh"

#include <algorithm>

namespace l2k
{
namespace
{

// --------------------------------------------------------------------------
// kv_lens += q_lens; max_q / max_kv by block reduction. One CTA of 1024
// threads loops over any batch size (the reference asserts batch <= 512:
// src/kernel/update_q_kv_lens.cu:9-61). Results stay on the device.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) update_lens_kernel(const uint32_t *__restrict__ q_lens,
                                                           uint32_t *__restrict__ kv_lens, int64_t batch,
                                                           uint32_t *__restrict__ max_q, uint32_t *__restrict__ max_kv)
{
    __shared__ uint32_t red_q[32], red_kv[32];
    uint32_t mq = 0, mkv = 0;
    for (int64_t i = threadIdx.x; i < batch; i += blockDim.x)
    {
        const uint32_t q = q_lens[i];
        const uint32_t kv = kv_lens[i] + q;
        kv_lens[i] = kv;
        mq = max(mq, q);
        mkv = max(mkv, kv);
    }
    mq = warp_max_u32(mq);
    mkv = warp_max_u32(mkv);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0)
    {
        red_q[warp] = mq;
        red_kv[warp] = mkv;
    }
    __syncthreads();
    if (warp == 0)
    {
        const int nw = blockDim.x >> 5;
        mq = warp_max_u32(lane < nw ? red_q[lane] : 0u);
        mkv = warp_max_u32(lane < nw ? red_kv[lane] : 0u);
        if (lane == 0)
        {
            *max_q = mq;
            *max_kv = mkv;
        }
    }
}

// --------------------------------------------------------------------------
// Causal mask with the reference's 32-bit unsigned expression
// (src/kernel/build_causal_mask.cu:35). Thread = 16 consecutive keys of one
// (seq, q) row; full 16-key groups are one 16-byte store when the row start
// is 16-byte aligned.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256) causal_mask_kernel(const uint32_t *__restrict__ q_lens,
                                                          const uint32_t *__restrict__ kv_lens,
                                                          uint8_t *__restrict__ mask, int64_t batch, int64_t qc,
                                                          int64_t S, uint32_t max_q, uint32_t max_kv, bool vec)
{
    const uint32_t k0 = (uint32_t)((blockIdx.x * blockDim.x + threadIdx.x) * 16u);
    if (k0 >= max_kv)
        return;
    for (int64_t b = blockIdx.z; b < batch; b += gridDim.z)
    {
        const uint32_t q_len = q_lens[b];
        const uint32_t kv_len = kv_lens[b];
        const uint32_t hist = kv_len - q_len;
        for (uint32_t qi = blockIdx.y; qi < max_q; qi += gridDim.y)
        {
            uint8_t *row = mask + ((int64_t)b * qc + qi) * S;
            uint8_t m[16];
#pragma unroll
            for (int e = 0; e < 16; ++e)
            {
                const uint32_t ki = k0 + e;
                m[e] = (uint8_t)(qi < q_len && ki < kv_len && qi >= (uint32_t)(ki - hist));
            }
            if (vec && k0 + 16 <= max_kv)
            {
                uint4 u;
                __builtin_memcpy(&u, m, 16);
                *reinterpret_cast<uint4 *>(row + k0) = u;
            }
            else
            {
                for (int e = 0; e < 16 && k0 + e < max_kv; ++e)
                    row[k0 + e] = m[e];
            }
        }
    }
}

// --------------------------------------------------------------------------
// Unpad -> pad index map. Every CTA scans seq_lens into shared memory
// (exclusive offsets), CTA 0 writes seq_offsets for every sequence, and the
// grid walks tokens, finding each token's sequence by binary search over the
// offsets: O(log B) per token instead of the reference's O(B) scan
// (src/kernel/build_padding_index_maps.cu:8-28).
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(1024) padding_maps_kernel(int64_t n_tokens, const uint32_t *__restrict__ seq_lens,
                                                            int64_t batch, int64_t qc, uint32_t *__restrict__ unpad,
                                                            uint32_t *__restrict__ offsets)
{
    extern __shared__ uint32_t incl[]; // inclusive prefix sums, batch entries
    __shared__ uint32_t warp_tot[32];
    const int tid = threadIdx.x, nt = blockDim.x;
    const int64_t per = (batch + nt - 1) / nt;
    const int64_t s0 = tid * per, s1 = min(batch, s0 + per);
    uint32_t local = 0;
    for (int64_t s = s0; s < s1; ++s)
        local += seq_lens[s];
    // exclusive scan of `local` across the block
    const int lane = tid & 31, warp = tid >> 5;
    uint32_t inc = local;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1)
    {
        const uint32_t n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o)
            inc += n;
    }
    if (lane == 31)
        warp_tot[warp] = inc;
    __syncthreads();
    if (warp == 0)
    {
        uint32_t w = lane < (nt >> 5) ? warp_tot[lane] : 0u;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1)
        {
            const uint32_t n = __shfl_up_sync(0xffffffffu, w, o);
            if (lane >= o)
                w += n;
        }
        warp_tot[lane] = w;
    }
    __syncthreads();
    uint32_t run = (warp ? warp_tot[warp - 1] : 0u) + inc - local;
    for (int64_t s = s0; s < s1; ++s)
    {
        if (blockIdx.x == 0)
            offsets[s] = run;
        run += seq_lens[s];
        incl[s] = run;
    }
    __syncthreads();
    for (int64_t t = (int64_t)blockIdx.x * nt + tid; t < n_tokens; t += (int64_t)gridDim.x * nt)
    {
        // first sequence whose inclusive end exceeds t
        int64_t lo = 0, hi = batch;
        while (lo < hi)
        {
            const int64_t mid = (lo + hi) >> 1;
            if (incl[mid] > (uint32_t)t)
                hi = mid;
            else
                lo = mid + 1;
        }
        if (lo >= batch)
            continue; // more tokens than sum(seq_lens): nothing to map
        const uint32_t start = lo ? incl[lo - 1] : 0u;
        unpad[t] = (uint32_t)(lo * qc) + ((uint32_t)t - start);
    }
}

// --------------------------------------------------------------------------
// Pointer arrays (src/kernel/build_q_k_v_qk_qkv_array.cu:9-64).
// --------------------------------------------------------------------------
struct PtrArgs
{
    char *base[8];
    int64_t stride_bytes[8];
    void **out[8];
};

__global__ void __launch_bounds__(256) ptr_arrays_kernel(const PtrArgs a, int64_t batch, int64_t hq, int64_t group,
                                                         int64_t hkv)
{
    const int64_t n = batch * hq;
    for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < n; idx += (int64_t)gridDim.x * blockDim.x)
    {
        const int64_t b = idx / hq, qh = idx - b * hq;
        const int64_t kv_idx = b * hkv + qh / group;
#pragma unroll
        for (int j = 0; j < 8; ++j)
        {
            const int64_t slot = (j == 2 || j == 3) ? kv_idx : idx;
            a.out[j][idx] = a.base[j] + slot * a.stride_bytes[j];
        }
    }
}

} // namespace
} // namespace l2k

extern "C" int l2k_update_q_kv_lens(const uint32_t *q_lens, uint32_t *kv_lens, int64_t batch, uint32_t *max_q_len,
                                    uint32_t *max_kv_len, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(batch >= 0, "l2k_update_q_kv_lens: negative batch");
    L2K_REQUIRE(max_q_len && max_kv_len, "l2k_update_q_kv_lens: null max pointer");
    L2K_REQUIRE(batch == 0 || (q_lens && kv_lens), "l2k_update_q_kv_lens: null lens pointer");
    const int block = batch >= 1024 ? 1024 : (int)std::max<int64_t>(32, ceil_div(batch, 32) * 32);
    update_lens_kernel<<<1, block, 0, stream>>>(q_lens, kv_lens, batch, max_q_len, max_kv_len);
    return check_launch("l2k_update_q_kv_lens");
}

extern "C" int l2k_build_causal_mask(uint32_t max_q_len, uint32_t max_kv_len, const uint32_t *q_lens,
                                     const uint32_t *kv_lens, uint8_t *mask, int64_t batch, int64_t q_cache_len,
                                     int64_t kv_cache_len, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(batch >= 0 && q_cache_len >= 0 && kv_cache_len >= 0, "l2k_build_causal_mask: negative size");
    L2K_REQUIRE(max_q_len <= q_cache_len && max_kv_len <= kv_cache_len,
                "l2k_build_causal_mask: max_q_len/max_kv_len exceed the mask's cache dims");
    if (batch == 0 || max_q_len == 0 || max_kv_len == 0)
        return L2K_OK;
    L2K_REQUIRE(q_lens && kv_lens && mask, "l2k_build_causal_mask: null pointer");
    const bool vec = kv_cache_len % 16 == 0 && is_aligned(mask, 16);
    const int64_t groups = ceil_div(max_kv_len, 16);
    const int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ceil_div(groups, 32) * 32));
    const dim3 grid((unsigned)ceil_div(groups, block), (unsigned)std::min<int64_t>(max_q_len, 65535),
                    (unsigned)std::min<int64_t>(batch, 65535));
    causal_mask_kernel<<<grid, block, 0, stream>>>(q_lens, kv_lens, mask, batch, q_cache_len, kv_cache_len, max_q_len,
                                                   max_kv_len, vec);
    return check_launch("l2k_build_causal_mask");
}

extern "C" int l2k_build_padding_index_maps(int64_t num_tokens, const uint32_t *seq_lens, int64_t batch,
                                            int64_t q_cache_len, uint32_t *unpad_to_pad_idx, uint32_t *seq_offsets,
                                            l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(num_tokens >= 0 && batch >= 0 && q_cache_len >= 0, "l2k_build_padding_index_maps: negative size");
    L2K_REQUIRE_SHAPE(batch <= 16384, "l2k_build_padding_index_maps: batch %lld > 16384", (long long)batch);
    if (batch == 0)
        return L2K_OK;
    L2K_REQUIRE(seq_lens && seq_offsets && (num_tokens == 0 || unpad_to_pad_idx),
                "l2k_build_padding_index_maps: null pointer");
    const size_t smem = (size_t)batch * sizeof(uint32_t);
    if (smem > 48 * 1024 &&
        cudaFuncSetAttribute(padding_maps_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
        return check_launch("l2k_build_padding_index_maps: shared-memory attribute");
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(num_tokens, 1024), num_sms()));
    padding_maps_kernel<<<grid, 1024, smem, stream>>>(num_tokens, seq_lens, batch, q_cache_len, unpad_to_pad_idx,
                                                      seq_offsets);
    return check_launch("l2k_build_padding_index_maps");
}

extern "C" int l2k_build_q_k_v_qk_qkv_array(void *const bases[8], const int64_t slice_elems[8], int64_t elem_size,
                                            int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                            void **const arrays[8], l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(bases && slice_elems && arrays, "l2k_build_q_k_v_qk_qkv_array: null argument array");
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && elem_size > 0,
                "l2k_build_q_k_v_qk_qkv_array: bad size");
    if (batch == 0 || q_head_num == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_build_q_k_v_qk_qkv_array: q_head_num must be a multiple of kv_head_num");
    PtrArgs a;
    for (int j = 0; j < 8; ++j)
    {
        L2K_REQUIRE(arrays[j] && slice_elems[j] >= 0, "l2k_build_q_k_v_qk_qkv_array: null output array %d", j);
        a.base[j] = static_cast<char *>(bases[j]);
        a.stride_bytes[j] = slice_elems[j] * elem_size;
        a.out[j] = arrays[j];
    }
    const int64_t n = batch * q_head_num;
    const int grid = (int)std::min<int64_t>(ceil_div(n, 256), num_sms() * 4);
    ptr_arrays_kernel<<<grid, 256, 0, stream>>>(a, batch, q_head_num, q_head_num / kv_head_num, kv_head_num);
    return check_launch("l2k_build_q_k_v_qk_qkv_array");
}
