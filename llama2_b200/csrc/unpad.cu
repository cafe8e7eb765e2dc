// Transpose + unpad of the attention output:
//   unpad_qkv[t, h * hd + d] = qkv[b, h, i, d],  b * Qc + i = unpad_to_pad_idx[t].
//
// HBM-bound gather copy. Each CTA walks output tokens (stride gridDim.x),
// reads the token's padded slot once, and its threads copy the H head rows
// (each hd * sizeof(T) bytes, Qc rows apart in the source) into the
// contiguous output row in 16-byte units, four per thread with all four
// loads in flight before the stores: read-once loads that skip L1, plain
// stores. Rows whose byte size or base alignment is not a multiple of
// 16 take the 2-byte path. A slot >= batch * Qc gives a zero row.
//
// Reference: src/kernel/fused_transpose_unpad.cu:11-73 (a grid capped at
// NUM_BLOCKS_X heads x NUM_BLOCKS_Y tokens, one vector per thread, the slot
// re-read and divided for every head).
#include "common.cuh"

#include <algorithm>

namespace l2k
{
namespace
{

constexpr int kUnroll = 4; // 16-byte units in flight per thread

template <typename Unit>
__global__ void __launch_bounds__(256) transpose_unpad_kernel(const uint32_t *__restrict__ slots, int64_t n_tokens,
                                                              int64_t n_slots, int64_t q_cache_len, int64_t heads,
                                                              int64_t units_per_head, const Unit *__restrict__ src,
                                                              Unit *__restrict__ dst)
{
    const int64_t units_per_row = heads * units_per_head;
    const int64_t head_stride = q_cache_len * units_per_head; // one head's plane of the padded layout
    for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x)
    {
        const uint32_t p = __ldg(slots + t);
        Unit *out = dst + t * units_per_row;
        if (p < n_slots)
        {
            const int64_t b = p / q_cache_len, i = p - b * q_cache_len;
            const Unit *base = src + (b * heads * q_cache_len + i) * units_per_head; // (b, head 0, i)
            // kUnroll units per thread, every load issued before the stores
            for (int64_t u0 = threadIdx.x; u0 < units_per_row; u0 += kUnroll * blockDim.x)
            {
                Unit v[kUnroll];
#pragma unroll
                for (int k = 0; k < kUnroll; ++k)
                {
                    const int64_t u = u0 + k * blockDim.x;
                    if (u < units_per_row)
                    {
                        const int64_t h = u / units_per_head, c = u - h * units_per_head;
                        if constexpr (sizeof(Unit) == 16)
                            v[k] = ldg_stream(base + h * head_stride + c);
                        else
                            v[k] = __ldg(base + h * head_stride + c);
                    }
                }
#pragma unroll
                for (int k = 0; k < kUnroll; ++k)
                {
                    const int64_t u = u0 + k * blockDim.x;
                    if (u < units_per_row)
                    {
                        if constexpr (sizeof(Unit) == 16)
                            stg(out + u, v[k]);
                        else
                            out[u] = v[k];
                    }
                }
            }
        }
        else
        {
            for (int64_t u = threadIdx.x; u < units_per_row; u += blockDim.x)
                out[u] = Unit{};
        }
    }
}

template <typename Unit>
void launch(const uint32_t *slots, int64_t n_tokens, int64_t n_slots, int64_t qc, int64_t heads, int64_t uph,
            const void *src, void *dst, cudaStream_t stream)
{
    const int64_t units = heads * uph;
    const int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ceil_div(ceil_div(units, kUnroll), 32) * 32));
    const int grid = (int)std::min<int64_t>(n_tokens, (int64_t)num_sms() * 16);
    transpose_unpad_kernel<Unit><<<grid, block, 0, stream>>>(slots, n_tokens, n_slots, qc, heads, uph,
                                                             static_cast<const Unit *>(src), static_cast<Unit *>(dst));
}

} // namespace
} // namespace l2k

extern "C" int l2k_fused_transpose_unpad(int64_t num_input_tokens, const void *qkv, const uint32_t *unpad_to_pad_idx,
                                         void *unpad_qkv, int64_t batch, int64_t q_head_num, int64_t q_cache_len,
                                         int64_t head_dim, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_fused_transpose_unpad: unsupported dtype %d", dtype);
    L2K_REQUIRE(num_input_tokens >= 0 && batch >= 0 && q_head_num >= 0 && q_cache_len >= 0 && head_dim >= 0,
                "l2k_fused_transpose_unpad: negative size");
    L2K_REQUIRE(num_input_tokens <= batch * q_cache_len,
                "l2k_fused_transpose_unpad: %lld tokens exceed the %lld padded slots", (long long)num_input_tokens,
                (long long)(batch * q_cache_len));
    if (num_input_tokens == 0 || q_head_num == 0 || head_dim == 0)
        return L2K_OK;
    L2K_REQUIRE(qkv && unpad_to_pad_idx && unpad_qkv, "l2k_fused_transpose_unpad: null pointer");
    const int64_t head_bytes = head_dim * (int64_t)dtype_size(dtype);
    const int64_t n_slots = batch * q_cache_len;
    if (head_bytes % 16 == 0 && is_aligned(qkv, 16) && is_aligned(unpad_qkv, 16))
        launch<uint4>(unpad_to_pad_idx, num_input_tokens, n_slots, q_cache_len, q_head_num, head_bytes / 16, qkv,
                      unpad_qkv, stream);
    else
        launch<uint16_t>(unpad_to_pad_idx, num_input_tokens, n_slots, q_cache_len, q_head_num, head_bytes / 2, qkv,
                         unpad_qkv, stream);
    return check_launch("l2k_fused_transpose_unpad");
}
