// Host construction of the RoPE cos/sin table.
//
// table[pos * (head_dim/2) + i] = {cosf(a), sinf(a)},
//   a = (float)pos * theta_i,  theta_i = 1 / powf(10000, 2i / head_dim)
// with the C library's float functions and the reference's float operation
// order (include/kernel/rope.cuh:14-17; its CPU oracle in
// test/kernel/test_fused_reshape_rope_kvcache_decode.cu:26-30). That is the
// reference's angle exactly whenever the sequence length is <= 4096, where
// its length-scaling factor alpha = 1 / powf(max(1, len / 4096), ...) is
// exactly 1 and pos * alpha = pos. Built with -ffp-contract=off.
#include <cmath>
#include <cstdint>

#include "llama2_b200.h"

extern "C" int64_t l2k_rope_table_floats(int64_t head_dim, int64_t num_positions)
{
    if (head_dim <= 0 || num_positions < 0 || head_dim % 2)
        return -1;
    return num_positions * head_dim; // (head_dim / 2) pairs of 2 floats per position
}

extern "C" int l2k_rope_table_fill(float *host_table, int64_t head_dim, int64_t num_positions)
{
    if (!host_table || head_dim <= 0 || head_dim % 2 || num_positions < 0 || num_positions > (int64_t(1) << 24))
        return L2K_ERR_INVALID_ARGUMENT;
    const int64_t half = head_dim / 2;
    const unsigned int hd = (unsigned int)head_dim;
    for (int64_t i = 0; i < half; ++i)
    {
        const float theta = 1.f / powf(10000.f, 2.f * (float)(unsigned int)i / (float)hd);
        for (int64_t pos = 0; pos < num_positions; ++pos)
        {
            const float angle = (float)(unsigned int)pos * 1.f * theta;
            float *e = host_table + 2 * (pos * half + i);
            e[0] = cosf(angle);
            e[1] = sinf(angle);
        }
    }
    return L2K_OK;
}
