// RoPE arithmetic shared by the RoPE + KV-append kernels and the fused
// decode step.
//
// Angles: from the host-built cos/sin table (rope_table.cpp) when the
// reference's length-scaling factor is exactly 1 (sequence length <= 4096)
// and the position is inside the table; otherwise the reference formula is
// evaluated on the device (include/kernel/rope.cuh:14-17). Rotation of the
// pair (x0, x1): o0 = c*x0 - s*x1, o1 = s*x0 + c*x1 with round-to-nearest
// intrinsics and no FMA contraction — the reference oracle's order, so the
// table path is bit-identical to it.
#pragma once

#include "common.cuh"

namespace l2k
{

// Reference angle formula on the device (include/kernel/rope.cuh:14-17).
__device__ __forceinline__ void rope_cos_sin_device(int64_t i, int64_t hd, uint32_t pos, uint32_t seq_len, float &c,
                                                    float &s)
{
    const float theta = __fdiv_rn(1.f, powf(10000.f, __fdiv_rn(2.f * (float)i, (float)hd)));
    const float ratio = __fdiv_rn((float)seq_len, 4096.f);
    const float alpha = __fdiv_rn(1.f, powf(fmaxf(1.f, ratio), __fdiv_rn(2.f * (float)i, (float)(uint32_t)(hd - 2))));
    const float angle = __fmul_rn(__fmul_rn((float)pos, alpha), theta);
    c = cosf(angle);
    s = sinf(angle);
}

// cos/sin of pair i at `pos` for a sequence of length seq_len.
__device__ __forceinline__ void rope_cos_sin(const float2 *table, int64_t table_pos, int64_t i, int64_t hd,
                                             uint32_t pos, uint32_t seq_len, float &c, float &s)
{
    if (table && seq_len <= 4096u && (int64_t)pos < table_pos)
    {
        const float2 cs = __ldg(table + (int64_t)pos * (hd / 2) + i);
        c = cs.x;
        s = cs.y;
    }
    else
        rope_cos_sin_device(i, hd, pos, seq_len, c, s);
}

__device__ __forceinline__ float rope_o0(float c, float s, float x0, float x1)
{
    return __fsub_rn(__fmul_rn(c, x0), __fmul_rn(s, x1));
}
__device__ __forceinline__ float rope_o1(float c, float s, float x0, float x1)
{
    return __fadd_rn(__fmul_rn(s, x0), __fmul_rn(c, x1));
}

} // namespace l2k
