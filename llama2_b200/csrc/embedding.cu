// Token-embedding gather: out[t, :] = table[ids[t], :].
//
// HBM-bound row copy. Each CTA walks tokens (stride gridDim.x); its threads
// copy the row in 16-byte chunks (read-once loads that skip L1; plain stores
// so the rows stay in L2 for the RMSNorm that reads them next). The token id
// is read once per row. Rows whose byte size or base alignment is not a
// multiple of 16 take the 2-byte path. Out-of-range ids give a zero row.
//
// Reference: src/kernel/embedding.cu:10-49 (one vector per thread in a flat
// grid-stride loop that re-reads ids[token] for every vector).
#include "common.cuh"

namespace l2k
{
namespace
{

template <typename Unit>
__global__ void __launch_bounds__(256) embedding_kernel(const uint32_t *__restrict__ ids, int64_t n_tokens,
                                                        const Unit *__restrict__ table, int64_t vocab,
                                                        int64_t units_per_row, Unit *__restrict__ out)
{
    for (int64_t t = blockIdx.x; t < n_tokens; t += gridDim.x)
    {
        const uint32_t id = __ldg(ids + t);
        Unit *dst = out + t * units_per_row;
        if (id < vocab)
        {
            const Unit *src = table + (int64_t)id * units_per_row;
            for (int64_t c = threadIdx.x; c < units_per_row; c += blockDim.x)
            {
                if constexpr (sizeof(Unit) == 16)
                    stg(dst + c, ldg_stream(src + c));
                else
                    dst[c] = __ldg(src + c);
            }
        }
        else
        {
            for (int64_t c = threadIdx.x; c < units_per_row; c += blockDim.x)
                dst[c] = Unit{};
        }
    }
}

} // namespace
} // namespace l2k

extern "C" int l2k_embedding(const uint32_t *input_ids, int64_t num_tokens, const void *embed_table,
                             int64_t vocab_size, int64_t embed_dim, void *output, int dtype, l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_embedding: unsupported dtype %d", dtype);
    L2K_REQUIRE(num_tokens >= 0 && vocab_size >= 0 && embed_dim >= 0, "l2k_embedding: negative size");
    if (num_tokens == 0 || embed_dim == 0)
        return L2K_OK;
    L2K_REQUIRE(input_ids && embed_table && output, "l2k_embedding: null pointer");
    const int64_t row_bytes = embed_dim * (int64_t)dtype_size(dtype);
    const int grid = (int)std::min<int64_t>(num_tokens, (int64_t)num_sms() * 16);
    if (row_bytes % 16 == 0 && is_aligned(embed_table, 16) && is_aligned(output, 16))
    {
        const int64_t units = row_bytes / 16;
        const int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ceil_div(units, 32) * 32));
        embedding_kernel<uint4><<<grid, block, 0, stream>>>(input_ids, num_tokens,
                                                           static_cast<const uint4 *>(embed_table), vocab_size,
                                                           units, static_cast<uint4 *>(output));
    }
    else
    {
        const int64_t units = row_bytes / 2;
        const int block = (int)std::min<int64_t>(256, std::max<int64_t>(32, ceil_div(units, 32) * 32));
        embedding_kernel<uint16_t><<<grid, block, 0, stream>>>(input_ids, num_tokens,
                                                               static_cast<const uint16_t *>(embed_table),
                                                               vocab_size, units, static_cast<uint16_t *>(output));
    }
    return check_launch("l2k_embedding");
}
