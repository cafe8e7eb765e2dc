// Fused prefill attention scores entry point.
//
// Dispatch: BF16/F16 with head_dim 128 run the tcgen05 kernel
// (prefill_scores_tc.cu). Other BF16/F16 shapes run the cluster score-row
// kernel (decode_scores.cu) with one cluster per query row, fp32 logits until
// the final store. F32 runs
// QK^T on the CUDA cores (gemm.cu) followed by the causal masked softmax
// (masked_softmax.cu): two kernels, the fp32 scores round-trip through HBM.
#include "common.cuh"

namespace l2k
{
int qk_scores_cuda_cores(const void *q, const void *k, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t qc,
                         int64_t S, int64_t hd, int64_t m, int64_t n, const uint32_t *row_lens, int dtype,
                         cudaStream_t stream);
int masked_softmax_causal(void *qk, const uint32_t *q_lens, const uint32_t *kv_lens, int64_t batch, int64_t H,
                          int64_t qc, int64_t S, int64_t max_q, int64_t max_kv, int64_t head_dim, int dtype,
                          cudaStream_t stream);
int prefill_score_rows(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens,
                       uint32_t max_kv, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc, int64_t S,
                       int64_t hd, int dtype, cudaStream_t stream);
bool prefill_tc_supported(int dtype, int64_t head_dim, int64_t S, int64_t Qc, const void *q, const void *k,
                          const void *qk, int64_t grid);
int prefill_scores_tc(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens, uint32_t max_q,
                      uint32_t max_kv, void *qk, int64_t batch, int64_t Hq, int64_t Hkv, int64_t Qc, int64_t S,
                      int dtype, cudaStream_t stream, const uint32_t *block_table = nullptr, int64_t max_pages = 0,
                      int64_t num_pages = 0);
} // namespace l2k

extern "C" int l2k_prefill_attention_scores(const void *q, const void *k, const uint32_t *q_lens,
                                            const uint32_t *kv_lens, uint32_t max_q_len, uint32_t max_kv_len,
                                            void *qk, int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                            int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim, int dtype,
                                            l2k_stream_t stream)
{
    using namespace l2k;
    L2K_REQUIRE(dtype_ok(dtype), "l2k_prefill_attention_scores: unsupported dtype %d", dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim > 0 && q_cache_len >= 0 &&
                    kv_cache_len >= 0,
                "l2k_prefill_attention_scores: bad size");
    L2K_REQUIRE(max_q_len <= q_cache_len && max_kv_len <= kv_cache_len,
                "l2k_prefill_attention_scores: max_q_len/max_kv_len exceed the cache dims");
    if (batch == 0 || q_head_num == 0 || max_q_len == 0 || max_kv_len == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0,
                "l2k_prefill_attention_scores: q_head_num must be a multiple of kv_head_num");
    L2K_REQUIRE(q && k && q_lens && kv_lens && qk, "l2k_prefill_attention_scores: null pointer");
    L2K_REQUIRE_SHAPE(batch <= 65535 && q_head_num <= 65535, "l2k_prefill_attention_scores: grid too large");
    const int64_t tc_grid = ceil_div(max_q_len, 128) * batch * q_head_num;
    if (prefill_tc_supported(dtype, head_dim, kv_cache_len, q_cache_len, q, k, qk, tc_grid))
        return prefill_scores_tc(q, k, q_lens, kv_lens, max_q_len, max_kv_len, qk, batch, q_head_num, kv_head_num,
                                 q_cache_len, kv_cache_len, dtype, stream);
    if (dtype != L2K_F32)
    {
        // 16-bit storage: keep the logits in fp32 until the final store (a QK^T
        // round trip through a bf16/f16 qk buffer would cost ~1% accuracy).
        return prefill_score_rows(q, k, q_lens, kv_lens, max_kv_len, qk, batch, q_head_num, kv_head_num,
                                  q_cache_len, kv_cache_len, head_dim, dtype, stream);
    }
    if (int st = qk_scores_cuda_cores(q, k, qk, batch, q_head_num, kv_head_num, q_cache_len, kv_cache_len, head_dim,
                                      max_q_len, max_kv_len, q_lens, dtype, stream))
        return st;
    return masked_softmax_causal(qk, q_lens, kv_lens, batch, q_head_num, q_cache_len, kv_cache_len, max_q_len,
                                 max_kv_len, head_dim, dtype, stream);
}

// Paged K cache: the tcgen05 kernel with each 128-key tile loaded as two
// 64-row pages (16-bit, head_dim 128 only: one page is 16 KB of rows).
extern "C" int l2k_prefill_attention_scores_paged(const void *q, const void *k_pages, const uint32_t *block_table,
                                                  int64_t max_pages, int64_t num_pages, const uint32_t *q_lens,
                                                  const uint32_t *kv_lens, uint32_t max_q_len, uint32_t max_kv_len,
                                                  void *qk, int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                  int64_t q_cache_len, int64_t head_dim, int dtype,
                                                  l2k_stream_t stream)
{
    using namespace l2k;
    const char *name = "l2k_prefill_attention_scores_paged";
    L2K_REQUIRE(dtype_ok(dtype), "%s: unsupported dtype %d", name, dtype);
    L2K_REQUIRE(batch >= 0 && q_head_num >= 0 && kv_head_num >= 0 && head_dim > 0 && q_cache_len >= 0 &&
                    max_pages >= 0 && num_pages >= 0,
                "%s: bad size", name);
    const int64_t S = max_pages * 64;
    L2K_REQUIRE(max_q_len <= q_cache_len && max_kv_len <= S, "%s: max_q_len/max_kv_len exceed the cache dims", name);
    if (batch == 0 || q_head_num == 0 || max_q_len == 0 || max_kv_len == 0)
        return L2K_OK;
    L2K_REQUIRE(kv_head_num > 0 && q_head_num % kv_head_num == 0, "%s: q_head_num must be a multiple of kv_head_num",
                name);
    L2K_REQUIRE(q && k_pages && block_table && q_lens && kv_lens && qk && num_pages > 0, "%s: null pointer or no pages",
                name);
    L2K_REQUIRE_SHAPE(batch <= 65535 && q_head_num <= 65535 && num_pages * kv_head_num < (int64_t(1) << 31),
                      "%s: grid or page pool too large", name);
    const int64_t tc_grid = ceil_div(max_q_len, 128) * batch * q_head_num;
    L2K_REQUIRE_SHAPE((dtype == L2K_BF16 || dtype == L2K_F16) && head_dim == 128 &&
                          prefill_tc_supported(dtype, head_dim, S, q_cache_len, q, k_pages, qk, tc_grid),
                      "%s: the paged path takes 16-bit data with head_dim 128, 16-byte aligned", name);
    return prefill_scores_tc(q, k_pages, q_lens, kv_lens, max_q_len, max_kv_len, qk, batch, q_head_num, kv_head_num,
                             q_cache_len, S, dtype, stream, block_table, max_pages, num_pages);
}
