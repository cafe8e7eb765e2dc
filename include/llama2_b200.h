/*
 * llama2_b200.h — C ABI of the B200 (sm_100a) Llama-2 layer kernels.
 *
 * One entry point per operator of the reference's operator API
 * (pentatracy5/llama2, include/kernel/*.h), plus the fused score kernels and
 * the fused decode step. Every entry point:
 *   - takes plain device pointers and 64-bit sizes (no C++ or torch types);
 *   - enqueues its work on `stream` and returns without synchronizing;
 *   - never allocates device memory (the caller owns every buffer);
 *   - returns L2K_OK (0) or a nonzero l2k_status; on error nothing was
 *     launched and l2k_last_error_message() describes the problem (the
 *     message is per host thread).
 * Shapes follow the reference: row-major, caches laid out as
 * (batch, kv_head, kv_cache_len, head_dim).
 *
 * Element types (`dtype`): L2K_F32, L2K_F16, L2K_BF16. Arithmetic is fp32 in
 * every kernel; 16-bit types are rounded to nearest-even on store. The fp8
 * K/V cache entries (l2k_*_fp8_*) store cache elements as e4m3 bytes with a
 * per-cache fp32 scale (value = scale * e4m3) next to 16-bit activations.
 */
#ifndef LLAMA2_B200_H
#define LLAMA2_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st *l2k_stream_t; /* same handle as cudaStream_t; NULL = legacy default stream */

enum l2k_dtype
{
    L2K_F32 = 0,
    L2K_F16 = 1,
    L2K_BF16 = 2,
    L2K_E4M3 = 3 /* fp8 e4m3 K/V cache elements: only l2k_paged_block_rows takes this code */
};

enum l2k_status
{
    L2K_OK = 0,
    L2K_ERR_INVALID_ARGUMENT = 1,  /* null pointer, negative size, inconsistent shapes */
    L2K_ERR_UNSUPPORTED_DTYPE = 2, /* dtype not handled by this operator */
    L2K_ERR_UNSUPPORTED_SHAPE = 3, /* valid but outside what this operator implements */
    L2K_ERR_CUDA = 4               /* a CUDA runtime call or launch failed */
};

/* RoPE pairings: (2i, 2i+1) as in the reference's generic kernels, or
 * (i, i + head_dim/2) as in its "_llama2" kernels. */
enum l2k_rope_pairing
{
    L2K_ROPE_INTERLEAVED = 0,
    L2K_ROPE_HALF = 1
};

const char *l2k_status_string(int status);
const char *l2k_last_error_message(void);
int l2k_abi_version(void);

/* ------------------------------------------------------------------------
 * Token-embedding gather: output[t, :] = embed_table[input_ids[t], :].
 * Replaces launch_embedding (include/kernel/embedding.h:6-9,
 * src/kernel/embedding.cu:35-49). Ids >= vocab_size produce a zero row
 * (the reference reads out of bounds there).
 * ------------------------------------------------------------------------ */
int l2k_embedding(const uint32_t *input_ids, int64_t num_tokens, const void *embed_table, int64_t vocab_size,
                  int64_t embed_dim, void *output, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused add-residual + RMSNorm, in place:
 *   if add_residual: x = x + residual (written back to x)
 *   residual = x * weights * 1/sqrt(mean(x^2) + 1e-5)
 * Replaces launch_fused_add_residual_rmsnorm<T, add_residual>
 * (include/kernel/fused_add_residual_rmsnorm.h:16-19,
 * src/kernel/fused_add_residual_rmsnorm.cu:104-126).
 * ------------------------------------------------------------------------ */
int l2k_fused_add_residual_rmsnorm(const void *weights, void *x, void *residual, int64_t num_tokens,
                                   int64_t embed_dim, int add_residual, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * RoPE cos/sin table. The RoPE entry points take an optional device table of
 * num_positions x (head_dim/2) float pairs {cos, sin} for the angle
 * pos / 10000^(2i/head_dim), which is the reference's angle whenever the
 * sequence length is <= 4096 (its length-scaling factor is then exactly 1).
 * l2k_rope_table_fill computes the table on the host with the C library's
 * powf/cosf/sinf, the functions the reference's CPU oracle uses, so the
 * kernels' rotations agree with that oracle bit for bit. Positions beyond
 * the table, and sequences longer than 4096, fall back to on-device
 * evaluation of the reference formula (include/kernel/rope.cuh:14-17).
 * ------------------------------------------------------------------------ */
int64_t l2k_rope_table_floats(int64_t head_dim, int64_t num_positions);
int l2k_rope_table_fill(float *host_table, int64_t head_dim, int64_t num_positions);

/* ------------------------------------------------------------------------
 * Decode RoPE + KV-cache append. input: (batch, (Hq + 2 Hkv) * head_dim);
 * q: (batch, Hq, 1, head_dim); k, v: (batch, Hkv, kv_cache_len, head_dim).
 * For each sequence with is_done == 0 and pos = kv_lens[b] - 1: rotate the
 * q and k heads at pos, write q and k row pos, copy v row pos.
 * l2k_fused_reshape_rope_kvcache_decode replaces
 * launch_fused_reshape_rope_kvcache_decode (interleaved pairs;
 * include/kernel/fused_reshape_rope_kvcache_decode.h:6-12,
 * src/kernel/fused_reshape_rope_kvcache_decode.cu:86-125);
 * l2k_fused_reshape_rope_kvcache_llama2_decode replaces
 * launch_fused_reshape_rope_kvcache_llama2_decode (half pairs;
 * include/kernel/fused_reshape_rope_kvcache_llama2_decode.h:6-12,
 * src/kernel/fused_reshape_rope_kvcache_llama2_decode.cu:76-114), which
 * the reference restricts to head_dim 128; here any even head_dim works.
 * rope_table may be NULL (on-device evaluation).
 * ------------------------------------------------------------------------ */
int l2k_fused_reshape_rope_kvcache_decode(const void *input, const uint8_t *is_done, const uint32_t *kv_lens,
                                          void *q, void *k, void *v, int64_t batch, int64_t q_head_num,
                                          int64_t kv_head_num, int64_t head_dim, int64_t kv_cache_len,
                                          const float *rope_table, int64_t rope_table_positions, int dtype,
                                          l2k_stream_t stream);
int l2k_fused_reshape_rope_kvcache_llama2_decode(const void *input, const uint8_t *is_done,
                                                 const uint32_t *kv_lens, void *q, void *k, void *v, int64_t batch,
                                                 int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
                                                 int64_t kv_cache_len, const float *rope_table,
                                                 int64_t rope_table_positions, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Prefill RoPE + pad/transpose + KV-cache append. input: (num_tokens,
 * (Hq + 2 Hkv) * head_dim), unpadded; unpad_to_pad_idx from
 * l2k_build_padding_index_maps; q: (batch, Hq, q_cache_len, head_dim).
 * Token t of sequence b is at pos = kv_lens[b] - q_lens[b] + t.
 * Replaces launch_fused_pad_reshape_transpose_rope_kvcache
 * (include/kernel/fused_pad_reshape_transpose_rope_kvcache.h:6-13,
 * src/kernel/fused_pad_reshape_transpose_rope_kvcache.cu:85-126) and the
 * "_llama2" variant (…_llama2.h:6-13, …_llama2.cu:77-117).
 * ------------------------------------------------------------------------ */
int l2k_fused_pad_reshape_transpose_rope_kvcache(const void *input, const uint32_t *q_lens,
                                                 const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx,
                                                 void *q, void *k, void *v, int64_t num_tokens, int64_t batch,
                                                 int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
                                                 int64_t q_cache_len, int64_t kv_cache_len,
                                                 const float *rope_table, int64_t rope_table_positions, int dtype,
                                                 l2k_stream_t stream);
int l2k_fused_pad_reshape_transpose_rope_kvcache_llama2(const void *input, const uint32_t *q_lens,
                                                        const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx,
                                                        void *q, void *k, void *v, int64_t num_tokens,
                                                        int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                        int64_t head_dim, int64_t q_cache_len,
                                                        int64_t kv_cache_len, const float *rope_table,
                                                        int64_t rope_table_positions, int dtype,
                                                        l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Length update: kv_lens[b] += q_lens[b]; *max_q_len = max(q_lens);
 * *max_kv_len = max(kv_lens) (device pointers; no host synchronization).
 * Replaces launch_update_q_kv_lens (include/kernel/update_q_kv_lens.h:6-9,
 * src/kernel/update_q_kv_lens.cu:43-61), without its batch <= 512 limit.
 * ------------------------------------------------------------------------ */
int l2k_update_q_kv_lens(const uint32_t *q_lens, uint32_t *kv_lens, int64_t batch, uint32_t *max_q_len,
                         uint32_t *max_kv_len, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Causal mask, u8 (batch, q_cache_len, kv_cache_len), written over
 * [0, max_q_len) x [0, max_kv_len) with the reference's expression
 *   q < q_len && k < kv_len && q >= k - (kv_len - q_len)
 * evaluated in 32-bit unsigned arithmetic, bit-identical to the reference
 * (src/kernel/build_causal_mask.cu:35), including its wrap-around for
 * k < kv_len - q_len. Replaces launch_build_causal_mask
 * (include/kernel/build_causal_mask.h:6-11, src/kernel/build_causal_mask.cu:45-67).
 * ------------------------------------------------------------------------ */
int l2k_build_causal_mask(uint32_t max_q_len, uint32_t max_kv_len, const uint32_t *q_lens,
                          const uint32_t *kv_lens, uint8_t *mask, int64_t batch, int64_t q_cache_len,
                          int64_t kv_cache_len, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Unpad -> pad index map: unpad_to_pad_idx[off_b + i] = b * q_cache_len + i,
 * seq_offsets[b] = sum(seq_lens[:b]). Replaces launch_build_padding_index_maps
 * (include/kernel/build_padding_index_maps.h:6-10,
 * src/kernel/build_padding_index_maps.cu:30-43). batch <= 16384.
 * ------------------------------------------------------------------------ */
int l2k_build_padding_index_maps(int64_t num_tokens, const uint32_t *seq_lens, int64_t batch, int64_t q_cache_len,
                                 uint32_t *unpad_to_pad_idx, uint32_t *seq_offsets, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Batched-GEMM pointer arrays. For slot idx = b * Hq + qh (kv slot
 * b * Hkv + qh / (Hq / Hkv) for entries 2 and 3):
 *   arrays[a][idx] = bases[a] + slot * slice_elems[a] * elem_size
 * with a = 0..7 the reference's q, q_decode, k, v, qk, qk_decode, qkv,
 * qkv_decode. bases, slice_elems and arrays are host arrays of 8; each
 * arrays[a] is a device array of batch * Hq pointers.
 * Replaces launch_build_q_k_v_qk_qkv_array
 * (include/kernel/build_q_k_v_qk_qkv_array.h:6-22,
 * src/kernel/build_q_k_v_qk_qkv_array.cu:66-137).
 * ------------------------------------------------------------------------ */
int l2k_build_q_k_v_qk_qkv_array(void *const bases[8], const int64_t slice_elems[8], int64_t elem_size,
                                 int64_t batch, int64_t q_head_num, int64_t kv_head_num, void **const arrays[8],
                                 l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Row-major GEMM C = op(A) op(B) (C is m x n), fp32 accumulation.
 * batch_count == 0: plain GEMM on a, b, c. batch_count > 0: one GEMM per
 * entry of the device pointer arrays a_array, b_array, c_array (a, b, c
 * ignored). lda/ldb/ldc are the row strides of the stored matrices.
 * Replaces launch_linear (include/kernel/linear.h:9-24,
 * src/kernel/linear.cu:42-155), which calls cuBLAS; here it is a kernel of
 * this library: plain 16-bit GEMMs with trans_a = 0 (16-byte aligned bases
 * and row strides) run on the tcgen05 tensor cores, everything else on the
 * CUDA cores. (The reference accumulates fp16 in fp16.)
 * ------------------------------------------------------------------------ */
int l2k_linear(int trans_a, int trans_b, int64_t m, int64_t n, int64_t k, const void *a, int64_t lda,
               const void *b, int64_t ldb, void *c, int64_t ldc, int64_t batch_count, const void *const *a_array,
               const void *const *b_array, void *const *c_array, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * QK^T at the reference's launch_linear call site (trans_B = true), per
 * (b, q head) with grouped KV heads, without pointer arrays:
 *   qk[b, h, i, j] = sum_d q[b, h, i, d] * k[b, h / (Hq/Hkv), j, d],
 * i < m, j < n. q: (B, Hq, q_cache_len, hd); k: (B, Hkv, kv_cache_len, hd);
 * qk: (B, Hq, q_cache_len, kv_cache_len). Other entries are left as is.
 * ------------------------------------------------------------------------ */
int l2k_qk_scores(const void *q, const void *k, void *qk, int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                  int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim, int64_t m, int64_t n, int dtype,
                  l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * P.V at the reference's launch_linear call site (trans_A = trans_B =
 * false), per (b, q head) with grouped KV heads, without pointer arrays:
 *   qkv[b, h, i, d] = sum_{j < n} qk[b, h, i, j] * v[b, h / (Hq/Hkv), j, d],
 * i < m (fp32 accumulation). qk: (B, Hq, q_cache_len, kv_cache_len);
 * v: (B, Hkv, kv_cache_len, hd); qkv: (B, Hq, q_cache_len, hd). Other rows
 * are left as is. This is the batched launch_linear of the reference's
 * qk x v product (src/kernel/linear.cu:96-128 with the qk, v and qkv
 * arrays of include/kernel/build_q_k_v_qk_qkv_array.h:6-22), M = m,
 * N = head_dim, K = n.
 * ------------------------------------------------------------------------ */
int l2k_attention_qkv(const void *qk, const void *v, void *qkv, int64_t batch, int64_t q_head_num,
                      int64_t kv_head_num, int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim, int64_t m,
                      int64_t n, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Masked attention score, in place on qk (B, H, q_cache_len, kv_cache_len):
 * for rows q < q_lens[b] and keys k < max_kv_len,
 *   qk = mask[b, q, k] ? exp(qk / sqrt(head_dim) - m) / (sum + 1e-6) : 0
 * (m, sum over the masked-in keys); every other entry is left untouched.
 * Replaces launch_compute_masked_attention_score<T, unsigned char>
 * (include/kernel/compute_masked_attention_score.h:6-12,
 * src/kernel/compute_masked_attention_score.cu:105-140).
 * ------------------------------------------------------------------------ */
int l2k_compute_masked_attention_score(int64_t head_dim, uint32_t max_q_len, uint32_t max_kv_len,
                                       const uint32_t *q_lens, const uint8_t *mask, void *qk, int64_t batch,
                                       int64_t q_head_num, int64_t q_cache_len, int64_t kv_cache_len, int dtype,
                                       l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * SwiGLU: output[t, i] = silu(input[t, i]) * input[t, F + i].
 * Replaces launch_swiglu (include/kernel/swiglu.h:6-8, src/kernel/swiglu.cu:55-72).
 * ------------------------------------------------------------------------ */
int l2k_swiglu(const void *input, void *output, int64_t num_tokens, int64_t intermediate_size, int dtype,
               l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Projection GEMMs with the following operator in their epilogue (tcgen05,
 * 16-bit, trans_A = false; B row-major K x N, or N x K with trans_b). The
 * product is never stored: results are bit-identical to l2k_linear into a
 * [m, n] buffer followed by the separate operator on that buffer (when
 * l2k_linear takes its tensor-core path, i.e. m > 8). Shapes these kernels
 * do not take return L2K_ERR_UNSUPPORTED_SHAPE, f32 returns
 * L2K_ERR_UNSUPPORTED_DTYPE: run the two operators instead.
 *
 * l2k_linear_swiglu: out[t, i] = silu(P[t, i]) * P[t, inter + i],
 *   P = A op(B) with op(B) k x 2 inter (gate columns, then up columns):
 *   launch_linear (src/kernel/linear.cu:42-155) then launch_swiglu
 *   (src/kernel/swiglu.cu:55-72). inter % 8 == 0.
 * l2k_linear_rope_kvcache_decode: P = A op(B), A = the batch's normed rows
 *   [batch, dim], op(B) dim x (Hq + 2 Hkv) hd; then the decode RoPE + K/V
 *   append of l2k_fused_reshape_rope_kvcache[_llama2]_decode on P (pairing
 *   selects which; src/kernel/fused_reshape_rope_kvcache_decode.cu:11-84,
 *   ..._llama2_decode.cu:11-74). head_dim 64 or 128; q, k, v and the table
 *   16-byte aligned.
 * l2k_linear_pad_rope_kvcache_prefill: the same for num_tokens unpadded
 *   token rows, then l2k_fused_pad_reshape_transpose_rope_kvcache[_llama2]
 *   (src/kernel/fused_pad_reshape_transpose_rope_kvcache.cu:11-83,
 *   ..._llama2.cu:11-75).
 * ------------------------------------------------------------------------ */
int l2k_linear_swiglu(int trans_b, int64_t m, int64_t inter, int64_t k, const void *a, int64_t lda, const void *b,
                      int64_t ldb, void *out, int64_t ldo, int dtype, l2k_stream_t stream);
int l2k_linear_rope_kvcache_decode(int trans_b, const void *a, int64_t lda, const void *b, int64_t ldb, int64_t dim,
                                   const uint8_t *is_done, const uint32_t *kv_lens, void *q, void *k, void *v,
                                   int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t head_dim,
                                   int64_t kv_cache_len, const float *rope_table, int64_t rope_table_positions,
                                   int pairing, int dtype, l2k_stream_t stream);
int l2k_linear_pad_rope_kvcache_prefill(int trans_b, const void *a, int64_t lda, const void *b, int64_t ldb,
                                        int64_t dim, const uint32_t *q_lens, const uint32_t *kv_lens,
                                        const uint32_t *unpad_to_pad_idx, void *q, void *k, void *v,
                                        int64_t num_tokens, int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                        int64_t head_dim, int64_t q_cache_len, int64_t kv_cache_len,
                                        const float *rope_table, int64_t rope_table_positions, int pairing,
                                        int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Transpose + unpad of the attention output (a byte-exact copy):
 *   unpad_qkv[t, h * hd + d] = qkv[b, h, i, d]
 * for t < num_input_tokens, with b * q_cache_len + i = unpad_to_pad_idx[t].
 * qkv: (batch, Hq, q_cache_len, hd); unpad_to_pad_idx: (batch * q_cache_len)
 * (e.g. from l2k_build_padding_index_maps); unpad_qkv: (num_input_tokens,
 * Hq * hd). A slot >= batch * q_cache_len gives a zero row (the reference
 * reads out of bounds there).
 * Replaces launch_fused_transpose_unpad (include/kernel/fused_transpose_unpad.h:6-11,
 * src/kernel/fused_transpose_unpad.cu:51-73).
 * ------------------------------------------------------------------------ */
int l2k_fused_transpose_unpad(int64_t num_input_tokens, const void *qkv, const uint32_t *unpad_to_pad_idx,
                              void *unpad_qkv, int64_t batch, int64_t q_head_num, int64_t q_cache_len,
                              int64_t head_dim, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused decode attention scores: QK^T + 1/sqrt(head_dim) scale + causal
 * length mask + softmax in one pass over the K cache, for one query token
 * per sequence. qk: (B, Hq, 1, kv_cache_len). With kv_len = kv_lens[b] and
 * M = *max_kv_len (device pointer, e.g. from l2k_update_q_kv_lens):
 *   qk[b,h,0,j] = exp(s_j - max) / (sum + 1e-6)  for j < kv_len,
 *   s_j = (q[b,h] . k[b,h/(Hq/Hkv),j]) / sqrt(head_dim);
 *   qk[b,h,0,j] = 0 for kv_len <= j < M; untouched for j >= M.
 * This is the composition of the reference's QK^T call site
 * (src/kernel/linear.cu:96-128), its masked softmax
 * (src/kernel/compute_masked_attention_score.cu:12-103) and the mask
 * "positions 0..pos" (k <= kv_len - 1), without materializing the mask.
 * ------------------------------------------------------------------------ */
int l2k_decode_attention_scores(const void *q, const void *k, const uint32_t *kv_lens, const uint32_t *max_kv_len,
                                void *qk, int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                int64_t kv_cache_len, int64_t head_dim, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused decode attention: the probabilities of l2k_decode_attention_scores
 * (written to qk exactly as that operator writes them) and the attention
 * output P.V, in one pass over the K and V caches:
 *   qkv[b, h, 0, d] = sum_{j < kv_len} p[b, h, j] * v[b, h / (Hq/Hkv), j, d]
 * (fp32 probabilities and accumulation). v: (B, Hkv, kv_cache_len, hd);
 * qkv: (B, Hq, 1, hd), which is also the unpadded (B, Hq * hd) layout of one
 * token per sequence. The composition it replaces: the QK^T call site,
 * the masked softmax, and the qk x v launch_linear call
 * (src/kernel/linear.cu:96-128) over the keys j < max_kv_len, whose
 * probabilities past kv_len are 0.
 * Head sizes whose K rows are not 64, 128, 256 or 512 bytes (or unaligned
 * operands) run the score operator and then l2k_attention_qkv's kernel.
 * ------------------------------------------------------------------------ */
int l2k_decode_attention(const void *q, const void *k, const void *v, const uint32_t *kv_lens,
                         const uint32_t *max_kv_len, void *qk, void *qkv, int64_t batch, int64_t q_head_num,
                         int64_t kv_head_num, int64_t kv_cache_len, int64_t head_dim, int dtype,
                         l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused prefill attention scores: the same composition for q_len query rows
 * per sequence, with the causal mask k <= (kv_len - q_len) + q:
 *   qk[b,h,i,j] = softmax over j < kv_len, j <= kv_len - q_len + i   (i < q_len)
 *   qk[b,h,i,j] = 0 for masked j < max_kv_len; untouched for j >= max_kv_len
 *   or i >= q_len.
 * q: (B, Hq, q_cache_len, hd) from the prefill RoPE; k as for decode.
 * BF16/F16 run QK^T on the tcgen05 tensor cores (fp32 accumulation in
 * tensor memory); F32 runs it on the CUDA cores.
 * ------------------------------------------------------------------------ */
int l2k_prefill_attention_scores(const void *q, const void *k, const uint32_t *q_lens, const uint32_t *kv_lens,
                                 uint32_t max_q_len, uint32_t max_kv_len, void *qk, int64_t batch,
                                 int64_t q_head_num, int64_t kv_head_num, int64_t q_cache_len,
                                 int64_t kv_cache_len, int64_t head_dim, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Fused decode step: the whole decode chain of one layer step in one launch,
 * with the results of running, in order,
 *   l2k_update_q_kv_lens (kv_lens += q_lens; max_lens[0] = max q_len,
 *                         max_lens[1] = max kv_len, on the device),
 *   l2k_embedding (x = embed_table[input_ids]),
 *   l2k_fused_add_residual_rmsnorm without add (normed = RMSNorm(x)),
 *   l2k_fused_reshape_rope_kvcache_decode (pairing L2K_ROPE_INTERLEAVED) or
 *     ..._llama2_decode (L2K_ROPE_HALF): q, and K/V rows appended at
 *     kv_len - 1, skipping sequences with is_done set,
 *   l2k_decode_attention_scores (qk over keys 0..kv_len-1, max_kv_len =
 *     max_lens[1]),
 *   l2k_swiglu (ffn_out from gate_up),
 * one token per sequence. It composes the reference's update_q_kv_lens,
 * embedding, fused_add_residual_rmsnorm, fused_reshape_rope_kvcache[_llama2]_decode,
 * QK^T (launch_linear) + compute_masked_attention_score and swiglu
 * operators; the reference has no fused step.
 *
 * workspace: l2k_decode_step_workspace_bytes() bytes of device memory,
 * zero before the first call; every completed call leaves it zero again. It
 * holds the counter through which the last CTA of the grid performs the
 * length update, so two steps that may run at the same time (different
 * streams) need different workspaces.
 *
 * Supported: head_dim * element size of 64, 128, 256 or 512 bytes; dim and
 * hidden multiples of 16 bytes of elements; 16-byte aligned tensors; for the
 * half pairing head_dim / 2 a multiple of 16 bytes of elements. Other shapes
 * return L2K_ERR_UNSUPPORTED_SHAPE (run the separate operators instead);
 * l2k_decode_step_supported answers without launching.
 * ------------------------------------------------------------------------ */
typedef struct l2k_decode_step_args
{
    /* lengths, u32 [batch]; kv_lens is updated in place; max_lens is u32 [2] */
    const uint32_t *q_lens;
    uint32_t *kv_lens;
    uint32_t *max_lens;
    /* embedding + RMSNorm */
    const uint32_t *input_ids; /* [batch] */
    const void *embed_table;   /* [vocab_size, dim] */
    const void *norm_weight;   /* [dim] */
    void *x;                   /* [batch, dim] */
    void *normed;              /* [batch, dim] */
    /* RoPE + KV append + attention scores */
    const void *qkv;           /* [batch, (q_head_num + 2 kv_head_num) * head_dim] */
    const uint8_t *is_done;    /* [batch] */
    void *q;                   /* (batch, q_head_num, 1, head_dim) */
    void *k_cache;             /* (batch, kv_head_num, kv_cache_len, head_dim) */
    void *v_cache;             /* same */
    void *qk;                  /* (batch, q_head_num, 1, kv_cache_len) */
    const float *rope_table;   /* l2k_rope_table_fill layout, or NULL */
    int64_t rope_table_positions;
    /* SwiGLU */
    const void *gate_up;       /* [batch, 2 * hidden] */
    void *ffn_out;             /* [batch, hidden] */
    /* sizes */
    int64_t batch;
    int64_t vocab_size;
    int64_t dim;
    int64_t q_head_num;
    int64_t kv_head_num;
    int64_t head_dim;
    int64_t kv_cache_len;
    int64_t hidden;
    int pairing; /* l2k_rope_pairing */
    int dtype;   /* l2k_dtype */
} l2k_decode_step_args;

int64_t l2k_decode_step_workspace_bytes(void);
int l2k_decode_step_supported(const l2k_decode_step_args *args);
int l2k_decode_step(const l2k_decode_step_args *args, uint32_t *workspace, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Paged K/V caches (decode). A paged cache is a pool of pages
 * (num_pages, Hkv, page_rows, head_dim); sequence b's cache positions
 * [j * page_rows, (j + 1) * page_rows) live in page block_table[b * max_pages
 * + j] (u32, device). page_rows is l2k_paged_block_rows(head_dim, dtype)
 * (16 KB of rows per page and kv head: one streamed block of the score
 * kernels); 0 when the head size is not one the streaming kernels take.
 * Page ids past the pool are not dereferenced (rows for them are not
 * written; the attention reads page 0 and records l2k_device_error).
 * No counterpart in the reference, whose caches are (batch, kv_head,
 * kv_cache_len, head_dim) (include/kernel/fused_reshape_rope_kvcache_decode.h:11-12).
 *
 * l2k_fused_reshape_rope_kvcache_paged_decode: the decode RoPE + append
 *   of l2k_fused_reshape_rope_kvcache[_llama2]_decode (pairing selects which)
 *   with K/V row pos = kv_lens[b] - 1 written to its page.
 * l2k_decode_attention_paged: l2k_decode_attention over the paged caches;
 *   qk is (B, Hq, 1, max_pages * page_rows), qkv (B, Hq, 1, hd).
 * ------------------------------------------------------------------------ */
int64_t l2k_paged_block_rows(int64_t head_dim, int dtype);
int l2k_fused_reshape_rope_kvcache_paged_decode(const void *input, const uint8_t *is_done, const uint32_t *kv_lens,
                                                void *q, void *k_pages, void *v_pages, const uint32_t *block_table,
                                                int64_t max_pages, int64_t num_pages, int64_t page_rows,
                                                int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                int64_t head_dim, const float *rope_table,
                                                int64_t rope_table_positions, int pairing, int dtype,
                                                l2k_stream_t stream);
int l2k_decode_attention_paged(const void *q, const void *k_pages, const void *v_pages, const uint32_t *block_table,
                               int64_t max_pages, int64_t num_pages, const uint32_t *kv_lens,
                               const uint32_t *max_kv_len, void *qk, void *qkv, int64_t batch, int64_t q_head_num,
                               int64_t kv_head_num, int64_t head_dim, int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * fp8 (e4m3) K/V caches (decode). No counterpart in the reference, whose
 * DataType stops at FP32/FP16/INT8 (include/common/types.h:60-71); each
 * replaces the 16-bit operator named beside it for caches of one byte per
 * element, holding value / scale rounded to e4m3 (nearest even, saturating
 * at +-448), with one positive fp32 scale per cache (k_scale, v_scale).
 * dtype is the activation type, L2K_BF16 or L2K_F16.
 *
 * l2k_fused_reshape_rope_kvcache_fp8_decode: the decode RoPE + append of
 *   l2k_fused_reshape_rope_kvcache[_llama2]_decode (pairing selects which):
 *   q in dtype; the rotated k and the v row scaled by 1 / scale (fp32) and
 *   rounded once to e4m3 at row kv_lens[b] - 1 of the byte caches
 *   (batch, kv_head_num, kv_cache_len, head_dim).
 * l2k_decode_attention_fp8: l2k_decode_attention over those caches: logits
 *   (q . k8) * (k_scale / sqrt(head_dim)), output v_scale * sum p_j v8_j,
 *   fp32 arithmetic on the exact e4m3 values; head_dim 64/128/256/512,
 *   16-byte aligned operands; qk (B, Hq, 1, kv_cache_len) and qkv in dtype.
 * l2k_decode_attention_fp8_paged: the same over page pools (num_pages,
 *   kv_head_num, 16384 / head_dim, head_dim) of bytes and a block table as
 *   for l2k_decode_attention_paged (l2k_paged_block_rows(head_dim,
 *   L2K_E4M3) rows per page); qk is (B, Hq, 1, max_pages * page_rows).
 * ------------------------------------------------------------------------ */
int l2k_fused_reshape_rope_kvcache_fp8_decode(const void *input, const uint8_t *is_done, const uint32_t *kv_lens,
                                              void *q, void *k_cache, void *v_cache, float k_scale, float v_scale,
                                              int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                              int64_t head_dim, int64_t kv_cache_len, const float *rope_table,
                                              int64_t rope_table_positions, int pairing, int dtype,
                                              l2k_stream_t stream);
int l2k_decode_attention_fp8(const void *q, const void *k_cache, const void *v_cache, float k_scale, float v_scale,
                             const uint32_t *kv_lens, const uint32_t *max_kv_len, void *qk, void *qkv, int64_t batch,
                             int64_t q_head_num, int64_t kv_head_num, int64_t kv_cache_len, int64_t head_dim,
                             int dtype, l2k_stream_t stream);
int l2k_decode_attention_fp8_paged(const void *q, const void *k_pages, const void *v_pages, float k_scale,
                                   float v_scale, const uint32_t *block_table, int64_t max_pages, int64_t num_pages,
                                   const uint32_t *kv_lens, const uint32_t *max_kv_len, void *qk, void *qkv,
                                   int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t head_dim, int dtype,
                                   l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Paged K/V caches (prefill), same pool layout and block table as above.
 * No counterpart in the reference; each replaces the contiguous operator
 * named beside it, whose reference counterpart it keeps:
 *
 * l2k_fused_pad_reshape_transpose_rope_kvcache_paged: the prefill RoPE +
 *   append of l2k_fused_pad_reshape_transpose_rope_kvcache[_llama2]
 *   (src/kernel/fused_pad_reshape_transpose_rope_kvcache*.cu:11-126; pairing
 *   selects which) with K/V row pos = kv_len - q_len + t written to page
 *   block_table[b][pos / page_rows], row pos % page_rows.
 * l2k_prefill_attention_scores_paged: l2k_prefill_attention_scores over a
 *   paged K cache; 16-bit data, head_dim 128 (page_rows 64: a 128-key tile of
 *   the tensor-core kernel is two pages). qk is (B, Hq, q_cache_len,
 *   max_pages * 64). Other shapes return L2K_ERR_UNSUPPORTED_SHAPE.
 * l2k_attention_qkv_paged: l2k_attention_qkv over a paged V cache, same
 *   shape coverage (one page is one 64-key block). kv_lens (device) are the
 *   sequences' lengths: a block wholly past a sequence's length reads pool
 *   page 0 (its probabilities are zero), so unset table entries past a
 *   sequence's pages are never dereferenced. As with the contiguous operator,
 *   rows after a sequence's length (here up to the end of its last page) are
 *   read and multiplied by zero probabilities.
 * ------------------------------------------------------------------------ */
int l2k_fused_pad_reshape_transpose_rope_kvcache_paged(const void *input, const uint32_t *q_lens,
                                                       const uint32_t *kv_lens, const uint32_t *unpad_to_pad_idx,
                                                       void *q, void *k_pages, void *v_pages,
                                                       const uint32_t *block_table, int64_t max_pages,
                                                       int64_t num_pages, int64_t page_rows, int64_t num_tokens,
                                                       int64_t batch, int64_t q_head_num, int64_t kv_head_num,
                                                       int64_t head_dim, int64_t q_cache_len, const float *rope_table,
                                                       int64_t rope_table_positions, int pairing, int dtype,
                                                       l2k_stream_t stream);
int l2k_prefill_attention_scores_paged(const void *q, const void *k_pages, const uint32_t *block_table,
                                       int64_t max_pages, int64_t num_pages, const uint32_t *q_lens,
                                       const uint32_t *kv_lens, uint32_t max_q_len, uint32_t max_kv_len, void *qk,
                                       int64_t batch, int64_t q_head_num, int64_t kv_head_num, int64_t q_cache_len,
                                       int64_t head_dim, int dtype, l2k_stream_t stream);
int l2k_attention_qkv_paged(const void *qk, const void *v_pages, const uint32_t *block_table, int64_t max_pages,
                            int64_t num_pages, const uint32_t *kv_lens, void *qkv, int64_t batch, int64_t q_head_num,
                            int64_t kv_head_num, int64_t q_cache_len, int64_t head_dim, int64_t m, int64_t n,
                            int dtype, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * The fused decode step with the attention output: everything
 * l2k_decode_step computes, and in the same launch
 *   attn_out[b, h, 0, :] = sum_{j <= pos} qk[b, h, 0, j] * v_cache[b, h / (Hq/Hkv), j, :]
 * over the appended cache (fp32 probabilities and accumulation), i.e. the
 * results of l2k_decode_attention in place of l2k_decode_attention_scores.
 * attn_out: (batch, Hq, 1, head_dim), 16-byte aligned — also the unpadded
 * (batch, Hq * head_dim) layout. Same shape coverage as l2k_decode_step
 * (l2k_decode_step_supported).
 * ------------------------------------------------------------------------ */
int l2k_decode_step_attention(const l2k_decode_step_args *args, void *attn_out, uint32_t *workspace,
                              l2k_stream_t stream);
/* The same on the library's static scratch (see l2k_decode_step_no_alloc). */
int l2k_decode_step_attention_no_alloc(const l2k_decode_step_args *args, void *attn_out, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * The fused decode step (with or without the attention output) over paged
 * K/V caches: args->k_cache and args->v_cache are page pools
 * (num_pages, kv_head_num, page_rows, head_dim) with page_rows =
 * l2k_paged_block_rows(head_dim, dtype); args->kv_cache_len must be
 * max_pages * page_rows (the logical cache length). Positions
 * [j * page_rows, (j + 1) * page_rows) of sequence b live in page
 * block_table[b * max_pages + j] (u32, device; every entry a sequence's keys
 * reach must name a page of the pool). The appended K/V rows go to the page
 * holding the position; results are bit-identical to l2k_decode_step /
 * l2k_decode_step_attention on the contiguous caches those pages form.
 * The reference's caches are contiguous (batch, kv_head, kv_cache_len,
 * head_dim) (include/kernel/fused_reshape_rope_kvcache_decode.h:11-12) and it
 * has no fused step; paging widens that cache contract.
 * ------------------------------------------------------------------------ */
int l2k_decode_step_paged(const l2k_decode_step_args *args, const uint32_t *block_table, int64_t max_pages,
                          int64_t num_pages, uint32_t *workspace, l2k_stream_t stream);
int l2k_decode_step_attention_paged(const l2k_decode_step_args *args, const uint32_t *block_table,
                                    int64_t max_pages, int64_t num_pages, void *attn_out, uint32_t *workspace,
                                    l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * l2k_decode_step without a workspace argument, for callers that cannot
 * provide device memory (for example a binding whose host side only passes
 * the tensors it already has and owns no device allocator). The workspace is
 * a 256-byte scratch array inside this library, one per device; nothing is
 * allocated. (No counterpart in the reference, which has no fused step.)
 *  - The stream must belong to the current device (a stream of another
 *    device returns L2K_ERR_INVALID_ARGUMENT); the scratch used is that
 *    device's.
 *  - The first call on a device looks the scratch up (cudaGetSymbolAddress,
 *    with that device current); make it before any stream capture. A call
 *    that finds a different driver context current than at the lookup (after
 *    cudaDeviceReset, or with a non-primary context made current) looks it
 *    up again in that context.
 *  - The scratch is zero when its context loads the library's kernels, and
 *    every call whose kernel runs to its end leaves it zero — also one whose
 *    bounded waits expired (l2k_device_error != 0): every CTA still takes its
 *    ticket. Only a call whose context is lost (a sticky CUDA error) can
 *    leave it nonzero; the new context a reset creates starts from zero.
 *  - Calls on one device share the scratch: two steps that may run at the
 *    same time (different streams) race and give wrong lengths. Use
 *    l2k_decode_step with separate workspaces for that.
 *  - Returns L2K_ERR_UNSUPPORTED_SHAPE if the step's workspace
 *    (l2k_decode_step_workspace_bytes) exceeds the 256-byte scratch or the
 *    device ordinal is >= 64.
 * ------------------------------------------------------------------------ */
int l2k_decode_step_no_alloc(const l2k_decode_step_args *args, l2k_stream_t stream);

/* ------------------------------------------------------------------------
 * Device-side error code recorded by kernels that wait on mbarriers (the
 * tcgen05 prefill scores, the streaming score rows, the fused decode step):
 * 0 = none. Every such wait is bounded; a wait that
 * expires records its code here and the kernel exits instead of hanging.
 * Synchronizes with the device. clear != 0 resets the code. Returns -1 if
 * the code could not be read. (No counterpart in the reference, which has
 * no such waits.)
 * ------------------------------------------------------------------------ */
int l2k_device_error(int clear);

#ifdef __cplusplus
}
#endif

#endif /* LLAMA2_B200_H */
