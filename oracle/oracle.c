/*
 * CPU oracle for the fused Llama-2 layer-kernel path.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates, in plain C11, the CPU
 * helper functions that the reference (pentatracy5/llama2) uses as the
 * expected-result oracle in its own unit tests (test/kernel/*.cu). It is
 * the checker for the CUDA kernels of this repository; it is never linked
 * into the product library and never called on a product path.
 *
 * Numeric contract (kept identical to the reference helpers):
 *   - fp32 arithmetic in the same operation order as the reference helper,
 *     using the C library float functions (powf, cosf, sinf, expf, sqrtf)
 *     that std::pow/std::cos/std::sin/std::exp/std::sqrt resolve to for
 *     float arguments in the reference's C++ code;
 *   - compiled with -ffp-contract=off so that a*b-c*d is not fused;
 *   - indices widened to 64 bits (the reference uses 32-bit unsigned int;
 *     the results are the same wherever the reference does not overflow).
 *
 * Each function names the reference file:line it follows.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

/* Constants from the reference's include/common/config.h:13-16. */
#define ORC_SOFTMAX_EPS 1e-6f
#define ORC_RMSNORM_EPS 1e-5f
#define ORC_ROPE_BASE 10000.f
#define ORC_TRAIN_SEQ_LEN 4096.f

/* ------------------------------------------------------------------------
 * Embedding gather.
 * Follows test/kernel/test_embedding.cu:50-61: out[t, :] = table[ids[t], :].
 * Byte-generic so that it covers every element type bit-exactly.
 * ------------------------------------------------------------------------ */
void orc_embedding(const uint32_t *ids, int64_t n_tokens, const void *table,
                   int64_t dim, int64_t elem_size, void *out)
{
    const int64_t row_bytes = dim * elem_size;
    for (int64_t t = 0; t < n_tokens; ++t)
        memcpy((char *)out + t * row_bytes,
               (const char *)table + (int64_t)ids[t] * row_bytes, (size_t)row_bytes);
}

/* ------------------------------------------------------------------------
 * Fused add-residual + RMSNorm.
 * Follows test/kernel/test_fused_add_residual_rmsnorm.cu:21-52:
 *   x_after = add ? x + residual : x
 *   inv_rms = 1 / sqrt(sum(x_after^2) / D + eps)   (sequential fp32 sum)
 *   residual_out = x_after * w * inv_rms
 * ------------------------------------------------------------------------ */
void orc_fused_add_residual_rmsnorm(const float *x, const float *residual, const float *w,
                                    int64_t n_tokens, int64_t dim, int add_residual,
                                    float *x_after, float *residual_out)
{
    for (int64_t t = 0; t < n_tokens; ++t)
    {
        float sq_sum = 0.0f;
        for (int64_t d = 0; d < dim; ++d)
        {
            const int64_t idx = t * dim + d;
            const float x_val = add_residual ? x[idx] + residual[idx] : x[idx];
            x_after[idx] = x_val;
            sq_sum += x_val * x_val;
        }
        const float inv_rms = 1.0f / sqrtf(sq_sum / (float)dim + ORC_RMSNORM_EPS);
        for (int64_t d = 0; d < dim; ++d)
        {
            const int64_t idx = t * dim + d;
            residual_out[idx] = x_after[idx] * w[d] * inv_rms;
        }
    }
}

/* ------------------------------------------------------------------------
 * RoPE angle for pair index i of a head of size head_dim, at position pos,
 * for a sequence whose total length is seq_len.
 * Follows test/kernel/test_fused_reshape_rope_kvcache_decode.cu:26-30
 * (same expression in the three other RoPE tests):
 *   theta = 1 / powf(10000, 2i / hd)
 *   alpha = 1 / powf(max(1, seq_len / 4096), 2i / (hd - 2))
 *   angle = pos * alpha * theta
 * ------------------------------------------------------------------------ */
void orc_rope_cos_sin(uint32_t i, uint32_t head_dim, uint32_t pos, uint32_t seq_len,
                      float *cos_out, float *sin_out)
{
    const float theta = 1.f / powf(ORC_ROPE_BASE, 2.f * (float)i / (float)head_dim);
    const float ratio = (float)seq_len / ORC_TRAIN_SEQ_LEN;
    const float alpha = 1.f / powf(ratio > 1.f ? ratio : 1.f,
                                   2.f * (float)i / (float)(uint32_t)(head_dim - 2u));
    const float angle = (float)pos * alpha * theta;
    *cos_out = cosf(angle);
    *sin_out = sinf(angle);
}

/* Rotates one head (head_dim floats) in place semantics: out may not alias in.
 * pairing 0: pairs (2i, 2i+1) — test_fused_reshape_rope_kvcache_decode.cu:14-35.
 * pairing 1: pairs (i, i+hd/2) — test_fused_reshape_rope_kvcache_llama2_decode.cu:14-36. */
static void orc_rotate_head(int pairing, const float *head, int64_t head_dim,
                            uint32_t pos, uint32_t seq_len, float *out)
{
    const int64_t half = head_dim / 2;
    for (int64_t i = 0; i < half; ++i)
    {
        const int64_t i0 = pairing ? i : 2 * i;
        const int64_t i1 = pairing ? i + half : 2 * i + 1;
        const float x0 = head[i0];
        const float x1 = head[i1];
        float c, s;
        orc_rope_cos_sin((uint32_t)i, (uint32_t)head_dim, pos, seq_len, &c, &s);
        out[i0] = c * x0 - s * x1;
        out[i1] = s * x0 + c * x1;
    }
}

/* One head rotated as above (exported for the CPU chain runner). */
void orc_rotate_one_head(int pairing, const float *head, int64_t head_dim, uint32_t pos, uint32_t seq_len,
                         float *out)
{
    orc_rotate_head(pairing, head, head_dim, pos, seq_len, out);
}

/* ------------------------------------------------------------------------
 * Decode RoPE + KV-cache append.
 * Follows compute_expected_decode, test_fused_reshape_rope_kvcache_decode.cu:37-97
 * (pairing 0) and test_fused_reshape_rope_kvcache_llama2_decode.cu:38-98
 * (pairing 1). For every sequence that is not done, with kv_len = kv_lens[b]
 * and pos = kv_len - 1:
 *   q[b, h, 0, :]      = rope(input head h)
 *   k[b, h, pos, :]    = rope(input head Hq + h)
 *   v[b, h, pos, :]    = input head Hq + Hkv + h
 * Only those rows are written; everything else in q, k, v is left as is.
 * input: [batch, (Hq + 2 Hkv) * hd]; q: [batch, Hq, 1, hd];
 * k, v: [batch, Hkv, kv_cache_len, hd].
 * ------------------------------------------------------------------------ */
void orc_rope_kvcache_decode(int pairing, const float *input, const uint8_t *is_done,
                             const uint32_t *kv_lens, int64_t batch, int64_t q_heads,
                             int64_t kv_heads, int64_t head_dim, int64_t kv_cache_len,
                             float *q, float *k, float *v)
{
    const int64_t total_heads = q_heads + 2 * kv_heads;
    for (int64_t b = 0; b < batch; ++b)
    {
        if (is_done[b])
            continue;
        const uint32_t kv_len = kv_lens[b];
        const uint32_t pos = kv_len - 1u;
        for (int64_t h = 0; h < q_heads; ++h)
            orc_rotate_head(pairing, input + (b * total_heads + h) * head_dim, head_dim, pos,
                            kv_len, q + (b * q_heads + h) * head_dim);
        for (int64_t h = 0; h < kv_heads; ++h)
            orc_rotate_head(pairing, input + (b * total_heads + q_heads + h) * head_dim, head_dim,
                            pos, kv_len,
                            k + ((b * kv_heads + h) * kv_cache_len + pos) * head_dim);
        for (int64_t h = 0; h < kv_heads; ++h)
            memcpy(v + ((b * kv_heads + h) * kv_cache_len + pos) * head_dim,
                   input + (b * total_heads + q_heads + kv_heads + h) * head_dim,
                   (size_t)head_dim * sizeof(float));
    }
}

/* ------------------------------------------------------------------------
 * Prefill RoPE + pad/transpose + KV-cache append.
 * Follows compute_expected, test_fused_pad_reshape_transpose_rope_kvcache.cu:57-124
 * (pairing 0) and compute_expected_llama2,
 * test_fused_pad_reshape_transpose_rope_kvcache_llama2.cu:60-127 (pairing 1).
 * Unpadded token idx maps to (seq, t) = divmod(unpad_to_pad[idx], q_cache_len);
 * history = kv_len - q_len; pos = history + t:
 *   q[seq, h, t, :]   = rope(input[idx] head h)
 *   k[seq, h, pos, :] = rope(input[idx] head Hq + h)
 *   v[seq, h, pos, :] = input[idx] head Hq + Hkv + h
 * ------------------------------------------------------------------------ */
void orc_rope_kvcache_prefill(int pairing, const float *input, const uint32_t *q_lens,
                              const uint32_t *kv_lens, const uint32_t *unpad_to_pad,
                              int64_t n_tokens, int64_t q_heads, int64_t kv_heads,
                              int64_t head_dim, int64_t q_cache_len, int64_t kv_cache_len,
                              float *q, float *k, float *v)
{
    const int64_t total_heads = q_heads + 2 * kv_heads;
    for (int64_t idx = 0; idx < n_tokens; ++idx)
    {
        const int64_t padded = unpad_to_pad[idx];
        const int64_t seq = padded / q_cache_len;
        const int64_t t = padded - q_cache_len * seq;
        const uint32_t kv_len = kv_lens[seq];
        const uint32_t history = kv_len - q_lens[seq];
        const uint32_t pos = (uint32_t)t + history;
        for (int64_t h = 0; h < q_heads; ++h)
            orc_rotate_head(pairing, input + (idx * total_heads + h) * head_dim, head_dim, pos,
                            kv_len, q + ((seq * q_heads + h) * q_cache_len + t) * head_dim);
        for (int64_t h = 0; h < kv_heads; ++h)
            orc_rotate_head(pairing, input + (idx * total_heads + q_heads + h) * head_dim,
                            head_dim, pos, kv_len,
                            k + ((seq * kv_heads + h) * kv_cache_len + pos) * head_dim);
        for (int64_t h = 0; h < kv_heads; ++h)
            memcpy(v + ((seq * kv_heads + h) * kv_cache_len + pos) * head_dim,
                   input + (idx * total_heads + q_heads + kv_heads + h) * head_dim,
                   (size_t)head_dim * sizeof(float));
    }
}

/* ------------------------------------------------------------------------
 * Length update.
 * Follows compute_expected, test/kernel/test_update_q_kv_lens.cu:11-28:
 *   kv_lens[i] += q_lens[i]; max_q = max(q_lens); max_kv = max(new kv_lens).
 * ------------------------------------------------------------------------ */
void orc_update_q_kv_lens(const uint32_t *q_lens, uint32_t *kv_lens, int64_t batch,
                          uint32_t *max_q_len, uint32_t *max_kv_len)
{
    uint32_t mq = 0, mkv = 0;
    for (int64_t i = 0; i < batch; ++i)
    {
        mq = q_lens[i] > mq ? q_lens[i] : mq;
        kv_lens[i] = kv_lens[i] + q_lens[i];
        mkv = kv_lens[i] > mkv ? kv_lens[i] : mkv;
    }
    *max_q_len = mq;
    *max_kv_len = mkv;
}

/* ------------------------------------------------------------------------
 * Causal mask, reference expression.
 * Follows compute_expected_causal_mask, test/kernel/test_build_causal_mask.cu:13-44,
 * evaluated in 32-bit unsigned arithmetic exactly as the reference does
 * (src/kernel/build_causal_mask.cu:35). Note: kv_id - (kv_len - q_len)
 * wraps for kv_id < kv_len - q_len, so history positions come out 0 when
 * kv_len > q_len. Only [0, max_q) x [0, max_kv) of each sequence is
 * written; mask is [batch, q_cache_len, kv_cache_len] u8.
 * ------------------------------------------------------------------------ */
void orc_build_causal_mask(const uint32_t *q_lens, const uint32_t *kv_lens, int64_t batch,
                           uint32_t max_q_len, uint32_t max_kv_len, int64_t q_cache_len,
                           int64_t kv_cache_len, uint8_t *mask)
{
    for (int64_t s = 0; s < batch; ++s)
    {
        const uint32_t q_len = q_lens[s];
        const uint32_t kv_len = kv_lens[s];
        for (uint32_t qi = 0; qi < max_q_len; ++qi)
            for (uint32_t ki = 0; ki < max_kv_len; ++ki)
            {
                const int is_one = qi < q_len && ki < kv_len && qi >= (uint32_t)(ki - (kv_len - q_len));
                mask[(s * q_cache_len + qi) * kv_cache_len + ki] = (uint8_t)is_one;
            }
    }
}

/* Intended causal mask of the fused score kernels: query row qi of a
 * sequence with q_len new tokens and kv_len total tokens may see key ki iff
 * qi < q_len, ki < kv_len and ki <= (kv_len - q_len) + qi (positions 0..pos).
 * This equals the reference expression whenever kv_len == q_len. Same
 * storage rules as orc_build_causal_mask. */
void orc_build_intended_mask(const uint32_t *q_lens, const uint32_t *kv_lens, int64_t batch,
                             uint32_t max_q_len, uint32_t max_kv_len, int64_t q_cache_len,
                             int64_t kv_cache_len, uint8_t *mask)
{
    for (int64_t s = 0; s < batch; ++s)
    {
        const int64_t q_len = q_lens[s];
        const int64_t kv_len = kv_lens[s];
        for (int64_t qi = 0; qi < (int64_t)max_q_len; ++qi)
            for (int64_t ki = 0; ki < (int64_t)max_kv_len; ++ki)
            {
                const int is_one = qi < q_len && ki < kv_len && ki <= (kv_len - q_len) + qi;
                mask[(s * q_cache_len + qi) * kv_cache_len + ki] = (uint8_t)is_one;
            }
    }
}

/* ------------------------------------------------------------------------
 * Unpad -> pad index map and sequence offsets.
 * Follows compute_expected_maps, test/kernel/test_build_padding_index_maps.cu:10-34:
 *   seq_offsets[s] = sum(seq_lens[:s]); unpad_to_pad[off_s + i] = s * q_cache_len + i.
 * ------------------------------------------------------------------------ */
void orc_build_padding_index_maps(const uint32_t *seq_lens, int64_t batch, int64_t q_cache_len,
                                  uint32_t *unpad_to_pad, uint32_t *seq_offsets)
{
    uint32_t acc = 0;
    for (int64_t s = 0; s < batch; ++s)
    {
        seq_offsets[s] = acc;
        for (uint32_t i = 0; i < seq_lens[s]; ++i)
            unpad_to_pad[acc + i] = (uint32_t)(s * q_cache_len + i);
        acc += seq_lens[s];
    }
}

/* ------------------------------------------------------------------------
 * Batched-GEMM pointer arrays (as byte addresses).
 * Follows the pointer expectations of run_pointer_array_test,
 * test/kernel/test_build_q_k_v_qk_qkv_array.cu:84-130: for slot
 * idx = b * Hq + qh, kv_idx = b * Hkv + qh / (Hq / Hkv):
 *   out[0] q + idx * stride_q,        out[1] q_decode + idx * stride_q_decode,
 *   out[2] k + kv_idx * stride_k,     out[3] v + kv_idx * stride_v,
 *   out[4] qk + idx * stride_qk,      out[5] qk_decode + idx * stride_qk_decode,
 *   out[6] qkv + idx * stride_qkv,    out[7] qkv_decode + idx * stride_qkv_decode.
 * bases and strides are in bytes; out is [8][batch * Hq].
 * ------------------------------------------------------------------------ */
void orc_build_ptr_arrays(const uint64_t *bases, const uint64_t *strides, int64_t batch,
                          int64_t q_heads, int64_t kv_heads, uint64_t *out)
{
    const int64_t n = batch * q_heads;
    const int64_t group = q_heads / kv_heads;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t qh = 0; qh < q_heads; ++qh)
        {
            const int64_t idx = b * q_heads + qh;
            const int64_t kv_idx = b * kv_heads + qh / group;
            for (int a = 0; a < 8; ++a)
            {
                const int64_t slot = (a == 2 || a == 3) ? kv_idx : idx;
                out[a * n + idx] = bases[a] + (uint64_t)slot * strides[a];
            }
        }
}

/* ------------------------------------------------------------------------
 * Row-major GEMM C[M, N] = op(A) op(B).
 * Follows compute_expected_linear, test/kernel/test_linear.cu:78-108
 * (sequential fp32 accumulation over k).
 * ------------------------------------------------------------------------ */
void orc_linear(const float *A, const float *B, int trans_a, int trans_b, int64_t M, int64_t N,
                int64_t K, float *C)
{
    const int64_t a_row = trans_a ? 1 : K, a_col = trans_a ? M : 1;
    const int64_t b_row = trans_b ? 1 : N, b_col = trans_b ? K : 1;
    for (int64_t i = 0; i < M; ++i)
        for (int64_t j = 0; j < N; ++j)
        {
            float sum = 0.0f;
            for (int64_t kk = 0; kk < K; ++kk)
                sum += A[i * a_row + kk * a_col] * B[kk * b_row + j * b_col];
            C[i * N + j] = sum;
        }
}

/* ------------------------------------------------------------------------
 * QK^T at the launch_linear call site (trans_B = true), per (b, q head),
 * with GQA (kv head = qh / (Hq / Hkv)), over rows i < M and keys j < N:
 *   qk[b, qh, i, j] = sum_d q[b, qh, i, d] * k[b, kvh, j, d]
 * Same accumulation as orc_linear. q: [B, Hq, Qc, hd]; k: [B, Hkv, S, hd];
 * qk: [B, Hq, Qc, S]; entries outside i < M, j < N are left as is.
 * ------------------------------------------------------------------------ */
void orc_qk_scores(const float *q, const float *k, int64_t batch, int64_t q_heads,
                   int64_t kv_heads, int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim,
                   int64_t M, int64_t N, float *qk)
{
    const int64_t group = q_heads / kv_heads;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t qh = 0; qh < q_heads; ++qh)
        {
            const float *qs = q + (b * q_heads + qh) * q_cache_len * head_dim;
            const float *ks = k + (b * kv_heads + qh / group) * kv_cache_len * head_dim;
            float *out = qk + (b * q_heads + qh) * q_cache_len * kv_cache_len;
            for (int64_t i = 0; i < M; ++i)
                for (int64_t j = 0; j < N; ++j)
                {
                    float sum = 0.0f;
                    for (int64_t d = 0; d < head_dim; ++d)
                        sum += qs[i * head_dim + d] * ks[j * head_dim + d];
                    out[i * kv_cache_len + j] = sum;
                }
        }
}

/* ------------------------------------------------------------------------
 * Masked attention score (scale + mask + softmax), in place.
 * Follows compute_expected_masked_attention_score,
 * test/kernel/test_compute_masked_attention_score.cu:21-89, and the
 * kernel's storage rules (src/kernel/compute_masked_attention_score.cu:40-47):
 * for rows q < q_lens[b] and keys k < max_kv_len,
 *   qk = mask ? expf(qk * s - m) / (sum + 1e-6) : 0,   s = 1 / sqrtf(hd),
 * m and sum taken over masked-in keys; all other entries are left as is.
 * qk: [B, H, Qc, S] fp32; mask: [B, Qc, S] u8.
 * ------------------------------------------------------------------------ */
void orc_masked_attention_score(float *qk, const uint8_t *mask, const uint32_t *q_lens,
                                int64_t batch, int64_t q_heads, int64_t q_cache_len,
                                int64_t kv_cache_len, int64_t max_kv_len, int64_t head_dim)
{
    const float scale = 1.f / sqrtf((float)head_dim);
    for (int64_t s = 0; s < batch; ++s)
        for (int64_t h = 0; h < q_heads; ++h)
            for (int64_t qi = 0; qi < (int64_t)q_lens[s]; ++qi)
            {
                float *row = qk + ((s * q_heads + h) * q_cache_len + qi) * kv_cache_len;
                const uint8_t *mrow = mask + (s * q_cache_len + qi) * kv_cache_len;
                float max_val = -INFINITY;
                for (int64_t ki = 0; ki < max_kv_len; ++ki)
                    if (mrow[ki])
                    {
                        const float val = row[ki] * scale;
                        max_val = val > max_val ? val : max_val;
                    }
                float sum = 0.f;
                for (int64_t ki = 0; ki < max_kv_len; ++ki)
                    if (mrow[ki])
                        sum += expf(row[ki] * scale - max_val);
                for (int64_t ki = 0; ki < max_kv_len; ++ki)
                    row[ki] = mrow[ki] ? expf(row[ki] * scale - max_val) / (sum + ORC_SOFTMAX_EPS) : 0.f;
            }
}

/* ------------------------------------------------------------------------
 * SwiGLU.
 * Follows compute_expected_swiglu, test/kernel/test_swiglu.cu:72-91:
 *   out[t, i] = x * (1 / (1 + exp(-x))) * y,  x = in[t, i], y = in[t, F + i].
 * ------------------------------------------------------------------------ */
void orc_swiglu(const float *in, int64_t n_tokens, int64_t inter, float *out)
{
    for (int64_t t = 0; t < n_tokens; ++t)
        for (int64_t i = 0; i < inter; ++i)
        {
            const float x = in[t * 2 * inter + i];
            const float y = in[t * 2 * inter + inter + i];
            const float sigmoid_x = 1.0f / (1.0f + expf(-x));
            out[t * inter + i] = x * sigmoid_x * y;
        }
}

/* ------------------------------------------------------------------------
 * Transpose + unpad of the attention output (byte copy, any element size).
 * Follows the expected-result loop of run_fused_transpose_unpad_test,
 * test/kernel/test_fused_transpose_unpad.cu:148-167, with the token's padded
 * slot taken from unpad_to_pad (the reference kernel's addressing,
 * src/kernel/fused_transpose_unpad.cu:30-38):
 *   p = unpad_to_pad[t], b = p / Qc, i = p % Qc,
 *   out[t, h * hd + d] = qkv[b, h, i, d].
 * A slot p >= batch * Qc (which the reference would read out of bounds)
 * gives a zero row here, as the CUDA operator does.
 * ------------------------------------------------------------------------ */
void orc_transpose_unpad(const void *qkv, const uint32_t *unpad_to_pad, int64_t n_tokens, int64_t batch,
                         int64_t heads, int64_t q_cache_len, int64_t head_dim, int64_t elem_size, void *out)
{
    const int64_t row = head_dim * elem_size;
    const char *src = (const char *)qkv;
    char *dst = (char *)out;
    for (int64_t t = 0; t < n_tokens; ++t)
    {
        const int64_t p = unpad_to_pad[t];
        for (int64_t h = 0; h < heads; ++h)
        {
            char *d = dst + (t * heads + h) * row;
            if (p >= batch * q_cache_len)
            {
                memset(d, 0, (size_t)row);
                continue;
            }
            const int64_t b = p / q_cache_len, i = p % q_cache_len;
            memcpy(d, src + ((b * heads + h) * q_cache_len + i) * row, (size_t)row);
        }
    }
}

/* ------------------------------------------------------------------------
 * P.V at the reference's launch_linear call site (trans_A = trans_B =
 * false), per (b, q head) with grouped KV heads:
 *   qkv[b, h, i, d] = sum_{j < n} qk[b, h, i, j] * v[b, h / (Hq/Hkv), j, d]
 * for rows i < m; other rows untouched. Summation in j order in fp32, as
 * compute_expected_linear does (test/kernel/test_linear.cu:78-108).
 * qk: (B, Hq, Qc, S); v: (B, Hkv, S, hd); qkv: (B, Hq, Qc, hd).
 * ------------------------------------------------------------------------ */
void orc_attention_qkv(const float *qk, const float *v, int64_t batch, int64_t q_heads, int64_t kv_heads,
                       int64_t q_cache_len, int64_t kv_cache_len, int64_t head_dim, int64_t m, int64_t n,
                       float *qkv)
{
    const int64_t group = q_heads / kv_heads;
    for (int64_t b = 0; b < batch; ++b)
        for (int64_t h = 0; h < q_heads; ++h)
        {
            const float *vh = v + (b * kv_heads + h / group) * kv_cache_len * head_dim;
            for (int64_t i = 0; i < m; ++i)
            {
                const float *p = qk + ((b * q_heads + h) * q_cache_len + i) * kv_cache_len;
                float *o = qkv + ((b * q_heads + h) * q_cache_len + i) * head_dim;
                for (int64_t d = 0; d < head_dim; ++d)
                {
                    float acc = 0.f;
                    for (int64_t j = 0; j < n; ++j)
                        acc += p[j] * vh[j * head_dim + d];
                    o[d] = acc;
                }
            }
        }
}

/* ------------------------------------------------------------------------
 * fp8 (e4m3) cache elements — no counterpart in the reference (its DataType
 * stops at FP32/FP16/INT8, include/common/types.h:60-71). The format is the
 * OCP 8-bit floating point "E4M3": sign bit, 4 exponent bits with bias 7,
 * 3 mantissa bits, no infinities, largest finite magnitude 448 = 1.75 * 2^8,
 * smallest normal 2^-6, subnormals m * 2^-9 (m = 1..7), NaN = S.1111.111.
 *
 * orc_e4m3_from_f32: y = x * inv_scale (one fp32 multiply), then y rounded
 *   to the nearest e4m3 value, ties to an even mantissa; magnitudes above
 *   448 saturate to 448 (the saturating conversion the cache writers use);
 *   NaN -> 0x7F.
 * orc_e4m3_to_f32: the exact value of each byte, times scale (fp32).
 * ------------------------------------------------------------------------ */
static uint8_t orc_e4m3_round(float y)
{
    if (y != y)
        return 0x7F;
    const uint8_t sign = (uint8_t)(signbit(y) ? 0x80 : 0x00);
    double a = fabs((double)y);
    if (a >= 448.0)
        return (uint8_t)(sign | 0x7E);
    if (a < 0.015625) /* below 2^-6: subnormal multiples of 2^-9 (8 * 2^-9 is the smallest normal) */
    {
        const double m = nearbyint(a * 512.0); /* default rounding mode: to nearest, ties to even */
        return (uint8_t)(sign | (uint8_t)m);
    }
    int e2;
    const double f = frexp(a, &e2); /* a = f * 2^e2, f in [0.5, 1) */
    int e = e2 - 1;                 /* a = (2 f) * 2^e, 2 f in [1, 2) */
    double q = nearbyint((2.0 * f - 1.0) * 8.0);
    if (q == 8.0)
    {
        q = 0.0;
        ++e;
    }
    if (e > 8 || (e == 8 && q == 7.0)) /* 480 is not finite in e4m3: saturate */
        return (uint8_t)(sign | 0x7E);
    return (uint8_t)(sign | (uint8_t)((e + 7) << 3) | (uint8_t)q);
}

void orc_e4m3_from_f32(const float *x, int64_t n, float inv_scale, uint8_t *out)
{
    for (int64_t i = 0; i < n; ++i)
    {
        const float y = x[i] * inv_scale;
        out[i] = orc_e4m3_round(y);
    }
}

static float orc_e4m3_value(uint8_t b)
{
    const int e = (b >> 3) & 0xF, m = b & 7;
    if (e == 0xF && m == 7)
        return NAN;
    const double mag = e == 0 ? ldexp((double)m, -9) : ldexp(1.0 + m / 8.0, e - 7);
    return (float)((b & 0x80) ? -mag : mag);
}

void orc_e4m3_to_f32(const uint8_t *x, int64_t n, float scale, float *out)
{
    for (int64_t i = 0; i < n; ++i)
        out[i] = orc_e4m3_value(x[i]) * scale;
}
