// Glue for test/kernel/test_compute_masked_attention_score.cu (reference).
#include "test/kernel/test_compute_masked_attention_score.cu"
#include "common.h"

extern "C" void ref_fill_random_qk_f32(float *out, unsigned int n)
{
    std::vector<float> v(n);
    fill_random_qk(v);
    ref_glue_out(v, out);
}

extern "C" void ref_fill_random_qk_f16(unsigned short *out, unsigned int n)
{
    std::vector<half> v(n);
    fill_random_qk(v);
    std::memcpy(out, v.data(), n * sizeof(half));
}

extern "C" void ref_masked_attention_score_f32(const float *qk, const unsigned char *mask, const unsigned int *q_lens,
                                               unsigned int B, unsigned int H, unsigned int Qc, unsigned int S,
                                               unsigned int max_kv, unsigned int hd, float *expected)
{
    std::vector<float> e;
    compute_expected_masked_attention_score(ref_glue_vec(qk, size_t(B) * H * Qc * S),
                                            ref_glue_vec(mask, size_t(B) * Qc * S), ref_glue_vec(q_lens, B), B, H, Qc,
                                            S, max_kv, hd, e);
    ref_glue_out(e, expected);
}

extern "C" void ref_masked_attention_score_f16(const unsigned short *qk, const unsigned char *mask,
                                               const unsigned int *q_lens, unsigned int B, unsigned int H,
                                               unsigned int Qc, unsigned int S, unsigned int max_kv, unsigned int hd,
                                               unsigned short *expected)
{
    const size_t n = size_t(B) * H * Qc * S;
    std::vector<half> in(n), e;
    std::memcpy(in.data(), qk, n * sizeof(half));
    compute_expected_masked_attention_score(in, ref_glue_vec(mask, size_t(B) * Qc * S), ref_glue_vec(q_lens, B), B, H,
                                            Qc, S, max_kv, hd, e);
    std::memcpy(expected, e.data(), n * sizeof(half));
}
