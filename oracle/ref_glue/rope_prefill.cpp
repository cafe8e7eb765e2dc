// Glue for test/kernel/test_fused_pad_reshape_transpose_rope_kvcache.cu (reference).
#include "test/kernel/test_fused_pad_reshape_transpose_rope_kvcache.cu"
#include "common.h"

extern "C" void ref_prefill_unpad_to_pad_idx(const unsigned int *q_lens, unsigned int B, unsigned int Qc,
                                             unsigned int *out)
{
    std::vector<unsigned int> m;
    compute_unpad_to_pad_idx(ref_glue_vec(q_lens, B), Qc, m);
    ref_glue_out(m, out);
}

extern "C" void ref_rope_kvcache_prefill(const float *input, const unsigned int *q_lens, const unsigned int *kv_lens,
                                         const unsigned int *unpad_to_pad, unsigned int T, unsigned int B,
                                         unsigned int Hq, unsigned int Hkv, unsigned int hd, unsigned int Qc,
                                         unsigned int S, float *q, float *k, float *v)
{
    std::vector<float> eq, ek, ev;
    compute_expected(ref_glue_vec(q_lens, B), ref_glue_vec(kv_lens, B), ref_glue_vec(unpad_to_pad, T), Qc, S, Hq, Hkv,
                     hd, ref_glue_vec(input, size_t(T) * (Hq + 2 * Hkv) * hd), eq, ek, ev);
    ref_glue_out(eq, q);
    ref_glue_out(ek, k);
    ref_glue_out(ev, v);
}
