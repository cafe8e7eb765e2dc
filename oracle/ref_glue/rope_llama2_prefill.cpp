// Glue for test/kernel/test_fused_pad_reshape_transpose_rope_kvcache_llama2.cu (reference).
#include "test/kernel/test_fused_pad_reshape_transpose_rope_kvcache_llama2.cu"
#include "common.h"

extern "C" void ref_rope_kvcache_llama2_prefill(const float *input, const unsigned int *q_lens,
                                                const unsigned int *kv_lens, const unsigned int *unpad_to_pad,
                                                unsigned int T, unsigned int B, unsigned int Hq, unsigned int Hkv,
                                                unsigned int Qc, unsigned int S, float *q, float *k, float *v)
{
    std::vector<float> eq, ek, ev;
    compute_expected_llama2(ref_glue_vec(q_lens, B), ref_glue_vec(kv_lens, B), ref_glue_vec(unpad_to_pad, T), Qc, S,
                            Hq, Hkv, ref_glue_vec(input, size_t(T) * (Hq + 2 * Hkv) * 128), eq, ek, ev);
    ref_glue_out(eq, q);
    ref_glue_out(ek, k);
    ref_glue_out(ev, v);
}
