// Glue for test/kernel/test_build_causal_mask.cu (reference).
#include "test/kernel/test_build_causal_mask.cu"
#include "common.h"

extern "C" void ref_build_causal_mask(const unsigned int *q_lens, const unsigned int *kv_lens, unsigned int B,
                                      unsigned int max_q, unsigned int max_kv, unsigned int Qc, unsigned int S,
                                      unsigned char *mask)
{
    std::vector<unsigned char> m;
    compute_expected_causal_mask(ref_glue_vec(q_lens, B), ref_glue_vec(kv_lens, B), max_q, max_kv, Qc, S, m);
    ref_glue_out(m, mask);
}
