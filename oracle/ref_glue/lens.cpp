// Glue for test/kernel/test_update_q_kv_lens.cu (reference).
#include "test/kernel/test_update_q_kv_lens.cu"
#include "common.h"

extern "C" void ref_update_q_kv_lens(const unsigned int *q_lens, const unsigned int *kv_lens, unsigned int B,
                                     unsigned int *kv_lens_out, unsigned int *max_q, unsigned int *max_kv)
{
    std::vector<unsigned int> e;
    compute_expected(ref_glue_vec(q_lens, B), ref_glue_vec(kv_lens, B), e, *max_q, *max_kv);
    ref_glue_out(e, kv_lens_out);
}
