// Glue for test/kernel/test_fused_transpose_unpad.cu (reference).
#include "test/kernel/test_fused_transpose_unpad.cu"
#include "common.h"

// compute_unpad_to_pad_idx: the (batch * q_cache_len) index map the test
// hands to the kernel (entries past the token count stay 0).
extern "C" void ref_unpad_to_pad_idx(const unsigned int *q_lens, unsigned int batch, unsigned int q_cache_len,
                                     unsigned int *out)
{
    ref_glue_out(compute_unpad_to_pad_idx(batch, q_cache_len, ref_glue_vec(q_lens, batch)), out);
}
