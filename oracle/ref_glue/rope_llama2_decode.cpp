// Glue for test/kernel/test_fused_reshape_rope_kvcache_llama2_decode.cu (reference).
#include "test/kernel/test_fused_reshape_rope_kvcache_llama2_decode.cu"
#include "common.h"

extern "C" void ref_rope_kvcache_llama2_decode(const float *input, const unsigned char *is_done,
                                               const unsigned int *kv_lens, unsigned int B, unsigned int Hq,
                                               unsigned int Hkv, unsigned int S, float *q, float *k, float *v)
{
    std::vector<float> eq, ek, ev;
    compute_expected_decode(ref_glue_vec(is_done, B), ref_glue_vec(kv_lens, B), S, Hq, Hkv,
                            ref_glue_vec(input, size_t(B) * (Hq + 2 * Hkv) * 128), eq, ek, ev);
    ref_glue_out(eq, q);
    ref_glue_out(ek, k);
    ref_glue_out(ev, v);
}

// One head rotated by the reference's own apply_rotation_llama2_decode (:14-36),
// without compute_expected_decode's whole-cache output buffers.
extern "C" void ref_rotate_head_llama2(const float *head, unsigned int hd, unsigned int pos, unsigned int seq_len,
                                       float *out)
{
    std::vector<float> o;
    apply_rotation_llama2_decode(ref_glue_vec(head, hd), hd, pos, seq_len, o);
    ref_glue_out(o, out);
}
