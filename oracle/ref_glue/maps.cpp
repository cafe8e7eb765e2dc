// Glue for test/kernel/test_build_padding_index_maps.cu (reference).
#include "test/kernel/test_build_padding_index_maps.cu"
#include "common.h"

extern "C" void ref_build_padding_index_maps(const unsigned int *seq_lens, unsigned int B, unsigned int max_seq_len,
                                             unsigned int *unpad_to_pad, unsigned int *seq_offsets)
{
    std::vector<unsigned int> u, o;
    compute_expected_maps(ref_glue_vec(seq_lens, B), max_seq_len, u, o);
    ref_glue_out(u, unpad_to_pad);
    ref_glue_out(o, seq_offsets);
}
