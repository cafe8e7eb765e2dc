// Glue for test/kernel/test_embedding.cu (reference). The test has no
// separate expected-value helper: its expectation is the inline loop at
// test_embedding.cu:50-61 (out[t, d] = table[ids[t] * D + d]), written
// here as the same loop. fill_sequential (:11-16) is the reference's own.
#include "test/kernel/test_embedding.cu"
#include "common.h"

extern "C" void ref_fill_sequential(float *data, unsigned int n, float start) { fill_sequential(data, n, start); }

extern "C" void ref_embedding(const unsigned int *ids, unsigned int token_num, const float *table,
                              unsigned int embed_dim, float *out)
{
    for (unsigned int t = 0; t < token_num; ++t)
        for (unsigned int d = 0; d < embed_dim; ++d)
            out[t * embed_dim + d] = table[ids[t] * embed_dim + d];
}
