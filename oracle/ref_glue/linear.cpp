// Glue for test/kernel/test_linear.cu (reference).
#include "test/kernel/test_linear.cu"
#include "common.h"

extern "C" void ref_linear(const float *A, const float *B, int trans_a, int trans_b, unsigned int M, unsigned int N,
                           unsigned int K, float *C)
{
    std::vector<float> c;
    compute_expected_linear(ref_glue_vec(A, size_t(M) * K), ref_glue_vec(B, size_t(K) * N), trans_a != 0,
                            trans_b != 0, M, N, K, c);
    ref_glue_out(c, C);
}
