// Glue for test/kernel/test_swiglu.cu (reference).
#include "test/kernel/test_swiglu.cu"
#include "common.h"
#include <random>

extern "C" void ref_swiglu(const float *in, unsigned int T, unsigned int F, float *out)
{
    std::vector<float> e;
    compute_expected_swiglu(ref_glue_vec(in, size_t(T) * 2 * F), T, F, e);
    ref_glue_out(e, out);
}

// Inputs of the randomized cases (LargeBatchRandomValues, :169-184, :217-230).
extern "C" void ref_swiglu_random_inputs(unsigned int seed, unsigned int n, float *out)
{
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> dist(-2.0f, 2.0f);
    for (unsigned int i = 0; i < n; ++i)
        out[i] = dist(gen);
}
