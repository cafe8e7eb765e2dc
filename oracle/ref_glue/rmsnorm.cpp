// Glue for test/kernel/test_fused_add_residual_rmsnorm.cu (reference).
#include "test/kernel/test_fused_add_residual_rmsnorm.cu"
#include "common.h"
#include <random>

extern "C" void ref_fused_add_residual_rmsnorm(const float *x, const float *residual, const float *w,
                                               unsigned int T, unsigned int D, int add_residual,
                                               float *x_after, float *residual_out)
{
    std::vector<float> xa, ro;
    compute_expected_fused_add_residual_rmsnorm(ref_glue_vec(x, size_t(T) * D), ref_glue_vec(residual, size_t(T) * D),
                                                ref_glue_vec(w, D), T, D, add_residual != 0, xa, ro);
    ref_glue_out(xa, x_after);
    ref_glue_out(ro, residual_out);
}

// Inputs of the randomized cases (LargeBatchRandomValues, :234-259, :322-347,
// :398-423, :471-494): the same generator, distributions and draw order.
extern "C" void ref_rmsnorm_random_inputs(unsigned int seed, int with_residual, unsigned int T, unsigned int D,
                                          float *x, float *residual, float *w)
{
    std::mt19937 gen(seed);
    std::uniform_real_distribution<float> x_dist(-2.0f, 2.0f);
    std::uniform_real_distribution<float> residual_dist(-1.0f, 1.0f);
    std::uniform_real_distribution<float> weight_dist(0.1f, 2.0f);
    for (unsigned int i = 0; i < T * D; ++i)
    {
        x[i] = x_dist(gen);
        residual[i] = with_residual ? residual_dist(gen) : 0.0f;
    }
    for (unsigned int d = 0; d < D; ++d)
        w[d] = weight_dist(gen);
}
