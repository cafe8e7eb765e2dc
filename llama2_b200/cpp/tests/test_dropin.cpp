// Tests of the C++ operator API (drop-in for the reference's
// include/kernel/*.h), written the way the reference's own GoogleTest cases
// are: host inputs -> Tensor<T> on the GPU -> launch_* -> copy back ->
// compare with the CPU expectation. The expectations come from the oracle
// (oracle/oracle.c, linked as test infrastructure). A minimal test runner
// replaces GoogleTest (not available offline). Exit status 0 = all passed.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <functional>
#include <random>
#include <string>
#include <vector>

#include "core/Tensor.cuh"
#include "kernel/attention_scores.h"
#include "kernel/build_causal_mask.h"
#include "kernel/build_padding_index_maps.h"
#include "kernel/build_q_k_v_qk_qkv_array.h"
#include "kernel/compute_masked_attention_score.h"
#include "kernel/embedding.h"
#include "kernel/fused_add_residual_rmsnorm.h"
#include "kernel/fused_pad_reshape_transpose_rope_kvcache_llama2.h"
#include "kernel/fused_reshape_rope_kvcache_decode.h"
#include "kernel/fused_reshape_rope_kvcache_llama2_decode.h"
#include "kernel/fused_transpose_unpad.h"
#include "kernel/linear.h"
#include "kernel/swiglu.h"
#include "kernel/update_q_kv_lens.h"

extern "C"
{
void orc_fused_add_residual_rmsnorm(const float *, const float *, const float *, int64_t, int64_t, int, float *,
                                    float *);
void orc_rope_kvcache_decode(int, const float *, const uint8_t *, const uint32_t *, int64_t, int64_t, int64_t,
                             int64_t, int64_t, float *, float *, float *);
void orc_rope_kvcache_prefill(int, const float *, const uint32_t *, const uint32_t *, const uint32_t *, int64_t,
                              int64_t, int64_t, int64_t, int64_t, int64_t, float *, float *, float *);
void orc_build_causal_mask(const uint32_t *, const uint32_t *, int64_t, uint32_t, uint32_t, int64_t, int64_t,
                           uint8_t *);
void orc_build_intended_mask(const uint32_t *, const uint32_t *, int64_t, uint32_t, uint32_t, int64_t, int64_t,
                             uint8_t *);
void orc_build_padding_index_maps(const uint32_t *, int64_t, int64_t, uint32_t *, uint32_t *);
void orc_linear(const float *, const float *, int, int, int64_t, int64_t, int64_t, float *);
void orc_qk_scores(const float *, const float *, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                   int64_t, float *);
void orc_masked_attention_score(float *, const uint8_t *, const uint32_t *, int64_t, int64_t, int64_t, int64_t,
                                int64_t, int64_t);
void orc_swiglu(const float *, int64_t, int64_t, float *);
void orc_embedding(const uint32_t *, int64_t, const void *, int64_t, int64_t, void *);
void orc_update_q_kv_lens(const uint32_t *, uint32_t *, int64_t, uint32_t *, uint32_t *);
void orc_transpose_unpad(const void *, const uint32_t *, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, void *);
void orc_attention_qkv(const float *, const float *, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                       int64_t, float *);
}

// ---------------------------------------------------------------------------
// minimal runner
// ---------------------------------------------------------------------------
static std::vector<std::pair<std::string, std::function<void()>>> &registry()
{
    static std::vector<std::pair<std::string, std::function<void()>>> r;
    return r;
}
struct Reg
{
    Reg(const char *n, std::function<void()> f) { registry().emplace_back(n, std::move(f)); }
};
static int g_failures = 0;
#define TEST(suite, name)                                   \
    static void suite##_##name();                           \
    static Reg reg_##suite##_##name(#suite "." #name, suite##_##name); \
    static void suite##_##name()
#define EXPECT_TRUE(cond)                                                           \
    do                                                                              \
    {                                                                               \
        if (!(cond))                                                                \
        {                                                                           \
            std::printf("  FAILED %s:%d: %s\n", __FILE__, __LINE__, #cond);         \
            ++g_failures;                                                           \
            return;                                                                 \
        }                                                                           \
    } while (0)

template <typename T>
static void upload(Tensor<T> &t, const std::vector<T> &h)
{
    CUDA_CHECK(cudaMemcpy(t.data(), h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
}
template <typename T>
static std::vector<T> download(const Tensor<T> &t)
{
    std::vector<T> h(t.numel());
    CUDA_CHECK(cudaMemcpy(h.data(), t.data(), h.size() * sizeof(T), cudaMemcpyDeviceToHost));
    return h;
}
static std::vector<float> pattern(size_t n, int mod, float mul, float sub)
{
    std::vector<float> v(n);
    for (size_t i = 0; i < n; ++i)
        v[i] = static_cast<float>(mod ? i % mod : i) * mul - sub;
    return v;
}
static float max_rel(const std::vector<float> &got, const std::vector<float> &want)
{
    float m = 0.f;
    for (size_t i = 0; i < got.size(); ++i)
    {
        const float d = std::fabs(got[i] - want[i]);
        if (d > 0.f)
            m = std::fmax(m, d / std::fabs(want[i]));
    }
    return m;
}
static std::vector<float> to_f(const std::vector<half> &v)
{
    std::vector<float> o(v.size());
    for (size_t i = 0; i < v.size(); ++i)
        o[i] = __half2float(v[i]);
    return o;
}

// ---------------------------------------------------------------------------
TEST(EmbeddingTest, BasicLookup)
{
    std::vector<unsigned int> ids = {0, 2, 1, 3};
    std::vector<float> table(4 * 8);
    for (size_t i = 0; i < table.size(); ++i)
        table[i] = 0.1f + static_cast<float>(i);
    Tensor<unsigned int> ids_d({4}, GPU);
    Tensor<float> table_d({4, 8}, GPU);
    Tensor<float> out_d({4, 8}, GPU);
    upload(ids_d, ids);
    upload(table_d, table);
    launch_embedding(ids_d, table_d, out_d);
    const auto out = download(out_d);
    for (int t = 0; t < 4; ++t)
        for (int d = 0; d < 8; ++d)
            EXPECT_TRUE(out[t * 8 + d] == table[ids[t] * 8 + d]);
}

TEST(FusedAddResidualRMSNormTest, Fp32AndHalf)
{
    const unsigned int n = 64, d = 64;
    std::mt19937 gen(123);
    std::uniform_real_distribution<float> xd(-2.f, 2.f), rd(-1.f, 1.f), wd(0.1f, 2.f);
    std::vector<float> x(n * d), r(n * d), w(d);
    for (unsigned int i = 0; i < n * d; ++i)
    {
        x[i] = xd(gen);
        r[i] = rd(gen);
    }
    for (auto &v : w)
        v = wd(gen);
    std::vector<float> xa(n * d), ro(n * d);
    orc_fused_add_residual_rmsnorm(x.data(), r.data(), w.data(), n, d, 1, xa.data(), ro.data());
    Tensor<float> w_d({d}, GPU), x_d({n, d}, GPU), r_d({n, d}, GPU);
    upload(w_d, w);
    upload(x_d, x);
    upload(r_d, r);
    launch_fused_add_residual_rmsnorm<float, true>(w_d, x_d, r_d);
    EXPECT_TRUE(download(x_d) == xa);
    EXPECT_TRUE(max_rel(download(r_d), ro) <= 1e-5f);
    // fp16, reference tolerance 1e-2 (test_fused_add_residual_rmsnorm.cu:471-494)
    std::vector<half> wh(d), xh(n * d), rh(n * d);
    for (unsigned int i = 0; i < n * d; ++i)
    {
        xh[i] = __float2half(x[i]);
        rh[i] = __float2half(r[i]);
    }
    for (unsigned int i = 0; i < d; ++i)
        wh[i] = __float2half(w[i]);
    Tensor<half> wh_d({d}, GPU), xh_d({n, d}, GPU), rh_d({n, d}, GPU);
    upload(wh_d, wh);
    upload(xh_d, xh);
    upload(rh_d, rh);
    launch_fused_add_residual_rmsnorm<half, true>(wh_d, xh_d, rh_d);
    const auto got = to_f(download(rh_d));
    for (unsigned int i = 0; i < n * d; ++i)
        EXPECT_TRUE(std::fabs(got[i] - ro[i]) <= 1e-2f);
}

TEST(FusedReshapeRopeKVCacheDecodeTest, WithDoneSequences)
{
    const unsigned int b = 4, hq = 8, hkv = 4, hd = 64, s = 64;
    std::vector<unsigned char> done = {0, 1, 0, 1};
    std::vector<unsigned int> kv = {4, 9, 15, 20};
    const auto input = pattern(b * (hq + 2 * hkv) * hd, 23, 0.05f, 0.5f);
    std::vector<float> eq(b * hq * hd, 0.f), ek(b * hkv * s * hd, 0.f), ev(b * hkv * s * hd, 0.f);
    orc_rope_kvcache_decode(0, input.data(), done.data(), kv.data(), b, hq, hkv, hd, s, eq.data(), ek.data(),
                            ev.data());
    Tensor<float> in_d({b, (hq + 2 * hkv) * hd}, GPU), q_d({b, hq, 1, hd}, GPU), k_d({b, hkv, s, hd}, GPU),
        v_d({b, hkv, s, hd}, GPU);
    Tensor<unsigned char> done_d({b}, GPU);
    Tensor<unsigned int> kv_d({b}, GPU);
    upload(in_d, input);
    upload(done_d, done);
    upload(kv_d, kv);
    launch_fused_reshape_rope_kvcache_decode(in_d, done_d, kv_d, q_d, k_d, v_d);
    EXPECT_TRUE(download(q_d) == eq);
    EXPECT_TRUE(download(k_d) == ek);
    EXPECT_TRUE(download(v_d) == ev);
}

TEST(FusedReshapeRopeKVCacheLlama2DecodeTest, LargeBatchLoopOverGrid)
{
    const unsigned int b = 300, hq = 4, hkv = 2, hd = 128, s = 128;
    std::vector<unsigned char> done(b, 0);
    std::vector<unsigned int> kv(b);
    for (unsigned int i = 0; i < b; ++i)
        kv[i] = (i % 63) + 1;
    const auto input = pattern(b * (hq + 2 * hkv) * hd, 31, 0.03f, 0.4f);
    std::vector<float> eq(b * hq * hd, 0.f), ek(b * hkv * s * hd, 0.f), ev(b * hkv * s * hd, 0.f);
    orc_rope_kvcache_decode(1, input.data(), done.data(), kv.data(), b, hq, hkv, hd, s, eq.data(), ek.data(),
                            ev.data());
    Tensor<float> in_d({b, (hq + 2 * hkv) * hd}, GPU), q_d({b, hq, 1, hd}, GPU), k_d({b, hkv, s, hd}, GPU),
        v_d({b, hkv, s, hd}, GPU);
    Tensor<unsigned char> done_d({b}, GPU);
    Tensor<unsigned int> kv_d({b}, GPU);
    upload(in_d, input);
    upload(done_d, done);
    upload(kv_d, kv);
    launch_fused_reshape_rope_kvcache_llama2_decode(in_d, done_d, kv_d, q_d, k_d, v_d);
    EXPECT_TRUE(download(q_d) == eq);
    EXPECT_TRUE(download(k_d) == ek);
    EXPECT_TRUE(download(v_d) == ev);
}

TEST(PrefillChainTest, MapsRopeAndScores)
{
    const unsigned int b = 2, hq = 4, hkv = 2, hd = 128, qc = 160, s = 192;
    std::vector<unsigned int> q_lens = {150, 37}, kv_lens = {150, 60}; // second: 23 tokens of history
    const unsigned int n = 150 + 37;
    Tensor<unsigned int> ql_d({b}, GPU), kl_d({b}, GPU), unpad_d({b, qc}, GPU), off_d({b}, GPU);
    upload(ql_d, q_lens);
    upload(kl_d, kv_lens);
    launch_build_padding_index_maps(n, ql_d, unpad_d, off_d);
    std::vector<uint32_t> eu(n), eo(b);
    orc_build_padding_index_maps(q_lens.data(), b, qc, eu.data(), eo.data());
    auto u = download(unpad_d);
    u.resize(n);
    EXPECT_TRUE(u == eu);
    EXPECT_TRUE(download(off_d) == eo);
    const auto input = pattern(n * (hq + 2 * hkv) * hd, 19, 0.07f, 0.6f);
    std::vector<float> eq(b * hq * qc * hd, 0.f), ek(b * hkv * s * hd, 0.f), ev(b * hkv * s * hd, 0.f);
    orc_rope_kvcache_prefill(1, input.data(), q_lens.data(), kv_lens.data(), eu.data(), n, hq, hkv, hd, qc, s,
                             eq.data(), ek.data(), ev.data());
    Tensor<float> in_d({n, (hq + 2 * hkv) * hd}, GPU), q_d({b, hq, qc, hd}, GPU), k_d({b, hkv, s, hd}, GPU),
        v_d({b, hkv, s, hd}, GPU);
    upload(in_d, input);
    launch_fused_pad_reshape_transpose_rope_kvcache_llama2(in_d, ql_d, kl_d, unpad_d, q_d, k_d, v_d);
    EXPECT_TRUE(download(q_d) == eq);
    EXPECT_TRUE(download(k_d) == ek);
    // fused causal scores (fp32: QK^T on the CUDA cores + masked softmax)
    Tensor<float> qk_d({b, hq, qc, s}, GPU);
    launch_prefill_attention_scores(q_d, k_d, ql_d, kl_d, 150, 150, qk_d);
    std::vector<float> eqk(b * hq * qc * s, 0.f);
    orc_qk_scores(eq.data(), ek.data(), b, hq, hkv, qc, s, hd, 150, 150, eqk.data());
    std::vector<uint8_t> mask(b * qc * s, 0);
    orc_build_intended_mask(q_lens.data(), kv_lens.data(), b, 150, 150, qc, s, mask.data());
    orc_masked_attention_score(eqk.data(), mask.data(), q_lens.data(), b, hq, qc, s, 150, hd);
    const auto got = download(qk_d);
    for (unsigned int bi = 0; bi < b; ++bi)
        for (unsigned int h = 0; h < hq; ++h)
            for (unsigned int i = 0; i < q_lens[bi]; ++i)
                for (unsigned int j = 0; j < s; ++j)
                {
                    const size_t o = ((size_t)(bi * hq + h) * qc + i) * s + j;
                    const float d = std::fabs(got[o] - eqk[o]);
                    EXPECT_TRUE(d == 0.f || d <= 1e-5f * std::fabs(eqk[o]));
                }
}

TEST(BuildCausalMaskTest, CacheLargerThanActual)
{
    std::vector<unsigned int> q = {2, 3}, kv = {4, 5};
    Tensor<unsigned int> q_d({2}, GPU), kv_d({2}, GPU);
    upload(q_d, q);
    upload(kv_d, kv);
    Tensor<unsigned char> m_d({2, 4, 6}, GPU);
    launch_build_causal_mask(3, 5, q_d, kv_d, m_d);
    std::vector<uint8_t> e(2 * 4 * 6, 0);
    orc_build_causal_mask(q.data(), kv.data(), 2, 3, 5, 4, 6, e.data());
    EXPECT_TRUE(download(m_d) == e);
}

TEST(UpdateQKVLensTest, HostMaxima)
{
    std::vector<unsigned int> q = {2, 5, 3}, kv = {0, 0, 0};
    Tensor<unsigned int> q_d({3}, GPU), kv_d({3}, GPU), mq({1}, CPU), mkv({1}, CPU);
    upload(q_d, q);
    upload(kv_d, kv);
    launch_update_q_kv_lens(q_d, kv_d, mq, mkv);
    EXPECT_TRUE(mq.devtype() == CPU_PINNED && mq.data()[0] == 5 && mkv.data()[0] == 5);
    EXPECT_TRUE(download(kv_d) == std::vector<unsigned int>({2, 5, 3}));
}

TEST(BuildQKVArrayTest, GqaMultiBatch)
{
    const unsigned int b = 3, hq = 6, hkv = 2, qc = 4, s = 10, hs = 8;
    Tensor<float> q({b, hq, qc, hs}, GPU), qd({b, hq, 1, hs}, GPU), k({b, hkv, s, hs}, GPU), v({b, hkv, s, hs}, GPU),
        qk({b, hq, qc, s}, GPU), qkd({b, hq, 1, s}, GPU), qkv({b, hq, qc, hs}, GPU), qkvd({b, hq, 1, hs}, GPU);
    std::vector<Tensor<void *>> arr;
    for (int i = 0; i < 8; ++i)
        arr.emplace_back(std::vector<unsigned int>{b * hq}, GPU);
    launch_build_q_k_v_qk_qkv_array(q, qd, k, v, qk, qkd, qkv, qkvd, arr[0], arr[1], arr[2], arr[3], arr[4], arr[5],
                                    arr[6], arr[7]);
    const auto ka = download(arr[2]);
    const auto qa = download(arr[0]);
    for (unsigned int bi = 0; bi < b; ++bi)
        for (unsigned int h = 0; h < hq; ++h)
        {
            const unsigned int idx = bi * hq + h;
            EXPECT_TRUE(qa[idx] == static_cast<void *>(q.data() + (size_t)idx * qc * hs));
            EXPECT_TRUE(ka[idx] == static_cast<void *>(k.data() + (size_t)(bi * hkv + h / 3) * s * hs));
        }
}

TEST(LinearTest, BatchedTransB)
{
    const unsigned int bt = 2, m = 4, n = 5, kk = 6;
    std::vector<float> a(bt * m * kk), bm(bt * n * kk);
    for (size_t i = 0; i < a.size(); ++i)
        a[i] = static_cast<float>(static_cast<int>(i % 7) - 3);
    for (size_t i = 0; i < bm.size(); ++i)
        bm[i] = static_cast<float>(static_cast<int>(i % 5) - 2);
    Tensor<float> a_d({bt, m, kk}, GPU), b_d({bt, n, kk}, GPU), c_d({bt, m, n}, GPU);
    upload(a_d, a);
    upload(b_d, bm);
    Tensor<void *> aa({bt}, GPU), ba({bt}, GPU), ca({bt}, GPU);
    std::vector<void *> ap, bp, cp;
    for (unsigned int i = 0; i < bt; ++i)
    {
        ap.push_back(a_d.data() + i * m * kk);
        bp.push_back(b_d.data() + i * n * kk);
        cp.push_back(c_d.data() + i * m * n);
    }
    upload(aa, ap);
    upload(ba, bp);
    upload(ca, cp);
    cublasHandle_t handle = nullptr;
    launch_linear(handle, false, true, m, n, kk, a_d, b_d, c_d, aa, ba, ca);
    const auto c = download(c_d);
    for (unsigned int i = 0; i < bt; ++i)
    {
        std::vector<float> e(m * n);
        orc_linear(a.data() + i * m * kk, bm.data() + i * n * kk, 0, 1, m, n, kk, e.data());
        for (unsigned int j = 0; j < m * n; ++j)
            EXPECT_TRUE(c[i * m * n + j] == e[j]);
    }
}

TEST(ComputeMaskedAttentionScoreTest, BatchWithPadding)
{
    const unsigned int b = 3, h = 2, qc = 8, s = 8;
    std::vector<unsigned int> ql = {3, 6, 2};
    std::vector<uint8_t> mask(b * qc * s, 0);
    for (unsigned int bi = 0; bi < b; ++bi)
        for (unsigned int i = 0; i < ql[bi]; ++i)
            for (unsigned int j = 0; j < s; j += 2)
                mask[(bi * qc + i) * s + j] = 1;
    std::mt19937 gen(42);
    std::uniform_real_distribution<float> dist(-2.f, 2.f);
    std::vector<float> qk(b * h * qc * s);
    for (auto &v : qk)
        v = dist(gen);
    Tensor<unsigned int> ql_d({b}, GPU);
    Tensor<unsigned char> m_d({b, qc, s}, GPU);
    Tensor<float> qk_d({b, h, qc, s}, GPU);
    upload(ql_d, ql);
    upload(m_d, mask);
    upload(qk_d, qk);
    launch_compute_masked_attention_score<float, unsigned char>(32, 6, 8, ql_d, m_d, qk_d);
    orc_masked_attention_score(qk.data(), mask.data(), ql.data(), b, h, qc, s, 8, 32);
    EXPECT_TRUE(max_rel(download(qk_d), qk) <= 1e-5f);
}

TEST(SwiGLUTest, LargeBatchRandomValues)
{
    const unsigned int n = 64, f = 64;
    std::mt19937 gen(42);
    std::uniform_real_distribution<float> dist(-2.f, 2.f);
    std::vector<float> in(n * 2 * f), e(n * f);
    for (auto &v : in)
        v = dist(gen);
    orc_swiglu(in.data(), n, f, e.data());
    Tensor<float> in_d({n, 2 * f}, GPU), out_d({n, f}, GPU);
    upload(in_d, in);
    launch_swiglu(in_d, out_d);
    EXPECT_TRUE(max_rel(download(out_d), e) <= 1e-5f);
}

// The reference's BasicTwoSequences and HalfBasic cases
// (test/kernel/test_fused_transpose_unpad.cu:180-190, 233-241): the padded
// (B, H, Qc, hd) attention output back to (tokens, H * hd), byte-exact.
TEST(FusedTransposeUnpadTest, BasicTwoSequencesAndHalf)
{
    const unsigned int b = 3, h = 4, qc = 16, hd = 16;
    const std::vector<unsigned int> lens = {2, 5, 3};
    std::vector<unsigned int> idx(b * qc, 0u);
    unsigned int t = 0;
    for (unsigned int s = 0; s < b; ++s)
        for (unsigned int i = 0; i < lens[s]; ++i)
            idx[t++] = s * qc + i;
    Tensor<unsigned int> idx_d({b, qc}, GPU);
    upload(idx_d, idx);
    const std::vector<float> x = pattern(size_t(b) * h * qc * hd, 53, 0.1f, 1.0f);
    {
        Tensor<float> qkv({b, h, qc, hd}, GPU), out({t, h * hd}, GPU);
        upload(qkv, x);
        launch_fused_transpose_unpad(t, qkv, idx_d, out);
        std::vector<float> e(size_t(t) * h * hd);
        orc_transpose_unpad(x.data(), idx.data(), t, b, h, qc, hd, sizeof(float), e.data());
        EXPECT_TRUE(download(out) == e);
    }
    {
        std::vector<half> xh(x.size());
        for (size_t i = 0; i < x.size(); ++i)
            xh[i] = __float2half(x[i]);
        Tensor<half> qkv({b, h, qc, hd}, GPU), out({t, h * hd}, GPU);
        upload(qkv, xh);
        launch_fused_transpose_unpad(t, qkv, idx_d, out);
        std::vector<half> e(size_t(t) * h * hd);
        orc_transpose_unpad(xh.data(), idx.data(), t, b, h, qc, hd, sizeof(half), e.data());
        const std::vector<half> got = download(out);
        EXPECT_TRUE(std::memcmp(got.data(), e.data(), e.size() * sizeof(half)) == 0);
    }
}

TEST(DecodeAttentionScoresTest, Fp32)
{
    const unsigned int b = 3, h = 4, hd = 128, s = 1000;
    std::vector<unsigned int> kv = {1, 517, 1000};
    std::mt19937 gen(7);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<float> q(b * h * hd), k(b * h * s * hd);
    for (auto &v : q)
        v = nd(gen);
    for (auto &v : k)
        v = nd(gen);
    Tensor<float> q_d({b, h, 1, hd}, GPU), k_d({b, h, s, hd}, GPU), qk_d({b, h, 1, s}, GPU);
    Tensor<unsigned int> kv_d({b}, GPU), mkv({1}, GPU);
    upload(q_d, q);
    upload(k_d, k);
    upload(kv_d, kv);
    upload(mkv, std::vector<unsigned int>{1000});
    launch_decode_attention_scores(q_d, k_d, kv_d, mkv, qk_d);
    std::vector<float> e(b * h * s, 0.f);
    orc_qk_scores(q.data(), k.data(), b, h, h, 1, s, hd, 1, 1000, e.data());
    std::vector<uint8_t> mask(b * s, 0);
    std::vector<unsigned int> ones(b, 1);
    orc_build_intended_mask(ones.data(), kv.data(), b, 1, 1000, 1, s, mask.data());
    orc_masked_attention_score(e.data(), mask.data(), ones.data(), b, h, 1, s, 1000, hd);
    EXPECT_TRUE(max_rel(download(qk_d), e) <= 1e-5f);
}

// Decode attention: the scores and P.V through the fused operator, against
// the oracle composition (scores, then the P.V of the launch_linear site).
TEST(DecodeAttentionTest, Fp32ScoresAndOutput)
{
    const unsigned int b = 2, h = 4, hd = 128, s = 700;
    std::vector<unsigned int> kv = {700, 33};
    std::mt19937 gen(9);
    std::normal_distribution<float> nd(0.f, 1.f);
    std::vector<float> q(b * h * hd), k(b * h * s * hd), v(b * h * s * hd);
    for (auto *vec : {&q, &k, &v})
        for (auto &x : *vec)
            x = nd(gen);
    Tensor<float> q_d({b, h, 1, hd}, GPU), k_d({b, h, s, hd}, GPU), v_d({b, h, s, hd}, GPU), qk_d({b, h, 1, s}, GPU),
        o_d({b, h, 1, hd}, GPU);
    Tensor<unsigned int> kv_d({b}, GPU), mkv({1}, GPU);
    upload(q_d, q);
    upload(k_d, k);
    upload(v_d, v);
    upload(kv_d, kv);
    upload(mkv, std::vector<unsigned int>{700});
    launch_decode_attention(q_d, k_d, v_d, kv_d, mkv, qk_d, o_d);
    std::vector<float> e(b * h * s, 0.f), eo(b * h * hd, 0.f);
    orc_qk_scores(q.data(), k.data(), b, h, h, 1, s, hd, 1, 700, e.data());
    std::vector<uint8_t> mask(b * s, 0);
    std::vector<unsigned int> ones(b, 1);
    orc_build_intended_mask(ones.data(), kv.data(), b, 1, 700, 1, s, mask.data());
    orc_masked_attention_score(e.data(), mask.data(), ones.data(), b, h, 1, s, 700, hd);
    orc_attention_qkv(e.data(), v.data(), b, h, h, 1, s, hd, 1, 700, eo.data());
    EXPECT_TRUE(max_rel(download(qk_d), e) <= 1e-5f);
    // P.V elements may cancel towards 0: relative to each output row's largest magnitude
    const std::vector<float> got = download(o_d);
    for (unsigned int r = 0; r < b * h; ++r)
    {
        float mx = 0.f, err = 0.f;
        for (unsigned int d = 0; d < hd; ++d)
        {
            mx = std::fmax(mx, std::fabs(eo[r * hd + d]));
            err = std::fmax(err, std::fabs(got[r * hd + d] - eo[r * hd + d]));
        }
        EXPECT_TRUE(err <= 1e-5f * mx);
    }
}

TEST(DecodeStepTest, WholeChainOneLaunch)
{
    // The fused step against the oracle composition of the operators it replaces.
    const unsigned int b = 2, h = 4, hd = 128, s = 256, d = h * hd, f = 768, vocab = 1000;
    std::mt19937 gen(11);
    std::normal_distribution<float> nd(0.f, 1.f);
    auto rnd = [&](size_t n, float sc) {
        std::vector<float> v(n);
        for (auto &e : v)
            e = nd(gen) * sc;
        return v;
    };
    std::vector<float> table = rnd((size_t)vocab * d, 0.02f), w(d), qkv = rnd((size_t)b * 3 * d, 1.f),
                       gate_up = rnd((size_t)b * 2 * f, 1.f), kc = rnd((size_t)b * h * s * hd, 1.f),
                       vc = rnd((size_t)b * h * s * hd, 1.f);
    for (unsigned int i = 0; i < d; ++i)
        w[i] = 0.5f + (float)(i % 97) / 97.f;
    std::vector<unsigned int> ids = {7, 998}, ql = {1, 1}, kv = {100, 255};
    std::vector<unsigned char> done = {0, 0};
    Tensor<float> table_d({vocab, d}, GPU), w_d({d}, GPU), x_d({b, d}, GPU), n_d({b, d}, GPU), qkv_d({b, 3 * d}, GPU),
        q_d({b, h, 1, hd}, GPU), k_d({b, h, s, hd}, GPU), v_d({b, h, s, hd}, GPU), qk_d({b, h, 1, s}, GPU),
        gu_d({b, 2 * f}, GPU), ffn_d({b, f}, GPU);
    Tensor<unsigned int> ids_d({b}, GPU), ql_d({b}, GPU), kv_d({b}, GPU), ml_d({2}, GPU);
    Tensor<unsigned char> done_d({b}, GPU);
    upload(table_d, table);
    upload(w_d, w);
    upload(qkv_d, qkv);
    upload(gu_d, gate_up);
    upload(k_d, kc);
    upload(v_d, vc);
    upload(ids_d, ids);
    upload(ql_d, ql);
    upload(kv_d, kv);
    upload(done_d, done);
    launch_decode_step(ql_d, kv_d, ml_d, ids_d, table_d, w_d, x_d, n_d, qkv_d, done_d, q_d, k_d, v_d, qk_d, gu_d,
                       ffn_d, true);
    // expectations
    std::vector<unsigned int> kv_e = kv, mq(1), mkv(1);
    orc_update_q_kv_lens(ql.data(), kv_e.data(), b, mq.data(), mkv.data());
    std::vector<float> x_e((size_t)b * d), res((size_t)b * d, 0.f), n_e((size_t)b * d);
    orc_embedding(ids.data(), b, table.data(), d, 4, x_e.data());
    std::vector<float> xa((size_t)b * d);
    orc_fused_add_residual_rmsnorm(x_e.data(), res.data(), w.data(), b, d, 0, xa.data(), n_e.data());
    std::vector<float> q_e((size_t)b * h * hd, 0.f), k_e = kc, v_e = vc;
    orc_rope_kvcache_decode(1, qkv.data(), done.data(), kv_e.data(), b, h, h, hd, s, q_e.data(), k_e.data(),
                            v_e.data());
    std::vector<float> qk_e((size_t)b * h * s, 0.f);
    orc_qk_scores(q_e.data(), k_e.data(), b, h, h, 1, s, hd, 1, mkv[0], qk_e.data());
    std::vector<uint8_t> mask((size_t)b * s, 0);
    orc_build_intended_mask(ql.data(), kv_e.data(), b, 1, mkv[0], 1, s, mask.data());
    orc_masked_attention_score(qk_e.data(), mask.data(), ql.data(), b, h, 1, s, mkv[0], hd);
    std::vector<float> ffn_e((size_t)b * f);
    orc_swiglu(gate_up.data(), b, f, ffn_e.data());
    EXPECT_TRUE(download(kv_d) == kv_e);
    const std::vector<unsigned int> ml = download(ml_d);
    EXPECT_TRUE(ml[0] == mq[0] && ml[1] == mkv[0]);
    EXPECT_TRUE(download(x_d) == x_e);
    EXPECT_TRUE(max_rel(download(n_d), n_e) <= 1e-5f);
    EXPECT_TRUE(download(q_d) == q_e);
    EXPECT_TRUE(download(k_d) == k_e);
    EXPECT_TRUE(download(v_d) == v_e);
    EXPECT_TRUE(max_rel(download(qk_d), qk_e) <= 1e-5f);
    EXPECT_TRUE(max_rel(download(ffn_d), ffn_e) <= 1e-5f);
    // The same step with the attention output: a second run on fresh lengths
    // and caches, whose P.V is checked against the oracle's P.V of the
    // probabilities above over the appended V cache.
    upload(kv_d, kv);
    upload(k_d, kc);
    upload(v_d, vc);
    Tensor<float> o_d({b, h, 1, hd}, GPU);
    launch_decode_step_attention(ql_d, kv_d, ml_d, ids_d, table_d, w_d, x_d, n_d, qkv_d, done_d, q_d, k_d, v_d, qk_d,
                                 gu_d, ffn_d, o_d, true);
    EXPECT_TRUE(download(v_d) == v_e);
    EXPECT_TRUE(max_rel(download(qk_d), qk_e) <= 1e-5f);
    std::vector<float> o_e((size_t)b * h * hd, 0.f);
    orc_attention_qkv(qk_e.data(), v_e.data(), b, h, h, 1, s, hd, 1, mkv[0], o_e.data());
    const std::vector<float> o = download(o_d);
    for (unsigned int r = 0; r < b * h; ++r)
    {
        float mx = 0.f, err = 0.f;
        for (unsigned int e = 0; e < hd; ++e)
        {
            mx = std::fmax(mx, std::fabs(o_e[r * hd + e]));
            err = std::fmax(err, std::fabs(o[r * hd + e] - o_e[r * hd + e]));
        }
        EXPECT_TRUE(err <= 1e-5f * mx);
    }
}

int main()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
    {
        std::printf("no CUDA device\n");
        return 2;
    }
    for (auto &t : registry())
    {
        const int before = g_failures;
        t.second();
        std::printf("[%s] %s\n", g_failures == before ? "  OK  " : "FAILED", t.first.c_str());
    }
    std::printf("%zu tests, %d failed\n", registry().size(), g_failures);
    return g_failures ? 1 : 0;
}
