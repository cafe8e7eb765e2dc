// C++ operator API (the reference's include/kernel/*.h signatures) over the
// C ABI in include/llama2_b200.h.
//
// Each launch_* reads its shapes from the Tensor arguments the way the
// reference's host wrappers do, checks them (the reference's asserts), and
// enqueues the library kernel on the legacy default stream. Any failure
// prints the message and exits, which is what the reference's
// CUDA_KERNEL_LAUNCH_CHECK does (include/common/macro.h:32-40).
//
// RoPE angle tables are built once per (device, head_dim) on the host and
// kept on that device for the life of the process; they make the rotations
// match the reference's CPU oracle bit for bit.
#include <cstdio>
#include <cstdlib>
#include <map>
#include <mutex>
#include <vector>

#include "core/Tensor.cuh"
#include "kernel/attention_scores.h"
#include "kernel/build_causal_mask.h"
#include "kernel/build_padding_index_maps.h"
#include "kernel/build_q_k_v_qk_qkv_array.h"
#include "kernel/compute_masked_attention_score.h"
#include "kernel/embedding.h"
#include "kernel/fused_add_residual_rmsnorm.h"
#include "kernel/fused_pad_reshape_transpose_rope_kvcache.h"
#include "kernel/fused_pad_reshape_transpose_rope_kvcache_llama2.h"
#include "kernel/fused_reshape_rope_kvcache_decode.h"
#include "kernel/fused_reshape_rope_kvcache_llama2_decode.h"
#include "kernel/fused_transpose_unpad.h"
#include "kernel/linear.h"
#include "kernel/swiglu.h"
#include "kernel/update_q_kv_lens.h"
#include "llama2_b200.h"

namespace
{

constexpr int64_t kRopePositions = 4096;

template <typename T>
constexpr int dtype_of();
template <>
constexpr int dtype_of<float>() { return L2K_F32; }
template <>
constexpr int dtype_of<half>() { return L2K_F16; }
template <>
constexpr int dtype_of<__nv_bfloat16>() { return L2K_BF16; }

void check(int status, const char *what)
{
    if (status != L2K_OK)
    {
        std::fprintf(stderr, "%s failed: %s: %s\n", what, l2k_status_string(status), l2k_last_error_message());
        std::exit(EXIT_FAILURE);
    }
}

void require(bool cond, const char *msg)
{
    if (!cond)
    {
        std::fprintf(stderr, "%s\n", msg);
        std::exit(EXIT_FAILURE);
    }
}

const float *rope_table(int64_t head_dim)
{
    static std::mutex mu;
    static std::map<std::pair<int, int64_t>, float *> tables;
    int dev = 0;
    CUDA_CHECK(cudaGetDevice(&dev));
    std::lock_guard<std::mutex> lock(mu);
    auto key = std::make_pair(dev, head_dim);
    auto it = tables.find(key);
    if (it != tables.end())
        return it->second;
    const int64_t n = l2k_rope_table_floats(head_dim, kRopePositions);
    require(n > 0, "rope table: bad head_dim");
    std::vector<float> host((size_t)n);
    check(l2k_rope_table_fill(host.data(), head_dim, kRopePositions), "l2k_rope_table_fill");
    float *d = nullptr;
    CUDA_CHECK(cudaMalloc((void **)&d, (size_t)n * sizeof(float)));
    CUDA_CHECK(cudaMemcpy(d, host.data(), (size_t)n * sizeof(float), cudaMemcpyHostToDevice));
    tables[key] = d;
    return d;
}

} // namespace

template <typename T>
void launch_embedding(const Tensor<unsigned int> &input_ids, const Tensor<T> &embed_table, Tensor<T> &output)
{
    require(embed_table.ndim() == 2 && output.ndim() == 2, "launch_embedding: tables must be 2-D");
    require(output.shape()[0] == input_ids.shape()[0] && output.shape()[1] == embed_table.shape()[1],
            "launch_embedding: Incorrect output size");
    check(l2k_embedding(input_ids.data(), input_ids.shape()[0], embed_table.data(), embed_table.shape()[0],
                        embed_table.shape()[1], output.data(), dtype_of<T>(), nullptr),
          "launch_embedding");
}

template <typename T, bool add_residual>
void launch_fused_add_residual_rmsnorm(const Tensor<T> &weights, Tensor<T> &x, Tensor<T> &residual)
{
    const unsigned int n = x.shape()[0], d = x.shape()[1];
    require(residual.shape()[0] == n && residual.shape()[1] == d, "Incorrect residual size");
    require(weights.shape()[0] == d, "Incorrect rmsnorm weight size");
    check(l2k_fused_add_residual_rmsnorm(weights.data(), x.data(), residual.data(), n, d, add_residual ? 1 : 0,
                                         dtype_of<T>(), nullptr),
          "launch_fused_add_residual_rmsnorm");
}

namespace
{
template <typename T, int PAIRING>
void rope_decode(const Tensor<T> &input, const Tensor<unsigned char> &is_done, const Tensor<unsigned int> &kv_lens,
                 Tensor<T> &q, Tensor<T> &k, Tensor<T> &v, const char *name)
{
    const unsigned int b = input.shape()[0], hd = q.shape()[3], hq = q.shape()[1], hkv = k.shape()[1];
    require(hd % 2 == 0, "Head dim should be even");
    require(k.shape()[3] == hd && v.shape()[3] == hd, "Head dim of q k v do not match");
    require(v.shape()[1] == hkv, "Head num of k v do not match");
    require(input.shape()[1] == (hq + 2 * hkv) * hd, "Incorrect embedding dim");
    require(is_done.shape()[0] == b && kv_lens.shape()[0] == b, "Incorrect batch size");
    require(q.shape()[0] == b && k.shape()[0] == b && v.shape()[0] == b, "Batch size of q k v do not match");
    require(q.shape()[2] == 1, "Incorrect q cache length");
    require(k.shape()[2] == v.shape()[2], "k v cache length do not match");
    auto fn = PAIRING == L2K_ROPE_HALF ? l2k_fused_reshape_rope_kvcache_llama2_decode
                                       : l2k_fused_reshape_rope_kvcache_decode;
    check(fn(input.data(), is_done.data(), kv_lens.data(), q.data(), k.data(), v.data(), b, hq, hkv, hd,
             k.shape()[2], rope_table(hd), kRopePositions, dtype_of<T>(), nullptr),
          name);
}

template <typename T, int PAIRING>
void rope_prefill(const Tensor<T> &input, const Tensor<unsigned int> &q_lens, const Tensor<unsigned int> &kv_lens,
                  const Tensor<unsigned int> &unpad, Tensor<T> &q, Tensor<T> &k, Tensor<T> &v, const char *name)
{
    const unsigned int n = input.shape()[0], b = q.shape()[0], hq = q.shape()[1], hd = q.shape()[3],
                       hkv = k.shape()[1];
    require(hd % 2 == 0, "Head dim should be even");
    require(k.shape()[3] == hd && v.shape()[3] == hd, "Head dim of q k v do not match");
    require(v.shape()[1] == hkv, "Head num of k v do not match");
    require(input.shape()[1] == (hq + 2 * hkv) * hd, "Incorrect embedding dim");
    require(q_lens.shape()[0] == b && kv_lens.shape()[0] == b, "Incorrect batch size of sequence length");
    require(k.shape()[0] == b && v.shape()[0] == b, "Batch size of k v do not match");
    require(k.shape()[2] == v.shape()[2], "k v cache length do not match");
    require(unpad.numel() >= n, "unpad_to_pad_idx too small");
    auto fn = PAIRING == L2K_ROPE_HALF ? l2k_fused_pad_reshape_transpose_rope_kvcache_llama2
                                       : l2k_fused_pad_reshape_transpose_rope_kvcache;
    check(fn(input.data(), q_lens.data(), kv_lens.data(), unpad.data(), q.data(), k.data(), v.data(), n, b, hq, hkv,
             hd, q.shape()[2], k.shape()[2], rope_table(hd), kRopePositions, dtype_of<T>(), nullptr),
          name);
}
} // namespace

template <typename T>
void launch_fused_reshape_rope_kvcache_decode(const Tensor<T> &input, const Tensor<unsigned char> &is_done,
                                              const Tensor<unsigned int> &kv_lens, Tensor<T> &q, Tensor<T> &k,
                                              Tensor<T> &v)
{
    rope_decode<T, L2K_ROPE_INTERLEAVED>(input, is_done, kv_lens, q, k, v, "launch_fused_reshape_rope_kvcache_decode");
}

template <typename T>
void launch_fused_reshape_rope_kvcache_llama2_decode(const Tensor<T> &input, const Tensor<unsigned char> &is_done,
                                                     const Tensor<unsigned int> &kv_lens, Tensor<T> &q, Tensor<T> &k,
                                                     Tensor<T> &v)
{
    rope_decode<T, L2K_ROPE_HALF>(input, is_done, kv_lens, q, k, v, "launch_fused_reshape_rope_kvcache_llama2_decode");
}

template <typename T>
void launch_fused_pad_reshape_transpose_rope_kvcache(const Tensor<T> &input, const Tensor<unsigned int> &q_lens,
                                                     const Tensor<unsigned int> &kv_lens,
                                                     const Tensor<unsigned int> &unpad_to_pad_idx, Tensor<T> &q,
                                                     Tensor<T> &k, Tensor<T> &v)
{
    rope_prefill<T, L2K_ROPE_INTERLEAVED>(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v,
                                          "launch_fused_pad_reshape_transpose_rope_kvcache");
}

template <typename T>
void launch_fused_pad_reshape_transpose_rope_kvcache_llama2(const Tensor<T> &input,
                                                            const Tensor<unsigned int> &q_lens,
                                                            const Tensor<unsigned int> &kv_lens,
                                                            const Tensor<unsigned int> &unpad_to_pad_idx,
                                                            Tensor<T> &q, Tensor<T> &k, Tensor<T> &v)
{
    rope_prefill<T, L2K_ROPE_HALF>(input, q_lens, kv_lens, unpad_to_pad_idx, q, k, v,
                                   "launch_fused_pad_reshape_transpose_rope_kvcache_llama2");
}

void launch_update_q_kv_lens(const Tensor<unsigned int> &q_lens, Tensor<unsigned int> &kv_lens,
                             Tensor<unsigned int> &max_q_len, Tensor<unsigned int> &max_kv_len)
{
    const unsigned int b = q_lens.shape()[0];
    require(kv_lens.shape()[0] == b, "Incorrect kv_lens size");
    if (max_q_len.devtype() == GPU && max_kv_len.devtype() == GPU)
    {
        check(l2k_update_q_kv_lens(q_lens.data(), kv_lens.data(), b, max_q_len.data(), max_kv_len.data(), nullptr),
              "launch_update_q_kv_lens");
        return;
    }
    // Host results, as the reference: move to the device, run, move to pinned host.
    max_q_len.to_device();
    max_kv_len.to_device();
    check(l2k_update_q_kv_lens(q_lens.data(), kv_lens.data(), b, max_q_len.data(), max_kv_len.data(), nullptr),
          "launch_update_q_kv_lens");
    max_q_len.to_host_pinned();
    max_kv_len.to_host_pinned();
}

template <typename T>
void launch_build_causal_mask(const unsigned int max_q_len, const unsigned int max_kv_len,
                              const Tensor<unsigned int> &q_lens, const Tensor<unsigned int> &kv_lens, Tensor<T> &mask)
{
    static_assert(sizeof(T) == 1, "mask elements are bytes");
    check(l2k_build_causal_mask(max_q_len, max_kv_len, q_lens.data(), kv_lens.data(),
                                reinterpret_cast<uint8_t *>(mask.data()), mask.shape()[0], mask.shape()[1],
                                mask.shape()[2], nullptr),
          "launch_build_causal_mask");
}

void launch_build_padding_index_maps(const unsigned int num_input_tokens, const Tensor<unsigned int> &seq_lens,
                                     Tensor<unsigned int> &unpad_to_pad_idx, Tensor<unsigned int> &seq_offsets)
{
    const int64_t qc = unpad_to_pad_idx.ndim() >= 2 ? unpad_to_pad_idx.shape()[1] : unpad_to_pad_idx.shape()[0];
    check(l2k_build_padding_index_maps(num_input_tokens, seq_lens.data(), seq_lens.shape()[0], qc,
                                       unpad_to_pad_idx.data(), seq_offsets.data(), nullptr),
          "launch_build_padding_index_maps");
}

template <typename T>
void launch_build_q_k_v_qk_qkv_array(Tensor<T> &q, Tensor<T> &q_decode, Tensor<T> &k, Tensor<T> &v, Tensor<T> &qk,
                                     Tensor<T> &qk_decode, Tensor<T> &qkv, Tensor<T> &qkv_decode,
                                     Tensor<void *> &q_array, Tensor<void *> &q_decode_array,
                                     Tensor<void *> &k_array, Tensor<void *> &v_array, Tensor<void *> &qk_array,
                                     Tensor<void *> &qk_decode_array, Tensor<void *> &qkv_array,
                                     Tensor<void *> &qkv_decode_array)
{
    Tensor<T> *ts[8] = {&q, &q_decode, &k, &v, &qk, &qk_decode, &qkv, &qkv_decode};
    Tensor<void *> *as[8] = {&q_array, &q_decode_array, &k_array, &v_array,
                             &qk_array, &qk_decode_array, &qkv_array, &qkv_decode_array};
    const unsigned int b = q.shape()[0], hq = q.shape()[1], hkv = k.shape()[1];
    require(hkv > 0 && hq % hkv == 0, "q_head_num is not divisible by kv_head_num");
    void *bases[8];
    int64_t slices[8];
    void **outs[8];
    for (int i = 0; i < 8; ++i)
    {
        require(as[i]->numel() == (uint64_t)b * hq, "Incorrect pointer array size");
        bases[i] = ts[i]->data();
        slices[i] = (int64_t)ts[i]->shape()[2] * ts[i]->shape()[3];
        outs[i] = as[i]->data();
    }
    check(l2k_build_q_k_v_qk_qkv_array(bases, slices, sizeof(T), b, hq, hkv, outs, nullptr),
          "launch_build_q_k_v_qk_qkv_array");
}

template <typename T>
void launch_linear(cublasHandle_t &, const bool trans_A, const bool trans_B, const unsigned int M,
                   const unsigned int N, const unsigned int K, const Tensor<T> &A, const Tensor<T> &B, Tensor<T> &C,
                   const Tensor<void *> &A_array, const Tensor<void *> &B_array, Tensor<void *> &C_array)
{
    const unsigned int dim = C.ndim();
    require(dim >= 2 && A.ndim() == dim && B.ndim() == dim, "Matrix dim do not match");
    const int64_t lda = A.shape()[dim - 1], ldb = B.shape()[dim - 1], ldc = C.shape()[dim - 1];
    if (dim > 2)
    {
        uint64_t batch = 1;
        for (unsigned int i = 0; i + 2 < dim; ++i)
            batch *= C.shape()[i];
        require(A_array.numel() == batch && B_array.numel() == batch && C_array.numel() == batch,
                "Illegal pointer array size");
        check(l2k_linear(trans_A, trans_B, M, N, K, nullptr, lda, nullptr, ldb, nullptr, ldc, (int64_t)batch,
                         A_array.data(), B_array.data(), C_array.data(), dtype_of<T>(), nullptr),
              "launch_linear");
    }
    else
        check(l2k_linear(trans_A, trans_B, M, N, K, A.data(), lda, B.data(), ldb, C.data(), ldc, 0, nullptr, nullptr,
                         nullptr, dtype_of<T>(), nullptr),
              "launch_linear");
}

template <typename T, typename MASK_T>
void launch_compute_masked_attention_score(const unsigned int head_dim, const unsigned int max_q_len,
                                           const unsigned int max_kv_len, const Tensor<unsigned int> &q_lens,
                                           const Tensor<MASK_T> &mask, Tensor<T> &qk)
{
    static_assert(sizeof(MASK_T) == 1, "mask elements are bytes");
    const unsigned int b = qk.shape()[0], hq = qk.shape()[1], qc = qk.shape()[2], s = qk.shape()[3];
    require(q_lens.shape()[0] == b, "Incorrect q_lens size");
    require(mask.shape()[0] == b && mask.shape()[1] == qc && mask.shape()[2] == s, "Incorrect mask size");
    require(max_q_len <= qc && max_kv_len <= s, "Incorrect max_q_len / max_kv_len");
    check(l2k_compute_masked_attention_score(head_dim, max_q_len, max_kv_len, q_lens.data(),
                                             reinterpret_cast<const uint8_t *>(mask.data()), qk.data(), b, hq, qc, s,
                                             dtype_of<T>(), nullptr),
          "launch_compute_masked_attention_score");
}

template <typename T>
void launch_swiglu(const Tensor<T> &input, Tensor<T> &output)
{
    const unsigned int n = output.shape()[0], f = output.shape()[1];
    require(input.shape()[0] == n && input.shape()[1] == 2 * f, "Incorrect input size");
    check(l2k_swiglu(input.data(), output.data(), n, f, dtype_of<T>(), nullptr), "launch_swiglu");
}

template <typename T>
void launch_fused_transpose_unpad(const unsigned int num_input_tokens, const Tensor<T> &qkv,
                                  const Tensor<unsigned int> &unpad_to_pad_idx, Tensor<T> &unpad_qkv)
{
    const unsigned int b = qkv.shape()[0], h = qkv.shape()[1], qc = qkv.shape()[2], hd = qkv.shape()[3];
    require(unpad_qkv.shape()[1] == h * hd, "Incorrect embed dim");
    require(unpad_qkv.shape()[0] >= num_input_tokens && unpad_to_pad_idx.numel() >= num_input_tokens,
            "Incorrect number of input tokens");
    check(l2k_fused_transpose_unpad(num_input_tokens, qkv.data(), unpad_to_pad_idx.data(), unpad_qkv.data(), b, h, qc,
                                    hd, dtype_of<T>(), nullptr),
          "launch_fused_transpose_unpad");
}

template <typename T>
void launch_decode_attention_scores(const Tensor<T> &q, const Tensor<T> &k, const Tensor<unsigned int> &kv_lens,
                                    const Tensor<unsigned int> &max_kv_len, Tensor<T> &qk)
{
    require(max_kv_len.devtype() == GPU, "max_kv_len must be a device tensor");
    check(l2k_decode_attention_scores(q.data(), k.data(), kv_lens.data(), max_kv_len.data(), qk.data(), q.shape()[0],
                                      q.shape()[1], k.shape()[1], k.shape()[2], q.shape()[3], dtype_of<T>(), nullptr),
          "launch_decode_attention_scores");
}

template <typename T>
void launch_decode_attention(const Tensor<T> &q, const Tensor<T> &k, const Tensor<T> &v,
                             const Tensor<unsigned int> &kv_lens, const Tensor<unsigned int> &max_kv_len, Tensor<T> &qk,
                             Tensor<T> &qkv)
{
    require(max_kv_len.devtype() == GPU, "max_kv_len must be a device tensor");
    require(v.shape() == k.shape(), "Incorrect v size");
    check(l2k_decode_attention(q.data(), k.data(), v.data(), kv_lens.data(), max_kv_len.data(), qk.data(), qkv.data(),
                               q.shape()[0], q.shape()[1], k.shape()[1], k.shape()[2], q.shape()[3], dtype_of<T>(),
                               nullptr),
          "launch_decode_attention");
}

template <typename T>
void launch_attention_qkv(const Tensor<T> &qk, const Tensor<T> &v, Tensor<T> &qkv, const unsigned int M,
                          const unsigned int N)
{
    check(l2k_attention_qkv(qk.data(), v.data(), qkv.data(), qk.shape()[0], qk.shape()[1], v.shape()[1], qk.shape()[2],
                            qk.shape()[3], v.shape()[3], M, N, dtype_of<T>(), nullptr),
          "launch_attention_qkv");
}

template <typename T>
void launch_prefill_attention_scores(const Tensor<T> &q, const Tensor<T> &k, const Tensor<unsigned int> &q_lens,
                                     const Tensor<unsigned int> &kv_lens, const unsigned int max_q_len,
                                     const unsigned int max_kv_len, Tensor<T> &qk)
{
    check(l2k_prefill_attention_scores(q.data(), k.data(), q_lens.data(), kv_lens.data(), max_q_len, max_kv_len,
                                       qk.data(), q.shape()[0], q.shape()[1], k.shape()[1], q.shape()[2], k.shape()[2],
                                       q.shape()[3], dtype_of<T>(), nullptr),
          "launch_prefill_attention_scores");
}

// The arguments of one fused decode step, read from the tensors as the
// separate launch_* functions read theirs.
template <typename T>
l2k_decode_step_args step_args(const Tensor<unsigned int> &q_lens, Tensor<unsigned int> &kv_lens,
                               Tensor<unsigned int> &max_lens, const Tensor<unsigned int> &input_ids,
                               const Tensor<T> &embed_table, const Tensor<T> &norm_weight, Tensor<T> &x,
                               Tensor<T> &normed, const Tensor<T> &qkv, const Tensor<unsigned char> &is_done,
                               Tensor<T> &q, Tensor<T> &k_cache, Tensor<T> &v_cache, Tensor<T> &qk,
                               const Tensor<T> &gate_up, Tensor<T> &ffn_out, bool llama2_pairs)
{
    const unsigned int b = input_ids.shape()[0];
    const unsigned int hq = q.shape()[1], hd = q.shape()[3], hkv = k_cache.shape()[1], s = k_cache.shape()[2];
    require(q.shape()[0] == b && q.shape()[2] == 1, "Incorrect q size");
    require(qk.shape()[0] == b && qk.shape()[1] == hq && qk.shape()[3] == s, "Incorrect qk size");
    require(max_lens.numel() >= 2, "max_lens needs two elements");
    l2k_decode_step_args a = {};
    a.q_lens = q_lens.data();
    a.kv_lens = kv_lens.data();
    a.max_lens = max_lens.data();
    a.input_ids = input_ids.data();
    a.embed_table = embed_table.data();
    a.norm_weight = norm_weight.data();
    a.x = x.data();
    a.normed = normed.data();
    a.qkv = qkv.data();
    a.is_done = is_done.data();
    a.q = q.data();
    a.k_cache = k_cache.data();
    a.v_cache = v_cache.data();
    a.qk = qk.data();
    a.rope_table = rope_table(hd);
    a.rope_table_positions = kRopePositions;
    a.gate_up = gate_up.data();
    a.ffn_out = ffn_out.data();
    a.batch = b;
    a.vocab_size = embed_table.shape()[0];
    a.dim = embed_table.shape()[1];
    a.q_head_num = hq;
    a.kv_head_num = hkv;
    a.head_dim = hd;
    a.kv_cache_len = s;
    a.hidden = ffn_out.shape()[1];
    a.pairing = llama2_pairs ? L2K_ROPE_HALF : L2K_ROPE_INTERLEAVED;
    a.dtype = dtype_of<T>();
    return a;
}

template <typename T>
void launch_decode_step(const Tensor<unsigned int> &q_lens, Tensor<unsigned int> &kv_lens,
                        Tensor<unsigned int> &max_lens, const Tensor<unsigned int> &input_ids,
                        const Tensor<T> &embed_table, const Tensor<T> &norm_weight, Tensor<T> &x, Tensor<T> &normed,
                        const Tensor<T> &qkv, const Tensor<unsigned char> &is_done, Tensor<T> &q, Tensor<T> &k_cache,
                        Tensor<T> &v_cache, Tensor<T> &qk, const Tensor<T> &gate_up, Tensor<T> &ffn_out,
                        bool llama2_pairs)
{
    const l2k_decode_step_args a = step_args<T>(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x,
                                                normed, qkv, is_done, q, k_cache, v_cache, qk, gate_up, ffn_out,
                                                llama2_pairs);
    check(l2k_decode_step_no_alloc(&a, nullptr), "launch_decode_step");
}

template <typename T>
void launch_decode_step_attention(const Tensor<unsigned int> &q_lens, Tensor<unsigned int> &kv_lens,
                                  Tensor<unsigned int> &max_lens, const Tensor<unsigned int> &input_ids,
                                  const Tensor<T> &embed_table, const Tensor<T> &norm_weight, Tensor<T> &x,
                                  Tensor<T> &normed, const Tensor<T> &qkv, const Tensor<unsigned char> &is_done,
                                  Tensor<T> &q, Tensor<T> &k_cache, Tensor<T> &v_cache, Tensor<T> &qk,
                                  const Tensor<T> &gate_up, Tensor<T> &ffn_out, Tensor<T> &attn_out,
                                  bool llama2_pairs)
{
    require(attn_out.numel() == q.numel(), "Incorrect attn_out size");
    const l2k_decode_step_args a = step_args<T>(q_lens, kv_lens, max_lens, input_ids, embed_table, norm_weight, x,
                                                normed, qkv, is_done, q, k_cache, v_cache, qk, gate_up, ffn_out,
                                                llama2_pairs);
    check(l2k_decode_step_attention_no_alloc(&a, attn_out.data(), nullptr), "launch_decode_step_attention");
}

// Explicit instantiations: float, half and bfloat16, as the reference
// instantiates float and half (e.g. src/kernel/embedding.cu:51-56).
#define L2K_INSTANTIATE(T)                                                                                          \
    template void launch_embedding<T>(const Tensor<unsigned int> &, const Tensor<T> &, Tensor<T> &);                \
    template void launch_fused_add_residual_rmsnorm<T, false>(const Tensor<T> &, Tensor<T> &, Tensor<T> &);         \
    template void launch_fused_add_residual_rmsnorm<T, true>(const Tensor<T> &, Tensor<T> &, Tensor<T> &);          \
    template void launch_fused_reshape_rope_kvcache_decode<T>(const Tensor<T> &, const Tensor<unsigned char> &,     \
                                                              const Tensor<unsigned int> &, Tensor<T> &,            \
                                                              Tensor<T> &, Tensor<T> &);                            \
    template void launch_fused_reshape_rope_kvcache_llama2_decode<T>(                                               \
        const Tensor<T> &, const Tensor<unsigned char> &, const Tensor<unsigned int> &, Tensor<T> &, Tensor<T> &,   \
        Tensor<T> &);                                                                                               \
    template void launch_fused_pad_reshape_transpose_rope_kvcache<T>(                                               \
        const Tensor<T> &, const Tensor<unsigned int> &, const Tensor<unsigned int> &,                              \
        const Tensor<unsigned int> &, Tensor<T> &, Tensor<T> &, Tensor<T> &);                                       \
    template void launch_fused_pad_reshape_transpose_rope_kvcache_llama2<T>(                                        \
        const Tensor<T> &, const Tensor<unsigned int> &, const Tensor<unsigned int> &,                              \
        const Tensor<unsigned int> &, Tensor<T> &, Tensor<T> &, Tensor<T> &);                                       \
    template void launch_build_q_k_v_qk_qkv_array<T>(                                                               \
        Tensor<T> &, Tensor<T> &, Tensor<T> &, Tensor<T> &, Tensor<T> &, Tensor<T> &, Tensor<T> &, Tensor<T> &,     \
        Tensor<void *> &, Tensor<void *> &, Tensor<void *> &, Tensor<void *> &, Tensor<void *> &,                   \
        Tensor<void *> &, Tensor<void *> &, Tensor<void *> &);                                                      \
    template void launch_linear<T>(cublasHandle_t &, const bool, const bool, const unsigned int,                    \
                                   const unsigned int, const unsigned int, const Tensor<T> &, const Tensor<T> &,    \
                                   Tensor<T> &, const Tensor<void *> &, const Tensor<void *> &, Tensor<void *> &);  \
    template void launch_compute_masked_attention_score<T, unsigned char>(                                          \
        const unsigned int, const unsigned int, const unsigned int, const Tensor<unsigned int> &,                   \
        const Tensor<unsigned char> &, Tensor<T> &);                                                                \
    template void launch_swiglu<T>(const Tensor<T> &, Tensor<T> &);                                                 \
    template void launch_fused_transpose_unpad<T>(const unsigned int, const Tensor<T> &,                            \
                                                  const Tensor<unsigned int> &, Tensor<T> &);                       \
    template void launch_decode_attention_scores<T>(const Tensor<T> &, const Tensor<T> &,                           \
                                                    const Tensor<unsigned int> &, const Tensor<unsigned int> &,     \
                                                    Tensor<T> &);                                                   \
    template void launch_decode_attention<T>(const Tensor<T> &, const Tensor<T> &, const Tensor<T> &,               \
                                             const Tensor<unsigned int> &, const Tensor<unsigned int> &, Tensor<T> &, \
                                             Tensor<T> &);                                                          \
    template void launch_attention_qkv<T>(const Tensor<T> &, const Tensor<T> &, Tensor<T> &, const unsigned int,    \
                                          const unsigned int);                                                      \
    template void launch_prefill_attention_scores<T>(const Tensor<T> &, const Tensor<T> &,                          \
                                                     const Tensor<unsigned int> &, const Tensor<unsigned int> &,    \
                                                     const unsigned int, const unsigned int, Tensor<T> &);          \
    template void launch_decode_step_attention<T>(                                                                  \
        const Tensor<unsigned int> &, Tensor<unsigned int> &, Tensor<unsigned int> &, const Tensor<unsigned int> &, \
        const Tensor<T> &, const Tensor<T> &, Tensor<T> &, Tensor<T> &, const Tensor<T> &,                          \
        const Tensor<unsigned char> &, Tensor<T> &, Tensor<T> &, Tensor<T> &, Tensor<T> &, const Tensor<T> &,       \
        Tensor<T> &, Tensor<T> &, bool);                                                                            \
    template void launch_decode_step<T>(const Tensor<unsigned int> &, Tensor<unsigned int> &,                       \
                                        Tensor<unsigned int> &, const Tensor<unsigned int> &, const Tensor<T> &,    \
                                        const Tensor<T> &, Tensor<T> &, Tensor<T> &, const Tensor<T> &,             \
                                        const Tensor<unsigned char> &, Tensor<T> &, Tensor<T> &, Tensor<T> &,       \
                                        Tensor<T> &, const Tensor<T> &, Tensor<T> &, bool);

L2K_INSTANTIATE(float)
L2K_INSTANTIATE(half)
L2K_INSTANTIATE(__nv_bfloat16)

template void launch_build_causal_mask<unsigned char>(const unsigned int, const unsigned int,
                                                      const Tensor<unsigned int> &, const Tensor<unsigned int> &,
                                                      Tensor<unsigned char> &);
