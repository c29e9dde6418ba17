// ref_attn_harness.cpp — runs the reference's OWN attention block.
//
// TEST INFRASTRUCTURE ONLY (the checker; never the product path).
//
// LEAP keeps its attention inline in the private run_layer() of each engine
// and its RoPE table in a private constructor helper.  oracle/Makefile cuts
// those exact line ranges out of the reference sources at build time into
// oracle/_ref/ (never committed) and checks their first/last lines:
//   fp32 block   src/inference/FloatTransformer.cpp:404-662
//   fp32 softmax src/inference/FloatTransformer.cpp:216-238
//   RoPE table   src/inference/FloatTransformer.cpp:56-72  (theta 500000,
//                and a copy with the literal set to 10000 for TinyLlama)
//   W8A8 block   src/inference/QuantizedTransformer.cpp:680-923
//   W8A8 softmax src/inference/QuantizedTransformer.cpp:314-336
// and the support ops around the block, for kernel-level parity:
//   fp32 rmsnorm    src/inference/FloatTransformer.cpp:79-214
//   fp32 matmul     src/inference/FloatTransformer.cpp:240-382
//   W8A8 dequantize src/inference/QuantizedTransformer.cpp:136-216
//   W8A8 quantize   src/inference/QuantizedTransformer.cpp:338-357
//   W8A8 matmul     src/inference/QuantizedTransformer.cpp:359-652
// This file compiles them, with the reference's release flags, inside a
// scope that supplies what run_layer() would have in scope (p, s,
// k / k_cache_ptr, loff, kv_dim, kv_mul, head_size, pos, rope_cos,
// rope_sin).  The run-state members are thin views over caller memory, so a
// call does not copy the cache.
#include <algorithm>
#include <cmath>
#include <cstddef>
#include <cstring>
#include <immintrin.h>
#include <vector>

#include "Config.h"  // reference src/inference/Config.h

namespace leapref {

template <typename T> struct View {
    T *p = nullptr;
    T *data() const { return p; }
    T &operator[](std::size_t i) const { return p[i]; }
};

struct RunStateView {
    View<float> q, att, key_cache, value_cache, xb;
};

struct FloatTransformer {
    Inference::Config config{};
    std::vector<float> rope_cos, rope_sin;
    void precompute_freqs();
    static void softmax(float *x, int size);
    static void rmsnorm(float *o, const float *x, const float *weight, int size);
    static void matmul(float *xout, const float *x, const float *w, int n, int d);
};
#include "fp32_softmax.inc"
#include "fp32_rope.inc"
#include "fp32_rmsnorm.inc"
#include "fp32_matmul.inc"

struct QuantizedTensor {
    int8_t *q;
    float *s;
};

struct QuantizedTransformer {
    int group_size = 64;
    static void softmax(float *x, int size);
    void dequantize(const QuantizedTensor *qx, float *x, int n) const;
    void quantize(const QuantizedTensor *qx, const float *x, int n) const;
    void matmul(float *xout, const QuantizedTensor *x, const QuantizedTensor *w, int n,
                int d) const;
};
#include "w8a8_softmax.inc"
#include "w8a8_dequantize.inc"
#include "w8a8_quantize.inc"
#include "w8a8_matmul.inc"

struct Fp32Block : FloatTransformer {
    static void run(const Inference::Config *p, RunStateView *s, float *k,
                    int loff, int kv_dim, int kv_mul, int head_size, int pos,
                    const float *rope_cos, const float *rope_sin) {
#include "fp32_block.inc"
    }
};

struct W8A8Block : QuantizedTransformer {
    static void run(const Inference::Config *p, RunStateView *s,
                    float *k_cache_ptr, int loff, int kv_dim, int kv_mul,
                    int head_size, int pos, const float *rope_cos,
                    const float *rope_sin) {
#include "w8a8_block.inc"
    }
};

}  // namespace leapref

namespace leapref10k {
struct FloatTransformer {
    Inference::Config config{};
    std::vector<float> rope_cos, rope_sin;
    void precompute_freqs();
};
#include "fp32_rope_theta10k.inc"
}  // namespace leapref10k

// One layer's attention as the reference computes it.  The caller has put
// the new un-rotated k/v in row `pos` of k_cache/v_cache ([seq_len][kv_dim]);
// q [n_heads*head_size] and that k row are rotated in place; xb receives the
// output; att is scratch [n_heads*seq_len].  which = 0 fp32 block, 1 W8A8.
extern "C" void leapref_attn_block(int which, int n_heads, int n_kv_heads,
                                   int head_size, int seq_len, int pos,
                                   const float *rope_cos, const float *rope_sin,
                                   float *q, float *k_cache, float *v_cache,
                                   float *att, float *xb) {
    Inference::Config cfg{};
    cfg.dim = n_heads * head_size;
    cfg.n_heads = n_heads;
    cfg.n_kv_heads = n_kv_heads;
    cfg.seq_len = seq_len;
    cfg.n_layers = 1;
    leapref::RunStateView s;
    s.q.p = q;
    s.att.p = att;
    s.key_cache.p = k_cache;
    s.value_cache.p = v_cache;
    s.xb.p = xb;
    const int kv_dim = n_kv_heads * head_size;
    const int kv_mul = n_heads / n_kv_heads;
    float *krow = k_cache + static_cast<std::size_t>(pos) * kv_dim;
    if (which == 0)
        leapref::Fp32Block::run(&cfg, &s, krow, 0, kv_dim, kv_mul, head_size,
                                pos, rope_cos, rope_sin);
    else
        leapref::W8A8Block::run(&cfg, &s, krow, 0, kv_dim, kv_mul, head_size,
                                pos, rope_cos, rope_sin);
}

// The reference's support ops around the block (FloatTransformer.cpp:79-214
// rmsnorm, :240-382 matmul; QuantizedTransformer.cpp:136-216 dequantize,
// :338-357 quantize, :359-652 int8 matmul), for kernel-level parity.
extern "C" void leapref_rmsnorm(float *o, const float *x, const float *w, int n) {
    leapref::FloatTransformer::rmsnorm(o, x, w, n);
}
extern "C" void leapref_matmul(float *xout, const float *x, const float *w, int n, int d) {
    leapref::FloatTransformer::matmul(xout, x, w, n, d);
}
extern "C" void leapref_quantize(int gs, int8_t *q, float *s, const float *x, int n) {
    leapref::QuantizedTransformer t;
    t.group_size = gs;
    leapref::QuantizedTensor qt{q, s};
    t.quantize(&qt, x, n);
}
extern "C" void leapref_dequantize(int gs, float *x, int8_t *q, float *s, int n) {
    leapref::QuantizedTransformer t;
    t.group_size = gs;
    leapref::QuantizedTensor qt{q, s};
    t.dequantize(&qt, x, n);
}
extern "C" void leapref_qmatmul(int gs, float *xout, int8_t *xq, float *xs, int8_t *wq,
                                float *ws, int n, int d) {
    leapref::QuantizedTransformer t;
    t.group_size = gs;
    leapref::QuantizedTensor xt{xq, xs}, wt{wq, ws};
    t.matmul(xout, &xt, &wt, n, d);
}

// The reference's RoPE table for a model of `dim`/`n_heads`/`seq_len`,
// [seq_len][head_size/2].  theta_10k = 0: the shipped literal 500000;
// theta_10k = 1: the same code with the literal set to 10000.
extern "C" void leapref_rope_table(int theta_10k, int dim, int n_heads,
                                   int seq_len, float *cos_out,
                                   float *sin_out) {
    const std::size_t n =
        static_cast<std::size_t>(seq_len) * ((dim / n_heads) / 2);
    if (theta_10k) {
        leapref10k::FloatTransformer t;
        t.config.dim = dim;
        t.config.n_heads = n_heads;
        t.config.seq_len = seq_len;
        t.precompute_freqs();
        std::memcpy(cos_out, t.rope_cos.data(), n * sizeof(float));
        std::memcpy(sin_out, t.rope_sin.data(), n * sizeof(float));
    } else {
        leapref::FloatTransformer t;
        t.config.dim = dim;
        t.config.n_heads = n_heads;
        t.config.seq_len = seq_len;
        t.precompute_freqs();
        std::memcpy(cos_out, t.rope_cos.data(), n * sizeof(float));
        std::memcpy(sin_out, t.rope_sin.data(), n * sizeof(float));
    }
}
