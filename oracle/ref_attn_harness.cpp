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
};
#include "fp32_softmax.inc"
#include "fp32_rope.inc"

struct QuantizedTransformer {
    static void softmax(float *x, int size);
};
#include "w8a8_softmax.inc"

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
