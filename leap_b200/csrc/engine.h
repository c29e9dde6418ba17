// engine.h — the transformer forward around attention (host side) and the
// support kernels it launches (engine_kernels.cu).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "ctx.h"

namespace leap {
namespace eng {

int embed(cudaStream_t st, float *x, const float *emb_f32, const int8_t *emb_q, const float *emb_s,
          const int *tok_dev, int n, int dim, int gs, int vocab, int *err);
int rmsnorm(cudaStream_t st, float *o, const float *x, const float *w, int rows, int dim);
int rmsnorm_quantize(cudaStream_t st, int8_t *q, float *s, const float *x, const float *w, int rows,
                     int dim);
int quantize(cudaStream_t st, int8_t *q, float *s, const float *x, size_t n, int gs);
int gemv_q8(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
            const float *ws, int n, int d, const float *res, int *err = nullptr);
// gemv_q8 of q(rmsnorm(x, nw)) (nw non-null) or q(x): the norm and the
// quantization in the persistent kernel's prologue where it can, else
// through (aq, as).  Same bits as the separate kernels.
int gemv_q8_fused(cudaStream_t st, float *y, const float *x, const float *nw, int8_t *aq,
                  float *as, const int8_t *wq, const float *ws, int n, int d, const float *res,
                  int *err = nullptr);
extern bool g_q8_slice;  // int8 GEMV: sliced one-row-per-lane kernel (else register-staged)
extern bool g_q8_tma;    // int8 GEMV: persistent bulk-copy kernel (default; takes precedence)
// int8 GEMM (prompt chunks, T tokens): the tcgen05 kind::i8 kernel
// (gemm_q8_tc.cu) where gemm_q8_tc_supported() holds and g_q8_gemm_tc is
// set (the default), else the CUDA-core dp4a kernel; both give the same bits.
extern bool g_q8_gemm_tc;
bool gemm_q8_tc_supported(const int8_t *xq, const float *xs, const int8_t *wq, const float *ws,
                          int n, int T);
int gemm_q8_tc(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
               const float *ws, int n, int d, int T, const float *res, int *err);
int gemm_q8(cudaStream_t st, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
            const float *ws, int n, int d, int T, const float *res, int *err = nullptr);
// y = W . a (+ res); a = x, or rmsnorm(x, nw) formed in the GEMV's prologue
// (same bits as rmsnorm followed by the GEMV; xb: a scratch row for the
// unfused route, used when x is misaligned or too long for shared memory).
int gemv_f32(cudaStream_t st, float *y, const float *x, const float *w, int n, int d,
             const float *res, const float *nw = nullptr, float *xb = nullptr);
int gemm_f32(cudaStream_t st, float *y, const float *x, const float *w, int n, int d, int T,
             const float *res);
int silu_mul(cudaStream_t st, float *h, const float *h3, size_t n);
int silu_mul_quantize(cudaStream_t st, int8_t *q, float *s, const float *h, const float *h3,
                      size_t n);
int argmax(cudaStream_t st, int *out, const float *v, int n);
}  // namespace eng
// One Sampler::sample on device logits (sampler.cu).
int sampler_launch(leap_sampler *s, cudaStream_t st, const float *logits, int *token_dev);
namespace eng {
int synth_normal(cudaStream_t st, float *w, size_t n, uint64_t seed, float std, float fill);

// A weight matrix [rows][cols]: FP32, or int8 with one float scale per group
// of `gs` consecutive values (the reference QuantizedTensor,
// src/inference/QuantizedTransformer.h:9-12).
struct Mat {
    float *f = nullptr;
    int8_t *q = nullptr;
    float *s = nullptr;
    int rows = 0, cols = 0;
};

}  // namespace eng
}  // namespace leap

struct leap_engine {
    leap_model_config cfg{};
    int head_dim = 0, kv_dim = 0, group = 0;
    int layer_begin = 0, layer_end = 0, n_local = 0;
    bool has_embed = false, has_head = false;
    int device = 0;
    cudaStream_t own_stream = nullptr, stream = nullptr;
    leap_ctx *attn = nullptr;

    std::vector<void *> allocs;  // every device allocation, freed at destroy

    // weights of the local layers
    float *rms_att = nullptr, *rms_ffn = nullptr, *rms_final = nullptr;
    std::vector<leap::eng::Mat> wqkv, wo, w13, w2;  // [wq;wk;wv], [w1;w3] stacked by rows
    leap::eng::Mat emb, wcls;                        // embedding; classifier (may alias emb)

    // single-token activations
    float *x = nullptr, *xb = nullptr, *qkv = nullptr, *att = nullptr, *h13 = nullptr;
    float *logits = nullptr;
    int8_t *aq = nullptr;
    float *as = nullptr;
    int *tok_dev = nullptr, *argmax_dev = nullptr;
    leap_sampler *sampler = nullptr;  // not owned; NULL = greedy argmax
    int *h_tok = nullptr;  // pinned host mirror for token ids

    // prompt-chunk activations, max_chunk tokens
    int max_chunk = 0;
    float *bx = nullptr, *bxb = nullptr, *bq = nullptr, *bk = nullptr, *bv = nullptr;
    float *batt = nullptr, *bh1 = nullptr, *bh3 = nullptr;
    int8_t *baq = nullptr;
    float *bas = nullptr;
    int *btok = nullptr;

    size_t device_bytes = 0;
};
