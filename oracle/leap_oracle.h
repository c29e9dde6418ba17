/*
 * leap_oracle.h — CPU restatement of LEAP's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is the checker that the CUDA path is
 * compared against; only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product path never calls it.
 *
 * Every function restates, in plain C, the arithmetic of the reference file
 * and lines it cites (Harikeshav-R/LEAP, src/inference/...).  Parity of this
 * restatement is pinned against the reference itself compiled from its own
 * sources (oracle/Makefile -> oracle/_ref/) through the golden fixtures in
 * tests/golden/.
 */
#ifndef LEAP_ORACLE_H
#define LEAP_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* RoPE table, FloatTransformer.cpp:56-72: for even i < head_size,
 * freq = 1/powf(theta, i/head_size), cos/sin(pos*freq) at [pos][i/2]. */
void orc_rope_table(int seq_len, int head_size, float theta, float *rope_cos,
                    float *rope_sin);

/* softmax in place over `size` values, FloatTransformer.cpp:216-238. */
void orc_softmax(float *x, int size);

/*
 * The attention block, FloatTransformer.cpp:404-662 (twin:
 * QuantizedTransformer.cpp:680-923).  The caller has already written the new
 * un-rotated k and v into row `pos` of the layer's caches, as the projection
 * matmuls do in the reference (:397-402).  On return q and cache row `pos`
 * of K are rotated in place and xb holds the output.
 *   q       [n_heads*head_size]
 *   k_cache [seq_len][kv_dim], v_cache [seq_len][kv_dim]  (one layer)
 *   att     scratch [n_heads*seq_len]
 *   xb      [n_heads*head_size]
 * n_threads > 1 splits the head loop like the reference's `omp parallel for`
 * over heads (:500).
 */
void orc_attn_block(int n_heads, int n_kv_heads, int head_size, int seq_len,
                    int pos, const float *rope_cos, const float *rope_sin,
                    float *q, float *k_cache, float *v_cache, float *att,
                    float *xb, int n_threads);

/*
 * Causal prefill as the reference does it: the block above for
 * pos = pos0 .. pos0+n_tok-1 in order (src/inference/main.cpp:80-89), each
 * step first writing token i's un-rotated k/v into cache row pos0+i.
 *   q [n_tok][n_heads*hs], k/v [n_tok][kv_dim], out [n_tok][n_heads*hs]
 */
void orc_attn_prefill(int n_heads, int n_kv_heads, int head_size, int seq_len,
                      int pos0, int n_tok, const float *rope_cos,
                      const float *rope_sin, const float *q, const float *k,
                      const float *v, float *k_cache, float *v_cache,
                      float *out, int n_threads);

/* RMSNorm, FloatTransformer.cpp:79-214 (AVX2 branch: 8-lane sum of squares,
 * rsqrt estimate refined by one Newton step is replaced by 1/sqrtf, see the
 * function comment). */
void orc_rmsnorm(float *o, const float *x, const float *weight, int size);

/* FP32 GEMV W(d,n).x(n) -> xout(d), FloatTransformer.cpp:240-382. */
void orc_matmul(float *xout, const float *x, const float *w, int n, int d,
                int n_threads);

/* Per-group int8 quantization, QuantizedTransformer.cpp:338-357 and
 * src/export/Utils.cpp:58-85: s = max|x|/127, q = round_half_away(x/s). */
void orc_quantize(int8_t *q, float *s, const float *x, int n, int gs);

/* W8A8 GEMV, QuantizedTransformer.cpp:359-652: per output row the sum over
 * groups of float(int32 dot) * w_s * x_s. */
void orc_qmatmul(float *xout, const int8_t *xq, const float *xs,
                 const int8_t *wq, const float *ws, int n, int d, int gs,
                 int n_threads);

#ifdef __cplusplus
}
#endif

#endif /* LEAP_ORACLE_H */
