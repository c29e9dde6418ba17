/*
 * leap_oracle.c — CPU restatement of LEAP's attention hot path (and of the
 * support ops around it), in plain C.
 *
 * TEST INFRASTRUCTURE ONLY: the checker for the CUDA path.  Only tests/,
 * __graft_entry__.smoke() and bench.py's CPU baseline leg load it; the
 * product path never calls it and has no CPU fallback.
 *
 * Each function restates the arithmetic of the reference file:line it cites
 * (paths inside Harikeshav-R/LEAP).  Where the reference's x86 build runs an
 * AVX2 branch, the restatement follows that branch's operation order (8-lane
 * FMA partial sums, then the lo+hi / hadd / hadd horizontal sum) so that the
 * results track the reference to the last few ulps.  Built with
 * -ffp-contract=off so that only the explicit fmaf() calls fuse.
 *
 * Parity of this file is pinned against the reference compiled from its own
 * sources (oracle/Makefile -> oracle/_ref/) by tests/test_oracle.py through
 * the fixtures in tests/golden/.
 */
#include "leap_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* FloatTransformer.cpp:56-72 (QuantizedTransformer.cpp:65-81).  The shipped
 * reference hard-codes theta = 500000 (:65); theta is a parameter here so the
 * same table can be made for other models.
 * The source says freq = 1/std::pow(theta, i/hs), but the reference's release
 * build (-ffast-math, CMakeLists.txt:33) evaluates that as
 * expf(-(i/hs) * logf(theta)); the two differ by an ulp in freq, which moves
 * cos/sin(pos*freq) by up to 5e-4 at pos 8192.  This follows what the
 * compiled reference computes, and matches its table bit for bit. */
void orc_rope_table(int seq_len, int head_size, float theta, float *rope_cos,
                    float *rope_sin) {
    const int half = head_size / 2;
    const float log_theta = logf(theta);
    for (int pos = 0; pos < seq_len; pos++) {
        for (int i = 0; i < head_size; i += 2) {
            const float e = (float)i / (float)head_size;
            const float freq = expf(-(e * log_theta));
            const float val = (float)pos * freq;
            rope_cos[pos * half + i / 2] = cosf(val);
            rope_sin[pos * half + i / 2] = sinf(val);
        }
    }
}

/* FloatTransformer.cpp:216-238: max, exp(x - max) with running sum,
 * multiply by 1/sum. */
void orc_softmax(float *x, int size) {
    float max_val = x[0];
    for (int i = 1; i < size; i++)
        if (x[i] > max_val) max_val = x[i];
    float sum = 0.0f;
    for (int i = 0; i < size; i++) {
        x[i] = expf(x[i] - max_val);
        sum += x[i];
    }
    const float inv_sum = 1.0f / sum;
    for (int i = 0; i < size; i++) x[i] *= inv_sum;
}

/* Interleaved-pair rotation of one head, FloatTransformer.cpp:446-493.  The
 * AVX2 branch computes x*c and swap(x)*s as two rounded products and then
 * _mm256_addsub_ps: even lane x0*c - x1*s, odd lane x1*c + x0*s. */
static void rope_rotate(float *x, const float *c, const float *s, int hs) {
    for (int j = 0; j < hs; j += 2) {
        const float fcr = c[j / 2], fci = s[j / 2];
        const float x0 = x[j], x1 = x[j + 1];
        const float a = x0 * fcr, b = x1 * fci; /* rounded products */
        const float e = x1 * fcr, f = x0 * fci;
        x[j] = a - b;
        x[j + 1] = e + f;
    }
}

/* 8-lane FMA dot product with the AVX2 horizontal sum of
 * FloatTransformer.cpp:527-556 / :609-624 (head_size is a multiple of 8 for
 * every shape the engine supports; a scalar tail follows :580-586). */
static float dot_avx2_order(const float *a, const float *b, int n) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int i = 0;
    for (; i + 8 <= n; i += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(a[i + l], b[i + l], acc[l]);
    /* lo + hi, then two hadd: ((a0+a4)+(a1+a5)) + ((a2+a6)+(a3+a7)) */
    const float t0 = acc[0] + acc[4], t1 = acc[1] + acc[5];
    const float t2 = acc[2] + acc[6], t3 = acc[3] + acc[7];
    float r = (t0 + t1) + (t2 + t3);
    /* Scalar tail (:330-339 / :375-377).  The release build (-O3
     * -ffast-math) turns 4 or more leftover elements into one 4-wide step:
     * separately rounded products, summed (p0+p2)+(p1+p3) and added to the
     * running value; the rest become fma.  Checked against the compiled
     * reference for tails of 1..7. */
    if (n - i >= 4) {
        const float p0 = a[i] * b[i], p1 = a[i + 1] * b[i + 1];
        const float p2 = a[i + 2] * b[i + 2], p3 = a[i + 3] * b[i + 3];
        r = r + ((p0 + p2) + (p1 + p3));
        i += 4;
    }
    for (; i < n; i++) r = fmaf(a[i], b[i], r);
    return r;
}

/* One query head, FloatTransformer.cpp:501-661: scores over t = 0..pos,
 * softmax (:632), weighted V sum into xb with FMA (:637-661). */
static void attn_head(int h, int head_size, int kv_dim, int kv_mul,
                      int seq_len, int pos, const float *q,
                      const float *k_cache, const float *v_cache, float *att,
                      float *xb) {
    const float att_scale = 1.0f / sqrtf((float)head_size); /* :497 */
    const float *qh = q + h * head_size;
    float *ah = att + (size_t)h * seq_len;
    const int kvh = h / kv_mul; /* :508 */
    for (int t = 0; t <= pos; t++) {
        const float *kr = k_cache + (size_t)t * kv_dim + kvh * head_size;
        ah[t] = dot_avx2_order(qh, kr, head_size) * att_scale;
    }
    orc_softmax(ah, pos + 1);
    float *o = xb + h * head_size;
    memset(o, 0, sizeof(float) * head_size);
    for (int t = 0; t <= pos; t++) {
        const float *vr = v_cache + (size_t)t * kv_dim + kvh * head_size;
        const float a = ah[t];
        for (int i = 0; i < head_size; i++) o[i] = fmaf(a, vr[i], o[i]);
    }
}

/* FloatTransformer.cpp:404-662 (QuantizedTransformer.cpp:680-923). */
void orc_attn_block(int n_heads, int n_kv_heads, int head_size, int seq_len,
                    int pos, const float *rope_cos, const float *rope_sin,
                    float *q, float *k_cache, float *v_cache, float *att,
                    float *xb, int n_threads) {
    const int kv_dim = n_kv_heads * head_size;
    const int kv_mul = n_heads / n_kv_heads;
    const int half = head_size / 2;
    const float *c = rope_cos + (size_t)pos * half; /* rope_offset, :405 */
    const float *s = rope_sin + (size_t)pos * half;
    float *krow = k_cache + (size_t)pos * kv_dim;
    /* RoPE: every q head; k heads of the new cache row (:437, :468, :487) */
    for (int i = 0; i < n_heads; i++) {
        rope_rotate(q + i * head_size, c, s, head_size);
        if (i < n_kv_heads) rope_rotate(krow + i * head_size, c, s, head_size);
    }
    if (n_threads < 1) n_threads = 1;
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int h = 0; h < n_heads; h++)
        attn_head(h, head_size, kv_dim, kv_mul, seq_len, pos, q, k_cache,
                  v_cache, att, xb);
}

/* main.cpp:80-89 feeds the prompt through forward() one position at a
 * time; per position the projections write row pos of the caches
 * (FloatTransformer.cpp:397-402) and the block runs. */
void orc_attn_prefill(int n_heads, int n_kv_heads, int head_size, int seq_len,
                      int pos0, int n_tok, const float *rope_cos,
                      const float *rope_sin, const float *q, const float *k,
                      const float *v, float *k_cache, float *v_cache,
                      float *out, int n_threads) {
    const int dim = n_heads * head_size;
    const int kv_dim = n_kv_heads * head_size;
    float *qbuf = (float *)malloc(sizeof(float) * dim);
    float *att = (float *)malloc(sizeof(float) * (size_t)n_heads * seq_len);
    for (int i = 0; i < n_tok; i++) {
        const int pos = pos0 + i;
        memcpy(qbuf, q + (size_t)i * dim, sizeof(float) * dim);
        memcpy(k_cache + (size_t)pos * kv_dim, k + (size_t)i * kv_dim,
               sizeof(float) * kv_dim);
        memcpy(v_cache + (size_t)pos * kv_dim, v + (size_t)i * kv_dim,
               sizeof(float) * kv_dim);
        orc_attn_block(n_heads, n_kv_heads, head_size, seq_len, pos, rope_cos,
                       rope_sin, qbuf, k_cache, v_cache, att,
                       out + (size_t)i * dim, n_threads);
    }
    free(att);
    free(qbuf);
}

/* FloatTransformer.cpp:79-214.  Sum of squares in the AVX2 8-lane FMA
 * order, ss/size + 1e-5, then the scalar branch's 1/sqrtf (:164).  The AVX2
 * branch's rsqrt estimate + one Newton step (:155-162) depends on the CPU's
 * rsqrt approximation table and lands within ~1 ulp of 1/sqrtf. */
void orc_rmsnorm(float *o, const float *x, const float *weight, int size) {
    float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    int j = 0;
    for (; j + 8 <= size; j += 8)
        for (int l = 0; l < 8; l++) acc[l] = fmaf(x[j + l], x[j + l], acc[l]);
    const float t0 = acc[0] + acc[4], t1 = acc[1] + acc[5];
    const float t2 = acc[2] + acc[6], t3 = acc[3] + acc[7];
    float ss = (t0 + t1) + (t2 + t3);
    for (; j < size; j++) ss += x[j] * x[j];
    ss /= (float)size;
    ss += 1e-5f;
    ss = 1.0f / sqrtf(ss);
    for (j = 0; j < size; j++) o[j] = weight[j] * (ss * x[j]);
}

/* FloatTransformer.cpp:240-382: each output row is an 8-lane FMA dot
 * product with the AVX2 horizontal sum. */
void orc_matmul(float *xout, const float *x, const float *w, int n, int d,
                int n_threads) {
    if (n_threads < 1) n_threads = 1;
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < d; i++) xout[i] = dot_avx2_order(w + (size_t)i * n, x, n);
}

/* QuantizedTransformer.cpp:338-357 (same math as the exporter,
 * src/export/Utils.cpp:58-85).  std::round rounds half away from zero,
 * which is C roundf.  The source computes scale = max / 127.0f and
 * id = 1.0f / scale; the reference's release build (-ffast-math) evaluates
 * them as scale = max * (1/127) and id = 127 / max (checked against the
 * compiled reference: the source's quotient differs in the last bit for ~5%
 * of groups, and 1/scale moves a code across a rounding boundary about once
 * in 10^5 values).  This follows the compiled form. */
void orc_quantize(int8_t *q, float *s, const float *x, int n, int gs) {
    const float inv127 = 1.0f / 127.0f;
    for (int i = 0; i < n; i += gs) {
        const int cur = (gs < n - i) ? gs : n - i;
        float max_val = 0.0f;
        for (int j = 0; j < cur; j++) {
            const float a = fabsf(x[i + j]);
            if (a > max_val) max_val = a;
        }
        const float scale = max_val * inv127;
        const float id = scale != 0.0f ? 127.0f / max_val : 0.0f;
        s[i / gs] = scale;
        for (int j = 0; j < cur; j++) q[i + j] = (int8_t)roundf(x[i + j] * id);
    }
}

/* QuantizedTransformer.cpp:359-652: per output row, groups in order; the
 * int32 group dot is exact, then val += float(ival) * w_s * x_s, which the
 * reference's release build evaluates as val = fma(float(ival), w_s*x_s, val)
 * (bit-exact against the compiled reference; the literal left-to-right
 * order matches only ~30% of outputs). */
void orc_qmatmul(float *xout, const int8_t *xq, const float *xs,
                 const int8_t *wq, const float *ws, int n, int d, int gs,
                 int n_threads) {
    if (n_threads < 1) n_threads = 1;
#ifdef _OPENMP
#pragma omp parallel for num_threads(n_threads) schedule(static)
#endif
    for (int i = 0; i < d; i++) {
        const size_t in = (size_t)i * n;
        float val = 0.0f;
        for (int j = 0; j + gs <= n; j += gs) {
            int32_t ival = 0;
            for (int k = 0; k < gs; k++)
                ival += (int32_t)xq[j + k] * (int32_t)wq[in + j + k];
            const float t = ws[(in + j) / gs] * xs[j / gs];
            val = fmaf((float)ival, t, val);
        }
        xout[i] = val;
    }
}
