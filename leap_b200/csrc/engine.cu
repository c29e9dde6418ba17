// engine.cu — the transformer forward around attention: LEAP's .bin loader
// and the per-layer step of run_layer on the GPU, for a contiguous range of
// layers (the whole model, or one pipeline stage).
//
// Reference: src/inference/TransformerFactory.cpp:59-135 (header, formats),
// FloatTransformer.cpp:947-978 / QuantizedTransformer.cpp:88-134 (weight
// order), FloatTransformer.cpp:384-797 / QuantizedTransformer.cpp:654-1061
// (forward).  Attention runs through the leap_ctx kernels of this library.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

#include "engine.h"

using leap::eng::Mat;

namespace {

constexpr int kMagic = 0x616B3432;

struct Mapped {
    int fd = -1;
    void *p = MAP_FAILED;
    size_t size = 0;
    ~Mapped() {
        if (p != MAP_FAILED) munmap(p, size);
        if (fd >= 0) close(fd);
    }
};

struct DevGuard {
    int prev = -1;
    explicit DevGuard(int d) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(d);
    }
    ~DevGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

#define ETRY(expr)                       \
    do {                                 \
        const int st_ = (expr);          \
        if (st_ != LEAP_OK) return st_;  \
    } while (0)

int dalloc(leap_engine *e, void **p, size_t bytes) {
    *p = nullptr;
    if (bytes == 0) return LEAP_OK;
    const cudaError_t err = cudaMalloc(p, bytes);
    if (err != cudaSuccess) return leap::cuda_status(err, "cudaMalloc(engine)");
    e->allocs.push_back(*p);
    e->device_bytes += bytes;
    return LEAP_OK;
}

template <class T>
int dalloc_t(leap_engine *e, T **p, size_t n) {
    return dalloc(e, reinterpret_cast<void **>(p), n * sizeof(T));
}

void free_engine(leap_engine *e) {
    if (!e) return;
    DevGuard g(e->device);
    if (e->own_stream) cudaStreamSynchronize(e->own_stream);
    if (e->stream && e->stream != e->own_stream) cudaStreamSynchronize(e->stream);
    if (e->attn) leap_ctx_destroy(e->attn);
    for (void *p : e->allocs) cudaFree(p);
    if (e->h_tok) cudaFreeHost(e->h_tok);
    if (e->own_stream) cudaStreamDestroy(e->own_stream);
    delete e;
}

// Header: TransformerFactory.cpp:59-118.
int parse_header(const unsigned char *b, size_t size, leap_model_config *c, size_t *hdr) {
    if (size < 28) {
        leap::set_error("model file too short for a header");
        return LEAP_ERR_INVALID;
    }
    int magic;
    std::memcpy(&magic, b, 4);
    int cfg[7];
    c->quantized = 0;
    c->group_size = 0;
    int shared = 0;
    if (magic == kMagic) {
        int version;
        std::memcpy(&version, b + 4, 4);
        std::memcpy(cfg, b + 8, sizeof(cfg));
        if (version == 1) {
            *hdr = 256;
        } else if (version == 2) {
            c->quantized = 1;
            shared = b[36];
            std::memcpy(&c->group_size, b + 37, 4);
            *hdr = 256;
        } else {
            leap::set_error("Bad file version %d", version);
            return LEAP_ERR_INVALID;
        }
    } else {  // legacy v0: the Config struct at offset 0
        std::memcpy(cfg, b, sizeof(cfg));
        *hdr = sizeof(cfg);
    }
    c->dim = cfg[0];
    c->hidden_dim = cfg[1];
    c->n_layers = cfg[2];
    c->n_heads = cfg[3];
    c->n_kv_heads = cfg[4];
    c->vocab_size = cfg[5];
    c->seq_len = cfg[6];
    if (!c->quantized) {  // :115-118 — FP32 files tie the classifier unless vocab < 0
        shared = c->vocab_size > 0 ? 1 : 0;
        c->vocab_size = std::abs(c->vocab_size);
    }
    c->shared_classifier = shared;
    return LEAP_OK;
}

int check_config(const leap_model_config &c) {
    if (c.dim <= 0 || c.hidden_dim <= 0 || c.n_layers <= 0 || c.n_heads <= 0 ||
        c.n_kv_heads <= 0 || c.vocab_size <= 0 || c.seq_len <= 0 || c.dim % c.n_heads ||
        c.n_heads % c.n_kv_heads) {
        leap::set_error("invalid model config dim %d hidden %d layers %d heads %d/%d vocab %d seq %d",
                        c.dim, c.hidden_dim, c.n_layers, c.n_heads, c.n_kv_heads, c.vocab_size,
                        c.seq_len);
        return LEAP_ERR_INVALID;
    }
    if (c.quantized && (c.group_size <= 0 || c.group_size != 64 || c.dim % 64 || c.hidden_dim % 64)) {
        leap::set_error("W8A8 engine supports group size 64 with dim/hidden multiples of 64 (got gs %d)",
                        c.group_size);
        return LEAP_ERR_INVALID;
    }
    if (c.dim % 4 || c.hidden_dim % 4) {
        leap::set_error("dim and hidden_dim must be multiples of 4");
        return LEAP_ERR_INVALID;
    }
    return LEAP_OK;
}

// Allocate the matrices and activations of the engine's range (weights not
// yet filled).
int allocate(leap_engine *e) {
    const leap_model_config &c = e->cfg;
    const bool q8 = c.quantized;
    const int dim = c.dim, hid = c.hidden_dim, kv = e->kv_dim;
    auto mat = [&](Mat &m, int rows, int cols) -> int {
        m.rows = rows;
        m.cols = cols;
        const size_t n = size_t(rows) * cols;
        if (q8) {
            ETRY(dalloc_t(e, &m.q, n));
            ETRY(dalloc_t(e, &m.s, n / c.group_size));
        } else {
            ETRY(dalloc_t(e, &m.f, n));
        }
        return LEAP_OK;
    };
    e->wqkv.resize(e->n_local);
    e->wo.resize(e->n_local);
    e->w13.resize(e->n_local);
    e->w2.resize(e->n_local);
    ETRY(dalloc_t(e, &e->rms_att, size_t(e->n_local) * dim));
    ETRY(dalloc_t(e, &e->rms_ffn, size_t(e->n_local) * dim));
    for (int i = 0; i < e->n_local; ++i) {
        ETRY(mat(e->wqkv[i], dim + 2 * kv, dim));
        ETRY(mat(e->wo[i], dim, dim));
        ETRY(mat(e->w13[i], 2 * hid, dim));
        ETRY(mat(e->w2[i], dim, hid));
    }
    if (e->has_embed) ETRY(mat(e->emb, c.vocab_size, dim));
    if (e->has_head) {
        ETRY(dalloc_t(e, &e->rms_final, dim));
        if (c.shared_classifier && e->has_embed)
            e->wcls = e->emb;
        else
            ETRY(mat(e->wcls, c.vocab_size, dim));
        ETRY(dalloc_t(e, &e->logits, c.vocab_size));
    }
    const int mx = dim > hid ? dim : hid;
    ETRY(dalloc_t(e, &e->x, dim));
    ETRY(dalloc_t(e, &e->xb, dim));
    ETRY(dalloc_t(e, &e->qkv, dim + 2 * kv));
    ETRY(dalloc_t(e, &e->att, dim));
    ETRY(dalloc_t(e, &e->h13, 2 * size_t(hid)));
    ETRY(dalloc_t(e, &e->aq, mx));
    ETRY(dalloc_t(e, &e->as, mx / 16 + 4));
    ETRY(dalloc_t(e, &e->tok_dev, 4));
    ETRY(dalloc_t(e, &e->argmax_dev, 4));
    const size_t T = e->max_chunk;
    ETRY(dalloc_t(e, &e->bx, T * dim));
    ETRY(dalloc_t(e, &e->bxb, T * dim));
    ETRY(dalloc_t(e, &e->bq, T * dim));
    ETRY(dalloc_t(e, &e->bk, T * kv));
    ETRY(dalloc_t(e, &e->bv, T * kv));
    ETRY(dalloc_t(e, &e->batt, T * dim));
    ETRY(dalloc_t(e, &e->bh1, T * hid));
    ETRY(dalloc_t(e, &e->bh3, T * hid));
    ETRY(dalloc_t(e, &e->baq, T * mx));
    ETRY(dalloc_t(e, &e->bas, T * mx / 16 + 4));
    ETRY(dalloc_t(e, &e->btok, T));
    const cudaError_t err = cudaMallocHost(&e->h_tok, 64 * sizeof(int));
    if (err != cudaSuccess) return leap::cuda_status(err, "cudaMallocHost(engine)");
    return LEAP_OK;
}

int make_attention(leap_engine *e, float theta) {
    const leap_model_config &c = e->cfg;
    std::vector<float> rc(size_t(c.seq_len) * (e->head_dim / 2)), rs(rc.size());
    ETRY(leap_rope_table(c.seq_len, e->head_dim, theta, rc.data(), rs.data()));
    leap_ctx_desc d{};
    d.n_layers = e->n_local;
    d.layer0 = e->layer_begin;
    d.n_heads = c.n_heads;
    d.n_kv_heads = c.n_kv_heads;
    d.head_dim = e->head_dim;
    d.max_seq = c.seq_len;
    d.max_batch = 1;
    d.device = e->device;
    d.rope_cos = rc.data();
    d.rope_sin = rs.data();
    ETRY(leap_ctx_create(&d, &e->attn));
    ETRY(leap_ctx_set_stream(e->attn, e->stream));
    size_t b = 0;
    leap_ctx_device_bytes(e->attn, &b);
    e->device_bytes += b;
    return LEAP_OK;
}

int begin(leap_engine **out, const leap_model_config &cfg, int device, int lb, int le,
          int max_chunk, leap_engine **pe) {
    *out = nullptr;
    ETRY(check_config(cfg));
    if (le < 0) le = cfg.n_layers;
    if (lb < 0 || lb >= le || le > cfg.n_layers) {
        leap::set_error("layer range [%d,%d) invalid for %d layers", lb, le, cfg.n_layers);
        return LEAP_ERR_INVALID;
    }
    const int hd = cfg.dim / cfg.n_heads;
    if (hd != 64 && hd != 128) {
        leap::set_error("head_dim %d unsupported (64 or 128)", hd);
        return LEAP_ERR_INVALID;
    }
    leap_engine *e = new (std::nothrow) leap_engine();
    if (!e) {
        leap::set_error("host allocation failed");
        return LEAP_ERR_NOMEM;
    }
    e->cfg = cfg;
    e->head_dim = hd;
    e->kv_dim = cfg.n_kv_heads * hd;
    e->group = cfg.n_heads / cfg.n_kv_heads;
    e->layer_begin = lb;
    e->layer_end = le;
    e->n_local = le - lb;
    e->has_embed = lb == 0;
    e->has_head = le == cfg.n_layers;
    e->device = device;
    e->max_chunk = max_chunk > 0 ? max_chunk : 512;
    *pe = e;
    const cudaError_t err = cudaStreamCreateWithFlags(&e->own_stream, cudaStreamNonBlocking);
    if (err != cudaSuccess) return leap::cuda_status(err, "cudaStreamCreate(engine)");
    e->stream = e->own_stream;
    return LEAP_OK;
}

// ---- file upload -------------------------------------------------------------
struct Cursor {
    const unsigned char *p;
    const unsigned char *end;
    bool ok = true;
    const unsigned char *take(size_t bytes) {
        if (size_t(end - p) < bytes) {
            ok = false;
            return nullptr;
        }
        const unsigned char *r = p;
        p += bytes;
        return r;
    }
};

int up(leap_engine *e, void *dst, const void *src, size_t bytes) {
    if (!bytes) return LEAP_OK;
    return leap::cuda_status(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice), "upload");
}

int load_fp32(leap_engine *e, Cursor &cur) {
    const leap_model_config &c = e->cfg;
    const size_t dim = c.dim, hid = c.hidden_dim, kv = e->kv_dim, L = c.n_layers;
    const size_t lb = e->layer_begin, nl = e->n_local;
    const float *rms_att = reinterpret_cast<const float *>(cur.take(L * dim * 4));
    const float *rms_ffn = reinterpret_cast<const float *>(cur.take(L * dim * 4));
    const float *rms_final = reinterpret_cast<const float *>(cur.take(dim * 4));
    const unsigned char *emb = cur.take(size_t(c.vocab_size) * dim * 4);
    const unsigned char *wq = cur.take(L * dim * dim * 4);
    const unsigned char *wk = cur.take(L * kv * dim * 4);
    const unsigned char *wv = cur.take(L * kv * dim * 4);
    const unsigned char *wo = cur.take(L * dim * dim * 4);
    const unsigned char *w1 = cur.take(L * hid * dim * 4);
    const unsigned char *w2 = cur.take(L * dim * hid * 4);
    const unsigned char *w3 = cur.take(L * hid * dim * 4);
    const unsigned char *wcls = c.shared_classifier ? emb : cur.take(size_t(c.vocab_size) * dim * 4);
    if (!cur.ok) {
        leap::set_error("model file shorter than its config requires");
        return LEAP_ERR_INVALID;
    }
    ETRY(up(e, e->rms_att, rms_att + lb * dim, nl * dim * 4));
    ETRY(up(e, e->rms_ffn, rms_ffn + lb * dim, nl * dim * 4));
    for (size_t i = 0; i < nl; ++i) {
        const size_t l = lb + i;
        float *qkv = e->wqkv[i].f;
        ETRY(up(e, qkv, wq + l * dim * dim * 4, dim * dim * 4));
        ETRY(up(e, qkv + dim * dim, wk + l * kv * dim * 4, kv * dim * 4));
        ETRY(up(e, qkv + dim * dim + kv * dim, wv + l * kv * dim * 4, kv * dim * 4));
        ETRY(up(e, e->wo[i].f, wo + l * dim * dim * 4, dim * dim * 4));
        ETRY(up(e, e->w13[i].f, w1 + l * hid * dim * 4, hid * dim * 4));
        ETRY(up(e, e->w13[i].f + hid * dim, w3 + l * hid * dim * 4, hid * dim * 4));
        ETRY(up(e, e->w2[i].f, w2 + l * dim * hid * 4, dim * hid * 4));
    }
    if (e->has_embed) ETRY(up(e, e->emb.f, emb, size_t(c.vocab_size) * dim * 4));
    if (e->has_head) {
        ETRY(up(e, e->rms_final, rms_final, dim * 4));
        if (e->wcls.f != e->emb.f) ETRY(up(e, e->wcls.f, wcls, size_t(c.vocab_size) * dim * 4));
    }
    return LEAP_OK;
}

// QuantizedTransformer.cpp:88-134: each tensor is int8[numel] then
// float[numel / gs]; per-layer tensors follow one another.
struct QT {
    const unsigned char *q = nullptr, *s = nullptr;
};

int load_q8(leap_engine *e, Cursor &cur) {
    const leap_model_config &c = e->cfg;
    const size_t dim = c.dim, hid = c.hidden_dim, kv = e->kv_dim, L = c.n_layers;
    const size_t gs = c.group_size, lb = e->layer_begin, nl = e->n_local;
    const float *rms_att = reinterpret_cast<const float *>(cur.take(L * dim * 4));
    const float *rms_ffn = reinterpret_cast<const float *>(cur.take(L * dim * 4));
    const float *rms_final = reinterpret_cast<const float *>(cur.take(dim * 4));
    auto qt = [&](size_t numel) {
        QT t;
        t.q = cur.take(numel);
        t.s = cur.take(numel / gs * 4);
        return t;
    };
    const QT tok = qt(size_t(c.vocab_size) * dim);
    std::vector<QT> wq(L), wk(L), wv(L), wo(L), w1(L), w2(L), w3(L);
    for (auto &t : wq) t = qt(dim * dim);
    for (auto &t : wk) t = qt(dim * kv);
    for (auto &t : wv) t = qt(dim * kv);
    for (auto &t : wo) t = qt(dim * dim);
    for (auto &t : w1) t = qt(dim * hid);
    for (auto &t : w2) t = qt(hid * dim);
    for (auto &t : w3) t = qt(dim * hid);
    const QT cls = c.shared_classifier ? tok : qt(dim * size_t(c.vocab_size));
    if (!cur.ok) {
        leap::set_error("model file shorter than its config requires");
        return LEAP_ERR_INVALID;
    }
    auto put = [&](int8_t *dq, float *ds, size_t row0, const QT &t, size_t numel) -> int {
        ETRY(up(e, dq + row0, t.q, numel));
        ETRY(up(e, ds + row0 / gs, t.s, numel / gs * 4));
        return LEAP_OK;
    };
    ETRY(up(e, e->rms_att, rms_att + lb * dim, nl * dim * 4));
    ETRY(up(e, e->rms_ffn, rms_ffn + lb * dim, nl * dim * 4));
    for (size_t i = 0; i < nl; ++i) {
        const size_t l = lb + i;
        ETRY(put(e->wqkv[i].q, e->wqkv[i].s, 0, wq[l], dim * dim));
        ETRY(put(e->wqkv[i].q, e->wqkv[i].s, dim * dim, wk[l], dim * kv));
        ETRY(put(e->wqkv[i].q, e->wqkv[i].s, dim * dim + dim * kv, wv[l], dim * kv));
        ETRY(put(e->wo[i].q, e->wo[i].s, 0, wo[l], dim * dim));
        ETRY(put(e->w13[i].q, e->w13[i].s, 0, w1[l], dim * hid));
        ETRY(put(e->w13[i].q, e->w13[i].s, dim * hid, w3[l], dim * hid));
        ETRY(put(e->w2[i].q, e->w2[i].s, 0, w2[l], hid * dim));
    }
    if (e->has_embed) ETRY(put(e->emb.q, e->emb.s, 0, tok, size_t(c.vocab_size) * dim));
    if (e->has_head) {
        ETRY(up(e, e->rms_final, rms_final, dim * 4));
        if (e->wcls.q != e->emb.q) ETRY(put(e->wcls.q, e->wcls.s, 0, cls, size_t(c.vocab_size) * dim));
    }
    return LEAP_OK;
}

// ---- synthetic weights ---------------------------------------------------------
uint64_t mix(uint64_t a, uint64_t b) {
    uint64_t z = a * 0x9E3779B97F4A7C15ull + b + 0x632BE59BD9B4E019ull;
    z = (z ^ (z >> 31)) * 0xBF58476D1CE4E5B9ull;
    return z ^ (z >> 29);
}

int synth_mat(leap_engine *e, Mat &m, uint64_t seed, float *tmp, size_t tmp_n) {
    const size_t n = size_t(m.rows) * m.cols;
    if (m.f) return leap::eng::synth_normal(e->stream, m.f, n, seed, 0.02f, 0.f);
    const size_t gs = e->cfg.group_size;
    size_t chunk = tmp_n / gs * gs;
    for (size_t o = 0, k = 0; o < n; o += chunk, ++k) {
        const size_t nn = (n - o) < chunk ? (n - o) : chunk;
        ETRY(leap::eng::synth_normal(e->stream, tmp, nn, mix(seed, k), 0.02f, 0.f));
        ETRY(leap::eng::quantize(e->stream, m.q + o, m.s + o / gs, tmp, nn, int(gs)));
    }
    return LEAP_OK;
}

int synthesize(leap_engine *e, uint64_t seed) {
    const leap_model_config &c = e->cfg;
    float *tmp = nullptr;
    const size_t tmp_n = size_t(64) << 20;  // 256 MB of FP32 staging
    if (c.quantized) ETRY(dalloc_t(e, &tmp, tmp_n));
    ETRY(leap::eng::synth_normal(e->stream, e->rms_att, size_t(e->n_local) * c.dim, 0, 0.f, 1.f));
    ETRY(leap::eng::synth_normal(e->stream, e->rms_ffn, size_t(e->n_local) * c.dim, 0, 0.f, 1.f));
    for (int i = 0; i < e->n_local; ++i) {
        const uint64_t l = uint64_t(e->layer_begin + i);
        ETRY(synth_mat(e, e->wqkv[i], mix(seed, l * 8 + 1), tmp, tmp_n));
        ETRY(synth_mat(e, e->wo[i], mix(seed, l * 8 + 2), tmp, tmp_n));
        ETRY(synth_mat(e, e->w13[i], mix(seed, l * 8 + 3), tmp, tmp_n));
        ETRY(synth_mat(e, e->w2[i], mix(seed, l * 8 + 4), tmp, tmp_n));
    }
    if (e->has_embed) ETRY(synth_mat(e, e->emb, mix(seed, 1ull << 40), tmp, tmp_n));
    if (e->has_head) {
        ETRY(leap::eng::synth_normal(e->stream, e->rms_final, c.dim, 0, 0.f, 1.f));
        // a tied classifier on a stage without the embedding regenerates it
        if (e->wcls.f != e->emb.f || e->wcls.q != e->emb.q)
            ETRY(synth_mat(e, e->wcls, mix(seed, c.shared_classifier ? (1ull << 40) : (1ull << 41)),
                           tmp, tmp_n));
    }
    ETRY(leap::cuda_status(cudaStreamSynchronize(e->stream), "synthesize"));
    return LEAP_OK;
}

// ---- forward pieces ------------------------------------------------------------
using namespace leap::eng;

int linear_vec(leap_engine *e, float *y, const float *x, const Mat &w, int row0, int rows,
               const float *res) {
    const int n = w.cols;
    if (w.f) return gemv_f32(e->stream, y, x, w.f + size_t(row0) * n, n, rows, res);
    return gemv_q8(e->stream, y, e->aq, e->as, w.q + size_t(row0) * n,
                   w.s + size_t(row0) * n / e->cfg.group_size, n, rows, res, e->attn->d_err);
}

int linear_mat(leap_engine *e, float *y, const float *x, const Mat &w, int row0, int rows, int T,
               const float *res) {
    const int n = w.cols;
    if (w.f) return gemm_f32(e->stream, y, x, w.f + size_t(row0) * n, n, rows, T, res);
    return gemm_q8(e->stream, y, e->baq, e->bas, w.q + size_t(row0) * n,
                   w.s + size_t(row0) * n / e->cfg.group_size, n, rows, T, res, e->attn->d_err);
}

// One token through the local layers (run_layer, FloatTransformer.cpp:384-749;
// W8A8: QuantizedTransformer.cpp:654-1012).
int layers_one(leap_engine *e, int pos, float *x) {
    const leap_model_config &c = e->cfg;
    const int dim = c.dim, hid = c.hidden_dim, kv = e->kv_dim;
    const bool q8 = c.quantized;
    // FP32: the projections of a normalised x form the norm in the GEMV's
    // prologue (gemv_f32 with the norm weight); W8A8 projections whose input
    // is normalised or freshly computed take it in fp32 and quantize (and
    // normalise) it in the GEMV's prologue (gemv_q8_fused)
    auto norm_vec = [&](float *y, const float *nw, const Mat &w, int rows) {
        return gemv_f32(e->stream, y, x, w.f, w.cols, rows, nullptr, nw, e->xb);
    };
    auto fused = [&](float *y, const float *in, const float *nw, const Mat &w, int rows,
                     const float *res) {
        return gemv_q8_fused(e->stream, y, in, nw, e->aq, e->as, w.q, w.s, w.cols, rows, res,
                             e->attn->d_err);
    };
    for (int i = 0; i < e->n_local; ++i) {
        if (q8) {
            ETRY(fused(e->qkv, x, e->rms_att + size_t(i) * dim, e->wqkv[i], dim + 2 * kv, nullptr));
        } else {
            ETRY(norm_vec(e->qkv, e->rms_att + size_t(i) * dim, e->wqkv[i], dim + 2 * kv));
        }
        ETRY(leap_attn_decode(e->attn, i, pos, e->qkv, e->qkv + dim, e->qkv + dim + kv, e->att));
        if (q8)
            ETRY(fused(x, e->att, nullptr, e->wo[i], dim, x));  // x += wo . q(att)
        else
            ETRY(linear_vec(e, x, e->att, e->wo[i], 0, dim, x));  // x += wo . att
        if (q8) {
            ETRY(fused(e->h13, x, e->rms_ffn + size_t(i) * dim, e->w13[i], 2 * hid, nullptr));
        } else {
            ETRY(norm_vec(e->h13, e->rms_ffn + size_t(i) * dim, e->w13[i], 2 * hid));
        }
        if (q8)
            ETRY(silu_mul_quantize(e->stream, e->aq, e->as, e->h13, e->h13 + hid, hid));
        else
            ETRY(silu_mul(e->stream, e->h13, e->h13 + hid, hid));
        ETRY(linear_vec(e, x, e->h13, e->w2[i], 0, dim, x));  // x += w2 . h
    }
    return LEAP_OK;
}

// A prompt chunk of T tokens at pos0.. through the local layers: the same
// arithmetic per token, with the projections as GEMMs and causal attention.
int layers_chunk(leap_engine *e, int pos0, int T, float *x) {
    const leap_model_config &c = e->cfg;
    const int dim = c.dim, hid = c.hidden_dim, kv = e->kv_dim, gs = c.group_size;
    const bool q8 = c.quantized;
    auto norm = [&](const float *w) {
        return q8 ? rmsnorm_quantize(e->stream, e->baq, e->bas, x, w, T, dim)
                  : rmsnorm(e->stream, e->bxb, x, w, T, dim);
    };
    for (int i = 0; i < e->n_local; ++i) {
        ETRY(norm(e->rms_att + size_t(i) * dim));
        ETRY(linear_mat(e, e->bq, e->bxb, e->wqkv[i], 0, dim, T, nullptr));
        ETRY(linear_mat(e, e->bk, e->bxb, e->wqkv[i], dim, kv, T, nullptr));
        ETRY(linear_mat(e, e->bv, e->bxb, e->wqkv[i], dim + kv, kv, T, nullptr));
        ETRY(leap_attn_prefill(e->attn, 0, i, pos0, T, e->bq, e->bk, e->bv, e->batt));
        if (q8) ETRY(quantize(e->stream, e->baq, e->bas, e->batt, size_t(T) * dim, gs));
        ETRY(linear_mat(e, x, e->batt, e->wo[i], 0, dim, T, x));
        ETRY(norm(e->rms_ffn + size_t(i) * dim));
        ETRY(linear_mat(e, e->bh1, e->bxb, e->w13[i], 0, hid, T, nullptr));
        ETRY(linear_mat(e, e->bh3, e->bxb, e->w13[i], hid, hid, T, nullptr));
        if (q8)
            ETRY(silu_mul_quantize(e->stream, e->baq, e->bas, e->bh1, e->bh3, size_t(T) * hid));
        else
            ETRY(silu_mul(e->stream, e->bh1, e->bh3, size_t(T) * hid));
        ETRY(linear_mat(e, x, e->bh1, e->w2[i], 0, dim, T, x));
    }
    return LEAP_OK;
}

int head(leap_engine *e, float *x, float *logits, int *token) {
    const leap_model_config &c = e->cfg;
    float *lg = logits ? logits : e->logits;
    if (c.quantized && !e->wcls.f) {
        // x is only consumed quantized (QuantizedTransformer.cpp:1056-1059):
        // norm and quantization in the classifier GEMV's prologue
        ETRY(gemv_q8_fused(e->stream, lg, x, e->rms_final, e->aq, e->as, e->wcls.q, e->wcls.s,
                           e->wcls.cols, c.vocab_size, nullptr, e->attn->d_err));
    } else {
        if (c.quantized)
            ETRY(rmsnorm_quantize(e->stream, e->aq, e->as, x, e->rms_final, 1, c.dim));
        else
            ETRY(rmsnorm(e->stream, x, x, e->rms_final, 1, c.dim));
        ETRY(linear_vec(e, lg, x, e->wcls, 0, c.vocab_size, nullptr));
    }
    if (token)
        ETRY(e->sampler ? leap::sampler_launch(e->sampler, e->stream, lg, token)
                        : argmax(e->stream, token, lg, c.vocab_size));
    return LEAP_OK;
}

}  // namespace

extern "C" {

int leap_engine_open(const char *path, int device, int layer_begin, int layer_end,
                     float rope_theta, int max_chunk, leap_engine **out) {
    leap::clear_error();
    if (!path || !out) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    *out = nullptr;
    Mapped m;
    m.fd = open(path, O_RDONLY);
    if (m.fd < 0) {
        leap::set_error("Couldn't open file %s", path);
        return LEAP_ERR_INVALID;
    }
    struct stat sb;
    if (fstat(m.fd, &sb) != 0 || sb.st_size < 28) {
        leap::set_error("cannot stat %s", path);
        return LEAP_ERR_INVALID;
    }
    m.size = size_t(sb.st_size);
    m.p = mmap(nullptr, m.size, PROT_READ, MAP_PRIVATE, m.fd, 0);
    if (m.p == MAP_FAILED) {
        leap::set_error("mmap failed for %s", path);
        return LEAP_ERR_INVALID;
    }
    madvise(m.p, m.size, MADV_SEQUENTIAL);
    madvise(m.p, m.size, MADV_WILLNEED);
    const unsigned char *b = static_cast<const unsigned char *>(m.p);
    leap_model_config cfg{};
    size_t hdr = 0;
    ETRY(parse_header(b, m.size, &cfg, &hdr));
    DevGuard g(device);
    leap_engine *e = nullptr;
    int st = begin(out, cfg, device, layer_begin, layer_end, max_chunk, &e);
    if (st == LEAP_OK) st = allocate(e);
    if (st == LEAP_OK) {
        Cursor cur{b + hdr, b + m.size};
        st = cfg.quantized ? load_q8(e, cur) : load_fp32(e, cur);
    }
    if (st == LEAP_OK) st = make_attention(e, rope_theta > 0.f ? rope_theta : 500000.f);
    if (st != LEAP_OK) {
        free_engine(e);
        return st;
    }
    *out = e;
    return LEAP_OK;
}

int leap_engine_synthetic(const leap_model_config *cfg, unsigned long long seed, int device,
                          int layer_begin, int layer_end, float rope_theta, int max_chunk,
                          leap_engine **out) {
    leap::clear_error();
    if (!cfg || !out) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(device);
    leap_engine *e = nullptr;
    int st = begin(out, *cfg, device, layer_begin, layer_end, max_chunk, &e);
    if (st == LEAP_OK) st = allocate(e);
    if (st == LEAP_OK) st = synthesize(e, seed);
    if (st == LEAP_OK) st = make_attention(e, rope_theta > 0.f ? rope_theta : 500000.f);
    if (st != LEAP_OK) {
        free_engine(e);
        return st;
    }
    *out = e;
    return LEAP_OK;
}

int leap_engine_destroy(leap_engine *e) {
    leap::clear_error();
    free_engine(e);
    return LEAP_OK;
}

int leap_engine_config(const leap_engine *e, leap_model_config *cfg, int *lb, int *le) {
    leap::clear_error();
    if (!e || !cfg) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    *cfg = e->cfg;
    if (lb) *lb = e->layer_begin;
    if (le) *le = e->layer_end;
    return LEAP_OK;
}

int leap_engine_device_bytes(const leap_engine *e, size_t *bytes) {
    if (!e || !bytes) {
        leap::set_error("null argument");
        return LEAP_ERR_INVALID;
    }
    *bytes = e->device_bytes;
    return LEAP_OK;
}

int leap_engine_set_stream(leap_engine *e, void *stream) {
    leap::clear_error();
    if (!e) {
        leap::set_error("null engine");
        return LEAP_ERR_INVALID;
    }
    e->stream = static_cast<cudaStream_t>(stream);
    return leap_ctx_set_stream(e->attn, stream);
}

int leap_engine_sync(leap_engine *e) {
    leap::clear_error();
    if (!e) {
        leap::set_error("null engine");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    ETRY(leap::cuda_status(cudaStreamSynchronize(e->stream), "engine sync"));
    return leap_sync(e->attn);
}

int leap_engine_clear_kv(leap_engine *e) {
    leap::clear_error();
    if (!e) {
        leap::set_error("null engine");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    return leap_kv_clear(e->attn);
}

int leap_engine_embed(leap_engine *e, const int *tokens, int n, float *x) {
    leap::clear_error();
    if (!e || !tokens || !x || n < 1 || n > e->max_chunk) {
        leap::set_error("embed: bad arguments (n %d, max_chunk %d)", n, e ? e->max_chunk : 0);
        return LEAP_ERR_INVALID;
    }
    if (!e->has_embed) {
        leap::set_error("embed: this engine's layer range does not start at layer 0");
        return LEAP_ERR_INVALID;
    }
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= e->cfg.vocab_size) {
            leap::set_error("token %d out of range", tokens[i]);
            return LEAP_ERR_INVALID;
        }
    DevGuard g(e->device);
    int *dtok = n == 1 ? e->tok_dev : e->btok;
    if (n == 1) {
        // pinned mirror: keep the previous copy from racing the host write
        ETRY(leap::cuda_status(cudaStreamSynchronize(e->stream), "embed sync"));
        e->h_tok[0] = tokens[0];
        ETRY(leap::cuda_status(cudaMemcpyAsync(dtok, e->h_tok, 4, cudaMemcpyHostToDevice, e->stream),
                               "embed tokens"));
    } else {
        ETRY(leap::cuda_status(
            cudaMemcpyAsync(dtok, tokens, size_t(n) * 4, cudaMemcpyHostToDevice, e->stream),
            "embed tokens"));
    }
    return embed(e->stream, x, e->emb.f, e->emb.q, e->emb.s, dtok, n, e->cfg.dim,
                 e->cfg.group_size, e->cfg.vocab_size, e->attn->d_err);
}

int leap_engine_embed_device(leap_engine *e, const int *tokens_dev, int n, float *x) {
    leap::clear_error();
    if (!e || !tokens_dev || !x || n < 1 || n > e->max_chunk) {
        leap::set_error("embed_device: bad arguments (n %d)", n);
        return LEAP_ERR_INVALID;
    }
    if (!e->has_embed) {
        leap::set_error("embed: this engine's layer range does not start at layer 0");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    return embed(e->stream, x, e->emb.f, e->emb.q, e->emb.s, tokens_dev, n, e->cfg.dim,
                 e->cfg.group_size, e->cfg.vocab_size, e->attn->d_err);
}

int leap_engine_layers(leap_engine *e, int pos0, int n, float *x) {
    leap::clear_error();
    if (!e || !x || n < 1 || n > e->max_chunk || pos0 < 0 || pos0 + n > e->cfg.seq_len) {
        leap::set_error("layers: bad arguments (pos0 %d, n %d)", pos0, n);
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    return n == 1 ? layers_one(e, pos0, x) : layers_chunk(e, pos0, n, x);
}

int leap_engine_head(leap_engine *e, float *x, float *logits, int *token) {
    leap::clear_error();
    if (!e || !x) {
        leap::set_error("head: bad arguments");
        return LEAP_ERR_INVALID;
    }
    if (!e->has_head) {
        leap::set_error("head: this engine's layer range does not end at the last layer");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    return head(e, x, logits, token);
}

int leap_engine_forward(leap_engine *e, int token, int pos, float *logits, int *next_token) {
    leap::clear_error();
    if (!e || !e->has_embed || !e->has_head) {
        leap::set_error("forward needs a single-stage engine (all layers)");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    ETRY(leap_engine_embed(e, &token, 1, e->x));
    ETRY(leap_engine_layers(e, pos, 1, e->x));
    ETRY(head(e, e->x, e->logits, e->argmax_dev));
    if (logits)
        ETRY(leap::cuda_status(cudaMemcpyAsync(logits, e->logits, size_t(e->cfg.vocab_size) * 4,
                                               cudaMemcpyDeviceToHost, e->stream),
                               "copy logits"));
    ETRY(leap::cuda_status(
        cudaMemcpyAsync(e->h_tok + 1, e->argmax_dev, 4, cudaMemcpyDeviceToHost, e->stream),
        "copy token"));
    ETRY(leap_engine_sync(e));
    if (next_token) *next_token = e->h_tok[1];
    return LEAP_OK;
}

int leap_engine_prefill(leap_engine *e, const int *tokens, int n, int pos0, int *next_token) {
    leap::clear_error();
    if (!e || !e->has_embed || !e->has_head || !tokens || n < 1 || pos0 < 0 ||
        pos0 + n > e->cfg.seq_len) {
        leap::set_error("prefill needs a single-stage engine and a prompt that fits seq_len");
        return LEAP_ERR_INVALID;
    }
    DevGuard g(e->device);
    const int dim = e->cfg.dim;
    for (int c0 = 0; c0 < n; c0 += e->max_chunk) {
        const int nc = (n - c0) < e->max_chunk ? (n - c0) : e->max_chunk;
        ETRY(leap_engine_embed(e, tokens + c0, nc, e->bx));
        ETRY(leap_engine_layers(e, pos0 + c0, nc, e->bx));
        if (c0 + nc == n)
            ETRY(leap::cuda_status(cudaMemcpyAsync(e->x, e->bx + size_t(nc - 1) * dim, size_t(dim) * 4,
                                                   cudaMemcpyDeviceToDevice, e->stream),
                                   "last row"));
    }
    ETRY(head(e, e->x, e->logits, e->argmax_dev));
    ETRY(leap::cuda_status(
        cudaMemcpyAsync(e->h_tok + 1, e->argmax_dev, 4, cudaMemcpyDeviceToHost, e->stream),
        "copy token"));
    ETRY(leap_engine_sync(e));
    if (next_token) *next_token = e->h_tok[1];
    return LEAP_OK;
}


// ---- support ops, one kernel each ------------------------------------------------
int leap_op_rmsnorm(void *stream, float *o, const float *x, const float *w, int rows, int dim) {
    leap::clear_error();
    if (!o || !x || !w || rows < 1 || dim < 1) {
        leap::set_error("rmsnorm: bad arguments");
        return LEAP_ERR_INVALID;
    }
    return rmsnorm(static_cast<cudaStream_t>(stream), o, x, w, rows, dim);
}

int leap_op_rmsnorm_quantize(void *stream, int8_t *q, float *s, const float *x, const float *w,
                             int rows, int dim) {
    leap::clear_error();
    if (!q || !s || !x || !w || rows < 1 || dim < 64 || dim % 64) {
        leap::set_error("rmsnorm_quantize: bad arguments (dim %d must be a multiple of 64)", dim);
        return LEAP_ERR_INVALID;
    }
    return rmsnorm_quantize(static_cast<cudaStream_t>(stream), q, s, x, w, rows, dim);
}

int leap_op_quantize(void *stream, int8_t *q, float *s, const float *x, long long n, int gs) {
    leap::clear_error();
    if (!q || !s || !x || n < 1 || gs < 1 || n % gs) {
        leap::set_error("quantize: n %lld must be a positive multiple of gs %d", n, gs);
        return LEAP_ERR_INVALID;
    }
    return quantize(static_cast<cudaStream_t>(stream), q, s, x, size_t(n), gs);
}

int leap_op_matmul(void *stream, float *y, const float *x, const float *w, int n, int d, int T,
                   const float *res) {
    leap::clear_error();
    if (!y || !x || !w || n < 4 || n % 4 || d < 1 || T < 1) {
        leap::set_error("matmul: bad arguments (n %d, d %d, T %d)", n, d, T);
        return LEAP_ERR_INVALID;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    return T == 1 ? gemv_f32(st, y, x, w, n, d, res) : gemm_f32(st, y, x, w, n, d, T, res);
}

int leap_op_qmatmul(void *stream, float *y, const int8_t *xq, const float *xs, const int8_t *wq,
                    const float *ws, int n, int d, int T, int gs, const float *res) {
    leap::clear_error();
    if (!y || !xq || !xs || !wq || !ws || gs != 64 || n < 64 || n % 64 || d < 1 || T < 1) {
        leap::set_error("qmatmul: bad arguments (n %d, d %d, T %d, gs %d; gs must be 64)", n, d, T,
                        gs);
        return LEAP_ERR_INVALID;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    return T == 1 ? gemv_q8(st, y, xq, xs, wq, ws, n, d, res)
                  : gemm_q8(st, y, xq, xs, wq, ws, n, d, T, res);
}

int leap_op_matmul_fused(void *stream, float *y, const float *x, const float *nw, const float *w,
                         int n, int d, const float *res) {
    leap::clear_error();
    if (!y || !x || !w || n < 4 || n % 4 || d < 1) {
        leap::set_error("matmul_fused: bad arguments (n %d, d %d)", n, d);
        return LEAP_ERR_INVALID;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the normalised row of the unfused route, stream-ordered on `st`
    void *xb = nullptr;
    if (nw)
        ETRY(leap::cuda_status(cudaMallocAsync(&xb, size_t(n) * 4, st),
                               "cudaMallocAsync(matmul_fused)"));
    const int rc = gemv_f32(st, y, x, w, n, d, res, nw, static_cast<float *>(xb));
    if (xb) cudaFreeAsync(xb, st);
    return rc;
}

int leap_op_qmatmul_fused(void *stream, float *y, const float *x, const float *nw,
                          const int8_t *wq, const float *ws, int n, int d, const float *res) {
    leap::clear_error();
    if (!y || !x || !wq || !ws || n < 64 || n % 64 || d < 1 ||
        (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(nw) & 15)) {
        leap::set_error("qmatmul_fused: bad arguments (n %d, d %d; x, nw 16-byte aligned)", n, d);
        return LEAP_ERR_INVALID;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    // (q, s) of the unfused route, stream-ordered on `st`
    void *aq = nullptr, *as = nullptr;
    ETRY(leap::cuda_status(cudaMallocAsync(&aq, size_t(n), st), "cudaMallocAsync(qmatmul_fused)"));
    if (int rc = leap::cuda_status(cudaMallocAsync(&as, size_t(n / 64) * 4, st),
                                   "cudaMallocAsync(qmatmul_fused)")) {
        cudaFreeAsync(aq, st);
        return rc;
    }
    const int rc = gemv_q8_fused(st, y, x, nw, static_cast<int8_t *>(aq), static_cast<float *>(as),
                                 wq, ws, n, d, res);
    cudaFreeAsync(aq, st);
    cudaFreeAsync(as, st);
    return rc;
}

int leap_op_set_q8_gemv(int impl) {
    leap::clear_error();
    if (impl < 0 || impl > 2) {
        leap::set_error("q8 gemv impl %d (0 sliced, 1 register-staged, 2 persistent bulk-copy)", impl);
        return LEAP_ERR_INVALID;
    }
    leap::eng::g_q8_slice = impl == 0;
    leap::eng::g_q8_tma = impl == 2;
    return LEAP_OK;
}

int leap_op_set_q8_gemm(int impl) {
    leap::clear_error();
    if (impl < 0 || impl > 1) {
        leap::set_error("q8 gemm impl %d (0 CUDA-core dp4a, 1 tcgen05 kind::i8)", impl);
        return LEAP_ERR_INVALID;
    }
    leap::eng::g_q8_gemm_tc = impl == 1;
    return LEAP_OK;
}

int leap_engine_set_sampler(leap_engine *e, leap_sampler *s) {
    leap::clear_error();
    if (!e) {
        leap::set_error("null engine");
        return LEAP_ERR_INVALID;
    }
    e->sampler = s;
    return LEAP_OK;
}

int leap_op_argmax(void *stream, int *token, const float *v, int n) {
    leap::clear_error();
    if (!token || !v || n < 1) {
        leap::set_error("argmax: bad arguments");
        return LEAP_ERR_INVALID;
    }
    return argmax(static_cast<cudaStream_t>(stream), token, v, n);
}

}  // extern "C"
