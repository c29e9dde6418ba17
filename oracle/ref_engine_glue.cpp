// ref_engine_glue.cpp — a C surface over the UNMODIFIED reference engine.
//
// TEST INFRASTRUCTURE ONLY (end-to-end checker and CPU baseline).
//
// Links against the reference's own src/inference/{FloatTransformer,
// QuantizedTransformer,TransformerFactory,Sampler}.cpp compiled by
// oracle/Makefile.  The reference's CLI (src/inference/main.cpp) needs
// CLI11, which is fetched from the network at configure time and is not
// available, so this glue stands in for it: it drives the public API
// Transformer::create (src/inference/TransformerFactory.cpp:59) and
// forward(token, pos) (src/inference/Transformer.h:56) exactly as
// generate() does (src/inference/main.cpp:64-108).
#include <cstring>
#include <exception>
#include <memory>
#include <string>

#include "Sampler.h"
#include "Transformer.h"

namespace {
thread_local std::string g_err;
}

extern "C" {

const char *leapref_engine_error() { return g_err.c_str(); }

void *leapref_engine_create(const char *path) {
    try {
        auto t = Inference::Transformer::create(path);
        return t.release();
    } catch (const std::exception &e) {
        g_err = e.what();
        return nullptr;
    }
}

void leapref_engine_destroy(void *h) {
    delete static_cast<Inference::Transformer *>(h);
}

// Config fields in the order of src/inference/Config.h:5-13.
void leapref_engine_config(void *h, int *out7) {
    const auto &c = static_cast<Inference::Transformer *>(h)->config;
    out7[0] = c.dim;
    out7[1] = c.hidden_dim;
    out7[2] = c.n_layers;
    out7[3] = c.n_heads;
    out7[4] = c.n_kv_heads;
    out7[5] = c.vocab_size;
    out7[6] = c.seq_len;
}

// forward(token, pos) of the single-process engine; returns the engine-owned
// logits[vocab] or null on error.
const float *leapref_engine_forward(void *h, int token, int pos) {
    try {
        return static_cast<Inference::Transformer *>(h)->forward(token, pos);
    } catch (const std::exception &e) {
        g_err = e.what();
        return nullptr;
    }
}

void leapref_engine_clear(void *h) {
    static_cast<Inference::Transformer *>(h)->clear_kv_cache();
}

// Greedy sampling through the reference Sampler (temperature 0 takes the
// argmax branch, src/inference/Sampler.cpp:199-202).
int leapref_sample_argmax(const float *logits, int vocab) {
    Inference::Sampler s(vocab, 0.0f, 0.9f, 0ULL);
    std::unique_ptr<float[]> tmp(new float[vocab]);
    std::memcpy(tmp.get(), logits, sizeof(float) * vocab);
    return s.sample(tmp.get());
}

// One draw of the reference Sampler (src/inference/Sampler.cpp:187-232) with
// the given temperature and top-p, its RNG state starting at *state.  The
// Sampler keeps its state private, so the caller advances *state itself
// (one random_f32 per draw when temperature != 0, src/inference/Utils.h:18-29).
int leapref_sample(const float *logits, int vocab, float temperature, float topp,
                   unsigned long long state) {
    Inference::Sampler s(vocab, temperature, topp, state);
    std::unique_ptr<float[]> tmp(new float[vocab]);
    std::memcpy(tmp.get(), logits, sizeof(float) * vocab);
    return s.sample(tmp.get());
}

}  // extern "C"
