// ref_binding_attn.cpp — the reference engine's attention block bound to the
// C ABI of libleap_b200.so (include/leap_b200.h).
//
// TEST INFRASTRUCTURE: it shows that the boundary is a drop-in for the
// reference's own engine.  oracle/Makefile (target `binding`) copies the
// reference's src/inference/FloatTransformer.cpp and QuantizedTransformer.cpp
// into oracle/_ref/binding/, replacing each run_layer's attention block
// (FloatTransformer.cpp:404-662, QuantizedTransformer.cpp:680-923: RoPE,
// scores, softmax, weighted V sum) by one call of leap_binding_attention
// below, and links the result with the reference's unmodified
// TransformerFactory.cpp and Sampler.cpp.  Everything else of the engine
// (weights, projections, the FFN, sampling) is the reference's own code.
//
// At the call the engine's projections have written the token's q into
// state.q and its un-rotated k and v into its host cache row `pos`
// (FloatTransformer.cpp:397-402); leap_attn_decode_host rotates q and k with
// the engine's own RoPE table (handed over when the context is made),
// appends k and v to the context's device cache and writes the attention
// output into state.xb, which the engine's wo projection reads next
// (:664).  Errors become std::runtime_error, the reference's convention.
#include <map>
#include <mutex>
#include <stdexcept>
#include <string>
#include <tuple>

#include "leap_b200.h"

namespace {

// One device context per engine object (and shape, and RoPE table).
using Key = std::tuple<const void *, int, int, int, int, int, const float *>;
std::mutex g_mu;
std::map<Key, leap_ctx *> g_ctx;

void check(int st) {
    if (st != LEAP_OK) throw std::runtime_error(std::string("leap_b200: ") + leap_last_error());
}

}  // namespace

extern "C" void leap_binding_attention(const void *engine, int n_layers, int n_heads,
                                       int n_kv_heads, int head_dim, int seq_len,
                                       const float *rope_cos, const float *rope_sin, int layer,
                                       int pos, const float *q, const float *k, const float *v,
                                       float *out) {
    leap_ctx *ctx = nullptr;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        const Key key{engine, n_layers, n_heads, n_kv_heads, head_dim, seq_len, rope_cos};
        auto it = g_ctx.find(key);
        if (it == g_ctx.end()) {
            leap_ctx_desc d{};
            d.n_layers = n_layers;
            d.layer0 = 0;
            d.n_heads = n_heads;
            d.n_kv_heads = n_kv_heads;
            d.head_dim = head_dim;
            d.max_seq = seq_len;
            d.max_batch = 1;
            d.device = 0;
            d.rope_cos = rope_cos;  // the engine's own table (precompute_freqs)
            d.rope_sin = rope_sin;
            check(leap_ctx_create(&d, &ctx));
            g_ctx.emplace(key, ctx);
        } else {
            ctx = it->second;
        }
    }
    check(leap_attn_decode_host(ctx, layer, pos, q, k, v, out));
}
