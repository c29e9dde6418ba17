/*
 * leap_b200.h — C ABI of the B200 attention engine for LEAP.
 *
 * LEAP (Harikeshav-R/LEAP) runs its GQA attention block inline in the private
 * `run_layer()` of its CPU engines:
 *   src/inference/FloatTransformer.cpp:404-662      (FP32 engine)
 *   src/inference/QuantizedTransformer.cpp:680-923  (W8A8 engine, same math)
 * That block is: RoPE on q and on the new k row of the cache, the new k/v rows
 * written into the FP32 KV cache, scores q.k/sqrt(head_size) over positions
 * 0..pos, softmax, and the softmax-weighted sum of V rows into `xb`.
 *
 * This header is the drop-in boundary a LEAP engine binds to replace that
 * block: plain C types, device pointers, an `int` status on every call
 * (0 = ok) and a thread-local message from leap_last_error().  A C++ caller
 * turns a non-zero status into std::runtime_error, which is the reference's
 * own error convention (src/inference/main.cpp:498-501).
 *
 * Threading: one caller thread per context, like the reference engine (its
 * run state is shared, src/inference/FloatTransformer.h:24-37).  Work is
 * stream-ordered on the context's stream; *_host entry points block.
 *
 * Device KV-cache layout (owned by the context, FP32):
 *   [slot][layer][kv_head][max_seq_padded][head_dim]
 * i.e. each (slot, layer, kv_head) is one contiguous stream of rows, so one
 * bulk copy moves a whole tile of positions.  The reference keeps
 * [layer][pos][kv_head][head_dim] (src/inference/FloatTransformer.cpp:50-51,
 * :396); leap_kv_write/leap_kv_read convert from/to that layout.
 */
#ifndef LEAP_B200_H
#define LEAP_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LEAP_API __attribute__((visibility("default")))
#else
#define LEAP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LEAP_OK 0
#define LEAP_ERR_INVALID 1   /* bad argument (shape, range, null pointer)     */
#define LEAP_ERR_CUDA 2      /* a CUDA runtime call failed                     */
#define LEAP_ERR_DEVICE 3    /* a kernel reported an error (bounded wait hit)  */
#define LEAP_ERR_NOMEM 4     /* device allocation failed                       */
#define LEAP_ERR_COMM 5      /* a stage-to-stage transfer failed or timed out  */

typedef struct leap_ctx leap_ctx; /* opaque */

/*
 * Engine description.  Mirrors the reference `Config`
 * (src/inference/Config.h:5-13) for the fields attention needs, plus the
 * layer range this context holds (the pipeline split of
 * src/inference/Transformer.h:17-23) and the number of sequence slots.
 */
typedef struct leap_ctx_desc {
    int n_layers;        /* layers whose KV cache this context holds            */
    int layer0;          /* global index of local layer 0 (pipeline stages)     */
    int n_heads;         /* query heads                                          */
    int n_kv_heads;      /* key/value heads; n_heads % n_kv_heads == 0           */
    int head_dim;        /* 64 or 128                                            */
    int max_seq;         /* cache capacity per slot (reference seq_len)          */
    int max_batch;       /* sequence slots (1 for the single-stream engine)      */
    int device;          /* CUDA device ordinal                                  */
    /* Host RoPE table [max_seq][head_dim/2], as the reference precomputes it
     * (src/inference/FloatTransformer.cpp:56-72).  The engine passes its own
     * table, so the device rotation uses exactly the same cos/sin values.   */
    const float *rope_cos;
    const float *rope_sin;
} leap_ctx_desc;

/* Last error message of the calling thread ("" if none). */
LEAP_API const char *leap_last_error(void);

/* Library version string. */
LEAP_API const char *leap_version(void);

/*
 * The reference RoPE table, host side: for even i < head_dim,
 *   cos/sin(pos * freq_i)  at [pos][i/2],  pos < seq_len.
 * Replaces FloatTransformer::precompute_freqs
 * (src/inference/FloatTransformer.cpp:56-72).  The source writes
 * freq = 1/pow(theta, i/hd); the reference's release build (-ffast-math)
 * evaluates it as expf(-(i/hd) * logf(theta)), and this function computes
 * that form with the C library's float functions, so its table equals the
 * compiled reference's bit for bit.  The shipped reference hard-codes
 * theta = 500000 (:65).
 */
LEAP_API int leap_rope_table(int seq_len, int head_dim, float theta,
                             float *rope_cos, float *rope_sin);

/*
 * Create / destroy a context: device KV cache (zeroed), RoPE table, split-KV
 * scratch and a non-blocking stream on desc->device.
 * Replaces FloatTransformer::init_run_state + precompute_freqs
 * (src/inference/FloatTransformer.cpp:39-72) for the attention state.
 */
LEAP_API int leap_ctx_create(const leap_ctx_desc *desc, leap_ctx **out);
LEAP_API int leap_ctx_destroy(leap_ctx *ctx);

/* Use `stream` (a cudaStream_t; NULL = the CUDA default stream, as
 * everywhere in CUDA) for all following work of this context. */
LEAP_API int leap_ctx_set_stream(leap_ctx *ctx, void *stream);

/* Go back to the context's own non-blocking stream (the initial state). */
LEAP_API int leap_ctx_use_own_stream(leap_ctx *ctx);

/*
 * Launch overlap (default on).  A decode launch may start streaming its
 * layer's K/V cache into shared memory while the previous kernel on the
 * stream is still finishing (programmatic dependent launch); it reads its
 * q/k/v inputs and writes anything only after that kernel has completed.
 * The context turns the overlap off by itself for a launch whose layer the
 * previous operation of this context wrote (or after leap_kv_write,
 * leap_kv_clear or a stream change), so results never depend on it.
 */
LEAP_API int leap_set_overlap(leap_ctx *ctx, int enable);

/*
 * Decode kernel selection (results agree within the decode tolerance):
 *   0 = auto: one sequence uses a 16-CTA thread-block cluster per kv head
 *       whose split-KV reduction runs in distributed shared memory, when
 *       every head's cluster fits on the device at once; otherwise the
 *       split-KV kernel (128-thread CTAs, two per SM) whose last CTA per
 *       (sequence, kv head) combines the partials;
 *   1 = that split-KV kernel;  2 = cluster kernel;
 *   3 = split-KV kernel with 256-thread CTAs, one per SM;
 *   4 = the split-KV kernel of 1 publishing its partials only, combined by a
 *       second launch (one CTA per query head) that starts under
 *       programmatic dependent launch.
 */
LEAP_API int leap_set_decode_impl(leap_ctx *ctx, int impl);

/* Number of 16-CTA decode clusters the device holds at once. */
LEAP_API int leap_decode_cluster_capacity(const leap_ctx *ctx, int *n);

/* Block until the context's queued work is done; reports kernel errors. */
LEAP_API int leap_sync(leap_ctx *ctx);

/* Bytes of device memory held by the context. */
LEAP_API int leap_ctx_device_bytes(const leap_ctx *ctx, size_t *bytes);

/*
 * Zero every slot's K and V cache.  Replaces
 * FloatTransformer::clear_kv_cache (src/inference/FloatTransformer.cpp:74-77).
 */
LEAP_API int leap_kv_clear(leap_ctx *ctx);

/*
 * Copy rows [pos0, pos0+n_pos) of (slot, layer) into / out of the cache.
 * `k`, `v` are in the reference row layout [n_pos][n_kv_heads][head_dim]
 * (src/inference/FloatTransformer.cpp:396-398).  from_host / to_host select
 * host or device pointers.  Used to load a KV snapshot, and by tests.
 */
LEAP_API int leap_kv_write(leap_ctx *ctx, int slot, int layer, int pos0, int n_pos,
                  const float *k, const float *v, int from_host);
LEAP_API int leap_kv_read(leap_ctx *ctx, int slot, int layer, int pos0, int n_pos,
                 float *k, float *v, int to_host);

/*
 * Decode attention for one token of slot 0, fused:
 *   RoPE(q), RoPE(k_new)                 FloatTransformer.cpp:404-494
 *   cache[layer][pos] <- (rot k_new, v)  FloatTransformer.cpp:397-402
 *   out = softmax(q.K^T/sqrt(hd)) . V    FloatTransformer.cpp:496-662
 * over positions 0..pos inclusive.
 *   q     [n_heads][head_dim]     (un-rotated, as the wq matmul leaves it)
 *   k_new [n_kv_heads][head_dim]  (un-rotated)
 *   v_new [n_kv_heads][head_dim]
 *   out   [n_heads][head_dim]     (the reference's `xb`)
 * Device pointers, 16-byte aligned; asynchronous on the context stream.
 */
LEAP_API int leap_attn_decode(leap_ctx *ctx, int layer, int pos, const float *q,
                     const float *k_new, const float *v_new, float *out);

/*
 * The same call with HOST pointers: the reference-facing form, for an
 * engine whose activations live in host memory like the reference's
 * run_layer.  Copies in, runs, copies out and blocks until `out` is ready
 * (inputs staged through pinned memory that a small kernel reads directly,
 * chained to the decode kernel by programmatic dependent launch; the decode
 * kernel stores the output into that pinned memory itself).
 */
LEAP_API int leap_attn_decode_host(leap_ctx *ctx, int layer, int pos, const float *q,
                          const float *k_new, const float *v_new, float *out);

/*
 * Ragged batched decode: one new token for each of n_seq sequences, each in
 * its own cache slot at its own position.  Semantics = leap_attn_decode per
 * sequence (the reference has no batched path; it is the reference block
 * applied to each sequence).
 *   slots[i], positions[i]: HOST int arrays of length n_seq
 *   q [n_seq][n_heads][hd], k_new/v_new [n_seq][n_kv][hd], out like q.
 * Slots must be distinct within one call.
 */
LEAP_API int leap_attn_decode_batched(leap_ctx *ctx, int layer, int n_seq,
                             const int *slots, const int *positions,
                             const float *q, const float *k_new,
                             const float *v_new, float *out);

/*
 * Causal prefill of n_tok prompt tokens of `slot` starting at pos0.
 * Semantics = the reference decode block run for pos = pos0 .. pos0+n_tok-1
 * in order (the reference feeds prompts token by token,
 * src/inference/main.cpp:80-89): each token's k/v are rotated and appended,
 * and token i attends to cache rows 0..pos0+i.
 *   q [n_tok][n_heads][hd], k/v [n_tok][n_kv][hd] (un-rotated), out like q.
 */
LEAP_API int leap_attn_prefill(leap_ctx *ctx, int slot, int layer, int pos0, int n_tok,
                      const float *q, const float *k, const float *v,
                      float *out);

/*
 * Decode attention that allocates nothing.  (No counterpart in the
 * reference: LEAP's CPU engine owns all its memory in std::vectors.)
 *
 * For callers that cannot call cudaMalloc: a host whose device memory is all
 * owned by one allocator (a framework's caching allocator) or by a fixed arena
 * reserved at start-up, or an embedding that is not allowed to touch CUDA's
 * allocator.  Such a caller cannot create
 * a leap_ctx (which allocates the cache and scratch), so this entry point
 * takes everything as caller-owned device memory and keeps its own scratch
 * (split-KV partials, combine tickets, an error word) in a 4 MiB array
 * compiled into the library, which every GPU that loads the library holds
 * until the process exits.  It calls no cudaMalloc, cudaFree or other
 * allocating routine.
 *
 * Same computation as leap_attn_decode for one token at `pos`, with the
 * caller's cache: k_cache/v_cache are [n_kv_heads][head_stride] floats, row t
 * of kv head h at k_cache + h*head_stride + t*head_dim, rows 0..pos-1
 * already rotated; row pos is written (rotated k, raw v).  rope_cos/rope_sin
 * are device tables [>= pos+1][head_dim/2] (leap_rope_table's values).  All
 * pointers device, 16-byte aligned; head_stride a multiple of 4 floats and
 * >= (pos+1)*head_dim.  Runs on `stream` (NULL = default stream).
 *
 * The first call on a device looks up the array's device address (once per
 * device), so make that first call before any stream capture.  Every call
 * shares the one array and clears the part of it that must start at zero;
 * calls that overlap on the GPU (different streams, or different host
 * threads) race on it and must not be issued.  A context too long for the
 * scratch (more split-KV partials than fit in 4 MiB, about 64k positions
 * for 8 kv heads of 4x128) is rejected with LEAP_ERR_INVALID and a message.
 *
 * The kernel's copy waits are bounded (about two seconds, never reached on a
 * healthy GPU).  A wait that gives up leaves `out` unwritten for the heads
 * it served and cannot be reported through this entry point; callers that
 * need that report use leap_attn_decode.
 */
LEAP_API int leap_attn_decode_noalloc(void *stream, int n_heads, int n_kv_heads,
                                      int head_dim, int pos,
                                      const float *rope_cos,
                                      const float *rope_sin, float *k_cache,
                                      float *v_cache, long long head_stride,
                                      const float *q, const float *k_new,
                                      const float *v_new, float *out);

/* ======================================================================
 * The forward pass around attention (decode-step driver).
 *
 * leap_engine holds the weights of a contiguous layer range of a LEAP model
 * on one GPU — all layers for the single-process engine, or one pipeline
 * stage's range (the split of src/inference/Transformer.h:17-23) — plus
 * that range's KV cache.  It reads the reference's own .bin files (v0/v1
 * FP32, v2 W8A8: src/inference/TransformerFactory.cpp:59-135, weight order
 * of FloatTransformer.cpp:947-978 / QuantizedTransformer.cpp:102-134) and
 * runs, per layer, what run_layer does (FloatTransformer.cpp:384-749,
 * QuantizedTransformer.cpp:654-1012) on sm_100a kernels.
 * ====================================================================== */

typedef struct leap_model_config {
    /* src/inference/Config.h:5-13 */
    int dim, hidden_dim, n_layers, n_heads, n_kv_heads, vocab_size, seq_len;
    int quantized;         /* 0: FP32 (.bin v0/v1); 1: W8A8 (.bin v2)       */
    int group_size;        /* W8A8 quantization group (v2 header)            */
    int shared_classifier; /* classifier tied to the token embedding         */
} leap_model_config;

typedef struct leap_engine leap_engine; /* opaque */

/*
 * Load layers [layer_begin, layer_end) of the model file at `path` onto
 * `device` (layer_end = -1: to the last layer).  The range holding layer 0
 * also holds the embedding; the range holding the last layer also holds the
 * final norm and the classifier.  rope_theta 0 = the reference's hard-coded
 * 500000 (FloatTransformer.cpp:65).  max_chunk = the most prompt tokens one
 * leap_engine_layers call takes (0 = 512).
 */
LEAP_API int leap_engine_open(const char *path, int device, int layer_begin,
                              int layer_end, float rope_theta, int max_chunk,
                              leap_engine **out);

/* Same, with N(0, 0.02) weights (RMSNorm weights 1) generated on the device
 * from `seed` — for shapes too large to write to a file. */
LEAP_API int leap_engine_synthetic(const leap_model_config *cfg,
                                   unsigned long long seed, int device,
                                   int layer_begin, int layer_end,
                                   float rope_theta, int max_chunk,
                                   leap_engine **out);

LEAP_API int leap_engine_destroy(leap_engine *e);
LEAP_API int leap_engine_config(const leap_engine *e, leap_model_config *cfg,
                                int *layer_begin, int *layer_end);
LEAP_API int leap_engine_device_bytes(const leap_engine *e, size_t *bytes);
LEAP_API int leap_engine_set_stream(leap_engine *e, void *stream);
LEAP_API int leap_engine_sync(leap_engine *e);

/* Transformer::clear_kv_cache (FloatTransformer.cpp:74-77). */
LEAP_API int leap_engine_clear_kv(leap_engine *e);

/* Stage operations on device buffers (asynchronous on the engine stream):
 *   embed:  x[n][dim] <- embedding rows of tokens[0..n) (host ints)
 *   embed_device: the same from device ints (no host round trip, so a
 *           pipeline's first stage can embed the token the last stage sent;
 *           ids outside [0, vocab) read row 0 and set the engine's error,
 *           reported by leap_engine_sync)
 *   layers: this engine's layers on x[n][dim] in place, for positions
 *           pos0..pos0+n-1 (n = 1 is the decode step; n > 1 a prompt chunk,
 *           n <= max_chunk)
 *   head:   final RMSNorm of x[dim] (in place, as the reference), classifier
 *           into logits[vocab] (device, or NULL) and the greedy token into
 *           *token (device int, or NULL). */
LEAP_API int leap_engine_embed(leap_engine *e, const int *tokens, int n, float *x);
LEAP_API int leap_engine_embed_device(leap_engine *e, const int *tokens_dev, int n, float *x);
LEAP_API int leap_engine_layers(leap_engine *e, int pos0, int n, float *x);
LEAP_API int leap_engine_head(leap_engine *e, float *x, float *logits, int *token);

/* Transformer::forward(token, pos) of a single-stage engine
 * (FloatTransformer.cpp:751-797): logits[vocab] into host memory (or
 * NULL) and the greedy next token (Sampler at temperature 0,
 * src/inference/Sampler.cpp:199-202) into *next_token (or NULL). Blocks. */
LEAP_API int leap_engine_forward(leap_engine *e, int token, int pos,
                                 float *logits, int *next_token);

/* Prefill of n prompt tokens at pos0.. through a single-stage engine in
 * chunks of max_chunk; *next_token = greedy token after the last one. */
LEAP_API int leap_engine_prefill(leap_engine *e, const int *tokens, int n,
                                 int pos0, int *next_token);

/* Prefill kernel selection (for tests and benchmarks):
 *   0 = tensor-core 3xTF32, software-pipelined across warp roles
 *       (softmax, operand conversion and MMA issue overlap),
 *   1 = CUDA-core FP32 path,
 *   2 = tensor-core 3xTF32, one tile at a time (no overlap),
 *   3 = default: as 0 with the two correction products (hi*lo, lo*hi) in
 *       BF16 (kind::f16, K = 16): 40 instead of 60 tensor-core instructions
 *       per 32-key tile, about 2^-19 relative per product. */
LEAP_API int leap_set_prefill_impl(leap_ctx *ctx, int impl);

/* ---- support ops of the layer, one kernel each --------------------------
 * Device pointers, stream-ordered on `stream` (NULL = default stream).  The
 * engine above launches exactly these; they are exported so that each one
 * can be checked against the reference function it replaces. */

/* rows x rmsnorm over `dim` (FloatTransformer.cpp:79-214): o = w * x *
 * 1/sqrt(mean(x^2) + 1e-5).  o may equal x. */
LEAP_API int leap_op_rmsnorm(void *stream, float *o, const float *x,
                             const float *w, int rows, int dim);
/* rmsnorm followed by the activation quantize below, in one kernel (the
 * W8A8 engine consumes the normalised row only quantized,
 * QuantizedTransformer.cpp:925-951): q/s as leap_op_quantize with gs 64 of
 * the rows leap_op_rmsnorm would produce.  dim % 64 == 0. */
LEAP_API int leap_op_rmsnorm_quantize(void *stream, int8_t *q, float *s,
                                      const float *x, const float *w,
                                      int rows, int dim);
/* Activation quantize (QuantizedTransformer.cpp:338-357): per group of gs,
 * s = max|x| * (1/127), q = round(x / s).  n % gs == 0. */
LEAP_API int leap_op_quantize(void *stream, int8_t *q, float *s,
                              const float *x, long long n, int gs);
/* y[t][d] = W[d][n] . x[t] (+ res[t]) in FP32 for T tokens
 * (FloatTransformer.cpp:240-382 per token); T == 1 is the decode GEMV,
 * T > 1 the prompt-chunk GEMM.  res may equal y. */
LEAP_API int leap_op_matmul(void *stream, float *y, const float *x,
                            const float *w, int n, int d, int T,
                            const float *res);
/* W8A8 grouped GEMV/GEMM (QuantizedTransformer.cpp:359-652 per token):
 * y[t][i] = sum over groups g, in order, of (int32 dot of group g) *
 * ws[i][g] * xs[t][g]; gs == 64.  res may equal y. */
LEAP_API int leap_op_qmatmul(void *stream, float *y, const int8_t *xq,
                             const float *xs, const int8_t *wq,
                             const float *ws, int n, int d, int T, int gs,
                             const float *res);
/* The FP32 GEMV of a normalised vector, as the engine's decode step
 * launches it for wq;wk;wv and w1;w3 (FloatTransformer.cpp:397-402,
 * :663-669): y = W . rmsnorm(x, nw) (+ res) (nw != NULL; NULL: y = W . x +
 * res), the norm formed in the GEMV's prologue with leap_op_rmsnorm's
 * operation order: bit-identical to leap_op_rmsnorm followed by
 * leap_op_matmul with T == 1.  n % 4 == 0; res may equal y. */
LEAP_API int leap_op_matmul_fused(void *stream, float *y, const float *x,
                                  const float *nw, const float *w, int n,
                                  int d, const float *res);
/* The W8A8 GEMV of a freshly normalised or computed fp32 vector, as the
 * engine's decode step launches it for wq;wk;wv, wo, w1;w3 and the
 * classifier (QuantizedTransformer.cpp:680-683, :925-951, :1056-1059):
 * y = W . q(a) (+ res), a = rmsnorm(x, nw) for nw != NULL (leap_op_rmsnorm)
 * else a = x, q the 64-group quantization of leap_op_quantize.  The
 * persistent kernel quantizes (and normalises) in its prologue; results are
 * bit-identical to leap_op_rmsnorm_quantize / leap_op_quantize followed by
 * leap_op_qmatmul with T == 1.  x, nw 16-byte aligned; n % 64 == 0; res
 * may equal y. */
LEAP_API int leap_op_qmatmul_fused(void *stream, float *y, const float *x,
                                   const float *nw, const int8_t *wq,
                                   const float *ws, int n, int d,
                                   const float *res);
/* W8A8 GEMV kernel selection for T == 1 (process-wide; tests/benchmarks):
 * 0 = one row per lane with the row's groups sliced over lanes,
 * 1 = register-staged rows with 4-lane group shuffles,
 * 2 = persistent CTAs streaming 8-row x 2 KB items through a bulk-copy
 *     pipeline, warp-specialised (dot warps, a copy producer, a chain warp;
 *     the default).  All compute the same bits. */
LEAP_API int leap_op_set_q8_gemv(int impl);
/* W8A8 GEMM kernel selection for T > 1, the prompt chunks of
 * leap_engine_prefill / leap_op_qmatmul (process-wide; tests/benchmarks):
 * 0 = CUDA-core dp4a tiles, 1 = tcgen05 kind::i8 tensor-core tiles whose
 * int32 group dots feed the same ordered FP32 chain (the default; used where
 * n % 256 == 0 and the operands are 16-byte aligned).  Both compute the bits
 * of QuantizedTransformer.cpp:359-652. */
LEAP_API int leap_op_set_q8_gemm(int impl);
/* Greedy sampling (Sampler.cpp:20-120 at temperature 0): index of the
 * first maximum in the reference's scan order. */
LEAP_API int leap_op_argmax(void *stream, int *token, const float *v, int n);

/* ---- sampler (src/inference/Sampler.cpp, Utils.h:18-29) ------------------
 * The reference Sampler(vocab, temperature, topp, seed) on the GPU.  Each
 * leap_sampler_sample is one Sampler::sample(logits): temperature 0 ->
 * argmax; else softmax(logits / temperature) and a coin from the same
 * xorshift* state (advanced on the host, one draw per call), then
 * multinomial (topp <= 0 or >= 1) or top-p sampling.  Logits are device
 * memory and are not modified; the token is written to device memory,
 * stream-ordered.  Equal probabilities are taken in index order; a token can
 * differ from the reference's only when a running probability sum lies
 * within float rounding of the coin or of topp. */
typedef struct leap_sampler leap_sampler;
LEAP_API int leap_sampler_create(int vocab, float temperature, float topp,
                                 unsigned long long seed, int device, leap_sampler **out);
LEAP_API int leap_sampler_destroy(leap_sampler *s);
LEAP_API int leap_sampler_sample(leap_sampler *s, void *stream, const float *logits,
                                 int *token_dev);
/* The RNG state after the draws so far (the reference's rng_state). */
LEAP_API int leap_sampler_state(const leap_sampler *s, unsigned long long *state);

/* Tokens from leap_engine_forward / _head come from this sampler instead of
 * the greedy argmax (NULL restores argmax).  The engine does not own it. */
LEAP_API int leap_engine_set_sampler(leap_engine *e, leap_sampler *s);

/* ---- stage-to-stage transport (layer-range pipelines in one box) --------
 * Replaces the reference's ring transport between a master and its workers
 * (src/inference/FloatTransformer.cpp:772-793 and :800-946, TCP/UDP or the
 * kernel module; src/inference/Transformer.h:17-23) for GPUs of one node:
 * point-to-point NCCL sends over NVLink, ordered on the caller's stream.
 * One process per GPU.  NCCL is loaded at run time (the process's own copy
 * when it already has one).  Creation and every enqueue wait at most
 * `timeout_ms` (0 = 60 s); on a timeout the communicator is aborted and the
 * call returns LEAP_ERR_COMM. */
typedef struct leap_pp leap_pp; /* opaque */

/* Rank 0 creates the job's id (128 bytes) and hands it to every rank by any
 * host channel (a TCP store, an MPI broadcast, a file). */
LEAP_API int leap_pp_unique_id(void *id_out);
LEAP_API int leap_pp_init(const void *id, int rank, int world, int device,
                          int timeout_ms, leap_pp **out);
/* x[bytes] of this stage to stage rank+1 / from stage rank-1 (device
 * buffers; stream = cudaStream_t, NULL = default stream). */
LEAP_API int leap_pp_send_next(leap_pp *pp, const void *buf, size_t bytes,
                               void *stream);
LEAP_API int leap_pp_recv_prev(leap_pp *pp, void *buf, size_t bytes,
                               void *stream);
/* Any peer (the last stage returns the sampled token id to stage 0). */
LEAP_API int leap_pp_send(leap_pp *pp, int peer, const void *buf, size_t bytes,
                          void *stream);
LEAP_API int leap_pp_recv(leap_pp *pp, int peer, void *buf, size_t bytes,
                          void *stream);
/* End every transfer in flight (a peer died or stopped answering); the
 * communicator cannot be used afterwards.  Then leap_pp_destroy. */
LEAP_API int leap_pp_abort(leap_pp *pp);
LEAP_API int leap_pp_destroy(leap_pp *pp);

#ifdef __cplusplus
}
#endif

#endif /* LEAP_B200_H */
