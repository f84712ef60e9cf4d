/*
 * malaga_b200 — B200-native NLLB-200 / M2M100 decode engine, C ABI.
 *
 * The entry points replace the CUDA decode path of rzafiamy/malaga
 * (crates/malaga-core). Each declaration names the reference interface it
 * stands in for (path:line inside the reference project). Plain pointers and
 * sizes only; every call is synchronous with respect to its host outputs and
 * runs on the context's own CUDA stream.
 *
 * Threading: one context per (thread, GPU). A context is not thread-safe; the
 * library keeps no global mutable state except the thread-local error text, so
 * N contexts on N threads drive N GPUs independently.
 *
 * Errors: every call returns an mgb_status; mgb_last_error() gives the text of
 * the calling thread's last failure. Device allocation failures return
 * MGB_ERR_OOM and their text contains "OUT_OF_MEMORY", the substring the
 * reference matches to trigger its graph-off retry and batch halving
 * (crates/malaga-core/src/graph.rs:214-222, translator.rs:150-158, 338-340).
 */
#ifndef MALAGA_B200_H
#define MALAGA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MGB_ABI_VERSION 1

#if defined(__GNUC__)
#define MGB_API __attribute__((visibility("default")))
#else
#define MGB_API
#endif

typedef struct mgb_ctx mgb_ctx;
typedef struct mgb_batch mgb_batch;

typedef enum {
    MGB_OK = 0,
    MGB_ERR_INVALID = 1,     /* bad argument, shape or token id */
    MGB_ERR_OOM = 2,         /* device allocation failed ("OUT_OF_MEMORY") */
    MGB_ERR_CUDA = 3,        /* any other CUDA error */
    MGB_ERR_IO = 4,          /* file missing or not a valid NLLB GGUF */
    MGB_ERR_UNSUPPORTED = 5, /* tensor type or dimension the kernels do not handle */
} mgb_status;

typedef struct {
    /* Capture the decoder step once per shape bucket as a CUDA graph and replay it
     * (graph.rs:273-294). 0 runs the same kernels eagerly (MALAGA_NO_CUDA_GRAPH). */
    int use_graphs;
    /* Byte budget of cached static states + graphs, LRU-evicted (graph.rs:183, 302-323;
     * MALAGA_GRAPH_CACHE_MB). Default 8 GiB: the reference's 512 MiB default is
     * sized for a 24 GB card, while one batch-64 state here (K/V caches of 128
     * positions, 128-key cross K/V, split-K buffers) takes about 0.85 GB and a
     * length-sorted batch set touches up to four source buckets. */
    uint64_t graph_cache_bytes;
    /* Test hook: when >= 0, the n-th device allocation made after mgb_open returns
     * MGB_ERR_OOM, without touching the GPU's memory. -1 = off. */
    int fail_alloc_after;
} mgb_options;

typedef struct {
    uint32_t vocab_size, d_model, encoder_layers, decoder_layers, encoder_heads, decoder_heads;
    uint32_t encoder_ffn, decoder_ffn, max_position_embeddings, max_length;
    uint32_t pad_token_id, eos_token_id, decoder_start_token_id, bos_token_id, scale_embedding;
    uint64_t weight_bytes;        /* device bytes of all weights */
    uint64_t decoder_step_bytes;  /* weight bytes one greedy step reads: decoder layers + LM head */
    uint64_t lm_head_bytes;       /* bytes of the tied LM head (token embedding) */
} mgb_model_info;

/* Fills `o` with the defaults (graphs on, 8 GiB cache, no fault injection). */
MGB_API void mgb_default_options(mgb_options *o);

/* Loads a GGUF written by malaga's converter onto GPU `device`.
 * Replaces Translator::load + Nllb::load (translator.rs:63-73, model.rs:343-433). */
MGB_API mgb_status mgb_open(const char *gguf_path, int device, const mgb_options *opts, mgb_ctx **out);

/* Frees the context and every device buffer it owns. */
MGB_API void mgb_close(mgb_ctx *ctx);

/* Text of the calling thread's last error ("" if none). */
MGB_API const char *mgb_last_error(void);

/* Architecture and memory figures of the loaded model (config.rs:15-35). */
MGB_API mgb_status mgb_model_info_get(const mgb_ctx *ctx, mgb_model_info *out);

/* Runs the encoder on a right-padded batch and projects every decoder layer's
 * cross-attention K/V once. ids: [b, s_stride] row-major (tokens past lens[i]
 * are ignored); lens: [b], 1 <= lens[i] <= s_stride <= max_position_embeddings - 2.
 * Replaces Nllb::encode_cross (model.rs:463-500). */
MGB_API mgb_status mgb_encode(mgb_ctx *ctx, const uint32_t *ids, const uint32_t *lens, uint32_t b, uint32_t s_stride,
                      mgb_batch **out);

/* Frees an encoded batch. Its device buffer goes back to the context's pool,
 * reused by the next mgb_encode (at most 4 GiB kept; mgb_clear_cache and
 * mgb_close release them). A batch freed after its context was closed releases
 * its buffer itself. */
MGB_API void mgb_batch_free(mgb_batch *batch);

/* Copies cross-attention K (which=0) or V (which=1) of decoder layer `layer`,
 * [b, heads, s, head_dim] as IEEE f16 bits, to the host (a parity / debug hook;
 * the reference keeps these as candle tensors, model.rs:471-475). */
MGB_API mgb_status mgb_batch_cross(mgb_ctx *ctx, const mgb_batch *batch, uint32_t layer, int which, uint16_t *out);

/* Greedy decoding of an encoded batch: step 0 consumes decoder_start, the target
 * language token is forced, then up to max_new tokens are generated per row.
 * out_ids: [b, max_new] raw columns (pad after a row's eos); out_lens: [b] tokens
 * before the first eos. force_steps = 1 ignores eos (every row decodes max_new
 * tokens; the benchmark configurations' "EOS ignored"). sync_every: host check
 * of the all-finished flag every n steps (translator.rs:47).
 * Replaces GraphCache::greedy (graph.rs:204-298). */
MGB_API mgb_status mgb_greedy(mgb_ctx *ctx, const mgb_batch *batch, uint32_t tgt_lang, uint32_t max_new, uint32_t sync_every,
                      int force_steps, uint32_t *out_ids, uint32_t *out_lens);

/* Same decode run eagerly with the logits of every generated step copied out:
 * logits [max_new, b, vocab] f32 (may be NULL), out_ids as mgb_greedy. A parity
 * hook: the graph path never writes logits to memory (model.rs:607-608). */
MGB_API mgb_status mgb_greedy_logits(mgb_ctx *ctx, const mgb_batch *batch, uint32_t tgt_lang, uint32_t max_new,
                             int force_steps, uint32_t *out_ids, float *logits);

/* Index of the vocabulary shortlist stored for language code `code` (GGUF
 * metadata nllb.shortlist.<code> with tensor lm_head.<code>.weight, written by
 * the converter's shortlist option, convert.rs:218-232), or -1. */
MGB_API int mgb_shortlist_find(const mgb_ctx *ctx, const char *code);

/* mgb_greedy over a vocabulary shortlist (--fast-vocab, not exact; model.rs:229-250,
 * 556-612, graph.rs:98-105, malaga.cu:280-326): each step scores the shortlist's
 * rows of the LM head plus the row's source tokens (dot products of the final
 * LayerNorm output with their embeddings) and picks the best of the two lists
 * (lowest index on ties, shortlist first). decoder_start and tgt_lang must be
 * in the shortlist (translator.rs:186-192), else MGB_ERR_INVALID. */
MGB_API mgb_status mgb_greedy_shortlist(mgb_ctx *ctx, const mgb_batch *batch, uint32_t tgt_lang, int shortlist,
                                uint32_t max_new, uint32_t sync_every, int force_steps, uint32_t *out_ids,
                                uint32_t *out_lens);

/* Beam search over an encoded batch (Translator::beam_search, translator.rs:250-358):
 * beam width k (1..8), length penalty (score / (len+1)^penalty), at most max_new
 * tokens; batch * k <= 64 rows. The prefix [decoder_start, tgt_lang] is fed first.
 * out_ids: [b, max_new] the best hypothesis per sentence (eos not included, pad
 * after it); out_lens: [b] its length. Log-softmax statistics and per-row top-k
 * run on the device, the k*k candidate merge on the host, as in the reference. */
MGB_API mgb_status mgb_beam(mgb_ctx *ctx, const mgb_batch *batch, uint32_t tgt_lang, uint32_t k, float length_penalty,
                    uint32_t max_new, uint32_t *out_ids, uint32_t *out_lens);

/* The device half of one beam-search step on caller logits: per row,
 * log_softmax (model.rs:615-617) and the k largest values with their indices
 * (translator.rs:343-358, k argmax passes: larger value first, lower index on
 * ties), on the kernel mgb_beam runs. logits: host [rows, vocab] f32;
 * vals / idx: host [rows, k]. A row with fewer than k non-NaN values pads with
 * (-inf, 0); NaN logits are never selected. k in 1..8. */
MGB_API mgb_status mgb_log_softmax_topk(mgb_ctx *ctx, const float *logits, uint32_t rows, uint32_t vocab, uint32_t k,
                                float *vals, uint32_t *idx);

/* Frees every cached static state and CUDA graph (GraphCache::clear, graph.rs:193-200). */
MGB_API mgb_status mgb_clear_cache(mgb_ctx *ctx);

/* The context's CUDA stream (a cudaStream_t), for callers that time or order work on it. */
MGB_API void *mgb_cuda_stream(mgb_ctx *ctx);

/* Number of the library's kernel launches so far (graph replays count every kernel node). */
MGB_API uint64_t mgb_kernel_launches(const mgb_ctx *ctx);

/* Instrumentation for the benchmark: runs `iters` greedy steps eagerly on an
 * encoded batch (forced, in the batch's graph bucket) and reports the mean
 * device time of the fused LM-head kernel and of a whole step, from CUDA events
 * recorded on the context's stream. No reference counterpart (the reference
 * times whole translations, crates/malaga/src/main.rs:409-457). */
MGB_API mgb_status mgb_profile_step(mgb_ctx *ctx, const mgb_batch *batch, uint32_t tgt_lang, uint32_t iters,
                            float *lm_head_ms, float *step_ms);

/* Greedy token choice (highest logit, lowest index on ties) for `rows` rows of
 * `vocab` f32 logits that are already in device memory, without allocating any
 * device memory. No counterpart in the reference: malaga's greedy_select
 * allocates its partial buffers on every call (crates/malaga-core/src/
 * kernels.rs:306-307). For callers that cannot allocate at this point: code
 * inside another framework's CUDA stream capture, hosts whose caching allocator
 * already holds the GPU's memory, serving loops that forbid allocation.
 *   logits: [rows, vocab] device memory; ids: [rows] device memory; vals: [rows]
 *   device memory or NULL (the winning logits); stream: a cudaStream_t (NULL =
 *   the legacy default stream) on the current device.
 * rows must be <= 64 (the fixed scratch size); larger requests fail with
 * MGB_ERR_INVALID. The scratch is a 128 KiB static device array that every
 * GPU loading the library keeps until exit, shared by all calls: calls that
 * overlap on the GPU race. The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture. The cached address belongs to the device's current context:
 * after cudaDeviceReset on that device it is stale and the library must be
 * reloaded. NaN logits never win; a row of only NaNs gives id 0 and value
 * -inf. Asynchronous: results are ready when the stream reaches them. */
MGB_API mgb_status mgb_argmax_noalloc(const float *logits, uint32_t rows, uint32_t vocab, uint32_t *ids, float *vals,
                                      void *stream);

#ifdef __cplusplus
}
#endif

#endif /* MALAGA_B200_H */
