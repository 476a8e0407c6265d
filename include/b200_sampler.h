/*
 * b200_sampler.h -- C ABI of the B200 token sampler.
 *
 * A drop-in for the CPU sampler of llama.zig (src/sampler.zig).  The entry
 * points below are what a Zig caller binds with @cImport; they take plain
 * pointers, sizes and a CUDA stream passed as void*.
 *
 * Interfaces replaced (reference file:line):
 *   bs_config            <- SamplerConfig            src/sampler.zig:4-13
 *   bs_create            <- Sampler.init             src/sampler.zig:19-24
 *   bs_sample            <- Sampler.sample           src/sampler.zig:26-28
 *                           (sampleWithRandom        src/sampler.zig:43-169)
 *   bs_sample_host       <- Sampler.sample with host logits, as engine.zig:355
 *                           and main.zig:667 call it today
 *   bs_argmax            <- sampleArgmax             src/sampler.zig:31-41
 *                           and Dispatcher.executeTopK src/compute_graph.zig:948-985
 *   bs_argmax_ex         <- executeTopK's logit_scale_bits (src/shaders/topk_bda.glsl:38-40)
 *                           and the host soft-cap before sampleArgmax (src/engine.zig:341-354)
 *   bs_set_logit_prologue <- the engine's logit prologue before Sampler.sample
 *                           (src/engine.zig:341-354, src/main.zig:653-666), from
 *                           ModelConfig.final_logit_softcapping / logit_scale (src/model.zig:34-35)
 *   bs_get/set_rng_state <- the DefaultPrng field    src/sampler.zig:17
 *   bs_seed_state        <- its initialisation in Sampler.init, host only
 *                           src/sampler.zig:22
 *   bs_destroy           <- (Zig: the Sampler goes out of scope)
 *   bs_status            <- error.OutOfMemory        src/sampler.zig:26 (!TokenID)
 *
 * Semantics: every row r of a handle is one Sampler.  Its xoshiro256++ state
 * is seeded like Sampler.init (seed, or 0xDEADBEEF when the seed is 0) and it
 * advances only when a row actually draws, exactly as in sampler.zig.  Token
 * ids are bit-identical to sampleWithRandom's on the same logits and state.
 *
 * Threading: a handle owns device buffers and per-row RNG state; calls on one
 * handle must be ordered (same stream or externally synchronised), as a Zig
 * Sampler is single-threaded.  Logits are borrowed device pointers; nothing is
 * copied unless the _host variant is used.
 *
 * Rows the sampler could not finish: such a row's token comes back as
 * 0xFFFFFFFF and its RNG state is left as it was (no draw).  With a handle,
 * bs_last_device_status reports why; the condition is per call, so the next
 * call starts clean.  The causes are a bounded device wait that gave up
 * (BS_ETIMEOUT) and, for the vocabulary-sharded draw only, a shard whose
 * candidates overflowed (BS_EINTERNAL).  A row whose candidate set or
 * typical-p band fails its cover check is not among them: it is sorted again
 * over the whole vocabulary on the device (slower, same result).
 *
 * Repetition penalty: the last min(n_prev, repetition_window) previous ids of
 * each row are penalised once each, for windows of any length (sampler.zig:
 * 54-75); ids outside the vocabulary match nothing.
 */
#ifndef B200_SAMPLER_H
#define B200_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes (replace Zig error unions). */
typedef enum bs_status {
    BS_OK = 0,
    BS_EINVAL = 1,     /* bad argument (null pointer, size out of range)        */
    BS_ENOMEM = 2,     /* device or host allocation failed (error.OutOfMemory)  */
    BS_ECUDA = 3,      /* a CUDA runtime call failed                            */
    BS_ENCCL = 4,      /* an NCCL call failed (vocab-sharded path)              */
    BS_ETIMEOUT = 5,   /* a bounded device-side wait gave up                    */
    BS_ENOTSUP = 6,    /* configuration outside what this build implements      */
    BS_EINTERNAL = 7   /* a device-side consistency check failed                */
} bs_status;

/* SamplerConfig, field for field (src/sampler.zig:4-13); 40 bytes. */
typedef struct bs_config {
    float temperature;          /* :5  default 0.8 */
    uint32_t top_k;             /* :6  default 0   */
    float top_p;                /* :7  default 0.9 */
    float min_p;                /* :8  default 0.0 */
    float typical_p;            /* :9  default 1.0 */
    uint32_t _pad0;             /* keeps seed 8-byte aligned; must be 0 */
    uint64_t seed;              /* :10 default 0 (-> 0xDEADBEEF)        */
    uint32_t repetition_window; /* :11 default 32  */
    float repetition_penalty;   /* :12 default 1.1 */
} bs_config;

typedef struct bs_sampler bs_sampler;

/* Fill *cfg with SamplerConfig's defaults (src/sampler.zig:5-12). */
void bs_config_default(bs_config *cfg);

/* Sampler.init for `batch` rows of `vocab` logits on CUDA device `device`.
 * Row r is seeded with cfg->seed + r (0 -> 0xDEADBEEF), unless `seeds` is
 * non-NULL, in which case row r is seeded with seeds[r]. */
bs_status bs_create(const bs_config *cfg, uint32_t batch, uint32_t vocab, int device,
                    const uint64_t *seeds, bs_sampler **out);

/* Sampler.sample for rows [row0, row0 + rows) of the handle.
 *   d_logits : device pointer, row i at d_logits + i*ld (ld >= vocab floats)
 *   d_prev   : device pointer to rows x n_prev previous token ids (row-major),
 *              or NULL; used only by the repetition penalty
 *   d_out    : device pointer, rows token ids
 *   stream   : cudaStream_t (NULL = legacy default stream)
 * Stream-ordered; returns once the work is enqueued. */
bs_status bs_sample(bs_sampler *s, const float *d_logits, size_t ld, uint32_t row0, uint32_t rows,
                    const uint32_t *d_prev, uint32_t n_prev, uint32_t *d_out, void *stream);

/* Compatibility path with host buffers (what engine.zig:355 passes today):
 * copies logits (and prev) to the device, samples, copies ids back and
 * synchronises the handle's stream.  h_prev may be NULL. */
bs_status bs_sample_host(bs_sampler *s, const float *h_logits, size_t ld, uint32_t row0,
                         uint32_t rows, const uint32_t *h_prev, uint32_t n_prev, uint32_t *h_out);

/* sampleArgmax on `rows` device rows: first index of the maximum (strict >,
 * lowest index on ties, a NaN never wins unless it is element 0). */
bs_status bs_argmax(const float *d_logits, size_t ld, uint32_t rows, uint32_t vocab,
                    uint32_t *d_out, void *stream);

/* sampleArgmax after the engine's logit prologue: with a soft-cap s > 0 each
 * logit is taken as tanh(v / s) * s (Zig's f32 std.math.tanh), then, unless
 * logit_scale is 1 or 0, multiplied by the f32 reciprocal of logit_scale.
 * softcap <= 0 and logit_scale 1 give bs_argmax.  The logits are not changed
 * in memory. */
bs_status bs_argmax_ex(const float *d_logits, size_t ld, uint32_t rows, uint32_t vocab,
                       float final_logit_softcapping, float logit_scale, uint32_t *d_out, void *stream);

/* The engine's logit prologue, fused into every later bs_sample on this
 * handle (the engine.zig loop applies it to the host logits before
 * Sampler.sample): soft-cap tanh(v / s) * s when final_logit_softcapping > 0,
 * then v * (1 / logit_scale) unless logit_scale is 1 or 0.  It comes before
 * the repetition penalty, and the T <= 0 argmax sees it too.  The logits are
 * read, not rewritten.  (0, 1) turns it off. */
bs_status bs_set_logit_prologue(bs_sampler *s, float final_logit_softcapping, float logit_scale);

/* Vocabulary sharding for a tensor-parallel LM head:
 * rank g of `world` holds columns [col0, col0 + vocab) of every row, the
 * handle created with the shard width as its vocab and the same seeds on
 * every rank.  Replaces the reference's LM head -> host logits -> sample
 * sequence (src/compute_graph.zig:505-528, src/engine.zig:339-355) when the
 * head is split over GPUs.  Exact: the tokens and RNG states equal a single
 * Sampler's over the whole row.  One call is five steps on every rank, with
 * the caller's collectives between them (stream-ordered, device buffers):
 *   1 bs_vshard_stats   -> d_part (rows entries); all-gather -> [world][rows]
 *   2 bs_vshard_main(parts, world, rank)
 *   3 bs_vshard_walk(entry, exit): entry = NULL on rank 0, else the exit sums
 *     received from rank - 1; send exit to rank + 1; the last rank's exit is
 *     the row normaliser S: broadcast it from rank world - 1
 *   4 bs_vshard_export -> d_cand (rows x BS_VSHARD_CAND_CAP), d_count (rows);
 *     all-gather both -> [world][rows][..], [world][rows]
 *   5 bs_vshard_draw(cand_all, count_all, world, S) -> d_out (rows tokens,
 *     the same on every rank)
 * Needs temperature > 0, 0 < top_k <= 256 and typical-p off (BS_ENOTSUP
 * otherwise); a shard with more than BS_VSHARD_CAND_CAP candidates in a row
 * fails that row (token 0xFFFFFFFF). */
typedef struct bs_vshard_part { float max_logit; uint32_t nonfinite; double sum; } bs_vshard_part;
typedef struct bs_vshard_cand { uint32_t id; float logit; } bs_vshard_cand;
#define BS_VSHARD_CAND_CAP 512
bs_status bs_vshard_stats(bs_sampler *s, const float *d_shard, size_t ld, uint32_t col0, uint32_t rows,
                          const uint32_t *d_prev, uint32_t n_prev, bs_vshard_part *d_part, void *stream);
bs_status bs_vshard_main(bs_sampler *s, const bs_vshard_part *d_parts, uint32_t world, uint32_t rank,
                         void *stream);
bs_status bs_vshard_walk(bs_sampler *s, const float *d_entry, float *d_exit, void *stream);
bs_status bs_vshard_export(bs_sampler *s, uint32_t col0, bs_vshard_cand *d_cand, uint32_t *d_count, void *stream);
bs_status bs_vshard_draw(bs_sampler *s, const bs_vshard_cand *d_cand_all, const uint32_t *d_count_all,
                         uint32_t world, const float *d_S, uint32_t *d_out, void *stream);

/* The same step through peer memory over NVLink instead of host-issued
 * collectives (one process per GPU, all GPUs of one node):
 *   bs_vshard_ipc_handle  the 64-byte CUDA IPC handle of this rank's exchange
 *                         words for `world` ranks (allocated on first use)
 *   (the caller all-gathers the handles: world x 64 bytes of host memory)
 *   bs_vshard_ipc_open    maps the other ranks' exchange words
 * Then, with the handle's whole batch in every call:
 *   bs_vshard_stats       with d_part = NULL stores each row's partial in
 *                         every rank's words (no all-gather)
 *   bs_vshard_main        with d_parts = NULL waits (bounded) for each row's
 *                         partials of every rank
 *   bs_vshard_export      with d_cand = d_count = NULL stores the candidates
 *                         in every rank's words (no all-gather)
 *   bs_vshard_chain       replaces bs_vshard_walk and the exit / S exchange:
 *                         the walk of a row on rank g waits for rank g-1's
 *                         exit of that row and stores its own into rank g+1's
 *                         words; the last rank stores S into every rank's
 *   bs_vshard_draw        with d_cand_all = d_count_all = d_S = NULL takes
 *                         them from this rank's words.
 * Every word is tagged with the step (a counter every rank advances in
 * bs_vshard_stats), so a replayed CUDA graph works; every rank must make the
 * same sequence of calls on its handle. */
bs_status bs_vshard_ipc_handle(bs_sampler *s, uint32_t world, void *h_handle64);
bs_status bs_vshard_ipc_open(bs_sampler *s, uint32_t world, uint32_t rank, const void *h_handles);
bs_status bs_vshard_chain(bs_sampler *s, void *stream);

/* Per-row xoshiro256++ state, batch x 4 u64 (host memory).  Synchronous. */
bs_status bs_get_rng_state(bs_sampler *s, uint64_t *h_state);
bs_status bs_set_rng_state(bs_sampler *s, const uint64_t *h_state);

/* The xoshiro256++ state that Sampler.init gives a seed (replaces the prng
 * field's initialisation at src/sampler.zig:19-23: DefaultPrng.init(seed, or
 * 0xDEADBEEF when seed is 0), i.e. four SplitMix64 outputs).  Host only: it
 * touches no device and allocates nothing, so a Sampler can be initialised
 * before any device exists and hand the state over with bs_set_rng_state
 * when it first samples. */
bs_status bs_seed_state(uint64_t seed, uint64_t *h_state4);

/* Status of the last bs_sample on this handle after the stream reached it:
 * BS_OK, or the first device-side error (e.g. BS_EINTERNAL).  Synchronous. */
bs_status bs_last_device_status(bs_sampler *s);

/* Profiling (the counterpart of the engine's --report-json timers,
 * src/engine.zig:14-26 and :457-462): when enabled, each of the next
 * `max_calls` bs_sample calls records CUDA events around its kernel groups.
 * bs_profile_read synchronises and writes, for up to `cap` calls, the
 * durations in ms: ms[3i] the statistics pass (the one HBM read of the
 * logits, and the per-row reduction), ms[3i+1] the main pass (with typical-p
 * also the normaliser walk and the entropy main pass), ms[3i+2] the final
 * walk/draw pass; then it resets the ring. */
bs_status bs_profile_enable(bs_sampler *s, uint32_t max_calls);
bs_status bs_profile_read(bs_sampler *s, float *ms, uint32_t cap, uint32_t *n_calls);

/* No counterpart in the reference (sampler.zig always allocates through the
 * caller's allocator).  bs_sample for callers that must not allocate device
 * memory while sampling: no handle, no cudaMalloc.  Scratch is one fixed
 * static device array of this library (about 14 MB per device), so at most
 * BS_STATIC_MAX_ROWS rows of at most BS_STATIC_MAX_VOCAB logits per call;
 * larger calls return BS_EINVAL with a message on stderr.
 *   cfg    : the sampler settings
 *   d_rng  : device buffer of rows x 4 u64 xoshiro256++ states, in the layout
 *            bs_get_rng_state returns; advanced in place like bs_sample's
 * Other arguments as bs_sample (row i of this call uses d_rng[4i..4i+3]).
 * All calls on one device share the scratch: calls that may overlap in time
 * (different streams or host threads) race and must be ordered by the
 * caller.  The first call on each device resolves the scratch address
 * (cudaGetSymbolAddress) and must not be made while a stream is capturing.
 * There is no handle to ask for a status: a row this call could not finish
 * comes back as token 0xFFFFFFFF (its RNG state unchanged), and only that
 * call's rows are affected. */
#define BS_STATIC_MAX_ROWS 4
#define BS_STATIC_MAX_VOCAB 131072
bs_status bs_sample_static(const bs_config *cfg, uint64_t *d_rng, const float *d_logits, size_t ld,
                           uint32_t rows, uint32_t vocab, const uint32_t *d_prev, uint32_t n_prev,
                           uint32_t *d_out, void *stream);

void bs_destroy(bs_sampler *s);

const char *bs_status_string(bs_status st);

#ifdef __cplusplus
}
#endif
#endif /* B200_SAMPLER_H */
