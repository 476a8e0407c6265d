/*
 * CPU oracle for the token sampler -- TEST INFRASTRUCTURE ONLY.
 *
 * This library is the checker for the CUDA sampler in llama.zig_b200/.  Only
 * tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference leg
 * may load it.  It is never linked into, or called by, the product path.
 *
 * It restates, operation for operation, src/sampler.zig of llama.zig
 * (Sampler.init :19-24, Sampler.sample :26-28, sampleArgmax :31-41,
 * sampleWithRandom :43-169) in C11, including the pieces that sampler.zig takes
 * from the Zig standard library / compiler_rt (xoshiro256++ seeded by
 * SplitMix64, Random.float(f32), a stable sort, f32 exp and log).
 *
 * Parity status: PARTIALLY PINNED.  The two reference tests
 * (sampler.zig:171-193 determinism, :195-213 top-k=1 -> argmax) are reproduced
 * as known-answer tests.  Zig is not installed, so the RNG stream, the
 * Random.float(f32) mapping and the exp/log ulps are restated from the
 * published algorithms and cannot be checked against Zig itself here
 * ("parity unpinned" for those three pieces).
 */
#ifndef REF_SAMPLER_H
#define REF_SAMPLER_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Field-for-field mirror of SamplerConfig (sampler.zig:4-13); same layout as
 * bs_config in include/b200_sampler.h. */
typedef struct orc_config {
    float temperature;
    uint32_t top_k;
    float top_p;
    float min_p;
    float typical_p;
    uint32_t _pad0;
    uint64_t seed;
    uint32_t repetition_window;
    float repetition_penalty;
} orc_config;

/* Sampler (sampler.zig:15-18): the config plus the xoshiro256++ state. */
typedef struct orc_sampler {
    orc_config cfg;
    uint64_t s[4];
} orc_sampler;

/* Per-call diagnostics (all fields are what the reference computed). */
typedef struct orc_trace {
    uint32_t token;
    uint32_t path;          /* see ORC_PATH_* */
    uint32_t n_kept;        /* tokens still selected before the draw */
    uint32_t draws;         /* u64 words consumed from the PRNG this call */
    float max_logit;
    float sum;              /* sequential f32 normaliser (sampler.zig:83-88) */
    float entropy;          /* typical-p entropy (sampler.zig:129-132), 0 if off */
    float total;            /* kept mass (sampler.zig:156-159) */
    float u;                /* Random.float(f32) (NaN if no draw) */
    float r0;               /* u * total */
    double sum_f64;         /* exact-ish f64 sum of the same p_i (diagnostic) */
    uint32_t cut_topp;      /* sorted position of the first token top-p cut (n if none) */
    uint32_t _pad;
    /* Parity classification (diagnostics, not part of the reference):
     * draw_margin: distance of the draw u to the nearest boundary of the kept
     *   tokens' CDF, in units of u (r before and after the winning subtraction,
     *   divided by the kept mass); +inf without a draw.
     * thr_margin: the smallest relative distance of a filter decision to its
     *   threshold (top-p's running sum against top_p at the cut, min-p's
     *   kept/cut probabilities against p_max * min_p, typical-p's running sum
     *   against typical_p at its cut); +inf when no such decision was made. */
    double draw_margin;
    double thr_margin;
} orc_trace;

enum {
    ORC_PATH_ARGMAX_T = 0,      /* temperature <= 0            (sampler.zig:50) */
    ORC_PATH_ARGMAX_SUM = 1,    /* sum <= 0                    (sampler.zig:89) */
    ORC_PATH_EMPTY = 2,         /* total_selected <= 0         (sampler.zig:160) */
    ORC_PATH_DRAW = 3,          /* r crossed zero              (sampler.zig:166) */
    ORC_PATH_DRAW_FALLBACK = 4  /* loop ended without return   (sampler.zig:168) */
};

/* --- Zig standard-library pieces, restated from their published algorithms -- */
void orc_rng_seed(uint64_t s[4], uint64_t seed);   /* Xoshiro256.init */
uint64_t orc_rng_next(uint64_t s[4]);              /* Xoshiro256.next */
float orc_rng_float(uint64_t s[4], uint32_t *words);/* Random.float(f32) */
float orc_expf(float x);                           /* compiler_rt expf */
float orc_logf(float x);                           /* compiler_rt logf */
float orc_expm1f(float x);                         /* std.math.expm1 (f32) */
float orc_tanhf(float x);                          /* std.math.tanh (f32) */
/* The engine's logit prologue (engine.zig:341-354): soft-cap, then 1/scale. */
void orc_prologue(float *logits, size_t n, float softcap, float logit_scale);

/* --- sampler.zig ---------------------------------------------------------- */
void orc_sampler_init(orc_sampler *sp, const orc_config *cfg);
uint32_t orc_argmax(const float *logits, size_t n);
/* Returns the token; 0xFFFFFFFF on allocation failure (error.OutOfMemory). */
uint32_t orc_sample(orc_sampler *sp, const float *logits, size_t n,
                    const uint32_t *prev, size_t n_prev, orc_trace *trace);

/* Batch helper for the harnesses: row r uses samplers[r], logits + r*ld.
 * prev (nullable) is rows x n_prev, row-major.  nthreads <= 0 -> all cores. */
int orc_sample_batch(orc_sampler *samplers, const float *logits, size_t rows,
                     size_t n, size_t ld, const uint32_t *prev, size_t n_prev,
                     uint32_t *out, orc_trace *traces, int nthreads);

#ifdef __cplusplus
}
#endif
#endif
