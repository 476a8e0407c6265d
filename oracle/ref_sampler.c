/*
 * CPU oracle for the token sampler -- TEST INFRASTRUCTURE ONLY (see
 * ref_sampler.h).  Build with -O2 -fno-fast-math -ffp-contract=off so that
 * every f32 operation below is one IEEE-754 binary32 operation with
 * round-to-nearest-even, in the order written, exactly as the Zig reference
 * evaluates it (Zig's default float mode is strict: no contraction, no
 * reassociation).
 */
#include "ref_sampler.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

static inline uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static inline float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

/* ------------------------------------------------------------------------ */
/* PRNG: std.Random.DefaultPrng = Xoshiro256 (xoshiro256++, Blackman & Vigna
 * 2018), seeded by four outputs of SplitMix64 (Steele, Lea & Flood 2014) run
 * from the seed.  Used at sampler.zig:17,22,27,162.                           */

static uint64_t splitmix64_next(uint64_t *x) {
    uint64_t z;
    *x += 0x9e3779b97f4a7c15ULL;
    z = *x;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

void orc_rng_seed(uint64_t s[4], uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; i++) s[i] = splitmix64_next(&x);
}

static inline uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

uint64_t orc_rng_next(uint64_t s[4]) {
    const uint64_t result = rotl64(s[0] + s[3], 23) + s[0];
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}

static inline unsigned clz64(uint64_t x) { return x ? (unsigned)__builtin_clzll(x) : 64u; }
static inline unsigned clz32(uint32_t x) { return x ? (unsigned)__builtin_clz(x) : 32u; }

/* Random.float(f32): one u64 gives 23 mantissa bits (its low bits) and an
 * exponentially distributed exponent 126 - clz64; if the 41 high bits are all
 * zero, further words extend the exponent.  Random.int(u64) reads one
 * little-endian 8-byte fill == one next(); Random.int(u32) reads the low four
 * bytes of one next(). */
float orc_rng_float(uint64_t s[4], uint32_t *words) {
    uint64_t r = orc_rng_next(s);
    unsigned lz = clz64(r);
    uint32_t used = 1;
    if (lz >= 41) {
        lz = 41 + clz64(orc_rng_next(s));
        used++;
        if (lz == 41 + 64) {
            lz += clz32((uint32_t)orc_rng_next(s) | 0x7FFu);
            used++;
        }
    }
    if (words) *words += used;
    return u2f(((uint32_t)(126 - lz) << 23) | ((uint32_t)r & 0x7FFFFFu));
}

/* ------------------------------------------------------------------------ */
/* f32 exp: Zig's std.math.exp lowers to the compiler_rt expf, which follows
 * the classic FreeBSD msun / musl (pre-2018) scheme: reduce x = k*ln2 + r with
 * ln2 split into a short high part and a low part, approximate
 * exp(r) = 1 + r + r*c/(2-c) with c = r - r^2*(P1 + r^2*P2) (the Remez
 * coefficients published with that scheme), then scale by 2^k. */
static const float EXP_LN2HI = 6.9314575195e-1f;  /* 0x3f317200 */
static const float EXP_LN2LO = 1.4286067653e-6f;  /* 0x35bfbe8e */
static const float EXP_INVLN2 = 1.4426950216e+0f; /* 0x3fb8aa3b */
static const float EXP_P1 = 1.6666625440e-1f;     /* 0xaaaa8f.0p-26 */
static const float EXP_P2 = -2.7667332906e-3f;    /* -0xb55215.0p-32 */

/* y * 2^k rounded once to nearest (what scalbn does for these arguments). */
static float scale2k(float y, int k) {
    if (k > 127) {
        y = y * 0x1p127f;
        k -= 127;
        if (k > 127) k = 127;
    } else if (k < -126) {
        y = y * 0x1p-102f;   /* exact: |y| ~ 1 stays normal */
        k += 102;
        if (k < -126) {
            y = y * 0x1p-102f;
            k += 102;
            if (k < -126) k = -126;
        }
    }
    return y * u2f((uint32_t)(0x7f + k) << 23);
}

float orc_expf(float x) {
    uint32_t hx = f2u(x);
    const int sign = (int)(hx >> 31);
    hx &= 0x7fffffffu;
    if (x != x) return x;
    if (hx >= 0x42aeac50u) {                   /* |x| >= 87.33655 */
        if (hx > 0x7f800000u) return x;        /* NaN */
        if (hx >= 0x42b17218u && !sign) return x * 0x1p127f; /* overflow */
        if (sign && hx >= 0x42cff1b5u) return 0.0f;          /* x <= -103.972084 */
    }
    int k;
    float hi, lo;
    if (hx > 0x3eb17218u) {                    /* |x| > ln2/2 */
        if (hx > 0x3f851592u) {                /* |x| > 3ln2/2 */
            const float t = EXP_INVLN2 * x + (sign ? -0.5f : 0.5f);
            k = (int)t;                        /* truncation, as the C/Zig cast */
        } else {
            k = 1 - sign - sign;
        }
        const float fk = (float)k;
        hi = x - fk * EXP_LN2HI;
        lo = fk * EXP_LN2LO;
        x = hi - lo;
    } else if (hx > 0x39000000u) {             /* |x| > 2^-14 */
        k = 0;
        hi = x;
        lo = 0.0f;
    } else {
        return 1.0f + x;
    }
    const float xx = x * x;
    const float c = x - xx * (EXP_P1 + xx * EXP_P2);
    const float y = 1.0f + ((x * c / (2.0f - c) - lo) + hi);
    if (k == 0) return y;
    return scale2k(y, k);
}

/* f32 natural log: compiler_rt logf, the FreeBSD msun / musl (pre-2018)
 * scheme: x = 2^k * (1+f) with 1+f in [sqrt(2)/2, sqrt(2)], s = f/(2+f),
 * log(1+f) = f - hfsq + s*(hfsq + R(s^2)) with the published degree-4
 * minimax R, plus k*ln2 split into high and low parts. */
static const float LOG_LN2HI = 6.9313812256e-01f; /* 0x3f317180 */
static const float LOG_LN2LO = 9.0580006145e-06f; /* 0x3717f7d1 */
static const float LOG_LG1 = 0xaaaaaa.0p-24f;     /* 0.66666662693 */
static const float LOG_LG2 = 0xccce13.0p-25f;     /* 0.40000972152 */
static const float LOG_LG3 = 0x91e9ee.0p-25f;     /* 0.28498786688 */
static const float LOG_LG4 = 0xf89e26.0p-26f;     /* 0.24279078841 */

/* exp(x) - 1 in f32 as Zig's std.math.expm1 computes it (a port of the
 * musl / FreeBSD msun expm1f): reduction x = k ln2 + r with ln2 split in two,
 * the scheme's published two-coefficient rational correction (Q1, Q2), and
 * the scheme's case split on k for the reconstruction. */
float orc_expm1f(float x) {
    const float o_threshold = 8.8721679688e+01f;   /* 0x42b17180 */
    const float ln2_hi = 6.9313812256e-01f;        /* 0x3f317180 */
    const float ln2_lo = 9.0580006145e-06f;        /* 0x3717f7d1 */
    const float invln2 = 1.4426950216e+00f;        /* 0x3fb8aa3b */
    const float Q1 = -3.3333212137e-2f;            /* -0x888868.0p-28 */
    const float Q2 = 1.5807170421e-3f;             /* 0xcf3010.0p-33 */
    float y, hi, lo, c = 0.0f, t, e, hxs, hfx, r1, twopk;
    const uint32_t ux = f2u(x);
    const uint32_t hx = ux & 0x7fffffffu;
    const int sign = (int)(ux >> 31);
    int k;
    if (hx >= 0x4195b844u) {                       /* |x| >= 27 ln2 */
        if (hx > 0x7f800000u) return x;            /* NaN */
        if (sign) return -1.0f;
        if (x > o_threshold) return x * 0x1p127f;  /* overflow */
    }
    if (hx > 0x3eb17218u) {                        /* |x| > ln2/2 */
        if (hx < 0x3f851592u) {                    /* and |x| < 3ln2/2 */
            if (!sign) { hi = x - ln2_hi; lo = ln2_lo; k = 1; }
            else       { hi = x + ln2_hi; lo = -ln2_lo; k = -1; }
        } else {
            k = (int)(invln2 * x + (sign ? -0.5f : 0.5f));
            t = (float)k;
            hi = x - t * ln2_hi;
            lo = t * ln2_lo;
        }
        x = hi - lo;
        c = (hi - x) - lo;
    } else if (hx < 0x33000000u) {                 /* |x| < 2^-25 */
        return x;
    } else {
        k = 0;
    }
    hfx = 0.5f * x;
    hxs = x * hfx;
    r1 = 1.0f + hxs * (Q1 + hxs * Q2);
    t = 3.0f - r1 * hfx;
    e = hxs * ((r1 - t) / (6.0f - x * t));
    if (k == 0) return x - (x * e - hxs);
    e = x * (e - c) - c;
    e -= hxs;
    if (k == -1) return 0.5f * (x - e) - 0.5f;
    if (k == 1) {
        if (x < -0.25f) return -2.0f * (e - (x + 0.5f));
        return 1.0f + 2.0f * (x - e);
    }
    twopk = u2f((uint32_t)(0x7f + k) << 23);
    if (k < 0 || k > 56) {
        y = x - e + 1.0f;
        if (k == 128) y = y * 2.0f * 0x1p127f;
        else y = y * twopk;
        return y - 1.0f;
    }
    const float uf = u2f((uint32_t)(0x7f - k) << 23);
    if (k < 23) return (x - e + (1.0f - uf)) * twopk;
    return (x - (e + uf) + 1.0f) * twopk;
}

/* tanh in f32 as Zig's std.math.tanh computes it (a port of musl tanhf):
 * three ranges of |x| through expm1, |x| > 10 saturating to 1. */
float orc_tanhf(float x) {
    const uint32_t u = f2u(x);
    const uint32_t ux = u & 0x7fffffffu;
    const float ax = u2f(ux);
    const int sign = (int)(u >> 31);
    float t;
    if (ux > 0x3f0c9f54u) {                        /* |x| > log(3)/2, or NaN */
        if (ux > 0x41200000u) {                    /* |x| > 10 */
            t = 1.0f + 0.0f / x;
        } else {
            t = orc_expm1f(2.0f * ax);
            t = 1.0f - 2.0f / (t + 2.0f);
        }
    } else if (ux > 0x3e82c578u) {                 /* |x| > log(5/3)/2 */
        t = orc_expm1f(2.0f * ax);
        t = t / (t + 2.0f);
    } else if (ux >= 0x00800000u) {                /* |x| >= 2^-126 */
        t = orc_expm1f(-2.0f * ax);
        t = -t / (t + 2.0f);
    } else {                                       /* subnormal */
        t = ax;
    }
    return sign ? -t : t;
}

/* The engine's logit prologue before sampling (engine.zig:341-354,
 * main.zig:653-666): with a soft-cap s > 0 every logit becomes
 * tanh(v / s) * s; then, unless logit_scale is 1 or 0, v *= 1 / logit_scale
 * (the reciprocal rounded once, as f32). */
void orc_prologue(float *logits, size_t n, float softcap, float logit_scale) {
    if (softcap > 0.0f)
        for (size_t i = 0; i < n; i++) logits[i] = orc_tanhf(logits[i] / softcap) * softcap;
    if (logit_scale != 1.0f && logit_scale != 0.0f) {
        const float inv = 1.0f / logit_scale;
        for (size_t i = 0; i < n; i++) logits[i] *= inv;
    }
}

float orc_logf(float x) {
    uint32_t ix = f2u(x);
    int k = 0;
    if (ix < 0x00800000u || (ix >> 31)) {      /* x < 2^-126, or negative */
        if ((ix << 1) == 0) return -INFINITY;  /* log(+-0) */
        if (ix >> 31) return NAN;              /* log(negative) */
        k -= 25;                               /* subnormal: scale up */
        x = x * 0x1p25f;
        ix = f2u(x);
    } else if (ix >= 0x7f800000u) {
        return x;                              /* inf or NaN */
    } else if (ix == 0x3f800000u) {
        return 0.0f;
    }
    ix += 0x3f800000u - 0x3f3504f3u;
    k += (int)(ix >> 23) - 0x7f;
    ix = (ix & 0x007fffffu) + 0x3f3504f3u;
    x = u2f(ix);
    const float f = x - 1.0f;
    const float s = f / (2.0f + f);
    const float z = s * s;
    const float w = z * z;
    const float t1 = w * (LOG_LG2 + w * LOG_LG4);
    const float t2 = z * (LOG_LG1 + w * LOG_LG3);
    const float R = t2 + t1;
    const float hfsq = 0.5f * f * f;
    const float dk = (float)k;
    return (((s * (hfsq + R) + dk * LOG_LN2LO) - hfsq) + f) + dk * LOG_LN2HI;
}

/* ------------------------------------------------------------------------ */
/* Stable sort of an index permutation by a float key.  std.mem.sort is a
 * stable block sort; every stable sort driven by the same strict ordering
 * yields the same permutation, so a bottom-up merge sort is used here.
 * desc != 0: order key[a] > key[b] (sampler.zig:96-100);
 * desc == 0: order key[a] < key[b] (sampler.zig:142-146).                     */
static inline int before(const float *key, uint32_t a, uint32_t b, int desc) {
    return desc ? (key[a] > key[b]) : (key[a] < key[b]);
}

static void stable_sort_idx(uint32_t *idx, uint32_t *tmp, size_t n, const float *key, int desc) {
    /* insertion sort runs of 16, then merge */
    const size_t RUN = 16;
    for (size_t lo = 0; lo < n; lo += RUN) {
        size_t hi = lo + RUN < n ? lo + RUN : n;
        for (size_t i = lo + 1; i < hi; i++) {
            uint32_t v = idx[i];
            size_t j = i;
            while (j > lo && before(key, v, idx[j - 1], desc)) {
                idx[j] = idx[j - 1];
                j--;
            }
            idx[j] = v;
        }
    }
    uint32_t *src = idx, *dst = tmp;
    for (size_t w = RUN; w < n; w *= 2) {
        for (size_t lo = 0; lo < n; lo += 2 * w) {
            size_t mid = lo + w < n ? lo + w : n;
            size_t hi = lo + 2 * w < n ? lo + 2 * w : n;
            size_t a = lo, b = mid, o = lo;
            while (a < mid && b < hi) {
                /* take from the right run only if it strictly precedes */
                if (before(key, src[b], src[a], desc)) dst[o++] = src[b++];
                else dst[o++] = src[a++];
            }
            while (a < mid) dst[o++] = src[a++];
            while (b < hi) dst[o++] = src[b++];
        }
        uint32_t *t = src; src = dst; dst = t;
    }
    if (src != idx) memcpy(idx, src, n * sizeof(uint32_t));
}

/* ------------------------------------------------------------------------ */
void orc_sampler_init(orc_sampler *sp, const orc_config *cfg) {
    /* sampler.zig:19-24 -- a zero seed becomes 0xDEADBEEF */
    sp->cfg = *cfg;
    orc_rng_seed(sp->s, cfg->seed != 0 ? cfg->seed : 0xDEADBEEFULL);
}

uint32_t orc_argmax(const float *logits, size_t n) {
    /* sampler.zig:31-41 -- strict '>' keeps the lowest index on ties; a NaN
     * never compares greater (and a leading NaN wins). */
    size_t best = 0;
    float max_v = logits[0];
    for (size_t i = 1; i < n; i++) {
        if (logits[i] > max_v) {
            max_v = logits[i];
            best = i;
        }
    }
    return (uint32_t)best;
}

uint32_t orc_sample(orc_sampler *sp, const float *logits, size_t n,
                    const uint32_t *prev, size_t n_prev, orc_trace *tr) {
    const orc_config *cfg = &sp->cfg;
    orc_trace local;
    if (!tr) tr = &local;
    memset(tr, 0, sizeof(*tr));
    tr->u = NAN;
    tr->r0 = NAN;
    tr->cut_topp = (uint32_t)n;
    tr->draw_margin = INFINITY;
    tr->thr_margin = INFINITY;

    /* sampler.zig:50 */
    if (cfg->temperature <= 0.0f) {
        tr->path = ORC_PATH_ARGMAX_T;
        tr->token = orc_argmax(logits, n);
        return tr->token;
    }

    float *penalized = (float *)malloc(n * sizeof(float));
    float *probs = (float *)malloc(n * sizeof(float));
    uint32_t *indices = (uint32_t *)malloc(n * sizeof(uint32_t));
    uint32_t *tmp = (uint32_t *)malloc(n * sizeof(uint32_t));
    unsigned char *selected = (unsigned char *)malloc(n);
    if (!penalized || !probs || !indices || !tmp || !selected) {
        free(penalized); free(probs); free(indices); free(tmp); free(selected);
        return 0xFFFFFFFFu;
    }
    uint32_t token;

    /* sampler.zig:54-75 repetition penalty: each id in the last `window`
     * previous tokens is penalised once. */
    memcpy(penalized, logits, n * sizeof(float));
    if (cfg->repetition_penalty != 1.0f && n_prev > 0) {
        size_t window = n_prev < (size_t)cfg->repetition_window ? n_prev : (size_t)cfg->repetition_window;
        size_t start = n_prev - window;
        for (size_t i = 0; i < n; i++) {
            for (size_t j = start; j < n_prev; j++) {
                if ((uint32_t)i == prev[j]) {
                    if (penalized[i] > 0.0f) penalized[i] = penalized[i] / cfg->repetition_penalty;
                    else penalized[i] = penalized[i] * cfg->repetition_penalty;
                    break;
                }
            }
        }
    }

    /* :80-81 max via @max (maxnum: a NaN operand is ignored) */
    float max_logit = penalized[0];
    for (size_t i = 1; i < n; i++) max_logit = fmaxf(max_logit, penalized[i]);
    tr->max_logit = max_logit;

    /* :83-88 p_i = exp((v - max) / T), summed sequentially in f32 */
    float sum = 0.0f;
    double sum64 = 0.0;
    for (size_t i = 0; i < n; i++) {
        const float p = orc_expf((penalized[i] - max_logit) / cfg->temperature);
        probs[i] = p;
        sum = sum + p;
        sum64 += (double)p;
    }
    tr->sum = sum;
    tr->sum_f64 = sum64;
    /* :89 */
    if (sum <= 0.0f) {
        tr->path = ORC_PATH_ARGMAX_SUM;
        token = orc_argmax(logits, n);
        goto done;
    }
    /* :90 */
    for (size_t i = 0; i < n; i++) probs[i] = probs[i] / sum;

    /* :92-100 stable sort, probability descending */
    for (size_t i = 0; i < n; i++) indices[i] = (uint32_t)i;
    stable_sort_idx(indices, tmp, n, probs, 1);

    memset(selected, 1, n);

    /* :106-109 top-k */
    if (cfg->top_k > 0 && (size_t)cfg->top_k < n) {
        for (size_t j = cfg->top_k; j < n; j++) selected[indices[j]] = 0;
    }
    /* :111-118 top-p: the token whose cumulative mass first exceeds top_p is
     * itself deselected (add, then test). */
    if (cfg->top_p > 0.0f && cfg->top_p < 1.0f) {
        float cum_p = 0.0f;
        for (size_t j = 0; j < n; j++) {
            const uint32_t idx = indices[j];
            if (!selected[idx]) continue;
            const float before = cum_p;
            cum_p = cum_p + probs[idx];
            if (cum_p > cfg->top_p) {
                if (tr->cut_topp == (uint32_t)n) {
                    tr->cut_topp = (uint32_t)j;
                    const double m = fmin((double)cum_p - cfg->top_p, (double)cfg->top_p - before) / cfg->top_p;
                    if (m < tr->thr_margin) tr->thr_margin = m;
                }
                selected[idx] = 0;
            }
        }
    }
    /* :120-126 min-p against the global maximum probability */
    if (cfg->min_p > 0.0f) {
        const float max_prob = probs[indices[0]];
        const float p_thresh = max_prob * cfg->min_p;
        for (size_t j = 0; j < n; j++) {
            const uint32_t idx = indices[j];
            if (!selected[idx]) continue;
            if (p_thresh > 0.0f) {
                const double m = fabs((double)probs[idx] - p_thresh) / p_thresh;
                if (m < tr->thr_margin) tr->thr_margin = m;
            }
            if (probs[idx] < p_thresh) selected[idx] = 0;
        }
    }
    /* :128-154 typical-p: entropy over the full distribution (index order),
     * then a stable ascending sort by |-log p - H|. */
    if (cfg->typical_p > 0.0f && cfg->typical_p < 1.0f) {
        float entropy = 0.0f;
        for (size_t i = 0; i < n; i++) {
            const float p = probs[i];
            if (p > 0.0f) entropy = entropy - p * orc_logf(p);
        }
        tr->entropy = entropy;
        float *dev = (float *)malloc(n * sizeof(float));
        uint32_t *order = (uint32_t *)malloc(n * sizeof(uint32_t));
        if (!dev || !order) {
            free(dev); free(order);
            token = 0xFFFFFFFFu;
            goto done;
        }
        for (size_t i = 0; i < n; i++) {
            const float p = probs[i];
            const float surprise = p > 0.0f ? -orc_logf(p) : INFINITY;
            dev[i] = fabsf(surprise - entropy);
            order[i] = (uint32_t)i;
        }
        stable_sort_idx(order, tmp, n, dev, 0);
        float cum_typ = 0.0f;
        int cut = 0;
        for (size_t j = 0; j < n; j++) {
            const uint32_t idx = order[j];
            if (!selected[idx]) continue;
            const float before = cum_typ;
            cum_typ = cum_typ + probs[idx];
            if (cum_typ > cfg->typical_p) {
                if (!cut) {
                    cut = 1;
                    const double m =
                        fmin((double)cum_typ - cfg->typical_p, (double)cfg->typical_p - before) / cfg->typical_p;
                    if (m < tr->thr_margin) tr->thr_margin = m;
                }
                selected[idx] = 0;
            }
        }
        free(dev);
        free(order);
    }

    /* :156-160 kept mass, summed in probability order */
    {
        float total = 0.0f;
        uint32_t kept = 0;
        for (size_t j = 0; j < n; j++) {
            const uint32_t idx = indices[j];
            if (selected[idx]) {
                total = total + probs[idx];
                kept++;
            }
        }
        tr->total = total;
        tr->n_kept = kept;
        if (total <= 0.0f) {
            tr->path = ORC_PATH_EMPTY;
            token = indices[0];
            goto done;
        }
        /* :162-168 inverse-CDF draw in probability order */
        const float u = orc_rng_float(sp->s, &tr->draws);
        float r = u * total;
        tr->u = u;
        tr->r0 = r;
        token = indices[0];
        tr->path = ORC_PATH_DRAW_FALLBACK;
        for (size_t j = 0; j < n; j++) {
            const uint32_t idx = indices[j];
            if (!selected[idx]) continue;
            const float before = r;
            r = r - probs[idx];
            if (r <= 0.0f) {
                token = idx;
                tr->path = ORC_PATH_DRAW;
                tr->draw_margin = fmin((double)before, -(double)r) / (double)total;
                break;
            }
        }
    }

done:
    tr->token = token;
    free(penalized);
    free(probs);
    free(indices);
    free(tmp);
    free(selected);
    return token;
}

/* ------------------------------------------------------------------------ */
typedef struct {
    orc_sampler *samplers;
    const float *logits;
    size_t rows, n, ld, n_prev;
    const uint32_t *prev;
    uint32_t *out;
    orc_trace *traces;
    size_t next;
    pthread_mutex_t mu;
    int failed;
} batch_job;

static void *batch_worker(void *arg) {
    batch_job *job = (batch_job *)arg;
    for (;;) {
        pthread_mutex_lock(&job->mu);
        size_t r = job->next++;
        pthread_mutex_unlock(&job->mu);
        if (r >= job->rows) break;
        const uint32_t *pv = job->prev ? job->prev + r * job->n_prev : NULL;
        uint32_t t = orc_sample(&job->samplers[r], job->logits + r * job->ld, job->n,
                                pv, job->prev ? job->n_prev : 0,
                                job->traces ? &job->traces[r] : NULL);
        job->out[r] = t;
        if (t == 0xFFFFFFFFu) job->failed = 1;
    }
    return NULL;
}

int orc_sample_batch(orc_sampler *samplers, const float *logits, size_t rows,
                     size_t n, size_t ld, const uint32_t *prev, size_t n_prev,
                     uint32_t *out, orc_trace *traces, int nthreads) {
    batch_job job;
    memset(&job, 0, sizeof(job));
    job.samplers = samplers; job.logits = logits; job.rows = rows; job.n = n;
    job.ld = ld; job.prev = prev; job.n_prev = n_prev; job.out = out; job.traces = traces;
    pthread_mutex_init(&job.mu, NULL);
    if (nthreads <= 0) nthreads = (int)sysconf(_SC_NPROCESSORS_ONLN);
    if ((size_t)nthreads > rows) nthreads = (int)rows;
    if (nthreads <= 1) {
        batch_worker(&job);
    } else {
        pthread_t *th = (pthread_t *)malloc(sizeof(pthread_t) * (size_t)nthreads);
        for (int i = 0; i < nthreads; i++) pthread_create(&th[i], NULL, batch_worker, &job);
        for (int i = 0; i < nthreads; i++) pthread_join(th[i], NULL);
        free(th);
    }
    pthread_mutex_destroy(&job.mu);
    return job.failed ? -1 : 0;
}
