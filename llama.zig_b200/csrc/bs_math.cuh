// bs_math.cuh -- bit-exact f32 arithmetic shared by the sampler kernels.
//
// Every operation on the exact path is one IEEE-754 binary32 operation with
// round-to-nearest-even, written with the __f*_rn intrinsics so that nvcc can
// neither contract a multiply-add into an FMA nor reorder anything.  The
// results are therefore identical to the Zig reference (strict float mode)
// and to the CPU checker built with -ffp-contract=off.
#pragma once

#include <cstdint>

namespace bs {

// ---------------------------------------------------------------------------
// xoshiro256++ (Blackman & Vigna) seeded by SplitMix64 (Steele, Lea & Flood):
// the Zig std.Random.DefaultPrng used at src/sampler.zig:17,22,27,162.
__host__ __device__ __forceinline__ uint64_t splitmix64_next(uint64_t &x) {
    x += 0x9e3779b97f4a7c15ULL;
    uint64_t z = x;
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ void rng_seed(uint64_t s[4], uint64_t seed) {
    uint64_t x = seed;
    s[0] = splitmix64_next(x);
    s[1] = splitmix64_next(x);
    s[2] = splitmix64_next(x);
    s[3] = splitmix64_next(x);
}

__host__ __device__ __forceinline__ uint64_t rotl64(uint64_t x, int k) {
    return (x << k) | (x >> (64 - k));
}

__host__ __device__ __forceinline__ uint64_t rng_next(uint64_t s[4]) {
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

#ifdef __CUDA_ARCH__
__device__ __forceinline__ unsigned clz64(uint64_t x) { return (unsigned)__clzll((long long)x); }
__device__ __forceinline__ unsigned clz32(uint32_t x) { return (unsigned)__clz((int)x); }
#else
inline unsigned clz64(uint64_t x) { return x ? (unsigned)__builtin_clzll(x) : 64u; }
inline unsigned clz32(uint32_t x) { return x ? (unsigned)__builtin_clz(x) : 32u; }
#endif

// Random.float(f32): mantissa = low 23 bits of one u64, exponent 126 - clz64;
// more words extend the exponent when the 41 high bits are zero.
__host__ __device__ __forceinline__ float rng_float(uint64_t s[4]) {
    const uint64_t r = rng_next(s);
    unsigned lz = clz64(r);
    if (lz >= 41) {
        lz = 41 + clz64(rng_next(s));
        if (lz == 41 + 64) lz += clz32((uint32_t)rng_next(s) | 0x7FFu);
    }
    const uint32_t bits = ((uint32_t)(126 - lz) << 23) | ((uint32_t)r & 0x7FFFFFu);
#ifdef __CUDA_ARCH__
    return __uint_as_float(bits);
#else
    float f;
    __builtin_memcpy(&f, &bits, 4);
    return f;
#endif
}

#ifdef __CUDACC__
// ---------------------------------------------------------------------------
// f32 exp as Zig's compiler_rt expf computes it (the FreeBSD msun / musl
// pre-2018 scheme): x = k*ln2 + r with ln2 split into a short high part and a
// low part, exp(r) = 1 + r + r*c/(2-c), c = r - r^2*(P1 + r^2*P2) with that
// scheme's published Remez coefficients, then a single rounding by 2^k.
__device__ __forceinline__ float scale2k(float y, int k) {
    if (k > 127) {
        y = __fmul_rn(y, __int_as_float(0x7f000000));  // 2^127
        k -= 127;
        if (k > 127) k = 127;
    } else if (k < -126) {
        y = __fmul_rn(y, __int_as_float(0x0c800000));  // 2^-102, exact here
        k += 102;
        if (k < -126) {
            y = __fmul_rn(y, __int_as_float(0x0c800000));
            k += 102;
            if (k < -126) k = -126;
        }
    }
    return __fmul_rn(y, __int_as_float((0x7f + k) << 23));
}

__device__ __forceinline__ float exp_ref(float x) {
    const float LN2HI = __int_as_float(0x3f317200);
    const float LN2LO = __int_as_float(0x35bfbe8e);
    const float INVLN2 = __int_as_float(0x3fb8aa3b);
    const float P1 = 1.6666625440e-1f;   // 0xaaaa8f.0p-26
    const float P2 = -2.7667332906e-3f;  // -0xb55215.0p-32
    uint32_t hx = __float_as_uint(x);
    const int sign = (int)(hx >> 31);
    hx &= 0x7fffffffu;
    if (hx > 0x7f800000u) return x;  // NaN
    if (hx >= 0x42aeac50u) {
        if (hx >= 0x42b17218u && !sign) return __fmul_rn(x, __int_as_float(0x7f000000));
        if (sign && hx >= 0x42cff1b5u) return 0.0f;
    }
    int k;
    float hi, lo;
    if (hx > 0x3eb17218u) {
        if (hx > 0x3f851592u) {
            const float t = __fadd_rn(__fmul_rn(INVLN2, x), sign ? -0.5f : 0.5f);
            k = __float2int_rz(t);
        } else {
            k = 1 - sign - sign;
        }
        const float fk = __int2float_rn(k);
        hi = __fsub_rn(x, __fmul_rn(fk, LN2HI));
        lo = __fmul_rn(fk, LN2LO);
        x = __fsub_rn(hi, lo);
    } else if (hx > 0x39000000u) {
        k = 0;
        hi = x;
        lo = 0.0f;
    } else {
        return __fadd_rn(1.0f, x);
    }
    const float xx = __fmul_rn(x, x);
    const float c = __fsub_rn(x, __fmul_rn(xx, __fadd_rn(P1, __fmul_rn(xx, P2))));
    const float q = __fdiv_rn(__fmul_rn(x, c), __fsub_rn(2.0f, c));
    const float y = __fadd_rn(1.0f, __fadd_rn(__fsub_rn(q, lo), hi));
    if (k == 0) return y;
    return scale2k(y, k);
}

// f32 natural log as Zig's compiler_rt logf computes it (FreeBSD msun / musl
// pre-2018): x = 2^k (1+f), s = f/(2+f), log(1+f) = f - hfsq + s(hfsq + R(s^2))
// with that scheme's published degree-4 minimax R, plus k*ln2 in two parts.
__device__ __forceinline__ float log_ref(float x) {
    const float LN2HI = __int_as_float(0x3f317180);
    const float LN2LO = __int_as_float(0x3717f7d1);
    const float LG1 = __int_as_float(0x3f2aaaaa);  // 0xaaaaaa.0p-24
    const float LG2 = __int_as_float(0x3eccce13);  // 0xccce13.0p-25
    const float LG3 = __int_as_float(0x3e91e9ee);  // 0x91e9ee.0p-25
    const float LG4 = __int_as_float(0x3e789e26);  // 0xf89e26.0p-26
    uint32_t ix = __float_as_uint(x);
    int k = 0;
    if (ix < 0x00800000u || (ix >> 31)) {
        if ((ix << 1) == 0) return __int_as_float(0xff800000);  // -inf
        if (ix >> 31) return __int_as_float(0x7fc00000);        // NaN
        k -= 25;
        x = __fmul_rn(x, 33554432.0f);  // 2^25
        ix = __float_as_uint(x);
    } else if (ix >= 0x7f800000u) {
        return x;
    } else if (ix == 0x3f800000u) {
        return 0.0f;
    }
    ix += 0x3f800000u - 0x3f3504f3u;
    k += (int)(ix >> 23) - 0x7f;
    ix = (ix & 0x007fffffu) + 0x3f3504f3u;
    x = __uint_as_float(ix);
    const float f = __fsub_rn(x, 1.0f);
    const float s = __fdiv_rn(f, __fadd_rn(2.0f, f));
    const float z = __fmul_rn(s, s);
    const float w = __fmul_rn(z, z);
    const float t1 = __fmul_rn(w, __fadd_rn(LG2, __fmul_rn(w, LG4)));
    const float t2 = __fmul_rn(z, __fadd_rn(LG1, __fmul_rn(w, LG3)));
    const float R = __fadd_rn(t2, t1);
    const float hfsq = __fmul_rn(__fmul_rn(0.5f, f), f);
    const float dk = __int2float_rn(k);
    float r = __fadd_rn(__fmul_rn(s, __fadd_rn(hfsq, R)), __fmul_rn(dk, LN2LO));
    r = __fsub_rn(r, hfsq);
    r = __fadd_rn(r, f);
    return __fadd_rn(r, __fmul_rn(dk, LN2HI));
}

// exp(x) - 1 in f32 as Zig's std.math.expm1 computes it (a port of the
// musl / FreeBSD msun expm1f): x = k ln2 + r with ln2 in two parts, the
// scheme's published two-coefficient correction (Q1, Q2) and its case split on
// k for the reconstruction.  Every operation is one IEEE f32 operation.
__device__ __forceinline__ float expm1_ref(float x) {
    const float o_threshold = 8.8721679688e+01f;   // 0x42b17180
    const float ln2_hi = 6.9313812256e-01f;        // 0x3f317180
    const float ln2_lo = 9.0580006145e-06f;        // 0x3717f7d1
    const float invln2 = 1.4426950216e+00f;        // 0x3fb8aa3b
    const float Q1 = -3.3333212137e-2f;            // -0x888868.0p-28
    const float Q2 = 1.5807170421e-3f;             // 0xcf3010.0p-33
    const uint32_t ux = __float_as_uint(x);
    const uint32_t hx = ux & 0x7fffffffu;
    const bool sign = (ux >> 31) != 0;
    float hi, lo, c = 0.0f, t;
    int k;
    if (hx >= 0x4195b844u) {                       // |x| >= 27 ln2
        if (hx > 0x7f800000u) return x;            // NaN
        if (sign) return -1.0f;
        if (x > o_threshold) return __fmul_rn(x, 0x1p127f);
    }
    if (hx > 0x3eb17218u) {                        // |x| > ln2/2
        if (hx < 0x3f851592u) {                    // and |x| < 3ln2/2
            if (!sign) {
                hi = __fsub_rn(x, ln2_hi);
                lo = ln2_lo;
                k = 1;
            } else {
                hi = __fadd_rn(x, ln2_hi);
                lo = -ln2_lo;
                k = -1;
            }
        } else {
            k = __float2int_rz(__fadd_rn(__fmul_rn(invln2, x), sign ? -0.5f : 0.5f));
            t = __int2float_rn(k);
            hi = __fsub_rn(x, __fmul_rn(t, ln2_hi));
            lo = __fmul_rn(t, ln2_lo);
        }
        x = __fsub_rn(hi, lo);
        c = __fsub_rn(__fsub_rn(hi, x), lo);
    } else if (hx < 0x33000000u) {                 // |x| < 2^-25
        return x;
    } else {
        k = 0;
    }
    const float hfx = __fmul_rn(0.5f, x);
    const float hxs = __fmul_rn(x, hfx);
    const float r1 = __fadd_rn(1.0f, __fmul_rn(hxs, __fadd_rn(Q1, __fmul_rn(hxs, Q2))));
    t = __fsub_rn(3.0f, __fmul_rn(r1, hfx));
    float e = __fmul_rn(hxs, __fdiv_rn(__fsub_rn(r1, t), __fsub_rn(6.0f, __fmul_rn(x, t))));
    if (k == 0) return __fsub_rn(x, __fsub_rn(__fmul_rn(x, e), hxs));
    e = __fsub_rn(__fmul_rn(x, __fsub_rn(e, c)), c);
    e = __fsub_rn(e, hxs);
    if (k == -1) return __fsub_rn(__fmul_rn(0.5f, __fsub_rn(x, e)), 0.5f);
    if (k == 1) {
        if (x < -0.25f) return __fmul_rn(-2.0f, __fsub_rn(e, __fadd_rn(x, 0.5f)));
        return __fadd_rn(1.0f, __fmul_rn(2.0f, __fsub_rn(x, e)));
    }
    const float twopk = __uint_as_float((uint32_t)(0x7f + k) << 23);
    if (k < 0 || k > 56) {
        float y = __fadd_rn(__fsub_rn(x, e), 1.0f);
        y = (k == 128) ? __fmul_rn(__fmul_rn(y, 2.0f), 0x1p127f) : __fmul_rn(y, twopk);
        return __fsub_rn(y, 1.0f);
    }
    const float uf = __uint_as_float((uint32_t)(0x7f - k) << 23);
    if (k < 23) return __fmul_rn(__fadd_rn(__fsub_rn(x, e), __fsub_rn(1.0f, uf)), twopk);
    return __fmul_rn(__fadd_rn(__fsub_rn(x, __fadd_rn(e, uf)), 1.0f), twopk);
}

// tanh in f32 as Zig's std.math.tanh computes it (a port of musl tanhf):
// three ranges of |x| through expm1, |x| > 10 saturating to 1.
__device__ __forceinline__ float tanh_ref(float x) {
    const uint32_t u = __float_as_uint(x);
    const uint32_t ux = u & 0x7fffffffu;
    const float ax = __uint_as_float(ux);
    float t;
    if (ux > 0x3f0c9f54u) {                        // |x| > log(3)/2, or NaN
        if (ux > 0x41200000u) {                    // |x| > 10
            t = __fadd_rn(1.0f, __fdiv_rn(0.0f, x));
        } else {
            t = expm1_ref(__fmul_rn(2.0f, ax));
            t = __fsub_rn(1.0f, __fdiv_rn(2.0f, __fadd_rn(t, 2.0f)));
        }
    } else if (ux > 0x3e82c578u) {                 // |x| > log(5/3)/2
        t = expm1_ref(__fmul_rn(2.0f, ax));
        t = __fdiv_rn(t, __fadd_rn(t, 2.0f));
    } else if (ux >= 0x00800000u) {                // |x| >= 2^-126
        t = expm1_ref(__fmul_rn(-2.0f, ax));
        t = __fdiv_rn(-t, __fadd_rn(t, 2.0f));
    } else {                                       // subnormal
        t = ax;
    }
    return (u >> 31) ? -t : t;
}

// The engine's logit prologue before sampling (engine.zig:341-354): with a
// soft-cap s > 0, tanh(v / s) * s; then, when `scale_on`, v * inv (inv the
// f32 reciprocal of logit_scale).
__device__ __forceinline__ float prologue_ref(float v, float softcap, bool cap_on, float inv, bool scale_on) {
    if (cap_on) v = __fmul_rn(tanh_ref(__fdiv_rn(v, softcap)), softcap);
    if (scale_on) v = __fmul_rn(v, inv);
    return v;
}

// p_i = exp((v - max) / T) exactly as sampler.zig:85 evaluates it.
__device__ __forceinline__ float prob_unnorm(float v, float m, float t) {
    return exp_ref(__fdiv_rn(__fsub_rn(v, m), t));
}

// The entropy term of sampler.zig:131-133 for logit v: with P = fl(p / S),
// `entropy -= P * @log(P)` adds fl(P * -logf(P)) (negation is exact and the
// rounding symmetric); 0 when P is not positive.
__device__ __forceinline__ float entropy_term(float v, float m, float t, float S) {
    const float P = __fdiv_rn(prob_unnorm(v, m, t), S);
    if (!(P > 0.0f)) return 0.0f;
    return __fmul_rn(P, -log_ref(P));
}
#endif  // __CUDACC__

}  // namespace bs
