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
