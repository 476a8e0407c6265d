// sampler.cu -- B200 token sampler: CUDA kernels (sm_100a) and the C ABI.
//
// The reference (llama.zig src/sampler.zig:43-169, sampleWithRandom) turns a
// row of V logits into one token on one CPU core:
//   p_i = exp((v_i - max)/T); sum = p_0 + p_1 + ... (sequential f32, index
//   order); probs = p/sum; stable sort; top-k / top-p / min-p / typical-p
//   masks; total = sum of kept probs in sorted order; r = float() * total;
//   walk sorted kept tokens until r <= 0.
// Every decision downstream of `sum` depends on its exact f32 value, so this
// implementation reproduces the sequential f32 sum bit for bit, in parallel:
//
//   k0_penalty  (a repetition penalty only) one bit per token of the row's
//               last `window` previous ids; the passes below apply the
//               penalty (and the engine's logit prologue, if one is set)
//               while loading.
//   k1_stats    one CTA per 8192-logit segment, one 32-logit tile per thread,
//               the segment bulk-copied into shared memory (the one full HBM
//               read): tile maxima and approximate tile sums of
//               2^((v - tile max) log2e / T); segment maxima and sums; the
//               histograms the candidate floor (top-p) or the typical-p band
//               need.
//   k1_rows     one CTA per row: the row maximum M, an approximate running
//               sum at every segment start, and the candidate floor: top-k
//               from the tile maxima, top-p from a tail-mass bound, min-p
//               from its threshold.
//   k2_main     one CTA per segment again: each tile gets the binades
//               [lo, hi] its running sum can be in.  Inside one binade e the
//               f32 add s + p is exactly s + u_e round(p / u_e) (u_e the ulp
//               of binade e; round half to even, whose tie direction depends
//               on the parity of s), so a tile whose window is one binade
//               (SIMPLE) reduces to a pair of integer counts (entry parity
//               0/1).  The counts come from ex2.approx bracketed by a proven
//               error bound; a tile whose bracket is ambiguous, or that spans
//               more binades (WINDOW / COMPLEX), is counted exactly by one
//               warp with the restated expf, COMPLEX tiles keeping their exact
//               terms.  Runs of tiles become walk items; tokens above the
//               floor become candidates (index, logit).
//   kernel_b    one CTA per row: warp 0 walks the ~40 items with the exact
//               state (binade, integer mantissa): an item applies in O(1)
//               when the state is in its binade and stays there; otherwise
//               the tile is added element by element with the reference's
//               f32 adds.  The result is the reference's `sum`, bit for bit,
//               for every input (a wrong prediction only costs time).
//               Meanwhile the other warps sort the candidates; then exact
//               probs, the filters, the kept mass and the draw follow the
//               reference's sequential f32 order on the candidate prefix.
//   Typical-p runs k2_main and kernel_b once more over the entropy terms
//   P (-ln P), which reproduces H bit for bit in the same way.
//
// Candidates: k2_main keeps only tokens above a floor that provably contains
// the kept prefix and the token that ends it; kernel_b verifies the cover,
// and a row whose check fails is sorted again over its whole vocabulary in
// the same CTA (the reference's full sort; slower, same token).
//
// Also here: argmax_kernel (T <= 0), persistent forms of the first three
// passes (k_fused, k_resident; opt-in), the vocabulary-sharded entry points
// (bs_vshard_*), and the allocation-free entry point (bs_sample_static).
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>

#include "../../include/b200_sampler.h"
#include "bs_math.cuh"
#include "sampler_kernels.cuh"

namespace bs {

constexpr uint32_t QSAT = 1u << 30;      // saturation of grid counts
constexpr uint32_t QLIM = 1u << 24;      // mantissa range of one binade
constexpr float NEG_INF = -__builtin_huge_valf();

// ---------------------------------------------------------------------------
// Grid-count composites.  Within binade e (ulp u_e = 2^(e-23); e = -126 also
// covers the subnormals) the state is s = m * u_e, m < 2^24.  Adding p gives
// m + round_e(p); a tie goes to the even result, so its count depends on the
// parity of m.  A composite stores the total count for entry parity 0 and 1.
struct Comp {
    uint32_t q0, q1;
};

// Per-tile prefix (binade lo) and suffix (binade lo+1) counts inside a
// WINDOW stretch: the walker locates the crossing tile with them.
struct WTile {
    Comp pre_lo;   // counts from the stretch start through this tile, binade lo
    Comp suf_hi;   // counts from this tile through the stretch end, binade lo+1
    uint32_t slot; // stored exact p of this tile (window/complex store) or ~0u
    uint32_t pad;
};

__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) {
    const uint32_t s = a + b;
    return s > QSAT ? QSAT : s;
}

// a then b
__device__ __forceinline__ Comp comp_then(Comp a, Comp b) {
    Comp r;
    r.q0 = sat_add(a.q0, (a.q0 & 1u) ? b.q1 : b.q0);
    r.q1 = sat_add(a.q1, (a.q1 & 1u) ? b.q0 : b.q1);
    return r;
}

// Count contributed by p (>= 0, finite) inside binade e.
__device__ __forceinline__ Comp elem_comp(float p, int e) {
    const uint32_t b = __float_as_uint(p);
    const uint32_t E = b >> 23;
    uint32_t mant = b & 0x7FFFFFu;
    int ep;
    if (E == 0) {
        ep = -126;
    } else {
        mant |= 0x800000u;
        ep = (int)E - 127;
    }
    const int d = e - ep;
    if (d < 0) return {QSAT, QSAT};          // p >= 2^(e+1): leaves the binade
    if (d == 0) return {mant, mant};
    if (d > 25) return {0u, 0u};
    const uint32_t qf = mant >> d;
    const uint32_t rem = mant & ((1u << d) - 1u);
    const uint32_t half = 1u << (d - 1);
    if (rem > half) return {qf + 1u, qf + 1u};
    if (rem < half) return {qf, qf};
    return {qf + (qf & 1u), qf + ((qf + 1u) & 1u)};
}

// floor(log2 x), clamped below at -126 (the subnormal grid is binade -126's).
__device__ __forceinline__ int binade_of(double x) {
    if (!(x >= 0x1p-126)) return -126;
    const unsigned long long b = (unsigned long long)__double_as_longlong(x);
    return (int)((b >> 52) & 0x7FF) - 1023;
}

struct SumState {
    int e;        // binade
    uint32_t m;   // s = m * 2^(e-23)
};

__device__ __forceinline__ SumState state_of(float s) {
    const uint32_t b = __float_as_uint(s);
    const uint32_t E = b >> 23;
    if (E == 0) return {-126, b & 0x7FFFFFu};
    return {(int)E - 127, (b & 0x7FFFFFu) | 0x800000u};
}

__device__ __forceinline__ float float_of(SumState st) {
    if (st.e == -126 && st.m < 0x800000u) return __uint_as_float(st.m);
    return __uint_as_float(((uint32_t)(st.e + 127) << 23) | (st.m & 0x7FFFFFu));
}

__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

__device__ __forceinline__ uint32_t warp_incl_scan_u(uint32_t v) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += t;
    }
    return v;
}

// s = fl(...fl(fl(s + p[0]) + p[1])... + p[31]) for 32 values in shared
// memory (16-byte aligned).  Every lane reads them with eight broadcast
// float4 loads and runs the same 32 dependent adds from registers.
__device__ __forceinline__ float seq_add32_smem(float s, const float *p) {
    const float4 *p4 = reinterpret_cast<const float4 *>(p);
    float4 q[8];
#pragma unroll
    for (int k = 0; k < 8; k++) q[k] = p4[k];
#pragma unroll
    for (int k = 0; k < 8; k++) {
        s = __fadd_rn(s, q[k].x);
        s = __fadd_rn(s, q[k].y);
        s = __fadd_rn(s, q[k].z);
        s = __fadd_rn(s, q[k].w);
    }
    return s;
}

// The composite of a warp's 32 lane composites in lane order.  Without ties
// (every count parity-free) and with every count below 2^24, it is a plain
// sum (one warp reduction, below 2^29); otherwise the ordered composition.
// The result is valid in lane 0.
__device__ __forceinline__ Comp warp_comp_reduce(Comp c);
__device__ __forceinline__ Comp warp_tile_comp(Comp c) {
    if (__all_sync(0xffffffffu, c.q0 == c.q1 && c.q0 < QLIM)) {
        const uint32_t q = __reduce_add_sync(0xffffffffu, c.q0);
        return Comp{q, q};
    }
    return warp_comp_reduce(c);
}

// Ordered reduction of lane composites (lane 0 = first element).  Result in lane 0.
__device__ __forceinline__ Comp warp_comp_reduce(Comp c) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        Comp r;
        r.q0 = __shfl_down_sync(0xffffffffu, c.q0, o);
        r.q1 = __shfl_down_sync(0xffffffffu, c.q1, o);
        if ((lane & (2 * o - 1)) == 0) c = comp_then(c, r);
    }
    return c;
}

// raw argmax element: NaN never wins (treated as -inf), ties -> lower index.
struct ArgBest {
    float v;
    uint32_t i;
};
__device__ __forceinline__ ArgBest arg_better(ArgBest a, ArgBest b) {
    if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
    return a;
}
__device__ __forceinline__ ArgBest warp_arg(ArgBest a) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ArgBest b;
        b.v = __shfl_xor_sync(0xffffffffu, a.v, o);
        b.i = __shfl_xor_sync(0xffffffffu, a.i, o);
        a = arg_better(a, b);
    }
    return a;
}

__device__ __forceinline__ float4 ldg_stream(const float4 *p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// The engine's logit prologue (engine.zig:341-354) as applied here: PRO_CAP
// the soft-cap tanh(v / softcap) * softcap, then PRO_SCALE v * pinv (pinv the
// f32 reciprocal of logit_scale).  pro == 0: the logits as given.
enum : uint32_t { PRO_CAP = 1u, PRO_SCALE = 2u };
struct Prologue {
    uint32_t pro;
    float softcap, pinv;
    __device__ __forceinline__ float operator()(float v) const {
        return prologue_ref(v, softcap, (pro & PRO_CAP) != 0u, pinv, (pro & PRO_SCALE) != 0u);
    }
};

// ---------------------------------------------------------------------------
// sampleArgmax (sampler.zig:31-41): one CTA per row, of the logits after the
// prologue (the engine applies it before sampling).
__global__ void __launch_bounds__(512) argmax_kernel(const float *__restrict__ logits, size_t ld,
                                                     uint32_t vocab, uint32_t *__restrict__ out, Prologue pr) {
    const uint32_t row = blockIdx.x;
    const float *x = logits + (size_t)row * ld;
    ArgBest best{NEG_INF, 0xFFFFFFFFu};
    const bool vec = ((reinterpret_cast<uintptr_t>(x) & 15u) == 0);
    uint32_t done = 0;
    if (vec) {
        const uint32_t n4 = vocab / 4;
        const float4 *x4 = reinterpret_cast<const float4 *>(x);
        for (uint32_t i = threadIdx.x; i < n4; i += blockDim.x) {
            const float4 v = ldg_stream(x4 + i);
            float a[4] = {v.x, v.y, v.z, v.w};
            if (pr.pro) {
#pragma unroll
                for (int k = 0; k < 4; k++) a[k] = pr(a[k]);
            }
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float f = a[k] != a[k] ? NEG_INF : a[k];
                best = arg_better(best, ArgBest{f, 4 * i + k});
            }
        }
        done = n4 * 4;
    }
    for (uint32_t i = done + threadIdx.x; i < vocab; i += blockDim.x) {
        const float f = pr.pro ? pr(x[i]) : x[i];
        best = arg_better(best, ArgBest{f != f ? NEG_INF : f, i});
    }
    best = warp_arg(best);
    __shared__ ArgBest wb[16];
    if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgBest b = wb[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) b = arg_better(b, wb[w]);
        const float x0 = pr.pro ? pr(x[0]) : x[0];
        uint32_t r = b.i;
        if (x0 != x0 || b.i == 0xFFFFFFFFu) r = 0;  // leading NaN wins; all -inf -> 0
        out[row] = r;
    }
}

// ---------------------------------------------------------------------------

struct TileParam {   // per-tile values of K2's main loop (16 bytes)
    float K;           // 23 - lo: log2(p / u_lo) = x2 + K
    float fhi, flo;    // 1 +- the certificate's relative error bound
    uint32_t info;     // TP_* flags | cls << 2 | (lo + 128) << 8
};
constexpr uint32_t TP_SPECIAL = 1u;   // counted by the warp-cooperative exact pass
constexpr uint32_t TP_CAND = 2u;      // the tile maximum reaches the candidate floor

struct TileRec {
    int32_t lo;
    uint32_t cls;
    uint32_t aux;
    Comp qlo;
    Comp qhi;
};

// Block-wide exclusive scan of n (<= 2*NT) uint32 in place; returns the total.
template <int NT>
__device__ uint32_t block_exscan_u(uint32_t *a, uint32_t n, uint32_t *wtmp) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t i0 = 2 * tid, i1 = 2 * tid + 1;
    const uint32_t a0 = (tid < NT && i0 < n) ? a[i0] : 0u;
    const uint32_t a1 = (tid < NT && i1 < n) ? a[i1] : 0u;
    uint32_t v = a0 + a1, incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31 && warp < NW) wtmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < NW ? wtmp[lane] : 0u, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < NW) wtmp[lane] = wi - w;
        if (lane == NW - 1) wtmp[NW] = wi;
    }
    __syncthreads();
    if (tid < NT) {
        const uint32_t ex = wtmp[warp] + incl - v;
        if (i0 < n) a[i0] = ex;
        if (i1 < n) a[i1] = ex + a0;
    }
    const uint32_t total = wtmp[NW];
    __syncthreads();
    return total;
}

// Segmented inclusive scan of composites over n (<= 2*NT) elements by the
// first NT threads.  Forward (REV = false): flag[i] starts a segment,
// c[i] <- c[start..i].  Reverse (REV = true): flag[i] ends a segment,
// c[i] <- c[i..end] (composition order is always index order).
struct SegComp {
    uint32_t f;
    Comp c;
};
template <bool REV>
__device__ __forceinline__ SegComp seg_then(SegComp a, SegComp b) {   // a precedes b in scan order
    if (b.f) return b;
    return SegComp{a.f, REV ? comp_then(b.c, a.c) : comp_then(a.c, b.c)};
}
template <bool REV, int NT>
__device__ void block_segscan_comp(Comp *c, const uint32_t *flag, uint32_t n, SegComp *wtmp) {
    constexpr int NW = NT / 32;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t j0 = 2 * tid, j1 = 2 * tid + 1;           // scan order
    const uint32_t i0 = REV ? n - 1 - j0 : j0, i1 = REV ? n - 2 - j0 : j1;   // physical
    const bool act = tid < NT;
    SegComp s0{(act && j0 < n) ? flag[i0] : 1u, (act && j0 < n) ? c[i0] : Comp{0, 0}};
    SegComp s1{(act && j1 < n) ? flag[i1] : 1u, (act && j1 < n) ? c[i1] : Comp{0, 0}};
    SegComp v = seg_then<REV>(s0, s1);
    SegComp incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        SegComp t;
        t.f = __shfl_up_sync(0xffffffffu, incl.f, o);
        t.c.q0 = __shfl_up_sync(0xffffffffu, incl.c.q0, o);
        t.c.q1 = __shfl_up_sync(0xffffffffu, incl.c.q1, o);
        if (lane >= o) incl = seg_then<REV>(t, incl);
    }
    if (lane == 31 && warp < NW) wtmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        SegComp w = lane < NW ? wtmp[lane] : SegComp{0u, {0, 0}};
        SegComp wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            SegComp t;
            t.f = __shfl_up_sync(0xffffffffu, wi.f, o);
            t.c.q0 = __shfl_up_sync(0xffffffffu, wi.c.q0, o);
            t.c.q1 = __shfl_up_sync(0xffffffffu, wi.c.q1, o);
            if (lane >= o) wi = seg_then<REV>(t, wi);
        }
        __syncwarp();
        if (lane < NW) wtmp[NW + 1 + lane] = wi;  // inclusive over warps 0..lane
    }
    __syncthreads();
    SegComp excl_lane;
    {
        SegComp t;
        t.f = __shfl_up_sync(0xffffffffu, incl.f, 1);
        t.c.q0 = __shfl_up_sync(0xffffffffu, incl.c.q0, 1);
        t.c.q1 = __shfl_up_sync(0xffffffffu, incl.c.q1, 1);
        excl_lane = lane > 0 ? t : SegComp{0u, {0, 0}};
    }
    SegComp carry = (warp > 0 && warp <= NW) ? wtmp[NW + 1 + warp - 1] : SegComp{0u, {0, 0}};
    SegComp pre = lane > 0 ? seg_then<REV>(carry, excl_lane) : carry;
    SegComp r0 = seg_then<REV>(pre, s0);
    SegComp r1 = seg_then<REV>(r0, s1);
    __syncthreads();
    if (act && j0 < n) c[i0] = r0.c;
    if (act && j1 < n) c[i1] = r1.c;
    __syncthreads();
}
// ===========================================================================
// Decoupled passes.  A row is cut into segments of SEG_TILES tiles; K1 and K2
// run one CTA per segment with one thread per tile (32 logits in registers).
//   K1 (k1_stats) streams the logits from HBM (L2 evict_first) and writes
//      per-tile maxima and sums (relative to the tile maximum) plus
//      per-segment aggregates and histograms; k1_rows, one CTA per row,
//      reduces them to the row maximum, the prefix estimate at every segment
//      start and the candidate floors (no CTA ever waits for another).
//   K2 (k2_main) re-reads each segment in segment-major order (every row's
//      first segment first), classifies tiles, computes the certified grid
//      counts, writes the walk items and the candidates.
// ===========================================================================
constexpr int SEG_TILES = 256;               // tiles per segment == K1/K2 block size
constexpr int SEG_ELEMS = SEG_TILES * TILE;  // 8192 logits
constexpr int K12_THREADS = SEG_TILES;
constexpr int MAX_SEG = 64;                  // vocab <= 524288
constexpr int KH_BINS = 256;                 // quarter-octave bins over 64 octaves
constexpr int RED_CHUNK = 4;                 // segments per step of the row reduction

// Speculation window of the running sum around the raw prefix estimate: the
// reference's sum lies below the exact prefix (elements under half an ulp are
// dropped) by up to ~2e-3 on flat rows, and above it by rounding noise only.
constexpr double WIN_LO = 4e-3;
constexpr double WIN_HI = 3e-5;

// Typical-p band (sampler.zig:128-154 with typical-p alone): the dev bound is
// chosen on a 1/32-nat grid from the statistics pass's mass histograms,
// assuming |H_raw - H| <= TB_H_REL |H| + TB_H_ABS; the walk checks that
// assumption against the exact H and reports BS_ENOTSUP when it fails.
constexpr int TB_CELLS = 1024;
constexpr double TB_PER_NAT = 32.0;
constexpr double TB_H_REL = 4e-3;
constexpr double TB_H_ABS = 1e-3;
constexpr float TB_MASS_REL = 0.01f;
constexpr float TB_MASS_ABS = 0.005f;
constexpr float TB_D_PAD = 0.01f;
constexpr float TB_OCTAVES = 12.0f;   // band histogram depth below each segment maximum

// Relative error bound, for the main loop's certificate, between
// y = ex2.approx(min(fma(d, c2, K), 17.5)) and the exact p / u_lo, where
// p = exp_ref(fdiv_rn(d, T)), d = fsub_rn(v, M), c2 = fl(log2(e) / T).
// Only elements with y >= 1/2 can count, so |x2| <= K + 1 for them.  Terms
// (relative error of y, natural-log units of the exponent times ln 2):
//   the reference's divide: |x2| ln2 2^-24;  its expf: 2^-23 (one ulp);
//   c2's rounding: |x2| ln2 2^-24;  the FFMA's rounding: 17.5 ln2 2^-24;
//   ex2.approx: 2^-22 (documented 2^-22.5 or better).
// The bound is doubled; the caller also floors it at 2^-17 so that the
// clamped values (y = 2^17.5) always fail the certificate.  The GPU suite
// checks it against the exact count on random inputs (bs_debug_cert_check).
__host__ __device__ __forceinline__ float cert_eps(float K) {
    return 2.0f * ((K + 1.0f) * 8.27e-8f + 1.2e-7f + 7.3e-7f + 2.4e-7f);
}

// The same for the entropy term h = P (-ln P), P = p / S, approximated as
// y = min(ex2.approx(min(z + K, 40)) * (-z ln2), 2^17.5) with
// z = fma(d, c2, -log2 S) ~ log2 P.  zmin: the tile's smallest |z| (its
// largest P; tiles with zmin < 1/16 go to the exact pass), l2s = |log2 S|.
// Elements that can count (y >= 1/2) have |z| <= K + 8, so |x2| <= K + 8 + l2s.
//   reference: P's error eP = (|x| + 3) 2^-24 (divide by T, expf, divide by
//     S) also moves -logf(P) by eP / (zmin ln2) relative; logf's ulp 2^-23;
//     the product's rounding 2^-24;
//   approximation: z's error dz = (|x2| + 2 l2s + K + 8) 2^-24 (log2 units)
//     moves 2^z by ln2 dz and -z by dz / zmin; the add's rounding 40 ln2
//     2^-24; ex2.approx 2^-22; two multiplies and ln2 3 2^-24.
// The bound is doubled; the caller floors it at 2^-17 like cert_eps.
__host__ __device__ __forceinline__ float cert_eps_h(float K, float zmin, float l2s) {
    const float u = 5.9604645e-8f;   // 2^-24
    const float x2m = K + 8.0f + l2s;
    const float eP = (x2m * 0.6931472f + 3.0f) * u;
    const float dz = (x2m + 2.0f * l2s + K + 8.0f) * u;
    const float inv = 1.0f / (zmin * 0.6931472f);
    const float ref = eP * (1.0f + inv) + 2.0f * u + u;
    const float apx = 0.6931472f * dz + dz / zmin + 40.0f * 0.6931472f * u + 4.0f * u + 3.0f * u;
    return 2.0f * (ref + apx);
}

__device__ __forceinline__ double pow2d(int k) {   // 2^k, -1022 <= k <= 1023
    return __longlong_as_double((long long)(k + 1023) << 52);
}

struct TileStat {
    float tmax;   // tile maximum (penalised logits)
    float tsr;    // sum of 2^r over the tile, r = (v - tmax) log2e / T
    float tsr2;   // sum of 2^r r (the entropy estimate's second moment)
    float pad;
};

struct SegStat {
    float smax;        // segment maximum
    uint32_t nonfin;   // a non-finite logit in the segment
    double ssum;       // sum of 2^x over the segment, x = (v - smax) log2e / T
    double base;       // (row reduction) raw prefix estimate at the segment start
    double ssum2;      // sum of 2^x x
};

// Vocabulary sharding: one shard's partial of a row (its maximum, its sum of
// 2^x relative to that maximum, a non-finite flag); 16 bytes.
struct VsPart {
    float m;
    uint32_t nonfin;
    double S;
};

struct RowInfo {   // written by the row reduction, read by the main and walk passes
    float M;
    float xf2;         // candidate floor, log2 p units
    uint32_t binding;  // 0 none (all p > 0), 1 top-k, 2 top-p, 3 min-p, 4 typical top ties
    uint32_t check_nan;
    double S_raw;
    double H_raw;      // typical-p: entropy estimate from the tile statistics
    float dband;       // TYP_BAND: dev bound of the candidate band
    uint32_t tmode;    // TYP_*
};

// Typical-p mode of the configuration (sampler.zig:128-154): off, over a
// selected set bounded by another filter, or alone (band candidates).
__host__ __device__ __forceinline__ uint32_t typical_mode(float typical_p, uint32_t top_k, uint32_t vocab,
                                                          float top_p, float min_p) {
    if (!(typical_p > 0.0f && typical_p < 1.0f)) return TYP_OFF;
    const bool other = (top_k > 0 && top_k < vocab) || (top_p > 0.0f && top_p < 1.0f) || min_p > 0.0f;
    return other ? TYP_SELECTED : TYP_BAND;
}

struct K12Params {
    const float *logits;
    size_t ld;
    const uint32_t *pen_bm;   // per handle row: ntiles_total words, bit k of word t = token 32 t + k is
                              // penalised; nullptr when the repetition penalty is off for this call
    uint32_t vocab;
    uint32_t row0;
    uint32_t rows;
    float T;
    float c2;                 // log2(e) / T (approximate paths only)
    uint32_t top_k;
    float top_p;
    float min_p;
    float rep_penalty;
    float typical_p;
    uint32_t tmode;           // TYP_*
    uint32_t nseg;
    uint32_t ntiles_total;
    TileStat *tstat;          // per handle row: ntiles_total
    SegStat *sstat;           // per handle row: MAX_SEG
    float *mhist;             // per handle row: MAX_SEG x KH_BINS masses
    RowInfo *rinfo;           // per handle row
    RowHdr *hdr;
    Item *items;
    WTile *wpre;
    float *wcdata;
    Candidate *cand;          // per handle row: cand_stride entries (idx, logit)
    uint32_t cand_stride;
    uint32_t *kerr;           // per handle: the call whose bounded device wait gave up
    uint32_t seq;             // this call's sequence number (never 0)
    // logit prologue (engine.zig:341-354): PRO_CAP soft-cap tanh(v / softcap) * softcap,
    // then PRO_SCALE v * pinv
    uint32_t pro;
    float softcap, pinv;
    // vocabulary sharding: the gathered partials of every shard ([world][rows]),
    // or nullptr; this shard's rank
    const VsPart *vs_parts;
    uint32_t vs_world, vs_rank;
    // the partials through peer memory: rank h's partial of row r is valid
    // once vs_ptag[h * rows + r] carries the step's tag (*vs_epoch)
    const unsigned long long *vs_ptag;
    const uint32_t *vs_epoch;
    // persistent kernel (k_fused): task scheduler state of this call
    uint32_t *ctl;            // [0] next statistics task, [1] next main task, [2] ready rows;
                              // then per call row: statistics tasks done; all zeroed before the call
    unsigned long long *ready;   // per slot: (seq << 32) | row once the slot publishes that row's main tasks
};

__device__ __forceinline__ bool penalty_active(const K12Params &P) { return P.pen_bm != nullptr; }

__device__ __forceinline__ Prologue prologue_of(const K12Params &P) { return Prologue{P.pro, P.softcap, P.pinv}; }

// The repetition penalty of one logit (sampler.zig:62-66).
__device__ __forceinline__ float penalize(float a, float pen) {
    return a > 0.0f ? __fdiv_rn(a, pen) : __fmul_rn(a, pen);
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ float4 ldg_policy(const float4 *p, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

// Block-wide (K12_THREADS) exclusive scan of one double per thread.
__device__ double block_exscan1_d(double v, double *wtmp, double *total) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    constexpr int NW = K12_THREADS / 32;
    double incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) wtmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        double w = lane < NW ? wtmp[lane] : 0.0, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < NW) wtmp[lane] = wi - w;
        if (lane == NW - 1) wtmp[NW] = wi;
    }
    __syncthreads();
    const double ex = wtmp[warp] + incl - v;
    *total = wtmp[NW];
    __syncthreads();
    return ex;
}

// Logits g .. g+3 (g a multiple of 4) from global memory (-inf past the
// vocabulary) with the repetition penalty applied to the ids marked in the
// row's bitmap `bm` (nullptr: no penalty).  Not inlined: it is the path for
// rows that cannot be staged in shared memory, and one out-of-line copy keeps
// the staged loops' instruction footprint small.
__device__ __noinline__ float4 load_quad(const float *x, uint32_t g, uint32_t vocab, float rep_penalty, uint64_t pol,
                                         const uint32_t *bm, Prologue pr) {
    float4 q;
    if (g + 4 <= vocab && (reinterpret_cast<uintptr_t>(x + g) & 15u) == 0) {
        q = ldg_policy(reinterpret_cast<const float4 *>(x + g), pol);
    } else {
        q.x = g < vocab ? x[g] : NEG_INF;
        q.y = g + 1 < vocab ? x[g + 1] : NEG_INF;
        q.z = g + 2 < vocab ? x[g + 2] : NEG_INF;
        q.w = g + 3 < vocab ? x[g + 3] : NEG_INF;
    }
    if (pr.pro) {   // the logit prologue comes before the penalty (the engine applies it first)
        q.x = pr(q.x);
        q.y = pr(q.y);
        q.z = pr(q.z);
        q.w = pr(q.w);
    }
    if (bm) {
        const uint32_t bits = (bm[g >> 5] >> (g & 31u)) & 0xFu;
        if (bits & 1u) q.x = penalize(q.x, rep_penalty);
        if (bits & 2u) q.y = penalize(q.y, rep_penalty);
        if (bits & 4u) q.z = penalize(q.z, rep_penalty);
        if (bits & 8u) q.w = penalize(q.w, rep_penalty);
    }
    return q;
}

// The logit prologue on the staged copy of tile `tl` (32 logits at
// sf[32 tl ..]), by the tile's owner thread, before the penalty.
__device__ __forceinline__ void prologue_tile_smem(const K12Params &P, uint32_t tl, float *sf) {
    const Prologue pr = prologue_of(P);
#pragma unroll 4
    for (int k = 0; k < TILE; k++) sf[tl * TILE + k] = pr(sf[tl * TILE + k]);
}

// The repetition penalty on the staged copy of tile `tl` (32 logits at
// sf[32 tl ..]) of segment `seg`: each id marked in the row's bitmap, once.
// Called by the tile's owner thread right after the copy landed.
__device__ __forceinline__ void patch_tile_smem(const K12Params &P, uint32_t hrow, uint32_t seg, uint32_t tl,
                                                float *sf) {
    uint32_t bits = P.pen_bm[(size_t)hrow * P.ntiles_total + seg * SEG_TILES + tl];
    while (bits) {
        const int k = __ffs(bits) - 1;
        bits &= bits - 1u;
        sf[tl * TILE + k] = penalize(sf[tl * TILE + k], P.rep_penalty);
    }
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch: the kernels after the statistics pass are
// launched so that their CTAs may start while the previous kernel drains;
// each waits for its producer's results (all of its memory operations) before
// reading them.  Every kernel lets its dependents launch once all of its CTAs
// have started.  Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------------------
// Segment staging: one bulk copy (cp.async.bulk, global -> shared, completion
// on an mbarrier) of a CTA's 32 KB segment.  Thread t then reduces tile t from
// shared memory, reading its eight float4 in the order j ^ (t & 7) so that the
// eight threads of a quarter-warp hit distinct banks.
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes, uint64_t *bar, uint64_t pol) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// System-scope forms (words another GPU writes or reads over NVLink).
__device__ __forceinline__ unsigned long long ld_acquire_sys_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
constexpr uint64_t PEER_WAIT_NS = 1000000000ull;   // one second for a peer's word
// Waits (one thread) for the word to carry this step's tag: true and its
// 32-bit payload, or false after a second without it (the call's error word
// `seq` then says so).
__device__ bool wait_peer_bits(const unsigned long long *p, uint32_t tag, uint32_t seq, uint32_t *kerr,
                               uint32_t &bits) {
    const uint64_t t0 = global_ns();
    for (uint32_t it = 0;; it++) {
        const unsigned long long v = ld_acquire_sys_u64(p);
        if ((uint32_t)(v >> 32) == tag) {
            bits = (uint32_t)v;
            return true;
        }
        if (global_ns() - t0 > PEER_WAIT_NS || it > (1u << 26)) {
            atomicExch(kerr, seq);
            bits = 0u;
            return false;
        }
        __nanosleep(64);
    }
}
// The f32 payload, or NaN when the wait gave up.
__device__ float wait_peer_word(const unsigned long long *p, uint32_t tag, uint32_t seq, uint32_t *kerr) {
    uint32_t b;
    return wait_peer_bits(p, tag, seq, kerr, b) ? __uint_as_float(b) : __int_as_float(0x7fc00000);
}

// Waits for phase `parity` of the barrier; false once `limit_ns` have passed
// (or after 2^20 tries).  Each try lets the hardware suspend the thread until
// the phase completes or a microsecond passes, so waiting threads do not
// spin on the issue slots the SM's other CTAs need.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < (1u << 20); i++) {
        uint32_t done;
        asm volatile(
            "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
            : "=r"(done)
            : "r"(smem_u32(bar)), "r"(parity), "r"(1000u)
            : "memory");
        if (done) return true;
        if (global_ns() - t0 > limit_ns) return false;
    }
    return false;
}
constexpr uint64_t MBAR_WAIT_NS = 1000000000ull;   // one second

// Per-thread asynchronous global -> shared copies (cp.async).  A thread
// issues all of its copies and then waits once, so a table gathered from many
// places costs one memory latency instead of one per load/store pair.
__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async8(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// The segment can be bulk copied: a 16-byte aligned start and a whole number
// of 16-byte chunks.
__device__ __forceinline__ bool seg_bulk_ok(const float *xs, uint32_t n) {
    return (reinterpret_cast<uintptr_t>(xs) & 15u) == 0 && (n & 3u) == 0;
}

// Issues the segment's bulk copy (thread 0) if it is possible; the caller
// waits with seg_wait.  Returns whether the copy was issued (block-uniform).
__device__ __forceinline__ bool seg_issue(const float *xs, uint32_t n, float4 *sbuf, uint64_t *bar, uint64_t pol) {
    const bool bulk = seg_bulk_ok(xs, n);
    if (bulk && threadIdx.x == 0) {
        // a persistent CTA's earlier task wrote this buffer with ordinary
        // stores (seen by this thread after the task's closing barrier):
        // order them before the copy's asynchronous-proxy writes
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_init(bar, 1);
        bulk_load(sbuf, xs, n * 4u, bar, pol);
    }
    return bulk;
}

// Waits for the copy (bounded).  On a timeout the block loads from global
// memory instead and the handle's error word records the failure; thread 0
// then waits once more (bounded) so that a late copy cannot land in a later
// CTA's shared memory.  Returns whether the shared copy is usable
// (block-uniform).
__device__ __forceinline__ bool seg_wait(const K12Params &P, uint64_t *bar) {
    const bool ok = mbar_wait(bar, 0u, MBAR_WAIT_NS);
    const bool all = __syncthreads_and(ok) != 0;
    if (!all && threadIdx.x == 0) {
        atomicExch(P.kerr, P.seq);
        mbar_wait(bar, 0u, MBAR_WAIT_NS);
    }
    return all;
}

// Tile `tl` of the segment (32 logits, -inf past the vocabulary), from the
// shared copy or, without one, from global memory with the penalty applied.
// The logits come back permuted: v[4 j + c] is element 4 (j ^ (tl & 7)) + c of
// the tile (a register array must be indexed by compile-time constants).
__device__ __forceinline__ uint32_t tile_elem(uint32_t tl, int j, int c) {
    return 4u * ((uint32_t)j ^ (tl & 7u)) + (uint32_t)c;
}
__device__ __forceinline__ void load_tile32(const K12Params &P, const float *x, uint32_t seg, uint32_t tl,
                                            const float4 *sbuf, bool staged, const uint32_t *bm, uint64_t pol,
                                            float v[TILE]) {
    const uint32_t g0 = seg * SEG_ELEMS + tl * TILE;
    if (staged && g0 + TILE <= P.vocab) {   // every tile but the row's last
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 q = sbuf[tl * 8 + ((uint32_t)j ^ (tl & 7u))];
            v[4 * j] = q.x;
            v[4 * j + 1] = q.y;
            v[4 * j + 2] = q.z;
            v[4 * j + 3] = q.w;
        }
    } else if (staged) {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const uint32_t jj = (uint32_t)j ^ (tl & 7u);
            const float4 q = sbuf[tl * 8 + jj];
            const uint32_t g = g0 + 4 * jj;
            v[4 * j] = g < P.vocab ? q.x : NEG_INF;
            v[4 * j + 1] = g + 1 < P.vocab ? q.y : NEG_INF;
            v[4 * j + 2] = g + 2 < P.vocab ? q.z : NEG_INF;
            v[4 * j + 3] = g + 3 < P.vocab ? q.w : NEG_INF;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 q = load_quad(x, g0 + tile_elem(tl, j, 0), P.vocab, P.rep_penalty, pol, bm, prologue_of(P));
            v[4 * j] = q.x;
            v[4 * j + 1] = q.y;
            v[4 * j + 2] = q.z;
            v[4 * j + 3] = q.w;
        }
    }
}

// Chunk j of tile `tl` (logits 4 (j ^ (tl & 7)) .. +3, -inf past the
// vocabulary), from the shared copy or from global memory.
__device__ __forceinline__ float4 tile_quad(const K12Params &P, const float *x, uint32_t seg, uint32_t tl, int j,
                                            const float4 *sbuf, bool staged, const uint32_t *bm, uint64_t pol) {
    const uint32_t g = seg * SEG_ELEMS + tl * TILE + tile_elem(tl, j, 0);
    if (!staged) return load_quad(x, g, P.vocab, P.rep_penalty, pol, bm, prologue_of(P));
    float4 q = sbuf[tl * 8 + ((uint32_t)j ^ (tl & 7u))];
    if (g + 4 > P.vocab) {
        q.x = g < P.vocab ? q.x : NEG_INF;
        q.y = g + 1 < P.vocab ? q.y : NEG_INF;
        q.z = g + 2 < P.vocab ? q.z : NEG_INF;
        q.w = g + 3 < P.vocab ? q.w : NEG_INF;
    }
    return q;
}

// ---------------------------------------------------------------------------
// K1: tile statistics of one segment per CTA (the HBM pass).  Per tile: the
// maximum and the sum of 2^((v - tile max) log2e / T); per segment: the
// maximum, the sum relative to it, a non-finite flag and, for top-p without a
// top-k floor, the tail-element histogram.  No cross-CTA step: the row
// reduction is k1_rows.
// Shared memory of one statistics task (segment `seg` of row `row`).
struct __align__(16) StatsSmem {
    uint32_t mh[KH_BINS];                // tail element counts per bin
    float th[KH_BINS];                   // typical band: mass per bin
    float wm[K12_THREADS / 32];
    uint32_t wf[K12_THREADS / 32];
    double wd[K12_THREADS / 32], wd2[K12_THREADS / 32];
};

// `sbuf` (SEG_ELEMS floats of shared memory, 16-byte aligned) receives the
// segment; returns whether it was staged there, with the prologue and the
// penalty applied (block-uniform), so that a main task of the same segment
// on the same CTA can run from it.
__device__ __forceinline__ bool stats_task(const K12Params &P, uint32_t seg, uint32_t row, StatsSmem &ss_,
                                           float4 *const sbuf, uint64_t *barp) {
    const uint32_t hrow = P.row0 + row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = K12_THREADS / 32;
    const float *x = P.logits + (size_t)row * P.ld;
    const float c2 = P.c2;
    const uint32_t ntile = min((uint32_t)SEG_TILES, P.ntiles_total - seg * SEG_TILES);
    const uint32_t nseg_el = min((uint32_t)SEG_ELEMS, P.vocab - seg * SEG_ELEMS);
    uint64_t &bar = *barp;
    uint32_t *const mh = ss_.mh;
    float *const th = ss_.th;
    float *const wm = ss_.wm;
    uint32_t *const wf = ss_.wf;
    double *const wd = ss_.wd;
    double *const wd2 = ss_.wd2;
    // the logits stream through L2 once here: marked evict-first, they do not
    // push out what later kernels reuse (their code, the tile statistics)
    const uint64_t pol = l2_policy_evict_first();
    const bool bulk = seg_issue(x + seg * SEG_ELEMS, nseg_el, sbuf, &bar, pol);
    const uint32_t *bm = penalty_active(P) ? P.pen_bm + (size_t)hrow * P.ntiles_total : nullptr;
    const bool k_floor = P.top_k > 0 && P.top_k < P.vocab && P.top_k <= KSEL_MAX;
    const bool p_active = P.top_p > 0.0f && P.top_p < 1.0f;
    const double p_margin = fmax(2e-3, 0.05 * (1.0 - (double)P.top_p));
    const bool p_floor = p_active && (1.0 - (double)P.top_p) > 2.0 * p_margin && !k_floor;
    const bool t_band = P.tmode == TYP_BAND;
    if (p_floor)
        for (uint32_t b = tid; b < KH_BINS; b += K12_THREADS) mh[b] = 0u;
    if (t_band)
        for (uint32_t b = tid; b < KH_BINS; b += K12_THREADS) th[b] = 0.0f;
    __syncthreads();   // the barrier's initialisation, mh, th
    const bool staged = bulk && seg_wait(P, &bar);

    const bool live = (uint32_t)tid < ntile;
    // the prologue and the penalty on this thread's own staged tile (read
    // back by it alone)
    if (staged && P.pro && live) prologue_tile_smem(P, tid, reinterpret_cast<float *>(sbuf));
    if (staged && bm && live) patch_tile_smem(P, hrow, seg, tid, reinterpret_cast<float *>(sbuf));
    float v[TILE];
    load_tile32(P, x, seg, live ? tid : 0u, sbuf, staged, bm, pol, v);
    float tm = NEG_INF;
#pragma unroll
    for (int k = 0; k < TILE; k++) tm = fmaxf(tm, v[k]);
    float s = 0.0f, s2 = 0.0f;
    if (live && tm > NEG_INF) {
        const float tc = tm * c2;
        if (P.tmode == TYP_OFF) {
#pragma unroll
            for (int k = 0; k < TILE; k++) s += ex2_approx(fmaf(v[k], c2, -tc));
        } else {
#pragma unroll
            for (int k = 0; k < TILE; k++) {
                const float r = fmaf(v[k], c2, -tc);
                const float e = ex2_approx(r);
                s += e;
                s2 = fmaf(e, fmaxf(r, -1e30f), s2);   // 2^r r (0 for -inf logits)
            }
        }
    }
    uint32_t nonfin = 0;
    if (live) {
        // a non-finite logit may make the sum NaN: +inf shows in the tile
        // maximum, a NaN (and -inf with T = +inf) in the tile sum
        nonfin = (!(fabsf(tm) <= 3.4028235e38f) || s != s) ? 1u : 0u;
        if (s != s) s = 0.0f;
        if (s2 != s2) s2 = 0.0f;
        P.tstat[(size_t)hrow * P.ntiles_total + seg * SEG_TILES + tid] = TileStat{tm, s, s2, 0.0f};
    } else {
        tm = NEG_INF;
    }
    float smax = warp_max(tm);
    nonfin = __any_sync(0xffffffffu, nonfin != 0) ? 1u : 0u;
    if (lane == 0) {
        wm[warp] = smax;
        wf[warp] = nonfin;
    }
    __syncthreads();
    float sm = wm[0];
    uint32_t nfs = wf[0];
#pragma unroll
    for (int w = 1; w < NW; w++) {
        sm = fmaxf(sm, wm[w]);
        nfs |= wf[w];
    }
    // segment sums relative to the segment maximum
    double ss = 0.0, ss2 = 0.0;
    if (live && tm > NEG_INF) {
        const float o = (tm - sm) * c2;
        const double et = (double)ex2_approx(o);
        ss = (double)s * et;
        ss2 = et * ((double)s2 + (double)o * (double)s);
    }
    // typical-p alone: mass per quarter-octave below the segment maximum.
    // The band needs only a lower bound of mass, so logits more than
    // TB_OCTAVES below the segment maximum are left out (their mass is at
    // most 2^-TB_OCTAVES of the maximum's each); a tile whose maximum is that
    // low is skipped whole
    if (t_band && sm > NEG_INF && live && (tm - sm) * c2 > -TB_OCTAVES) {
        const float sc = sm * c2;
#pragma unroll
        for (int k = 0; k < TILE; k++) {
            const float xr = fmaf(v[k], c2, -sc);
            if (xr > -TB_OCTAVES) atomicAdd(&th[min(KH_BINS - 1, (int)(-xr * 4.0f))], ex2_approx(xr));
        }
    }
    // top-p without a top-k floor: tail-element histogram relative to the
    // segment maximum
    if (p_floor && sm > NEG_INF && live) {
        const float sc = sm * c2;
#pragma unroll
        for (int k = 0; k < TILE; k++) {
            const float xr = fmaf(v[k], c2, -sc);   // log2(p / p(segment max))
            if (xr > -64.0f) atomicAdd(&mh[min(KH_BINS - 1, (int)(-xr * 4.0f))], 1u);
        }
    }
    ss = warp_sum_d(ss);
    ss2 = warp_sum_d(ss2);
    if (lane == 0) {
        wd[warp] = ss;
        wd2[warp] = ss2;
    }
    __syncthreads();
    if (tid == 0) {
        double sacc = 0.0, sacc2 = 0.0;
        for (int w = 0; w < NW; w++) {
            sacc += wd[w];
            sacc2 += wd2[w];
        }
        SegStat st;
        st.smax = sm;
        st.nonfin = nfs;
        st.ssum = sacc;
        st.base = 0.0;
        st.ssum2 = sacc2;
        P.sstat[(size_t)hrow * MAX_SEG + seg] = st;
    }
    if (p_floor)
        for (uint32_t b = tid; b < KH_BINS; b += K12_THREADS)   // mass bound: count x the bin's upper edge
            P.mhist[((size_t)hrow * MAX_SEG + seg) * KH_BINS + b] = (float)mh[b] * exp2f(-0.25f * (float)b);
    if (t_band)
        for (uint32_t b = tid; b < KH_BINS; b += K12_THREADS) P.mhist[((size_t)hrow * MAX_SEG + seg) * KH_BINS + b] = th[b];
    return staged;
}

__global__ void __launch_bounds__(K12_THREADS, 5) k1_stats(K12Params P) {
    __shared__ __align__(128) float4 sbuf[SEG_ELEMS / 4];
    __shared__ StatsSmem sm;
    __shared__ __align__(8) uint64_t bar;
    grid_dep_launch();
    stats_task(P, blockIdx.x, blockIdx.y, sm, sbuf, &bar);
}

// Row reduction, one CTA per row: the row maximum M, the raw prefix estimate
// at every segment start, and the candidate floor (log2 p relative to M):
//   top-k: from the tile maxima, binned by quarter octaves below M: the
//     first bin edge with at least k tiles above it (so at least k logits);
//   top-p without top-k: from the segments' tail-element histograms (a
//     bound on the mass below each grid point);
//   min-p: ln(min_p) in log2 units, minus a margin.
// Shared memory of one row reduction.
struct __align__(16) RowsSmem {
    float off[MAX_SEG];   // (segment max - M) log2e / T
    float ssc[MAX_SEG];   // segment tail mass scale 2^off
    RowInfo ri;
    uint32_t kh[KH_BINS];
    int kj_w[K12_THREADS / 32], pj_w[K12_THREADS / 32];
    float dh[TB_CELLS];
    float cumm[RED_CHUNK * KH_BINS];
    float mtot[RED_CHUNK];
};

// Loads of data another CTA of the same grid wrote (the persistent kernel's
// tasks): through L2, never from a possibly stale L1 line.
__device__ __forceinline__ SegStat ld_segstat(const SegStat *p) {
    SegStat st;
    st.smax = __ldcg(&p->smax);
    st.nonfin = __ldcg(&p->nonfin);
    st.ssum = __ldcg(&p->ssum);
    st.base = __ldcg(&p->base);
    st.ssum2 = __ldcg(&p->ssum2);
    return st;
}
__device__ __forceinline__ TileStat ld_tilestat(const TileStat *p) {
    const float4 v = __ldcg(reinterpret_cast<const float4 *>(p));
    return TileStat{v.x, v.y, v.z, v.w};
}

__device__ __forceinline__ void rows_task(const K12Params &P, uint32_t row, RowsSmem &rs_) {
    const uint32_t hrow = P.row0 + row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = K12_THREADS / 32;
    const float c2 = P.c2;
    const bool k_floor = P.top_k > 0 && P.top_k < P.vocab && P.top_k <= KSEL_MAX;
    const bool p_active = P.top_p > 0.0f && P.top_p < 1.0f;
    const double p_margin = fmax(2e-3, 0.05 * (1.0 - (double)P.top_p));
    const bool p_floor = p_active && (1.0 - (double)P.top_p) > 2.0 * p_margin && !k_floor;

    float *const off = rs_.off;
    float *const ssc = rs_.ssc;
    RowInfo &ri = rs_.ri;
    uint32_t *const kh = rs_.kh;
    int *const kj_w = rs_.kj_w;
    int *const pj_w = rs_.pj_w;
    const SegStat *S = P.sstat + (size_t)hrow * MAX_SEG;
    const uint32_t ns = P.nseg;
    for (uint32_t b = tid; b < KH_BINS; b += K12_THREADS) kh[b] = 0u;
    // top-k: every thread requests its first tile maxima now, so that their
    // loads overlap the row reduction below
    constexpr int KT = 16;
    const TileStat *ts = P.tstat + (size_t)hrow * P.ntiles_total;
    float tmv[KT];
    if (k_floor) {
#pragma unroll
        for (int k = 0; k < KT; k++) {
            const uint32_t t = (uint32_t)k * K12_THREADS + tid;
            tmv[k] = t < P.ntiles_total ? __ldcg(&ts[t].tmax) : NEG_INF;
        }
    }
    if (warp == 0) {
        float m = NEG_INF;
        uint32_t nf = 0;
        for (uint32_t c = lane; c < ns; c += 32) {
            const SegStat st = ld_segstat(S + c);
            m = fmaxf(m, st.smax);
            nf |= st.nonfin;
        }
        m = warp_max(m);
        nf = __any_sync(0xffffffffu, nf != 0) ? 1u : 0u;
        // raw prefix at each segment start, in units of p(M) = 1
        double run = 0.0, vs_after = 0.0;
        if (P.vs_parts) {
            // a vocabulary shard: the row maximum over all shards, and the
            // estimate of the lower-index shards' mass at this shard's start
            if (P.vs_ptag) {   // lane h waits for rank h's partial of this row
                const uint32_t tag = *P.vs_epoch;
                for (uint32_t h = lane; h < P.vs_world; h += 32) {
                    uint32_t b;
                    wait_peer_bits(P.vs_ptag + (size_t)h * P.rows + row, tag, P.seq, P.kerr, b);
                }
            }
            float gm = NEG_INF;
            uint32_t gnf = 0;
            for (uint32_t h = lane; h < P.vs_world; h += 32) {
                const VsPart q = P.vs_parts[(size_t)h * P.rows + row];
                gm = fmaxf(gm, q.m);
                gnf |= q.nonfin;
            }
            m = warp_max(gm);
            nf = __any_sync(0xffffffffu, gnf != 0) ? 1u : 0u;
            double before = 0.0, after = 0.0;
            for (uint32_t h = lane; h < P.vs_world; h += 32) {
                const VsPart q = P.vs_parts[(size_t)h * P.rows + row];
                const double v = q.m > NEG_INF ? q.S * (double)ex2_approx((q.m - m) * c2) : 0.0;
                if (h < P.vs_rank) before += v;
                if (h > P.vs_rank) after += v;
            }
            run = warp_sum_d(before);
            vs_after = warp_sum_d(after);
        }
        for (uint32_t c0 = 0; c0 < ns; c0 += 32) {
            const uint32_t c = c0 + lane;
            double sv = 0.0;
            float o = NEG_INF;
            if (c < ns) {
                const SegStat st = ld_segstat(S + c);
                o = (st.smax > NEG_INF) ? (st.smax - m) * c2 : NEG_INF;
                sv = st.smax > NEG_INF ? st.ssum * (double)ex2_approx(o) : 0.0;
                off[c] = o;
                ssc[c] = ex2_approx(o);
            }
            double incl = sv;
#pragma unroll
            for (int k = 1; k < 32; k <<= 1) {
                const double u = __shfl_up_sync(0xffffffffu, incl, k);
                if (lane >= k) incl += u;
            }
            if (c < ns) P.sstat[(size_t)hrow * MAX_SEG + c].base = run + incl - sv;
            run += __shfl_sync(0xffffffffu, incl, 31);
        }
        // entropy estimate (typical-p alone): H = ln S - ln2 sum(e x) / S,
        // e = 2^x, x = (v - M) log2e / T
        double e2 = 0.0;
        if (P.tmode == TYP_BAND) {
            for (uint32_t c = lane; c < ns; c += 32) {
                const SegStat st = ld_segstat(S + c);
                if (st.smax > NEG_INF) {
                    const double o = (double)((st.smax - m) * c2);
                    e2 += (double)ex2_approx((float)o) * (st.ssum2 + o * st.ssum);
                }
            }
            e2 = warp_sum_d(e2);
        }
        if (lane == 0) {
            ri.M = m;
            ri.check_nan = nf | ((P.T != P.T) ? 1u : 0u);
            ri.S_raw = run + vs_after;
            ri.H_raw = (P.tmode == TYP_BAND && run > 0.0) ? log(run) - 0.6931471805599453 * e2 / run : 0.0;
            ri.dband = __int_as_float(0x7f800000);
            ri.tmode = P.tmode;
        }
    }
    __syncthreads();
    const float M = ri.M;
    // typical-p alone: the smallest dev bound d whose band [H - d, H + d] of
    // surprise surely holds more than typical_p of the mass.  Each source bin
    // (segment c, quarter-octave b) lies wholly inside the band once
    // d >= max(H_hi - s_lo, s_hi - H_lo); those d are histogrammed by mass.
    if (P.tmode == TYP_BAND && ri.S_raw > 0.0) {
        float *const dh = rs_.dh;
        for (uint32_t j = tid; j < TB_CELLS; j += K12_THREADS) dh[j] = 0.0f;
        __syncthreads();
        const double lnS = log(ri.S_raw), H = ri.H_raw;
        const double dH = TB_H_REL * fabs(H) + TB_H_ABS;   // assumed bound on |H_raw - H|
        const float *TH = P.mhist + (size_t)hrow * MAX_SEG * KH_BINS;
        for (uint32_t i = tid; i < ns * KH_BINS; i += K12_THREADS) {
            const uint32_t c = i / KH_BINS, b = i - c * KH_BINS;
            const float o = off[c];
            const float mass = __ldcg(TH + i);
            if (!(o > NEG_INF) || !(mass > 0.0f)) continue;
            const double xs_hi = (double)o - 0.25 * (double)b, xs_lo = (double)o - 0.25 * (double)(b + 1);
            const double s_lo = lnS - xs_hi * 0.6931471805599453, s_hi = lnS - xs_lo * 0.6931471805599453;
            const double d = fmax(fmax((H + dH) - s_lo, s_hi - (H - dH)), 0.0);
            const int cell = (int)fmin(ceil(d * TB_PER_NAT), (double)(TB_CELLS - 1));
            atomicAdd(&dh[cell], (float)((double)mass * (double)ssc[c] / ri.S_raw));
        }
        __syncthreads();
        if (warp == 0) {
            // first cell whose cumulative (lower-bound) mass reaches the target
            const float target = P.typical_p * (1.0f + TB_MASS_REL) + TB_MASS_ABS;
            float run2 = 0.0f;
            int found = -1;
            for (uint32_t j0 = 0; j0 < TB_CELLS && found < 0; j0 += 32) {
                const float v = dh[j0 + lane];
                float incl = v;
#pragma unroll
                for (int o2 = 1; o2 < 32; o2 <<= 1) {
                    const float t = __shfl_up_sync(0xffffffffu, incl, o2);
                    if (lane >= o2) incl += t;
                }
                const uint32_t hit = __ballot_sync(0xffffffffu, run2 + incl >= target);
                if (hit) found = (int)(j0 + __ffs(hit) - 1);
                run2 += __shfl_sync(0xffffffffu, incl, 31);
            }
            if (lane == 0 && found >= 0 && found < TB_CELLS - 1)
                ri.dband = (float)(found + 1) / (float)TB_PER_NAT + TB_D_PAD;
        }
        __syncthreads();
    }
    // top-k: tile maxima per quarter-octave bin below M (the same x2 as the
    // main pass's per-logit candidate test, which is monotone in the logit)
    uint32_t kcount = 0;   // tiles whose maximum is above the bin edge -(tid+1)/4
    if (k_floor) {
        // all of a thread's tile maxima are requested before the first atomic
        // (the first KT were requested before the row reduction)
        for (uint32_t t0 = 0; t0 < P.ntiles_total; t0 += KT * K12_THREADS) {
            if (t0 > 0) {
#pragma unroll
                for (int k = 0; k < KT; k++) {
                    const uint32_t t = t0 + (uint32_t)k * K12_THREADS + tid;
                    tmv[k] = t < P.ntiles_total ? __ldcg(&ts[t].tmax) : NEG_INF;
                }
            }
#pragma unroll
            for (int k = 0; k < KT; k++) {
                const float d = __fsub_rn(tmv[k], M);
                const float x2 = (d == 0.0f) ? 0.0f : d * c2;
                if (x2 > -64.0f) atomicAdd(&kh[min(KH_BINS - 1, (int)(-x2 * 4.0f))], 1u);
            }
        }
        __syncthreads();
        // inclusive prefix over bins 0..tid (bins hold x2 in (-(b+1)/4, -b/4])
        const uint32_t v = kh[tid];
        const uint32_t incl = warp_incl_scan_u(v);
        if (lane == 31) kj_w[warp] = (int)incl;
        __syncthreads();
        uint32_t base = 0;
        for (int w = 0; w < warp; w++) base += (uint32_t)kj_w[w];
        kcount = base + incl;
        __syncthreads();
    }
    // top-p without top-k: mass possibly below the grid point f_j = -j/4.
    // Segment c's bin b spans [off_c - (b+1)/4, off_c - b/4).  Segments are
    // processed in chunks of RED_CHUNK: one warp per segment turns its
    // histogram into a cumulative one in shared memory, then thread j
    // accumulates grid point j.
    float *const cumm = rs_.cumm;
    float *const mtot = rs_.mtot;
    const float *MH = P.mhist + (size_t)hrow * MAX_SEG * KH_BINS;
    float mbelow = 0.0f;   // mass possibly below f_j (over-count), units of p(M)
    if (p_floor) {
        for (uint32_t c0 = 0; c0 < ns; c0 += RED_CHUNK) {
            const uint32_t nc = min((uint32_t)RED_CHUNK, ns - c0);
            __syncthreads();
            for (uint32_t cc = warp; cc < nc; cc += NW) {
                const uint32_t c = c0 + cc;
                float mc[8];
                float ms = 0.0f;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    ms += __ldcg(MH + (size_t)c * KH_BINS + lane * 8 + j);
                    mc[j] = ms;
                }
                float mi = ms;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float w2 = __shfl_up_sync(0xffffffffu, mi, o);
                    if (lane >= o) mi += w2;
                }
#pragma unroll
                for (int j = 0; j < 8; j++) cumm[cc * KH_BINS + lane * 8 + j] = mc[j] + mi - ms;
                if (lane == 31) mtot[cc] = mi;
            }
            __syncthreads();
            for (uint32_t cc = 0; cc < nc; cc++) {
                const float o = off[c0 + cc];
                if (!(o > NEG_INF)) continue;
                // bins entirely above f_j: b <= floor(4 o) + j - 1
                const float fb = floorf(4.0f * o);
                const int bmax = fb < -1e6f ? -1 : min(KH_BINS - 1, (int)fb + tid - 1);
                const float ma = bmax >= 0 ? cumm[cc * KH_BINS + bmax] : 0.0f;
                // mass below -64 octaves of the segment maximum is not binned:
                // at most SEG_ELEMS * 2^-64 of it
                mbelow += (mtot[cc] - ma + 4.4e-16f) * ssc[c0 + cc];
            }
        }
    }
    const uint32_t kmask = __ballot_sync(0xffffffffu, kcount >= P.top_k);
    const double budget = (1.0 - (double)P.top_p - p_margin) * fmax(1.0, 0.99 * ri.S_raw);
    const uint32_t pmask = __ballot_sync(0xffffffffu, (double)mbelow * 1.01 + 1e-30 <= budget);
    if (lane == 0) {
        kj_w[warp] = kmask ? warp * 32 + __ffs(kmask) - 1 : 1 << 20;
        pj_w[warp] = pmask ? warp * 32 + __ffs(pmask) - 1 : 1 << 20;
    }
    __syncthreads();
    if (tid == 0) {
        int kj = 1 << 20, pj = 1 << 20;
        for (int w = 0; w < NW; w++) {
            kj = min(kj, kj_w[w]);
            pj = min(pj, pj_w[w]);
        }
        float xf2 = -150.01f;   // every p > 0
        uint32_t binding = 0;
        if (k_floor && kj < KH_BINS) {
            // at least top_k tiles have their maximum above -(kj+1)/4
            const float xk = -(float)(kj + 1) * 0.25f - 1e-3f;
            if (xk > xf2) { xf2 = xk; binding = 1; }
        }
        if (p_floor && pj < KH_BINS) {
            const float xp = -(float)pj * 0.25f - 1e-3f;
            if (xp > xf2) { xf2 = xp; binding = 2; }
        }
        if (P.min_p > 0.0f) {
            const float xm = fminf(0.0f, log2f(P.min_p)) - 0.01f;
            if (xm > xf2) { xf2 = xm; binding = 3; }
        }
        if (P.tmode == TYP_BAND) {
            // the probability order only matters for indices[0] (ties at the top)
            xf2 = -0.01f;
            binding = 4;
        }
        RowInfo r = ri;
        r.xf2 = xf2;
        r.binding = binding;
        P.rinfo[hrow] = r;
        RowHdr *hdr = P.hdr + hrow;
        hdr->M = r.M;
        hdr->v_floor = xf2;
        hdr->binding = binding;
        hdr->s_approx = (float)r.S_raw;
        hdr->n_cand = 0;
        hdr->n_wc = 0;
        hdr->flags = 0;
        hdr->nseg = ns;
    }
}

__global__ void __launch_bounds__(K12_THREADS) k1_rows(K12Params P) {
    __shared__ RowsSmem rs;
    grid_dep_wait();     // the statistics pass's results
    grid_dep_launch();   // after the wait: the main pass may read the statistics before its own wait
    rows_task(P, blockIdx.x, rs);
}

// ---------------------------------------------------------------------------
// K2: classification, certified grid counts, candidates, walk items.
// TERM_P: the terms p_i of the normaliser S (sampler.zig:83-88).
// TERM_H: the terms h_i of the entropy H (sampler.zig:130-133), after S is
// known; only for typical-p rows whose token is not yet final.
enum : int { TERM_P = 0, TERM_H = 1 };

// Shared memory of one main-pass task (segment `seg` of row `row`).
constexpr uint32_t RC_CAP = 512;   // uncertified terms recounted one per thread (entropy pass)
struct __align__(16) MainSmem {
    TileRec rec[SEG_TILES];
    double wtmp_d[K12_THREADS / 32 + 1];
    double hbase;
    SegComp wtmp_s[2 * (K12_THREADS / 32) + 2];
    uint32_t wtmp_u[K12_THREADS / 32 + 1];
    uint32_t wlist[SEG_TILES];
    uint16_t rcl[RC_CAP];               // (tile << 5) | element
    uint32_t nrc, rc_fb[SEG_TILES / 32];
    uint32_t nlist, nanflag;
    uint32_t wuni[K12_THREADS / 32];
    uint32_t wsum_u[K12_THREADS / 32];
    uint64_t ch_a[K12_THREADS / 32], ch_b[K12_THREADS / 32];
    uint32_t ch_heads[K12_THREADS / 32], ch_start[K12_THREADS / 32];
};

__device__ __forceinline__ RowInfo ld_rowinfo(const RowInfo *p) {
    RowInfo r;
    r.M = __ldcg(&p->M);
    r.xf2 = __ldcg(&p->xf2);
    r.binding = __ldcg(&p->binding);
    r.check_nan = __ldcg(&p->check_nan);
    r.S_raw = __ldcg(&p->S_raw);
    r.H_raw = __ldcg(&p->H_raw);
    r.dband = __ldcg(&p->dband);
    r.tmode = __ldcg(&p->tmode);
    return r;
}

// `sbuf` (SEG_ELEMS floats of shared memory, 16-byte aligned) holds the
// segment's logits, later the item phase's arrays.  `pre`: the statistics
// task of this segment left it staged there, prologue and penalty applied.
template <int TERM>
__device__ __forceinline__ void main_task(const K12Params &P, uint32_t seg, uint32_t row, MainSmem &ms_,
                                          float4 *const sbuf, uint64_t *barp, bool pre = false) {
    const uint32_t hrow = P.row0 + row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NW = K12_THREADS / 32;
    const uint32_t ntile = min((uint32_t)SEG_TILES, P.ntiles_total - seg * SEG_TILES);
    const bool live = (uint32_t)tid < ntile;   // thread-per-tile phases below
    grid_dep_launch();
    const float *x = P.logits + (size_t)row * P.ld;
    const float c2 = P.c2, T = P.T;
    RowHdr *hdr = P.hdr + hrow;

    double *const wtmp_d = ms_.wtmp_d;
    double &hbase = ms_.hbase;
    uint32_t *const wtmp_u = ms_.wtmp_u;
    SegComp *const wtmp_s = ms_.wtmp_s;
    TileRec *const rec = ms_.rec;
    uint64_t &bar = *barp;
    // the item phase's arrays reuse the segment copy, which is dead by then
    // (6 KB less shared memory per CTA: five CTAs fit an SM instead of four)
    uint32_t *const uarr = reinterpret_cast<uint32_t *>(sbuf);
    uint32_t *const uarr2 = uarr + SEG_TILES;
    Comp *const carr = reinterpret_cast<Comp *>(uarr2 + SEG_TILES);   // 8-byte aligned: read as uint64_t too
    Comp *const carr2 = carr + SEG_TILES;
    uint32_t *const wlist = ms_.wlist;
    // uncertified terms of SIMPLE tiles, recounted exactly one per thread:
    // (tile << 5) | element, and the tiles that still need the warp pass
    uint16_t *const rcl = ms_.rcl;
    uint32_t &nrc = ms_.nrc;
    uint32_t *const rc_fb = ms_.rc_fb;
    uint32_t &nlist = ms_.nlist, &nanflag = ms_.nanflag;
    // the segment's bulk copy overlaps the prologue (and, for the normaliser,
    // the wait for the row reduction: it needs only the logits); it is read
    // once more only by the exact pass, so it need not stay in L2
    const uint64_t pol = l2_policy_evict_first();
    const uint32_t nseg_el = min((uint32_t)SEG_ELEMS, P.vocab - seg * SEG_ELEMS);
    const uint32_t *bm = penalty_active(P) ? P.pen_bm + (size_t)hrow * P.ntiles_total : nullptr;
    bool bulk = false;
    if (TERM == TERM_P && !pre) bulk = seg_issue(x + seg * SEG_ELEMS, nseg_el, sbuf, &bar, pol);
    // the tile statistics come from the statistics pass, complete before this
    // grid could start (the row reduction lets it launch only after its own
    // wait): load them before waiting for the row reduction
    TileStat ts_pre = TileStat{NEG_INF, 0.0f, 0.0f, 0.0f};
    if (live) ts_pre = ld_tilestat(P.tstat + (size_t)hrow * P.ntiles_total + seg * SEG_TILES + tid);
    grid_dep_wait();   // the row reduction (and, for the entropy, the normaliser's walk)
    const RowInfo ri = ld_rowinfo(P.rinfo + hrow);
    // the segment's prefix estimate, requested with the row's information
    // (one round trip for both)
    const double base_p = TERM == TERM_P ? __ldcg(&P.sstat[(size_t)hrow * MAX_SEG + seg].base) : 0.0;
    const float M = ri.M;
    if (TERM == TERM_H && __ldcg(&hdr->tdone)) return;   // the row's token is already final
    if (TERM == TERM_H) bulk = seg_issue(x + seg * SEG_ELEMS, nseg_el, sbuf, &bar, pol);
    // the entropy pass: S exact, log2 S for the terms' exponents
    const float S = TERM == TERM_H ? __ldcg(&hdr->S_exact) : 1.0f;
    const double lnS = TERM == TERM_H ? log((double)S) : 0.0;
    const float l2S = (float)(lnS * 1.4426950408889634);
    if (tid == 0) {
        nlist = 0;
        nanflag = 0;
        nrc = 0;
    }
    if ((uint32_t)tid < SEG_TILES / 32) rc_fb[tid] = 0u;

    // raw prefix estimate at every tile start of the segment, and from it
    // each tile's candidate binades of the running sum and its main-loop
    // parameters (thread t owns tile t)
    const float xf2 = ri.xf2;
    const bool band = TERM == TERM_H && ri.tmode == TYP_BAND;
    const float Hr = (float)ri.H_raw, dband = ri.dband;
    TileParam tp;
    {
        double ct = 0.0;
        float tmax = NEG_INF;
        if (live) {
            const TileStat ts = ts_pre;
            tmax = ts.tmax;
            if (ts.tmax > NEG_INF) {
                const float o = (ts.tmax - M) * c2;
                const double et = (double)ex2_approx(o);
                if (TERM == TERM_P) {
                    ct = (double)ts.tsr * et;
                } else {   // sum of P (-ln P) = 2^o (ln S tsr - ln2 (tsr2 + o tsr)) / S
                    ct = fmax(0.0, et * (lnS * ts.tsr - 0.6931471805599453 * ((double)ts.tsr2 + (double)o * ts.tsr)) /
                                       (double)S);
                }
            }
        }
        double base;
        if (TERM == TERM_P) {
            base = base_p;
        } else {
            // entropy mass of the earlier segments, from their statistics
            if (warp == 0) {
                double hb = 0.0;
                for (uint32_t c = lane; c < seg; c += 32) {
                    const SegStat st = ld_segstat(P.sstat + (size_t)hrow * MAX_SEG + c);
                    if (st.smax > NEG_INF) {
                        const double o = (double)((st.smax - M) * c2);
                        hb += fmax(0.0, (double)ex2_approx((float)o) *
                                            (lnS * st.ssum - 0.6931471805599453 * (st.ssum2 + o * st.ssum)) /
                                            (double)S);
                    }
                }
                hb = warp_sum_d(hb);
                if (lane == 0) hbase = hb;
            }
            __syncthreads();
            base = hbase;
        }
        double segtot;
        const double Ps = base + block_exscan1_d(ct, wtmp_d, &segtot);
        const double Pe = Ps + ct;
        const int lo = binade_of(Ps * (1.0 - WIN_LO));
        const int hi = binade_of(Pe * (1.0 + WIN_HI));
        const uint32_t cls = hi == lo ? CLS_SIMPLE : (hi == lo + 1 ? CLS_WINDOW : CLS_COMPLEX);
        // SIMPLE and WINDOW tiles are counted here (WINDOW in both binades);
        // COMPLEX tiles and tiny binades go to the exact pass.  So do the
        // WINDOW tiles of a segment that has few of them: the exact pass
        // stores their p, so the walker finds a binade crossing in shared
        // memory instead of recomputing the tile from the logits
        const uint32_t nwin_seg = __syncthreads_count(live && cls == CLS_WINDOW);
        bool special = cls == CLS_COMPLEX || lo < -100 || (cls == CLS_WINDOW && nwin_seg <= 32u);
        const float K = (float)(23 - max(lo, -100));   // log2(term / u_lo) = exponent + K
        // may hold candidates: the per-element test below is monotone in the
        // logit, so the tile maximum decides
        const float dm = __fsub_rn(tmax, M);
        const float xm = (dm == 0.0f) ? 0.0f : dm * c2;
        bool cand = tmax > NEG_INF && xm >= xf2;
        float e;
        if (TERM == TERM_P) {
            e = fmaxf(cert_eps(K), 0x1p-17f);
        } else {
            // the tile's largest P: a P near 1 has a tiny -ln P whose relative
            // error the certificate cannot bound, so its tile is exact
            const float zt = xm - l2S;
            special = special || zt > -0.0625f;
            e = fmaxf(cert_eps_h(K, fmaxf(-zt, 0.0625f), fabsf(l2S)), 0x1p-17f);
            // band candidates: surprises of the tile are at least -zt ln2
            cand = band && tmax > NEG_INF && -zt * 0.6931472f <= Hr + dband + 0.01f;
        }
        tp.K = K;
        tp.fhi = 1.0f + e;
        tp.flo = 1.0f - e;
        tp.info = (special ? TP_SPECIAL : 0u) | (cand ? TP_CAND : 0u) | (cls << 2) | ((uint32_t)(lo + 128) << 8);
    }

    const bool t_nan = T != T, t_inf = isinf(T);
    const bool check_nan = ri.check_nan != 0;
    Candidate *cand = P.cand + (size_t)hrow * P.cand_stride;
    const bool staged = pre || (bulk && seg_wait(P, &bar));
    // the prologue and the penalty on this thread's own staged tile; other
    // threads read it only after the barriers below
    if (!pre && staged && P.pro && live) prologue_tile_smem(P, tid, reinterpret_cast<float *>(sbuf));
    if (!pre && staged && bm && live) patch_tile_smem(P, hrow, seg, tid, reinterpret_cast<float *>(sbuf));
    const uint32_t tt = live ? (uint32_t)tid : 0u;
    auto quad = [&](int j) { return tile_quad(P, x, seg, tt, j, sbuf, staged, bm, pol); };
    const uint32_t g0 = seg * SEG_ELEMS + (uint32_t)tid * TILE;
    // certified grid counts of binade lo: y = p / u_lo from the fast exp;
    // y (1 - e) and y (1 + e) bracket the exact value, and the count is the
    // common rounding of both (a tie, or a value too close to one, makes them
    // differ).  The clamp makes large values differ too.  The permuted order
    // of v does not matter: without ties the counts simply add.
    // the term over u_lo: p / u_lo = 2^(x2 + K), or for the entropy
    // P (-ln P) / u_lo = 2^(z + K) (-z ln2) with z = x2 - log2 S
    auto term_y = [&](float d) {
        if (TERM == TERM_P) return ex2_approx(fminf(fmaf(d, c2, tp.K), 17.5f));
        const float z = fmaf(d, c2, -l2S);
        const float w = fminf(z * -0.6931472f, 1e30f);   // -ln P (finite for P = 0)
        return fminf(ex2_approx(fminf(z + tp.K, 40.0f)) * w, 185363.8f);   // 2^17.5
    };
    // The normaliser pass sums both roundings: r1 >= r2 element by element
    // (fhi > flo and y >= 0), and a tile's differences stay far below 2^32,
    // so the two sums agree exactly when every element's do.  The entropy
    // pass marks the terms whose roundings differ instead (bit 4 j + c of
    // `bad`): its uncertified terms are recounted one by one below.
    constexpr bool RC = TERM == TERM_H;
    uint32_t acc = 0u, diff = 0u, bad = 0u;
    const uint32_t cls_t = (tp.info >> 2) & 3u;
    const bool win = live && cls_t == CLS_WINDOW;
    uint32_t acch = 0u;
    {
        uint32_t acc2 = 0u;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const float4 q = quad(j);
            const float a4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float y = term_y(__fsub_rn(a4[c], M));
                const uint32_t r1 = __float_as_uint(fmaf(y, tp.fhi, 12582912.0f));
                const uint32_t r2 = __float_as_uint(fmaf(y, tp.flo, 12582912.0f));
                acc += r1;
                if (RC) {
                    bad |= r1 != r2 ? 1u << (4 * j + c) : 0u;
                } else {
                    acc2 += r2;
                }
            }
        }
        diff |= RC ? bad : (acc ^ acc2);
        acc -= (uint32_t)TILE * 0x4B400000u;   // a tile sums to < 2^22.5
        if (win) {
            const float hh = 0.5f * tp.fhi, hl = 0.5f * tp.flo;
            uint32_t acch2 = 0u;
#pragma unroll 2
            for (int j = 0; j < 8; j++) {
                const float4 q = quad(j);
                const float a4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const float y = term_y(__fsub_rn(a4[c], M));
                    acch += __float_as_uint(fmaf(y, hh, 12582912.0f));
                    acch2 += __float_as_uint(fmaf(y, hl, 12582912.0f));
                }
            }
            diff |= acch ^ acch2;
            acch -= (uint32_t)TILE * 0x4B400000u;
        }
    }
    uint32_t nanl = 0;
    if (TERM == TERM_P && check_nan && live) {
#pragma unroll 1
        for (int j = 0; j < 8; j++) {
            const float4 q = quad(j);
            const float a4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float d = __fsub_rn(a4[c], M);
                nanl |= (g0 + tile_elem(tid, j, c) < P.vocab && ((d != d) || t_nan || (isinf(d) && t_inf))) ? 1u
                                                                                                          : 0u;
            }
        }
    }
    // Entropy pass: a SIMPLE tile with a few uncertified terms keeps its
    // other counts.  The uncertified terms' estimates come off its sum here
    // and their exact counts (exp, divide and log each) are added below, one
    // term per thread, instead of a warp pass over the whole tile.  The tile
    // still goes to the warp pass if a term is a tie (its count would depend
    // on the parity), leaves the binade, or the list is full.  (For the
    // normaliser's cheaper terms the warp pass measured faster.)
    const bool recount = RC && live && !(tp.info & TP_SPECIAL) && cls_t == CLS_SIMPLE && diff != 0u;
    if (recount) {
        uint32_t mb = bad;
        while (mb) {
            const int b = __ffs(mb) - 1;
            mb &= mb - 1u;
            const float4 q = quad(b >> 2);
            const float a = (b & 3) == 0 ? q.x : ((b & 3) == 1 ? q.y : ((b & 3) == 2 ? q.z : q.w));
            acc -= __float_as_uint(fmaf(term_y(__fsub_rn(a, M)), tp.fhi, 12582912.0f)) - 0x4B400000u;
            const uint32_t slot = atomicAdd(&nrc, 1u);
            if (slot < RC_CAP) {
                rcl[slot] = (uint16_t)(((uint32_t)tid << 5) | tile_elem(tid, b >> 2, b & 3));
            } else {
                atomicOr(&rc_fb[tid >> 5], 1u << (tid & 31));
            }
        }
    }
    const bool special = live && ((tp.info & TP_SPECIAL) || (diff != 0u && !recount));
    if (live) {
        TileRec rr;
        rr.lo = (int32_t)(tp.info >> 8) - 128;
        rr.cls = cls_t;
        rr.aux = 0xFFFFFFFFu;
        rr.qlo = Comp{acc, acc};
        rr.qhi = win ? Comp{acch, acch} : Comp{0u, 0u};
        rec[tid] = rr;
    }
    {   // special tiles to the exact pass: one reservation per warp
        const uint32_t m = __ballot_sync(0xffffffffu, special);
        uint32_t base = 0;
        if (lane == 0 && m) base = atomicAdd(&nlist, (uint32_t)__popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (special) wlist[base + __popc(m & ((1u << lane) - 1u))] = tid;
    }
    if (__any_sync(0xffffffffu, nanl != 0) && lane == 0) atomicOr(&nanflag, 1u);
    __syncthreads();
    if (nanflag && tid == 0) atomicOr(&hdr->flags, RF_NAN);
    if (RC && nrc > 0) {   // block-uniform: read after the barrier
        // the listed terms' exact counts
        const uint32_t nr = min(nrc, RC_CAP);
        const float *sb = reinterpret_cast<const float *>(sbuf);
        for (uint32_t i = tid; i < nr; i += K12_THREADS) {
            const uint32_t e = rcl[i], lt = e >> 5;
            const uint32_t g = seg * SEG_ELEMS + lt * TILE + (e & 31u);
            float a = staged ? sb[lt * TILE + (e & 31u)] : x[g];
            if (!staged) a = prologue_of(P)(a);
            if (!staged && bm && ((bm[g >> 5] >> (g & 31u)) & 1u)) a = penalize(a, P.rep_penalty);
            const float pt = TERM == TERM_P ? prob_unnorm(a, M, T) : entropy_term(a, M, T, S);
            const Comp c = elem_comp(pt, rec[lt].lo);
            if (c.q0 == c.q1 && c.q0 < QLIM) {
                atomicAdd(&rec[lt].qlo.q0, c.q0);
                atomicAdd(&rec[lt].qlo.q1, c.q0);
            } else {
                atomicOr(&rc_fb[lt >> 5], 1u << (lt & 31));
            }
        }
        __syncthreads();
        // a recounted tile with a tie, a term out of the binade or a sum of
        // 2^24 or more joins the exact pass (which composes such tiles)
        const bool sp = recount && (((rc_fb[tid >> 5] >> (tid & 31)) & 1u) || rec[tid].qlo.q0 >= QLIM);
        const uint32_t m = __ballot_sync(0xffffffffu, sp);
        uint32_t base = 0;
        if (lane == 0 && m) base = atomicAdd(&nlist, (uint32_t)__popc(m));
        base = __shfl_sync(0xffffffffu, base, 0);
        if (sp) wlist[base + __popc(m & ((1u << lane) - 1u))] = tid;
        __syncthreads();
    }
    // warp-cooperative exact pass (lane = element, index order) for tiles
    // whose counts need ordered composition (ties), tiny binades or several
    // binades; several-binade tiles also keep their exact p for the walker
    const uint32_t nl = nlist;
    float *wcd = P.wcdata + (size_t)hrow * WC_CAP * TILE;
    for (uint32_t li = warp; li < nl; li += NW) {
        const uint32_t lt = wlist[li];
        const uint32_t tt = seg * SEG_TILES + lt;
        TileRec r = rec[lt];
        const uint32_t g = tt * TILE + lane;
        float a = NEG_INF;
        if (g < P.vocab) a = staged ? reinterpret_cast<const float *>(sbuf)[lt * TILE + lane] : x[g];
        // the prologue and the penalty (the staged copy has them already)
        if (!staged && g < P.vocab) a = prologue_of(P)(a);
        if (!staged && bm && g < P.vocab && ((bm[g >> 5] >> (g & 31u)) & 1u)) a = penalize(a, P.rep_penalty);
        const float p = g < P.vocab ? (TERM == TERM_P ? prob_unnorm(a, M, T) : entropy_term(a, M, T, S)) : 0.0f;
        r.qlo = warp_tile_comp(elem_comp(p, r.lo));
        if (r.cls == CLS_WINDOW) r.qhi = warp_tile_comp(elem_comp(p, r.lo + 1));
        if (r.cls != CLS_SIMPLE) {   // several binades: the walker may need the exact p
            uint32_t slot = 0;
            if (lane == 0) slot = atomicAdd(&hdr->n_wc, 1u);
            slot = __shfl_sync(0xffffffffu, slot, 0);
            if (slot < WC_CAP) {
                wcd[slot * TILE + lane] = p;
                r.aux = slot;
            }
        }
        if (lane == 0) rec[lt] = r;
    }
    // candidates (index, logit), after the warp's exact-pass tiles and in
    // the same barrier interval: warp-aggregated reservation.  The
    // normaliser pass takes every token above the floor; the entropy pass,
    // for typical-p alone, every token whose approximate dev = |-ln P - H|
    // is inside the band
    auto is_cand = [&](float d) {
        if (TERM == TERM_P) return (d == 0.0f ? 0.0f : d * c2) >= xf2;
        const float w = fminf(fmaf(d, c2, -l2S) * -0.6931472f, 1e30f);
        return fabsf(w - Hr) <= dband;
    };
    const bool tc = live && (tp.info & TP_CAND);
    if (__any_sync(0xffffffffu, tc)) {
        uint32_t nc = 0;
        if (tc) {
#pragma unroll 1
            for (int j = 0; j < 8; j++) {
                const float4 q = quad(j);
                const float a4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int c = 0; c < 4; c++) nc += is_cand(__fsub_rn(a4[c], M)) ? 1u : 0u;
            }
        }
        const uint32_t incl = warp_incl_scan_u(nc);
        const uint32_t wtot = __shfl_sync(0xffffffffu, incl, 31);
        uint32_t cb = 0;
        if (lane == 31 && wtot) cb = atomicAdd(&hdr->n_cand, wtot);
        cb = __shfl_sync(0xffffffffu, cb, 31);
        uint32_t pos = cb + incl - nc;
        if (nc) {
#pragma unroll 1
            for (int j = 0; j < 8; j++) {
                const float4 q = quad(j);
                const float a4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    if (is_cand(__fsub_rn(a4[c], M))) {
                        if (pos < P.cand_stride) cand[pos] = Candidate{g0 + tile_elem(tid, j, c), a4[c]};
                        pos++;
                    }
                }
            }
        }
    }
    __syncthreads();

    // ---- items: a stretch of SIMPLE tiles of one binade, a stretch of WINDOW
    // tiles of one lower binade, or one COMPLEX tile
    const uint32_t NT = ntile;
    const uint32_t tile0 = seg * SEG_TILES;
    Item *items = P.items + (size_t)hrow * P.ntiles_total + tile0;
    WTile *wpre = P.wpre + (size_t)hrow * P.ntiles_total + tile0;
    // the common segment (past the row start): every tile SIMPLE in one
    // binade with parity-free counts -- a single item, from a block sum
    {
        // (the tile records are final after the exact pass's barrier)
        uint32_t *const wsum_u = ms_.wsum_u;
        uint32_t *const wuni = ms_.wuni;
        const int32_t lo0 = rec[0].lo;
        const TileRec rt = live ? rec[tid] : rec[0];
        const bool mine = rt.cls == CLS_SIMPLE && rt.lo == lo0 && rt.qlo.q0 == rt.qlo.q1;
        // a tile counts < 2^22.5, so 256 of them fit 32 bits
        const uint32_t qw = __reduce_add_sync(0xffffffffu, live ? rt.qlo.q0 : 0u);
        const bool wall = __all_sync(0xffffffffu, mine);
        if (lane == 0) {
            wsum_u[warp] = qw;
            wuni[warp] = wall ? 1u : 0u;
        }
        __syncthreads();
        bool uni = true;
#pragma unroll
        for (int w = 0; w < NW; w++) uni = uni && wuni[w] != 0u;
        if (uni) {
            if (tid == 0) {
                uint32_t tot = 0;
                for (int w = 0; w < NW; w++) tot += wsum_u[w];
                const uint32_t qa = min(tot, QSAT);
                Item it;
                it.kind = CLS_SIMPLE;
                it.lo = lo0;
                it.q[0] = qa;
                it.q[1] = qa;
                it.q[2] = 0u;
                it.q[3] = 0u;
                it.tile = tile0;
                it.aux = NT;
                items[0] = it;
                hdr->seg_items[seg] = 1u;
                hdr->seg_tile0[seg] = tile0;
            }
            return;
        }
    }
    // counts that depend on the entry parity (ties) need ordered composition;
    // otherwise plain sums suffice and the warps build the items in parallel
    const bool ties = __syncthreads_or(live && (rec[tid].qlo.q0 != rec[tid].qlo.q1 ||
                                                rec[tid].qhi.q0 != rec[tid].qhi.q1)) != 0;
    if (!ties) {
        // each warp builds the items of its chunk of 32 tiles; a stretch that
        // runs into a chunk from before is carried from the chunk summaries
        uint64_t *const ch_a = ms_.ch_a, *const ch_b = ms_.ch_b;   // counts from the chunk's last head (or start) to its end
        uint32_t *const ch_heads = ms_.ch_heads, *const ch_start = ms_.ch_start;
        uint32_t *sid = uarr;                                   // item of each WINDOW tile
        uint64_t *sb = reinterpret_cast<uint64_t *>(carr);      // hi prefix of each WINDOW tile
        uint64_t *itb = reinterpret_cast<uint64_t *>(carr2);    // hi total of each item
        const uint32_t c0 = (uint32_t)warp * 32u;
        const uint32_t j = c0 + lane;
        const bool valid = j < NT;
        TileRec r;
        r.lo = 0;
        r.cls = CLS_SIMPLE;
        r.aux = 0u;
        r.qlo = Comp{0u, 0u};
        r.qhi = Comp{0u, 0u};
        if (valid) r = rec[j];
        bool h = valid, e = valid;
        if (valid && j > 0) {
            const TileRec q = rec[j - 1];
            h = r.cls == CLS_COMPLEX || q.cls != r.cls || q.lo != r.lo;
        }
        if (valid && j + 1 < NT) {
            const TileRec q = rec[j + 1];
            e = r.cls == CLS_COMPLEX || q.cls != r.cls || q.lo != r.lo;
        }
        const uint32_t heads = __ballot_sync(0xffffffffu, h);
        const uint64_t a = r.qlo.q0, b = r.qhi.q0;
        uint64_t Pa = a, Pb = b;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint64_t ua = __shfl_up_sync(0xffffffffu, Pa, o);
            const uint64_t ub = __shfl_up_sync(0xffffffffu, Pb, o);
            if (lane >= o) {
                Pa += ua;
                Pb += ub;
            }
        }
        const uint32_t upto = lane == 31 ? 0xffffffffu : ((2u << lane) - 1u);
        const uint32_t m = heads & upto;
        const int sl = m ? 31 - __clz(m) : 0;
        const uint64_t pa0 = __shfl_sync(0xffffffffu, Pa, sl > 0 ? sl - 1 : 0);
        const uint64_t pb0 = __shfl_sync(0xffffffffu, Pb, sl > 0 ? sl - 1 : 0);
        const uint64_t loc_a = m ? Pa - (sl > 0 ? pa0 : 0) : Pa;
        const uint64_t loc_b = m ? Pb - (sl > 0 ? pb0 : 0) : Pb;
        if (lane == 31) {
            ch_a[warp] = loc_a;
            ch_b[warp] = loc_b;
            ch_heads[warp] = __popc(heads);
            ch_start[warp] = heads ? c0 + (31u - __clz(heads)) : 0xFFFFFFFFu;
        }
        __syncthreads();
        // the stretch open at this chunk's start: back to the nearest chunk
        // with a head (chunk 0 always starts with one)
        uint32_t nbefore = 0;
        for (int w2 = 0; w2 < warp; w2++) nbefore += ch_heads[w2];
        uint64_t carry_a = 0, carry_b = 0;
        uint32_t carry_start = 0;
        for (int w2 = warp - 1; w2 >= 0; w2--) {
            carry_a += ch_a[w2];
            carry_b += ch_b[w2];
            if (ch_heads[w2]) {
                carry_start = ch_start[w2];
                break;
            }
        }
        uint64_t seg_a, seg_b;
        uint32_t start, id;
        if (m) {
            seg_a = loc_a;
            seg_b = loc_b;
            start = c0 + (uint32_t)sl;
            id = nbefore + __popc(m) - 1u;
        } else {   // continues the stretch open at the chunk start
            seg_a = carry_a + Pa;
            seg_b = carry_b + Pb;
            start = carry_start;
            id = nbefore - 1u;
        }
        if (valid && r.cls == CLS_WINDOW) {
            const uint32_t pa = (uint32_t)min(seg_a, (uint64_t)QSAT);
            wpre[j] = WTile{Comp{pa, pa}, Comp{0u, 0u}, r.aux, 0u};
            sid[j] = id;
            sb[j] = seg_b - b;   // exclusive hi prefix
        }
        if (valid && e) {
            Item it;
            it.kind = r.cls;
            it.lo = r.lo;
            it.tile = tile0 + start;
            const uint32_t qa = (uint32_t)min(seg_a, (uint64_t)QSAT);
            const uint32_t qb = (uint32_t)min(seg_b, (uint64_t)QSAT);
            if (r.cls == CLS_COMPLEX) {
                it.q[0] = r.qlo.q0;
                it.q[1] = r.qlo.q1;
                it.q[2] = 0u;
                it.q[3] = 0u;
                it.aux = r.aux;
            } else {
                it.q[0] = qa;
                it.q[1] = qa;
                it.q[2] = r.cls == CLS_WINDOW ? qb : 0u;
                it.q[3] = r.cls == CLS_WINDOW ? qb : 0u;
                it.aux = j - start + 1u;
            }
            items[id] = it;
            itb[id] = seg_b;
        }
        __syncthreads();
        // suffix counts (binade lo+1) of the WINDOW tiles
        if (live) {
            const TileRec rr = rec[tid];
            if (rr.cls == CLS_WINDOW) {
                const uint64_t suf = itb[sid[tid]] - sb[tid];
                const uint32_t qs = (uint32_t)min(suf, (uint64_t)QSAT);
                wpre[tid].suf_hi = Comp{qs, qs};
            }
        }
        if (tid == 0) {
            uint32_t nitems = 0;
            for (int w2 = 0; w2 < NW; w2++) nitems += ch_heads[w2];
            hdr->seg_items[seg] = nitems;
            hdr->seg_tile0[seg] = tile0;
        }
        return;
    }
    if (live) {
        const TileRec r = rec[tid];
        uint32_t h = 1, e = 1;
        if (tid > 0) {
            const TileRec q = rec[tid - 1];
            h = (r.cls == CLS_COMPLEX || q.cls != r.cls || r.lo != q.lo) ? 1u : 0u;
        }
        if ((uint32_t)tid + 1 < NT) {
            const TileRec q = rec[tid + 1];
            e = (r.cls == CLS_COMPLEX || q.cls != r.cls || r.lo != q.lo) ? 1u : 0u;
        }
        uarr[tid] = h;
        uarr2[tid] = e;
        carr[tid] = r.qlo;
        carr2[tid] = r.qhi;
    }
    __syncthreads();
    block_segscan_comp<false, K12_THREADS / 2>(carr, uarr, NT, wtmp_s);
    block_segscan_comp<true, K12_THREADS / 2>(carr2, uarr2, NT, wtmp_s);
    const uint32_t nitems = block_exscan_u<K12_THREADS / 2>(uarr, NT, wtmp_u);
    uint32_t *sstart = uarr2;
    __syncthreads();
    if (live) {
        const uint32_t nxt = ((uint32_t)tid + 1 < NT) ? uarr[tid + 1] : nitems;
        if (nxt != uarr[tid]) sstart[uarr[tid]] = tid;
    }
    __syncthreads();
    if (live) {
        const uint32_t id = (((uint32_t)tid + 1 < NT) ? uarr[tid + 1] : nitems) - 1u;
        const TileRec r = rec[tid];
        if (r.cls == CLS_WINDOW) wpre[tid] = WTile{carr[tid], carr2[tid], r.aux, 0u};
        bool is_end = ((uint32_t)tid + 1 == NT);
        if (!is_end) {
            const uint32_t nxt2 = ((uint32_t)tid + 2 < NT) ? uarr[tid + 2] : nitems;
            is_end = (nxt2 != uarr[tid + 1]);
        }
        if (is_end) {
            const uint32_t start = sstart[id];
            Item it;
            it.kind = r.cls;
            it.lo = r.lo;
            it.tile = tile0 + start;
            if (r.cls == CLS_COMPLEX) {
                it.q[0] = r.qlo.q0;
                it.q[1] = r.qlo.q1;
                it.q[2] = 0u;
                it.q[3] = 0u;
                it.aux = r.aux;
            } else {
                const Comp c = carr[tid];
                const Comp hh = r.cls == CLS_WINDOW ? carr2[start] : Comp{0u, 0u};
                it.q[0] = c.q0;
                it.q[1] = c.q1;
                it.q[2] = hh.q0;
                it.q[3] = hh.q1;
                it.aux = tid - start + 1u;
            }
            items[id] = it;
        }
    }
    if (tid == 0) {
        hdr->seg_items[seg] = nitems;
        hdr->seg_tile0[seg] = tile0;
    }
}

template <int TERM>
__global__ void __launch_bounds__(K12_THREADS, 5) k2_main(K12Params P) {
    __shared__ __align__(128) float4 sbuf[SEG_ELEMS / 4];
    __shared__ MainSmem ms;
    __shared__ __align__(8) uint64_t bar;
    // segment-major order over a 1-D grid: every row's segment 0 first (the
    // row start holds most exact-pass tiles, so those CTAs live several times
    // longer), the last segments last, so the kernel's tail is short CTAs
    const uint32_t seg = blockIdx.x / P.rows, row = blockIdx.x - seg * P.rows;
    main_task<TERM>(P, seg, row, ms, sbuf, &bar);
}

// ---------------------------------------------------------------------------
// Persistent form of the statistics pass, the row reduction and the
// normaliser's main pass: one launch whose resident CTAs take tasks from
// counters in device memory.
//   statistics task (row, segment), in row-major order;
//   the CTA that finishes a row's last statistics task runs the row
//     reduction and then publishes the row's main tasks (a slot of the ready
//     list, released after everything the tasks read);
//   main task (slot, segment): taken first whenever one is published, so a
//     row's logits are read again soon after the statistics streamed them
//     (from L2), and the HBM-bound statistics of later rows overlap the
//     issue-bound main tasks of earlier ones.
// A CTA waits only for tasks that running CTAs hold, never for one that no
// CTA has taken; every wait is bounded (a timeout marks the call failed).
// Loads of data another task wrote go through L2 (__ldcg): L1 is not
// coherent across SMs.
enum : uint32_t { TK_STATS = 0, TK_MAIN = 1, TK_EXIT = 2 };
constexpr uint64_t FUSED_WAIT_NS = 1000000000ull;   // one second without a task

union __align__(16) FusedSmem {
    StatsSmem s;
    RowsSmem r;
    MainSmem m;
};

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_u64(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

constexpr int FUSED_CTAS_PER_SM = 4;
__global__ void __launch_bounds__(K12_THREADS, FUSED_CTAS_PER_SM) k_fused(K12Params P) {
    __shared__ __align__(128) float4 sbuf[SEG_ELEMS / 4];
    __shared__ FusedSmem u;
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t t_kind, t_row, t_seg, t_last;
    const uint32_t nseg = P.nseg, total = P.rows * P.nseg;
    uint32_t *const s_next = P.ctl, *const m_next = P.ctl + 1, *const n_ready = P.ctl + 2;
    uint32_t *const row_done = P.ctl + 4;
    // thread 0's scheduling state: the statistics tasks are all taken; the
    // main-task ticket it holds (a fetch-add on the main counter, taken only
    // when a reduced row is likely waiting, so claims never contend; a ticket
    // whose row is not published yet is kept while the CTA takes statistics
    // tasks)
    constexpr uint32_t NONE = 0xFFFFFFFFu;
    bool s_done = false;
    uint32_t ticket = NONE;
    for (;;) {
        if (threadIdx.x == 0) {
            uint32_t kind = TK_EXIT, row = 0, seg = 0;
            const uint64_t t0 = global_ns();
            for (uint32_t it = 0;; it++) {
                if (ticket == NONE && __ldcg(m_next) < min(__ldcg(n_ready) * nseg, total)) {
                    const uint32_t t = atomicAdd(m_next, 1u);
                    if (t < total) ticket = t;
                }
                if (ticket != NONE) {
                    const uint32_t slot = ticket / nseg;
                    const unsigned long long rv = ld_acquire_u64(P.ready + slot);
                    if ((uint32_t)(rv >> 32) == P.seq) {
                        kind = TK_MAIN;
                        row = (uint32_t)rv;
                        seg = ticket - slot * nseg;
                        ticket = NONE;
                        break;
                    }
                }
                if (!s_done) {
                    const uint32_t t = atomicAdd(s_next, 1u);
                    if (t < total) {
                        kind = TK_STATS;
                        row = t / nseg;
                        seg = t - row * nseg;
                        break;
                    }
                    s_done = true;
                }
                if (ticket == NONE && __ldcg(m_next) >= total) break;   // every task is taken
                // a main task remains whose row is not published yet: the
                // statistics it needs are in running CTAs' hands
                if (global_ns() - t0 > FUSED_WAIT_NS || it > (1u << 24)) {
                    atomicExch(P.kerr, P.seq);
                    break;
                }
                __nanosleep(128);
            }
            t_kind = kind;
            t_row = row;
            t_seg = seg;
        }
        __syncthreads();
        const uint32_t kind = t_kind, row = t_row, seg = t_seg;
        if (kind == TK_EXIT) break;
        if (kind == TK_STATS) {
            stats_task(P, seg, row, u.s, sbuf, &bar);
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence();   // the task's statistics before its count
                t_last = atomicAdd(row_done + row, 1u) + 1u == nseg ? 1u : 0u;
            }
            __syncthreads();
            if (t_last) {
                __threadfence();   // every statistics task of the row before its reduction
                rows_task(P, row, u.r);
                __syncthreads();
                if (threadIdx.x == 0) {
                    __threadfence();
                    const uint32_t slot = atomicAdd(n_ready, 1u);
                    st_release_u64(P.ready + slot, ((unsigned long long)P.seq << 32) | row);
                }
            }
        } else {
            __threadfence();   // after thread 0's acquire of the slot: the row's reduction
            main_task<TERM_P>(P, seg, row, u.m, sbuf, &bar);
        }
        __syncthreads();   // the task's shared memory is free again
    }
}

// ---------------------------------------------------------------------------
// Read-once persistent form of the statistics pass, the row reduction and
// the normaliser's main pass.  A CTA takes (row, segment) tasks in row-major
// order from one counter, stages the segment in shared memory and computes
// its statistics; the CTA that completes a row's statistics runs the row
// reduction and publishes the row; the others wait for that, and every CTA
// then runs the main pass on the segment it still holds.  The logits cross
// HBM once per call instead of twice.
// Progress: a CTA waits only for its own row, whose other segments are held
// by running CTAs or taken next (tasks are taken in order), so with at least
// one row's worth of CTAs running every wait ends; each is bounded anyway
// (a timeout marks the call failed through the error word).
constexpr int RES_CTAS_PER_SM = 4;
__global__ void __launch_bounds__(K12_THREADS, RES_CTAS_PER_SM) k_resident(K12Params P) {
    __shared__ __align__(128) float4 sbuf[SEG_ELEMS / 4];
    __shared__ FusedSmem u;
    __shared__ __align__(8) uint64_t bar;
    __shared__ uint32_t t_task, t_last;
    const uint32_t nseg = P.nseg, total = P.rows * P.nseg;
    uint32_t *const next = P.ctl;
    uint32_t *const row_done = P.ctl + 4;
    for (;;) {
        if (threadIdx.x == 0) t_task = atomicAdd(next, 1u);
        __syncthreads();
        const uint32_t t = t_task;
        if (t >= total) break;
        const uint32_t row = t / nseg, seg = t - row * nseg;
        const bool staged = stats_task(P, seg, row, u.s, sbuf, &bar);
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();   // the task's statistics before its count
            t_last = atomicAdd(row_done + row, 1u) + 1u == nseg ? 1u : 0u;
        }
        __syncthreads();
        if (t_last) {
            __threadfence();   // every statistics task of the row before its reduction
            rows_task(P, row, u.r);
            __syncthreads();
            if (threadIdx.x == 0) {
                __threadfence();
                st_release_u64(P.ready + row, ((unsigned long long)P.seq << 32) | row);
            }
        } else if (threadIdx.x == 0) {
            const uint64_t t0 = global_ns();
            for (uint32_t it = 0; (uint32_t)(ld_acquire_u64(P.ready + row) >> 32) != P.seq; it++) {
                if (global_ns() - t0 > FUSED_WAIT_NS || it > (1u << 24)) {
                    atomicExch(P.kerr, P.seq);
                    break;
                }
                __nanosleep(256);
            }
        }
        __syncthreads();
        __threadfence();   // after thread 0's acquire: the row's reduction
        main_task<TERM_P>(P, seg, row, u.m, sbuf, &bar, staged);
        __syncthreads();   // the task's shared memory is free again
    }
}

// ---------------------------------------------------------------------------
enum : uint32_t { VS_OFF = 0, VS_WALK = 1, VS_DRAW = 2 };
constexpr uint32_t VS_CAND_CAP = 512;   // candidates a shard exports per row (BS_VSHARD_CAND_CAP)

struct KBParams {
    const float *logits;
    size_t ld;
    const uint32_t *pen_bm;   // as K12Params::pen_bm
    uint32_t vocab;
    uint32_t row0;
    float T;
    uint32_t top_k;
    float top_p;
    float min_p;
    float typical_p;
    float rep_penalty;
    uint32_t ntiles_total;
    RowHdr *hdr;
    Item *items;
    float *wcdata;
    const WTile *wpre;
    Candidate *cand;     // per handle row: cand_stride entries (Kernel A output)
    unsigned long long *ctmp;  // per handle row: 2 x cand_stride keys (large-set path)
    uint32_t cand_stride;
    uint64_t *rng;       // per handle row, 4 words
    RowTrace *trace;     // per handle row
    const uint32_t *kerr;   // == seq: a bounded wait of this call gave up
    uint32_t seq;
    uint32_t pro;           // as K12Params
    float softcap, pinv;
    // vocabulary sharding: VS_WALK walks this shard's items from the running
    // sum vs_entry[row] (nullptr: the empty sum) and writes the sum after them
    // to vs_exit[row]; VS_DRAW takes the row's normaliser from vs_S[row] and
    // draws from the merged candidates of every shard
    uint32_t vs_mode;
    const float *vs_entry;
    float *vs_exit;
    const float *vs_S;
    // the chain through peer memory instead (vs_p2p): 64-bit words
    // (seq << 32) | f32 bits.  VS_WALK waits for its entry in vs_in[row]
    // (written by the previous rank; rank 0: the empty sum) and stores its
    // exit in the next rank's vs_next[row], or, on the last rank, the row's
    // S in every rank's S words (vs_xs[g] + vs_soff + row); VS_DRAW waits
    // for its S in vs_in[vs_soff + row]
    uint32_t vs_p2p, vs_world, vs_rank, vs_soff;
    const uint32_t *vs_epoch;   // the step's tag (a captured graph replays one seq)
    unsigned long long *vs_in;
    unsigned long long *vs_next;
    unsigned long long *const *vs_xs;
    const RowInfo *rinfo;   // per handle row
    uint32_t tmode;      // TYP_*
    uint32_t force_full;    // test hook: every row takes the full-vocabulary retry
    uint32_t *out;       // per call row
};

// The crossing inside a WINDOW stretch of ntl tiles: the first tile c whose
// prefix count (binade lo, entry parity pi, table wp) brings the running
// mantissa m to 2^24.  The caller guarantees that the whole stretch does.
// Called by a full warp: each round samples the window [lo_i, hi_i] at up
// to 32 evenly spaced tiles (every tile once it is a warp wide) and keeps
// the part between the last sample below 2^24 and the first at or above it
// (no division: lanes past the window take part as crossed).
struct Crossing {
    uint32_t c;        // the crossing tile
    uint32_t q_prev;   // prefix count through tile c - 1 (0 when c = 0)
    uint32_t slot;     // tile c's stored exact terms, or >= n_wc
    Comp suf;          // suffix counts (binade lo + 1) from tile c + 1, if c + 1 < ntl
};
__device__ __forceinline__ Crossing find_crossing(const WTile *wp, uint32_t ntl, uint32_t m, uint32_t pi) {
    const uint32_t lane = threadIdx.x & 31u;
    // invariant: the crossing lies in [lo_i, hi_i]
    uint32_t lo_i = 0, hi_i = ntl - 1;
    while (lo_i < hi_i) {
        const uint32_t step = (hi_i - lo_i + 32) / 32;
        const uint32_t pos = lo_i + lane * step;
        // a lane past the window counts as crossed (the crossing is at or
        // before hi_i), so an empty ballot means every lane's tile is below it
        bool pr = pos > hi_i;
        if (!pr) {
            const Comp c = wp[pos].pre_lo;
            pr = m + (pi ? c.q1 : c.q0) >= QLIM;
        }
        const uint32_t mask = __ballot_sync(0xffffffffu, pr);
        if (mask == 0) {
            lo_i = lo_i + 31 * step + 1;
        } else {
            const uint32_t f = __ffs(mask) - 1;
            hi_i = min(hi_i, lo_i + f * step);
            if (f > 0) lo_i = lo_i + (f - 1) * step + 1;
        }
    }
    Crossing x;
    x.c = lo_i;
    x.q_prev = 0u;
    if (x.c > 0) {
        const Comp pc = wp[x.c - 1].pre_lo;
        x.q_prev = pi ? pc.q1 : pc.q0;
    }
    x.slot = wp[x.c].slot;
    x.suf = x.c + 1 < ntl ? wp[x.c + 1].suf_hi : Comp{0u, 0u};
    return x;
}

// Check of find_crossing for the test harness: block b (one warp) takes
// stretches of ntl = b + 1 tiles and every crossing position, with a table
// that makes the answer known; failures are counted in out[0], cases in out[1].
__global__ void crossing_check_kernel(WTile *scratch, uint32_t max_ntl, unsigned long long *out) {
    const uint32_t ntl = blockIdx.x + 1, lane = threadIdx.x;
    WTile *wp = scratch + (size_t)blockIdx.x * max_ntl;
    for (uint32_t cs = 0; cs < ntl; cs++) {
        for (uint32_t pi = 0; pi < 2; pi++) {
            const uint32_t m = 5u + pi;
            for (uint32_t k = lane; k < ntl; k += 32) {
                // prefix counts below the crossing stay under 2^24 - m
                const uint32_t q = k < cs ? k : QLIM;
                wp[k] = WTile{Comp{pi ? 7u : q, pi ? q : 7u}, Comp{3 * k, 3 * k + 1}, 1000u + k, 0u};
            }
            __syncwarp();
            const Crossing x = find_crossing(wp, ntl, m, pi);
            bool ok = x.c == cs && x.slot == 1000u + cs && x.q_prev == (cs > 0 ? cs - 1 : 0u);
            if (cs + 1 < ntl) ok = ok && x.suf.q0 == 3 * (cs + 1) && x.suf.q1 == 3 * (cs + 1) + 1;
            if (lane == 0) {
                atomicAdd(&out[1], 1ull);
                if (!ok) atomicAdd(&out[0], 1ull);
            }
            __syncwarp();
        }
    }
}

// Exact p of element g (the logit prologue, then the repetition penalty when
// the row's bitmap `bm` marks it), for the recompute path.
__device__ __forceinline__ float exact_p_raw(const float *xrow, uint32_t vocab, uint32_t g, float M, float T,
                                             float pen, const uint32_t *bm, Prologue pr) {
    if (g >= vocab) return 0.0f;
    float v = xrow[g];
    if (pr.pro) v = pr(v);
    if (bm && ((bm[g >> 5] >> (g & 31u)) & 1u)) v = penalize(v, pen);
    return prob_unnorm(v, M, T);
}
__device__ __forceinline__ Prologue prologue_of(const KBParams &P) { return Prologue{P.pro, P.softcap, P.pinv}; }
__device__ __forceinline__ const uint32_t *row_bitmap(const KBParams &P, uint32_t hrow) {
    return P.pen_bm ? P.pen_bm + (size_t)hrow * P.ntiles_total : nullptr;
}
__device__ float exact_p_at(const KBParams &P, uint32_t row, uint32_t hrow, uint32_t g, float M) {
    return exact_p_raw(P.logits + (size_t)row * P.ld, P.vocab, g, M, P.T, P.rep_penalty, row_bitmap(P, hrow),
                       prologue_of(P));
}

// The walker's recompute path: the warp adds one tile's terms, p (TERM_P)
// or the entropy terms h (TERM_H, with the normaliser S), recomputed from
// the logits, to the running sum s in index order.  Out of line: it is rare,
// and inlined it would sit in the middle of the walk's hot code.
template <int TERM>
__device__ __noinline__ float walk_recompute_tile(float s, const float *xrow, uint32_t vocab, uint32_t tile, float M,
                                                  float T, float pen, const uint32_t *bm, Prologue pr, float S,
                                                  float *tilep) {
    const uint32_t lane = threadIdx.x & 31u;
    float t = exact_p_raw(xrow, vocab, tile * TILE + lane, M, T, pen, bm, pr);
    if (TERM == TERM_H) {
        const float Pn = __fdiv_rn(t, S);
        t = Pn > 0.0f ? __fmul_rn(Pn, -log_ref(Pn)) : 0.0f;
    }
    tilep[lane] = t;
    __syncwarp();
    s = seq_add32_smem(s, tilep);
    __syncwarp();
    return s;
}

// Bitonic sort (ascending) of npow keys in shared memory (npow a power of two,
// at least 32) by `nthr` threads of whole warps, t = 0 .. nthr - 1 their index
// among them, `sync()` their barrier.  Only the stages with a stride of 32 or
// more go through shared memory (one barrier each); the others run in
// registers, lane l of a warp holding key 32 b + l of each block b the warp
// takes, with shuffles: each merge's strides 16 .. 1, and the whole network up
// to size 32 at the start.
__device__ __forceinline__ unsigned long long bitonic_cmpx(unsigned long long k, uint32_t e, uint32_t s,
                                                           uint32_t size) {
    const unsigned long long o = __shfl_xor_sync(0xffffffffu, k, (int)s);
    const bool up = (e & size) == 0u, lower = (e & s) == 0u;
    return (lower == up) ? (k < o ? k : o) : (k < o ? o : k);
}
template <typename Sync>
__device__ void bitonic_sort_keys(unsigned long long *k, uint32_t npow, uint32_t t, uint32_t nthr, Sync sync) {
    const uint32_t lane = t & 31u, w = t >> 5, nw = nthr >> 5, nblk = npow >> 5;
    // sizes 2 .. 32 in registers
    for (uint32_t b = w; b < nblk; b += nw) {
        const uint32_t e = 32u * b + lane;
        unsigned long long v = k[e];
#pragma unroll
        for (uint32_t size = 2; size <= 32; size <<= 1)
#pragma unroll
            for (uint32_t st = size >> 1; st > 0; st >>= 1) v = bitonic_cmpx(v, e, st, size);
        k[e] = v;
    }
    for (uint32_t size = 64; size <= npow; size <<= 1) {
        for (uint32_t stride = size >> 1; stride >= 32; stride >>= 1) {
            sync();
            for (uint32_t i = t; i < npow / 2; i += nthr) {
                const uint32_t a = 2 * i - (i & (stride - 1));
                const uint32_t b = a + stride;
                const bool up = ((a & size) == 0);
                const unsigned long long ka = k[a], kb = k[b];
                if (up ? (ka > kb) : (ka < kb)) {
                    k[a] = kb;
                    k[b] = ka;
                }
            }
        }
        sync();
        for (uint32_t b = w; b < nblk; b += nw) {
            const uint32_t e = 32u * b + lane;
            unsigned long long v = k[e];
#pragma unroll
            for (uint32_t st = 16; st > 0; st >>= 1) v = bitonic_cmpx(v, e, st, size);
            k[e] = v;
        }
    }
    sync();
}

// Block-wide form (every thread of the block).
__device__ void block_bitonic(unsigned long long *k, uint32_t npow) {
    __syncthreads();
    bitonic_sort_keys(k, npow, threadIdx.x, blockDim.x, [] { __syncthreads(); });
}

// Candidate key: ascending key order == (p descending, index ascending).
__device__ __forceinline__ unsigned long long cand_key(uint32_t idx, float p) {
    return ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(p)) << 32) | idx;
}
__device__ __forceinline__ float key_p(unsigned long long k) {
    return __uint_as_float(0xFFFFFFFFu - (uint32_t)(k >> 32));
}

// Stable LSD radix sort (4-bit digits) of n keys by one CTA, global memory.
// Returns the buffer holding the sorted keys (a or b).
__device__ __noinline__ unsigned long long *cta_radix_sort(unsigned long long *a, unsigned long long *b, uint32_t n,
                                                           uint32_t *cnt /* smem, 16 * KB_THREADS */,
                                                           unsigned long long *red /* smem, 2 */) {
    const int tid = threadIdx.x;
    // bits that differ between keys
    unsigned long long o = 0, an = ~0ull;
    for (uint32_t i = tid; i < n; i += KB_THREADS) {
        o |= a[i];
        an &= a[i];
    }
    if (tid == 0) {
        red[0] = 0;
        red[1] = ~0ull;
    }
    __syncthreads();
    atomicOr(&red[0], o);
    atomicAnd(&red[1], an);
    __syncthreads();
    const unsigned long long vary = red[0] ^ red[1];
    const uint32_t chunk = (n + KB_THREADS - 1) / KB_THREADS;
    const uint32_t lo = min(n, tid * chunk), hi = min(n, lo + chunk);
    const int lane = tid & 31, warp = tid >> 5;
    // per-thread digit counters in shared memory, column `tid` of 16 rows
    // (a register array indexed by the digit would live in local memory)
    uint32_t *const col = cnt + tid;
    for (int sh = 0; sh < 64; sh += 4) {
        if (((vary >> sh) & 0xFull) == 0) continue;
#pragma unroll
        for (int d = 0; d < 16; d++) col[d * KB_THREADS] = 0u;
        for (uint32_t i = lo; i < hi; i++) col[((a[i] >> sh) & 0xF) * KB_THREADS]++;
        uint32_t c[16];
#pragma unroll
        for (int d = 0; d < 16; d++) c[d] = col[d * KB_THREADS];
        // exclusive scan of the counts in digit-major order (digit d of thread
        // t starts after every lower digit and after digit d of threads < t),
        // in parallel: within each warp by shuffles, then over the warps and
        // the digits through shared memory (the counter rows are free once
        // every thread holds its counts)
        __syncthreads();
        uint32_t *const wt = cnt;                              // [warp][16] warp totals
        uint32_t *const base = cnt + (KB_THREADS / 32) * 16;   // [warp][16] starts
#pragma unroll
        for (int d = 0; d < 16; d++) {
            uint32_t incl = c[d];
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t u = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += u;
            }
            if (lane == 31) wt[warp * 16 + d] = incl;
            c[d] = incl - c[d];   // within the warp
        }
        __syncthreads();
        if (tid < 32) {   // digit d = tid (< 16): where each warp's keys of digit d start
            const int d = tid & 15;
            uint32_t wcol[KB_THREADS / 32], tot = 0;
#pragma unroll
            for (int w = 0; w < KB_THREADS / 32; w++) {
                wcol[w] = tot;
                tot += wt[w * 16 + d];
            }
            uint32_t dincl = tid < 16 ? tot : 0u;   // prefix of the digit totals
#pragma unroll
            for (int o = 1; o < 16; o <<= 1) {
                const uint32_t u = __shfl_up_sync(0xffffffffu, dincl, o);
                if (lane >= o) dincl += u;
            }
            if (tid < 16) {
#pragma unroll
                for (int w = 0; w < KB_THREADS / 32; w++) base[w * 16 + d] = dincl - tot + wcol[w];
            }
        }
        __syncthreads();
#pragma unroll
        for (int d = 0; d < 16; d++) c[d] += base[warp * 16 + d];
        __syncthreads();   // (the starts are read before the columns are rewritten)
#pragma unroll
        for (int d = 0; d < 16; d++) col[d * KB_THREADS] = c[d];
        // stable scatter: each thread its contiguous range, in order
        for (uint32_t i = lo; i < hi; i++) {
            const unsigned long long k = a[i];
            b[col[((k >> sh) & 0xF) * KB_THREADS]++] = k;
        }
        __syncthreads();
        unsigned long long *t = a;
        a = b;
        b = t;
    }
    return a;
}

// Sequential f32 scans by one thread over long lists (top-p and cum_typ,
// kept mass, draw walk).  The adds stay strictly in list order; only the
// loads are issued eight ahead, so the loop runs at the add chain's latency
// instead of a load round trip per element.  `get(i)` returns element i.
// The terms are >= 0, so the running sum never decreases: the threshold is
// tested once per eight adds (off the add chain), and only the block that
// crosses it is searched.  If `cum_out` is given, the running sum after
// element i is stored there for every element added (the kept mass of any
// prefix is then read back instead of summed again).
template <typename Get>
__device__ __forceinline__ uint32_t seq_first_exceed(Get get, uint32_t n, float thr, float &cum,
                                                     float *cum_out = nullptr) {
    for (uint32_t i0 = 0; i0 < n; i0 += 8) {
        float v[8], c[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = i0 + k < n ? get(i0 + k) : 0.0f;
        float t = cum;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            t = __fadd_rn(t, v[k]);   // past n the terms are 0: t is unchanged
            c[k] = t;
        }
        if (cum_out) {
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (i0 + k < n) cum_out[i0 + k] = c[k];
        }
        if (t > thr) {
#pragma unroll
            for (int k = 0; k < 8; k++) {
                if (c[k] > thr) {
                    if (i0 + k >= n) break;
                    cum = c[k];
                    return i0 + k;
                }
            }
        }
        cum = t;
    }
    return n;
}
template <typename Get>
__device__ __forceinline__ float seq_sum(Get get, uint32_t n) {
    float t = 0.0f;
    for (uint32_t i0 = 0; i0 < n; i0 += 8) {
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = i0 + k < n ? get(i0 + k) : 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++)
            if (i0 + k < n) t = __fadd_rn(t, v[k]);
    }
    return t;
}
// r -= a[i] in order; the first i with r <= 0, or n.  The terms are >= 0,
// so r never increases: tested once per eight subtractions, as above.
template <typename Get>
__device__ __forceinline__ uint32_t seq_draw(Get get, uint32_t n, float r) {
    for (uint32_t i0 = 0; i0 < n; i0 += 8) {
        float v[8], c[8];
#pragma unroll
        for (int k = 0; k < 8; k++) v[k] = i0 + k < n ? get(i0 + k) : 0.0f;
#pragma unroll
        for (int k = 0; k < 8; k++) {
            r = __fsub_rn(r, v[k]);
            c[k] = r;
        }
        if (r <= 0.0f) {
#pragma unroll
            for (int k = 0; k < 8; k++)
                if (c[k] <= 0.0f) return i0 + k < n ? i0 + k : n;
        }
    }
    return n;
}

// Typical-p (sampler.zig:128-154) and the draw (:156-168), after the entropy
// walk.  The list is the selected set from the normaliser pass (TYP_SELECTED:
// (index, P) pairs) or the band candidates of the entropy pass (TYP_BAND:
// (index, logit)).  Exact dev = |fl(-logf P) - H| gives the stable dev order;
// cum_typ over it deselects the crossing token and everything after it; the
// kept tokens are then taken in probability order (stable) for the mass and
// the inverse-CDF draw.  In band mode the kept set is trusted only when every
// token up to the crossing's dev is surely inside the band.
__device__ void typical_tail(const KBParams &P, uint32_t row, uint32_t hrow, float H, unsigned long long *skeys,
                             float *sprobs, unsigned long long *red2) {
    const int tid = threadIdx.x;
    RowHdr *hdr = P.hdr + hrow;
    const RowInfo ri = P.rinfo[hrow];
    const float M = hdr->M, S = hdr->S_exact;
    const uint32_t mode = P.tmode;
    const Candidate *cl = P.cand + (size_t)hrow * P.cand_stride;
    unsigned long long *gk0 = P.ctmp + (size_t)hrow * 2 * P.cand_stride;
    unsigned long long *gk1 = gk0 + P.cand_stride;
    const uint32_t n_list = min(mode == TYP_SELECTED ? hdr->n_sel : hdr->n_cand, P.cand_stride);
    uint32_t *cnt = reinterpret_cast<uint32_t *>(sprobs);   // radix scratch (big lists keep P in global memory)
    __shared__ uint32_t n_keep_sh, status_sh, nk_pow_sh, retry_sh;

    // A band that cannot be shown to cover the kept set (or every band, with
    // the test hook) is replaced by the whole vocabulary: the reference's
    // full dev sort, by the whole CTA in global memory.
    uint32_t n = n_list;
    bool big = false;
    unsigned long long *keys = skeys;
    float *pd = sprobs;
    bool went_full = false;
    for (bool full = false;; full = true) {
        went_full = full;
        n = full ? P.vocab : n_list;
        big = full || n > (uint32_t)CAND_SMEM;
        // 1. keys (dev, index), ascending
        uint32_t npow = 32;   // (block_bitonic takes blocks of 32 keys)
        while (npow < n) npow <<= 1;
        keys = big ? gk0 : skeys;
        for (uint32_t i = tid; i < (big ? n : npow); i += KB_THREADS) {
            unsigned long long k = ~0ull;
            if (i < n) {
                float Pi;
                uint32_t id = i;
                if (full) {
                    Pi = __fdiv_rn(exact_p_at(P, row, hrow, i, M), S);
                } else {
                    const Candidate c = cl[i];
                    Pi = mode == TYP_SELECTED ? c.v : __fdiv_rn(prob_unnorm(c.v, M, P.T), S);
                    id = c.idx;
                }
                const float sur = Pi > 0.0f ? -log_ref(Pi) : __int_as_float(0x7f800000);
                const float dev = fabsf(__fsub_rn(sur, H));
                k = ((unsigned long long)__float_as_uint(dev) << 32) | id;
            }
            keys[i] = k;
        }
        __syncthreads();
        if (big) {
            keys = cta_radix_sort(gk0, gk1, n, cnt, red2);
        } else {
            block_bitonic(keys, npow);
        }
        // 2. P in dev order, recomputed from the logits as the normaliser pass did
        pd = big ? reinterpret_cast<float *>(keys == gk0 ? gk1 : gk0) : sprobs;
        for (uint32_t i = tid; i < n; i += KB_THREADS)
            pd[i] = __fdiv_rn(exact_p_at(P, row, hrow, (uint32_t)keys[i], M), S);
        __syncthreads();
        // 3. cum_typ (sequential f32 in dev order)
        if (tid == 0) {
            uint32_t nk = n, st = *P.kerr == P.seq ? (uint32_t)ROW_ETIMEOUT : (uint32_t)ROW_OK;
            float cum = 0.0f;
            nk = seq_first_exceed([&](uint32_t i) { return pd[i]; }, n, P.typical_p, cum);
            const bool crossed = nk < n;
            bool retry = false;
            if (mode == TYP_BAND && st == ROW_OK && !full) {
                // the band held every token with approximate dev <= dband, where
                // the approximation used H_raw: tokens with exact dev up to
                // dband - |H_raw - H| - (surprise error) are surely in it
                const float dcross = crossed ? __uint_as_float((uint32_t)(keys[nk] >> 32)) : __int_as_float(0x7f800000);
                const float herr = fabsf((float)ri.H_raw - H);
                const float safe = ri.dband - herr - (1e-4f * (fabsf(H) + dcross) + 1e-4f);
                retry = !crossed || !(dcross <= safe) || P.force_full;
            }
            uint32_t np2 = 32;
            while (np2 < nk) np2 <<= 1;
            n_keep_sh = nk;
            status_sh = st;
            nk_pow_sh = np2;
            retry_sh = retry ? 1u : 0u;
        }
        __syncthreads();
        if (!retry_sh) break;
    }
    const uint32_t nk = n_keep_sh, nkp = nk_pow_sh;
    // 4. the kept tokens by (P descending, index ascending): each thread
    // rewrites its own entries in place
    for (uint32_t i = tid; i < (big ? nk : nkp); i += KB_THREADS)
        keys[i] = i < nk ? cand_key((uint32_t)keys[i], pd[i]) : ~0ull;
    __syncthreads();
    if (big) {
        keys = cta_radix_sort(keys, keys == gk0 ? gk1 : gk0, nk, cnt, red2);
    } else {
        block_bitonic(keys, nkp);
    }
    if (tid != 0) return;
    // 5. kept mass (sorted order) and the draw
    uint32_t status = status_sh;
    uint32_t token = hdr->top_idx, path = 2;
    float total = 0.0f, u = __int_as_float(0x7fc00000);
    uint64_t *rng = P.rng + (size_t)hrow * 4;
    uint64_t s4[4] = {rng[0], rng[1], rng[2], rng[3]};
    if (status == ROW_OK) {
        total = seq_sum([&](uint32_t j) { return key_p(keys[j]); }, nk);
        if (total > 0.0f) {   // else indices[0] without a draw (sampler.zig:160)
            u = rng_float(s4);
            const uint32_t j = seq_draw([&](uint32_t i) { return key_p(keys[i]); }, nk, __fmul_rn(u, total));
            path = 4;
            if (j < nk) {
                token = (uint32_t)keys[j];
                path = 3;
            }
        }
        rng[0] = s4[0]; rng[1] = s4[1]; rng[2] = s4[2]; rng[3] = s4[3];
        P.out[row] = token;
    } else {
        P.out[row] = 0xFFFFFFFFu;
    }
    RowTrace tr;
    tr.S = S;
    tr.total = total;
    tr.u = u;
    tr.n_kept = nk;
    tr.path = path;
    tr.flags = hdr->flags | (big ? RF_CAND_BIG : 0u) | (went_full ? RF_FULL : 0u);
    tr.n_cand = n;
    tr.status = status;
    tr.n_items = 0;
    tr.n_wc = hdr->n_wc;
    tr.n_slow = 0;
    tr.H = H;
    P.trace[hrow] = tr;
}

template <int TERM>
__global__ void __launch_bounds__(KB_THREADS, 2) kernel_b(KBParams P) {
    const uint32_t row = blockIdx.x;
    const uint32_t hrow = P.row0 + row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    grid_dep_launch();
    grid_dep_wait();   // the main pass's results
    RowHdr *hdr = P.hdr + hrow;
    if (TERM == TERM_H && hdr->tdone) return;   // the row's token is already final
    const float Sx = TERM == TERM_H ? hdr->S_exact : 1.0f;

    __shared__ Item sitems[ITEM_CHUNK];
    __shared__ __align__(16) Item sall[ITEM_SMEM];   // the first `spec` items of every segment
    __shared__ uint32_t woff[ITEM_SMEM];         // WINDOW item: its prefix table in wpool, or ~0u
    __shared__ __align__(8) WTile wpool[WPOOL];
    __shared__ uint32_t s_nit[MAX_SEG], wsum[KB_THREADS / 32 + 1], wcnt[KB_THREADS / 32], n_fit;
    // the walk's order of items: slots of sall, or ITEM_SMEM + s for a
    // segment s with more items than its slots (walked from global memory)
    __shared__ uint16_t fidx[ITEM_SMEM + MAX_SEG];
    __shared__ uint32_t n_flat, n_items_all;
    __shared__ __align__(16) float tilep[TILE];   // a recomputed tile's p, for the walker
    __shared__ float S_sh;
    __shared__ uint32_t walk_flags, walk_items, walk_slow, n_zero;
    __shared__ unsigned long long red2[2];
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned long long *skeys = reinterpret_cast<unsigned long long *>(smem);  // CAND_SMEM
    float *wcs = reinterpret_cast<float *>(skeys + CAND_SMEM);                 // WC_CAP*32
    float *sprobs = wcs + WC_CAP * TILE;                                       // CAND_SMEM

    const float M = hdr->M;
    const uint32_t flags0 = hdr->flags;
    const uint32_t n_cand = min(hdr->n_cand, P.cand_stride);
    const uint32_t n_wc = min(hdr->n_wc, (uint32_t)WC_CAP);
    // (a bitonic network in shared memory, beside the walk, up to CAND_SMEM
    // keys; longer lists take the block-wide radix sort in global memory
    // after it)
    const bool big = TERM == TERM_P && n_cand > (uint32_t)CAND_SMEM;

    // the walk's inputs in shared memory, gathered with asynchronous copies
    // (one wait for all of them).  Segment s's items start at tile
    // s * SEG_TILES; its first `spec` items are fetched speculatively in the
    // same round trip as their count
    const uint32_t nseg = min((P.ntiles_total + SEG_TILES - 1) / SEG_TILES, (uint32_t)MAX_SEG);
    const uint32_t spec = ITEM_SMEM / nseg;
    const Item *ib = P.items + (size_t)hrow * P.ntiles_total;
    static_assert(sizeof(Item) == 32, "an item is two 16-byte chunks");
    const bool walks = P.vs_mode != VS_DRAW;   // (a shard draw takes S from the chain)
    for (uint32_t i = tid; walks && i < 2 * nseg * spec; i += KB_THREADS) {
        const uint32_t it = i >> 1, sg = it / spec, j = it - sg * spec;
        if (sg * SEG_TILES + j < P.ntiles_total && j < (uint32_t)SEG_TILES)
            cp_async16(reinterpret_cast<uint4 *>(sall) + i, reinterpret_cast<const uint4 *>(ib + sg * SEG_TILES + j) + (i & 1u));
    }
    // the stored exact terms (rows of WC_CAP * TILE floats, 16-byte aligned)
    const float *wcg = P.wcdata + (size_t)hrow * WC_CAP * TILE;
    for (uint32_t i = tid; walks && i < n_wc * (TILE / 4); i += KB_THREADS) cp_async16(wcs + 4 * i, wcg + 4 * i);
    if ((uint32_t)tid < nseg)
        s_nit[tid] = walks ? min(hdr->seg_items[tid], min((uint32_t)SEG_TILES, P.ntiles_total - tid * SEG_TILES)) : 0u;
    cp_async_wait_all();
    const Candidate *cg_ = P.cand + (size_t)hrow * P.cand_stride;
    unsigned long long *gk0 = P.ctmp + (size_t)hrow * 2 * P.cand_stride;
    unsigned long long *gk1 = gk0 + P.cand_stride;
    uint32_t npow = 32;   // (the sort's register phases take blocks of 32 keys)
    while (npow < n_cand) npow <<= 1;
    if (tid == 0) {
        walk_flags = 0;
        walk_items = 0;
        walk_slow = 0;
        n_zero = 0;
        S_sh = __int_as_float(0x7fc00000);
    }
    __syncthreads();
    if (warp == KB_THREADS / 32 - 1) {
        // the flat list the walk runs through (a loop over segments and their
        // items costs it several times more per item); two segments per lane
        const uint32_t s0 = lane, s1 = lane + 32;
        const uint32_t n0 = s0 < nseg ? s_nit[s0] : 0u, n1 = s1 < nseg ? s_nit[s1] : 0u;
        const uint32_t c0 = s0 < nseg ? (n0 <= spec ? n0 : 1u) : 0u;
        const uint32_t c1 = s1 < nseg ? (n1 <= spec ? n1 : 1u) : 0u;
        const uint32_t i0 = warp_incl_scan_u(c0);
        const uint32_t t0 = __shfl_sync(0xffffffffu, i0, 31);
        const uint32_t i1 = t0 + warp_incl_scan_u(c1);
        const uint32_t all = __reduce_add_sync(0xffffffffu, n0 + n1);
        if (s0 < nseg) {
            if (n0 <= spec) {
                for (uint32_t j = 0; j < n0; j++) fidx[i0 - c0 + j] = (uint16_t)(s0 * spec + j);
            } else {
                fidx[i0 - c0] = (uint16_t)(ITEM_SMEM + s0);
            }
        }
        if (s1 < nseg) {
            if (n1 <= spec) {
                for (uint32_t j = 0; j < n1; j++) fidx[i1 - c1 + j] = (uint16_t)(s1 * spec + j);
            } else {
                fidx[i1 - c1] = (uint16_t)(ITEM_SMEM + s1);
            }
        }
        if (lane == 31) {
            n_flat = i1;
            n_items_all = all;
        }
    }
    // prefix tables of the WINDOW items held in shared memory (offsets by a
    // block scan over the item slots, two per thread; tables that do not fit
    // stay in global memory).  Slots are scanned in order, so the tables that
    // fit are the first ones; their slots are listed (in sitems, unused
    // until the walk) and one warp per listed table issues its copies.
    {
        uint32_t *tlist = reinterpret_cast<uint32_t *>(sitems);
        static_assert(sizeof(sitems) >= ITEM_SMEM * sizeof(uint32_t), "the table list fits the item chunk");
        uint32_t len[2] = {0u, 0u};
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t i = 2 * tid + h;
            if (i < nseg * spec) {
                const uint32_t sg = i / spec;
                if (i - sg * spec < s_nit[sg] && sall[i].kind == CLS_WINDOW)
                    len[h] = min(sall[i].aux, P.ntiles_total - min(sall[i].tile, P.ntiles_total));
            }
        }
        const uint32_t mine = len[0] + len[1];
        const uint32_t nmine = (len[0] != 0u) + (len[1] != 0u);
        const uint32_t incl = warp_incl_scan_u(mine);
        const uint32_t nincl = warp_incl_scan_u(nmine);
        if (lane == 31) {
            wsum[warp] = incl;
            wcnt[warp] = nincl;
        }
        __syncthreads();
        if (tid == 0) {
            uint32_t r = 0, c = 0;
            for (int w = 0; w < KB_THREADS / 32; w++) {
                const uint32_t v = wsum[w], n = wcnt[w];
                wsum[w] = r;
                wcnt[w] = c;
                r += v;
                c += n;
            }
            n_fit = 0;
        }
        __syncthreads();
        uint32_t off = wsum[warp] + incl - mine, t = wcnt[warp] + nincl - nmine;
#pragma unroll
        for (int h = 0; h < 2; h++) {
            const uint32_t i = 2 * tid + h;
            const bool fits = len[h] && off + len[h] <= (uint32_t)WPOOL;
            woff[i] = fits ? off : 0xFFFFFFFFu;
            if (fits) {
                tlist[t] = i;
                atomicAdd(&n_fit, 1u);
            }
            t += len[h] ? 1u : 0u;
            off += len[h];
        }
        __syncthreads();
        // one warp per listed table issues its copies (8-byte chunks)
        static_assert(sizeof(WTile) == 24, "a prefix-table entry is three 8-byte chunks");
        const WTile *wrow_g = P.wpre + (size_t)hrow * P.ntiles_total;
        const uint32_t nf = n_fit;
        for (uint32_t t2 = warp; t2 < nf; t2 += KB_THREADS / 32) {
            const uint32_t i = tlist[t2];
            const Item &itm = sall[i];
            const uint32_t n = min(itm.aux, P.ntiles_total - min(itm.tile, P.ntiles_total));
            const uint2 *src = reinterpret_cast<const uint2 *>(wrow_g + itm.tile);
            uint2 *dst = reinterpret_cast<uint2 *>(wpool + woff[i]);
            for (uint32_t k = lane; k < 3 * n; k += 32) cp_async8(dst + k, src + k);
        }
        cp_async_wait_all();
    }
    __syncthreads();

    if (warp == 0 && P.vs_mode == VS_DRAW) {
        // the normaliser of every shard's terms, from the chain of walks
        if (lane == 0)
            S_sh = P.vs_p2p ? wait_peer_word(P.vs_in + P.vs_soff + row, *P.vs_epoch, P.seq,
                                             const_cast<uint32_t *>(P.kerr))
                            : P.vs_S[row];
    } else if (warp == 0) {
        // ---- the exact walk of the sequential f32 sum (skipped for a NaN
        // row, whose sum is NaN whatever the order; warp 0 must still stay
        // out of the sort's named barrier below) ----
        float entry = P.vs_entry ? P.vs_entry[row] : 0.0f;
        if (P.vs_p2p && P.vs_rank > 0) {   // the previous rank's exit (a peer's store)
            if (lane == 0)
                entry = wait_peer_word(P.vs_in + row, *P.vs_epoch, P.seq, const_cast<uint32_t *>(P.kerr));
            entry = __shfl_sync(0xffffffffu, entry, 0);
        }
        if (!(flags0 & RF_NAN) && entry == entry) {
        SumState st = state_of(entry);   // the empty sum: binade -126, count 0
        uint32_t wflags = 0, nitems_all = 0, nslow = 0;
        const WTile *wrow = P.wpre + (size_t)hrow * P.ntiles_total;
        // add one tile element by element, p recomputed from the logits
        const float *xrow = P.logits + (size_t)row * P.ld;
        auto add_tile = [&](uint32_t tile) {
            st = state_of(walk_recompute_tile<TERM>(float_of(st), xrow, P.vocab, tile, M, P.T, P.rep_penalty,
                                                    row_bitmap(P, hrow), prologue_of(P), Sx, tilep));
        };
        // everything but the common case: a WINDOW crossing, a stored or
        // recomputed tile, a running sum outside the item's binades
        auto slow_item = [&](const Item &it, uint32_t wo) {
            const uint32_t ntl = it.kind == CLS_COMPLEX ? 1u : min(it.aux, P.ntiles_total - it.tile);
            // 0 applied, 1 window crossing, 2 recompute every tile, 3 stored p
            int action = 2;
            const uint32_t par = st.m & 1u;
            if (st.e == it.lo) {
                const uint32_t q = par ? it.q[1] : it.q[0];
                if (st.m + q < QLIM && q < QSAT) {
                    st.m += q;
                    action = 0;
                } else if (it.kind == CLS_WINDOW) {
                    action = 1;
                }
            } else if (it.kind == CLS_WINDOW && st.e == it.lo + 1) {
                const uint32_t q = par ? it.q[3] : it.q[2];
                if (st.m + q < QLIM && q < QSAT) {
                    st.m += q;
                    action = 0;
                }
            }
            if (action == 2 && it.kind == CLS_COMPLEX && it.aux < n_wc) action = 3;
            if (action == 0) return;
            if (action == 3) {   // stored exact p
                st = state_of(seq_add32_smem(float_of(st), wcs + it.aux * TILE));
                return;
            }
            uint32_t from = 0;
            if (action == 1) {
                // the running sum leaves binade lo inside this stretch: first
                // tile c whose prefix count reaches 2^24, from the stretch's
                // prefix table (shared memory when it was gathered)
                const WTile *wp = wo != 0xFFFFFFFFu ? wpool + wo : wrow + it.tile;
                const uint32_t pi = par;
                const Crossing x = find_crossing(wp, ntl, st.m, pi);
                const uint32_t c = x.c, sl = x.slot;
                st.m += x.q_prev;
                if (sl < n_wc) {   // stored exact p
                    st = state_of(seq_add32_smem(float_of(st), wcs + sl * TILE));
                } else {
                    add_tile(it.tile + c);
                }
                from = c + 1;
                if (from < ntl && st.e == it.lo + 1) {
                    const uint32_t q = (st.m & 1u) ? x.suf.q1 : x.suf.q0;
                    if (st.m + q < QLIM && q < QSAT) {
                        st.m += q;
                        from = ntl;
                    }
                }
            }
            if (from < ntl) {
                wflags |= RF_SLOW_WALK;
                nslow += ntl - from;
                for (uint32_t tt = from; tt < ntl; tt++) add_tile(it.tile + tt);
            }
        };
        // The items in walk order from the flat list: the common case stays
        // in the tight loop (the running sum is in the item's binade and
        // stays there: a SIMPLE stretch, or a WINDOW stretch that does not
        // cross), with the next slot and item requested a step ahead; every
        // other item goes through the one call site of slow_item below (so
        // that it is inlined and the walk state stays in registers).  A
        // segment with more items than its shared slots is walked from
        // global memory in chunks.
        static_assert(ITEM_SMEM + MAX_SEG <= 65535, "slots fit 16 bits");
        const uint32_t nf = n_flat;
        nitems_all = n_items_all;
        uint32_t j = 0;
        uint32_t gseg = 0xFFFFFFFFu, gpos = 0, gn = 0;   // the segment walked from global memory
        uint32_t ix = nf > 0 ? fidx[0] : 0u, ixn = nf > 1 ? fidx[1] : 0u;
        for (;;) {
            Item it;
            uint32_t wo = 0xFFFFFFFFu;
            if (gseg != 0xFFFFFFFFu) {
                if (gpos == gn) {
                    gseg = 0xFFFFFFFFu;
                    continue;
                }
                const uint32_t k = gpos % ITEM_CHUNK;
                if (k == 0) {
                    const uint32_t nc = min((uint32_t)ITEM_CHUNK, gn - gpos);
                    __syncwarp();
                    for (uint32_t q = lane; q < nc; q += 32) sitems[q] = ib[gseg * SEG_TILES + gpos + q];
                    __syncwarp();
                }
                it = sitems[k];
                gpos++;
                if (st.e == it.lo) {
                    const uint32_t q = (st.m & 1u) ? it.q[1] : it.q[0];
                    if (st.m + q < QLIM && q < QSAT) {
                        st.m += q;
                        continue;
                    }
                }
            } else {
                for (; j < nf && ix < (uint32_t)ITEM_SMEM; j++) {
                    // kind, lo, q[0], q[1]: the first 16 bytes of the item
                    const uint4 f = *reinterpret_cast<const uint4 *>(sall + ix);
                    const uint32_t ixnn = j + 2 < nf ? fidx[j + 2] : 0u;
                    const uint32_t q = (st.m & 1u) ? f.w : f.z;
                    if (!(st.e == (int)f.y && st.m + q < QLIM && q < QSAT)) break;
                    st.m += q;
                    ix = ixn;
                    ixn = ixnn;
                }
                if (j >= nf) break;
                const uint32_t cur = ix;
                j++;
                ix = ixn;
                ixn = j + 1 < nf ? fidx[j + 1] : 0u;
                if (cur >= (uint32_t)ITEM_SMEM) {
                    gseg = cur - ITEM_SMEM;
                    gpos = 0;
                    gn = s_nit[gseg];
                    continue;
                }
                it = sall[cur];
                wo = woff[cur];
            }
            slow_item(it, wo);
        }
        if (lane == 0) {
            S_sh = float_of(st);
            walk_flags = wflags;
            walk_items = nitems_all;
            walk_slow = nslow;
        }
        }
    } else if (TERM == TERM_P && !big && P.vs_mode != VS_WALK) {
        // ---- candidate keys (exact p), then the sort in shared memory,
        // ascending key, while warp 0 walks ----
        const int t2 = tid - 32, nthr = KB_THREADS - 32;
        uint32_t nz = 0;
        for (uint32_t i = t2; i < npow; i += nthr) {
            unsigned long long k = ~0ull;
            if (i < n_cand) {
                const Candidate c = cg_[i];
                const float p = prob_unnorm(c.v, M, P.T);
                k = cand_key(c.idx, p);
                nz += p > 0.0f ? 0u : 1u;
            }
            skeys[i] = k;
        }
        if (nz) atomicAdd(&n_zero, nz);
        asm volatile("bar.sync 1, %0;" ::"r"(nthr));
        bitonic_sort_keys(skeys, npow, (uint32_t)t2, (uint32_t)nthr,
                          [nthr] { asm volatile("bar.sync 1, %0;" ::"r"(nthr)); });
    }
    __syncthreads();
    if (P.vs_mode == VS_WALK) {   // this shard's part of the chain ends here
        if (tid == 0 && P.vs_p2p) {
            const unsigned long long w = ((unsigned long long)*P.vs_epoch << 32) | __float_as_uint(S_sh);
            if (P.vs_next) {
                st_release_sys_u64(P.vs_next + row, w);
            } else {   // the last rank: the row's S to every rank
                for (uint32_t g = 0; g < P.vs_world; g++) st_release_sys_u64(P.vs_xs[g] + P.vs_soff + row, w);
            }
        } else if (tid == 0) {
            P.vs_exit[row] = S_sh;
        }
        return;
    }
    if (TERM == TERM_H) {
        typical_tail(P, row, hrow, S_sh, skeys, sprobs, red2);
        return;
    }

    const float S = S_sh;
    // a NaN anywhere in the row makes the sum NaN (for shards: the chain's S)
    const bool nan_row = P.vs_mode == VS_DRAW ? (S != S) : (flags0 & RF_NAN) != 0;
    __shared__ uint32_t rawarg_sh, retry_sh;
    __shared__ ArgBest rbest[KB_THREADS / 32];
    if (!nan_row && !(S > 0.0f) && P.vs_mode != VS_DRAW) {
        // sum <= 0 (sampler.zig:89): sampleArgmax of the raw logits.  Not
        // reachable with a finite maximum (its own term is exp(0) = 1).
        const float *x = P.logits + (size_t)row * P.ld;
        const Prologue pr = prologue_of(P);   // the logits the engine passed: with the prologue, unpenalised
        ArgBest b{NEG_INF, 0xFFFFFFFFu};
        for (uint32_t i = tid; i < P.vocab; i += KB_THREADS) {
            const float f = pr.pro ? pr(x[i]) : x[i];
            b = arg_better(b, ArgBest{f != f ? NEG_INF : f, i});
        }
        b = warp_arg(b);
        if (lane == 0) rbest[warp] = b;
        __syncthreads();
        if (tid == 0) {
            ArgBest bb = rbest[0];
            for (int w = 1; w < KB_THREADS / 32; w++) bb = arg_better(bb, rbest[w]);
            const float x0 = pr.pro ? pr(x[0]) : x[0];
            rawarg_sh = (x0 != x0 || bb.i == 0xFFFFFFFFu) ? 0u : bb.i;
        }
        __syncthreads();
    }

    // thread 0's state, kept across the retry below
    uint32_t status = *P.kerr == P.seq ? (uint32_t)ROW_ETIMEOUT : (uint32_t)ROW_OK;
    uint32_t flags = flags0 | walk_flags | (big ? RF_CAND_BIG : 0u);
    uint32_t n_sel = 0;
    bool cover_ok = false;
    float *cums = nullptr;
    uint32_t *idxs = nullptr;   // idxs[2*i] aliases the low word of keys[i]

    // The candidates are sorted by (p descending, index ascending), the
    // filters run over them, and the kept prefix is checked to lie inside
    // them.  A row whose check fails (or every row, with the test hook) goes
    // round once more with every token of the vocabulary as a candidate: the
    // reference's full sort, by the whole CTA in global memory.  Not for a
    // shard's draw, whose logits are spread over the shards.
    unsigned long long *keys = skeys;
    float *probs = sprobs;
    uint32_t n_pos = 0, nc = n_cand;
    for (bool full = false;; full = true) {
        nc = full ? P.vocab : n_cand;
        if (big || full) {
            // keys, then a stable radix sort in global memory (whole CTA)
            uint32_t nz = 0;
            for (uint32_t i = tid; i < nc; i += KB_THREADS) {
                float p;
                uint32_t id = i;
                if (full) {
                    p = exact_p_at(P, row, hrow, i, M);
                } else {
                    const Candidate c = cg_[i];
                    p = prob_unnorm(c.v, M, P.T);
                    id = c.idx;
                }
                gk0[i] = cand_key(id, p);
                nz += p > 0.0f ? 0u : 1u;
            }
            if (nz) atomicAdd(&n_zero, nz);
            __syncthreads();
            uint32_t *cnt = reinterpret_cast<uint32_t *>(sprobs);   // 16 * KB_THREADS words
            keys = cta_radix_sort(gk0, gk1, nc, cnt, red2);
            probs = reinterpret_cast<float *>(keys == gk0 ? gk1 : gk0);
            __syncthreads();
        }
        n_pos = nc - n_zero;   // p = 0 candidates sort last and never matter
        // exact probs in sorted order (sampler.zig:90)
        for (uint32_t i = tid; i < n_pos; i += KB_THREADS) probs[i] = __fdiv_rn(key_p(keys[i]), S);
        __syncthreads();
        // distinct p can round to equal probs; the stable sort then wants index
        // order among them.  Rare: the block checks adjacent pairs first
        bool tie_fix = false;
        {
            const uint32_t *ix = reinterpret_cast<const uint32_t *>(keys);
            bool mine = false;
            for (uint32_t i = tid + 1; i < n_pos; i += KB_THREADS)
                mine |= probs[i] == probs[i - 1] && ix[2 * (i - 1)] > ix[2 * i];
            tie_fix = __syncthreads_or(mine) != 0;
        }
        if (tid == 0) {
            bool retry = false;
            if (!nan_row && S > 0.0f) {
                idxs = reinterpret_cast<uint32_t *>(keys);
                // ties: equal probs from distinct p keep index order (stable sort)
                for (uint32_t i = 1; tie_fix && i < n_pos; i++) {
                    if (probs[i] == probs[i - 1] && idxs[2 * (i - 1)] > idxs[2 * i]) {
                        uint32_t j = i;
                        const uint32_t id = idxs[2 * j];
                        const float pr = probs[j];
                        while (j > 0 && probs[j - 1] == pr && idxs[2 * (j - 1)] > id) {
                            idxs[2 * j] = idxs[2 * (j - 1)];
                            j--;
                        }
                        idxs[2 * j] = id;
                    }
                }
                // The candidates are every token above a floor, i.e. a prefix of
                // the reference's sorted order.  The kept prefix is settled inside
                // it when some filter cuts before its end, when the candidates are
                // all tokens with p > 0, or when the floor is the binding filter's
                // own bound.
                n_sel = n_pos;
                const uint32_t binding = hdr->binding;
                const bool k_act = P.top_k > 0 && P.top_k < P.vocab;
                // top-k (sampler.zig:106-109)
                if (k_act && n_sel > P.top_k) n_sel = P.top_k;
                // top-p (sampler.zig:111-118): the crossing token is deselected
                // too.  Its running sums are kept (in the stored terms' area, free
                // after the walk): the kept mass below is the same sum over a prefix
                cums = nullptr;
                if (P.top_p > 0.0f && P.top_p < 1.0f) {
                    float cum = 0.0f;
                    if (n_sel <= (uint32_t)(WC_CAP * TILE)) cums = wcs;
                    n_sel = seq_first_exceed([&](uint32_t j) { return probs[j]; }, n_sel, P.top_p, cum, cums);
                }
                // min-p (sampler.zig:120-126) against probs[indices[0]]
                if (P.min_p > 0.0f && n_pos > 0) {
                    const float thr = __fmul_rn(probs[0], P.min_p);
                    uint32_t j = 0;
                    while (j < n_sel && !(probs[j] < thr)) j++;
                    n_sel = j;
                }
                cover_ok = full || ((binding == 0 || binding == 1 || binding == 3 || binding == 4 ||
                                     n_sel < n_pos || (k_act && P.top_k <= n_pos)) &&
                                    !(flags0 & RF_CAND_SHORT));   // (a shard's candidates overflowed)
                if (status == ROW_OK && !full && P.vs_mode != VS_DRAW && (!cover_ok || P.force_full))
                    retry = true;
            }
            if (full) flags |= RF_FULL | RF_CAND_BIG;
            n_zero = 0;
            retry_sh = retry ? 1u : 0u;
        }
        __syncthreads();
        if (!retry_sh) break;
    }
    if (tid != 0) return;

    bool pending = false;
    uint32_t token = 0;
    uint32_t path = 0;
    uint32_t n_kept = 0;
    float total = 0.0f, u = __int_as_float(0x7fc00000);
    uint64_t s4[4];
    uint64_t *rng = P.rng + (size_t)hrow * 4;
    s4[0] = rng[0]; s4[1] = rng[1]; s4[2] = rng[2]; s4[3] = rng[3];
    float S_rep = S;

    if (nan_row) {
        // sum is NaN (sampler.zig:87-90): every comparison is false, the stable
        // sort keeps index order, nothing is deselected, total is NaN, one
        // draw, and the walk never returns: indices[0] == 0.
        u = rng_float(s4);
        token = 0;
        path = 5;
        total = __int_as_float(0x7fc00000);
        S_rep = total;
    } else if (!(S > 0.0f)) {
        token = rawarg_sh;   // sampler.zig:89
        path = 1;
        if (P.vs_mode == VS_DRAW) status = ROW_EINTERNAL;   // the raw logits are spread over the shards
    } else {
        if (status != ROW_OK) {
            // a bounded device wait gave up: nothing of this call is trusted
        } else if (!cover_ok) {
            status = ROW_EINTERNAL;   // (only a shard's draw: other rows took the retry)
            flags |= RF_CAND_SHORT;
        } else if (P.tmode != TYP_OFF) {
            // typical-p follows in the entropy passes (sampler.zig:128-154):
            // hand over S, indices[0] and the selected set (index, P)
            pending = true;
            Candidate *cw = P.cand + (size_t)hrow * P.cand_stride;
            if (P.tmode == TYP_SELECTED)
                for (uint32_t j = 0; j < n_sel; j++) cw[j] = Candidate{idxs[2 * j], probs[j]};
            hdr->n_sel = P.tmode == TYP_SELECTED ? n_sel : 0u;
            hdr->top_idx = n_pos > 0 ? idxs[0] : 0u;
            hdr->flags = flags0 | (flags & RF_FULL);   // (the typical tail's trace reports it)
        } else {
            // kept mass in sorted order (sampler.zig:156-159): the same adds
            // from 0 as top-p's running sum, so its value at the last kept
            // token when that was recorded
            total = (cums && n_sel > 0) ? cums[n_sel - 1] : seq_sum([&](uint32_t j) { return probs[j]; }, n_sel);
            n_kept = n_sel;
            if (!(total > 0.0f)) {
                token = n_pos > 0 ? idxs[0] : 0u;  // sampler.zig:160
                path = 2;
            } else {
                u = rng_float(s4);
                const uint32_t j = seq_draw([&](uint32_t i) { return probs[i]; }, n_sel, __fmul_rn(u, total));
                token = idxs[0];
                path = 4;
                if (j < n_sel) {
                    token = idxs[2 * j];
                    path = 3;
                }
            }
        }
    }
    if (P.tmode != TYP_OFF) {
        hdr->S_exact = S;
        hdr->tdone = pending ? 0u : 1u;
        hdr->n_cand = 0;   // the entropy pass appends its own candidates
        hdr->n_wc = 0;
        if (pending) return;   // the typical tail writes token, state and trace
    }
    if (status == ROW_OK) {
        rng[0] = s4[0]; rng[1] = s4[1]; rng[2] = s4[2]; rng[3] = s4[3];
        P.out[row] = token;
    } else {
        P.out[row] = 0xFFFFFFFFu;
    }
    RowTrace tr;
    tr.S = S_rep;
    tr.total = total;
    tr.u = u;
    tr.n_kept = n_kept;
    tr.path = path;
    tr.flags = flags;
    tr.n_cand = nc;
    tr.status = status;
    tr.n_items = walk_items;
    tr.n_wc = hdr->n_wc;
    tr.n_slow = walk_slow;
    tr.H = __int_as_float(0x7fc00000);
    P.trace[hrow] = tr;
}

// A rank's exchange words for the vocabulary-sharded step through peer
// memory (u64 words; B = the handle's batch, G = the world):
//   [0, B)            entry: the previous rank's exit state of each row
//   [B, 2B)           S: the row's normaliser, from the last rank
//   [2B]              the step tag (low 32 bits)
//   then G x B        tags of the ranks' partials
//   then G x B x 2    the ranks' partials (VsPart)
//   then G x B        the ranks' candidate counts, tagged
//   then G x B x CAP  the ranks' candidates (Candidate)
// A tagged word is (tag << 32) | payload, stored with release semantics at
// system scope after the data it covers.
struct VsLayout {
    size_t ptag, parts, ctag, cand, words;
    __host__ __device__ VsLayout(uint32_t B, uint32_t G) {
        ptag = 2 * (size_t)B + 1;
        parts = ptag + (size_t)G * B;
        ctag = parts + 2 * (size_t)G * B;
        cand = ctag + (size_t)G * B;
        words = cand + (size_t)G * B * VS_CAND_CAP;
    }
};
struct VsPeer {
    unsigned long long *const *xs;   // every rank's exchange words (null: host collectives)
    unsigned long long *own;         // this rank's
    uint32_t world, rank, batch;
};

// The peer-memory chain's step tag: one increment at the start of every step
// (so a replayed CUDA graph tags each replay afresh; every rank makes the same
// calls, so the ranks' tags agree).  Never 0, the value of unwritten words.
__global__ void k_vs_epoch(uint32_t *epoch) {
    const uint32_t e = *epoch + 1u;
    *epoch = e == 0u ? 1u : e;
}

// Vocabulary sharding: each row's partial over this shard, from the
// statistics pass's segment aggregates (one warp per row).
__global__ void k_vs_partials(const SegStat *__restrict__ sstat, uint32_t nseg, uint32_t rows, float c2,
                              VsPart *__restrict__ out, VsPeer pe) {
    const uint32_t row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32, lane = threadIdx.x & 31u;
    if (row >= rows) return;
    const SegStat *S = sstat + (size_t)row * MAX_SEG;
    float m = NEG_INF;
    uint32_t nf = 0;
    for (uint32_t c = lane; c < nseg; c += 32) {
        m = fmaxf(m, S[c].smax);
        nf |= S[c].nonfin;
    }
    m = warp_max(m);
    nf = __any_sync(0xffffffffu, nf != 0) ? 1u : 0u;
    double sum = 0.0;
    for (uint32_t c = lane; c < nseg; c += 32)
        if (S[c].smax > NEG_INF) sum += S[c].ssum * (double)ex2_approx((S[c].smax - m) * c2);
    sum = warp_sum_d(sum);
    if (lane == 0 && !pe.xs) out[row] = VsPart{m, nf, sum};
    if (pe.xs) {   // to every rank's words (lane g, g + 32, ...), then the tag
        const VsLayout L(pe.batch, pe.world);
        const uint32_t tag = *reinterpret_cast<const uint32_t *>(pe.own + 2 * (size_t)pe.batch);
        const size_t k = (size_t)pe.rank * pe.batch + row;
        for (uint32_t g = lane; g < pe.world; g += 32) {
            unsigned long long *x = pe.xs[g];
            *reinterpret_cast<VsPart *>(x + L.parts + 2 * k) = VsPart{m, nf, sum};
            st_release_sys_u64(x + L.ptag + k, ((unsigned long long)tag << 32) | 1ull);
        }
    }
}

// This shard's candidates with global token ids (col0 added), at most
// VS_CAND_CAP per row; count[row] = VS_CAND_CAP + 1 marks an overflow.
__global__ void k_vs_export(const RowHdr *__restrict__ hdr, const Candidate *__restrict__ cand, uint32_t cand_stride,
                            uint32_t col0, Candidate *__restrict__ out, uint32_t *__restrict__ count, VsPeer pe) {
    const uint32_t row = blockIdx.x;
    const uint32_t n = hdr[row].n_cand;
    const uint32_t m = n < VS_CAND_CAP ? n : VS_CAND_CAP;
    const uint32_t cnt = n <= VS_CAND_CAP ? n : VS_CAND_CAP + 1;
    if (!pe.xs) {
        for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
            const Candidate c = cand[(size_t)row * cand_stride + i];
            out[(size_t)row * VS_CAND_CAP + i] = Candidate{c.idx + col0, c.v};
        }
        if (threadIdx.x == 0) count[row] = cnt;
        return;
    }
    // to every rank's words; then, once the block's stores are done, the
    // tagged counts
    const VsLayout L(pe.batch, pe.world);
    const size_t k = (size_t)pe.rank * pe.batch + row;
    for (uint32_t i = threadIdx.x; i < m; i += blockDim.x) {
        const Candidate c = cand[(size_t)row * cand_stride + i];
        const Candidate o{c.idx + col0, c.v};
        for (uint32_t g = 0; g < pe.world; g++)
            *reinterpret_cast<Candidate *>(pe.xs[g] + L.cand + k * VS_CAND_CAP + i) = o;
    }
    __syncthreads();
    if (threadIdx.x < pe.world) {
        __threadfence_system();
        const uint32_t tag = *reinterpret_cast<const uint32_t *>(pe.own + 2 * (size_t)pe.batch);
        st_release_sys_u64(pe.xs[threadIdx.x] + L.ctag + k, ((unsigned long long)tag << 32) | cnt);
    }
}

// The candidates of every shard ([world][rows][VS_CAND_CAP]) as this
// handle's candidate list of each row (a shard that overflowed flags the row).
__global__ void k_vs_merge(const Candidate *__restrict__ all, const uint32_t *__restrict__ counts, uint32_t world,
                           uint32_t rows, RowHdr *__restrict__ hdr, Candidate *__restrict__ cand, uint32_t cand_stride,
                           VsPeer pe, uint32_t seq, uint32_t *kerr) {
    const uint32_t row = blockIdx.x;
    __shared__ uint32_t base[65], pcount[64];
    if (pe.xs) {   // the ranks' candidates in this rank's words, once their counts carry the step's tag
        const VsLayout L(pe.batch, pe.world);
        all = reinterpret_cast<const Candidate *>(pe.own + L.cand);
        if (threadIdx.x < world) {
            const uint32_t tag = *reinterpret_cast<const uint32_t *>(pe.own + 2 * (size_t)pe.batch);
            uint32_t c = 0;
            wait_peer_bits(pe.own + L.ctag + (size_t)threadIdx.x * pe.batch + row, tag, seq, kerr, c);
            pcount[threadIdx.x] = c;   // (0 when the wait gave up: the call's rows then fail)
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        uint32_t b = 0, over = 0;
        for (uint32_t h = 0; h < world; h++) {
            const uint32_t c = pe.xs ? pcount[h] : counts[(size_t)h * rows + row];
            base[h] = b;
            over |= c > VS_CAND_CAP ? 1u : 0u;
            b += c > VS_CAND_CAP ? VS_CAND_CAP : c;
        }
        base[world] = b;
        hdr[row].n_cand = b < cand_stride ? b : cand_stride;
        if (over) atomicOr(&hdr[row].flags, RF_CAND_SHORT);   // the row cannot be drawn exactly
    }
    __syncthreads();
    for (uint32_t h = 0; h < world; h++) {
        const uint32_t n = base[h + 1] - base[h];
        for (uint32_t i = threadIdx.x; i < n; i += blockDim.x)
            if (base[h] + i < cand_stride)
                cand[(size_t)row * cand_stride + base[h] + i] =
                    all[((size_t)h * (pe.xs ? pe.batch : rows) + row) * VS_CAND_CAP + i];
    }
}

// Repetition-penalty pre-pass (sampler.zig:54-75), one CTA per row: the
// row's bitmap of penalised ids, bit k of word t for token 32 t + k.  The
// reference penalises each token id found among the last `win` previous
// tokens once, however often it occurs there; ids outside the vocabulary
// match no logit.
__global__ void __launch_bounds__(256) k0_penalty(const uint32_t *__restrict__ prev, uint32_t n_prev, uint32_t win,
                                                  uint32_t vocab, uint32_t col0, uint32_t row0, uint32_t words,
                                                  uint32_t *__restrict__ bm) {
    const uint32_t row = blockIdx.x;
    uint32_t *b = bm + (size_t)(row0 + row) * words;
    for (uint32_t i = threadIdx.x; i < words; i += blockDim.x) b[i] = 0u;
    __syncthreads();
    const uint32_t *p = prev + (size_t)row * n_prev + (n_prev - win);
    for (uint32_t j = threadIdx.x; j < win; j += blockDim.x) {
        const uint32_t id = p[j] - col0;   // this (shard's) slice of the vocabulary
        if (id < vocab) atomicOr(&b[id >> 5], 1u << (id & 31u));
    }
}

}  // namespace bs

// ===========================================================================
// C ABI
// ===========================================================================
using namespace bs;

struct bs_sampler {
    bs_config cfg;
    uint32_t batch;
    uint32_t vocab;
    int device;
    uint32_t nseg, ntiles_total;
    size_t smem_b;
    uint64_t *d_rng;
    RowHdr *d_hdr;
    TileStat *d_tstat;
    SegStat *d_sstat;
    uint32_t *d_penbm;       // repetition-penalty bitmaps, ntiles_total words per row
    uint32_t *d_fctl;        // persistent kernel: 4 control words + batch row counters (zeroed per call)
    unsigned long long *d_ready;   // persistent kernel: ready list, batch slots
    float *d_mhist;
    RowInfo *d_rinfo;
    Item *d_items;
    WTile *d_wpre;
    float *d_wc;
    Candidate *d_cand;
    unsigned long long *d_ctmp;
    uint32_t cand_stride;
    RowTrace *d_trace;
    uint32_t *d_kerr;        // sequence number of the last call whose bounded device wait gave up
    uint32_t seq;            // sequence number of the last call (0 before the first)
    uint32_t fused;          // 1: the persistent kernel instead of separate statistics / row / main kernels
    uint32_t force_full;     // test hook: every row takes the full-vocabulary retry
    Prologue pro;            // the logit prologue set by bs_set_logit_prologue (pro.pro == 0: none)
    // the vocabulary-shard call in progress (bs_vshard_stats sets it up)
    K12Params vs_A;
    KBParams vs_B;
    uint32_t vs_rows;
    bool vs_ready;
    // peer-memory chain: this rank's exchange words (entry, then S, batch
    // each), the ranks' exchange words as this device sees them (opened
    // peer mappings), and the device array of those pointers
    unsigned long long *d_xchg;
    unsigned long long *peer_xchg[64];
    unsigned long long **d_peer_xchg;
    uint32_t p2p_world, p2p_rank, xchg_world;
    float *d_logits_stage;   // host-path staging
    uint32_t *d_prev_stage;
    uint32_t *d_out_stage;
    size_t stage_floats;
    size_t stage_prev;
    cudaStream_t stream;
    cudaEvent_t *prof_ev;    // profiling ring: 4 events per bs_sample call
    uint32_t prof_cap, prof_n;
};

static bs_status cuda_status(cudaError_t e) { return e == cudaSuccess ? BS_OK : BS_ECUDA; }

#define BS_CUDA(call)                                                 \
    do {                                                              \
        cudaError_t err__ = (call);                                   \
        if (err__ != cudaSuccess) {                                   \
            fprintf(stderr, "b200_sampler: %s failed: %s\n", #call,   \
                    cudaGetErrorString(err__));                       \
            return BS_ECUDA;                                          \
        }                                                             \
    } while (0)

extern "C" void bs_config_default(bs_config *cfg) {
    if (!cfg) return;
    cfg->temperature = 0.8f;
    cfg->top_k = 0;
    cfg->top_p = 0.9f;
    cfg->min_p = 0.0f;
    cfg->typical_p = 1.0f;
    cfg->_pad0 = 0;
    cfg->seed = 0;
    cfg->repetition_window = 32;
    cfg->repetition_penalty = 1.1f;
}

extern "C" const char *bs_status_string(bs_status st) {
    switch (st) {
        case BS_OK: return "ok";
        case BS_EINVAL: return "invalid argument";
        case BS_ENOMEM: return "out of memory";
        case BS_ECUDA: return "CUDA error";
        case BS_ENCCL: return "NCCL error";
        case BS_ETIMEOUT: return "device wait timed out";
        case BS_ENOTSUP: return "not supported by this build";
        case BS_EINTERNAL: return "internal consistency check failed";
    }
    return "unknown status";
}

static void free_all(bs_sampler *s) {
    if (!s) return;
    cudaFree(s->d_rng);
    cudaFree(s->d_hdr);
    cudaFree(s->d_tstat);
    cudaFree(s->d_sstat);
    cudaFree(s->d_penbm);
    cudaFree(s->d_fctl);
    cudaFree(s->d_ready);
    cudaFree(s->d_mhist);
    cudaFree(s->d_rinfo);
    cudaFree(s->d_items);
    cudaFree(s->d_wpre);
    cudaFree(s->d_wc);
    cudaFree(s->d_cand);
    cudaFree(s->d_ctmp);
    cudaFree(s->d_trace);
    cudaFree(s->d_kerr);
    cudaFree(s->d_logits_stage);
    cudaFree(s->d_prev_stage);
    cudaFree(s->d_out_stage);
    for (uint32_t g = 0; g < s->p2p_world && g < 64; g++)
        if (g != s->p2p_rank && s->peer_xchg[g]) cudaIpcCloseMemHandle(s->peer_xchg[g]);
    cudaFree(s->d_peer_xchg);
    cudaFree(s->d_xchg);
    if (s->stream) cudaStreamDestroy(s->stream);
    for (uint32_t i = 0; s->prof_ev && i < 4 * s->prof_cap; i++) cudaEventDestroy(s->prof_ev[i]);
    delete[] s->prof_ev;
}

// Dynamic shared memory of the walk kernel (candidate keys, stored terms,
// probabilities).
constexpr size_t KB_SMEM = (size_t)CAND_SMEM * 8 + (size_t)WC_CAP * TILE * 4 + (size_t)CAND_SMEM * 4;

// Kernel attributes are per device: set them once on each device, with that
// device current.
constexpr int MAX_DEVICES = 64;
static bool g_attrs_set[MAX_DEVICES];
static std::mutex g_attrs_mu;
static cudaError_t ensure_kernel_attrs(int dev) {
    if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_attrs_mu);
    if (g_attrs_set[dev]) return cudaSuccess;
    cudaError_t e = cudaFuncSetAttribute(kernel_b<TERM_P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KB_SMEM);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kernel_b<TERM_H>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)KB_SMEM);
    if (e == cudaSuccess) g_attrs_set[dev] = true;
    return e;
}

// Resident CTAs of a persistent kernel on a device (all of them run at once):
// kind 1 the task-queue kernel k_fused, kind 2 the read-once kernel k_resident.
static int g_fused_ctas[MAX_DEVICES][2];
static cudaError_t fused_grid(int dev, int *ctas, uint32_t kind = 1) {
    if (dev < 0 || dev >= MAX_DEVICES || kind < 1 || kind > 2) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_attrs_mu);
    int &n = g_fused_ctas[dev][kind - 1];
    if (n == 0) {
        int per_sm = 0, sms = 0;
        cudaError_t e = kind == 1 ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_fused, K12_THREADS, 0)
                                  : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_resident, K12_THREADS, 0);
        if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess) return e;
        if (per_sm <= 0 || sms <= 0) return cudaErrorInvalidConfiguration;
        n = per_sm * sms;
    }
    *ctas = n;
    return cudaSuccess;
}

// The next sequence number of a call (never 0, the value of a clear error word).
static uint32_t next_seq(uint32_t &seq) {
    seq = seq + 1u == 0u ? 1u : seq + 1u;
    return seq;
}

extern "C" bs_status bs_create(const bs_config *cfg, uint32_t batch, uint32_t vocab, int device,
                               const uint64_t *seeds, bs_sampler **out) {
    if (!cfg || !out || batch == 0 || vocab == 0) return BS_EINVAL;
    if (vocab > (uint32_t)(MAX_SEG * SEG_ELEMS)) return BS_ENOTSUP;
    *out = nullptr;
    BS_CUDA(cudaSetDevice(device));
    bs_sampler *s = new (std::nothrow) bs_sampler();
    if (!s) return BS_ENOMEM;
    memset(s, 0, sizeof(*s));
    s->cfg = *cfg;
    s->batch = batch;
    s->vocab = vocab;
    s->device = device;
    s->ntiles_total = (vocab + TILE - 1) / TILE;
    s->nseg = (s->ntiles_total + SEG_TILES - 1) / SEG_TILES;
    s->smem_b = KB_SMEM;
    s->cand_stride = (vocab + 31u) & ~31u;

    cudaError_t e = cudaSuccess;
    e = cudaMalloc(&s->d_rng, (size_t)batch * 4 * sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_hdr, (size_t)batch * sizeof(RowHdr));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_tstat, (size_t)batch * s->ntiles_total * sizeof(TileStat));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_sstat, (size_t)batch * MAX_SEG * sizeof(SegStat));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_penbm, (size_t)batch * s->ntiles_total * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_fctl, (4 + (size_t)batch) * sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_ready, (size_t)batch * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(s->d_ready, 0, (size_t)batch * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_mhist, (size_t)batch * MAX_SEG * KH_BINS * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_rinfo, (size_t)batch * sizeof(RowInfo));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_items, (size_t)batch * s->ntiles_total * sizeof(Item));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_wpre, (size_t)batch * s->ntiles_total * sizeof(WTile));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_wc, (size_t)batch * WC_CAP * TILE * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_cand, (size_t)batch * s->cand_stride * sizeof(Candidate));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_ctmp, (size_t)batch * 2 * s->cand_stride * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_trace, (size_t)batch * sizeof(RowTrace));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_kerr, sizeof(uint32_t));
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        free_all(s);
        delete s;
        return e == cudaErrorMemoryAllocation ? BS_ENOMEM : BS_ECUDA;
    }
    // seed rows (Sampler.init: zero -> 0xDEADBEEF)
    uint64_t *h = new (std::nothrow) uint64_t[(size_t)batch * 4];
    if (!h) {
        free_all(s);
        delete s;
        return BS_ENOMEM;
    }
    for (uint32_t r = 0; r < batch; r++) {
        uint64_t sd = seeds ? seeds[r] : cfg->seed + r;
        if (sd == 0) sd = 0xDEADBEEFULL;
        rng_seed(h + 4 * (size_t)r, sd);
    }
    e = cudaMemcpy(s->d_rng, h, (size_t)batch * 4 * sizeof(uint64_t), cudaMemcpyHostToDevice);
    delete[] h;
    if (e == cudaSuccess) e = cudaMemset(s->d_trace, 0, (size_t)batch * sizeof(RowTrace));
    if (e == cudaSuccess) e = cudaMemset(s->d_kerr, 0, sizeof(uint32_t));
    if (e == cudaSuccess) e = ensure_kernel_attrs(device);
    if (e != cudaSuccess) {
        fprintf(stderr, "b200_sampler: setup failed: %s\n", cudaGetErrorString(e));
        free_all(s);
        delete s;
        return BS_ECUDA;
    }
    *out = s;
    return BS_OK;
}

extern "C" void bs_destroy(bs_sampler *s) {
    if (!s) return;
    cudaSetDevice(s->device);
    free_all(s);
    delete s;
}

// The prologue for a model's final_logit_softcapping and logit_scale, as the
// engine decides it (engine.zig:341,351): the soft-cap when it is > 0, the
// scale unless it is 1 or 0; the reciprocal is one f32 division, as
// `1.0 / cfg.logit_scale` in the engine.
static Prologue make_prologue(float softcap, float logit_scale) {
    Prologue p{0u, softcap, 1.0f};
    if (softcap > 0.0f) p.pro |= PRO_CAP;
    if (logit_scale != 1.0f && logit_scale != 0.0f) {
        p.pro |= PRO_SCALE;
        volatile float one = 1.0f;   // one IEEE f32 division at run time
        p.pinv = one / logit_scale;
    }
    return p;
}

static bs_status argmax_launch(const float *d_logits, size_t ld, uint32_t rows, uint32_t vocab, Prologue pr,
                               uint32_t *d_out, void *stream) {
    if (!d_logits || !d_out || vocab == 0 || ld < vocab) return BS_EINVAL;
    if (rows == 0) return BS_OK;
    argmax_kernel<<<rows, 512, 0, (cudaStream_t)stream>>>(d_logits, ld, vocab, d_out, pr);
    return cuda_status(cudaGetLastError());
}

extern "C" bs_status bs_argmax(const float *d_logits, size_t ld, uint32_t rows, uint32_t vocab,
                               uint32_t *d_out, void *stream) {
    return argmax_launch(d_logits, ld, rows, vocab, Prologue{0u, 0.0f, 1.0f}, d_out, stream);
}

extern "C" bs_status bs_argmax_ex(const float *d_logits, size_t ld, uint32_t rows, uint32_t vocab,
                                  float final_logit_softcapping, float logit_scale, uint32_t *d_out, void *stream) {
    return argmax_launch(d_logits, ld, rows, vocab, make_prologue(final_logit_softcapping, logit_scale), d_out,
                         stream);
}

extern "C" bs_status bs_set_logit_prologue(bs_sampler *s, float final_logit_softcapping, float logit_scale) {
    if (!s) return BS_EINVAL;
    s->pro = make_prologue(final_logit_softcapping, logit_scale);
    return BS_OK;
}

// A launch that may overlap the previous kernel of the stream (the kernel
// waits for it with griddepcontrol.wait before reading its results).
template <typename... Args>
static cudaError_t launch_dependent(void (*kern)(Args...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                    Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

// The kernels' parameters of one call (rows [row0, row0 + rows) of the
// handle, logits row i at d_logits + i ld).
static void make_params(const bs_sampler *s, uint32_t seq, const float *d_logits, size_t ld, uint32_t row0,
                        uint32_t rows, const uint32_t *d_prev, uint32_t n_prev, uint32_t *d_out, K12Params &A,
                        KBParams &B, bool &pen, uint32_t &win) {
    const bs_config &c = s->cfg;
    // sampler.zig:58 -- the penalty applies to the last min(n_prev, window) ids
    pen = c.repetition_penalty != 1.0f && d_prev != nullptr && n_prev > 0 && c.repetition_window > 0;
    win = pen ? (n_prev < c.repetition_window ? n_prev : c.repetition_window) : 0u;

    A.logits = d_logits;
    A.ld = ld;
    A.pen_bm = pen ? s->d_penbm : nullptr;
    A.vocab = s->vocab;
    A.row0 = row0;
    A.rows = rows;
    A.T = c.temperature;
    A.c2 = (float)(1.4426950408889634 / (double)c.temperature);
    A.top_k = c.top_k;
    A.top_p = c.top_p;
    A.min_p = c.min_p;
    A.rep_penalty = c.repetition_penalty;
    A.nseg = s->nseg;
    A.ntiles_total = s->ntiles_total;
    A.tstat = s->d_tstat;
    A.sstat = s->d_sstat;
    A.mhist = s->d_mhist;
    A.rinfo = s->d_rinfo;
    A.hdr = s->d_hdr;
    A.items = s->d_items;
    A.wpre = s->d_wpre;
    A.wcdata = s->d_wc;
    A.cand = s->d_cand;
    A.cand_stride = s->cand_stride;
    A.kerr = s->d_kerr;
    A.seq = seq;
    A.pro = s->pro.pro;
    A.softcap = s->pro.softcap;
    A.pinv = s->pro.pinv;
    A.ctl = s->d_fctl;
    A.ready = s->d_ready;
    A.vs_parts = nullptr;
    A.vs_world = 1;
    A.vs_rank = 0;
    A.vs_ptag = nullptr;
    A.vs_epoch = nullptr;
    A.typical_p = c.typical_p;
    A.tmode = typical_mode(c.typical_p, c.top_k, s->vocab, c.top_p, c.min_p);

    B.logits = d_logits;
    B.ld = ld;
    B.pen_bm = A.pen_bm;
    B.vocab = s->vocab;
    B.row0 = row0;
    B.T = c.temperature;
    B.top_k = c.top_k;
    B.top_p = c.top_p;
    B.min_p = c.min_p;
    B.typical_p = c.typical_p;
    B.rep_penalty = c.repetition_penalty;
    B.ntiles_total = s->ntiles_total;
    B.hdr = s->d_hdr;
    B.items = s->d_items;
    B.wcdata = s->d_wc;
    B.wpre = s->d_wpre;
    B.cand = s->d_cand;
    B.ctmp = s->d_ctmp;
    B.cand_stride = s->cand_stride;
    B.rng = s->d_rng;
    B.trace = s->d_trace;
    B.kerr = s->d_kerr;
    B.seq = seq;
    B.pro = s->pro.pro;
    B.softcap = s->pro.softcap;
    B.pinv = s->pro.pinv;
    B.rinfo = s->d_rinfo;
    B.tmode = A.tmode;
    B.force_full = s->force_full;
    B.out = d_out;
    B.vs_mode = VS_OFF;
    B.vs_entry = nullptr;
    B.vs_exit = nullptr;
    B.vs_S = nullptr;
    B.vs_p2p = 0;
    B.vs_world = 1;
    B.vs_rank = 0;
    B.vs_soff = 0;
    B.vs_in = nullptr;
    B.vs_epoch = nullptr;
    B.vs_next = nullptr;
    B.vs_xs = nullptr;

}

// Rows [row0, row0 + rows) of a call through the separate kernels on one
// stream: penalty bitmap, statistics, row reduction, main pass, walk and draw
// (with typical-p, the entropy main pass and walk).  The kernels after the
// statistics pass overlap their predecessors (programmatic dependent launch).
static cudaError_t launch_group(bs_sampler *s, uint32_t seq, const float *d_logits, size_t ld, uint32_t row0,
                                uint32_t rows, const uint32_t *d_prev, uint32_t n_prev, uint32_t *d_out,
                                cudaStream_t st) {
    K12Params A;
    KBParams B;
    bool pen = false;
    uint32_t win = 0;
    make_params(s, seq, d_logits, ld, row0, rows, d_prev, n_prev, d_out, A, B, pen, win);
    const dim3 g12(s->nseg, rows), g2(s->nseg * rows);
    if (pen) k0_penalty<<<rows, 256, 0, st>>>(d_prev, n_prev, win, s->vocab, 0u, row0, s->ntiles_total, s->d_penbm);
    k1_stats<<<g12, K12_THREADS, 0, st>>>(A);
    cudaError_t e = launch_dependent(k1_rows, dim3(rows), dim3(K12_THREADS), 0, st, A);
    if (e == cudaSuccess) e = launch_dependent(k2_main<TERM_P>, g2, dim3(K12_THREADS), 0, st, A);
    if (A.tmode != TYP_OFF) {
        if (e == cudaSuccess) e = launch_dependent(kernel_b<TERM_P>, dim3(rows), dim3(KB_THREADS), s->smem_b, st, B);
        if (e == cudaSuccess) e = launch_dependent(k2_main<TERM_H>, g2, dim3(K12_THREADS), 0, st, A);
    }
    if (e == cudaSuccess)
        e = launch_dependent(A.tmode != TYP_OFF ? kernel_b<TERM_H> : kernel_b<TERM_P>, dim3(rows), dim3(KB_THREADS),
                             s->smem_b, st, B);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) fprintf(stderr, "b200_sampler: launch failed: %s\n", cudaGetErrorString(e));
    return e;
}

// One sampling call; `seq` numbers it for the error word (never 0).
static bs_status sample_impl(bs_sampler *s, uint32_t seq, const float *d_logits, size_t ld, uint32_t row0,
                             uint32_t rows, const uint32_t *d_prev, uint32_t n_prev, uint32_t *d_out, void *stream) {
    if (!s || !d_logits || !d_out || ld < s->vocab) return BS_EINVAL;
    if (row0 > s->batch || rows > s->batch - row0) return BS_EINVAL;
    if (rows == 0) return BS_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const bs_config &c = s->cfg;
    // sampler.zig:50 -- temperature <= 0: argmax of the logits (after the
    // engine's prologue), no penalty, no draw
    if (c.temperature <= 0.0f) return argmax_launch(d_logits, ld, rows, s->vocab, s->pro, d_out, stream);

    K12Params A;
    KBParams B;
    bool pen = false;
    uint32_t win = 0;
    make_params(s, seq, d_logits, ld, row0, rows, d_prev, n_prev, d_out, A, B, pen, win);

    // statistics, row reduction | main pass | walk and draw.  With typical-p
    // the normaliser's walk hands over to a second main pass and walk over
    // the entropy terms (profiled with the main pass | the final walk).
    cudaEvent_t *ev = nullptr;
    if (s->prof_ev && s->prof_n < s->prof_cap) ev = s->prof_ev + 4 * s->prof_n++;
    // the persistent kernel for the statistics, row reduction and main pass
    // (one launch; the walk follows as an ordinary launch).  Profiling runs
    // the separate kernels, whose groups the events can split
    if (!ev && s->fused && s->d_fctl) {
        int ctas = 0;
        const uint32_t kind = s->fused == 2 ? 2u : 1u;
        cudaError_t e = fused_grid(s->device, &ctas, kind);
        const uint32_t tasks = rows * s->nseg;
        if (e == cudaSuccess) e = cudaMemsetAsync(s->d_fctl, 0, (4 + (size_t)rows) * sizeof(uint32_t), st);
        if (e == cudaSuccess && pen)
            k0_penalty<<<rows, 256, 0, st>>>(d_prev, n_prev, win, s->vocab, 0u, row0, s->ntiles_total, s->d_penbm);
        const uint32_t grid = (uint32_t)ctas < tasks ? (uint32_t)ctas : tasks;
        if (e == cudaSuccess) {
            if (kind == 2) k_resident<<<grid, K12_THREADS, 0, st>>>(A);
            else k_fused<<<grid, K12_THREADS, 0, st>>>(A);
        }
        const dim3 g2(s->nseg * rows);
        if (A.tmode != TYP_OFF) {
            if (e == cudaSuccess) {
                kernel_b<TERM_P><<<rows, KB_THREADS, s->smem_b, st>>>(B);
                e = launch_dependent(k2_main<TERM_H>, g2, dim3(K12_THREADS), 0, st, A);
            }
            if (e == cudaSuccess)
                e = launch_dependent(kernel_b<TERM_H>, dim3(rows), dim3(KB_THREADS), s->smem_b, st, B);
        } else if (e == cudaSuccess) {
            kernel_b<TERM_P><<<rows, KB_THREADS, s->smem_b, st>>>(B);
        }
        if (e == cudaSuccess) e = cudaGetLastError();
        if (e != cudaSuccess) fprintf(stderr, "b200_sampler: launch failed: %s\n", cudaGetErrorString(e));
        return cuda_status(e);
    }
    if (!ev) return cuda_status(launch_group(s, seq, d_logits, ld, row0, rows, d_prev, n_prev, d_out, st));
    // profiled: the same launches with event records between the kernel
    // groups (which keep them from overlapping)
    const dim3 g12(s->nseg, rows), g2(s->nseg * rows);
    if (ev) cudaEventRecord(ev[0], st);
    if (pen) k0_penalty<<<rows, 256, 0, st>>>(d_prev, n_prev, win, s->vocab, 0u, row0, s->ntiles_total, s->d_penbm);
    k1_stats<<<g12, K12_THREADS, 0, st>>>(A);
    cudaError_t e = launch_dependent(k1_rows, dim3(rows), dim3(K12_THREADS), 0, st, A);
    if (ev) cudaEventRecord(ev[1], st);
    if (e == cudaSuccess) e = launch_dependent(k2_main<TERM_P>, g2, dim3(K12_THREADS), 0, st, A);
    if (A.tmode != TYP_OFF) {
        if (e == cudaSuccess) e = launch_dependent(kernel_b<TERM_P>, dim3(rows), dim3(KB_THREADS), s->smem_b, st, B);
        if (e == cudaSuccess) e = launch_dependent(k2_main<TERM_H>, g2, dim3(K12_THREADS), 0, st, A);
    }
    if (ev) cudaEventRecord(ev[2], st);
    if (e == cudaSuccess)
        e = launch_dependent(A.tmode != TYP_OFF ? kernel_b<TERM_H> : kernel_b<TERM_P>, dim3(rows), dim3(KB_THREADS),
                             s->smem_b, st, B);
    if (ev) cudaEventRecord(ev[3], st);
    if (e == cudaSuccess) e = cudaGetLastError();
    if (e != cudaSuccess) fprintf(stderr, "b200_sampler: launch failed: %s\n", cudaGetErrorString(e));
    return cuda_status(e);
}

extern "C" bs_status bs_sample(bs_sampler *s, const float *d_logits, size_t ld, uint32_t row0,
                               uint32_t rows, const uint32_t *d_prev, uint32_t n_prev, uint32_t *d_out,
                               void *stream) {
    if (!s) return BS_EINVAL;
    return sample_impl(s, next_seq(s->seq), d_logits, ld, row0, rows, d_prev, n_prev, d_out, stream);
}

// ---------------------------------------------------------------------------
// Vocabulary sharding, exact (a tensor-parallel LM head: rank g holds
// columns [col0, col0 + vocab) of all rows; the handle's vocab is the shard
// width).  The reference's normaliser is one sequential f32 sum over the
// whole row in index order; it is reproduced as a chain over the shards in
// rank order.  Per call, on every rank, with the collectives between the
// steps done by the caller (NCCL):
//   bs_vshard_stats   the statistics pass on the shard; per-row partials
//   (all-gather of the partials, [world][rows])
//   bs_vshard_main    row reduction against the global maximum and the lower
//                     shards' mass estimate; the main pass (items, candidates)
//   bs_vshard_walk    the walk of this shard's items from the running sum the
//                     previous rank ended with (rank 0: the empty sum)
//   (rank g receives rank g-1's exit sums and sends its own on; the last
//    rank's exit is the normaliser S, broadcast to all ranks)
//   bs_vshard_export  this shard's candidates with global ids
//   (all-gather of the candidates)
//   bs_vshard_draw    filters and the draw on the merged candidates, with the
//                     row's RNG state (the same on every rank)
// Exact only with a top-k bound: every kept token is among its shard's local
// top-k, which each shard's candidates contain.
// The peer-memory exchange of this handle (all null before bs_vshard_ipc_open).
static VsPeer vs_peer(const bs_sampler *s) {
    VsPeer pe{};
    if (s->d_peer_xchg) {
        pe.xs = s->d_peer_xchg;
        pe.own = s->d_xchg;
        pe.world = s->p2p_world;
        pe.rank = s->p2p_rank;
        pe.batch = s->batch;
    }
    return pe;
}

static bool vs_supported(const bs_sampler *s) {
    const bs_config &c = s->cfg;
    return c.temperature > 0.0f && c.top_k > 0 && c.top_k <= (uint32_t)KSEL_MAX &&
           typical_mode(c.typical_p, c.top_k, s->vocab, c.top_p, c.min_p) == TYP_OFF;
}

extern "C" bs_status bs_vshard_stats(bs_sampler *s, const float *d_shard, size_t ld, uint32_t col0, uint32_t rows,
                                     const uint32_t *d_prev, uint32_t n_prev, bs_vshard_part *d_part, void *stream) {
    if (!s || !d_shard || ld < s->vocab || rows == 0 || rows > s->batch) return BS_EINVAL;
    if (!d_part && !s->d_peer_xchg) return BS_EINVAL;     // (NULL: the partials go to the peers' words)
    if (s->d_peer_xchg && rows != s->batch) return BS_EINVAL;   // (the exchange words are laid out by the batch)
    if (!vs_supported(s)) return BS_ENOTSUP;
    cudaStream_t st = (cudaStream_t)stream;
    bool pen = false;
    uint32_t win = 0;
    make_params(s, next_seq(s->seq), d_shard, ld, 0, rows, d_prev, n_prev, nullptr, s->vs_A, s->vs_B, pen, win);
    s->vs_rows = rows;
    s->vs_ready = true;
    if (s->d_peer_xchg) k_vs_epoch<<<1, 1, 0, st>>>(reinterpret_cast<uint32_t *>(s->d_xchg + 2 * (size_t)s->batch));
    if (pen)
        k0_penalty<<<rows, 256, 0, st>>>(d_prev, n_prev, win, s->vocab, col0, 0u, s->ntiles_total, s->d_penbm);
    k1_stats<<<dim3(s->nseg, rows), K12_THREADS, 0, st>>>(s->vs_A);
    VsPeer pe = vs_peer(s);
    if (d_part) pe.xs = nullptr;   // (partials to the caller's buffer, host collectives)
    k_vs_partials<<<(rows + 7) / 8, 256, 0, st>>>(s->d_sstat, s->nseg, rows, s->vs_A.c2,
                                                   reinterpret_cast<VsPart *>(d_part), pe);
    return cuda_status(cudaGetLastError());
}

extern "C" bs_status bs_vshard_main(bs_sampler *s, const bs_vshard_part *d_parts, uint32_t world, uint32_t rank,
                                    void *stream) {
    if (!s || world == 0 || world > 64 || rank >= world) return BS_EINVAL;
    if (!s->vs_ready || (!d_parts && !s->d_peer_xchg)) return BS_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    K12Params A = s->vs_A;
    A.vs_parts = reinterpret_cast<const VsPart *>(d_parts);
    if (!d_parts) {   // the partials in this rank's exchange words, each waited for by its tag
        const VsLayout L(s->batch, s->p2p_world);
        A.vs_parts = reinterpret_cast<const VsPart *>(s->d_xchg + L.parts);
        A.vs_ptag = s->d_xchg + L.ptag;
        A.vs_epoch = reinterpret_cast<const uint32_t *>(s->d_xchg + 2 * (size_t)s->batch);
    }
    A.vs_world = world;
    A.vs_rank = rank;
    k1_rows<<<s->vs_rows, K12_THREADS, 0, st>>>(A);
    cudaError_t e = launch_dependent(k2_main<TERM_P>, dim3(s->nseg * s->vs_rows), dim3(K12_THREADS), 0, st, A);
    if (e == cudaSuccess) e = cudaGetLastError();
    return cuda_status(e);
}

extern "C" bs_status bs_vshard_walk(bs_sampler *s, const float *d_entry, float *d_exit, void *stream) {
    if (!s || !d_exit || !s->vs_ready) return BS_EINVAL;
    KBParams B = s->vs_B;
    B.vs_mode = VS_WALK;
    B.vs_entry = d_entry;
    B.vs_exit = d_exit;
    kernel_b<TERM_P><<<s->vs_rows, KB_THREADS, s->smem_b, (cudaStream_t)stream>>>(B);
    return cuda_status(cudaGetLastError());
}

// Peer-memory chain.  Every rank exports the IPC handle of its exchange words
// (bs_vshard_ipc_handle), the caller all-gathers the handles (host memory,
// world x 64 bytes), and every rank opens the others' (bs_vshard_ipc_open).
// Then bs_vshard_chain replaces bs_vshard_walk and the exit/S exchange, and
// bs_vshard_draw takes d_S = NULL (S arrives in the exchange words).
extern "C" bs_status bs_vshard_ipc_handle(bs_sampler *s, uint32_t world, void *h_handle) {
    if (!s || !h_handle || world < 2 || world > 64 || (s->d_xchg && world != s->xchg_world)) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    if (!s->d_xchg) {   // the exchange words (VsLayout), zeroed: no word carries a tag yet
        const size_t bytes = VsLayout(s->batch, world).words * sizeof(unsigned long long);
        s->xchg_world = world;
        if (cudaMalloc(&s->d_xchg, bytes) != cudaSuccess) return BS_ENOMEM;
        BS_CUDA(cudaMemset(s->d_xchg, 0, bytes));
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "an IPC handle is 64 bytes");
    cudaIpcMemHandle_t h;
    BS_CUDA(cudaIpcGetMemHandle(&h, s->d_xchg));
    memcpy(h_handle, &h, sizeof(h));
    return BS_OK;
}

extern "C" bs_status bs_vshard_ipc_open(bs_sampler *s, uint32_t world, uint32_t rank, const void *h_handles) {
    if (!s || !h_handles || world < 2 || world > 64 || rank >= world || !s->d_xchg || s->d_peer_xchg ||
        world != s->xchg_world)
        return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    s->p2p_world = world;
    s->p2p_rank = rank;
    for (uint32_t g = 0; g < world; g++) {
        if (g == rank) {
            s->peer_xchg[g] = s->d_xchg;
            continue;
        }
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const unsigned char *>(h_handles) + 64 * (size_t)g, sizeof(h));
        void *ptr = nullptr;
        BS_CUDA(cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess));
        s->peer_xchg[g] = static_cast<unsigned long long *>(ptr);
    }
    if (cudaMalloc(&s->d_peer_xchg, world * sizeof(unsigned long long *)) != cudaSuccess) return BS_ENOMEM;
    BS_CUDA(cudaMemcpy(s->d_peer_xchg, s->peer_xchg, world * sizeof(unsigned long long *), cudaMemcpyHostToDevice));
    return BS_OK;
}

// The chain of walks through peer memory: rank g's walk of a row waits for
// rank g-1's exit word of that row and stores its own into rank g+1's; the
// last rank stores the row's S into every rank's words.  Rows pipeline across
// the ranks; no collective.  Every rank must make the same calls (the words
// are tagged with the call's sequence number).
extern "C" bs_status bs_vshard_chain(bs_sampler *s, void *stream) {
    if (!s || !s->vs_ready || !s->d_peer_xchg) return BS_EINVAL;
    KBParams B = s->vs_B;
    B.vs_mode = VS_WALK;
    B.vs_entry = nullptr;
    B.vs_exit = nullptr;
    B.vs_p2p = 1;
    B.vs_world = s->p2p_world;
    B.vs_rank = s->p2p_rank;
    B.vs_soff = s->batch;
    B.vs_in = s->d_xchg;
    B.vs_epoch = reinterpret_cast<const uint32_t *>(s->d_xchg + 2 * (size_t)s->batch);
    B.vs_next = s->p2p_rank + 1 < s->p2p_world ? s->peer_xchg[s->p2p_rank + 1] : nullptr;
    B.vs_xs = s->d_peer_xchg;
    kernel_b<TERM_P><<<s->vs_rows, KB_THREADS, s->smem_b, (cudaStream_t)stream>>>(B);
    return cuda_status(cudaGetLastError());
}

extern "C" bs_status bs_vshard_export(bs_sampler *s, uint32_t col0, bs_vshard_cand *d_cand, uint32_t *d_count,
                                      void *stream) {
    if (!s || !s->vs_ready) return BS_EINVAL;
    if ((!d_cand || !d_count) && !s->d_peer_xchg) return BS_EINVAL;   // (NULL: to the peers' words)
    VsPeer pe = vs_peer(s);
    if (d_cand) pe.xs = nullptr;
    k_vs_export<<<s->vs_rows, 256, 0, (cudaStream_t)stream>>>(s->d_hdr, s->d_cand, s->cand_stride, col0,
                                                               reinterpret_cast<Candidate *>(d_cand), d_count, pe);
    return cuda_status(cudaGetLastError());
}

extern "C" bs_status bs_vshard_draw(bs_sampler *s, const bs_vshard_cand *d_cand_all, const uint32_t *d_count_all,
                                    uint32_t world, const float *d_S, uint32_t *d_out, void *stream) {
    if (!s || !d_out || world == 0 || world > 64 || !s->vs_ready) return BS_EINVAL;
    // (NULL candidates / S: from this rank's exchange words)
    if ((!d_cand_all || !d_count_all || !d_S) && !s->d_peer_xchg) return BS_EINVAL;
    cudaStream_t st = (cudaStream_t)stream;
    VsPeer pe = vs_peer(s);
    if (d_cand_all) pe.xs = nullptr;
    k_vs_merge<<<s->vs_rows, 256, 0, st>>>(reinterpret_cast<const Candidate *>(d_cand_all), d_count_all, world,
                                          s->vs_rows, s->d_hdr, s->d_cand, s->cand_stride, pe, s->vs_B.seq,
                                          s->d_kerr);
    KBParams B = s->vs_B;
    B.vs_mode = VS_DRAW;
    B.vs_S = d_S;
    if (!d_S) {
        B.vs_p2p = 1;
        B.vs_soff = s->batch;
        B.vs_in = s->d_xchg;
        B.vs_epoch = reinterpret_cast<const uint32_t *>(s->d_xchg + 2 * (size_t)s->batch);
    }
    B.out = d_out;
    kernel_b<TERM_P><<<s->vs_rows, KB_THREADS, s->smem_b, st>>>(B);
    return cuda_status(cudaGetLastError());
}

extern "C" bs_status bs_sample_host(bs_sampler *s, const float *h_logits, size_t ld, uint32_t row0,
                                    uint32_t rows, const uint32_t *h_prev, uint32_t n_prev, uint32_t *h_out) {
    if (!s || !h_logits || !h_out || ld < s->vocab) return BS_EINVAL;
    if (row0 > s->batch || rows > s->batch - row0) return BS_EINVAL;
    if (rows == 0) return BS_OK;
    BS_CUDA(cudaSetDevice(s->device));
    const size_t nf = (size_t)rows * ld;
    if (nf > s->stage_floats) {
        cudaFree(s->d_logits_stage);
        s->d_logits_stage = nullptr;
        if (cudaMalloc(&s->d_logits_stage, nf * sizeof(float)) != cudaSuccess) return BS_ENOMEM;
        s->stage_floats = nf;
    }
    if (!s->d_out_stage) {
        if (cudaMalloc(&s->d_out_stage, (size_t)s->batch * sizeof(uint32_t)) != cudaSuccess) return BS_ENOMEM;
    }
    const uint32_t *dp = nullptr;
    if (h_prev && n_prev > 0) {
        const size_t np = (size_t)rows * n_prev;
        if (np > s->stage_prev) {
            cudaFree(s->d_prev_stage);
            s->d_prev_stage = nullptr;
            if (cudaMalloc(&s->d_prev_stage, np * sizeof(uint32_t)) != cudaSuccess) return BS_ENOMEM;
            s->stage_prev = np;
        }
        BS_CUDA(cudaMemcpyAsync(s->d_prev_stage, h_prev, np * sizeof(uint32_t), cudaMemcpyHostToDevice,
                                s->stream));
        dp = s->d_prev_stage;
    }
    BS_CUDA(cudaMemcpyAsync(s->d_logits_stage, h_logits, nf * sizeof(float), cudaMemcpyHostToDevice, s->stream));
    bs_status r = bs_sample(s, s->d_logits_stage, ld, row0, rows, dp, dp ? n_prev : 0, s->d_out_stage, s->stream);
    if (r != BS_OK) return r;
    BS_CUDA(cudaMemcpyAsync(h_out, s->d_out_stage, rows * sizeof(uint32_t), cudaMemcpyDeviceToHost, s->stream));
    BS_CUDA(cudaStreamSynchronize(s->stream));
    for (uint32_t i = 0; i < rows; i++)
        if (h_out[i] == 0xFFFFFFFFu) return bs_last_device_status(s);
    return BS_OK;
}

// Test and tuning hooks: 1 selects the task-queue persistent kernel, 2 the
// read-once persistent kernel, 0 the separate kernels (same results); the
// persistent kernels' grids on a device.
extern "C" bs_status bs_debug_set_fused(bs_sampler *s, uint32_t fused) {
    if (!s) return BS_EINVAL;
    s->fused = fused;
    return BS_OK;
}
// Test hook: 1 sends every row through the full-vocabulary retry (the path
// of rows whose candidates or typical-p band fail their cover check).
extern "C" bs_status bs_debug_set_force_full(bs_sampler *s, uint32_t on) {
    if (!s) return BS_EINVAL;
    s->force_full = on;
    return BS_OK;
}
extern "C" int bs_debug_fused_ctas(int device) {
    int ctas = 0;
    return fused_grid(device, &ctas) == cudaSuccess ? ctas : -1;
}
extern "C" int bs_debug_resident_ctas(int device) {
    int ctas = 0;
    return fused_grid(device, &ctas, 2u) == cudaSuccess ? ctas : -1;
}

extern "C" bs_status bs_get_rng_state(bs_sampler *s, uint64_t *h_state) {
    if (!s || !h_state) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    BS_CUDA(cudaDeviceSynchronize());
    BS_CUDA(cudaMemcpy(h_state, s->d_rng, (size_t)s->batch * 4 * sizeof(uint64_t), cudaMemcpyDeviceToHost));
    return BS_OK;
}

extern "C" bs_status bs_set_rng_state(bs_sampler *s, const uint64_t *h_state) {
    if (!s || !h_state) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    BS_CUDA(cudaDeviceSynchronize());
    BS_CUDA(cudaMemcpy(s->d_rng, h_state, (size_t)s->batch * 4 * sizeof(uint64_t), cudaMemcpyHostToDevice));
    return BS_OK;
}

extern "C" bs_status bs_seed_state(uint64_t seed, uint64_t *h_state4) {
    if (!h_state4) return BS_EINVAL;
    rng_seed(h_state4, seed != 0 ? seed : 0xDEADBEEFULL);
    return BS_OK;
}

extern "C" bs_status bs_last_device_status(bs_sampler *s) {
    if (!s) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    BS_CUDA(cudaDeviceSynchronize());
    RowTrace *h = new (std::nothrow) RowTrace[s->batch];
    if (!h) return BS_ENOMEM;
    cudaError_t e = cudaMemcpy(h, s->d_trace, (size_t)s->batch * sizeof(RowTrace), cudaMemcpyDeviceToHost);
    bs_status r = BS_OK;
    if (e != cudaSuccess) r = BS_ECUDA;
    for (uint32_t i = 0; r == BS_OK && i < s->batch; i++) {
        if (h[i].status == ROW_ENOTSUP) r = BS_ENOTSUP;
        else if (h[i].status == ROW_ETIMEOUT) r = BS_ETIMEOUT;
        else if (h[i].status != ROW_OK) r = BS_EINTERNAL;
    }
    delete[] h;
    return r;
}

// Self-check of the main loop's certificate (cert_eps): random logits placed
// so that p / u_lo falls near the rounding points; every certified count must
// equal the exact one (elem_comp of the restated expf's p).  out[0] counts
// violations, out[1] certified samples, out[2] samples.
__global__ void cert_check_kernel(uint32_t n, uint64_t seed, unsigned long long *out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t h = seed ^ (0x9E3779B97F4A7C15ull * (i + 1));
    auto nxt = [&]() {
        h += 0x9E3779B97F4A7C15ull;
        uint64_t z = h;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    auto unif = [&]() { return (float)((nxt() >> 40) * 0x1p-24); };
    const int lo = -100 + (int)(nxt() % 160);   // binades -100 .. 59
    const float K = (float)(23 - lo);
    const float T = 0.05f + 5.0f * unif();
    const float M = -50.0f + 100.0f * unif();
    const float c2 = (float)(1.4426950408889634 / (double)T);
    // target y: near k + 1/2 (half of the samples) or anywhere, 2^-3 .. 2^17.5
    const double ly = -3.0 + 20.5 * (double)unif();
    double y0 = exp2(ly);
    if (nxt() & 1) y0 = floor(y0) + 0.5 + (unif() - 0.5) * 2e-4 * y0;
    const double x2 = log2(y0) - (double)K;   // <= 0 needs y0 <= 2^K
    if (x2 > 0.0) return;
    const float v = __fadd_rn(M, (float)(x2 * (double)T / 1.4426950408889634));
    const float d = __fsub_rn(v, M);
    const float y = ex2_approx(fminf(fmaf(d, c2, K), 17.5f));
    const float e = fmaxf(cert_eps(K), 0x1p-17f);
    const uint32_t r1 = __float_as_uint(fmaf(y, 1.0f + e, 12582912.0f));
    const uint32_t r2 = __float_as_uint(fmaf(y, 1.0f - e, 12582912.0f));
    atomicAdd(&out[2], 1ull);
    if (r1 != r2) return;
    atomicAdd(&out[1], 1ull);
    const Comp ex = elem_comp(prob_unnorm(v, M, T), lo);
    if (ex.q0 != ex.q1 || ex.q0 != r1 - 0x4B400000u) atomicAdd(&out[0], 1ull);
}

// The same for the entropy terms (cert_eps_h): the certified count of
// y = min(ex2.approx(min(z + K, 40)) (-z ln2), 2^17.5), z = fma(d, c2, -log2 S),
// against elem_comp of the exact term fl(P * -logf(P)), P = fl(p / S).
__global__ void cert_check_h_kernel(uint32_t n, uint64_t seed, unsigned long long *out) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    uint64_t h = seed ^ (0xD1B54A32D192ED03ull * (i + 1));
    auto nxt = [&]() {
        h += 0x9E3779B97F4A7C15ull;
        uint64_t z = h;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        return z ^ (z >> 31);
    };
    auto unif = [&]() { return (double)(nxt() >> 11) * 0x1p-53; };
    const int lo = -60 + (int)(nxt() % 70);   // binades -60 .. 9
    const float K = (float)(23 - lo);
    const float T = (float)(0.05 + 5.0 * unif());
    const float M = (float)(-50.0 + 100.0 * unif());
    const float S = (float)exp2(10.0 * unif());   // 1 .. 1024
    const float c2 = (float)(1.4426950408889634 / (double)T);
    const float l2S = (float)(log((double)S) * 1.4426950408889634);
    // target y = P (-ln P) / u_lo: near k + 1/2 (half of the samples) or anywhere
    double ly = -3.0 + 20.0 * unif();
    double y0 = exp2(ly);
    if (nxt() & 1) y0 = floor(y0) + 0.5 + (unif() - 0.5) * 2e-4 * y0;
    // solve 2^(z + K) (-z ln2) = y0 for z < -1/16 (Newton on the branch below
    // the maximum at z = -1/ln2)
    double z = -2.0 - 30.0 * unif();
    for (int it = 0; it < 60; it++) {
        const double f = exp2(z + K) * (-z * 0.6931471805599453) - y0;
        const double fp = exp2(z + K) * 0.6931471805599453 * (-z * 0.6931471805599453 - 1.0);
        if (fp == 0.0) break;
        const double zn = z - f / fp;
        z = fmin(zn, -1.4426950408889634 - 1e-3);
    }
    if (!(z < -0.0625) || z + l2S > 0.0) return;
    const double x2 = z + (double)l2S;
    const float v = __fadd_rn(M, (float)(x2 * (double)T / 1.4426950408889634));
    const float d = __fsub_rn(v, M);
    const float zz = fmaf(d, c2, -l2S);
    if (!(zz < -0.0625f)) return;
    const float w = fminf(zz * -0.6931472f, 1e30f);
    const float y = fminf(ex2_approx(fminf(zz + K, 40.0f)) * w, 185363.8f);
    const float e = fmaxf(cert_eps_h(K, fmaxf(-zz, 0.0625f), fabsf(l2S)), 0x1p-17f);
    const uint32_t r1 = __float_as_uint(fmaf(y, 1.0f + e, 12582912.0f));
    const uint32_t r2 = __float_as_uint(fmaf(y, 1.0f - e, 12582912.0f));
    atomicAdd(&out[2], 1ull);
    if (r1 != r2) return;
    atomicAdd(&out[1], 1ull);
    const Comp ex = elem_comp(entropy_term(v, M, T, S), lo);
    if (ex.q0 != ex.q1 || ex.q0 != r1 - 0x4B400000u) atomicAdd(&out[0], 1ull);
}

extern "C" bs_status bs_debug_cert_check(uint32_t n, uint64_t seed, unsigned long long *h_out) {
    if (!h_out || n == 0) return BS_EINVAL;
    const bool entropy = (seed >> 63) != 0;   // the entropy terms' certificate
    unsigned long long *d = nullptr;
    BS_CUDA(cudaMalloc(&d, 3 * sizeof(unsigned long long)));
    cudaError_t e = cudaMemset(d, 0, 3 * sizeof(unsigned long long));
    if (e == cudaSuccess) {
        if (entropy) {
            cert_check_h_kernel<<<(n + 255) / 256, 256>>>(n, seed, d);
        } else {
            cert_check_kernel<<<(n + 255) / 256, 256>>>(n, seed, d);
        }
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(h_out, d, 3 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    return cuda_status(e);
}

// The crossing search on every stretch length 1..max_ntl and crossing
// position; h_out[0] = failures, h_out[1] = cases.  Synchronous.
extern "C" bs_status bs_debug_crossing_check(uint32_t max_ntl, unsigned long long *h_out) {
    if (!h_out || max_ntl == 0 || max_ntl > 4096) return BS_EINVAL;
    WTile *scratch = nullptr;
    unsigned long long *d = nullptr;
    BS_CUDA(cudaMalloc(&scratch, (size_t)max_ntl * max_ntl * sizeof(WTile)));
    cudaError_t e = cudaMalloc(&d, 2 * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMemset(d, 0, 2 * sizeof(unsigned long long));
    if (e == cudaSuccess) {
        crossing_check_kernel<<<max_ntl, 32>>>(scratch, max_ntl, d);
        e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaMemcpy(h_out, d, 2 * sizeof(unsigned long long), cudaMemcpyDeviceToHost);
    cudaFree(d);
    cudaFree(scratch);
    return cuda_status(e);
}

// Diagnostics for the test harness: per-row RowTrace of the last call
// (S, kept mass, draw, path, flags).  Synchronous.
extern "C" bs_status bs_debug_row_traces(bs_sampler *s, void *h_traces, size_t bytes) {
    if (!s || !h_traces || bytes < (size_t)s->batch * sizeof(RowTrace)) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    BS_CUDA(cudaDeviceSynchronize());
    BS_CUDA(cudaMemcpy(h_traces, s->d_trace, (size_t)s->batch * sizeof(RowTrace), cudaMemcpyDeviceToHost));
    return BS_OK;
}

extern "C" bs_status bs_profile_enable(bs_sampler *s, uint32_t max_calls) {
    if (!s) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    for (uint32_t i = 0; s->prof_ev && i < 4 * s->prof_cap; i++) cudaEventDestroy(s->prof_ev[i]);
    delete[] s->prof_ev;
    s->prof_ev = nullptr;
    s->prof_cap = s->prof_n = 0;
    if (max_calls == 0) return BS_OK;
    s->prof_ev = new (std::nothrow) cudaEvent_t[4 * (size_t)max_calls];
    if (!s->prof_ev) return BS_ENOMEM;
    for (uint32_t i = 0; i < 4 * max_calls; i++) BS_CUDA(cudaEventCreate(&s->prof_ev[i]));
    s->prof_cap = max_calls;
    return BS_OK;
}

extern "C" bs_status bs_profile_read(bs_sampler *s, float *ms, uint32_t cap, uint32_t *n_calls) {
    if (!s || !ms || !n_calls) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    const uint32_t n = s->prof_n < cap ? s->prof_n : cap;
    for (uint32_t i = 0; i < n; i++) {
        BS_CUDA(cudaEventSynchronize(s->prof_ev[4 * i + 3]));
        for (int j = 0; j < 3; j++)
            BS_CUDA(cudaEventElapsedTime(&ms[3 * i + j], s->prof_ev[4 * i + j], s->prof_ev[4 * i + j + 1]));
    }
    *n_calls = n;
    s->prof_n = 0;
    return BS_OK;
}

// ---------------------------------------------------------------------------
// bs_sample_static: the same three passes with every scratch buffer carved
// from one fixed static device array instead of a handle's allocations.  The
// caller owns the RNG state (a device buffer of rows x 4 u64).
constexpr size_t r256(size_t b) { return (b + 255) & ~(size_t)255; }
constexpr int STATIC_NBUF = 15;   // the buffers of a handle, in the order below
struct StaticSizes {
    size_t b[STATIC_NBUF];
};
constexpr StaticSizes static_sizes(uint32_t rows, uint32_t vocab) {
    const size_t nt = (vocab + TILE - 1) / TILE, cs = (vocab + 31u) & ~31u;
    return StaticSizes{{r256(rows * sizeof(RowHdr)), r256(rows * nt * sizeof(TileStat)),
                        r256(rows * MAX_SEG * sizeof(SegStat)), r256(rows * nt * sizeof(uint32_t)),
                        r256(rows * MAX_SEG * KH_BINS * sizeof(float)), r256(rows * sizeof(RowInfo)), r256(rows * nt * sizeof(Item)), r256(rows * nt * sizeof(WTile)),
                        r256(rows * WC_CAP * TILE * sizeof(float)), r256(rows * cs * sizeof(Candidate)),
                        r256(rows * 2 * cs * sizeof(unsigned long long)), r256(rows * sizeof(RowTrace)),
                        r256(sizeof(uint32_t)), r256((4 + rows) * sizeof(uint32_t)),
                        r256(rows * sizeof(unsigned long long))}};
}
constexpr size_t static_total(uint32_t rows, uint32_t vocab) {
    const StaticSizes s = static_sizes(rows, vocab);
    size_t t = 0;
    for (int i = 0; i < STATIC_NBUF; i++) t += s.b[i];
    return t;
}
// every buffer size grows with rows and vocab, so any call within the limits
// fits in the array sized for the limits
constexpr size_t STATIC_BYTES = static_total(BS_STATIC_MAX_ROWS, BS_STATIC_MAX_VOCAB);
static __device__ __align__(256) unsigned char g_static_scratch[STATIC_BYTES];

static unsigned char *g_static_base[MAX_DEVICES];
static uint32_t g_static_seq[MAX_DEVICES];   // sequence numbers of the static calls, per device
static std::mutex g_static_mu;

// Address of this device's copy of the static scratch, resolved once per
// device (with the kernel attributes set there), and the call's sequence
// number for the error word in that scratch.
static cudaError_t static_scratch_base(int dev, unsigned char **base, uint32_t *seq) {
    if (dev < 0 || dev >= MAX_DEVICES) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_static_mu);
    if (!g_static_base[dev]) {
        void *p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_static_scratch);
        if (e != cudaSuccess) return e;
        e = ensure_kernel_attrs(dev);
        if (e != cudaSuccess) return e;
        g_static_base[dev] = static_cast<unsigned char *>(p);
    }
    *base = g_static_base[dev];
    *seq = next_seq(g_static_seq[dev]);
    return cudaSuccess;
}

extern "C" bs_status bs_sample_static(const bs_config *cfg, uint64_t *d_rng, const float *d_logits, size_t ld,
                                      uint32_t rows, uint32_t vocab, const uint32_t *d_prev, uint32_t n_prev,
                                      uint32_t *d_out, void *stream) {
    if (!cfg || !d_rng || !d_logits || !d_out || vocab == 0 || ld < vocab) return BS_EINVAL;
    if (rows > BS_STATIC_MAX_ROWS || vocab > BS_STATIC_MAX_VOCAB) {
        fprintf(stderr,
                "b200_sampler: bs_sample_static: %u rows of %u logits exceed the static scratch "
                "(at most %u rows of at most %u logits); use a handle (bs_create)\n",
                rows, vocab, (unsigned)BS_STATIC_MAX_ROWS, (unsigned)BS_STATIC_MAX_VOCAB);
        return BS_EINVAL;
    }
    if (rows == 0) return BS_OK;
    if (cfg->temperature <= 0.0f) return bs_argmax(d_logits, ld, rows, vocab, d_out, stream);   // no prologue here
    int dev = 0;
    BS_CUDA(cudaGetDevice(&dev));
    unsigned char *base = nullptr;
    uint32_t seq = 0;
    const cudaError_t e = static_scratch_base(dev, &base, &seq);
    if (e != cudaSuccess) {
        fprintf(stderr, "b200_sampler: bs_sample_static: static scratch set-up failed: %s\n", cudaGetErrorString(e));
        return BS_ECUDA;
    }
    // a handle on the host stack whose buffers point into the static scratch
    bs_sampler s;
    memset(&s, 0, sizeof(s));
    s.cfg = *cfg;
    s.batch = rows;
    s.vocab = vocab;
    s.device = dev;
    s.ntiles_total = (vocab + TILE - 1) / TILE;
    s.nseg = (s.ntiles_total + SEG_TILES - 1) / SEG_TILES;
    s.smem_b = KB_SMEM;
    s.cand_stride = (vocab + 31u) & ~31u;
    s.d_rng = d_rng;
    const StaticSizes sz = static_sizes(rows, vocab);
    void *ptr[STATIC_NBUF];
    size_t off = 0;
    for (int i = 0; i < STATIC_NBUF; i++) {
        ptr[i] = base + off;
        off += sz.b[i];
    }
    s.d_hdr = static_cast<RowHdr *>(ptr[0]);
    s.d_tstat = static_cast<TileStat *>(ptr[1]);
    s.d_sstat = static_cast<SegStat *>(ptr[2]);
    s.d_penbm = static_cast<uint32_t *>(ptr[3]);
    s.d_mhist = static_cast<float *>(ptr[4]);
    s.d_rinfo = static_cast<RowInfo *>(ptr[5]);
    s.d_items = static_cast<Item *>(ptr[6]);
    s.d_wpre = static_cast<WTile *>(ptr[7]);
    s.d_wc = static_cast<float *>(ptr[8]);
    s.d_cand = static_cast<Candidate *>(ptr[9]);
    s.d_ctmp = static_cast<unsigned long long *>(ptr[10]);
    s.d_trace = static_cast<RowTrace *>(ptr[11]);
    s.d_kerr = static_cast<uint32_t *>(ptr[12]);
    s.d_fctl = static_cast<uint32_t *>(ptr[13]);        // zeroed by each call before use
    s.d_ready = static_cast<unsigned long long *>(ptr[14]);   // earlier calls' sequence numbers only
    // nothing in the scratch has to start at zero: every buffer a call reads
    // is written earlier in the same call, and the error word holds the
    // sequence number of a failed call (zero at load), never this call's
    // unless this call's own wait gave up
    return sample_impl(&s, seq, d_logits, ld, 0, rows, d_prev, n_prev, d_out, stream);
}
