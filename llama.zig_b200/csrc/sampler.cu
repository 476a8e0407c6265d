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
//   Kernel A (one thread-block cluster per row, one CTA per row segment, the
//   segment resident in shared memory; HBM is read once):
//     1. load the segment, row max M via DSMEM;
//     2. approximate tile sums (ex2.approx) -> cluster-wide prefix P_raw(t);
//     3. rounding-aware tile sums: each p rounded to the grid of the binade
//        the running sum is expected to be in -> prefix P(t), which tracks the
//        reference's running sum to ~1e-6;
//     4. every 32-element tile gets the candidate binades [lo, hi] of the
//        running sum over it; tiles with lo == hi are SIMPLE; inside one binade
//        e the f32 add s + p is exactly s + u_e * round_e(p) (u_e the ulp of
//        binade e, round-half-even whose tie direction depends on the parity
//        of s), so a tile reduces to two integer counts (entry parity 0/1);
//        WINDOW (hi = lo+1) and COMPLEX tiles keep their exact p for an
//        element-wise add;
//     5. consecutive SIMPLE tiles of one binade are composed into one item.
//   Kernel B (one CTA per row): a single warp walks the ~30-60 items with the
//   exact state (binade, integer mantissa): an item applies in O(1) when the
//   state is in its binade and does not leave it; otherwise the tile is added
//   element by element with the same f32 adds as the reference.  The result
//   is the reference's `sum`, bit for bit, for every input (a speculation miss
//   only costs time).  Meanwhile the other warps sort the candidate tokens;
//   then exact probs, the filters, the kept mass and the draw follow the
//   reference's sequential f32 order on the (small) candidate prefix.
//
// Candidates: Kernel A keeps only tokens above a floor that provably contains
// the kept prefix and the token that ends it (top-k: the k-th largest tile
// maximum; top-p: a mass bound; min-p: its threshold); Kernel B verifies the
// cover and reports BS_ENOTSUP if it ever fails.
#include <cooperative_groups.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>

#include "../../include/b200_sampler.h"
#include "bs_math.cuh"
#include "sampler_kernels.cuh"

namespace cg = cooperative_groups;

namespace bs {

constexpr uint32_t QSAT = 1u << 30;      // saturation of grid counts
constexpr uint32_t QLIM = 1u << 24;      // mantissa range of one binade
constexpr double DELTA = 1e-5;           // speculation window (relative)
constexpr float NEG_INF = -__builtin_huge_valf();

// ---------------------------------------------------------------------------
// Grid-count composites.  Within binade e (ulp u_e = 2^(e-23); e = -126 also
// covers the subnormals) the state is s = m * u_e, m < 2^24.  Adding p gives
// m + round_e(p); a tie goes to the even result, so its count depends on the
// parity of m.  A composite stores the total count for entry parity 0 and 1.
struct Comp {
    uint32_t q0, q1;
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

// ---------------------------------------------------------------------------
// sampleArgmax (sampler.zig:31-41): one CTA per row.
__global__ void __launch_bounds__(512) argmax_kernel(const float *__restrict__ logits, size_t ld,
                                                     uint32_t vocab, uint32_t *__restrict__ out) {
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
            const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const float f = a[k] != a[k] ? NEG_INF : a[k];
                best = arg_better(best, ArgBest{f, 4 * i + k});
            }
        }
        done = n4 * 4;
    }
    for (uint32_t i = done + threadIdx.x; i < vocab; i += blockDim.x) {
        const float f = x[i];
        best = arg_better(best, ArgBest{f != f ? NEG_INF : f, i});
    }
    best = warp_arg(best);
    __shared__ ArgBest wb[16];
    if ((threadIdx.x & 31) == 0) wb[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        ArgBest b = wb[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); w++) b = arg_better(b, wb[w]);
        const float x0 = x[0];
        uint32_t r = b.i;
        if (x0 != x0 || b.i == 0xFFFFFFFFu) r = 0;  // leading NaN wins; all -inf -> 0
        out[row] = r;
    }
}

// ---------------------------------------------------------------------------
struct KAParams {
    const float *logits;
    size_t ld;
    const uint32_t *prev;     // rows x n_prev (device) or null
    uint32_t n_prev;
    uint32_t vocab;
    uint32_t row0;            // first handle row of this call
    float T;                  // temperature
    float c2;                 // log2(e) / T (approximate paths only)
    uint32_t top_k;
    float top_p;
    float min_p;
    uint32_t rep_window;
    float rep_penalty;
    uint32_t C;               // cluster size (segments per row)
    uint32_t seg_len;         // elements per segment (multiple of 32)
    uint32_t ntiles_seg;      // seg_len / 32
    uint32_t ntiles_total;    // ceil(vocab / 32)
    uint32_t ksort;           // power of two >= ntiles_seg (top-k tile-max sort)
    RowHdr *hdr;              // per handle row
    Item *items;              // per handle row: ntiles_total slots
    float *wcdata;            // per handle row: WC_CAP x 32
    Candidate *cand;          // per handle row: cand_stride
    uint32_t cand_stride;     // >= vocab: every token can be a candidate
};

struct XSlot {   // per-CTA values exchanged through distributed shared memory
    float pmax;
    float rmax;
    uint32_t rarg;
    uint32_t nan_any;
    double tot_raw;
    double tot2;
    uint32_t klen;
    uint32_t pad;
};

struct TileRec {
    int32_t lo;
    uint32_t cls;
    uint32_t aux;
    Comp qlo;
    Comp qhi;
};

__device__ __forceinline__ bool penalty_active(const KAParams &P) {
    return P.rep_penalty != 1.0f && P.n_prev > 0 && P.prev != nullptr && P.rep_window > 0;
}

// Block-wide exclusive scan of n (<= 2*KA_THREADS) doubles in place; returns total.
__device__ double block_exscan_d(double *a, uint32_t n, double *wtmp) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t i0 = 2 * tid, i1 = 2 * tid + 1;
    const double a0 = i0 < n ? a[i0] : 0.0;
    const double a1 = i1 < n ? a[i1] : 0.0;
    double v = a0 + a1, incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const double t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) wtmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        double w = lane < KA_WARPS ? wtmp[lane] : 0.0, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const double t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < KA_WARPS) wtmp[lane] = wi - w;  // exclusive warp offsets
        if (lane == KA_WARPS - 1) wtmp[KA_WARPS] = wi;
    }
    __syncthreads();
    const double ex = wtmp[warp] + incl - v;
    if (i0 < n) a[i0] = ex;
    if (i1 < n) a[i1] = ex + a0;
    const double total = wtmp[KA_WARPS];
    __syncthreads();
    return total;
}

// Block-wide exclusive scan of n (<= 2*KA_THREADS) uint32 flags; returns total.
__device__ uint32_t block_exscan_u(uint32_t *a, uint32_t n, uint32_t *wtmp) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t i0 = 2 * tid, i1 = 2 * tid + 1;
    const uint32_t a0 = i0 < n ? a[i0] : 0u;
    const uint32_t a1 = i1 < n ? a[i1] : 0u;
    uint32_t v = a0 + a1, incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    if (lane == 31) wtmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        uint32_t w = lane < KA_WARPS ? wtmp[lane] : 0u, wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const uint32_t t = __shfl_up_sync(0xffffffffu, wi, o);
            if (lane >= o) wi += t;
        }
        if (lane < KA_WARPS) wtmp[lane] = wi - w;
        if (lane == KA_WARPS - 1) wtmp[KA_WARPS] = wi;
    }
    __syncthreads();
    const uint32_t ex = wtmp[warp] + incl - v;
    if (i0 < n) a[i0] = ex;
    if (i1 < n) a[i1] = ex + a0;
    const uint32_t total = wtmp[KA_WARPS];
    __syncthreads();
    return total;
}

// Segmented inclusive scan of composites: head[i] starts a new segment.
// In: c[i], head[i] for i < n (n <= 2*KA_THREADS).  Out: c[i] = composite
// from the segment start to i.
struct SegComp {
    uint32_t f;
    Comp c;
};
__device__ __forceinline__ SegComp seg_then(SegComp a, SegComp b) {
    if (b.f) return b;
    return SegComp{a.f, comp_then(a.c, b.c)};
}
__device__ void block_segscan_comp(Comp *c, const uint32_t *head, uint32_t n, SegComp *wtmp) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t i0 = 2 * tid, i1 = 2 * tid + 1;
    SegComp s0{i0 < n ? head[i0] : 1u, i0 < n ? c[i0] : Comp{0, 0}};
    SegComp s1{i1 < n ? head[i1] : 1u, i1 < n ? c[i1] : Comp{0, 0}};
    SegComp v = seg_then(s0, s1);
    SegComp incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        SegComp t;
        t.f = __shfl_up_sync(0xffffffffu, incl.f, o);
        t.c.q0 = __shfl_up_sync(0xffffffffu, incl.c.q0, o);
        t.c.q1 = __shfl_up_sync(0xffffffffu, incl.c.q1, o);
        if (lane >= o) incl = seg_then(t, incl);
    }
    if (lane == 31) wtmp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
        SegComp w = lane < KA_WARPS ? wtmp[lane] : SegComp{0u, {0, 0}};
        SegComp wi = w;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            SegComp t;
            t.f = __shfl_up_sync(0xffffffffu, wi.f, o);
            t.c.q0 = __shfl_up_sync(0xffffffffu, wi.c.q0, o);
            t.c.q1 = __shfl_up_sync(0xffffffffu, wi.c.q1, o);
            if (lane >= o) wi = seg_then(t, wi);
        }
        __syncwarp();
        if (lane < KA_WARPS) wtmp[KA_WARPS + 1 + lane] = wi;  // inclusive over warps 0..lane
    }
    __syncthreads();
    // exclusive prefix for this thread = (warp carry) then (lanes before me)
    SegComp excl_lane;
    {
        SegComp t;
        t.f = __shfl_up_sync(0xffffffffu, incl.f, 1);
        t.c.q0 = __shfl_up_sync(0xffffffffu, incl.c.q0, 1);
        t.c.q1 = __shfl_up_sync(0xffffffffu, incl.c.q1, 1);
        excl_lane = lane > 0 ? t : SegComp{0u, {0, 0}};
    }
    SegComp carry = warp > 0 ? wtmp[KA_WARPS + 1 + warp - 1] : SegComp{0u, {0, 0}};
    SegComp pre = lane > 0 ? seg_then(carry, excl_lane) : carry;
    // element 0 then element 1
    SegComp r0 = seg_then(pre, s0);
    SegComp r1 = seg_then(r0, s1);
    __syncthreads();
    if (i0 < n) c[i0] = r0.c;
    if (i1 < n) c[i1] = r1.c;
    __syncthreads();
}

__global__ void __launch_bounds__(KA_THREADS, 2) kernel_a(KAParams P) {
    cg::cluster_group cluster = cg::this_cluster();
    const uint32_t rank = cluster.block_rank();
    const uint32_t row = blockIdx.y;
    const uint32_t hrow = P.row0 + row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const uint32_t V = P.vocab;
    const uint32_t NT = P.ntiles_seg;

    extern __shared__ __align__(16) unsigned char smem[];
    float *seg = reinterpret_cast<float *>(smem);
    double *tsum = reinterpret_cast<double *>(seg + P.seg_len);          // NT
    double *pref = tsum + NT;                                             // NT
    float *tmax = reinterpret_cast<float *>(pref + NT);                   // ksort
    TileRec *rec = reinterpret_cast<TileRec *>(tmax + P.ksort);           // NT
    uint32_t *uarr = reinterpret_cast<uint32_t *>(rec + NT);              // NT
    Comp *carr = reinterpret_cast<Comp *>(uarr + NT);                     // NT
    __shared__ XSlot xs;
    __shared__ double wtmp_d[KA_WARPS + 1];
    __shared__ uint32_t wtmp_u[KA_WARPS + 1];
    __shared__ SegComp wtmp_s[2 * KA_WARPS + 2];
    __shared__ ArgBest wbest[KA_WARPS];
    __shared__ float wmax[KA_WARPS];
    __shared__ uint32_t wnan[KA_WARPS];
    __shared__ float kth_sh;
    __shared__ float kgather[MAX_CLUSTER * KSEL_MAX];
    __shared__ float hist[HIST_BINS];
    __shared__ float ghist[HIST_BINS];

    RowHdr *hdr = P.hdr + hrow;
    const uint32_t seg0 = rank * P.seg_len;
    const uint32_t segn = seg0 < V ? min(P.seg_len, V - seg0) : 0u;
    const uint32_t tile0 = rank * NT;
    const float *src = P.logits + (size_t)row * P.ld + seg0;

    if (rank == 0 && tid == 0) {
        hdr->n_cand = 0;
        hdr->n_wc = 0;
        hdr->flags = 0;
        hdr->nseg = P.C;
    }

    // ---- phase 1: segment -> shared memory; raw argmax; penalised max -----
    ArgBest best{NEG_INF, 0xFFFFFFFFu};
    float lmax = NEG_INF;
    {
        uint32_t done = 0;
        if ((reinterpret_cast<uintptr_t>(src) & 15u) == 0) {
            const uint32_t n4 = segn / 4;
            const float4 *s4 = reinterpret_cast<const float4 *>(src);
            float4 *d4 = reinterpret_cast<float4 *>(seg);
            uint32_t i = tid;
            for (; i + 3 * KA_THREADS < n4; i += 4 * KA_THREADS) {
                float4 v[4];
#pragma unroll
                for (int u = 0; u < 4; u++) v[u] = ldg_stream(s4 + i + u * KA_THREADS);
#pragma unroll
                for (int u = 0; u < 4; u++) {
                    d4[i + u * KA_THREADS] = v[u];
                    const float a[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                    for (int k = 0; k < 4; k++) {
                        lmax = fmaxf(lmax, a[k]);
                        best = arg_better(best, ArgBest{a[k] != a[k] ? NEG_INF : a[k],
                                                        seg0 + 4 * (i + u * KA_THREADS) + k});
                    }
                }
            }
            for (; i < n4; i += KA_THREADS) {
                const float4 v = ldg_stream(s4 + i);
                d4[i] = v;
                const float a[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    lmax = fmaxf(lmax, a[k]);
                    best = arg_better(best, ArgBest{a[k] != a[k] ? NEG_INF : a[k], seg0 + 4 * i + k});
                }
            }
            done = n4 * 4;
        }
        for (uint32_t i = done + tid; i < segn; i += KA_THREADS) {
            const float a = src[i];
            seg[i] = a;
            lmax = fmaxf(lmax, a);
            best = arg_better(best, ArgBest{a != a ? NEG_INF : a, seg0 + i});
        }
        for (uint32_t i = segn + tid; i < NT * TILE; i += KA_THREADS) seg[i] = NEG_INF;
    }
    if (rank == 0 && tid == 0) xs.nan_any = (segn > 0 && src[0] != src[0]) ? 1u : 0u;  // leading NaN
    // repetition penalty (sampler.zig:54-75): each distinct id of the last
    // `window` previous tokens, once.
    const bool pen = penalty_active(P);
    if (pen) {
        __syncthreads();
        const uint32_t win = min(P.n_prev, P.rep_window);
        const uint32_t start = P.n_prev - win;
        const uint32_t *pv = P.prev + (size_t)row * P.n_prev + start;
        for (uint32_t j = tid; j < win; j += KA_THREADS) {
            const uint32_t id = pv[j];
            bool first = true;
            for (uint32_t jj = 0; jj < j; jj++)
                if (pv[jj] == id) { first = false; break; }
            if (first && id >= seg0 && id < seg0 + segn) {
                const float v = seg[id - seg0];
                seg[id - seg0] = v > 0.0f ? __fdiv_rn(v, P.rep_penalty) : __fmul_rn(v, P.rep_penalty);
            }
        }
        __syncthreads();
        lmax = NEG_INF;
        for (uint32_t i = tid; i < segn; i += KA_THREADS) lmax = fmaxf(lmax, seg[i]);
    }
    best = warp_arg(best);
    lmax = warp_max(lmax);
    if (lane == 0) {
        wbest[warp] = best;
        wmax[warp] = lmax;
    }
    __syncthreads();
    if (tid == 0) {
        ArgBest b = wbest[0];
        float m = wmax[0];
        for (int w = 1; w < KA_WARPS; w++) {
            b = arg_better(b, wbest[w]);
            m = fmaxf(m, wmax[w]);
        }
        xs.pmax = m;
        xs.rmax = b.v;
        xs.rarg = b.i;
    }
    cluster.sync();  // #1

    // ---- phase 2: row max ----------------------------------------------------
    float M = NEG_INF;
    {
        ArgBest b{NEG_INF, 0xFFFFFFFFu};
        for (uint32_t r = 0; r < P.C; r++) {
            const XSlot *o = cluster.map_shared_rank(&xs, r);
            M = fmaxf(M, o->pmax);
            b = arg_better(b, ArgBest{o->rmax, o->rarg});
        }
        if (rank == 0 && tid == 0) {
            hdr->M = M;
            hdr->raw_max = b.v;
            hdr->raw_arg = (xs.nan_any || b.i == 0xFFFFFFFFu) ? 0u : b.i;
            for (uint32_t r = 0; r < P.C; r++) hdr->seg_tile0[r] = r * NT;
        }
    }
    const float T = P.T;
    const float c2 = P.c2;
    const bool t_nan = (T != T);
    const bool t_inf = isinf(T);

    // ---- phase 3a: approximate tile sums and tile maxima ---------------------
    uint32_t nan_local = 0;
    for (uint32_t t = warp; t < NT; t += KA_WARPS) {
        const float v = seg[t * TILE + lane];
        const float d = __fsub_rn(v, M);
        const bool real = seg0 + t * TILE + lane < V;   // not padding
        const bool isn = real && ((d != d) || t_nan || (isinf(d) && t_inf));
        nan_local |= isn ? 1u : 0u;
        const float x2 = (d == 0.0f) ? 0.0f : d * c2;
        const float pt = isn ? 0.0f : ex2_approx(x2);
        const float s = warp_sum(pt);
        const float mx = warp_max(v);
        if (lane == 0) {
            tsum[t] = (double)s;
            tmax[t] = mx;
        }
    }
    nan_local = __any_sync(0xffffffffu, nan_local != 0) ? 1u : 0u;
    if (lane == 0) wnan[warp] = nan_local;
    for (uint32_t t = NT + tid; t < P.ksort; t += KA_THREADS) tmax[t] = NEG_INF;
    __syncthreads();
    if (tid == 0) {
        uint32_t n = 0;
        for (int w = 0; w < KA_WARPS; w++) n |= wnan[w];
        xs.nan_any = n;   // (the leading-NaN bit was consumed in phase 2)
    }
    {
        for (uint32_t t = tid; t < NT; t += KA_THREADS) pref[t] = tsum[t];
        __syncthreads();
        const double tot = block_exscan_d(pref, NT, wtmp_d);
        if (tid == 0) xs.tot_raw = tot;
    }
    cluster.sync();  // #2
    double base_raw = 0.0, s_raw = 0.0;
    uint32_t row_nan = 0;
    for (uint32_t r = 0; r < P.C; r++) {
        const XSlot *o = cluster.map_shared_rank(&xs, r);
        if (r < rank) base_raw += o->tot_raw;
        s_raw += o->tot_raw;
        row_nan |= o->nan_any;
    }

    // top-p tail-mass histogram: elements with log2 p >= f0 (f0 bounds the mass
    // below it by a quarter of the top-p budget, V * 2^f0 <= (1-top_p) S / 4)
    const bool p_active = P.top_p > 0.0f && P.top_p < 1.0f;
    const bool hist_on = p_active && (1.0f - P.top_p) >= 1e-3f;
    const double s_lo = fmax(1.0, 0.99 * s_raw);
    const float f0 = hist_on ? (float)(log2((1.0 - (double)P.top_p) * s_lo / (4.0 * (double)V)) - 1e-3)
                             : 0.0f;
    const float binw = fmaxf(0.125f, -f0 / (float)HIST_BINS);
    const float inv_binw = 1.0f / binw;
    for (uint32_t b = tid; b < HIST_BINS; b += KA_THREADS) hist[b] = 0.0f;
    __syncthreads();

    // ---- phase 3b: rounding-aware tile sums ---------------------------------
    for (uint32_t t = warp; t < NT; t += KA_WARPS) {
        const double Pt = base_raw + pref[t];
        const int e = binade_of(Pt);
        const float v = seg[t * TILE + lane];
        const float d = __fsub_rn(v, M);
        const bool isn = (d != d) || t_nan || (isinf(d) && t_inf);
        const float x2 = (d == 0.0f) ? 0.0f : d * c2;
        float q = 0.0f, big = 0.0f;
        const float ex = x2 - (float)(e - 23);   // log2(p / u_e)
        if (!isn && ex >= -1.01f) {
            if (ex < 22.0f) {
                const float y = ex2_approx(ex);
                q = (y + 12582912.0f) - 12582912.0f;  // round to the grid (rint)
            } else {
                big = ex2_approx(x2);                 // far above the grid: p itself
            }
        }
        if (hist_on && !isn && x2 >= f0) {
            const int b = min(HIST_BINS - 1, (int)((x2 - f0) * inv_binw));
            atomicAdd(&hist[b], ex2_approx(x2));
        }
        const float s = warp_sum(q);
        const float sb = warp_sum(big);
        if (lane == 0) tsum[t] = (double)s * exp2((double)(e - 23)) + (double)sb;
    }
    __syncthreads();
    {
        for (uint32_t t = tid; t < NT; t += KA_THREADS) pref[t] = tsum[t];
        __syncthreads();
        const double tot = block_exscan_d(pref, NT, wtmp_d);
        if (tid == 0) xs.tot2 = tot;
    }

    // ---- candidate floor: top-k tile-max sort (local part) -------------------
    const bool k_active = P.top_k > 0 && P.top_k < V;
    const bool k_floor = k_active && P.top_k <= KSEL_MAX && P.ntiles_total >= P.top_k;
    if (k_floor) {
        // bitonic sort, descending, of tmax[0..ksort)
        for (uint32_t size = 2; size <= P.ksort; size <<= 1) {
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                __syncthreads();
                for (uint32_t i = tid; i < P.ksort / 2; i += KA_THREADS) {
                    const uint32_t lo_i = 2 * i - (i & (stride - 1));
                    const uint32_t hi_i = lo_i + stride;
                    const bool desc = ((lo_i & size) == 0);
                    const float a = tmax[lo_i], b = tmax[hi_i];
                    if (desc ? (a < b) : (a > b)) {
                        tmax[lo_i] = b;
                        tmax[hi_i] = a;
                    }
                }
            }
        }
        __syncthreads();
        if (tid == 0) xs.klen = min(P.top_k, NT);
    }
    cluster.sync();  // #3
    double base2 = 0.0, s_tot = 0.0;
    for (uint32_t r = 0; r < P.C; r++) {
        const XSlot *o = cluster.map_shared_rank(&xs, r);
        if (r < rank) base2 += o->tot2;
        s_tot += o->tot2;
    }
    if (hist_on) {
        for (uint32_t b = tid; b < HIST_BINS; b += KA_THREADS) {
            float m = 0.0f;
            for (uint32_t r = 0; r < P.C; r++) m += cluster.map_shared_rank(hist, r)[b];
            ghist[b] = m;
        }
        __syncthreads();
    }
    float xk2 = NEG_INF;
    if (k_floor) {
        const uint32_t K = P.top_k;
        // gather every CTA's sorted top list
        uint32_t lens[MAX_CLUSTER];
        for (uint32_t r = 0; r < P.C; r++) {
            const XSlot *o = cluster.map_shared_rank(&xs, r);
            lens[r] = o->klen;
            const float *lst = cluster.map_shared_rank(tmax, r);
            for (uint32_t j = tid; j < o->klen; j += KA_THREADS) kgather[r * KSEL_MAX + j] = lst[j];
        }
        if (tid == 0) kth_sh = NEG_INF;
        __syncthreads();
        // the K-th largest value w satisfies  #(> w) < K <= #(>= w)
        const uint32_t total = P.C * KSEL_MAX;
        for (uint32_t i = tid; i < total; i += KA_THREADS) {
            const uint32_t r0 = i / KSEL_MAX, j0 = i % KSEL_MAX;
            if (j0 >= lens[r0]) continue;
            const float w = kgather[i];
            uint32_t gt = 0, ge = 0;
            for (uint32_t r = 0; r < P.C; r++) {
                const float *l = kgather + r * KSEL_MAX;
                uint32_t a = 0, b = lens[r];  // count of l[j] > w (sorted desc)
                while (a < b) {
                    const uint32_t mid = (a + b) >> 1;
                    if (l[mid] > w) a = mid + 1; else b = mid;
                }
                gt += a;
                uint32_t a2 = a, b2 = lens[r];  // count of l[j] >= w
                while (a2 < b2) {
                    const uint32_t mid = (a2 + b2) >> 1;
                    if (l[mid] >= w) a2 = mid + 1; else b2 = mid;
                }
                ge += a2;
            }
            if (gt < K && K <= ge) kth_sh = w;   // unique value; benign race
        }
        __syncthreads();
        const float vk = kth_sh;
        const float dk = __fsub_rn(vk, M);
        xk2 = (dk == 0.0f ? 0.0f : dk * c2) - 1e-3f - fabsf(dk * c2) * 1e-6f;
    }
    cluster.sync();  // #4: no distributed shared memory access after this point

    // floors in log2 units of p (x2 = log2 p, approximately)
    float xf2 = -151.0f;   // p > 0 only
    uint32_t binding = 0;  // 0 none, 1 k, 2 p, 3 min-p
    if (k_floor && xk2 > xf2) { xf2 = xk2; binding = 1; }
    if (hist_on) {
        // highest bin edge f* with (mass in [f0, f*)) <= (1-top_p) S / 4, so the
        // mass below f* is at most half of the top-p budget: the cumulative
        // probability of the tokens above f* exceeds top_p with margin.
        const float budget = (float)((1.0 - (double)P.top_p) * s_lo / 4.0);
        float acc = 0.0f;
        int bstar = 0;
        for (int b = 0; b < HIST_BINS; b++) {
            acc += ghist[b] * 1.001f;
            if (acc > budget) break;
            bstar = b + 1;
        }
        const float xp = f0 + (float)bstar * binw - 1e-3f;
        if (xp > xf2) { xf2 = xp; binding = 2; }
    }
    if (P.min_p > 0.0f) {
        const double xm = fmin(0.0, log2((double)P.min_p)) - 0.01;
        if ((float)xm > xf2) { xf2 = (float)xm; binding = 3; }
    }
    if (rank == 0 && tid == 0) {
        hdr->s_approx = (float)s_tot;
        hdr->v_floor = xf2;
        hdr->binding = binding;
        if (row_nan) hdr->flags |= RF_NAN;
    }

    // ---- phase 4: classify tiles, grid counts, candidates ---------------------
    Candidate *cand = P.cand + (size_t)hrow * P.cand_stride;
    float *wcd = P.wcdata + (size_t)hrow * WC_CAP * TILE;
    for (uint32_t t = warp; t < NT; t += KA_WARPS) {
        const double Ps = base2 + pref[t];
        const double Pe = Ps + tsum[t];
        const int lo = binade_of(Ps * (1.0 - DELTA));
        const int hi = binade_of(Pe * (1.0 + DELTA));
        const uint32_t cls = hi == lo ? CLS_SIMPLE : (hi == lo + 1 ? CLS_WINDOW : CLS_COMPLEX);
        const uint32_t gidx = seg0 + t * TILE + lane;
        const float v = seg[t * TILE + lane];
        const float d = __fsub_rn(v, M);
        const float x2 = (d == 0.0f) ? 0.0f : d * c2;
        const bool valid = gidx < V && !row_nan;
        const bool sig = valid && (lo - 24 <= -149 || x2 >= (float)(lo - 24) - 0.01f);
        const bool cnd = valid && x2 >= xf2;
        float p = 0.0f;
        if (sig || cnd || (valid && cls != CLS_SIMPLE)) p = prob_unnorm(v, M, T);
        Comp clo{0u, 0u}, chi{0u, 0u};
        if (sig) {
            clo = elem_comp(p, lo);
            if (cls == CLS_WINDOW) chi = elem_comp(p, lo + 1);
        }
        if (__any_sync(0xffffffffu, sig)) {
            clo = warp_comp_reduce(clo);
            if (cls == CLS_WINDOW) chi = warp_comp_reduce(chi);
        }
        const uint32_t cmask = __ballot_sync(0xffffffffu, cnd && p > 0.0f);
        if (cmask) {
            uint32_t basec = 0;
            if (lane == 0) basec = atomicAdd(&hdr->n_cand, (uint32_t)__popc(cmask));
            basec = __shfl_sync(0xffffffffu, basec, 0);
            if (cnd && p > 0.0f) {
                const uint32_t pos = basec + __popc(cmask & ((1u << lane) - 1u));
                if (pos < P.cand_stride) cand[pos] = Candidate{gidx, p};
            }
        }
        uint32_t aux = 0;
        if (cls != CLS_SIMPLE) {
            uint32_t slot = 0;
            if (lane == 0) slot = atomicAdd(&hdr->n_wc, 1u);
            slot = __shfl_sync(0xffffffffu, slot, 0);
            if (slot < WC_CAP) {
                wcd[slot * TILE + lane] = sig ? p : 0.0f;
                aux = slot;
            } else {
                aux = 0xFFFFFFFFu;
            }
        }
        if (lane == 0) {
            TileRec r;
            r.lo = lo;
            r.cls = cls;
            r.aux = aux;
            r.qlo = clo;
            r.qhi = chi;
            rec[t] = r;
        }
    }
    __syncthreads();

    // ---- phase 5: items ------------------------------------------------------
    // head[t]: tile t starts an item (every WINDOW/COMPLEX tile, and a SIMPLE
    // tile whose predecessor is not a SIMPLE tile of the same binade).
    for (uint32_t t = tid; t < NT; t += KA_THREADS) {
        const TileRec r = rec[t];
        uint32_t h = 1;
        if (t > 0) {
            const TileRec q = rec[t - 1];
            h = (r.cls != CLS_SIMPLE || q.cls != CLS_SIMPLE || r.lo != q.lo) ? 1u : 0u;
        }
        uarr[t] = h;
        carr[t] = r.qlo;
    }
    __syncthreads();
    block_segscan_comp(carr, uarr, NT, wtmp_s);   // carr[t]: composite from item start to t
    const uint32_t nitems = block_exscan_u(uarr, NT, wtmp_u);  // uarr[t]: heads before t
    uint32_t *sstart = reinterpret_cast<uint32_t *>(tmax);     // free after the floor phase
    for (uint32_t t = tid; t < NT; t += KA_THREADS) {
        const uint32_t nxt = (t + 1 < NT) ? uarr[t + 1] : nitems;
        if (nxt != uarr[t]) sstart[uarr[t]] = t;             // t is a head
    }
    __syncthreads();
    Item *items = P.items + (size_t)hrow * P.ntiles_total + tile0;
    for (uint32_t t = tid; t < NT; t += KA_THREADS) {
        const uint32_t id = ((t + 1 < NT) ? uarr[t + 1] : nitems) - 1u;  // item of tile t
        bool is_end = (t + 1 == NT);
        if (!is_end) {
            const uint32_t nxt2 = (t + 2 < NT) ? uarr[t + 2] : nitems;
            is_end = (nxt2 != uarr[t + 1]);                                // t+1 is a head
        }
        if (is_end) {
            const TileRec r = rec[t];
            const uint32_t start = sstart[id];
            Item it;
            it.kind = r.cls;
            it.lo = r.lo;
            if (r.cls == CLS_SIMPLE) {
                const Comp c = carr[t];
                it.q[0] = c.q0;
                it.q[1] = c.q1;
                it.q[2] = 0u;
                it.q[3] = 0u;
                it.aux = t - start + 1u;
            } else {
                it.q[0] = r.qlo.q0;
                it.q[1] = r.qlo.q1;
                it.q[2] = r.qhi.q0;
                it.q[3] = r.qhi.q1;
                it.aux = r.aux;
            }
            it.tile = tile0 + start;
            items[id] = it;
        }
    }
    if (tid == 0) hdr->seg_items[rank] = nitems;
}

// ---------------------------------------------------------------------------
struct KBParams {
    const float *logits;
    size_t ld;
    const uint32_t *prev;
    uint32_t n_prev;
    uint32_t vocab;
    uint32_t row0;
    float T;
    uint32_t top_k;
    float top_p;
    float min_p;
    float typical_p;
    uint32_t rep_window;
    float rep_penalty;
    uint32_t ntiles_total;
    RowHdr *hdr;
    Item *items;
    float *wcdata;
    Candidate *cand;     // per handle row: cand_stride entries (Kernel A output)
    unsigned long long *ctmp;  // per handle row: 2 x cand_stride keys (large-set path)
    uint32_t cand_stride;
    uint64_t *rng;       // per handle row, 4 words
    RowTrace *trace;     // per handle row
    uint32_t *out;       // per call row
};

// Exact p of element g (with the repetition penalty), for the recompute path.
__device__ float exact_p_at(const KBParams &P, uint32_t row, uint32_t g, float M, const uint32_t *win,
                            uint32_t nwin) {
    if (g >= P.vocab) return 0.0f;
    float v = P.logits[(size_t)row * P.ld + g];
    for (uint32_t j = 0; j < nwin; j++) {
        if (win[j] == g) {
            v = v > 0.0f ? __fdiv_rn(v, P.rep_penalty) : __fmul_rn(v, P.rep_penalty);
            break;
        }
    }
    return prob_unnorm(v, M, P.T);
}

// Candidate key: ascending key order == (p descending, index ascending).
__device__ __forceinline__ unsigned long long cand_key(Candidate c) {
    return ((unsigned long long)(0xFFFFFFFFu - __float_as_uint(c.p)) << 32) | c.idx;
}
__device__ __forceinline__ float key_p(unsigned long long k) {
    return __uint_as_float(0xFFFFFFFFu - (uint32_t)(k >> 32));
}

// Stable LSD radix sort (4-bit digits) of n keys by one CTA, global memory.
// Returns the buffer holding the sorted keys (a or b).
__device__ unsigned long long *cta_radix_sort(unsigned long long *a, unsigned long long *b, uint32_t n,
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
    for (int sh = 0; sh < 64; sh += 4) {
        if (((vary >> sh) & 0xFull) == 0) continue;
        uint32_t c[16];
#pragma unroll
        for (int d = 0; d < 16; d++) c[d] = 0;
        for (uint32_t i = lo; i < hi; i++) c[(a[i] >> sh) & 0xF]++;
#pragma unroll
        for (int d = 0; d < 16; d++) cnt[d * KB_THREADS + tid] = c[d];
        __syncthreads();
        if (tid == 0) {   // exclusive scan, digit-major
            uint32_t run = 0;
            for (int i = 0; i < 16 * KB_THREADS; i++) {
                const uint32_t v = cnt[i];
                cnt[i] = run;
                run += v;
            }
        }
        __syncthreads();
#pragma unroll
        for (int d = 0; d < 16; d++) c[d] = cnt[d * KB_THREADS + tid];
        for (uint32_t i = lo; i < hi; i++) {
            const unsigned long long k = a[i];
            b[c[(k >> sh) & 0xF]++] = k;
        }
        __syncthreads();
        unsigned long long *t = a;
        a = b;
        b = t;
    }
    return a;
}

__global__ void __launch_bounds__(KB_THREADS) kernel_b(KBParams P) {
    const uint32_t row = blockIdx.x;
    const uint32_t hrow = P.row0 + row;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const RowHdr *hdr = P.hdr + hrow;

    __shared__ Item sitems[ITEM_CHUNK];
    __shared__ float tilep[TILE];
    __shared__ uint32_t swin[256];
    __shared__ float S_sh;
    __shared__ uint32_t walk_flags;
    __shared__ unsigned long long red2[2];
    extern __shared__ __align__(16) unsigned char smem[];
    unsigned long long *skeys = reinterpret_cast<unsigned long long *>(smem);  // CAND_SMEM
    float *wcs = reinterpret_cast<float *>(skeys + CAND_SMEM);                 // WC_CAP*32
    float *sprobs = wcs + WC_CAP * TILE;                                       // CAND_SMEM

    const float M = hdr->M;
    const uint32_t flags0 = hdr->flags;
    const uint32_t n_cand = min(hdr->n_cand, P.cand_stride);
    const uint32_t n_wc = min(hdr->n_wc, (uint32_t)WC_CAP);
    const bool big = n_cand > (uint32_t)CAND_SMEM;

    // penalty window (for the recompute path)
    uint32_t nwin = 0;
    if (P.rep_penalty != 1.0f && P.n_prev > 0 && P.prev != nullptr && P.rep_window > 0) {
        const uint32_t win = min(min(P.n_prev, P.rep_window), 256u);
        const uint32_t start = P.n_prev - win;
        for (uint32_t j = tid; j < win; j += KB_THREADS) swin[j] = P.prev[(size_t)row * P.n_prev + start + j];
        nwin = win;
    }
    const float *wcg = P.wcdata + (size_t)hrow * WC_CAP * TILE;
    for (uint32_t i = tid; i < n_wc * TILE; i += KB_THREADS) wcs[i] = wcg[i];
    const Candidate *cg_ = P.cand + (size_t)hrow * P.cand_stride;
    unsigned long long *gk0 = P.ctmp + (size_t)hrow * 2 * P.cand_stride;
    unsigned long long *gk1 = gk0 + P.cand_stride;
    uint32_t npow = 1;
    if (!big) {
        while (npow < n_cand) npow <<= 1;
        for (uint32_t i = tid; i < npow; i += KB_THREADS) skeys[i] = i < n_cand ? cand_key(cg_[i]) : ~0ull;
    }
    if (tid == 0) walk_flags = 0;
    __syncthreads();

    if (warp == 0) {
        // ---- the exact walk of the sequential f32 sum ----
        SumState st{-126, 0u};
        uint32_t wflags = 0;
        const uint32_t nseg = min(hdr->nseg, (uint32_t)MAX_CLUSTER);
        for (uint32_t sgi = 0; sgi < nseg; sgi++) {
            const uint32_t t0 = min(hdr->seg_tile0[sgi], P.ntiles_total);
            const uint32_t nit = min(hdr->seg_items[sgi], P.ntiles_total - t0);
            const Item *ig = P.items + (size_t)hrow * P.ntiles_total + t0;
            for (uint32_t i0 = 0; i0 < nit; i0 += ITEM_CHUNK) {
                const uint32_t nc = min((uint32_t)ITEM_CHUNK, nit - i0);
                __syncwarp();
                for (uint32_t j = lane; j < nc; j += 32) sitems[j] = ig[i0 + j];
                __syncwarp();
                for (uint32_t j = 0; j < nc; j++) {
                    const Item it = sitems[j];
                    bool done = false;
                    if (lane == 0) {
                        const uint32_t par = st.m & 1u;
                        if (st.e == it.lo) {
                            const uint32_t q = par ? it.q[1] : it.q[0];
                            if (st.m + q < QLIM && q < QSAT) { st.m += q; done = true; }
                        } else if (it.kind == CLS_WINDOW && st.e == it.lo + 1) {
                            const uint32_t q = par ? it.q[3] : it.q[2];
                            if (st.m + q < QLIM && q < QSAT) { st.m += q; done = true; }
                        }
                    }
                    done = __shfl_sync(0xffffffffu, done, 0);
                    if (done) continue;
                    // element-wise: stored p (valid when the state is at or above
                    // binade lo), else recomputed from the logits
                    const int e_now = __shfl_sync(0xffffffffu, st.e, 0);
                    const bool stored = it.kind != CLS_SIMPLE && it.aux != 0xFFFFFFFFu &&
                                        it.aux < n_wc && e_now >= it.lo;
                    const uint32_t ntl = it.kind == CLS_SIMPLE ? min(it.aux, P.ntiles_total) : 1u;
                    if (!stored) wflags |= RF_SLOW_WALK;
                    for (uint32_t tt = 0; tt < ntl; tt++) {
                        const float pv = stored ? wcs[it.aux * TILE + lane]
                                                : exact_p_at(P, row, (it.tile + tt) * TILE + lane, M, swin, nwin);
                        tilep[lane] = pv;
                        __syncwarp();
                        if (lane == 0) {
                            float s = float_of(st);
                            for (int k = 0; k < TILE; k++) s = __fadd_rn(s, tilep[k]);
                            st = state_of(s);
                        }
                        __syncwarp();
                    }
                }
            }
        }
        if (lane == 0) {
            S_sh = float_of(st);
            walk_flags = wflags;
        }
    } else if (!big) {
        // ---- candidate sort in shared memory: ascending key ----
        const int t2 = tid - 32, nthr = KB_THREADS - 32;
        for (uint32_t size = 2; size <= npow; size <<= 1) {
            for (uint32_t stride = size >> 1; stride > 0; stride >>= 1) {
                asm volatile("bar.sync 1, %0;" ::"r"(nthr));
                for (uint32_t i = t2; i < npow / 2; i += nthr) {
                    const uint32_t a = 2 * i - (i & (stride - 1));
                    const uint32_t b = a + stride;
                    const bool up = ((a & size) == 0);
                    const unsigned long long ka = skeys[a], kb = skeys[b];
                    if (up ? (ka > kb) : (ka < kb)) {
                        skeys[a] = kb;
                        skeys[b] = ka;
                    }
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(nthr));
    }
    __syncthreads();

    // large candidate sets: stable radix sort in global memory (whole CTA)
    unsigned long long *keys = skeys;
    float *probs = sprobs;
    if (big) {
        for (uint32_t i = tid; i < n_cand; i += KB_THREADS) gk0[i] = cand_key(cg_[i]);
        __syncthreads();
        uint32_t *cnt = reinterpret_cast<uint32_t *>(sprobs);   // 16 * KB_THREADS words
        keys = cta_radix_sort(gk0, gk1, n_cand, cnt, red2);
        probs = reinterpret_cast<float *>(keys == gk0 ? gk1 : gk0);
        __syncthreads();
    }

    const float S = S_sh;
    const bool nan_row = (flags0 & RF_NAN) != 0;
    // exact probs in sorted order (sampler.zig:90)
    for (uint32_t i = tid; i < n_cand; i += KB_THREADS) probs[i] = __fdiv_rn(key_p(keys[i]), S);
    __syncthreads();
    if (tid != 0) return;

    uint32_t status = ROW_OK;
    uint32_t token = 0;
    uint32_t path = 0;
    uint32_t n_kept = 0;
    float total = 0.0f, u = __int_as_float(0x7fc00000);
    uint64_t s4[4];
    uint64_t *rng = P.rng + (size_t)hrow * 4;
    s4[0] = rng[0]; s4[1] = rng[1]; s4[2] = rng[2]; s4[3] = rng[3];
    uint32_t flags = flags0 | walk_flags | (big ? RF_CAND_BIG : 0u);
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
        token = hdr->raw_arg;   // sampler.zig:89
        path = 1;
    } else {
        // idxs[2*i] aliases the low word of keys[i]
        uint32_t *idxs = reinterpret_cast<uint32_t *>(keys);
        // ties: equal probs from distinct p keep index order (stable sort)
        for (uint32_t i = 1; i < n_cand; i++) {
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
        // The candidates are every token above a floor, i.e. a prefix of the
        // reference's sorted order.  The kept prefix is settled inside it when
        // some filter cuts before its end, when the candidates are all tokens
        // with p > 0, or when the floor is the binding filter's own bound.
        uint32_t n_sel = n_cand;
        const uint32_t binding = hdr->binding;
        const bool k_act = P.top_k > 0 && P.top_k < P.vocab;
        // top-k (sampler.zig:106-109)
        if (k_act && n_sel > P.top_k) n_sel = P.top_k;
        // top-p (sampler.zig:111-118): the crossing token is deselected too
        if (P.top_p > 0.0f && P.top_p < 1.0f) {
            float cum = 0.0f;
            for (uint32_t j = 0; j < n_sel; j++) {
                cum = __fadd_rn(cum, probs[j]);
                if (cum > P.top_p) {
                    n_sel = j;
                    break;
                }
            }
        }
        // min-p (sampler.zig:120-126) against probs[indices[0]]
        if (P.min_p > 0.0f && n_cand > 0) {
            const float thr = __fmul_rn(probs[0], P.min_p);
            uint32_t j = 0;
            while (j < n_sel && !(probs[j] < thr)) j++;
            n_sel = j;
        }
        const bool cover_ok = binding == 0 || binding == 1 || binding == 3 || n_sel < n_cand ||
                              (k_act && P.top_k <= n_cand);
        if (!cover_ok) {
            status = ROW_EINTERNAL;
            flags |= RF_CAND_SHORT;
        } else if (P.typical_p > 0.0f && P.typical_p < 1.0f) {
            status = ROW_ENOTSUP;  // typical-p runs in its own pass (not in this build)
        } else {
            // kept mass in sorted order (sampler.zig:156-159)
            for (uint32_t j = 0; j < n_sel; j++) total = __fadd_rn(total, probs[j]);
            n_kept = n_sel;
            if (!(total > 0.0f)) {
                token = n_cand > 0 ? idxs[0] : 0u;  // sampler.zig:160
                path = 2;
            } else {
                u = rng_float(s4);
                float r = __fmul_rn(u, total);
                token = idxs[0];
                path = 4;
                for (uint32_t j = 0; j < n_sel; j++) {
                    r = __fsub_rn(r, probs[j]);
                    if (r <= 0.0f) {
                        token = idxs[2 * j];
                        path = 3;
                        break;
                    }
                }
            }
        }
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
    tr.n_cand = n_cand;
    tr.status = status;
    P.trace[hrow] = tr;
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
    uint32_t C, seg_len, ntiles_seg, ntiles_total, ksort;
    size_t smem_a, smem_b;
    uint64_t *d_rng;
    RowHdr *d_hdr;
    Item *d_items;
    float *d_wc;
    Candidate *d_cand;
    unsigned long long *d_ctmp;
    uint32_t cand_stride;
    RowTrace *d_trace;
    float *d_logits_stage;   // host-path staging
    uint32_t *d_prev_stage;
    uint32_t *d_out_stage;
    size_t stage_floats;
    size_t stage_prev;
    cudaStream_t stream;
    cudaEvent_t *prof_ev;    // profiling ring: 3 events per bs_sample call
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
    cudaFree(s->d_items);
    cudaFree(s->d_wc);
    cudaFree(s->d_cand);
    cudaFree(s->d_ctmp);
    cudaFree(s->d_trace);
    cudaFree(s->d_logits_stage);
    cudaFree(s->d_prev_stage);
    cudaFree(s->d_out_stage);
    if (s->stream) cudaStreamDestroy(s->stream);
    for (uint32_t i = 0; s->prof_ev && i < 3 * s->prof_cap; i++) cudaEventDestroy(s->prof_ev[i]);
    delete[] s->prof_ev;
}

// The dynamic shared-memory limit is a per-function attribute: keep it at the
// largest size any handle in this process needs.
static size_t g_smem_a = 0, g_smem_b = 0;
static cudaError_t raise_smem_limits(size_t a, size_t b) {
    cudaError_t e = cudaSuccess;
    if (a > g_smem_a) {
        e = cudaFuncSetAttribute(kernel_a, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)a);
        if (e == cudaSuccess) g_smem_a = a;
    }
    if (e == cudaSuccess && b > g_smem_b) {
        e = cudaFuncSetAttribute(kernel_b, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)b);
        if (e == cudaSuccess) g_smem_b = b;
    }
    return e;
}

extern "C" bs_status bs_create(const bs_config *cfg, uint32_t batch, uint32_t vocab, int device,
                               const uint64_t *seeds, bs_sampler **out) {
    if (!cfg || !out || batch == 0 || vocab == 0) return BS_EINVAL;
    if (vocab > (uint32_t)(MAX_CLUSTER * SEG_MAX)) return BS_ENOTSUP;
    *out = nullptr;
    BS_CUDA(cudaSetDevice(device));
    bs_sampler *s = new (std::nothrow) bs_sampler();
    if (!s) return BS_ENOMEM;
    memset(s, 0, sizeof(*s));
    s->cfg = *cfg;
    s->batch = batch;
    s->vocab = vocab;
    s->device = device;
    // segments: one CTA per ~SEG_TARGET elements, at most MAX_CLUSTER per row
    uint32_t C = (vocab + SEG_TARGET - 1) / SEG_TARGET;
    if (C < 1) C = 1;
    if (C > (uint32_t)MAX_CLUSTER) C = MAX_CLUSTER;
    uint32_t seg = (vocab + C - 1) / C;
    seg = (seg + TILE - 1) / TILE * TILE;
    while (C > 1 && (C - 1) * seg >= vocab) C--;   // no empty segment
    s->C = C;
    s->seg_len = seg;
    s->ntiles_seg = seg / TILE;
    s->ntiles_total = C * s->ntiles_seg;
    uint32_t ks = 1;
    while (ks < s->ntiles_seg) ks <<= 1;
    s->ksort = ks;
    s->smem_a = (size_t)seg * 4 + (size_t)s->ntiles_seg * 16 + (size_t)ks * 4 +
                (size_t)s->ntiles_seg * (sizeof(TileRec) + 4 + sizeof(Comp)) + 64;
    s->smem_b = (size_t)CAND_SMEM * 8 + (size_t)WC_CAP * TILE * 4 + (size_t)CAND_SMEM * 4;
    s->cand_stride = (vocab + 31u) & ~31u;

    cudaError_t e = cudaSuccess;
    e = cudaMalloc(&s->d_rng, (size_t)batch * 4 * sizeof(uint64_t));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_hdr, (size_t)batch * sizeof(RowHdr));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_items, (size_t)batch * s->ntiles_total * sizeof(Item));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_wc, (size_t)batch * WC_CAP * TILE * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_cand, (size_t)batch * s->cand_stride * sizeof(Candidate));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_ctmp, (size_t)batch * 2 * s->cand_stride * sizeof(unsigned long long));
    if (e == cudaSuccess) e = cudaMalloc(&s->d_trace, (size_t)batch * sizeof(RowTrace));
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
    if (e == cudaSuccess) e = raise_smem_limits(s->smem_a, s->smem_b);
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

extern "C" bs_status bs_argmax(const float *d_logits, size_t ld, uint32_t rows, uint32_t vocab,
                               uint32_t *d_out, void *stream) {
    if (!d_logits || !d_out || vocab == 0 || ld < vocab) return BS_EINVAL;
    if (rows == 0) return BS_OK;
    argmax_kernel<<<rows, 512, 0, (cudaStream_t)stream>>>(d_logits, ld, vocab, d_out);
    return cuda_status(cudaGetLastError());
}

extern "C" bs_status bs_sample(bs_sampler *s, const float *d_logits, size_t ld, uint32_t row0,
                               uint32_t rows, const uint32_t *d_prev, uint32_t n_prev, uint32_t *d_out,
                               void *stream) {
    if (!s || !d_logits || !d_out || ld < s->vocab) return BS_EINVAL;
    if (row0 > s->batch || rows > s->batch - row0) return BS_EINVAL;
    if (rows == 0) return BS_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const bs_config &c = s->cfg;
    // sampler.zig:50 -- temperature <= 0: argmax of the raw logits, no draw
    if (c.temperature <= 0.0f) return bs_argmax(d_logits, ld, rows, s->vocab, d_out, stream);

    KAParams A;
    A.logits = d_logits;
    A.ld = ld;
    A.prev = d_prev;
    A.n_prev = d_prev ? n_prev : 0;
    A.vocab = s->vocab;
    A.row0 = row0;
    A.T = c.temperature;
    A.c2 = (float)(1.4426950408889634 / (double)c.temperature);
    A.top_k = c.top_k;
    A.top_p = c.top_p;
    A.min_p = c.min_p;
    A.rep_window = c.repetition_window;
    A.rep_penalty = c.repetition_penalty;
    A.C = s->C;
    A.seg_len = s->seg_len;
    A.ntiles_seg = s->ntiles_seg;
    A.ntiles_total = s->ntiles_total;
    A.ksort = s->ksort;
    A.hdr = s->d_hdr;
    A.items = s->d_items;
    A.wcdata = s->d_wc;
    A.cand = s->d_cand;
    A.cand_stride = s->cand_stride;

    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(s->C, rows, 1);
    cfg.blockDim = dim3(KA_THREADS, 1, 1);
    cfg.dynamicSmemBytes = s->smem_a;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = s->C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaEvent_t *ev = nullptr;
    if (s->prof_ev && s->prof_n < s->prof_cap) ev = s->prof_ev + 3 * s->prof_n++;
    if (ev) cudaEventRecord(ev[0], st);
    cudaError_t e = cudaLaunchKernelEx(&cfg, kernel_a, A);
    if (e != cudaSuccess) {
        fprintf(stderr, "b200_sampler: kernel A launch failed: %s\n", cudaGetErrorString(e));
        return BS_ECUDA;
    }

    KBParams B;
    B.logits = d_logits;
    B.ld = ld;
    B.prev = A.prev;
    B.n_prev = A.n_prev;
    B.vocab = s->vocab;
    B.row0 = row0;
    B.T = c.temperature;
    B.top_k = c.top_k;
    B.top_p = c.top_p;
    B.min_p = c.min_p;
    B.typical_p = c.typical_p;
    B.rep_window = c.repetition_window;
    B.rep_penalty = c.repetition_penalty;
    B.ntiles_total = s->ntiles_total;
    B.hdr = s->d_hdr;
    B.items = s->d_items;
    B.wcdata = s->d_wc;
    B.cand = s->d_cand;
    B.ctmp = s->d_ctmp;
    B.cand_stride = s->cand_stride;
    B.rng = s->d_rng;
    B.trace = s->d_trace;
    B.out = d_out;
    if (ev) cudaEventRecord(ev[1], st);
    kernel_b<<<rows, KB_THREADS, s->smem_b, st>>>(B);
    if (ev) cudaEventRecord(ev[2], st);
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
        else if (h[i].status != ROW_OK) r = BS_EINTERNAL;
    }
    delete[] h;
    return r;
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
    for (uint32_t i = 0; s->prof_ev && i < 3 * s->prof_cap; i++) cudaEventDestroy(s->prof_ev[i]);
    delete[] s->prof_ev;
    s->prof_ev = nullptr;
    s->prof_cap = s->prof_n = 0;
    if (max_calls == 0) return BS_OK;
    s->prof_ev = new (std::nothrow) cudaEvent_t[3 * (size_t)max_calls];
    if (!s->prof_ev) return BS_ENOMEM;
    for (uint32_t i = 0; i < 3 * max_calls; i++) BS_CUDA(cudaEventCreate(&s->prof_ev[i]));
    s->prof_cap = max_calls;
    return BS_OK;
}

extern "C" bs_status bs_profile_read(bs_sampler *s, float *ms_a, float *ms_b, uint32_t *n_calls) {
    if (!s || !ms_a || !ms_b || !n_calls) return BS_EINVAL;
    BS_CUDA(cudaSetDevice(s->device));
    const uint32_t n = s->prof_n;
    for (uint32_t i = 0; i < n; i++) {
        BS_CUDA(cudaEventSynchronize(s->prof_ev[3 * i + 2]));
        BS_CUDA(cudaEventElapsedTime(&ms_a[i], s->prof_ev[3 * i], s->prof_ev[3 * i + 1]));
        BS_CUDA(cudaEventElapsedTime(&ms_b[i], s->prof_ev[3 * i + 1], s->prof_ev[3 * i + 2]));
    }
    *n_calls = n;
    s->prof_n = 0;
    return BS_OK;
}
