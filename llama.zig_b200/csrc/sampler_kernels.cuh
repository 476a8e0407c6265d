// sampler_kernels.cuh -- data layout shared by the sampler kernels and the
// host runtime.  See sampler.cu for the algorithm.
#pragma once

#include <cstdint>

namespace bs {

constexpr int TILE = 32;                 // elements per tile (one warp, one lane each)
constexpr int KA_THREADS = 512;          // Kernel A block size
constexpr int KA_WARPS = KA_THREADS / 32;
constexpr int KB_THREADS = 256;          // Kernel B block size
constexpr int MAX_CLUSTER = 8;           // portable cluster size
constexpr int SEG_TARGET = 16384;        // target elements per CTA segment
constexpr int SEG_MAX = 32768;           // hard cap (128 KB of shared memory)
constexpr int CAND_SMEM = 4096;          // candidates sorted in shared memory (fast path)
constexpr int HIST_BINS = 256;           // top-p tail-mass histogram bins
constexpr int WC_CAP = 256;              // window/complex tiles with stored p per row
constexpr int KSEL_MAX = 256;            // largest top_k served by the tile-max floor
constexpr int ITEM_CHUNK = 128;          // items staged per step in Kernel B (rows with many items)
constexpr int ITEM_SMEM = 512;           // items of a row held in shared memory (spread over its segments)
constexpr int WPOOL = 256;               // WINDOW prefix-table entries of a row held in shared memory

// Tile classes (running-sum binade candidates over the tile).
enum : uint32_t { CLS_SIMPLE = 0, CLS_WINDOW = 1, CLS_COMPLEX = 2 };

// Row flags.
enum : uint32_t {
    RF_NAN = 1u << 0,           // some p_i is NaN: sum is NaN (sampler.zig:87)
    RF_CAND_BIG = 1u << 1,      // more than CAND_SMEM candidates (global-memory path)
    RF_CAND_SHORT = 1u << 2,    // candidate set did not cover the kept prefix
    RF_SLOW_WALK = 1u << 3,     // walker needed the recompute path (diagnostic)
    RF_BAD_CONFIG = 1u << 4,
};

// Kernel output status per row (written by Kernel B).
enum : uint32_t { ROW_OK = 0, ROW_ETIMEOUT = 5, ROW_ENOTSUP = 6, ROW_EINTERNAL = 7 };

// Row header in scratch: written by Kernel A, read by Kernel B.
struct RowHdr {
    float M;             // max of penalised logits (sampler.zig:80-81)
    float raw_max;       // sampleArgmax of the raw logits, value ...
    uint32_t raw_arg;    // ... and index (sampler.zig:89 fallback)
    uint32_t flags;      // RF_*
    uint32_t n_cand;     // candidates appended
    uint32_t n_wc;       // window/complex tiles with stored p (may exceed WC_CAP)
    float s_approx;      // approximate normaliser
    float v_floor;       // candidate floor (logit domain)
    uint32_t seg_items[64];   // walk items per segment (MAX_SEG)
    uint32_t seg_tile0[64];
    uint32_t nseg;
    uint32_t binding;    // which filter set the candidate floor (0 none, 1 k, 2 p, 3 min-p)
    uint32_t pad[2];
};

// One walk item: a stretch of SIMPLE tiles with one binade, or one
// WINDOW/COMPLEX tile.  32 bytes.
struct Item {
    uint32_t kind;     // CLS_*
    int32_t lo;        // lowest candidate binade of the running sum
    uint32_t q[4];     // composite grid counts: lo parity 0/1, lo+1 parity 0/1
    uint32_t tile;     // first global tile index
    uint32_t aux;      // SIMPLE: tile count; WINDOW/COMPLEX: stored-p slot or ~0u
};

// Per-row diagnostics written by Kernel B (what the reference computed).
struct RowTrace {
    float S;           // sequential f32 normaliser
    float total;       // kept mass
    float u;           // Random.float draw (NaN if none)
    uint32_t n_kept;
    uint32_t path;     // 0 argmax(T<=0) 1 argmax(sum<=0) 2 empty 3 draw 4 fallback 5 NaN
    uint32_t flags;
    uint32_t n_cand;
    uint32_t status;
    uint32_t n_items;  // walk items of the row
    uint32_t n_wc;     // window/complex tiles
    uint32_t n_slow;   // tiles the walk recomputed from the logits
    uint32_t pad;
};

struct Candidate {
    uint32_t idx;
    float v;           // the (penalised) logit; the walk kernel computes p exactly
};

}  // namespace bs
