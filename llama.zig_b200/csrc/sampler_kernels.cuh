// sampler_kernels.cuh -- data layout shared by the sampler kernels and the
// host runtime.  See sampler.cu for the algorithm.
#pragma once

#include <cstdint>

namespace bs {

constexpr int TILE = 32;                 // elements per tile
constexpr int KB_THREADS = 256;          // walk/draw kernel block size
constexpr int CAND_SMEM = 4096;          // candidates sorted in shared memory (fast path)
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
    RF_TYP_BAND = 1u << 4,      // typical-p: the dev band did not cover the kept set
    RF_FULL = 1u << 5,          // resolved by the retry with every token as a candidate
};

// Typical-p modes of a row (sampler.zig:128-154).
enum : uint32_t {
    TYP_OFF = 0,       // typical_p outside (0, 1)
    TYP_SELECTED = 1,  // another filter bounds the selected set: typical-p runs over it
    TYP_BAND = 2,      // typical-p alone: candidates from a band of dev = |surprise - H|
};

// Per-row status (written by the walk/draw pass).
enum : uint32_t { ROW_OK = 0, ROW_ETIMEOUT = 5, ROW_ENOTSUP = 6, ROW_EINTERNAL = 7 };

// Row header in scratch: written by the statistics and main passes, read by
// the walk/draw pass.
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
    uint32_t binding;    // which filter set the candidate floor (0 none, 1 k, 2 p, 3 min-p, 4 typical)
    // typical-p (written by the normaliser's walk, read by the entropy passes)
    float S_exact;       // the sequential f32 normaliser
    uint32_t top_idx;    // indices[0]: the first token of the probability order
    uint32_t n_sel;      // TYP_SELECTED: size of the selected set
    uint32_t tdone;      // the row's token is final (NaN row, sum <= 0, ...)
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
    float H;           // typical-p: the sequential f32 entropy (NaN otherwise)
};

struct Candidate {
    uint32_t idx;
    float v;           // the (penalised) logit; the walk kernel computes p exactly
};

}  // namespace bs
