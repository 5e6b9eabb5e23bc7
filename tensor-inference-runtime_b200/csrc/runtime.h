// runtime.h -- device-side program description shared by the host driver
// (api.cpp) and the persistent sm_100a kernels (decode.cu).
//
// A "program" is the ordered list of phases of one forward step.  For the
// batch-1 decode loop of src/forward.rs:13-258 it is, per layer,
//   QKV  (rmsnorm -> fused q|k|v Q8_0 matvec -> RoPE -> KV-cache append)
//   ATTN (grouped-query attention over the cache, split over positions)
//   O    (output projection + residual)
//   GU   (rmsnorm -> fused gate|up matvec -> silu(gate)*up)
//   DOWN (down projection + residual)
// and finally LM (rmsnorm -> vocabulary matvec -> logits, argmax partials).
// Each phase of each step is a grid-wide dependency: its CTAs start once every
// CTA finished the previous phase (monotonic per-phase counters).  Weights never
// depend on activations, so every CTA streams its weight tiles into a
// shared-memory ring with TMA bulk copies, across phase and step boundaries,
// while its warps wait on dependencies.
#pragma once
#include <cstdint>

namespace tir {

// ---- launch geometry --------------------------------------------------------
constexpr int kWarps = 12;
constexpr int kThreads = kWarps * 32;            // one CTA of 12 warps per SM
constexpr int kTileMult = 2;                     // tile rows = row lanes x 2
constexpr int kChunkBytes = kTileMult * 32 * 34; // one warp's slice of a tile: 2 rows x 32 blocks
constexpr int kWarpSlots = 7;                    // per-warp ring depth (183 KB in flight per SM)
constexpr int kMaxK = 6144;                      // longest matvec row (columns)
constexpr int kMaxPhases = 128;                  // phases per step (5 per layer + 1)
constexpr int kHeadDim = 64;                     // attention head size supported
constexpr int kAttnChunk = 32;                   // positions per attention chunk
constexpr int kAttnHeadsPerPass = kWarps;
static_assert(kMaxK / 16 == kThreads, "input staging gives every thread one 16-column chunk");

enum PhaseKind : int32_t { PH_GEMV = 0, PH_ATTN = 1 };
// IN_ATTN: the attention output, merged from the per-split partial softmaxes
// by the reader when there are at most kReaderCombineMaxSplits splits.
enum InKind : int32_t { IN_RAW = 0, IN_X_NORM = 1, IN_X0_NORM = 2, IN_ATTN = 3 };
constexpr int kReaderCombineMaxSplits = 4;
constexpr int kAttnRec = 68;     // floats per split record: max, sum, 2 pad, o[64]
constexpr int kTraceFields = 8;  // per (phase, CTA): 4 stamps, data wait, tiles, dep wait, pad
enum EpiKind : int32_t { EPI_STORE = 0, EPI_QKV = 1, EPI_RESID = 2, EPI_GU = 3, EPI_LOGITS = 4 };

// Scale row stride (f16 elements) of the split Q8_0 layout: 16-byte rows.
__host__ __device__ constexpr int64_t scale_stride(int64_t k) { return ((k / 32) + 7) / 8 * 8; }

// GEMV geometry for rows of k columns (k / 32 Q8_0 blocks): a "row lane" of
// gemv_wpr(k) warps covers one row, lane j of the group owning column block j;
// the CTA's kWarps warps form gemv_row_lanes(k) row lanes, and a weight tile
// holds row_lanes x kTileMult rows: row lane rl takes tile rows rl and
// rl + row_lanes, so every thread handles kTileMult (row, block) units of
// every tile with the same column block.
__host__ __device__ constexpr int gemv_wpr(int64_t k) { return static_cast<int>((k / 32 + 31) / 32); }
__host__ __device__ constexpr int gemv_row_lanes(int64_t k) { return kWarps / gemv_wpr(k); }
__host__ __device__ constexpr int gemv_tile_rows(int64_t k) { return gemv_row_lanes(k) * kTileMult; }

// Warp-sliced tile-major Q8_0 layout (the layout the decode kernel streams).
// Tile t holds rows [t R, t R + R), R = gemv_tile_rows(k), the last tile
// padded with zero rows.  Inside a tile, the slice of warp (row lane rl,
// column warp wi) -- tile rows rl + row_lanes j (j < kTileMult), column
// blocks [32 wi, 32 wi + nbw) -- is one contiguous chunk: the rows' quants
// (kTileMult x nbw x 32 int8), then their f16 scales (kTileMult x nbwp,
// nbwp = nbw rounded up to 8).  Chunks follow in (rl, wi) order, so each
// warp streams its own slice of every tile with 16-byte copies.
__host__ __device__ constexpr int q8_slice_blocks(int64_t k, int wi) {
    return static_cast<int>((k / 32 - 32 * wi) < 32 ? (k / 32 - 32 * wi) : 32);
}
__host__ __device__ constexpr int64_t q8_slice_bytes(int64_t k, int wi) {
    return kTileMult * (q8_slice_blocks(k, wi) * 32 + ((q8_slice_blocks(k, wi) + 7) / 8 * 8) * 2);
}
__host__ __device__ constexpr int64_t q8_lane_bytes(int64_t k) {
    return (gemv_wpr(k) - 1) * q8_slice_bytes(k, 0) + q8_slice_bytes(k, gemv_wpr(k) - 1);
}
__host__ __device__ constexpr int64_t q8_tile_bytes(int64_t k) { return gemv_row_lanes(k) * q8_lane_bytes(k); }
__host__ __device__ constexpr int64_t q8_slice_offset(int64_t k, int64_t t, int rl, int wi) {
    return t * q8_tile_bytes(k) + rl * q8_lane_bytes(k) + wi * q8_slice_bytes(k, 0);
}
__host__ __device__ constexpr int64_t q8_tiled_matrix_bytes(int64_t n, int64_t k) {
    return (n + gemv_tile_rows(k) - 1) / gemv_tile_rows(k) * q8_tile_bytes(k);
}

struct PhaseDesc {
    int32_t kind, layer, in_kind, epi;
    int32_t n, k, sk;          // rows, columns, scale stride (halves)
    int32_t rows_per_tile, n_tiles;  // rows_per_tile = gemv_tile_rows(k)
    int32_t dump;              // EPI_RESID: also write the residual to the dump
    int32_t tiled;             // 1: wq is warp-sliced tile-major (q8_slice_offset), ws unused
    int32_t qact;              // 1: Mode::Quantize input -- activated_q8 blocks, integer block dots
    const uint8_t* wq;         // quants [n][k] signed int8 q (split layout), or the tiled matrix
    const uint16_t* ws;        // f16 scales [n][sk] (split layout)
    const float* in;           // IN_RAW input / IN_X_NORM residual buffer
    const float* norm_w;       // rmsnorm weights (IN_*_NORM)
    float* out;                // epilogue target
    float* kc;                 // EPI_QKV: key cache of this layer [kv][max_ctx][64]
    float* vc;                 // EPI_QKV: value cache of this layer
};

struct DecodeParams {
    const PhaseDesc* phases;   // device array; NULL -> use `single`
    PhaseDesc single;
    int32_t n_phases;
    int32_t n_steps, pos0;
    int32_t H, q_heads, kv_heads, group, kvd, max_ctx, vocab, max_splits;
    int32_t qact;              // some phase runs Mode::Quantize (PhaseDesc.qact): that kernel instantiation
    // token source of each step (IN_X0_NORM): x0 (step 0 only, optional),
    // else prompt[f] for f < n_prompt, else argmax of the previous logits.
    const float* x0;
    const int32_t* prompt;
    int32_t n_prompt;
    int32_t* out_ids;          // sampled ids of steps >= n_prompt
    const uint8_t* embd_q;     // token_embd, split layout
    const uint16_t* embd_s;
    int32_t embd_sk;
    float rms_eps;
    // state buffers
    float* x;                  // residual stream [H]
    float* dump;               // optional [(layers+1)][H]
    uint8_t* qdump;            // optional, Mode::Quantize: [(2 layers + 1)][H / 32] Q8_0 blocks of the quantised inputs
    int32_t n_layers;
    const float* rope_cos;     // [max_ctx][32]
    const float* rope_sin;
    float* attn_part;          // [kv][max_splits][group][kAttnRec]
    uint32_t* attn_cnt;        // [layers][kv]
    float* attn_out;           // [H]
    const float* q;            // [H] (written by EPI_QKV)
    uint32_t* counters;        // [n_phases]
    unsigned long long* argmax_part;  // [grid]
    uint32_t* error;           // [0] code, [1] phase, [2] step, [3] code again (sticky, read by the host);
                               // single matvec (phases == nullptr): [4] exit count, zero between launches
    unsigned long long timeout_ns;
    int32_t hold_phase;        // tests only: this phase's dependency is never met (-1: none)
    // Phase timeline of step `trace_step` (globaltimer ns), NULL when off:
    // trace[(phase * grid + cta) * kTraceFields + {0 start, 1 inputs ready,
    // 2 staged, 3 released, 4 ns waiting for ring data, 5 tiles, 6 ns waiting
    // for the previous phase}]
    unsigned long long* trace;
    int32_t trace_step;
};

// Host launchers (decode.cu).
int decode_launch(const DecodeParams& p, int grid, void* stream, bool cooperative);
int decode_grid_size(int device);
int decode_smem_bytes();
int decode_blocks_per_sm();

}  // namespace tir
