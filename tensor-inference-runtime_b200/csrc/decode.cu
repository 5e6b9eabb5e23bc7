// decode.cu -- persistent sm_100a kernel running a whole forward program
// (runtime.h): the batch-1 decode loop of src/forward.rs:13-258 /
// src/lib.rs:239-314, or a single Q8_0 matvec (src/math.rs:87-98).
//
// One CTA of 12 warps per SM (cooperative launch: all CTAs co-resident).
//
// Weight stream.  Each CTA's weight tiles, in schedule order over every GEMV
// phase of every step, are streamed warp by warp: the HBM layout keeps each
// warp's slice of a tile contiguous (runtime.h q8_slice_offset), and every
// warp copies its own slices with 16-byte cp.async into a private
// kWarpSlots-deep shared-memory ring, kWarpSlots tiles ahead of the tile it is
// computing.  No warp waits for another to free a slot, and no copy engine
// serialises small copies.  Weights never wait for activations, so HBM keeps
// streaming across phase boundaries while the warps wait on dependencies.
//
// Phases.  Every CTA waits (bounded) until all CTAs released the previous
// phase, stages the phase input once (rmsnorm fused) as per-block fixed-point
// digits, then all warps work through the CTA's tiles together: thread (row
// lane, column block b) owns block b of every row its row lane covers, keeps
// block b of the input in registers for the whole phase, and leaves one
// partial dot per (row, block); batches of up to 8 tiles are reduced with
// shuffles and one CTA barrier, and the fused epilogue (RoPE + KV append,
// residual, SiLU*up, logits + argmax) runs one thread per row.
//
// Arithmetic.  Weights stay signed int8.  The input of each 32-column block is
// encoded as integers q_i = round(x_i * 2^(22-E)), 2^E > max |x_i| of the
// block, split into three signed base-256 digits (q = d0 + 256 d1 + 65536 d2),
// so a block dot is three exact integer dp4a chains; the block's f16 weight
// scale and 2^(E-22) are applied in f32.  The relative error of a row dot is
// that of f32 accumulation (the fixed point keeps 22 bits below the block
// maximum), well inside the path's f32 tolerance.
//
// Every wait is bounded by DecodeParams::timeout_ns (globaltimer); on expiry the
// kernel records TIR_ERR_TIMEOUT, every CTA leaves at its next phase boundary,
// and thread 0 waits (bounded) for the copies still in flight before exiting.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstddef>
#include <cstdint>

#include "ptx.cuh"
#include "runtime.h"

namespace tir {

constexpr uint32_t kErrTimeout = 25;   // TIR_ERR_TIMEOUT
constexpr uint32_t kErrBadToken = 12;  // TIR_ERR_BAD_TOKEN
constexpr uint32_t FULL = 0xffffffffu;
constexpr uint32_t kBarAll = 1;  // named barrier id for the CTA's warps

// Where the weight stream reads a phase's tiles (cached in shared memory so
// refills need no global loads).
struct TileSrc {
    const uint8_t* wq;
    const uint16_t* ws;
    int32_t k, sk, n, rows, tiled;
};

struct AttnBufs {
    float aq[kAttnHeadsPerPass][kHeadDim];
    float akv[2][kAttnChunk][kHeadDim];  // K and V rows of one chunk (TMA target)
};

// Staged GEMV input: per 32-column block, three words-of-digits planes (word j
// of a plane holds the digit of columns 4j..4j+3) and the block's 2^(E-22);
// before encoding, the merged attention output of an IN_ATTN phase passes
// through xf (same storage, separated by a CTA barrier).
struct StageBufs {
    union {
        float xf[kMaxK];
        struct {
            uint32_t xd[3][kMaxK / 32][8];
            float xsc[kMaxK / 32];
        };
    };
};

struct __align__(128) Smem {
    uint8_t ring[kWarps][kWarpSlots][kChunkBytes];  // per-warp weight slices (cp.async targets)
    union {
        StageBufs st;
        AttnBufs attn;
    } u;
    uint64_t abar;  // attention K/V copies
    TileSrc src[kMaxPhases];
    float part[2][kWarps][8];  // per-warp row partials of a tile batch (double buffered)
    unsigned long long best[kWarps];
    float red[kWarps];
    int16_t nmine[kMaxPhases], tfirst[kMaxPhases];
    int32_t token, phase_ok, abort_flag, attn_last, ok0;
};

// TMA bulk-copy destinations must start on 16-byte boundaries.
static_assert(offsetof(Smem, ring) % 128 == 0 && kChunkBytes % 16 == 0, "ring slots must be 16-byte aligned");
static_assert((offsetof(Smem, u) + offsetof(AttnBufs, akv)) % 16 == 0, "akv must be 16-byte aligned");
static_assert(offsetof(Smem, u) % 16 == 0, "staged digits are read as 16-byte vectors");
static_assert(offsetof(Smem, abar) % 8 == 0, "mbarriers need 8-byte alignment");
static_assert(sizeof(Smem) <= 227 * 1024, "shared memory budget");

__device__ __forceinline__ const PhaseDesc& phase_at(const DecodeParams& p, int i) {
    return p.phases ? p.phases[i] : p.single;
}

__device__ __forceinline__ void cbar() { named_bar(kBarAll, kThreads); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL, v, o));
    return v;
}

// Key whose unsigned order is the IEEE total order (f32::total_cmp).
__device__ __forceinline__ uint32_t total_key(float v) {
    uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ unsigned long long pack_best(float v, int idx) {
    return (static_cast<unsigned long long>(total_key(v)) << 32) | static_cast<uint32_t>(idx);
}

// error[0..2]: the launch's first failure (code, phase, step), which makes
// every other wait give up; error[3]: the same code, left set for the host to
// collect (the launcher clears only words 0..2 before a launch).
__device__ __forceinline__ void set_error(const DecodeParams& p, uint32_t code, int ph, int f) {
    if (atomicCAS(p.error, 0u, code) == 0u) {
        p.error[1] = static_cast<uint32_t>(ph);
        p.error[2] = static_cast<uint32_t>(f);
        p.error[3] = code;
    }
}

__device__ __forceinline__ bool any_error(const DecodeParams& p) { return ld_relaxed_gpu(p.error) != 0u; }

// Bounded wait for a grid-wide phase counter (one thread).
__device__ __forceinline__ bool wait_counter(const DecodeParams& p, const uint32_t* ctr, uint32_t target, int ph,
                                             int f) {
    if (ld_acquire_gpu(ctr) >= target) return true;
    const uint64_t t0 = globaltimer_ns();
    for (;;) {
        if (ld_acquire_gpu(ctr) >= target) return true;
        if (any_error(p)) return false;
        if (globaltimer_ns() - t0 > p.timeout_ns) {
            set_error(p, kErrTimeout, ph, f);
            return false;
        }
        __nanosleep(32);
    }
}

// Bounded wait for an mbarrier phase (one thread).
__device__ __forceinline__ bool wait_mbar(const DecodeParams& p, uint64_t* bar, uint32_t parity, int ph, int f) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++n & 15u) == 0u) {
            if (any_error(p)) return false;
            if (globaltimer_ns() - t0 > p.timeout_ns) {
                set_error(p, kErrTimeout, ph, f);
                return false;
            }
        }
    }
    return true;
}

__device__ __forceinline__ void trace_mark(const DecodeParams& p, int ph, int f, int j) {
    if (p.trace && f == p.trace_step && threadIdx.x == 0)
        p.trace[(static_cast<size_t>(ph) * gridDim.x + blockIdx.x) * kTraceFields + j] = globaltimer_ns();
}

// ---------------------------------------------------------------------------
// weight stream
// ---------------------------------------------------------------------------

// Thread 0, at kernel start: this CTA's share of every phase (tile t of a
// phase belongs to CTA (t + rot) % G, rot continuing round-robin over the
// step's GEMV phases) and where its tiles are read from.
__device__ void build_schedule(const DecodeParams& p, Smem& s) {
    const int G = gridDim.x;
    int rot = 0;
    for (int ph = 0; ph < p.n_phases; ++ph) {
        const PhaseDesc& d = phase_at(p, ph);
        if (d.kind != PH_GEMV) {
            s.nmine[ph] = 0;
            s.tfirst[ph] = 0;
            continue;
        }
        const int t0 = (static_cast<int>(blockIdx.x) - rot + G) % G;
        s.tfirst[ph] = static_cast<int16_t>(t0);
        s.nmine[ph] = static_cast<int16_t>(t0 < d.n_tiles ? (d.n_tiles - 1 - t0) / G + 1 : 0);
        s.src[ph] = TileSrc{d.wq, d.ws, d.k, d.sk, d.n, d.rows_per_tile, d.tiled};
        rot = (rot + d.n_tiles) % G;
    }
}

// Position in the tile schedule: step, phase, ordinal within the phase.
struct Pos {
    int f, ph, k;
};

// Moves n tiles forward; false past the last tile.
__device__ __forceinline__ bool pos_advance(const DecodeParams& p, const Smem& s, Pos& c, int n) {
    c.k += n;
    while (c.k >= s.nmine[c.ph]) {
        c.k -= s.nmine[c.ph];
        if (++c.ph == p.n_phases) {
            c.ph = 0;
            if (++c.f >= p.n_steps) return false;
        }
    }
    return true;
}

// The warp's position in the CTA's tile schedule for its next copy, with the
// copy geometry of that position's phase cached (recomputed only when the
// cursor enters another phase): for the tile-major layout, the warp's slice in
// the CTA's first tile of the phase and the stride to its next tile.
struct Stream {
    Pos c;
    bool more;
    int bound_ph;           // phase the cache below describes (-1: none)
    const uint8_t* src0;    // tile-major: slice of tile tfirst
    long long stride;       // tile-major: bytes between the CTA's tiles
    int pieces;             // 16-byte pieces of the warp's slice (0: no slice)
};

__device__ __forceinline__ void stream_bind(const Smem& s, Stream& st, int warp) {
    const TileSrc& t = s.src[st.c.ph];
    const int wpr = gemv_wpr(t.k), RL = kWarps / wpr;
    const int rl = warp / wpr, wi = warp % wpr;
    st.bound_ph = st.c.ph;
    st.pieces = 0;
    if (rl < RL) {
        const int nbw = q8_slice_blocks(t.k, wi), nbwp = (nbw + 7) / 8 * 8;
        st.pieces = kTileMult * (nbw * 2 + nbwp / 8);
        if (t.tiled) {
            st.src0 = t.wq + q8_slice_offset(t.k, s.tfirst[st.c.ph], rl, wi);
            st.stride = static_cast<long long>(gridDim.x) * q8_tile_bytes(t.k);
        }
    }
}

// Warp `warp` copies its slice of schedule tile i (position st.c, when
// st.more) into its slot i % kWarpSlots with 16-byte cp.async (lane-strided,
// coalesced) and commits one group -- an empty one past the schedule's end or
// when the warp has no slice in that phase, so every thread's group count
// stays in step with the tiles.  Slot layout: the slice's quants
// (kTileMult rows x nbw blocks x 32 bytes), then its scales (kTileMult x nbwp
// f16), for the tile-major and the split source layouts alike.
__device__ __forceinline__ void issue_chunk(Smem& s, Stream& st, uint32_t i, int warp, int lane) {
    if (st.more) {
        if (st.bound_ph != st.c.ph) stream_bind(s, st, warp);
        const TileSrc& t = s.src[st.c.ph];
        uint8_t* dst = s.ring[warp][i % kWarpSlots];
        if (t.tiled) {
            const uint8_t* src = st.src0 + st.c.k * st.stride;
            for (int pc = lane; pc < st.pieces; pc += 32) cp_async16(dst + 16 * pc, src + 16 * pc);
        } else if (st.pieces > 0) {  // split layout (single-matrix launches)
            const int wpr = gemv_wpr(t.k), RL = kWarps / wpr;
            const int rl = warp / wpr, wi = warp % wpr;
            const int ti = s.tfirst[st.c.ph] + st.c.k * static_cast<int>(gridDim.x);
            const int nbw = q8_slice_blocks(t.k, wi), nbwp = (nbw + 7) / 8 * 8;
            const int qpr = nbw * 2, spr = nbwp / 8;  // 16-byte pieces per row
            const uint8_t* ws = reinterpret_cast<const uint8_t*>(t.ws);
            for (int pc = lane; pc < st.pieces; pc += 32) {
                const bool quant = pc < kTileMult * qpr;
                const int pp = quant ? pc : pc - kTileMult * qpr;
                const int per = quant ? qpr : spr;
                const int j = pp / per, q = pp % per;
                const int row = ti * t.rows + rl + RL * j;
                if (row < t.n) {
                    const uint8_t* src = quant ? t.wq + static_cast<size_t>(row) * t.k + 1024 * wi + 16 * q
                                               : ws + static_cast<size_t>(row) * t.sk * 2 + 64 * wi + 16 * q;
                    cp_async16(dst + 16 * pc, src);
                }
            }
        }
    }
    cp_async_commit();
}

// Issues the warp's next copy and moves its cursor one tile on.
__device__ __forceinline__ void stream_next(const DecodeParams& p, Smem& s, Stream& st, uint32_t i, int warp,
                                            int lane) {
    issue_chunk(s, st, i, warp, lane);
    if (st.more) st.more = pos_advance(p, s, st.c, 1);
}

// ---------------------------------------------------------------------------
// GEMV phases
// ---------------------------------------------------------------------------

// One thread's 32-column input block for a phase: digit planes of the half it
// reads first (columns 16 fh .. 16 fh + 15) and second, and 2^(E-22).  The
// half order fh = (b >> 2) & 1 spreads a warp's 16-byte shared-memory reads
// of consecutive 32-byte blocks over all banks.
struct XBlock {
    uint32_t a[3][4], b[3][4];
    float sc;
};

__device__ __forceinline__ void load_xblock(const Smem& s, int b, int fh, XBlock& x) {
#pragma unroll
    for (int d = 0; d < 3; ++d) {
        const uint4 u = *reinterpret_cast<const uint4*>(&s.u.st.xd[d][b][4 * fh]);
        const uint4 v = *reinterpret_cast<const uint4*>(&s.u.st.xd[d][b][4 * (fh ^ 1)]);
        x.a[d][0] = u.x; x.a[d][1] = u.y; x.a[d][2] = u.z; x.a[d][3] = u.w;
        x.b[d][0] = v.x; x.b[d][1] = v.y; x.b[d][2] = v.z; x.b[d][3] = v.w;
    }
    x.sc = s.u.st.xsc[b];
}

// Dot of one 32-weight block (signed int8, `q` = its first byte in shared
// memory, `scale` its f16 scale) with the thread's input block:
// sum_i q_i x_i = scale * 2^(E-22) * (S0 + 256 S1 + 65536 S2), S_d the exact
// integer dot of the weights with digit plane d (|S_d| < 2^19).
__device__ __forceinline__ float unit_dot(const uint8_t* q, uint16_t scale, const XBlock& x, int fh) {
    const uint4 wa = *reinterpret_cast<const uint4*>(q + 16 * fh);
    const uint4 wb = *reinterpret_cast<const uint4*>(q + 16 * (fh ^ 1));
    const int A[4] = {static_cast<int>(wa.x), static_cast<int>(wa.y), static_cast<int>(wa.z), static_cast<int>(wa.w)};
    const int B[4] = {static_cast<int>(wb.x), static_cast<int>(wb.y), static_cast<int>(wb.z), static_cast<int>(wb.w)};
    int sa[3] = {0, 0, 0}, sb[3] = {0, 0, 0};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int d = 0; d < 3; ++d) {
            sa[d] = __dp4a(A[j], static_cast<int>(x.a[d][j]), sa[d]);
            sb[d] = __dp4a(B[j], static_cast<int>(x.b[d][j]), sb[d]);
        }
    }
    const int s0 = sa[0] + sb[0], s1 = sa[1] + sb[1], s2 = sa[2] + sb[2];
    const float v = fmaf(static_cast<float>(s2), 65536.0f, static_cast<float>(s1 * 256 + s0));
    return v * (__half2float(__ushort_as_half(scale)) * x.sc);
}

struct StepCtx {
    int f, pos, token;
    bool x0_given;
    int S;  // attention splits of this step
};

// Attention splits for a context of n_ctx positions: one per kAttnChunk
// positions, at most max_splits (one CTA each).
__device__ __forceinline__ int attn_splits(const DecodeParams& p, int n_ctx) {
    const int S = (n_ctx + kAttnChunk - 1) / kAttnChunk;
    return max(1, min(S, p.max_splits));
}

// Sixteen consecutive input elements [k0, k0 + 16) (k0 % 16 == 0) in one
// round trip: the step input x0 (explicit vector, or the embedding row of the
// step's token, src/tokenizer.rs:10-32: f32(q) * f32(scale), exact) or the
// phase's input buffer.  Data written by other CTAs is read from L2 (never a
// stale L1 line).
__device__ __forceinline__ void load16(const DecodeParams& p, const PhaseDesc& d, const StepCtx& st, int k0,
                                       float* v) {
    if (d.in_kind == IN_X0_NORM && !st.x0_given) {
        const size_t row = static_cast<size_t>(st.token);
        const uint4 q = __ldg(reinterpret_cast<const uint4*>(p.embd_q + row * p.H + k0));
        const float sc = __half2float(__ushort_as_half(__ldg(p.embd_s + row * p.embd_sk + k0 / 32)));
        const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
            for (int b = 0; b < 4; ++b)
                v[4 * j + b] = __fmul_rn(static_cast<float>(static_cast<int8_t>((w[j] >> (8 * b)) & 0xffu)), sc);
    } else {
        const float* src = d.in_kind == IN_X0_NORM ? p.x0 : d.in;
        const float4* s4 = reinterpret_cast<const float4*>(src + k0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 t = __ldcg(s4 + j);
            v[4 * j] = t.x;
            v[4 * j + 1] = t.y;
            v[4 * j + 2] = t.z;
            v[4 * j + 3] = t.w;
        }
    }
}

// Eight attention-output elements [k0, k0 + 8) of head h = k0 / 64, merged
// from the S <= kReaderCombineMaxSplits per-split partial softmaxes the
// attention phase left (max m_j, sum l_j, unnormalised o_j): one round trip.
__device__ __forceinline__ void merge8(const DecodeParams& p, const StepCtx& st, int k0, float* v) {
    const int h = k0 / kHeadDim, d0 = k0 % kHeadDim;
    const int g = h / p.group, hh = h % p.group;
    float2 ml[kReaderCombineMaxSplits];
    float4 o[kReaderCombineMaxSplits][2];
#pragma unroll
    for (int j = 0; j < kReaderCombineMaxSplits; ++j) {
        if (j < st.S) {
            const float* rec = p.attn_part + ((static_cast<size_t>(g) * p.max_splits + j) * p.group + hh) * kAttnRec;
            ml[j] = __ldcg(reinterpret_cast<const float2*>(rec));
            o[j][0] = __ldcg(reinterpret_cast<const float4*>(rec + 4 + d0));
            o[j][1] = __ldcg(reinterpret_cast<const float4*>(rec + 4 + d0) + 1);
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < kReaderCombineMaxSplits; ++j)
        if (j < st.S) M = fmaxf(M, ml[j].x);
    float L = 0.f, acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.f;
#pragma unroll
    for (int j = 0; j < kReaderCombineMaxSplits; ++j) {
        if (j < st.S) {
            const float w = expf(ml[j].x - M);
            L = fmaf(ml[j].y, w, L);
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                acc[4 * q] = fmaf(o[j][q].x, w, acc[4 * q]);
                acc[4 * q + 1] = fmaf(o[j][q].y, w, acc[4 * q + 1]);
                acc[4 * q + 2] = fmaf(o[j][q].z, w, acc[4 * q + 2]);
                acc[4 * q + 3] = fmaf(o[j][q].w, w, acc[4 * q + 3]);
            }
        }
    }
    const float inv = 1.0f / L;
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = acc[i] * inv;
}

// Operands of a phase that do not depend on the previous phase, loaded before
// the dependency wait so their latency hides behind it: the rmsnorm weights of
// this thread's 16-column chunk and the position's RoPE cos/sin (lane i holds
// pair i).
struct Prefetch {
    float wr[16];
    float rc, rs;
};

__device__ __forceinline__ void prefetch_operands(const DecodeParams& p, const PhaseDesc& d, const StepCtx& st,
                                                  Prefetch& pf) {
    const int tid = threadIdx.x, lane = tid & 31;
    const bool norm = d.in_kind == IN_X_NORM || d.in_kind == IN_X0_NORM;
    const int k0 = tid * 16;
    if (norm && k0 < d.k) {
        const float4* w4 = reinterpret_cast<const float4*>(d.norm_w + k0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 t = __ldg(w4 + j);
            pf.wr[4 * j] = t.x;
            pf.wr[4 * j + 1] = t.y;
            pf.wr[4 * j + 2] = t.z;
            pf.wr[4 * j + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) pf.wr[i] = 1.0f;
    }
    pf.rc = 0.f;
    pf.rs = 0.f;
    if (d.epi == EPI_QKV) {
        pf.rc = __ldg(p.rope_cos + static_cast<size_t>(st.pos) * (kHeadDim / 2) + lane);
        pf.rs = __ldg(p.rope_sin + static_cast<size_t>(st.pos) * (kHeadDim / 2) + lane);
    }
}

// Four encoded values u (bytes 0..2 = digits + 128) -> the three digit words
// (byte e of word d = digit d of value e, as signed int8).
__device__ __forceinline__ void pack_digits(const uint32_t* u, uint32_t& w0, uint32_t& w1, uint32_t& w2) {
    const uint32_t p01 = __byte_perm(u[0], u[1], 0x5140), p23 = __byte_perm(u[2], u[3], 0x5140);
    const uint32_t q01 = __byte_perm(u[0], u[1], 0x0062), q23 = __byte_perm(u[2], u[3], 0x0062);
    w0 = __byte_perm(p01, p23, 0x5410) ^ 0x80808080u;
    w1 = __byte_perm(p01, p23, 0x7632) ^ 0x80808080u;
    w2 = __byte_perm(q01, q23, 0x5410) ^ 0x80808080u;
}

// Stages the phase input for the GEMV threads.  Thread t loads columns
// [16t, 16t + 16) (one round trip of loads), applies rmsnorm for IN_*_NORM
// phases (src/math.rs:141-150: x*w / sqrt(sum(x^2)/n + eps), the division as
// a multiplication by the correctly rounded reciprocal), and encodes its half
// of the 32-column block as fixed point: with m = max |value| of the block
// (the two halves sit in lanes t, t^1) and E = the exponent with
// 2^(E-1) <= m < 2^E, q = round(value * 2^(22-E)) so |q| <= 2^22;
// fma(value, 2^(22-E), 1.5 * 2^23) has q in its low mantissa bits, and adding
// 0x408080 leaves u = q + 0x808080 in bytes 0..2, i.e. digit + 128 per byte
// (q = d0 + 256 d1 + 65536 d2, |d2| <= 64).  Blocks with m < 2^-86 use E = -86.
// For the step input, one of the phase's CTAs also stores each chunk as the
// residual stream x (and dump row 0).
__device__ __forceinline__ void stage_load(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                                           const Prefetch& pf, float* v, float& inv, float& rms, int ph) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = d.k, nchunks = K / 16;
    const bool norm = d.in_kind == IN_X_NORM || d.in_kind == IN_X0_NORM;
    const int c = tid;
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = 0.f;
    if (d.in_kind == IN_ATTN && st.S <= kReaderCombineMaxSplits) {
        // merge the attention splits 8 columns per thread, then regroup
        for (int c8 = tid; c8 < K / 8; c8 += kThreads) {
            float m[8];
            merge8(p, st, c8 * 8, m);
            float4* xf4 = reinterpret_cast<float4*>(s.u.st.xf + c8 * 8);
            xf4[0] = make_float4(m[0], m[1], m[2], m[3]);
            xf4[1] = make_float4(m[4], m[5], m[6], m[7]);
        }
        cbar();
        if (c < nchunks) {
            const float4* xf4 = reinterpret_cast<const float4*>(s.u.st.xf + c * 16);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float4 t = xf4[q];
                v[4 * q] = t.x;
                v[4 * q + 1] = t.y;
                v[4 * q + 2] = t.z;
                v[4 * q + 3] = t.w;
            }
        }
        cbar();  // xf is read before the digits (same storage) are written
    } else if (c < nchunks) {
        load16(p, d, st, c * 16, v);
    }
    // chunk c is stored by one of the phase's CTAs with tiles (only they
    // stage), told apart by their first tile
    if (d.in_kind == IN_X0_NORM && c < nchunks && c % min(d.n_tiles, static_cast<int>(gridDim.x)) == s.tfirst[ph]) {
        float4* x4 = reinterpret_cast<float4*>(p.x + c * 16);
        float4* d4 = p.dump ? reinterpret_cast<float4*>(p.dump + c * 16) : nullptr;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float4 t = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            x4[j] = t;
            if (d4) d4[j] = t;
        }
    }
    inv = 1.0f;
    rms = 1.0f;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < 16; ++i) ss = fmaf(v[i], v[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s.red[warp] = ss;
        cbar();
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += s.red[w];
        rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), p.rms_eps));
        inv = __frcp_rn(rms);
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = __fmul_rn(v[i], pf.wr[i]);
    }
}

__device__ __forceinline__ void stage_input(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                                            const Prefetch& pf, int ph) {
    const int c = threadIdx.x, nchunks = d.k / 16;
    float v[16], inv, rms;
    stage_load(p, s, d, st, pf, v, inv, rms, ph);
    float mx = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) mx = fmaxf(mx, fabsf(v[i]));
    mx = fmaxf(mx, __shfl_xor_sync(FULL, mx, 1));
    uint32_t ex = __float_as_uint(__fmul_rn(mx, inv)) >> 23;  // biased exponent of m
    ex = max(ex, 40u);
    const float up = __uint_as_float((275u - ex) << 23);    // 2^(22-E), E = ex - 126
    const float down = __uint_as_float((ex - 21u) << 23);   // 2^(E-22)
    const float mul = inv * up;                             // exact: power-of-two scaling
    if (c < nchunks) {
        uint32_t u[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(fmaf(v[i], mul, 12582912.0f)) + 0x408080u;
        const int b = c >> 1, h = c & 1;
        uint32_t w[3][4];
#pragma unroll
        for (int g = 0; g < 4; ++g) pack_digits(u + 4 * g, w[0][g], w[1][g], w[2][g]);
#pragma unroll
        for (int dd = 0; dd < 3; ++dd)
            *reinterpret_cast<uint4*>(&s.u.st.xd[dd][b][4 * h]) = make_uint4(w[dd][0], w[dd][1], w[dd][2], w[dd][3]);
        if (h == 0) s.u.st.xsc[b] = down;
    }
    cbar();
}

// Mode::Quantize input staging (src/forward.rs:261-275): the phase input as
// stage_load leaves it, divided by rmsnorm's r (as the reference rounds it),
// then the block's Q8_0 quantisation by activated_q8 (src/kernels.rs:8-31) --
// scale = the signed element of largest |x| (the last of equal ones) / 127,
// q = round(x / scale) half away from zero, saturated to int8, NaN -> 0 -- as
// digit plane 0 (planes 1 and 2 zero), and the f16-rounded scale the block
// dot multiplies by (dot_prod_act_q8, src/math.rs:39-50): unit_dot then yields
// the exact integer block dot times scale_a * scale_w.  Compiled only into
// the kernel instantiation for Mode::Quantize (decode_kernel<true>).
__device__ __forceinline__ void stage_input_qact(const DecodeParams& p, Smem& s, const PhaseDesc& d,
                                                 const StepCtx& st, const Prefetch& pf, int ph) {
    const int c = threadIdx.x, nchunks = d.k / 16;
    float v[16], inv, rms;
    stage_load(p, s, d, st, pf, v, inv, rms, ph);
    uint32_t babs = 0u;
    float bval = 0.f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        v[i] = __fdiv_rn(v[i], rms);
        const uint32_t a = __float_as_uint(v[i]) & 0x7fffffffu;
        if (a >= babs) {
            babs = a;
            bval = v[i];
        }
    }
    const uint32_t oabs = __shfl_xor_sync(FULL, babs, 1);
    const float oval = __shfl_xor_sync(FULL, bval, 1);
    const int h = c & 1;  // half 1 follows half 0 in the block: it wins ties
    if (h == 0 ? oabs >= babs : oabs > babs) bval = oval;
    const float scale = __fdiv_rn(bval, 127.0f);
    if (c < nchunks) {
        uint32_t w0[4];
#pragma unroll
        for (int g = 0; g < 4; ++g) {
            uint32_t word = 0u;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float r = roundf(__fdiv_rn(v[4 * g + e], scale));
                const int qi = r != r ? 0 : static_cast<int>(fminf(fmaxf(r, -128.0f), 127.0f));
                word |= (static_cast<uint32_t>(qi) & 0xffu) << (8 * e);
            }
            w0[g] = word;
        }
        const int b = c >> 1;
        *reinterpret_cast<uint4*>(&s.u.st.xd[0][b][4 * h]) = make_uint4(w0[0], w0[1], w0[2], w0[3]);
        *reinterpret_cast<uint4*>(&s.u.st.xd[1][b][4 * h]) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(&s.u.st.xd[2][b][4 * h]) = make_uint4(0u, 0u, 0u, 0u);
        if (h == 0) s.u.st.xsc[b] = __half2float(__float2half_rn(scale));
        // the dump of the quantised input (Q8_0 blocks, as activated_q8 writes
        // them), by one of the phase's CTAs: slot 2 l (q|k|v of layer l),
        // 2 l + 1 (o of layer l), 2 L (lm_head)
        if (p.qdump && s.tfirst[ph] == 0) {
            const int slot = d.layer < 0 ? 2 * p.n_layers : 2 * d.layer + (d.epi == EPI_QKV ? 0 : 1);
            uint8_t* blk = p.qdump + (static_cast<size_t>(slot) * (d.k / 32) + b) * 34;
            if (h == 0) {
                const unsigned short hs = __half_as_ushort(__float2half_rn(scale));
                blk[0] = static_cast<uint8_t>(hs & 0xffu);
                blk[1] = static_cast<uint8_t>(hs >> 8);
            }
#pragma unroll
            for (int e = 0; e < 16; ++e) blk[2 + 16 * h + e] = static_cast<uint8_t>((w0[e / 4] >> (8 * (e % 4))) & 0xffu);
        }
    }
    (void)inv;
    cbar();
}


// Sums eight per-lane values over the warp with 9 shuffles; lane l ends with
// the total of value (l >> 2) & 7.
__device__ __forceinline__ float reduce8(const float* v, int lane) {
    const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
    float t[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) t[i] = (b4 ? v[4 + i] : v[i]) + __shfl_xor_sync(FULL, b4 ? v[i] : v[4 + i], 16);
    float u[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) u[i] = (b3 ? t[2 + i] : t[i]) + __shfl_xor_sync(FULL, b3 ? t[i] : t[2 + i], 8);
    float w = (b2 ? u[1] : u[0]) + __shfl_xor_sync(FULL, b2 ? u[0] : u[1], 4);
    w += __shfl_xor_sync(FULL, w, 2);
    w += __shfl_xor_sync(FULL, w, 1);
    return w;
}

// Trace accumulators of the traced step (thread 0 only).
struct TraceAcc {
    bool on;
    unsigned long long data_wait_ns, dep_wait_ns, tiles;
};

// Fused epilogue of matrix row n (or of the pair n, n + 1 for EPI_QKV / EPI_GU,
// n even): y (y1) = the row dot(s), pre = prefetched residual (EPI_RESID),
// (c, sn) = RoPE cos/sin of the pair.
__device__ __forceinline__ void epilogue(const DecodeParams& p, const PhaseDesc& d, const StepCtx& st, int n,
                                         float y, float y1, float pre, float c, float sn,
                                         unsigned long long& best) {
    switch (d.epi) {
        case EPI_STORE:
            d.out[n] = y;
            break;
        case EPI_LOGITS:
            d.out[n] = y;
            best = max(best, pack_best(y, n));
            break;
        case EPI_RESID: {  // src/forward.rs:192, :232-236
            const float x = __fadd_rn(pre, y);
            d.out[n] = x;
            if (d.dump && p.dump) p.dump[static_cast<size_t>(d.layer + 1) * p.H + n] = x;
            break;
        }
        case EPI_GU: {  // rows (2i, 2i+1) = (gate_i, up_i); src/math.rs:171-175
            const float silu = __fdiv_rn(y, __fadd_rn(1.0f, expf(-y)));
            d.out[n >> 1] = __fmul_rn(silu, y1);
            break;
        }
        case EPI_QKV: {
            // RoPE on adjacent pairs (src/math.rs:196-228), then q or the
            // KV-cache append (src/forward.rs:71, :83-84).
            const int H = p.H, kvd = p.kvd;
            int idx = n;
            float* dst;
            bool rope = true;
            if (idx < H) {
                dst = d.out + idx;
            } else if (idx < H + kvd) {
                idx -= H;
                dst = d.kc + (static_cast<size_t>(idx / kHeadDim) * p.max_ctx + st.pos) * kHeadDim + idx % kHeadDim;
            } else {
                idx -= H + kvd;
                dst = d.vc + (static_cast<size_t>(idx / kHeadDim) * p.max_ctx + st.pos) * kHeadDim + idx % kHeadDim;
                rope = false;
            }
            float e0 = y, e1 = y1;
            if (rope) {
                e0 = __fadd_rn(__fmul_rn(c, y), __fmul_rn(-sn, y1));
                e1 = __fadd_rn(__fmul_rn(sn, y), __fmul_rn(c, y1));
            }
            dst[0] = e0;
            dst[1] = e1;
            break;
        }
        default:
            break;
    }
}

// The CTA's tiles of one GEMV phase (schedule indices gidx + k, k < nmine),
// M units per thread per tile.  Batches of 8 / M tiles: every warp waits for
// its own slices of the batch's tiles (cp.async groups), computes all their
// units, and issues the copies kWarpSlots tiles ahead into the freed slots; the per-thread
// partials are reduced over each warp (reduce8) into s.part, and after one CTA
// barrier thread e runs the epilogue of batch row e, summing the partials of
// the row lane's warps in order (deterministic).  The last batch's copies are
// left to the caller (`deferred` of them), which issues them after the phase
// is released: issuing copies occupies a warp ~1k cycles per tile, which would
// otherwise delay the release that every CTA waits for.
template <int M>
__device__ __forceinline__ bool gemv_tiles(const DecodeParams& p, Smem& s, Stream& sw, const PhaseDesc& d,
                                           const StepCtx& st, int ph, uint32_t gidx, const Prefetch& pf,
                                           TraceAcc& tr, unsigned long long& best, int& deferred) {
    static_assert(M == kTileMult, "tiles hold kTileMult rows per row lane");
    constexpr int TB = 8 / M;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = gridDim.x;
    const int K = d.k, N = d.n, R = d.rows_per_tile;
    const int wpr = gemv_wpr(K), RL = kWarps / wpr;
    const int rl = warp / wpr, wi = warp % wpr, b = wi * 32 + lane;
    const int nbw = q8_slice_blocks(K, wi), nbwp = (nbw + 7) / 8 * 8;
    const bool warp_on = rl < RL;
    const bool lane_on = warp_on && lane < nbw;
    const int fh = (b >> 2) & 1;
    const int nm = s.nmine[ph], t0 = s.tfirst[ph];
    const bool pairs = d.epi == EPI_QKV || d.epi == EPI_GU;
    XBlock x;
    if (lane_on) load_xblock(s, b, fh, x);
    int buf = 0;
    for (int k0 = 0; k0 < nm; k0 += TB) {
        const int nt = min(TB, nm - k0);
        // this thread's epilogue row of the batch, and its residual operand
        const int eti = tid / R, er = tid - eti * R;
        const int en = (t0 + (k0 + eti) * G) * R + er;
        const bool e_on = tid < nt * R && en < N && (!pairs || (er & 1) == 0);
        float pre = 0.f;
        if (d.epi == EPI_RESID && e_on) pre = __ldcg(d.out + en);
        float t[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = 0.f;
        // 1. this warp's slices of the batch's tiles have landed (each thread
        //    waits for its own copies, the warp sync publishes the others')
        {
            const uint64_t w0 = tr.on ? globaltimer_ns() : 0;
            static_assert(TB <= kWarpSlots && TB <= 4, "batch waits below");
            switch (nt) {
                case 1: cp_async_wait<kWarpSlots - 1>(); break;
                case 2: cp_async_wait<kWarpSlots - 2>(); break;
                case 3: cp_async_wait<kWarpSlots - 3>(); break;
                default: cp_async_wait<kWarpSlots - 4>(); break;
            }
            if (tr.on) tr.data_wait_ns += globaltimer_ns() - w0;
        }
        __syncwarp();
        // 2. every unit of the batch: independent dot chains
        if (lane_on) {
#pragma unroll
            for (int ti = 0; ti < TB; ++ti) {
                if (ti < nt) {
                    const uint32_t i = gidx + static_cast<uint32_t>(k0 + ti);
                    const int r0 = (t0 + (k0 + ti) * G) * R;
                    const int rows = min(R, N - r0);
                    const uint8_t* ch = s.ring[warp][i % kWarpSlots];
                    const uint16_t* cs = reinterpret_cast<const uint16_t*>(ch + M * nbw * 32);
#pragma unroll
                    for (int j = 0; j < M; ++j) {
                        const int r = rl + RL * j;
                        if (r < rows) t[ti * M + j] = unit_dot(ch + (j * nbw + lane) * 32, cs[j * nbwp + lane], x, fh);
                    }
                }
            }
        }
        __syncwarp();  // the batch's slots are free
        // 3. refill them, kWarpSlots tiles ahead (the last batch's: after the release)
        if (k0 + TB < nm) {
            for (int ti = 0; ti < nt; ++ti)
                stream_next(p, s, sw, gidx + static_cast<uint32_t>(k0 + ti + kWarpSlots), warp, lane);
        } else {
            deferred = nt;
        }
        if (tr.on) tr.tiles += static_cast<unsigned long long>(nt);
        const float y8 = reduce8(t, lane);
        if (warp_on && (lane & 3) == 0) s.part[buf][warp][lane >> 2] = y8;
        // RoPE cos/sin of the epilogue pair (whole warps take part in the shuffles)
        float c = 0.f, sn = 0.f;
        if (d.epi == EPI_QKV) {
            const int pair = (en % kHeadDim) >> 1;
            c = __shfl_sync(FULL, pf.rc, pair & 31);
            sn = __shfl_sync(FULL, pf.rs, pair & 31);
        }
        cbar();
        if (e_on) {
            const int erl = er % RL, v = eti * M + er / RL;
            float y = 0.f, y1 = 0.f;
            for (int w = 0; w < wpr; ++w) y += s.part[buf][erl * wpr + w][v];
            if (pairs) {
                const int erl1 = (er + 1) % RL, v1 = eti * M + (er + 1) / RL;
                for (int w = 0; w < wpr; ++w) y1 += s.part[buf][erl1 * wpr + w][v1];
            }
            epilogue(p, d, st, en, y, y1, pre, c, sn, best);
        }
        buf ^= 1;
    }
    return true;
}

// One GEMV phase; returns false on timeout (this CTA then stops at the end
// of the phase, together with its other warps).
template <bool QACT>
__device__ __forceinline__ bool gemv_phase(const DecodeParams& p, Smem& s, Stream& sw, const PhaseDesc& d,
                                           const StepCtx& st, int ph, uint32_t gidx, const Prefetch& pf,
                                           TraceAcc& tr, int& deferred) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nm = s.nmine[ph];
    if (nm == 0) {
        if (d.epi == EPI_LOGITS && tid == 0) p.argmax_part[blockIdx.x] = 0ull;
        return true;
    }
    if (QACT && d.qact)
        stage_input_qact(p, s, d, st, pf, ph);
    else
        stage_input(p, s, d, st, pf, ph);
    trace_mark(p, ph, st.f, 2);
    unsigned long long best = 0ull;
    bool ok;
    ok = gemv_tiles<kTileMult>(p, s, sw, d, st, ph, gidx, pf, tr, best, deferred);
    if (d.epi == EPI_LOGITS) {
#pragma unroll
        for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(FULL, best, o));
        if (lane == 0) s.best[warp] = best;
    }
    return ok;
}

// ---------------------------------------------------------------------------
// attention
// ---------------------------------------------------------------------------

// Position range [t0, t1) of attention split j of S over n_ctx positions.
__device__ __forceinline__ void split_range(int j, int S, int n_ctx, int& t0, int& t1) {
    t0 = static_cast<int>(static_cast<long long>(j) * n_ctx / S);
    t1 = static_cast<int>(static_cast<long long>(j + 1) * n_ctx / S);
}

// Thread 0: TMA bulk copies of cache rows [a, b) of kv head g into chunk rows
// [a - c0, b - c0), K and V, accounted on s.abar (expect_tx only; the arrive
// comes with the chunk's last batch).
__device__ __forceinline__ void issue_kv_rows(const DecodeParams& p, Smem& s, const PhaseDesc& d, int g, int c0, int a,
                                              int b) {
    if (b <= a) return;
    fence_proxy_async_global();  // rows other CTAs stored, read by the TMA engine
    const uint32_t bytes = static_cast<uint32_t>(b - a) * kHeadDim * 4u;
    const size_t off = (static_cast<size_t>(g) * p.max_ctx + a) * kHeadDim;
    mbar_expect_tx(&s.abar, 2u * bytes);
    bulk_g2s(&s.u.attn.akv[0][a - c0][0], d.kc + off, bytes, &s.abar);
    bulk_g2s(&s.u.attn.akv[1][a - c0][0], d.vc + off, bytes, &s.abar);
}

// Grouped-query attention of one layer at position st.pos (src/forward.rs:86-174),
// split over positions (flash-decoding), one (kv head, split) tile per CTA.
// Cache rows of earlier positions were prefetched into shared memory before
// the dependency wait (attn_prefetch); the current position's row and q come
// after it.  Each split leaves (max, sum, unnormalised output) per query head;
// for few splits the O phase merges them while staging its input, otherwise
// the last split of each kv head to finish merges them here.
__device__ __forceinline__ bool attention_phase(const DecodeParams& p, Smem& s, const PhaseDesc& d,
                                                const StepCtx& st, uint32_t& abar_phase, bool prefetched) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_ctx = st.pos + 1;
    const int S = st.S;
    const int group = p.group;
    const int n_tiles = p.kv_heads * S;
    const int ti = blockIdx.x;
    if (ti >= n_tiles) return true;
    const int g = ti / S, j = ti % S;
    int t0, t1;
    split_range(j, S, n_ctx, t0, t1);
    const float scale = sqrtf(static_cast<float>(kHeadDim));
    AttnBufs& a = s.u.attn;
    bool ok = true;
    for (int hp = 0; hp < group && ok; hp += kAttnHeadsPerPass) {
        const int nh = min(kAttnHeadsPerPass, group - hp);
        float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
        for (int c0 = t0; c0 < t1; c0 += kAttnChunk) {
            const int nc = min(kAttnChunk, t1 - c0);
            const bool first = (c0 == t0 && hp == 0);
            cbar();  // previous users of aq / akv are done
            if (tid == 0) {
                // Rows of earlier positions (prefetched for the first chunk),
                // then the current position's row, written this step.
                if (!(first && prefetched)) issue_kv_rows(p, s, d, g, c0, c0, min(c0 + nc, st.pos));
                if (st.pos >= c0 && st.pos < c0 + nc) {
                    const uint32_t bytes = kHeadDim * 4u;
                    const size_t off = (static_cast<size_t>(g) * p.max_ctx + st.pos) * kHeadDim;
                    fence_proxy_async_global();
                    mbar_arrive_expect_tx(&s.abar, 2u * bytes);
                    bulk_g2s(&a.akv[0][st.pos - c0][0], d.kc + off, bytes, &s.abar);
                    bulk_g2s(&a.akv[1][st.pos - c0][0], d.vc + off, bytes, &s.abar);
                } else {
                    mbar_arrive(&s.abar);
                }
            }
            if (c0 == t0)
                for (int e = tid; e < nh * kHeadDim; e += kThreads)
                    a.aq[e / kHeadDim][e % kHeadDim] =
                        __ldcg(p.q + static_cast<size_t>(g * group + hp + e / kHeadDim) * kHeadDim + e % kHeadDim);
            if (tid == 0) s.ok0 = wait_mbar(p, &s.abar, abar_phase & 1u, -2, st.f) ? 1 : 0;
            cbar();
            ++abar_phase;
            if (!s.ok0) {
                ok = false;
                break;
            }
            // every thread observes the completed copy before reading it
            for (int n = 0; n < (1 << 20) && !mbar_try_wait(&s.abar, (abar_phase - 1) & 1u); ++n) {
            }
            if (warp < nh) {
                // scores: lane = position; rotated column order keeps the
                // shared-memory reads of K and q conflict-free
                float sc = -INFINITY;
                if (lane < nc) {
                    float acc = 0.f;
#pragma unroll 16
                    for (int dd = 0; dd < kHeadDim; ++dd) {
                        const int c = (dd + lane) & (kHeadDim - 1);
                        acc = fmaf(a.aq[warp][c], a.akv[0][lane][c], acc);
                    }
                    sc = acc / scale;
                }
                const float m_new = fmaxf(m, warp_max(sc));
                const float pr = lane < nc ? expf(sc - m_new) : 0.f;
                const float corr = expf(m - m_new);
                l = l * corr + warp_sum(pr);
                o0 *= corr;
                o1 *= corr;
                for (int t = 0; t < nc; ++t) {
                    const float pt = __shfl_sync(FULL, pr, t);
                    o0 = fmaf(pt, a.akv[1][t][lane], o0);
                    o1 = fmaf(pt, a.akv[1][t][lane + 32], o1);
                }
                m = m_new;
            }
        }
        if (ok && warp < nh) {
            float* rec = p.attn_part + ((static_cast<size_t>(g) * p.max_splits + j) * group + hp + warp) * kAttnRec;
            if (lane == 0) {
                rec[0] = m;
                rec[1] = l;
            }
            rec[4 + lane] = o0;
            rec[4 + lane + 32] = o1;
        }
    }
    if (!ok) return false;
    if (S > kReaderCombineMaxSplits) {
        cbar();
        if (tid == 0) {
            // acquire-release count: this CTA's records (ordered before it by
            // the barrier) are visible before it, and the last one sees every
            // record
            const uint32_t old = atom_add_acq_rel_gpu(p.attn_cnt + d.layer * p.kv_heads + g, 1u);
            s.attn_last = (old == static_cast<uint32_t>(S - 1)) ? 1 : 0;
        }
        cbar();
        if (s.attn_last) {
            for (int h = warp; h < group; h += kWarps) {
                const float* base = p.attn_part + (static_cast<size_t>(g) * p.max_splits * group + h) * kAttnRec;
                const size_t jstride = static_cast<size_t>(group) * kAttnRec;
                // the splits' maxima, lanes over splits; then the records in
                // batches of 4 whose loads are all in flight at once, folded
                // in split order (the same sums as one split at a time)
                float M = -INFINITY;
                for (int jj = lane; jj < S; jj += 32) M = fmaxf(M, __ldcg(base + jj * jstride));
                M = warp_max(M);
                float L = 0.f, O0 = 0.f, O1 = 0.f;
                for (int j0 = 0; j0 < S; j0 += 4) {
                    float m4[4], l4[4], a4[4], b4[4];
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float* pj = base + static_cast<size_t>(min(j0 + i, S - 1)) * jstride;
                        m4[i] = __ldcg(pj);
                        l4[i] = __ldcg(pj + 1);
                        a4[i] = __ldcg(pj + 4 + lane);
                        b4[i] = __ldcg(pj + 4 + lane + 32);
                    }
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        if (j0 + i < S) {
                            const float w = expf(m4[i] - M);
                            L = fmaf(l4[i], w, L);
                            O0 = fmaf(a4[i], w, O0);
                            O1 = fmaf(b4[i], w, O1);
                        }
                    }
                }
                float* out = p.attn_out + static_cast<size_t>(g * group + h) * kHeadDim;
                out[lane] = O0 / L;
                out[lane + 32] = O1 / L;
            }
            if (tid == 0) p.attn_cnt[d.layer * p.kv_heads + g] = 0u;
        }
    }
    return true;
}

// Before the ATTN dependency wait (thread 0): prefetch the cache rows of
// earlier positions for this CTA's first attention chunk.  Those rows were
// written in earlier steps, so they need nothing from this step.
__device__ __forceinline__ bool attn_prefetch(const DecodeParams& p, Smem& s, const PhaseDesc& d,
                                              const StepCtx& st) {
    const int ti = blockIdx.x;
    if (ti >= p.kv_heads * st.S) return false;
    const int g = ti / st.S, j = ti % st.S;
    int t0, t1;
    split_range(j, st.S, st.pos + 1, t0, t1);
    issue_kv_rows(p, s, d, g, t0, t0, min(min(t1, t0 + kAttnChunk), st.pos));
    return true;
}

// ---------------------------------------------------------------------------
// the program loop
// ---------------------------------------------------------------------------
template <bool QACT>
__device__ __forceinline__ void run(const DecodeParams& p, Smem& s, Stream& sw) {
    const int G = gridDim.x;
    const int tid = threadIdx.x;
    uint32_t gidx = 0;  // schedule index of the current phase's first tile
    uint32_t abar_phase = 0;
    for (int f = 0; f < p.n_steps; ++f) {
        StepCtx st{f, p.pos0 + f, 0, false, attn_splits(p, p.pos0 + f + 1)};
        TraceAcc tr{p.trace != nullptr && f == p.trace_step && tid == 0, 0ull, 0ull, 0ull};
        for (int ph = 0; ph < p.n_phases; ++ph) {
            const PhaseDesc d = phase_at(p, ph);  // registers
            trace_mark(p, ph, f, 0);
            // 0. operands independent of the previous phase, loaded first
            Prefetch pf;
            bool prefetched = false;
            if (d.kind == PH_GEMV)
                prefetch_operands(p, d, st, pf);
            else if (tid == 0)
                prefetched = attn_prefetch(p, s, d, st);
            // 1. dependency on the previous phase (bounded), by thread 0; warp 0
            //    then reads the step's token
            if (tid < 32) {
                int ok = 1;
                if (tid == 0) {
                    const uint64_t w0 = tr.on ? globaltimer_ns() : 0;
                    // hold_phase (tests only) waits for one release more than
                    // the grid makes, so that wait runs into its time limit
                    if (ph > 0)
                        ok = wait_counter(p, p.counters + ph - 1,
                                          static_cast<uint32_t>((f + 1) * G + (ph == p.hold_phase ? 1 : 0)), ph, f)
                                 ? 1
                                 : 0;
                    else if (f > 0)
                        ok = wait_counter(p, p.counters + p.n_phases - 1,
                                          static_cast<uint32_t>(f * G + (p.hold_phase == 0 ? 1 : 0)), ph, f)
                                 ? 1
                                 : 0;
                    if (tr.on) tr.dep_wait_ns += globaltimer_ns() - w0;
                }
                ok = __shfl_sync(FULL, ok, 0);
                __syncwarp();  // the other lanes read what thread 0's acquire covers
                if (ok && d.kind == PH_GEMV && d.in_kind == IN_X0_NORM) {
                    // The step's token: prompt id, or greedy argmax of the
                    // previous step's logits (src/tokenizer.rs:152-167): the
                    // CTAs' candidates (value key << 32 | index, so the max
                    // keeps the last of equal values) loaded by all 32 lanes
                    // at once and reduced over the warp.
                    int tok = 0;
                    if (f < p.n_prompt) {
                        tok = p.prompt ? p.prompt[f] : 0;
                    } else if (f > 0) {
                        unsigned long long c8[8];
#pragma unroll
                        for (int i = 0; i < 8; ++i) {
                            const int c = tid + 32 * i;
                            c8[i] = c < G ? __ldcg(p.argmax_part + c) : 0ull;
                        }
                        unsigned long long b = 0ull;
#pragma unroll
                        for (int i = 0; i < 8; ++i) b = max(b, c8[i]);
                        for (int c = tid + 256; c < G; c += 32) b = max(b, __ldcg(p.argmax_part + c));
#pragma unroll
                        for (int o = 16; o; o >>= 1) b = max(b, __shfl_xor_sync(FULL, b, o));
                        tok = static_cast<int>(b & 0xffffffffu);
                    }
                    if (tid == 0) {
                        // Ids from device memory are unchecked by the host: an id
                        // outside the vocabulary is reported, and row 0 is read
                        // instead so no access leaves the embedding table.
                        if (tok < 0 || tok >= p.vocab) {
                            set_error(p, kErrBadToken, ph, f);
                            tok = 0;
                        }
                        s.token = tok;
                        if (blockIdx.x == 0 && f >= p.n_prompt && p.out_ids) p.out_ids[f - p.n_prompt] = tok;
                    }
                }
                if (tid == 0) s.phase_ok = ok;
            }
            cbar();
            if (!s.phase_ok) {
                if (tid == 0) {
                    if (prefetched) {  // let the prefetch land before exiting
                        mbar_arrive(&s.abar);
                        wait_mbar(p, &s.abar, abar_phase & 1u, ph, f);
                    }
                }
                cp_async_wait_all();  // no weight copy may land after the CTA left
                return;
            }
            trace_mark(p, ph, f, 1);
            bool ok = true;
            int deferred = 0;  // weight copies of the phase's last batch, issued after the release
            if (d.kind == PH_ATTN) {
                ok = attention_phase(p, s, d, st, abar_phase, prefetched);
            } else {
                if (d.in_kind == IN_X0_NORM) {
                    st.token = s.token;
                    st.x0_given = (f == 0 && p.x0 != nullptr);
                }
                ok = gemv_phase<QACT>(p, s, sw, d, st, ph, gidx, pf, tr, deferred);
                gidx += static_cast<uint32_t>(s.nmine[ph]);
            }
            if (!ok) s.abort_flag = 1;  // any warp: the CTA stops after this phase
            // 2. release this phase once all warps wrote their outputs.
            cbar();
            if (s.abort_flag) {
                cp_async_wait_all();
                return;
            }
            if (tid == 0) {
                if (d.epi == EPI_LOGITS && s.nmine[ph] > 0) {
                    unsigned long long b = 0ull;
                    for (int w = 0; w < kWarps; ++w) b = max(b, s.best[w]);
                    p.argmax_part[blockIdx.x] = b;
                }
                // gpu-scope release of the phase: covers every store of the CTA
                // ordered before it by the barrier above
                red_release_gpu_add(p.counters + ph, 1u);
                if (tr.on) {
                    unsigned long long* rec =
                        p.trace + (static_cast<size_t>(ph) * gridDim.x + blockIdx.x) * kTraceFields;
                    rec[4] = tr.data_wait_ns;
                    rec[5] = tr.tiles;
                    rec[6] = tr.dep_wait_ns;
                    tr.data_wait_ns = tr.dep_wait_ns = tr.tiles = 0ull;
                }
            }
            trace_mark(p, ph, f, 3);
            // 3. the deferred copies of the phase's last batch
            {
                const int warp = tid >> 5, lane = tid & 31;
                for (int ti = 0; ti < deferred; ++ti)
                    stream_next(p, s, sw, gidx - static_cast<uint32_t>(deferred - ti) + kWarpSlots, warp, lane);
            }
        }
    }
}

// QACT: the instantiation that also runs Mode::Quantize phases (PhaseDesc.qact);
// the Normal-mode one carries none of that code.
template <bool QACT>
__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x;
    if (tid == 0) {
        mbar_init(&s.abar, 1);
        s.abort_flag = 0;
        fence_mbar_init();
        build_schedule(p, s);
    }
    __syncthreads();
    // every warp starts its weight stream: the first kWarpSlots tiles
    const int warp = tid >> 5, lane = tid & 31;
    Stream sw{Pos{0, 0, 0}, true, -1, nullptr, 0, 0};
    sw.more = s.nmine[0] > 0 || pos_advance(p, s, sw.c, 0);
    for (uint32_t i = 0; i < static_cast<uint32_t>(kWarpSlots); ++i) stream_next(p, s, sw, i, warp, lane);
    run<QACT>(p, s, sw);
    cp_async_wait_all();
    if (p.phases == nullptr) {
        // a single matvec: the last CTA to leave clears the launch's error
        // words 0..2 and the exit count (word 4); word 3 keeps a failure's
        // code for the host.  Nothing of this launch reads them any more.
        __syncthreads();
        if (tid == 0) {
            __threadfence();
            if (atomicAdd(p.error + 4, 1u) == gridDim.x - 1) {
                p.error[0] = 0u;
                p.error[1] = 0u;
                p.error[2] = 0u;
                p.error[4] = 0u;
            }
        }
    }
}

int decode_smem_bytes() { return static_cast<int>(sizeof(Smem)); }

int decode_blocks_per_sm() {
    if (cudaFuncSetAttribute(decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(Smem))) != cudaSuccess)
        return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel<false>, kThreads, sizeof(Smem)) != cudaSuccess)
        return 0;
    return n;
}

int decode_grid_size(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    return sms;
}

// p.qact selects the instantiation that runs Mode::Quantize phases.
int decode_launch(const DecodeParams& p, int grid, void* stream, bool cooperative) {
    static thread_local int configured_device = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_device != dev) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(Smem)));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(decode_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(sizeof(Smem)));
        if (e != cudaSuccess) return static_cast<int>(e);
        configured_device = dev;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void (*kernel)(DecodeParams) = p.qact ? decode_kernel<true> : decode_kernel<false>;
    if (cooperative) {
        void* args[] = {const_cast<DecodeParams*>(&p)};
        return static_cast<int>(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(kernel), dim3(grid),
                                                            dim3(kThreads), args, sizeof(Smem), st));
    }
    kernel<<<grid, kThreads, sizeof(Smem), st>>>(p);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace tir
