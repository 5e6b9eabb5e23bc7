// decode.cu -- persistent sm_100a kernel running a whole forward program
// (runtime.h): the batch-1 decode loop of src/forward.rs:13-258 /
// src/lib.rs:239-314, or a single Q8_0 matvec (src/math.rs:87-98).
//
// One CTA of 8 warps per SM (cooperative launch: all CTAs co-resident).
//
// Weight stream.  Each CTA's weight tiles, in schedule order over every GEMV
// phase of every step, flow through a kStages-deep shared-memory ring filled
// by TMA bulk copies (cp.async.bulk, mbarrier completion).  Tile i sits in slot
// i % kStages and is consumed by warp i % 8, which refills the slot with tile
// i + kStages as soon as it is done.  Weights never wait for activations, so
// HBM keeps streaming while the warps wait on phase dependencies.
//
// Phases.  Every CTA waits (bounded) until all CTAs released the previous
// phase, stages the phase input once into shared memory (rmsnorm fused), then
// each warp works through its tiles independently -- row dots, one butterfly
// reduction per tile, fused epilogue (RoPE + KV append, residual, SiLU*up,
// logits + argmax) -- and the CTA releases the phase.
//
// Q8_0 split layout: quants are stored as u = q + 128 (one byte), so a weight
// becomes an exact f32 with one byte permute and one add:
//   float(0x4B000000 | u) = 2^23 + u,   (2^23 + u) - (2^23 + 128) = q.
// Products and sums use packed f32x2 FMA (sm_100).
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
constexpr uint32_t kBarAll = 1;  // named barrier id for the CTA's 8 warps

// Where the weight stream reads a phase's tiles (cached in shared memory so
// refills need no global loads).
struct TileSrc {
    const uint8_t* wq;
    const uint16_t* ws;
    int32_t k, sk, n, rows;
};

struct AttnBufs {
    float aq[kAttnHeadsPerPass][kHeadDim];
    float akv[2][kAttnChunk][kHeadDim];  // K and V rows of one chunk (TMA target)
};

struct __align__(128) Smem {
    uint8_t ring[kStages][kStageBytes];  // weight tiles (TMA targets)
    union {
        float xs[kMaxK];  // phase input, permuted [i4][chunk][4] (conflict-free 16-B reads)
        AttnBufs attn;
    } u;
    uint64_t full[kStages];
    uint64_t abar;  // attention K/V copies
    TileSrc src[kMaxPhases];
    unsigned long long best[kWarps];
    float red[kWarps];
    int32_t slot_issued[kStages];
    int16_t nmine[kMaxPhases], tfirst[kMaxPhases];
    int32_t token, phase_ok, abort_flag, attn_last, ok0;
};

// TMA bulk-copy destinations must start on 16-byte boundaries.
static_assert(offsetof(Smem, ring) % 128 == 0 && kStageBytes % 128 == 0, "ring slots must be 16-byte aligned");
static_assert((offsetof(Smem, u) + offsetof(AttnBufs, akv)) % 16 == 0, "akv must be 16-byte aligned");
static_assert(offsetof(Smem, full) % 8 == 0 && offsetof(Smem, abar) % 8 == 0, "mbarriers need 8-byte alignment");
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

__device__ __forceinline__ void set_error(const DecodeParams& p, uint32_t code, int ph, int f) {
    if (atomicCAS(p.error, 0u, code) == 0u) {
        p.error[1] = static_cast<uint32_t>(ph);
        p.error[2] = static_cast<uint32_t>(f);
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
        s.src[ph] = TileSrc{d.wq, d.ws, d.k, d.sk, d.n, d.rows_per_tile};
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

// TMA copy of the tile at `c` (schedule index i) into slot i % kStages.
__device__ __forceinline__ void issue_tile(Smem& s, const Pos& c, uint32_t i) {
    const TileSrc& t = s.src[c.ph];
    const int slot = static_cast<int>(i % kStages);
    const int r0 = (s.tfirst[c.ph] + c.k * static_cast<int>(gridDim.x)) * t.rows;
    const int rows = min(t.rows, t.n - r0);
    const uint32_t bq = static_cast<uint32_t>(rows) * t.k;
    const uint32_t bs = static_cast<uint32_t>(rows) * t.sk * 2u;
    mbar_arrive_expect_tx(&s.full[slot], bq + bs);
    bulk_g2s(s.ring[slot], t.wq + static_cast<size_t>(r0) * t.k, bq, &s.full[slot]);
    bulk_g2s(s.ring[slot] + bq, t.ws + static_cast<size_t>(r0) * t.sk, bs, &s.full[slot]);
    s.slot_issued[slot] += 1;
}

// Abort path (thread 0): wait, bounded, for the last copy issued into each slot.
__device__ __forceinline__ void drain_ring(const DecodeParams& p, Smem& s) {
    for (int slot = 0; slot < kStages; ++slot) {
        const int n = *reinterpret_cast<volatile int32_t*>(&s.slot_issued[slot]);
        if (n > 0) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&s.full[slot], static_cast<uint32_t>(n - 1) & 1u) &&
                   globaltimer_ns() - t0 < p.timeout_ns) {
            }
        }
    }
}

// ---------------------------------------------------------------------------
// GEMV phases
// ---------------------------------------------------------------------------

// 16 weights (one uint4 of u = q+128 bytes) dotted with 16 activations.
__device__ __forceinline__ float dot16(const uint4 w, const float* x) {
    const float2 magic = make_float2(-8388736.0f, -8388736.0f);
    float2 a0 = make_float2(0.f, 0.f), a1 = make_float2(0.f, 0.f);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float2 lo = make_float2(__uint_as_float(__byte_perm(ws[j], 0x4B000000u, 0x7440)),
                                __uint_as_float(__byte_perm(ws[j], 0x4B000000u, 0x7441)));
        float2 hi = make_float2(__uint_as_float(__byte_perm(ws[j], 0x4B000000u, 0x7442)),
                                __uint_as_float(__byte_perm(ws[j], 0x4B000000u, 0x7443)));
        lo = __fadd2_rn(lo, magic);
        hi = __fadd2_rn(hi, magic);
        a0 = __ffma2_rn(make_float2(x[4 * j], x[4 * j + 1]), lo, a0);
        a1 = __ffma2_rn(make_float2(x[4 * j + 2], x[4 * j + 3]), hi, a1);
    }
    return (a0.x + a0.y) + (a1.x + a1.y);
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
// step's token, src/tokenizer.rs:10-32: f32(q) * f32(scale), exact), the
// attention output (merging the per-split partial softmaxes when the
// attention phase left that to its readers), or the phase's input buffer.
// Data written by other CTAs is read from L2 (never a stale L1 line).
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
                v[4 * j + b] = __fmul_rn(static_cast<float>(static_cast<int>((w[j] >> (8 * b)) & 0xffu) - 128), sc);
    } else if (d.in_kind == IN_ATTN && st.S <= kReaderCombineMaxSplits) {
        // softmax-weighted merge of the splits of head h = k0 / 64
        const int h = k0 / kHeadDim, d0 = k0 % kHeadDim;
        const int g = h / p.group, hh = h % p.group;
        float4 ml[kReaderCombineMaxSplits];
        float4 o[kReaderCombineMaxSplits][4];
#pragma unroll
        for (int j = 0; j < kReaderCombineMaxSplits; ++j) {
            if (j < st.S) {
                const float* rec =
                    p.attn_part + ((static_cast<size_t>(g) * p.max_splits + j) * p.group + hh) * kAttnRec;
                ml[j] = __ldcg(reinterpret_cast<const float4*>(rec));
#pragma unroll
                for (int q = 0; q < 4; ++q) o[j][q] = __ldcg(reinterpret_cast<const float4*>(rec + 4 + d0) + q);
            }
        }
        float M = -INFINITY;
#pragma unroll
        for (int j = 0; j < kReaderCombineMaxSplits; ++j)
            if (j < st.S) M = fmaxf(M, ml[j].x);
        float L = 0.f, acc[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = 0.f;
#pragma unroll
        for (int j = 0; j < kReaderCombineMaxSplits; ++j) {
            if (j < st.S) {
                const float w = expf(ml[j].x - M);
                L = fmaf(ml[j].y, w, L);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    acc[4 * q] = fmaf(o[j][q].x, w, acc[4 * q]);
                    acc[4 * q + 1] = fmaf(o[j][q].y, w, acc[4 * q + 1]);
                    acc[4 * q + 2] = fmaf(o[j][q].z, w, acc[4 * q + 2]);
                    acc[4 * q + 3] = fmaf(o[j][q].w, w, acc[4 * q + 3]);
                }
            }
        }
        const float inv = 1.0f / L;
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = acc[i] * inv;
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

// Each thread stages chunks c = tid and tid + 256 (16 columns each).
constexpr int kChunksPerThread = (kMaxK / 16 + kThreads - 1) / kThreads;

// Operands of a phase that do not depend on the previous phase, loaded before
// the dependency wait so their HBM latency hides behind it: the rmsnorm
// weights of this thread's chunks and the position's RoPE cos/sin (lane i
// holds pair i).
struct Prefetch {
    float wr[kChunksPerThread * 16];
    float rc, rs;
};

__device__ __forceinline__ void prefetch_operands(const DecodeParams& p, const PhaseDesc& d, const StepCtx& st,
                                                  Prefetch& pf) {
    const int tid = threadIdx.x, lane = tid & 31;
    const bool norm = d.in_kind == IN_X_NORM || d.in_kind == IN_X0_NORM;
#pragma unroll
    for (int ci = 0; ci < kChunksPerThread; ++ci) {
        const int k0 = (tid + ci * kThreads) * 16;
        if (norm && k0 < d.k) {
            const float4* w4 = reinterpret_cast<const float4*>(d.norm_w + k0);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const float4 t = __ldg(w4 + j);
                pf.wr[ci * 16 + 4 * j] = t.x;
                pf.wr[ci * 16 + 4 * j + 1] = t.y;
                pf.wr[ci * 16 + 4 * j + 2] = t.z;
                pf.wr[ci * 16 + 4 * j + 3] = t.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) pf.wr[ci * 16 + i] = 0.f;
        }
    }
    pf.rc = 0.f;
    pf.rs = 0.f;
    if (d.epi == EPI_QKV) {
        pf.rc = __ldg(p.rope_cos + static_cast<size_t>(st.pos) * (kHeadDim / 2) + lane);
        pf.rs = __ldg(p.rope_sin + static_cast<size_t>(st.pos) * (kHeadDim / 2) + lane);
    }
}

// Stages the phase input into s.u.xs (layout [i4][chunk][4], i.e. element
// 16c + 4q + j at ((q * nchunks) + c) * 4 + j), with rmsnorm applied for
// IN_*_NORM phases (src/math.rs:141-150: x*w / sqrt(sum(x^2)/n + eps); the
// division is a multiplication by the correctly rounded reciprocal).  One
// round trip of loads; for the step input, the CTA owning a chunk also
// materialises it as the residual stream x (and dump row 0).
__device__ __forceinline__ void stage_input(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                                            const Prefetch& pf) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = d.k, nchunks = K / 16;
    const bool norm = d.in_kind == IN_X_NORM || d.in_kind == IN_X0_NORM;
    float v[kChunksPerThread * 16];
#pragma unroll
    for (int ci = 0; ci < kChunksPerThread; ++ci) {
        const int c = tid + ci * kThreads;
        if (c < nchunks) {
            load16(p, d, st, c * 16, v + ci * 16);
        } else {
#pragma unroll
            for (int i = 0; i < 16; ++i) v[ci * 16 + i] = 0.f;
        }
    }
    if (d.in_kind == IN_X0_NORM) {
#pragma unroll
        for (int ci = 0; ci < kChunksPerThread; ++ci) {
            const int c = tid + ci * kThreads;
            if (c < nchunks && c % static_cast<int>(gridDim.x) == static_cast<int>(blockIdx.x)) {
                float4* x4 = reinterpret_cast<float4*>(p.x + c * 16);
                float4* d4 = p.dump ? reinterpret_cast<float4*>(p.dump + c * 16) : nullptr;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const float4 t = make_float4(v[ci * 16 + 4 * j], v[ci * 16 + 4 * j + 1], v[ci * 16 + 4 * j + 2],
                                                 v[ci * 16 + 4 * j + 3]);
                    x4[j] = t;
                    if (d4) d4[j] = t;
                }
            }
        }
    }
    float inv = 1.0f;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < kChunksPerThread * 16; ++i) ss = fmaf(v[i], v[i], ss);
        ss = warp_sum(ss);
        if (lane == 0) s.red[warp] = ss;
        cbar();
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) total += s.red[w];
        inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), p.rms_eps)));
    }
    float4* xs4 = reinterpret_cast<float4*>(s.u.xs);
#pragma unroll
    for (int ci = 0; ci < kChunksPerThread; ++ci) {
        const int c = tid + ci * kThreads;
        if (c < nchunks) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float4 t;
                const float* e = v + ci * 16 + 4 * q;
                const float* w = pf.wr + ci * 16 + 4 * q;
                if (norm) {
                    t = make_float4(__fmul_rn(__fmul_rn(e[0], w[0]), inv), __fmul_rn(__fmul_rn(e[1], w[1]), inv),
                                    __fmul_rn(__fmul_rn(e[2], w[2]), inv), __fmul_rn(__fmul_rn(e[3], w[3]), inv));
                } else {
                    t = make_float4(e[0], e[1], e[2], e[3]);
                }
                xs4[q * nchunks + c] = t;
            }
        }
    }
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

// One warp, one tile of `rows` (<= R) rows: per-lane partial dots over the
// lane's 16-column chunks (every 32nd), then the warp reduction.  Returns, in
// lane l, the dot of row (l >> 2) & 7 (R > 1) or of row 0 (R == 1).
template <int R>
__device__ __forceinline__ float warp_tile(const uint8_t* tq, const uint16_t* ts, const float* xs, int K, int sk,
                                           int rows) {
    const int lane = threadIdx.x & 31;
    const int nchunks = K / 16;
    const float4* xv = reinterpret_cast<const float4*>(xs);
    float acc[R];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = 0.f;
    for (int c = lane; c < nchunks; c += 32) {
        float x[16];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float4 t = xv[q * nchunks + c];
            x[4 * q] = t.x;
            x[4 * q + 1] = t.y;
            x[4 * q + 2] = t.z;
            x[4 * q + 3] = t.w;
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
            if (r < rows) {
                const uint4 w = *reinterpret_cast<const uint4*>(tq + static_cast<size_t>(r) * K + c * 16);
                const float sc = __half2float(__ushort_as_half(ts[r * sk + (c >> 1)]));
                acc[r] = fmaf(dot16(w, x), sc, acc[r]);
            }
        }
    }
    if constexpr (R == 1) {
        return warp_sum(acc[0]);
    } else {
        float v[8];
#pragma unroll
        for (int r = 0; r < 8; ++r) v[r] = r < R ? acc[r < R ? r : 0] : 0.f;
        return reduce8(v, lane);
    }
}

// Fused epilogue of one tile, run by the lanes l with (l & 3) == 0: row
// (l >> 2) & 7 of the tile (only lane 0 when R == 1); y = row dot, pre =
// prefetched residual (EPI_RESID), (rc, rs) = the warp's RoPE cos/sin row
// (lane i holds pair i).
__device__ __forceinline__ void epilogue(const DecodeParams& p, const PhaseDesc& d, const StepCtx& st, int r0,
                                         int rows, int R, float y, float pre, float rc, float rs,
                                         unsigned long long& best) {
    const int lane = threadIdx.x & 31;
    const int row = R == 1 ? 0 : (lane >> 2) & 7;
    const int n = r0 + row;
    const float y1 = __shfl_down_sync(FULL, y, 4);  // row + 1 (pairs need R >= 2)
    const int pair = (n % kHeadDim) >> 1;
    const float c = __shfl_sync(FULL, rc, pair & 31);
    const float sn = __shfl_sync(FULL, rs, pair & 31);
    if ((lane & 3) != 0 || row >= rows || (R == 1 && lane != 0)) return;
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
        case EPI_GU:  // rows (2i, 2i+1) = (gate_i, up_i); src/math.rs:171-175
            if ((row & 1) == 0) {
                const float silu = __fdiv_rn(y, __fadd_rn(1.0f, expf(-y)));
                d.out[n >> 1] = __fmul_rn(silu, y1);
            }
            break;
        case EPI_QKV:
            if ((row & 1) == 0) {
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
            }
            break;
        default:
            break;
    }
}

// Trace accumulators of the traced step (thread 0 only).
struct TraceAcc {
    bool on;
    unsigned long long data_wait_ns, dep_wait_ns, tiles;
};

// The warp's tiles of one GEMV phase: schedule indices gidx + k for the
// phase's ordinals k with (gidx + k) % 8 == warp.  Returns false on timeout.
template <int R>
__device__ __forceinline__ bool gemv_tiles(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                                           int ph, uint32_t gidx, const Prefetch& pf, TraceAcc& tr,
                                           unsigned long long& best) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nm = s.nmine[ph];
    const int G = gridDim.x;
    const int K = d.k, SK = d.sk, N = d.n;
    int k = (warp - static_cast<int>(gidx % kWarps) + kWarps) % kWarps;
    for (; k < nm; k += kWarps) {
        const uint32_t i = gidx + static_cast<uint32_t>(k);
        const int slot = static_cast<int>(i % kStages);
        const int r0 = (s.tfirst[ph] + k * G) * R;
        const int rows = min(R, N - r0);
        const int row = R == 1 ? 0 : (lane >> 2) & 7;
        float pre = 0.f;
        if (d.epi == EPI_RESID && (lane & 3) == 0 && row < rows) pre = __ldcg(d.out + r0 + row);
        // lane 0 waits for the tile's bytes; the warp sync orders the reads
        int ok = 1;
        if (lane == 0) {
            const uint64_t t0 = tr.on ? globaltimer_ns() : 0;
            ok = wait_mbar(p, &s.full[slot], (i / kStages) & 1u, ph, st.f) ? 1 : 0;
            if (tr.on) tr.data_wait_ns += globaltimer_ns() - t0;
        }
        ok = __shfl_sync(FULL, ok, 0);
        if (!ok) return false;
        const uint8_t* tq = s.ring[slot];
        const uint16_t* ts = reinterpret_cast<const uint16_t*>(tq + static_cast<size_t>(rows) * K);
        const float y = warp_tile<R>(tq, ts, s.u.xs, K, SK, rows);
        __syncwarp();
        // the slot is free: refill it with the tile kStages ahead
        if (lane == 0) {
            Pos c{st.f, ph, k};
            if (pos_advance(p, s, c, kStages)) issue_tile(s, c, i + kStages);
        }
        epilogue(p, d, st, r0, rows, R, y, pre, pf.rc, pf.rs, best);
        if (tr.on) tr.tiles += 1;
    }
    return true;
}

// One GEMV phase; returns false on timeout (this CTA then stops at the end
// of the phase, together with its other warps).
__device__ __forceinline__ bool gemv_phase(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                                           int ph, uint32_t gidx, const Prefetch& pf, TraceAcc& tr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nm = s.nmine[ph];
    if (nm == 0) {
        if (d.epi == EPI_LOGITS && tid == 0) p.argmax_part[blockIdx.x] = 0ull;
        return true;
    }
    stage_input(p, s, d, st, pf);
    trace_mark(p, ph, st.f, 2);
    unsigned long long best = 0ull;
    bool ok;
    switch (d.rows_per_tile) {
        case 1: ok = gemv_tiles<1>(p, s, d, st, ph, gidx, pf, tr, best); break;
        case 2: ok = gemv_tiles<2>(p, s, d, st, ph, gidx, pf, tr, best); break;
        case 4: ok = gemv_tiles<4>(p, s, d, st, ph, gidx, pf, tr, best); break;
        default: ok = gemv_tiles<8>(p, s, d, st, ph, gidx, pf, tr, best); break;
    }
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
            __threadfence();
            const uint32_t old = atomicAdd(p.attn_cnt + d.layer * p.kv_heads + g, 1u);
            s.attn_last = (old == static_cast<uint32_t>(S - 1)) ? 1 : 0;
        }
        cbar();
        if (s.attn_last) {
            __threadfence();
            for (int h = warp; h < group; h += kWarps) {
                const float* base = p.attn_part + (static_cast<size_t>(g) * p.max_splits * group + h) * kAttnRec;
                const size_t jstride = static_cast<size_t>(group) * kAttnRec;
                float M = -INFINITY;
                for (int jj = 0; jj < S; ++jj) M = fmaxf(M, __ldcg(base + jj * jstride));
                float L = 0.f, O0 = 0.f, O1 = 0.f;
                for (int jj = 0; jj < S; ++jj) {
                    const float* pj = base + jj * jstride;
                    const float w = expf(__ldcg(pj) - M);
                    L = fmaf(__ldcg(pj + 1), w, L);
                    O0 = fmaf(__ldcg(pj + 4 + lane), w, O0);
                    O1 = fmaf(__ldcg(pj + 4 + lane + 32), w, O1);
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
__device__ __forceinline__ void run(const DecodeParams& p, Smem& s) {
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
            // 1. dependency on the previous phase (bounded), by thread 0
            if (tid == 0) {
                const uint64_t w0 = tr.on ? globaltimer_ns() : 0;
                bool ok = true;
                if (ph > 0)
                    ok = wait_counter(p, p.counters + ph - 1, static_cast<uint32_t>((f + 1) * G), ph, f);
                else if (f > 0)
                    ok = wait_counter(p, p.counters + p.n_phases - 1, static_cast<uint32_t>(f * G), ph, f);
                if (tr.on) tr.dep_wait_ns += globaltimer_ns() - w0;
                if (ok && d.kind == PH_GEMV && d.in_kind == IN_X0_NORM) {
                    // The step's token: prompt id, or greedy argmax of the
                    // previous step's logits (src/tokenizer.rs:152-167).
                    int tok = 0;
                    if (f < p.n_prompt) {
                        tok = p.prompt ? p.prompt[f] : 0;
                    } else if (f > 0) {
                        unsigned long long b = 0ull;
                        for (int c = 0; c < G; ++c) b = max(b, __ldcg(p.argmax_part + c));
                        tok = static_cast<int>(b & 0xffffffffu);
                    }
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
                s.phase_ok = ok ? 1 : 0;
            }
            cbar();
            if (!s.phase_ok) {
                if (tid == 0) {
                    if (prefetched) {  // let the prefetch land before exiting
                        mbar_arrive(&s.abar);
                        wait_mbar(p, &s.abar, abar_phase & 1u, ph, f);
                    }
                    drain_ring(p, s);
                }
                return;
            }
            trace_mark(p, ph, f, 1);
            bool ok = true;
            if (d.kind == PH_ATTN) {
                ok = attention_phase(p, s, d, st, abar_phase, prefetched);
            } else {
                if (d.in_kind == IN_X0_NORM) {
                    st.token = s.token;
                    st.x0_given = (f == 0 && p.x0 != nullptr);
                }
                ok = gemv_phase(p, s, d, st, ph, gidx, pf, tr);
                gidx += static_cast<uint32_t>(s.nmine[ph]);
            }
            if (!ok) s.abort_flag = 1;  // any warp: the CTA stops after this phase
            // 2. release this phase once all warps wrote their outputs.
            cbar();
            if (s.abort_flag) {
                if (tid == 0) drain_ring(p, s);
                return;
            }
            if (tid == 0) {
                if (d.epi == EPI_LOGITS && s.nmine[ph] > 0) {
                    unsigned long long b = 0ull;
                    for (int w = 0; w < kWarps; ++w) b = max(b, s.best[w]);
                    p.argmax_part[blockIdx.x] = b;
                }
                __threadfence();
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
        }
    }
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Smem& s = *reinterpret_cast<Smem*>(smem_raw);
    const int tid = threadIdx.x;
    if (tid == 0) {
        for (int i = 0; i < kStages; ++i) {
            mbar_init(&s.full[i], 1);
            s.slot_issued[i] = 0;
        }
        mbar_init(&s.abar, 1);
        s.abort_flag = 0;
        fence_mbar_init();
        build_schedule(p, s);
        // fill the ring with the first kStages tiles of the schedule
        Pos c{0, 0, 0};
        bool more = s.nmine[0] > 0 || pos_advance(p, s, c, 0);
        for (uint32_t i = 0; more && i < static_cast<uint32_t>(kStages); ++i) {
            issue_tile(s, c, i);
            more = pos_advance(p, s, c, 1);
        }
    }
    __syncthreads();
    run(p, s);
}

int decode_smem_bytes() { return static_cast<int>(sizeof(Smem)); }

int decode_blocks_per_sm() {
    if (cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(Smem))) != cudaSuccess)
        return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_kernel, kThreads, sizeof(Smem)) != cudaSuccess)
        return 0;
    return n;
}

int decode_grid_size(int device) {
    int sms = 0;
    if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return 0;
    return sms;
}

int decode_launch(const DecodeParams& p, int grid, void* stream, bool cooperative) {
    static thread_local int configured_device = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured_device != dev) {
        cudaError_t e = cudaFuncSetAttribute(decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(Smem)));
        if (e != cudaSuccess) return static_cast<int>(e);
        configured_device = dev;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (cooperative) {
        void* args[] = {const_cast<DecodeParams*>(&p)};
        return static_cast<int>(cudaLaunchCooperativeKernel(reinterpret_cast<void*>(decode_kernel), dim3(grid),
                                                            dim3(kThreads), args, sizeof(Smem), st));
    }
    decode_kernel<<<grid, kThreads, sizeof(Smem), st>>>(p);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace tir
