// decode.cu -- persistent sm_100a kernel running a whole forward program
// (runtime.h): the batch-1 decode loop of src/forward.rs:13-258 /
// src/lib.rs:239-314, or a single Q8_0 matvec (src/math.rs:87-98).
//
// One CTA per SM (cooperative launch, so all CTAs are co-resident).
//   warp 8 (producer): one lane walks this CTA's weight tiles of every phase of
//     every step and streams them into a kStages-deep shared-memory ring with
//     TMA bulk copies (cp.async.bulk, mbarrier completion).  Weights never wait
//     for activations, so HBM keeps streaming across phase boundaries.
//   warps 0-7 (consumers): for each phase, wait (bounded) until every CTA has
//     released the previous phase, stage the phase input (rmsnorm fused) in
//     registers, then for each ring tile compute the row dot products and run
//     the fused epilogue (RoPE + KV append, residual, SiLU*up, logits+argmax).
//
// Q8_0 split layout: quants are stored as u = q + 128 (one byte), so a weight
// becomes an exact f32 with one byte permute and one add:
//   float(0x4B000000 | u) = 2^23 + u,   (2^23 + u) - (2^23 + 128) = q.
// Products and sums use packed f32x2 FMA (sm_100).
//
// Every wait is bounded by DecodeParams::timeout_ns (globaltimer); on expiry the
// kernel records TIR_ERR_TIMEOUT, the producer drains its in-flight copies, and
// all CTAs return.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "ptx.cuh"
#include "runtime.h"

namespace tir {

constexpr uint32_t kErrTimeout = 25;   // TIR_ERR_TIMEOUT
constexpr uint32_t kErrBadToken = 12;  // TIR_ERR_BAD_TOKEN
constexpr uint32_t FULL = 0xffffffffu;
constexpr uint32_t kBarConsumers = 1;  // named barrier id for the 256 consumer threads

struct __align__(128) Smem {
    uint8_t ring[kStages][kStageBytes];
    uint64_t full[kStages];
    uint64_t empty[kStages];
    float part[2][kMaxTileRows][kMaxSegs];
    float red[kConsumerWarps];
    float aq[kAttnHeadsPerPass][kHeadDim];
    float ak[kAttnChunk][kHeadDim + 1];
    float av[kAttnChunk][kHeadDim];
    int32_t abort_flag;
    int32_t token;
    int32_t attn_last;
    int32_t phase_ok;
    int32_t ok[2];
};

__device__ __forceinline__ const PhaseDesc& phase_at(const DecodeParams& p, int i) {
    return p.phases ? p.phases[i] : p.single;
}

__device__ __forceinline__ void cbar() { named_bar(kBarConsumers, kConsumerThreads); }

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

__device__ __forceinline__ bool any_error(const DecodeParams& p) {
    return ld_relaxed_gpu(p.error) != 0u;
}

// Bounded wait for a grid-wide phase counter (one thread).
__device__ bool wait_counter(const DecodeParams& p, const uint32_t* ctr, uint32_t target, int ph,
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

// Bounded wait for an mbarrier phase (one thread).  `watch_abort` lets the
// producer give up as soon as the consumers abort.
__device__ bool wait_mbar(const DecodeParams& p, Smem& s, uint64_t* bar, uint32_t parity,
                          bool watch_abort, int ph, int f) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    uint32_t n = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++n & 15u) == 0u) {
            if (watch_abort && (*reinterpret_cast<volatile int32_t*>(&s.abort_flag) || any_error(p)))
                return false;
            if (globaltimer_ns() - t0 > p.timeout_ns) {
                set_error(p, kErrTimeout, ph, f);
                return false;
            }
        }
    }
    return true;
}

// Every consumer thread observes the completed phase of a ring slot (already
// awaited by thread 0, so this returns at once) before reading bytes the TMA
// engine wrote; bounded in case the invariant is ever broken.
__device__ __forceinline__ void observe_full(Smem& s, uint32_t it) {
    for (int n = 0; n < (1 << 20) && !mbar_try_wait(&s.full[it % kStages], (it / kStages) & 1u); ++n) {
    }
}

__device__ __forceinline__ int first_tile(int rot, int G) {
    return (static_cast<int>(blockIdx.x) - rot + G) % G;
}

// ---------------------------------------------------------------------------
// producer
// ---------------------------------------------------------------------------
__device__ void producer(const DecodeParams& p, Smem& s) {
    const int G = gridDim.x;
    uint32_t it = 0;
    bool ok = true;
    for (int f = 0; f < p.n_steps && ok; ++f) {
        int rot = 0;
        for (int ph = 0; ph < p.n_phases && ok; ++ph) {
            const PhaseDesc& d = phase_at(p, ph);
            if (d.kind != PH_GEMV) continue;
            for (int t = first_tile(rot, G); t < d.n_tiles; t += G, ++it) {
                const int slot = static_cast<int>(it % kStages);
                const uint32_t round = it / kStages;
                if (round > 0 && !wait_mbar(p, s, &s.empty[slot], (round - 1) & 1u, true, ph, f)) {
                    ok = false;
                    break;
                }
                const int r0 = t * d.rows_per_tile;
                const int rows = min(d.rows_per_tile, d.n - r0);
                const uint32_t bq = static_cast<uint32_t>(rows) * d.k;
                const uint32_t bs = static_cast<uint32_t>(rows) * d.sk * 2u;
                mbar_arrive_expect_tx(&s.full[slot], bq + bs);
                bulk_g2s(s.ring[slot], d.wq + static_cast<size_t>(r0) * d.k, bq, &s.full[slot]);
                bulk_g2s(s.ring[slot] + bq, d.ws + static_cast<size_t>(r0) * d.sk, bs,
                         &s.full[slot]);
            }
            rot = (rot + d.n_tiles) % G;
        }
    }
    if (!ok) {
        // Abort: let every copy still in flight land before the CTA exits.
        const uint32_t lo = it > static_cast<uint32_t>(kStages) ? it - kStages : 0u;
        for (uint32_t j = lo; j < it; ++j)
            wait_mbar(p, s, &s.full[j % kStages], (j / kStages) & 1u, false, -1, -1);
    }
}

// ---------------------------------------------------------------------------
// consumer helpers
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
};

// Element k of the step input x0: the explicit vector, or the embedding row of
// the step's token (src/tokenizer.rs:10-32: f32(q) * f32(scale), exact).
__device__ __forceinline__ float x0_at(const DecodeParams& p, const StepCtx& st, int k) {
    if (st.x0_given) return __ldcg(p.x0 + k);
    const size_t row = static_cast<size_t>(st.token);
    const int q = static_cast<int>(p.embd_q[row * p.H + k]) - 128;
    return static_cast<float>(q) * __half2float(__ushort_as_half(p.embd_s[row * p.embd_sk + k / 32]));
}

__device__ __forceinline__ float in_at(const DecodeParams& p, const PhaseDesc& d,
                                       const StepCtx& st, int k) {
    return d.in_kind == IN_X0_NORM ? x0_at(p, st, k) : __ldcg(d.in + k);
}

// Stages the phase input into registers: xr[si*16 + i] is input element
// seg*512 + lane*16 + i of the warp's si-th segment (rmsnorm applied,
// src/math.rs:141-150: (x*w)/sqrt(sum(x^2)/n + eps)).
__device__ void stage_input(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                            int nseg_w, const int* segs, float* xr) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = d.k;
    float rms = 1.0f;
    const bool norm = d.in_kind != IN_RAW;
    if (norm) {
        float ss = 0.f;
        for (int k = tid; k < K; k += kConsumerThreads) {
            const float v = in_at(p, d, st, k);
            ss += v * v;
        }
        ss = warp_sum(ss);
        if (lane == 0) s.red[warp] = ss;
        cbar();
        float total = 0.f;
#pragma unroll
        for (int w = 0; w < kConsumerWarps; ++w) total += s.red[w];
        rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(K)), p.rms_eps));
    }
#pragma unroll
    for (int si = 0; si < kMaxSegsPerWarp; ++si) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
            float v = 0.f;
            if (si < nseg_w) {
                const int k = segs[si] * kSegK + lane * 16 + i;
                if (k < K) {
                    v = in_at(p, d, st, k);
                    if (norm) v = __fdiv_rn(__fmul_rn(v, __ldg(d.norm_w + k)), rms);
                }
            }
            xr[si * 16 + i] = v;
        }
    }
}

// Fused epilogue for rows r0 + lane (lane < rows) of one tile; y = row dot.
__device__ __forceinline__ void epilogue(const DecodeParams& p, const PhaseDesc& d,
                                         const StepCtx& st, int r0, int rows, float y,
                                         unsigned long long& best) {
    const int lane = threadIdx.x & 31;
    const float y1 = __shfl_down_sync(FULL, y, 1);
    if (lane >= rows) return;
    const int n = r0 + lane;
    switch (d.epi) {
        case EPI_STORE:
            d.out[n] = y;
            break;
        case EPI_LOGITS:
            d.out[n] = y;
            best = max(best, pack_best(y, n));
            break;
        case EPI_RESID: {  // src/forward.rs:192, :232-236
            const float x = __fadd_rn(__ldcg(d.out + n), y);
            d.out[n] = x;
            if (d.dump && p.dump) p.dump[static_cast<size_t>(d.layer + 1) * p.H + n] = x;
            break;
        }
        case EPI_GU:  // rows (2i, 2i+1) = (gate_i, up_i); src/math.rs:171-175
            if ((lane & 1) == 0) {
                const float silu = __fdiv_rn(y, __fadd_rn(1.0f, expf(-y)));
                d.out[n >> 1] = __fmul_rn(silu, y1);
            }
            break;
        case EPI_QKV:
            if ((lane & 1) == 0) {
                // RoPE on adjacent pairs (src/math.rs:196-228), then q or the
                // KV-cache append (src/forward.rs:71, :83-84).
                const int H = p.H, kvd = p.kvd;
                int idx = n, d0;
                float* dst;
                bool rope = true;
                if (idx < H) {
                    dst = d.out + idx;
                    d0 = idx % kHeadDim;
                } else if (idx < H + kvd) {
                    idx -= H;
                    d0 = idx % kHeadDim;
                    dst = d.kc + (static_cast<size_t>(idx / kHeadDim) * p.max_ctx + st.pos) * kHeadDim + d0;
                } else {
                    idx -= H + kvd;
                    d0 = idx % kHeadDim;
                    dst = d.vc + (static_cast<size_t>(idx / kHeadDim) * p.max_ctx + st.pos) * kHeadDim + d0;
                    rope = false;
                }
                float e0 = y, e1 = y1;
                if (rope) {
                    const int i = d0 >> 1;
                    const float c = __ldg(p.rope_cos + static_cast<size_t>(st.pos) * (kHeadDim / 2) + i);
                    const float sn = __ldg(p.rope_sin + static_cast<size_t>(st.pos) * (kHeadDim / 2) + i);
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

// One GEMV phase: returns false on abort.
__device__ bool gemv_phase(const DecodeParams& p, Smem& s, const PhaseDesc& d, const StepCtx& st,
                           int ph, int rot, uint32_t& it, int& buf) {
    const int G = gridDim.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t_first = first_tile(rot, G);
    const int n_mine = t_first < d.n_tiles ? (d.n_tiles - 1 - t_first) / G + 1 : 0;
    if (n_mine == 0) {
        if (d.epi == EPI_LOGITS && tid == 0) p.argmax_part[blockIdx.x] = 0ull;
        return true;
    }

    // Warp -> (segments, rows) assignment.
    const int NS = d.segs;
    const bool split_rows = NS <= kConsumerWarps && (kConsumerWarps % NS) == 0;
    int segs[kMaxSegsPerWarp] = {0, 0};
    int nseg_w = 0, rho0 = 0, rho_step = 1;
    if (split_rows) {
        segs[0] = warp % NS;
        nseg_w = 1;
        rho0 = warp / NS;
        rho_step = kConsumerWarps / NS;
    } else {
        for (int sgi = warp; sgi < NS && nseg_w < kMaxSegsPerWarp; sgi += kConsumerWarps) segs[nseg_w++] = sgi;
    }
    float xr[kMaxSegsPerWarp * 16];
    stage_input(p, s, d, st, nseg_w, segs, xr);

    unsigned long long best = 0ull;
    for (int i = 0; i < n_mine; ++i, ++it) {
        const int t = t_first + i * G;
        const int slot = static_cast<int>(it % kStages);
        const int r0 = t * d.rows_per_tile;
        const int rows = min(d.rows_per_tile, d.n - r0);
        const uint8_t* tq = s.ring[slot];
        const uint16_t* ts = reinterpret_cast<const uint16_t*>(tq + static_cast<size_t>(rows) * d.k);
        // Data of tile i was awaited by thread 0 before the previous barrier.
        observe_full(s, it);
#pragma unroll 1
        for (int rho = rho0; rho < rows; rho += rho_step) {
#pragma unroll
            for (int si = 0; si < kMaxSegsPerWarp; ++si) {
                if (si < nseg_w) {
                    const int kk = segs[si] * kSegK + lane * 16;
                    float acc = 0.f;
                    if (kk < d.k) {
                        const uint4 w = *reinterpret_cast<const uint4*>(tq + static_cast<size_t>(rho) * d.k + kk);
                        const float sc = __half2float(__ushort_as_half(ts[rho * d.sk + (kk >> 5)]));
                        acc = dot16(w, xr + si * 16) * sc;
                    }
                    acc = warp_sum(acc);
                    if (lane == 0) s.part[buf][rho][segs[si]] = acc;
                }
            }
        }
        // Thread 0 waits for the next tile's bytes before the barrier, so one
        // barrier per tile both publishes the partials and the next tile.
        if (tid == 0) {
            bool ok = true;
            if (i + 1 < n_mine) {
                const uint32_t nx = it + 1;
                ok = wait_mbar(p, s, &s.full[nx % kStages], (nx / kStages) & 1u, false, ph, st.f);
            }
            s.ok[i & 1] = ok ? 1 : 0;
        }
        cbar();
        const bool ok = s.ok[i & 1] != 0;
        if (tid == 0) mbar_arrive(&s.empty[slot]);
        if (warp == 0) {
            float y = 0.f;
            if (lane < rows)
                for (int sg = 0; sg < NS; ++sg) y += s.part[buf][lane][sg];
            epilogue(p, d, st, r0, rows, y, best);
        }
        buf ^= 1;
        if (!ok) return false;
    }
    if (d.epi == EPI_LOGITS && warp == 0) {
#pragma unroll
        for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(FULL, best, o));
        if (lane == 0) p.argmax_part[blockIdx.x] = best;
    }
    return true;
}

// Grouped-query attention of one layer at position st.pos, split over
// positions (flash-decoding): src/forward.rs:86-174.  Returns false on abort.
__device__ bool attention_phase(const DecodeParams& p, Smem& s, const PhaseDesc& d,
                                const StepCtx& st) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n_ctx = st.pos + 1;
    int S = (n_ctx + kAttnChunk - 1) / kAttnChunk;
    S = max(1, min(S, p.max_splits));
    const int group = p.group;
    const int n_tiles = p.kv_heads * S;
    const float scale = sqrtf(static_cast<float>(kHeadDim));
    for (int ti = blockIdx.x; ti < n_tiles; ti += gridDim.x) {
        const int g = ti / S, j = ti % S;
        const int t0 = static_cast<int>(static_cast<long long>(j) * n_ctx / S);
        const int t1 = static_cast<int>(static_cast<long long>(j + 1) * n_ctx / S);
        const float* Kg = d.kc + static_cast<size_t>(g) * p.max_ctx * kHeadDim;
        const float* Vg = d.vc + static_cast<size_t>(g) * p.max_ctx * kHeadDim;
        for (int hp = 0; hp < group; hp += kAttnHeadsPerPass) {
            const int nh = min(kAttnHeadsPerPass, group - hp);
            cbar();
            for (int e = tid; e < nh * kHeadDim; e += kConsumerThreads)
                s.aq[e / kHeadDim][e % kHeadDim] =
                    __ldcg(p.q + static_cast<size_t>(g * group + hp + e / kHeadDim) * kHeadDim + e % kHeadDim);
            float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
            for (int c0 = t0; c0 < t1; c0 += kAttnChunk) {
                const int nc = min(kAttnChunk, t1 - c0);
                cbar();
                for (int e = tid; e < nc * kHeadDim; e += kConsumerThreads) {
                    const int t = e / kHeadDim, dd = e % kHeadDim;
                    s.ak[t][dd] = __ldcg(Kg + static_cast<size_t>(c0 + t) * kHeadDim + dd);
                    s.av[t][dd] = __ldcg(Vg + static_cast<size_t>(c0 + t) * kHeadDim + dd);
                }
                cbar();
                if (warp < nh) {
                    float sc = -INFINITY;
                    if (lane < nc) {
                        float acc = 0.f;
#pragma unroll 16
                        for (int dd = 0; dd < kHeadDim; ++dd) acc = fmaf(s.aq[warp][dd], s.ak[lane][dd], acc);
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
                        o0 = fmaf(pt, s.av[t][lane], o0);
                        o1 = fmaf(pt, s.av[t][lane + 32], o1);
                    }
                    m = m_new;
                }
            }
            if (warp < nh) {
                const int h = hp + warp;
                if (S == 1) {
                    float* out = p.attn_out + static_cast<size_t>(g * group + h) * kHeadDim;
                    out[lane] = o0 / l;
                    out[lane + 32] = o1 / l;
                } else {
                    float* part = p.attn_part +
                                  ((static_cast<size_t>(g) * p.max_splits + j) * group + h) * (kHeadDim + 2);
                    if (lane == 0) {
                        part[0] = m;
                        part[1] = l;
                    }
                    part[2 + lane] = o0;
                    part[2 + lane + 32] = o1;
                }
            }
        }
        if (S > 1) {
            cbar();
            if (tid == 0) {
                __threadfence();
                const uint32_t old = atomicAdd(p.attn_cnt + d.layer * p.kv_heads + g, 1u);
                s.attn_last = (old == static_cast<uint32_t>(S - 1)) ? 1 : 0;
            }
            cbar();
            if (s.attn_last) {
                __threadfence();
                for (int h = warp; h < group; h += kConsumerWarps) {
                    const float* base = p.attn_part + (static_cast<size_t>(g) * p.max_splits * group + h) * (kHeadDim + 2);
                    const size_t jstride = static_cast<size_t>(group) * (kHeadDim + 2);
                    float M = -INFINITY;
                    for (int jj = 0; jj < S; ++jj) M = fmaxf(M, __ldcg(base + jj * jstride));
                    float L = 0.f, O0 = 0.f, O1 = 0.f;
                    for (int jj = 0; jj < S; ++jj) {
                        const float* pj = base + jj * jstride;
                        const float w = expf(__ldcg(pj) - M);
                        L = fmaf(__ldcg(pj + 1), w, L);
                        O0 = fmaf(__ldcg(pj + 2 + lane), w, O0);
                        O1 = fmaf(__ldcg(pj + 2 + lane + 32), w, O1);
                    }
                    float* out = p.attn_out + static_cast<size_t>(g * group + h) * kHeadDim;
                    out[lane] = O0 / L;
                    out[lane + 32] = O1 / L;
                }
                if (tid == 0) p.attn_cnt[d.layer * p.kv_heads + g] = 0u;
            }
        }
    }
    return true;
}

__device__ void consumer(const DecodeParams& p, Smem& s) {
    const int G = gridDim.x;
    const int tid = threadIdx.x;
    uint32_t it = 0;
    int buf = 0;
    for (int f = 0; f < p.n_steps; ++f) {
        StepCtx st{f, p.pos0 + f, 0, false};
        int rot = 0;
        for (int ph = 0; ph < p.n_phases; ++ph) {
            const PhaseDesc& d = phase_at(p, ph);
            // 1. dependency on the previous phase (bounded), plus the first
            //    ring tile of this phase, awaited by thread 0.
            if (tid == 0) {
                bool ok = true;
                if (ph > 0)
                    ok = wait_counter(p, p.counters + ph - 1, static_cast<uint32_t>((f + 1) * G), ph, f);
                else if (f > 0)
                    ok = wait_counter(p, p.counters + p.n_phases - 1, static_cast<uint32_t>(f * G), ph, f);
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
                if (ok && d.kind == PH_GEMV) {
                    const int t_first = first_tile(rot, G);
                    if (t_first < d.n_tiles)
                        ok = wait_mbar(p, s, &s.full[it % kStages], (it / kStages) & 1u, false, ph, f);
                }
                s.phase_ok = ok ? 1 : 0;
                if (!ok) s.abort_flag = 1;
            }
            cbar();
            if (!s.phase_ok) return;
            bool ok = true;
            if (d.kind == PH_ATTN) {
                ok = attention_phase(p, s, d, st);
            } else {
                if (d.in_kind == IN_X0_NORM) {
                    st.token = s.token;
                    st.x0_given = (f == 0 && p.x0 != nullptr);
                    // Materialise x0 as the residual stream (and dump row 0).
                    for (int n = blockIdx.x * kConsumerThreads + tid; n < p.H; n += G * kConsumerThreads) {
                        const float v = x0_at(p, st, n);
                        p.x[n] = v;
                        if (p.dump) p.dump[n] = v;
                    }
                }
                ok = gemv_phase(p, s, d, st, ph, rot, it, buf);
                rot = (rot + d.n_tiles) % G;
            }
            if (!ok) {
                if (tid == 0) s.abort_flag = 1;
                return;
            }
            // 2. release this phase once all consumer threads wrote outputs.
            cbar();
            if (tid == 0) {
                __threadfence();
                red_release_gpu_add(p.counters + ph, 1u);
            }
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
            mbar_init(&s.empty[i], 1);
        }
        s.abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (tid >= kConsumerThreads) {
        if (tid == kConsumerThreads) producer(p, s);
        return;
    }
    consumer(p, s);
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
