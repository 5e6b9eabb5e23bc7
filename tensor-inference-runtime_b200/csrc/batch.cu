// batch.cu -- forward passes over many tokens at once: batched greedy decode
// of independent sequences and batched prefill (the reference feeds one token
// of one sequence per forward, src/lib.rs:239-314; every sequence here gets
// the same arithmetic up to f32 rounding order).  Layer by layer, every
// projection runs on the tensor-core Q8_0 matmul (gemm.cu); RMSNorm, RoPE +
// KV append, causal grouped-query attention, SwiGLU and the residual adds are
// small CUDA-core kernels.  All sequences of a batch advance in lockstep.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "host.h"
#include "launch.cuh"
#include "parts.cuh"
#include "planes.cuh"
#include "ptx.cuh"
#include "runtime.h"

namespace tir {
namespace {

constexpr uint32_t kBErrBadToken = 12;
constexpr int kQBlock = 32;   // query tokens per prefill attention CTA (one per lane)
constexpr int kPage = 16;     // KV-cache positions per page

// A step's row layout and the paged KV cache.  Row r of the step's q|k|v (and
// attention output) is token r - seq_row0[s] of sequence s = row_seq[r], at
// position seq_len[s] + that index; position p of sequence s lives in page
// table[s * max_pages + p / kPage], slot p % kPage.  The cache of one layer
// is [pages][kPage][kvd] floats for K and the same for V.
struct Pages {
    int32_t* seq_len;         // [n_seqs] tokens before this step (advanced at its end)
    const int32_t* seq_row0;  // [n_seqs] first row of the sequence's new tokens
    const int32_t* seq_cnt;   // [n_seqs] new tokens this step (0: idle)
    const int32_t* row_seq;   // [rows] sequence of each row
    const int32_t* table;     // [n_seqs][max_pages]
    int32_t max_pages;
};

__device__ __forceinline__ size_t kv_slot(const Pages& pg, int s, int pos, int kvd) {
    const int page = pg.table[static_cast<size_t>(s) * pg.max_pages + pos / kPage];
    return (static_cast<size_t>(page) * kPage + pos % kPage) * kvd;
}

// Q8_0 blocks of a matrix held in the decode kernel's warp-sliced tile-major
// layout (runtime.h q8_slice_offset), written back as [n][k/32] 34-byte blocks.
__global__ void tiled_to_blocks_kernel(const uint8_t* __restrict__ tiled, int64_t n, int64_t k,
                                       uint8_t* __restrict__ blocks) {
    const int64_t nb = k / 32;
    const int R = gemv_tile_rows(k), RL = gemv_row_lanes(k);
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n * nb;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t row = i / nb, b = i % nb;
        const int64_t t = row / R, rr = row % R;
        const int rl = static_cast<int>(rr % RL), j = static_cast<int>(rr / RL);
        const int wi = static_cast<int>(b / 32), bl = static_cast<int>(b % 32);
        const int nbw = q8_slice_blocks(k, wi), nbwp = (nbw + 7) / 8 * 8;
        const uint8_t* base = tiled + q8_slice_offset(k, t, rl, wi);
        const uint8_t* q = base + (static_cast<int64_t>(j) * nbw + bl) * 32;
        const uint8_t* sc = base + kTileMult * nbw * 32 + (j * nbwp + bl) * 2;
        uint8_t* dst = blocks + i * 34;
        dst[0] = sc[0];
        dst[1] = sc[1];
        for (int e = 0; e < 32; ++e) dst[2 + e] = q[e];
    }
}

// X[t] = embedding row ids[t] (src/tokenizer.rs:10-32: f32(q) * f32(scale)).
__global__ void embed_rows_kernel(const int32_t* __restrict__ ids, const uint8_t* __restrict__ eq,
                                  const uint16_t* __restrict__ es, int64_t esk, int H, int vocab,
                                  float* __restrict__ X, uint32_t* err) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t t = blockIdx.x;
    int id = ids[t];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) atomicCAS(err, 0u, kBErrBadToken);
        id = 0;
    }
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        const float sc = __half2float(__ushort_as_half(es[static_cast<int64_t>(id) * esk + c / 32]));
        X[t * H + c] = __fmul_rn(static_cast<float>(static_cast<int8_t>(eq[static_cast<int64_t>(id) * H + c])), sc);
    }
}

// RoPE on the q and k parts of each row's fused q|k|v (src/math.rs:196-228),
// then the KV-cache append (src/forward.rs:83-84) at the row's sequence and
// position (Pages).
__global__ void rope_append_kernel(float* __restrict__ qkv, int parts, int64_t part, int64_t ld, Pages pg, int H,
                                   int kvd, const float* __restrict__ rc, const float* __restrict__ rs,
                                   float* __restrict__ kc, float* __restrict__ vc) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t t = blockIdx.x;
    const int s = pg.row_seq[t];
    const int pos = pg.seq_len[s] + static_cast<int>(t - pg.seq_row0[s]);
    float* row = qkv + t * ld;
    // the q|k|v row: the sum of the matmul's partial tiles (into tile 0)
    sum_parts_inplace(row, parts, part, H + 2 * kvd);
    auto val = [&](int c) { return row[c]; };
    const size_t cache_row = kv_slot(pg, s, pos, kvd);
    for (int pr = threadIdx.x; pr < (H + kvd) / 2; pr += blockDim.x) {
        const int c = 2 * pr;
        const int i = (c % kHeadDim) >> 1;
        const float cs = rc[static_cast<size_t>(pos) * (kHeadDim / 2) + i];
        const float sn = rs[static_cast<size_t>(pos) * (kHeadDim / 2) + i];
        const float y0 = val(c), y1 = val(c + 1);
        const float e0 = __fadd_rn(__fmul_rn(cs, y0), __fmul_rn(-sn, y1));
        const float e1 = __fadd_rn(__fmul_rn(sn, y0), __fmul_rn(cs, y1));
        if (c < H) {  // the attention kernels read q (roped) from partial tile 0
            row[c] = e0;
            row[c + 1] = e1;
        } else {
            kc[cache_row + (c - H)] = e0;
            kc[cache_row + (c - H) + 1] = e1;
        }
    }
    for (int c = threadIdx.x; c < kvd; c += blockDim.x) vc[cache_row + c] = val(H + kvd + c);
}

// Causal grouped-query attention for tps >= 2 new tokens per sequence
// (src/forward.rs:79-174 for every query position): CTA per (sequence, kv
// head and group of up to kPHeads of its query heads, block of 32 query
// tokens); warp w handles one query head, lane i query token i of the block, with its q and running output in
// registers; keys are staged kPChunk positions at a time in shared memory and
// taken four at a time (four independent score chains, one running-max
// update per four keys).  Online softmax (running max and sum), scale
// 1/sqrt(64).
constexpr int kPChunk = 64;
constexpr int kPHeads = 8;  // query heads (warps) per CTA

__global__ void __launch_bounds__(kPHeads * 32, 1) attn_prefill_kernel(const float* __restrict__ qkv, int64_t ld,
                                                                      Pages pg, int H, int kvd, int group,
                                                                      const float* __restrict__ kc,
                                                                      const float* __restrict__ vc,
                                                                      float* __restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ __align__(16) float4 ks[kPChunk][kHeadDim / 4];
    __shared__ __align__(16) float4 vs[kPChunk][kHeadDim / 4];
    const int n_hb = (group + kPHeads - 1) / kPHeads;
    const int s = blockIdx.x, g = blockIdx.y / n_hb, hb = blockIdx.y % n_hb, qb = blockIdx.z;
    const int cnt = pg.seq_cnt[s];
    if (qb * kQBlock >= cnt) return;  // the whole CTA: no query of this sequence in the block
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hg = hb * kPHeads + warp;  // query head within the group
    const int h = g * group + hg;
    const int qi = qb * kQBlock + lane;  // query token within the sequence's new tokens
    const bool active = qi < cnt && hg < group;
    const int pos0 = pg.seq_len[s];
    const int qpos = pos0 + qi;
    const int64_t t = static_cast<int64_t>(pg.seq_row0[s]) + qi;
    float q[kHeadDim], o[kHeadDim];
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) {
        q[d] = active ? qkv[t * ld + h * kHeadDim + d] : 0.f;
        o[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int last = pos0 + min(cnt, (qb + 1) * kQBlock) - 1;  // the block's last query position
    for (int c0 = 0; c0 <= last; c0 += kPChunk) {
        __syncthreads();
        for (int e = threadIdx.x; e < kPChunk * (kHeadDim / 4); e += blockDim.x) {
            const int j = e / (kHeadDim / 4), d4 = e % (kHeadDim / 4);
            const bool in = c0 + j <= last;
            const size_t off = in ? kv_slot(pg, s, c0 + j, kvd) + static_cast<size_t>(g) * kHeadDim : 0;
            ks[j][d4] = in ? reinterpret_cast<const float4*>(kc + off)[d4] : make_float4(0.f, 0.f, 0.f, 0.f);
            vs[j][d4] = in ? reinterpret_cast<const float4*>(vc + off)[d4] : make_float4(0.f, 0.f, 0.f, 0.f);
        }
        __syncthreads();
        if (!active) continue;
        const int jmax = min(kPChunk, qpos - c0 + 1);
        int j = 0;
        for (; j + 4 <= jmax; j += 4) {
            float sc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 kv = ks[j + u][d4];
                    sc[u] = fmaf(q[4 * d4], kv.x, sc[u]);
                    sc[u] = fmaf(q[4 * d4 + 1], kv.y, sc[u]);
                    sc[u] = fmaf(q[4 * d4 + 2], kv.z, sc[u]);
                    sc[u] = fmaf(q[4 * d4 + 3], kv.w, sc[u]);
                }
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) sc[u] = sc[u] / 8.0f;  // sqrt(64)
            const float mx = fmaxf(fmaxf(sc[0], sc[1]), fmaxf(sc[2], sc[3]));
            if (mx > m) {
                const float corr = expf(m - mx);
                l *= corr;
#pragma unroll
                for (int d = 0; d < kHeadDim; ++d) o[d] *= corr;
                m = mx;
            }
            float pj[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                pj[u] = expf(sc[u] - m);
                l += pj[u];
            }
#pragma unroll
            for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float4 vv = vs[j + u][d4];
                    o[4 * d4] = fmaf(pj[u], vv.x, o[4 * d4]);
                    o[4 * d4 + 1] = fmaf(pj[u], vv.y, o[4 * d4 + 1]);
                    o[4 * d4 + 2] = fmaf(pj[u], vv.z, o[4 * d4 + 2]);
                    o[4 * d4 + 3] = fmaf(pj[u], vv.w, o[4 * d4 + 3]);
                }
            }
        }
        for (; j < jmax; ++j) {
            float acc = 0.f;
#pragma unroll
            for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
                const float4 kv = ks[j][d4];
                acc = fmaf(q[4 * d4], kv.x, acc);
                acc = fmaf(q[4 * d4 + 1], kv.y, acc);
                acc = fmaf(q[4 * d4 + 2], kv.z, acc);
                acc = fmaf(q[4 * d4 + 3], kv.w, acc);
            }
            const float sc = acc / 8.0f;
            if (sc > m) {
                const float corr = expf(m - sc);
                l *= corr;
#pragma unroll
                for (int d = 0; d < kHeadDim; ++d) o[d] *= corr;
                m = sc;
            }
            const float pj = expf(sc - m);
            l += pj;
#pragma unroll
            for (int d4 = 0; d4 < kHeadDim / 4; ++d4) {
                const float4 vv = vs[j][d4];
                o[4 * d4] = fmaf(pj, vv.x, o[4 * d4]);
                o[4 * d4 + 1] = fmaf(pj, vv.y, o[4 * d4 + 1]);
                o[4 * d4 + 2] = fmaf(pj, vv.z, o[4 * d4 + 2]);
                o[4 * d4 + 3] = fmaf(pj, vv.w, o[4 * d4 + 3]);
            }
        }
    }
    if (active) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) out[t * H + h * kHeadDim + d] = o[d] * inv;
    }
}

// One new token per sequence (decode), src/forward.rs:79-174: CTA per
// (sequence, kv head).  The CTA finishes the q|k|v projection for its kv head
// (the sum of the matmul's `parts` partial tiles), applies RoPE to its query
// heads and key (src/math.rs:196-228) and appends key and value to the cache
// (src/forward.rs:83-84).  Key and value rows are read from shared memory, in
// windows of kAttnWin positions staged with cp.async.  The first window is
// requested before the wait on the q|k|v matmul: the positions before the
// new one were written by earlier forwards, and every forward starts after a
// stream operation that is not a programmatic launch (the decode graph's
// launch, or the copy of the step layout), so those forwards are complete;
// the page table and the step layout do not change during a forward.  Warp w
// takes the 32-key chunks w, w + kAttnWarps, ... of a window: lane j scores
// key j against every query head of the group (queries in shared memory),
// the chunk's probabilities go to shared memory, and the warp folds the
// chunk into a running (max, sum, output) per head with lanes over output
// dimensions; the warps' states merge at the end.  Scale 1/sqrt(64), softmax
// with the running-max shift.  The last of a sequence's kv-head CTAs to
// finish (head_done[s] counts them and is reset by that CTA) turns the
// sequence's output row into the activation planes of the o projection
// (planes.cuh), which the plane writer would otherwise do as a kernel of its
// own.
constexpr int kAttnWarps = 8;
constexpr int kAttnWin = 176;         // positions per staged window (two CTAs per SM)
constexpr int kKVPad = kHeadDim + 4;  // floats per staged row: 16-byte reads of 8 rows hit distinct banks
constexpr int kAttnPid = 256;         // page ids staged in shared memory (later pages: read from the table)
constexpr size_t kAttnDynSmem = 2u * kAttnWin * kKVPad * sizeof(float);  // [K | V][row][kKVPad]
static_assert(kAttnWarps * 32 == kPlaneThreads, "the decode attention CTA writes planes with all its threads");
constexpr int kMaxParts = 16;  // split-K partial tiles a reader sums

template <int G>  // query heads per kv head, rounded up (heads >= group are computed on zeros, not stored)
__global__ void __launch_bounds__(kAttnWarps * 32, 2) attn_decode_kernel(const float* __restrict__ qkv, int parts,
                                                                      int64_t part, int64_t ld, Pages pg, int H,
                                                                      int kvd, int group, const float* __restrict__ rc,
                                                                      const float* __restrict__ rs,
                                                                      float* __restrict__ kc,
                                                                      float* __restrict__ vc,
                                                                      float* __restrict__ out,
                                                                      uint32_t* __restrict__ head_done, int nt,
                                                                      uint8_t* __restrict__ planes,
                                                                      float* __restrict__ inv) {
    __shared__ __align__(16) float qs[G][kHeadDim];
    __shared__ __align__(16) float ps[kAttnWarps][32][G];  // a chunk's probabilities, [key][head]
    __shared__ int32_t pid[kAttnPid];
    __shared__ float ms[kAttnWarps][G], ls[kAttnWarps][G];
    extern __shared__ __align__(16) float kvs[];  // [K | V][kAttnWin][kKVPad]; then the warps' outputs
    static_assert(kAttnWarps * G * kHeadDim <= 2 * kAttnWin * kKVPad, "the warps' outputs fit the window");
    griddep_launch_dependents();
    const int s = blockIdx.x, g = blockIdx.y;
    const bool idle = pg.seq_cnt[s] == 0;  // the whole CTA: the sequence has no token this step
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = pg.seq_len[s], n = pos + 1;
    const size_t head = static_cast<size_t>(g) * kHeadDim;
    const int32_t* table = pg.table + static_cast<size_t>(s) * pg.max_pages;
    if (!idle)
        for (int i = threadIdx.x; i < min((n + kPage - 1) / kPage, kAttnPid); i += blockDim.x) pid[i] = table[i];
    __syncthreads();
    auto slot = [&](int j) {  // cache offset of position j's row of this kv head
        const int page = j / kPage < kAttnPid ? pid[j / kPage] : table[j / kPage];
        return (static_cast<size_t>(page) * kPage + j % kPage) * kvd + head;
    };
    // window w's rows, 16 sixteen-byte pieces of K, then of V, per position;
    // the new position only after it is written (w > 0)
    auto stage = [&](int w) {
        const int j0 = w * kAttnWin, cnt = min(n - j0, kAttnWin);
        for (int e = threadIdx.x; e < cnt * 32; e += blockDim.x) {
            const int jr = e >> 5, c = e & 31, isv = c >> 4;
            if (j0 + jr == pos && w == 0) continue;
            cp_async16(kvs + (isv * kAttnWin + jr) * kKVPad + (c & 15) * 4, (isv ? vc : kc) + slot(j0 + jr) + (c & 15) * 4);
        }
        cp_async_commit();
    };
    if (!idle) stage(0);
    griddep_wait();
    if (idle) return;
    const int64_t r = pg.seq_row0[s];  // the sequence's row in this step
    const float* row = qkv + r * ld;
    auto val = [&](int c) {  // partial loads first, then the sum in partial order
        float v[kMaxParts];
#pragma unroll
        for (int j = 0; j < kMaxParts; ++j) v[j] = j < parts ? row[j * part + c] : 0.f;
        float acc = v[0];
#pragma unroll
        for (int j = 1; j < kMaxParts; ++j)
            if (j < parts) acc = __fadd_rn(acc, v[j]);
        return acc;
    };
    const size_t cache_row = slot(pos);
    float* const win_k = pos < kAttnWin ? kvs + pos * kKVPad : nullptr;  // the new row's staged copy, if in window 0
    for (int pr = threadIdx.x; pr < (group + 1) * (kHeadDim / 2); pr += blockDim.x) {
        const bool isq = pr < group * (kHeadDim / 2);
        const int i = pr % (kHeadDim / 2);  // rotation pair within the head
        const int c = isq ? (g * group) * kHeadDim + 2 * pr : H + g * kHeadDim + 2 * i;
        const float cs = rc[static_cast<size_t>(pos) * (kHeadDim / 2) + i];
        const float sn = rs[static_cast<size_t>(pos) * (kHeadDim / 2) + i];
        const float y0 = val(c), y1 = val(c + 1);
        const float e0 = __fadd_rn(__fmul_rn(cs, y0), __fmul_rn(-sn, y1));
        const float e1 = __fadd_rn(__fmul_rn(sn, y0), __fmul_rn(cs, y1));
        if (isq) {
            qs[pr / (kHeadDim / 2)][2 * i] = e0;
            qs[pr / (kHeadDim / 2)][2 * i + 1] = e1;
        } else {
            kc[cache_row + 2 * i] = e0;
            kc[cache_row + 2 * i + 1] = e1;
            if (win_k) {
                win_k[2 * i] = e0;
                win_k[2 * i + 1] = e1;
            }
        }
    }
    for (int d = threadIdx.x; d < kHeadDim; d += blockDim.x) {
        const float v = val(H + kvd + g * kHeadDim + d);
        vc[cache_row + d] = v;
        if (win_k) win_k[kAttnWin * kKVPad + d] = v;
    }
    for (int e = group * kHeadDim + threadIdx.x; e < G * kHeadDim; e += blockDim.x) qs[e / kHeadDim][e % kHeadDim] = 0.f;
    __threadfence_block();  // the new row reaches the cache before a later window's copy reads it back
    float m[G], l[G], o0[G], o1[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
        o0[h] = 0.f;
        o1[h] = 0.f;
    }
    const float* kb = kvs;
    const float* vb = kvs + kAttnWin * kKVPad;
    for (int j0 = 0; j0 < n; j0 += kAttnWin) {
        if (j0 > 0) {
            __syncthreads();  // every warp is done with the previous window
            stage(j0 / kAttnWin);
        }
        cp_async_wait_all();
        __syncthreads();  // the window landed (and, at the first, the queries and the new row are staged)
        const int cnt = min(n - j0, kAttnWin);
        for (int c0 = warp * 32; c0 < cnt; c0 += kAttnWarps * 32) {
            const int jr = c0 + lane;
            const bool valid = jr < cnt;
            float p[G];
#pragma unroll
            for (int h = 0; h < G; ++h) p[h] = 0.f;
            const float4* kr = reinterpret_cast<const float4*>(kb + (valid ? jr : c0) * kKVPad);
#pragma unroll 4
            for (int i = 0; i < kHeadDim / 4; ++i) {
                const float4 kv = kr[i];
#pragma unroll
                for (int h = 0; h < G; ++h) {
                    const float4 qv = reinterpret_cast<const float4*>(qs[h])[i];
                    p[h] = fmaf(qv.x, kv.x, p[h]);
                    p[h] = fmaf(qv.y, kv.y, p[h]);
                    p[h] = fmaf(qv.z, kv.z, p[h]);
                    p[h] = fmaf(qv.w, kv.w, p[h]);
                }
            }
#pragma unroll
            for (int h = 0; h < G; ++h) p[h] = valid ? p[h] / 8.0f : -INFINITY;  // sqrt(64)
#pragma unroll
            for (int h = 0; h < G; ++h) {
                float mx = p[h];
#pragma unroll
                for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
                const float m_new = fmaxf(m[h], mx);  // finite: lane 0 of the chunk is a valid key
                const float pj = valid ? expf(p[h] - m_new) : 0.f;
                float sum = pj;
#pragma unroll
                for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
                const float corr = expf(m[h] - m_new);
                l[h] = l[h] * corr + sum;
                o0[h] *= corr;
                o1[h] *= corr;
                m[h] = m_new;
                ps[warp][lane][h] = pj;
            }
            __syncwarp();
            // value rows eight keys at a time, folded in key order, with the
            // keys' probabilities of every head read back as vectors
            const int nc = min(32, cnt - c0);
            for (int u0 = 0; u0 < nc; u0 += 8) {
                float v0[8], v1[8];
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const float* vr = vb + (c0 + min(u0 + u, nc - 1)) * kKVPad;
                    v0[u] = vr[lane];
                    v1[u] = vr[lane + 32];
                }
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    if (u0 + u < nc) {
                        float pt[G];
                        if constexpr (G % 4 == 0) {
#pragma unroll
                            for (int h4 = 0; h4 < G / 4; ++h4) {
                                const float4 q4 = reinterpret_cast<const float4*>(ps[warp][u0 + u])[h4];
                                pt[4 * h4] = q4.x;
                                pt[4 * h4 + 1] = q4.y;
                                pt[4 * h4 + 2] = q4.z;
                                pt[4 * h4 + 3] = q4.w;
                            }
                        } else {
#pragma unroll
                            for (int h = 0; h < G; ++h) pt[h] = ps[warp][u0 + u][h];
                        }
#pragma unroll
                        for (int h = 0; h < G; ++h) {
                            o0[h] = fmaf(pt[h], v0[u], o0[h]);
                            o1[h] = fmaf(pt[h], v1[u], o1[h]);
                        }
                    }
                }
            }
            __syncwarp();  // ps is rewritten by the warp's next chunk
        }
    }
    float(*os)[G][kHeadDim] = reinterpret_cast<float(*)[G][kHeadDim]>(kvs);  // [warp][head][dim]
    __syncthreads();  // every warp is done with the window
#pragma unroll
    for (int h = 0; h < G; ++h) {
        if (lane == 0) {
            ms[warp][h] = m[h];
            ls[warp][h] = l[h];
        }
        os[warp][h][lane] = o0[h];
        os[warp][h][lane + 32] = o1[h];
    }
    __syncthreads();
    for (int e = threadIdx.x; e < group * kHeadDim; e += blockDim.x) {
        const int h = e / kHeadDim, d = e % kHeadDim;
        float mx = ms[0][h];
#pragma unroll
        for (int w = 1; w < kAttnWarps; ++w) mx = fmaxf(mx, ms[w][h]);
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < kAttnWarps; ++w) {
            const float f = expf(ms[w][h] - mx);  // 0 for a warp that had no keys
            L = fmaf(ls[w][h], f, L);
            O = fmaf(os[w][h][d], f, O);
        }
        out[r * H + (g * group + h) * kHeadDim + d] = O / L;
    }
    __shared__ bool last;
    __syncthreads();  // the CTA's part of the row is written
    if (threadIdx.x == 0) {
        // acquire-release count: this CTA's part is visible before it, and the
        // last CTA sees every other head's part
        last = atom_add_acq_rel_gpu(&head_done[s], 1u) == gridDim.y - 1;
        if (last) head_done[s] = 0;  // ready for the next launch
    }
    __syncthreads();
    if (!last) return;
    const int nc = plane_chunks(H);
    float v[kPlaneMaxChunks * 8];
#pragma unroll
    for (int i = 0; i < kPlaneMaxChunks; ++i)
        if (i < nc) load8_cg(out + r * H + (threadIdx.x + i * kPlaneThreads) * 8, v + 8 * i);
    planes_store(v, nc, true, r, H, nt, planes, inv);
}

// Greedy sample per row (src/tokenizer.rs:152-167: total order, ties -> last)
// of logits that are the sum of `parts` partial tiles `part` floats apart.
__global__ void argmax_rows_kernel(const float* __restrict__ x, int parts, int64_t part, int64_t n,
                                   int32_t* __restrict__ out) {
    griddep_launch_dependents();
    griddep_wait();
    __shared__ unsigned long long red[32];
    const float* r = x + static_cast<int64_t>(blockIdx.x) * n;
    unsigned long long best = 0ull;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        float v = r[i];
        for (int j = 1; j < parts; ++j) v = __fadd_rn(v, r[j * part + i]);
        const uint32_t b = __float_as_uint(v);
        const uint32_t key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
        best = max(best, (static_cast<unsigned long long>(key) << 32) | static_cast<uint32_t>(i));
    }
    for (int o = 16; o; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned long long b = 0ull;
        for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) b = max(b, red[i]);
        out[blockIdx.x] = static_cast<int32_t>(b & 0xffffffffu);
    }
}

// Each sequence's last new row (-1 for an idle sequence: its logits row is
// zeros, and no live row is gathered twice); then every sequence's device
// length advances by its new tokens (every kernel of the forward that reads it
// has run by now).
// Layer outputs of the dumped rows: out[i] = X[rows[i]] + (Y's partial tiles
// summed in order), the residual add the next rmsnorm kernel would do (Y null:
// X as it is).
__global__ void dump_rows_kernel(const float* __restrict__ X, const float* __restrict__ Y, int parts, int64_t part,
                                 const int32_t* __restrict__ rows, int H, float* __restrict__ out, int64_t out_ld) {
    const int i = blockIdx.x;
    const int64_t r = rows[i];
    for (int c = threadIdx.x; c < H; c += blockDim.x) {
        float v = X[r * H + c];
        if (Y) {
            float y = Y[r * H + c];
            for (int j = 1; j < parts; ++j) y += Y[j * part + r * H + c];
            v += y;
        }
        out[static_cast<int64_t>(i) * out_ld + c] = v;
    }
}

__global__ void last_rows_kernel(int32_t* rows, Pages pg, int n_seqs) {
    griddep_launch_dependents();
    griddep_wait();
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < n_seqs) {
        const int cnt = pg.seq_cnt[s];
        rows[s] = cnt > 0 ? pg.seq_row0[s] + cnt - 1 : -1;
        pg.seq_len[s] += cnt;
    }
}

// Greedy decode feedback: the sampled ids are both the next input and
// generated output.
__global__ void feed_kernel(const int32_t* __restrict__ next, int32_t* __restrict__ ids, int32_t* __restrict__ gen,
                            int n_seqs) {
    griddep_launch_dependents();
    griddep_wait();
    for (int s = blockIdx.x * blockDim.x + threadIdx.x; s < n_seqs; s += gridDim.x * blockDim.x) {
        const int32_t v = next[s];
        ids[s] = v;
        gen[s] = v;
    }
}

unsigned g1(int64_t n, int threads) { return static_cast<unsigned>(std::min<int64_t>((n + threads - 1) / threads, 148 * 16)); }

}  // namespace
}  // namespace tir

using namespace tir;

struct tir_batch {
    struct GW {
        uint8_t* w = nullptr;
        float* p2 = nullptr;
        int64_t n = 0, k = 0;
    };
    tir_model* m = nullptr;
    int B = 0, max_ctx = 0, max_tps = 0, sms = 148;
    int max_pages = 0, n_pages = 0;  // pages per sequence at most; pages in the pool
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    std::vector<GW> qkv, o, gu, down;
    GW lm;
    float *kc = nullptr, *vc = nullptr, *rcos = nullptr, *rsin = nullptr;  // kc, vc: [layers][n_pages][kPage][kvd]
    float *X = nullptr, *Y = nullptr, *QKV = nullptr, *ATT = nullptr, *GU = nullptr, *LG = nullptr, *inv = nullptr;
    uint8_t* planes = nullptr;
    int32_t *ids = nullptr, *rows = nullptr, *next = nullptr, *h_next = nullptr;
    float* logits = nullptr;  // [B][V] summed lm_head rows (allocated on first tir_batch_logits)
    int lm_parts = 0;         // partial tiles of the last forward's lm_head output (0: no forward yet)
    uint32_t *err = nullptr, *h_err = nullptr;
    uint32_t* head_done = nullptr;  // [B] kv-head CTAs of the decode attention done (zero between launches)
    // Sequences and pages.  seq_len lives on the device (kernels read and
    // advance it, so graph replays stay valid); h_len mirrors it.
    int32_t* seq_len = nullptr;
    std::vector<int32_t> h_len;
    std::vector<std::vector<int32_t>> seq_pages;  // pages of each sequence, in position order
    std::vector<int32_t> free_pages;
    int32_t *table = nullptr, *h_table = nullptr;  // [B][max_pages], device and pinned host
    bool table_dirty = false;
    // Step layouts ([row0 B | cnt B | row_seq]): dyn for any step (pinned
    // host copy h_dyn), uni = every sequence one token (constant; the decode
    // graph reads it).
    int32_t *dyn = nullptr, *h_dyn = nullptr, *uni = nullptr;
    int32_t* gen = nullptr;  // generated ids [gen_cap][B] (tir_batch_generate)
    int gen_cap = 0;
    cudaGraphExec_t decode_graph = nullptr;  // one decode forward on `uni`, captured on first use
    bool capturing = false;                  // forward() is being recorded into decode_graph
    // tir_batch_dump_rows: per-layer outputs of chosen rows of the forwards
    // run outside the decode graph, [n][layers][H] (rows in step-row order).
    std::vector<int32_t> dump_rows;
    float* dump = nullptr;
    int32_t* dump_idx = nullptr;
    ~tir_batch() {
        cudaSetDevice(m ? m->device : 0);
        if (stream) cudaStreamSynchronize(stream);
        if (decode_graph) cudaGraphExecDestroy(decode_graph);
        if (gen) cudaFree(gen);
        if (logits) cudaFree(logits);
        if (dump) cudaFree(dump);
        if (dump_idx) cudaFree(dump_idx);
        for (void* p : allocs) cudaFree(p);
        if (h_next) cudaFreeHost(h_next);
        if (h_err) cudaFreeHost(h_err);
        if (h_table) cudaFreeHost(h_table);
        if (h_dyn) cudaFreeHost(h_dyn);
        if (stream) cudaStreamDestroy(stream);
    }
};

namespace {

tir_status bfail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? TIR_ERR_OOM : TIR_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorName(e));
}

template <class T>
bool balloc(tir_batch* b, size_t bytes, T** p) {
    void* q = nullptr;
    if (dev_malloc(&q, bytes ? bytes : 16) != cudaSuccess) return false;
    b->allocs.push_back(q);
    *p = static_cast<T*>(q);
    return true;
}

// Tensor-core layout of one decode-layout matrix (via a Q8_0 block staging buffer).
tir_status make_gw(tir_batch* b, const Mat& mt, uint8_t* staging, tir_batch::GW& g) {
    g.n = mt.n;
    g.k = mt.k;
    if (!balloc(b, static_cast<size_t>(gemm_q8_weight_bytes(mt.n, mt.k)), &g.w) ||
        !balloc(b, static_cast<size_t>(gemm_q8_rows_padded(mt.n)) * 4, &g.p2))
        return fail(TIR_ERR_OOM, "tensor-core weight allocation failed");
    tiled_to_blocks_kernel<<<g1(mt.n * (mt.k / 32), 256), 256, 0, b->stream>>>(mt.q, mt.n, mt.k, staging);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bfail(e, "weight layout");
    const int rc = launch_gemm_repack(staging, mt.n, mt.k, g.w, g.p2, b->stream);
    if (rc != 0) return bfail(static_cast<cudaError_t>(rc), "weight layout");
    return TIR_OK;
}

// The matmul of the activation planes in b->planes (as written for `tokens`
// rows) with g: *parts partial tiles of tokens x g.n floats from y on, whose
// sum in order is the product.
tir_status mm(tir_batch* b, int64_t tokens, const tir_batch::GW& g, float* y, int* parts) {
    const int splits = gemm_real_splits(g.k, gemm_splits(g.n, g.k, tokens, b->sms));
    if (splits > kMaxParts) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "more split-K partial tiles than a reader sums");
    const int rc = launch_gemm_q8(g.w, g.p2, b->planes, b->inv, g.n, g.k, tokens, y, g.n, splits, b->err,
                                  timeout_ns(), b->stream, true);
    if (rc != 0) return bfail(static_cast<cudaError_t>(rc), "tensor-core matmul");
    *parts = splits;
    return TIR_OK;
}

tir_status planes_rc(int rc) {
    return rc == 0 ? TIR_OK : bfail(static_cast<cudaError_t>(rc), "activation planes");
}

// The step layout `meta` ([row0 B | cnt B | row_seq]) as kernel arguments.
Pages pages_of(tir_batch* b, const int32_t* meta) {
    Pages pg;
    pg.seq_len = b->seq_len;
    pg.seq_row0 = meta;
    pg.seq_cnt = meta + b->B;
    pg.row_seq = meta + 2 * b->B;
    pg.table = b->table;
    pg.max_pages = b->max_pages;
    return pg;
}

// Decode attention (with the q|k|v partial sum, RoPE and KV append) over the
// group size rounded up to an instantiated width.
void attn_decode(tir_batch* b, const Pages& pg, int64_t rows, int parts, int group, int kv_heads, int H, int KVD,
                 int64_t ldq, float* kc, float* vc) {
    const dim3 grid(static_cast<unsigned>(b->B), static_cast<unsigned>(kv_heads));
    const unsigned th = kAttnWarps * 32;
    const int64_t part = rows * ldq;
#define TIR_ATTN(GM)                                                                                                   \
    do {                                                                                                               \
        cudaFuncSetAttribute(attn_decode_kernel<GM>, cudaFuncAttributeMaxDynamicSharedMemorySize,                      \
                             static_cast<int>(kAttnDynSmem));                                                          \
        launch_kernel(attn_decode_kernel<GM>, grid, dim3(th), kAttnDynSmem, b->stream, true, b->QKV, parts, part, ldq, \
                      pg, H, KVD, group, b->rcos, b->rsin, kc, vc, b->ATT, b->head_done, gemm_token_tile(rows),        \
                      b->planes, b->inv);                                                                              \
    } while (0)
    if (group <= 1)
        TIR_ATTN(1);
    else if (group <= 2)
        TIR_ATTN(2);
    else if (group <= 4)
        TIR_ATTN(4);
    else if (group <= 8)
        TIR_ATTN(8);
    else
        TIR_ATTN(16);
#undef TIR_ATTN
}

// One forward over the step layout `meta` (T rows; ids already in b->ids,
// sequence-major); greedy next id of every sequence into b->next.
// max_cnt: the most new tokens of one sequence (1: the decode attention, which
// also does RoPE and the KV append).  Per layer: the previous layer's residual
// add + rmsnorm fused into the activation planes of the q|k|v matmul, RoPE +
// KV append, attention, the o matmul (into Y), residual add + rmsnorm into the
// gate|up planes, SiLU * up into the down planes, the down matmul (into Y,
// added by the next norm).
tir_status forward(tir_batch* b, const int32_t* meta, int64_t T, int max_cnt) {
    tir_model* m = b->m;
    const tir_transformer& t = m->t;
    const int H = static_cast<int>(t.embed_dim), KVD = static_cast<int>(t.kv_dim), F = static_cast<int>(t.ffn_dim);
    const int V = static_cast<int>(t.vocab), L = static_cast<int>(t.layers);
    const int group = static_cast<int>(t.q_heads / t.k_v_heads);
    const int64_t ldq = H + 2 * KVD;
    const size_t layer_cache = static_cast<size_t>(b->n_pages) * kPage * KVD;
    const Pages pg = pages_of(b, meta);
    cudaStream_t st = b->stream;
    tir_status rc;
    launch_kernel(embed_rows_kernel, dim3(static_cast<unsigned>(T)), dim3(256), 0, st, true, b->ids, m->embd.q,
                  m->embd.s, m->embd.sk, H, V, b->X, b->err);
    int parts = 0, y_parts = 0;  // partial tiles of the latest matmul / of the one in Y
    const int n_dump = b->capturing ? 0 : static_cast<int>(b->dump_rows.size());
    auto dump_layer = [&](int l, const float* Y, int y_p) {  // output of layer l (0-based) into dump[row][l]
        dump_rows_kernel<<<n_dump, 256, 0, st>>>(b->X, Y, y_p, T * H, b->dump_idx, H,
                                                 b->dump + static_cast<size_t>(l) * H, static_cast<int64_t>(L) * H);
    };
    for (int i = 0; i < n_dump; ++i)
        if (b->dump_rows[static_cast<size_t>(i)] >= T) return fail(TIR_ERR_INVALID_ARG, "a dumped row is past the step's rows");
    for (int l = 0; l < L; ++l) {
        if (n_dump > 0 && l > 0) dump_layer(l - 1, b->Y, y_parts);
        // the residual add of the previous layer's down projection (none before layer 0)
        if ((rc = planes_rc(launch_gemm_norm_planes(b->X, l > 0 ? b->Y : nullptr, y_parts, T * H, nullptr, T, H,
                                                    m->attn_norm[l], 1e-5f, b->planes, b->inv, st, true))) != TIR_OK)
            return rc;
        if ((rc = mm(b, T, b->qkv[l], b->QKV, &parts)) != TIR_OK) return rc;
        float* kc = b->kc + l * layer_cache;
        float* vc = b->vc + l * layer_cache;
        if (max_cnt <= 1) {
            attn_decode(b, pg, T, parts, group, static_cast<int>(t.k_v_heads), H, KVD, ldq, kc, vc);  // + the planes
        } else {
            launch_kernel(rope_append_kernel, dim3(static_cast<unsigned>(T)), dim3(256), 0, st, true, b->QKV, parts,
                          T * ldq, ldq, pg, H, KVD, b->rcos, b->rsin, kc, vc);
            launch_kernel(attn_prefill_kernel,
                          dim3(b->B, static_cast<unsigned>(t.k_v_heads * ((group + kPHeads - 1) / kPHeads)),
                               (max_cnt + kQBlock - 1) / kQBlock),
                          dim3(kPHeads * 32), 0, st, true, b->QKV, ldq, pg, H, KVD, group, kc, vc, b->ATT);
            if ((rc = planes_rc(launch_gemm_x_planes(b->ATT, T, H, b->planes, b->inv, st, true))) != TIR_OK) return rc;
        }
        if ((rc = mm(b, T, b->o[l], b->Y, &y_parts)) != TIR_OK) return rc;
        if ((rc = planes_rc(launch_gemm_norm_planes(b->X, b->Y, y_parts, T * H, nullptr, T, H, m->ffn_norm[l], 1e-5f,
                                                    b->planes, b->inv, st, true))) != TIR_OK)
            return rc;
        if ((rc = mm(b, T, b->gu[l], b->GU, &parts)) != TIR_OK) return rc;
        if ((rc = planes_rc(launch_gemm_silu_planes(b->GU, parts, T * 2 * F, T, F, b->planes, b->inv, st, true))) !=
            TIR_OK)
            return rc;
        if ((rc = mm(b, T, b->down[l], b->Y, &y_parts)) != TIR_OK) return rc;
    }
    if (n_dump > 0 && L > 0) dump_layer(L - 1, b->Y, y_parts);
    launch_kernel(last_rows_kernel, dim3((b->B + 127) / 128), dim3(128), 0, st, true, b->rows, pg, b->B);
    // the last down projection's residual add, on the rows the logits need
    if ((rc = planes_rc(launch_gemm_norm_planes(b->X, b->Y, y_parts, T * H, b->rows, b->B, H, m->out_norm, 1e-5f,
                                                b->planes, b->inv, st, true))) != TIR_OK)
        return rc;
    if ((rc = mm(b, b->B, b->lm, b->LG, &parts)) != TIR_OK) return rc;
    b->lm_parts = parts;
    launch_kernel(argmax_rows_kernel, dim3(static_cast<unsigned>(b->B)), dim3(256), 0, st, true, b->LG, parts,
                  static_cast<int64_t>(b->B) * V, static_cast<int64_t>(V), b->next);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bfail(e, "batched forward");
    return TIR_OK;
}

// Pages for positions [0, new_len) of sequence s, from the pool; TIR_ERR_OOM
// (nothing taken) when the pool runs short.
tir_status ensure_pages(tir_batch* b, int s, int new_len) {
    const size_t need = static_cast<size_t>((new_len + kPage - 1) / kPage);
    std::vector<int32_t>& mine = b->seq_pages[static_cast<size_t>(s)];
    if (need <= mine.size()) return TIR_OK;
    if (need - mine.size() > b->free_pages.size()) return fail(TIR_ERR_OOM, "the batch's KV page pool is exhausted");
    while (mine.size() < need) {
        const int32_t pgid = b->free_pages.back();
        b->free_pages.pop_back();
        b->h_table[static_cast<size_t>(s) * b->max_pages + mine.size()] = pgid;
        mine.push_back(pgid);
    }
    b->table_dirty = true;
    return TIR_OK;
}

tir_status upload_table(tir_batch* b) {
    if (!b->table_dirty) return TIR_OK;
    const cudaError_t e = cudaMemcpyAsync(b->table, b->h_table, static_cast<size_t>(b->B) * b->max_pages * 4,
                                          cudaMemcpyHostToDevice, b->stream);
    if (e != cudaSuccess) return bfail(e, "page table upload");
    b->table_dirty = false;
    return TIR_OK;
}

// Sequence s empties: its pages back to the pool, its length 0 (host and device).
tir_status release_seq(tir_batch* b, int s) {
    std::vector<int32_t>& mine = b->seq_pages[static_cast<size_t>(s)];
    for (auto it = mine.rbegin(); it != mine.rend(); ++it) b->free_pages.push_back(*it);
    mine.clear();
    b->h_len[static_cast<size_t>(s)] = 0;
    const cudaError_t e = cudaMemsetAsync(b->seq_len + s, 0, 4, b->stream);
    return e == cudaSuccess ? TIR_OK : bfail(e, "sequence reset");
}

// Every sequence empty.  Pages may still be in use by queued work: the
// stream is drained first.
tir_status reset_all(tir_batch* b) {
    cudaError_t e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return bfail(e, "batch reset");
    for (int s = 0; s < b->B; ++s) {
        const tir_status rc = release_seq(b, s);
        if (rc != TIR_OK) return rc;
    }
    return TIR_OK;
}

// Decode forward on the constant one-token-per-sequence layout, through a
// CUDA graph captured on first use: the launch sequence depends only on the
// batch's buffers, and every kernel reads positions and pages from the device.
tir_status decode_forward(tir_batch* b) {
    if (!b->decode_graph) {
        cudaGraph_t g = nullptr;
        cudaError_t e = cudaStreamBeginCapture(b->stream, cudaStreamCaptureModeThreadLocal);
        if (e != cudaSuccess) return bfail(e, "decode graph capture");
        b->capturing = true;
        const tir_status rc = forward(b, b->uni, b->B, 1);
        b->capturing = false;
        e = cudaStreamEndCapture(b->stream, &g);
        if (rc != TIR_OK) {
            if (g) cudaGraphDestroy(g);
            return rc;
        }
        if (e != cudaSuccess) return bfail(e, "decode graph capture");
        e = cudaGraphInstantiate(&b->decode_graph, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) {
            b->decode_graph = nullptr;
            return bfail(e, "decode graph instantiation");
        }
    }
    const cudaError_t e = cudaGraphLaunch(b->decode_graph, b->stream);
    if (e != cudaSuccess) return bfail(e, "decode graph launch");
    for (int32_t& l : b->h_len) l += 1;
    return TIR_OK;
}

// Validates and lays out a step with counts[s] new tokens of sequence s
// (ids in sequence order), takes the pages it needs and uploads the layout,
// the page table and the ids.  *T = rows, *max_cnt = the largest count.
tir_status stage_step(tir_batch* b, const int32_t* ids_host, const int32_t* counts, int64_t* T, int* max_cnt) {
    int64_t rows = 0;
    int mc = 0;
    for (int s = 0; s < b->B; ++s) {
        const int c = counts[s];
        if (c < 0 || c > b->max_tps)
            return fail(TIR_ERR_INVALID_ARG, "a sequence's token count must be in [0, " + std::to_string(b->max_tps) +
                                                 "]");
        if (b->h_len[static_cast<size_t>(s)] + c > b->max_ctx)
            return fail(TIR_ERR_CTX_OVERFLOW, "sequence " + std::to_string(s) + " would exceed the batch context");
        rows += c;
        mc = std::max(mc, c);
    }
    // pages: all or nothing
    size_t need = 0;
    for (int s = 0; s < b->B; ++s) {
        const size_t want = static_cast<size_t>((b->h_len[static_cast<size_t>(s)] + counts[s] + kPage - 1) / kPage);
        need += want > b->seq_pages[static_cast<size_t>(s)].size() ? want - b->seq_pages[static_cast<size_t>(s)].size()
                                                                  : 0;
    }
    if (need > b->free_pages.size()) return fail(TIR_ERR_OOM, "the batch's KV page pool is exhausted");
    for (int s = 0; s < b->B; ++s) {
        const tir_status rc = ensure_pages(b, s, b->h_len[static_cast<size_t>(s)] + counts[s]);
        if (rc != TIR_OK) return rc;
    }
    int32_t* row0 = b->h_dyn;
    int32_t* cnt = b->h_dyn + b->B;
    int32_t* row_seq = b->h_dyn + 2 * b->B;
    int64_t r = 0;
    for (int s = 0; s < b->B; ++s) {
        row0[s] = static_cast<int32_t>(r);
        cnt[s] = counts[s];
        for (int i = 0; i < counts[s]; ++i) row_seq[r++] = s;
    }
    cudaError_t e = cudaMemcpyAsync(b->dyn, b->h_dyn, static_cast<size_t>(2 * b->B + rows) * 4,
                                    cudaMemcpyHostToDevice, b->stream);
    if (e == cudaSuccess && rows > 0)
        e = cudaMemcpyAsync(b->ids, ids_host, static_cast<size_t>(rows) * 4, cudaMemcpyHostToDevice, b->stream);
    if (e != cudaSuccess) return bfail(e, "step upload");
    const tir_status rc = upload_table(b);
    if (rc != TIR_OK) return rc;
    *T = rows;
    *max_cnt = mc;
    return TIR_OK;
}

tir_status check_err(tir_batch* b) {
    cudaError_t e = cudaMemcpyAsync(b->h_err, b->err, 4, cudaMemcpyDeviceToHost, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return bfail(e, "batched forward");
    const uint32_t code = *b->h_err;
    if (code == 0) return TIR_OK;
    // reset: every sequence and the error word
    *b->h_err = 0;
    e = cudaMemsetAsync(b->err, 0, 16, b->stream);
    if (e != cudaSuccess) return bfail(e, "batch reset");
    const tir_status rc = reset_all(b);
    if (rc != TIR_OK) return rc;
    if (code == kBErrBadToken) return fail(TIR_ERR_BAD_TOKEN, "a token id is not in the vocab; the batch was reset");
    return fail(TIR_ERR_TIMEOUT, "device wait timed out; the batch was reset");
}

}  // namespace

extern "C" {

tir_status tir_batch_create_paged(tir_model* m, int32_t n_seqs, int32_t max_ctx, int32_t max_tokens_per_seq,
                                  int32_t n_pages, tir_batch** out) {
    clear_error();
    if (!m || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const tir_transformer& t = m->t;
    if (n_seqs <= 0 || max_ctx <= 0 || max_tokens_per_seq <= 0 || max_tokens_per_seq > max_ctx || n_pages <= 0)
        return fail(TIR_ERR_INVALID_ARG,
                    "need n_seqs, max_ctx, n_pages > 0 and 0 < max_tokens_per_seq <= max_ctx");
    if (t.embed_dim % 64 != 0 || t.ffn_dim % 64 != 0 || t.q_heads / t.k_v_heads > 16)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "batched path needs embedding and FFN sizes that are multiples of 64 "
                                               "and at most 16 query heads per KV head");
    if (cudaSetDevice(m->device) != cudaSuccess) return fail(TIR_ERR_CUDA, "cudaSetDevice");
    tir_batch* b = new tir_batch;
    b->m = m;
    b->B = n_seqs;
    b->max_ctx = max_ctx;
    b->max_tps = max_tokens_per_seq;
    b->max_pages = (max_ctx + kPage - 1) / kPage;
    b->n_pages = n_pages;
    b->h_len.assign(static_cast<size_t>(n_seqs), 0);
    b->seq_pages.assign(static_cast<size_t>(n_seqs), {});
    for (int32_t p = n_pages - 1; p >= 0; --p) b->free_pages.push_back(p);  // page 0 handed out first
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, m->device);
    b->sms = sms > 0 ? sms : 148;
    if (cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess) {
        delete b;
        return fail(TIR_ERR_CUDA, "stream creation failed");
    }
    const int64_t H = t.embed_dim, KVD = t.kv_dim, F = t.ffn_dim, V = t.vocab, L = t.layers;
    const int64_t T = static_cast<int64_t>(n_seqs) * max_tokens_per_seq;
    const int64_t kmax = std::max(H, F);
    const size_t cache = static_cast<size_t>(L) * n_pages * kPage * KVD;
    // Rows of partial tiles a matmul of n x k leaves over every row count a
    // step can have (1 .. n_seqs x tokens_per_seq): split-K count x rows, at most.
    auto part_rows = [&](int64_t n, int64_t k) {
        size_t rows = 0;
        for (int64_t tok = 1; tok <= T; ++tok)
            rows = std::max(rows, static_cast<size_t>(gemm_real_splits(k, gemm_splits(n, k, tok, b->sms)) * tok));
        return rows;
    };
    bool ok = balloc(b, cache * 4, &b->kc) && balloc(b, cache * 4, &b->vc) &&
              balloc(b, static_cast<size_t>(max_ctx) * 32 * 4, &b->rcos) &&
              balloc(b, static_cast<size_t>(max_ctx) * 32 * 4, &b->rsin) && balloc(b, T * H * 4, &b->X) &&
              balloc(b, std::max(part_rows(H, H), part_rows(H, F)) * H * 4, &b->Y) &&
              balloc(b, part_rows(H + 2 * KVD, H) * (H + 2 * KVD) * 4, &b->QKV) && balloc(b, T * H * 4, &b->ATT) &&
              balloc(b, part_rows(2 * F, H) * 2 * F * 4, &b->GU) &&
              balloc(b, static_cast<size_t>(gemm_real_splits(H, gemm_splits(V, H, n_seqs, b->sms))) * n_seqs * V * 4,
                     &b->LG) &&
              balloc(b, static_cast<size_t>(n_seqs) * 4, &b->seq_len) &&
              balloc(b, static_cast<size_t>(n_seqs) * b->max_pages * 4, &b->table) &&
              balloc(b, static_cast<size_t>(2 * n_seqs + T) * 4, &b->dyn) &&
              balloc(b, static_cast<size_t>(3 * n_seqs) * 4, &b->uni) &&
              balloc(b, static_cast<size_t>(gemm_x_plane_bytes(T, kmax)), &b->planes) &&
              balloc(b, static_cast<size_t>(gemm_tokens_padded(T)) * 4, &b->inv) && balloc(b, T * 4, &b->ids) &&
              balloc(b, static_cast<size_t>(n_seqs) * 4, &b->rows) &&
              balloc(b, static_cast<size_t>(n_seqs) * 4, &b->next) && balloc(b, 16, &b->err) &&
              balloc(b, static_cast<size_t>(n_seqs) * 4, &b->head_done);
    if (!ok || host_malloc_pinned(&b->h_next, static_cast<size_t>(n_seqs) * 4) != cudaSuccess ||
        host_malloc_pinned(&b->h_err, 16) != cudaSuccess ||
        host_malloc_pinned(&b->h_table, static_cast<size_t>(n_seqs) * b->max_pages * 4) != cudaSuccess ||
        host_malloc_pinned(&b->h_dyn, static_cast<size_t>(2 * n_seqs + T) * 4) != cudaSuccess) {
        delete b;
        return fail(TIR_ERR_OOM, "batch allocation failed");
    }
    std::memset(b->h_table, 0, static_cast<size_t>(n_seqs) * b->max_pages * 4);
    std::vector<int32_t> uni(static_cast<size_t>(3 * n_seqs));
    for (int s_ = 0; s_ < n_seqs; ++s_) {
        uni[static_cast<size_t>(s_)] = s_;           // row0
        uni[static_cast<size_t>(n_seqs + s_)] = 1;   // cnt
        uni[static_cast<size_t>(2 * n_seqs + s_)] = s_;  // row_seq
    }
    std::vector<float> c, sn;
    rope_table(t.base_freq, kHeadDim, max_ctx, c, sn);
    if (cudaMemcpy(b->rcos, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(b->rsin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(b->uni, uni.data(), uni.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(b->table, 0, static_cast<size_t>(n_seqs) * b->max_pages * 4) != cudaSuccess ||
        cudaMemset(b->err, 0, 16) != cudaSuccess || cudaMemset(b->seq_len, 0, static_cast<size_t>(n_seqs) * 4) != cudaSuccess ||
        cudaMemset(b->head_done, 0, static_cast<size_t>(n_seqs) * 4) != cudaSuccess ||
        gemm_configure() != 0) {
        delete b;
        return fail(TIR_ERR_CUDA, "batch initialisation failed");
    }
    // tensor-core copies of every projection (through one block staging buffer)
    uint8_t* staging = nullptr;
    const size_t sbytes = static_cast<size_t>(std::max(m->lm.n * (m->lm.k / 32), m->gu[0].n * (m->gu[0].k / 32))) * 34;
    if (dev_malloc(&staging, sbytes) != cudaSuccess) {
        delete b;
        return fail(TIR_ERR_OOM, "staging allocation failed");
    }
    tir_status rc = TIR_OK;
    b->qkv.resize(L);
    b->o.resize(L);
    b->gu.resize(L);
    b->down.resize(L);
    for (int64_t l = 0; l < L && rc == TIR_OK; ++l) {
        if ((rc = make_gw(b, m->qkv[l], staging, b->qkv[l])) != TIR_OK) break;
        if ((rc = make_gw(b, m->o[l], staging, b->o[l])) != TIR_OK) break;
        if ((rc = make_gw(b, m->gu[l], staging, b->gu[l])) != TIR_OK) break;
        rc = make_gw(b, m->down[l], staging, b->down[l]);
    }
    if (rc == TIR_OK) rc = make_gw(b, m->lm, staging, b->lm);
    cudaStreamSynchronize(b->stream);
    cudaFree(staging);
    if (rc != TIR_OK) {
        delete b;
        return rc;
    }
    *out = b;
    return TIR_OK;
}

tir_status tir_batch_create(tir_model* m, int32_t n_seqs, int32_t max_ctx, int32_t max_tokens_per_seq,
                            tir_batch** out) {
    if (n_seqs <= 0 || max_ctx <= 0) {
        clear_error();
        return fail(TIR_ERR_INVALID_ARG, "need n_seqs, max_ctx > 0 and 0 < max_tokens_per_seq <= max_ctx");
    }
    return tir_batch_create_paged(m, n_seqs, max_ctx, max_tokens_per_seq, n_seqs * ((max_ctx + kPage - 1) / kPage),
                                  out);
}

void tir_batch_destroy(tir_batch* b) { delete b; }

tir_status tir_batch_reset(tir_batch* b) {
    clear_error();
    if (!b) return fail(TIR_ERR_INVALID_ARG, "null argument");
    cudaSetDevice(b->m->device);
    return reset_all(b);
}

tir_status tir_batch_reset_seq(tir_batch* b, int32_t seq) {
    clear_error();
    if (!b || seq < 0 || seq >= b->B) return fail(TIR_ERR_INVALID_ARG, "null batch or sequence out of range");
    cudaSetDevice(b->m->device);
    const cudaError_t e = cudaStreamSynchronize(b->stream);  // its pages may still be read
    if (e != cudaSuccess) return bfail(e, "sequence reset");
    return release_seq(b, seq);
}

int32_t tir_batch_len(const tir_batch* b) {
    if (!b) return 0;
    int32_t mx = 0;
    for (int32_t l : b->h_len) mx = std::max(mx, l);
    return mx;
}

int32_t tir_batch_seq_len(const tir_batch* b, int32_t seq) {
    return b && seq >= 0 && seq < b->B ? b->h_len[static_cast<size_t>(seq)] : 0;
}

int32_t tir_batch_free_pages(const tir_batch* b) { return b ? static_cast<int32_t>(b->free_pages.size()) : 0; }

void* tir_batch_stream(tir_batch* b) { return b ? static_cast<void*>(b->stream) : nullptr; }

tir_status tir_batch_step_ragged(tir_batch* b, const int32_t* ids_host, const int32_t* counts_host,
                                 int32_t* next_ids_host) {
    clear_error();
    if (!b || !counts_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    int64_t total = 0;
    for (int s_ = 0; s_ < b->B; ++s_) total += counts_host[s_] > 0 ? counts_host[s_] : 0;
    if (total > 0 && !ids_host) return fail(TIR_ERR_INVALID_ARG, "null ids");
    cudaSetDevice(b->m->device);
    int64_t T = 0;
    int max_cnt = 0;
    tir_status rc = stage_step(b, ids_host, counts_host, &T, &max_cnt);
    if (rc != TIR_OK) return rc;
    if (T == 0) return TIR_OK;
    rc = forward(b, b->dyn, T, max_cnt);
    if (rc != TIR_OK) return rc;
    if (next_ids_host) {
        const cudaError_t e =
            cudaMemcpyAsync(b->h_next, b->next, static_cast<size_t>(b->B) * 4, cudaMemcpyDeviceToHost, b->stream);
        if (e != cudaSuccess) return bfail(e, "id readback");
    }
    rc = check_err(b);
    if (rc != TIR_OK) return rc;
    for (int s_ = 0; s_ < b->B; ++s_) b->h_len[static_cast<size_t>(s_)] += counts_host[s_];
    if (next_ids_host) std::copy(b->h_next, b->h_next + b->B, next_ids_host);
    return TIR_OK;
}

tir_status tir_batch_step(tir_batch* b, const int32_t* ids_host, int32_t tokens_per_seq, int32_t* next_ids_host) {
    clear_error();
    if (!b || !ids_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (tokens_per_seq <= 0 || tokens_per_seq > b->max_tps)
        return fail(TIR_ERR_INVALID_ARG, "tokens_per_seq must be in [1, " + std::to_string(b->max_tps) + "]");
    const std::vector<int32_t> counts(static_cast<size_t>(b->B), tokens_per_seq);
    if (tokens_per_seq > 1) return tir_batch_step_ragged(b, ids_host, counts.data(), next_ids_host);
    // one token each: the captured decode forward on the constant layout
    cudaSetDevice(b->m->device);
    for (int s_ = 0; s_ < b->B; ++s_)
        if (b->h_len[static_cast<size_t>(s_)] + 1 > b->max_ctx)
            return fail(TIR_ERR_CTX_OVERFLOW, "sequence " + std::to_string(s_) + " would exceed the batch context");
    size_t need = 0;
    for (int s_ = 0; s_ < b->B; ++s_) {
        const size_t want = static_cast<size_t>((b->h_len[static_cast<size_t>(s_)] + 1 + kPage - 1) / kPage);
        need += want > b->seq_pages[static_cast<size_t>(s_)].size() ? 1 : 0;
    }
    if (need > b->free_pages.size()) return fail(TIR_ERR_OOM, "the batch's KV page pool is exhausted");
    tir_status rc = TIR_OK;
    for (int s_ = 0; s_ < b->B && rc == TIR_OK; ++s_) rc = ensure_pages(b, s_, b->h_len[static_cast<size_t>(s_)] + 1);
    if (rc == TIR_OK) rc = upload_table(b);
    if (rc != TIR_OK) return rc;
    cudaError_t e = cudaMemcpyAsync(b->ids, ids_host, static_cast<size_t>(b->B) * 4, cudaMemcpyHostToDevice, b->stream);
    if (e != cudaSuccess) return bfail(e, "id upload");
    rc = decode_forward(b);
    if (rc != TIR_OK) return rc;
    if (next_ids_host) {
        e = cudaMemcpyAsync(b->h_next, b->next, static_cast<size_t>(b->B) * 4, cudaMemcpyDeviceToHost, b->stream);
        if (e != cudaSuccess) return bfail(e, "id readback");
    }
    rc = check_err(b);
    if (rc == TIR_OK && next_ids_host) std::copy(b->h_next, b->h_next + b->B, next_ids_host);
    return rc;
}

#define CUDA_BTRY(expr, what)                         \
    do {                                              \
        cudaError_t e_ = (expr);                      \
        if (e_ != cudaSuccess) return bfail(e_, what); \
    } while (0)

tir_status tir_batch_dump_rows(tir_batch* b, const int32_t* rows_host, int32_t n_rows) {
    clear_error();
    if (!b || n_rows < 0 || (n_rows > 0 && !rows_host)) return fail(TIR_ERR_INVALID_ARG, "bad dump request");
    cudaSetDevice(b->m->device);
    cudaStreamSynchronize(b->stream);
    if (b->dump) cudaFree(b->dump);
    if (b->dump_idx) cudaFree(b->dump_idx);
    b->dump = nullptr;
    b->dump_idx = nullptr;
    b->dump_rows.assign(rows_host, rows_host + n_rows);
    if (n_rows == 0) return TIR_OK;
    const int64_t T = static_cast<int64_t>(b->B) * b->max_tps;
    for (int32_t r : b->dump_rows)
        if (r < 0 || r >= T) {
            b->dump_rows.clear();
            return fail(TIR_ERR_INVALID_ARG, "dump row out of range");
        }
    const size_t bytes = static_cast<size_t>(n_rows) * b->m->t.layers * b->m->t.embed_dim * 4;
    if (dev_malloc(&b->dump, bytes) != cudaSuccess || dev_malloc(&b->dump_idx, static_cast<size_t>(n_rows) * 4) != cudaSuccess) {
        b->dump_rows.clear();
        return fail(TIR_ERR_OOM, "dump allocation failed");
    }
    CUDA_BTRY(cudaMemset(b->dump, 0, bytes), "dump reset");
    CUDA_BTRY(cudaMemcpy(b->dump_idx, rows_host, static_cast<size_t>(n_rows) * 4, cudaMemcpyHostToDevice), "dump rows");
    return TIR_OK;
}

tir_status tir_batch_dump(tir_batch* b, float* out_host) {
    clear_error();
    if (!b || !out_host || b->dump_rows.empty()) return fail(TIR_ERR_INVALID_ARG, "no dump armed (tir_batch_dump_rows)");
    cudaSetDevice(b->m->device);
    const size_t bytes = b->dump_rows.size() * b->m->t.layers * b->m->t.embed_dim * 4;
    CUDA_BTRY(cudaMemcpyAsync(out_host, b->dump, bytes, cudaMemcpyDeviceToHost, b->stream), "dump readback");
    return check_err(b);
}

// Logits [n_seqs][vocab] of every sequence's last row in the last forward
// (what src/forward.rs:242-252 returns per sequence; a sequence that took no
// token in that step gets zeros): the lm_head partial tiles summed in order.
tir_status tir_batch_logits(tir_batch* b, float* logits_host) {
    clear_error();
    if (!b || !logits_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (b->lm_parts == 0) return fail(TIR_ERR_INVALID_ARG, "no forward has run on this batch");
    cudaSetDevice(b->m->device);
    const int64_t n = static_cast<int64_t>(b->B) * static_cast<int64_t>(b->m->t.vocab);
    if (!b->logits && dev_malloc(reinterpret_cast<void**>(&b->logits), static_cast<size_t>(n) * 4) != cudaSuccess)
        return fail(TIR_ERR_OOM, "logits allocation failed");
    int e = launch_gemm_sum_parts(b->LG, b->lm_parts, n, n, b->logits, b->stream, false);
    if (e != 0) return bfail(static_cast<cudaError_t>(e), "logits sum");
    cudaError_t ce = cudaMemcpyAsync(logits_host, b->logits, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost, b->stream);
    if (ce != cudaSuccess) return bfail(ce, "logits readback");
    return check_err(b);
}

// Per sequence: prefill n_prompt ids, then cap greedy steps (n_prompt + cap
// forwards, as generate_capped, src/lib.rs:239-314); out_ids [B][cap].  Every
// sequence starts empty; the pages for the whole generation are taken first.
tir_status tir_batch_generate(tir_batch* b, const int32_t* prompts_host, int32_t n_prompt, int32_t cap,
                              int32_t* out_ids_host) {
    clear_error();
    if (!b || !prompts_host || (cap > 0 && !out_ids_host)) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (n_prompt <= 0 || n_prompt > b->max_tps || cap < 0)
        return fail(TIR_ERR_INVALID_ARG, "n_prompt must be in [1, " + std::to_string(b->max_tps) + "], cap >= 0");
    if (n_prompt + cap > b->max_ctx) return fail(TIR_ERR_CTX_OVERFLOW, "prompt + cap exceeds the batch context");
    cudaSetDevice(b->m->device);
    tir_status rc = reset_all(b);
    if (rc != TIR_OK) return rc;
    const size_t per = static_cast<size_t>((n_prompt + cap + kPage - 1) / kPage);
    if (per * static_cast<size_t>(b->B) > b->free_pages.size())
        return fail(TIR_ERR_OOM, "the batch's KV page pool is too small for prompt + cap on every sequence");
    for (int s_ = 0; s_ < b->B && rc == TIR_OK; ++s_) rc = ensure_pages(b, s_, n_prompt + cap);
    if (rc != TIR_OK) return rc;
    if (cap > b->gen_cap) {  // generated ids [cap][B] on the device
        cudaStreamSynchronize(b->stream);
        if (b->gen) cudaFree(b->gen);
        b->gen = nullptr;
        b->gen_cap = 0;
        if (dev_malloc(reinterpret_cast<void**>(&b->gen), static_cast<size_t>(cap) * b->B * 4) != cudaSuccess)
            return fail(TIR_ERR_OOM, "output allocation failed");
        b->gen_cap = cap;
    }
    const std::vector<int32_t> counts(static_cast<size_t>(b->B), n_prompt);
    int64_t T = 0;
    int max_cnt = 0;
    rc = stage_step(b, prompts_host, counts.data(), &T, &max_cnt);  // uploads the page table too
    if (rc == TIR_OK) rc = forward(b, b->dyn, T, max_cnt);
    if (rc == TIR_OK)
        for (int32_t& l : b->h_len) l += n_prompt;
    const unsigned fb = static_cast<unsigned>((b->B + 255) / 256);
    for (int i = 0; rc == TIR_OK && i < cap; ++i) {
        feed_kernel<<<fb, 256, 0, b->stream>>>(b->next, b->ids, b->gen + static_cast<size_t>(i) * b->B, b->B);
        rc = decode_forward(b);
    }
    std::vector<int32_t> host(static_cast<size_t>(cap) * b->B);
    if (rc == TIR_OK && cap > 0) {
        const cudaError_t e = cudaMemcpyAsync(host.data(), b->gen, host.size() * 4, cudaMemcpyDeviceToHost, b->stream);
        if (e != cudaSuccess) rc = bfail(e, "id readback");
    }
    const tir_status rc2 = check_err(b);
    if (rc == TIR_OK) rc = rc2;
    if (rc == TIR_OK)
        for (int s_ = 0; s_ < b->B; ++s_)
            for (int i = 0; i < cap; ++i)
                out_ids_host[static_cast<size_t>(s_) * cap + i] = host[static_cast<size_t>(i) * b->B + s_];
    return rc;
}

}  // extern "C"
