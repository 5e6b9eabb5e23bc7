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
#include <string>
#include <vector>

#include "host.h"
#include "runtime.h"

namespace tir {
namespace {

constexpr uint32_t kBErrBadToken = 12;
constexpr int kQBlock = 32;   // query tokens per prefill attention CTA (one per lane)
constexpr int kKChunk = 32;   // key positions staged per step

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

// out[i] = rmsnorm(X[rows ? rows[i] : i]) * w  (src/math.rs:141-150; the
// division as a multiplication by the correctly rounded reciprocal).
__global__ void rmsnorm_rows_kernel(const float* __restrict__ X, const int32_t* __restrict__ rows, int H,
                                    const float* __restrict__ w, float eps, float* __restrict__ out) {
    __shared__ float red[32];
    const int64_t r = rows ? rows[blockIdx.x] : blockIdx.x;
    const float* x = X + r * H;
    float ss = 0.f;
    for (int c = threadIdx.x; c < H; c += blockDim.x) ss = fmaf(x[c], x[c], ss);
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
    for (int i = 0; i < static_cast<int>(blockDim.x >> 5); ++i) total += red[i];
    const float inv = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(H)), eps)));
    float* o = out + static_cast<int64_t>(blockIdx.x) * H;
    for (int c = threadIdx.x; c < H; c += blockDim.x) o[c] = __fmul_rn(__fmul_rn(x[c], w[c]), inv);
}

// RoPE on the q and k parts of each token's fused q|k|v row (src/math.rs:196-228),
// then the KV-cache append (src/forward.rs:83-84).  Token t belongs to
// sequence t / tps at position pos0 + t % tps; cache [seq][max_ctx][kvd].
__global__ void rope_append_kernel(float* __restrict__ qkv, int64_t ld, int tps, int pos0, int H, int kvd,
                                   int max_ctx, const float* __restrict__ rc, const float* __restrict__ rs,
                                   float* __restrict__ kc, float* __restrict__ vc) {
    const int64_t t = blockIdx.x;
    const int64_t s = t / tps;
    const int pos = pos0 + static_cast<int>(t % tps);
    float* row = qkv + t * ld;
    const size_t cache_row = (static_cast<size_t>(s) * max_ctx + pos) * kvd;
    for (int pr = threadIdx.x; pr < (H + kvd) / 2; pr += blockDim.x) {
        const int c = 2 * pr;
        const int i = (c % kHeadDim) >> 1;
        const float cs = rc[static_cast<size_t>(pos) * (kHeadDim / 2) + i];
        const float sn = rs[static_cast<size_t>(pos) * (kHeadDim / 2) + i];
        const float y0 = row[c], y1 = row[c + 1];
        const float e0 = __fadd_rn(__fmul_rn(cs, y0), __fmul_rn(-sn, y1));
        const float e1 = __fadd_rn(__fmul_rn(sn, y0), __fmul_rn(cs, y1));
        if (c < H) {
            row[c] = e0;
            row[c + 1] = e1;
        } else {
            kc[cache_row + (c - H)] = e0;
            kc[cache_row + (c - H) + 1] = e1;
        }
    }
    for (int c = threadIdx.x; c < kvd; c += blockDim.x) vc[cache_row + c] = row[H + kvd + c];
}

// Causal grouped-query attention for tps >= 2 new tokens per sequence
// (src/forward.rs:79-174 for every query position): CTA per (sequence, kv
// head, block of 32 query tokens); warp h handles query head g * group + h,
// lane i query token i of the block, with its q and running output in
// registers; keys are staged 32 positions at a time in shared memory.  Online
// softmax (running max and sum), scale 1/sqrt(64).
__global__ void attn_prefill_kernel(const float* __restrict__ qkv, int64_t ld, int tps, int pos0, int H, int kvd,
                                    int group, int max_ctx, const float* __restrict__ kc,
                                    const float* __restrict__ vc, float* __restrict__ out) {
    __shared__ float ks[kKChunk][kHeadDim];
    __shared__ float vs[kKChunk][kHeadDim];
    const int s = blockIdx.x, g = blockIdx.y, qb = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = g * group + warp;
    const int qi = qb * kQBlock + lane;  // query token within the sequence's new tokens
    const bool active = qi < tps && warp < group;
    const int qpos = pos0 + qi;
    const int64_t t = static_cast<int64_t>(s) * tps + qi;
    float q[kHeadDim], o[kHeadDim];
#pragma unroll
    for (int d = 0; d < kHeadDim; ++d) {
        q[d] = active ? qkv[t * ld + h * kHeadDim + d] : 0.f;
        o[d] = 0.f;
    }
    float m = -INFINITY, l = 0.f;
    const int last = pos0 + min(tps, (qb + 1) * kQBlock) - 1;  // the block's last query position
    const size_t head_base = static_cast<size_t>(s) * max_ctx * kvd + static_cast<size_t>(g) * kHeadDim;
    for (int c0 = 0; c0 <= last; c0 += kKChunk) {
        __syncthreads();
        for (int e = threadIdx.x; e < kKChunk * kHeadDim; e += blockDim.x) {
            const int j = e / kHeadDim, d = e % kHeadDim;
            const bool in = c0 + j <= last;
            ks[j][d] = in ? kc[head_base + static_cast<size_t>(c0 + j) * kvd + d] : 0.f;
            vs[j][d] = in ? vc[head_base + static_cast<size_t>(c0 + j) * kvd + d] : 0.f;
        }
        __syncthreads();
        if (active) {
            const int jmax = min(kKChunk, qpos - c0 + 1);
            for (int j = 0; j < jmax; ++j) {
                float acc = 0.f;
#pragma unroll
                for (int d = 0; d < kHeadDim; ++d) acc = fmaf(q[d], ks[j][d], acc);
                const float sc = acc / 8.0f;  // sqrt(64)
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
                for (int d = 0; d < kHeadDim; ++d) o[d] = fmaf(pj, vs[j][d], o[d]);
            }
        }
    }
    if (active) {
        const float inv = 1.0f / l;
#pragma unroll
        for (int d = 0; d < kHeadDim; ++d) out[t * H + h * kHeadDim + d] = o[d] * inv;
    }
}

// One new token per sequence (decode): CTA per (sequence, kv head), warp h
// for query head g * group + h, lanes over key positions for the scores and
// over dimensions (two each) for the output; keys staged 32 at a time.
__global__ void attn_decode_kernel(const float* __restrict__ qkv, int64_t ld, int pos, int H, int kvd, int group,
                                   int max_ctx, const float* __restrict__ kc, const float* __restrict__ vc,
                                   float* __restrict__ out) {
    __shared__ float ks[kKChunk][kHeadDim + 1];
    __shared__ float vs[kKChunk][kHeadDim];
    __shared__ float qs[16][kHeadDim];
    const int s = blockIdx.x, g = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int h = g * group + warp;
    const bool active = warp < group;
    for (int e = threadIdx.x; e < group * kHeadDim; e += blockDim.x)
        qs[e / kHeadDim][e % kHeadDim] = qkv[static_cast<int64_t>(s) * ld + (g * group) * kHeadDim + e];
    float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
    const size_t head_base = static_cast<size_t>(s) * max_ctx * kvd + static_cast<size_t>(g) * kHeadDim;
    for (int c0 = 0; c0 <= pos; c0 += kKChunk) {
        __syncthreads();
        const int nc = min(kKChunk, pos - c0 + 1);
        for (int e = threadIdx.x; e < kKChunk * kHeadDim; e += blockDim.x) {
            const int j = e / kHeadDim, d = e % kHeadDim;
            const bool in = j < nc;
            ks[j][d] = in ? kc[head_base + static_cast<size_t>(c0 + j) * kvd + d] : 0.f;
            vs[j][d] = in ? vc[head_base + static_cast<size_t>(c0 + j) * kvd + d] : 0.f;
        }
        __syncthreads();
        if (active) {
            float sc = -INFINITY;
            if (lane < nc) {
                float acc = 0.f;
#pragma unroll 16
                for (int d = 0; d < kHeadDim; ++d) acc = fmaf(qs[warp][d], ks[lane][d], acc);
                sc = acc / 8.0f;
            }
            float mx = sc;
            for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            const float m_new = fmaxf(m, mx);
            const float pj = lane < nc ? expf(sc - m_new) : 0.f;
            float ps = pj;
            for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
            const float corr = expf(m - m_new);
            l = l * corr + ps;
            o0 *= corr;
            o1 *= corr;
            for (int j = 0; j < nc; ++j) {
                const float pt = __shfl_sync(0xffffffffu, pj, j);
                o0 = fmaf(pt, vs[j][lane], o0);
                o1 = fmaf(pt, vs[j][lane + 32], o1);
            }
            m = m_new;
        }
    }
    if (active) {
        out[static_cast<int64_t>(s) * H + h * kHeadDim + lane] = o0 / l;
        out[static_cast<int64_t>(s) * H + h * kHeadDim + lane + 32] = o1 / l;
    }
}

__global__ void residual_add_kernel(float* __restrict__ x, const float* __restrict__ y, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        x[i] = __fadd_rn(x[i], y[i]);
}

// h[t][j] = silu(gate) * up from interleaved (gate_j, up_j) columns
// (src/math.rs:171-175).
__global__ void silu_pairs_kernel(const float* __restrict__ gu, int64_t tokens, int F, float* __restrict__ h) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < tokens * F;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t t = i / F, j = i % F;
        const float g = gu[t * 2 * F + 2 * j], u = gu[t * 2 * F + 2 * j + 1];
        h[i] = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
    }
}

// Greedy sample per row (src/tokenizer.rs:152-167: total order, ties -> last).
__global__ void argmax_rows_kernel(const float* __restrict__ x, int64_t n, int32_t* __restrict__ out) {
    __shared__ unsigned long long red[32];
    const float* r = x + static_cast<int64_t>(blockIdx.x) * n;
    unsigned long long best = 0ull;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const uint32_t b = __float_as_uint(r[i]);
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

__global__ void last_rows_kernel(int32_t* rows, int n_seqs, int tps) {
    const int s = blockIdx.x * blockDim.x + threadIdx.x;
    if (s < n_seqs) rows[s] = s * tps + tps - 1;
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
    int B = 0, max_ctx = 0, max_tps = 0, len = 0, sms = 148;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    std::vector<GW> qkv, o, gu, down;
    GW lm;
    float *kc = nullptr, *vc = nullptr, *rcos = nullptr, *rsin = nullptr;
    float *X = nullptr, *XN = nullptr, *QKV = nullptr, *ATT = nullptr, *GU = nullptr, *HH = nullptr, *Y = nullptr,
          *LG = nullptr, *inv = nullptr, *part = nullptr;
    uint8_t* planes = nullptr;
    int32_t *ids = nullptr, *rows = nullptr, *next = nullptr, *h_next = nullptr;
    uint32_t *err = nullptr, *h_err = nullptr;
    size_t part_floats = 0;
    ~tir_batch() {
        cudaSetDevice(m ? m->device : 0);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : allocs) cudaFree(p);
        if (h_next) cudaFreeHost(h_next);
        if (h_err) cudaFreeHost(h_err);
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
    if (cudaMalloc(&q, bytes ? bytes : 16) != cudaSuccess) return false;
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

tir_status gemm(tir_batch* b, const float* x, int64_t tokens, const tir_batch::GW& g, float* y) {
    int rc = launch_gemm_x_planes(x, tokens, g.k, b->planes, b->inv, b->stream);
    if (rc != 0) return bfail(static_cast<cudaError_t>(rc), "activation planes");
    const int64_t tiles = ((g.n + 127) / 128) * ((tokens + 127) / 128);
    int splits = 1;
    if (tiles < b->sms && tokens <= 256) {
        splits = static_cast<int>(std::min<int64_t>(g.k / 64, std::max<int64_t>(1, b->sms / tiles)));
        while (splits > 1 && static_cast<size_t>(splits) * tokens * g.n > b->part_floats) --splits;
    }
    rc = launch_gemm_q8(g.w, g.p2, b->planes, b->inv, g.n, g.k, tokens, y, g.n, splits, b->part, b->err,
                        2000ull * 1000000ull, b->stream);
    if (rc != 0) return bfail(static_cast<cudaError_t>(rc), "tensor-core matmul");
    return TIR_OK;
}

// One forward over tps new tokens of every sequence (ids already in b->ids,
// sequence-major); greedy next id of every sequence into b->next.
tir_status forward(tir_batch* b, int tps) {
    tir_model* m = b->m;
    const tir_transformer& t = m->t;
    const int H = static_cast<int>(t.embed_dim), KVD = static_cast<int>(t.kv_dim), F = static_cast<int>(t.ffn_dim);
    const int V = static_cast<int>(t.vocab), L = static_cast<int>(t.layers);
    const int group = static_cast<int>(t.q_heads / t.k_v_heads);
    const int64_t T = static_cast<int64_t>(b->B) * tps;
    const int64_t ldq = H + 2 * KVD;
    const size_t layer_cache = static_cast<size_t>(b->B) * b->max_ctx * KVD;
    cudaStream_t st = b->stream;
    tir_status rc;
    embed_rows_kernel<<<static_cast<unsigned>(T), 256, 0, st>>>(b->ids, m->embd.q, m->embd.s, m->embd.sk, H, V, b->X,
                                                                 b->err);
    for (int l = 0; l < L; ++l) {
        rmsnorm_rows_kernel<<<static_cast<unsigned>(T), 256, 0, st>>>(b->X, nullptr, H, m->attn_norm[l], 1e-5f, b->XN);
        if ((rc = gemm(b, b->XN, T, b->qkv[l], b->QKV)) != TIR_OK) return rc;
        float* kc = b->kc + l * layer_cache;
        float* vc = b->vc + l * layer_cache;
        rope_append_kernel<<<static_cast<unsigned>(T), 256, 0, st>>>(b->QKV, ldq, tps, b->len, H, KVD, b->max_ctx,
                                                                      b->rcos, b->rsin, kc, vc);
        if (tps == 1) {
            attn_decode_kernel<<<dim3(b->B, static_cast<unsigned>(t.k_v_heads)), group * 32, 0, st>>>(
                b->QKV, ldq, b->len, H, KVD, group, b->max_ctx, kc, vc, b->ATT);
        } else {
            attn_prefill_kernel<<<dim3(b->B, static_cast<unsigned>(t.k_v_heads), (tps + kQBlock - 1) / kQBlock),
                                  group * 32, 0, st>>>(b->QKV, ldq, tps, b->len, H, KVD, group, b->max_ctx, kc, vc,
                                                       b->ATT);
        }
        if ((rc = gemm(b, b->ATT, T, b->o[l], b->Y)) != TIR_OK) return rc;
        residual_add_kernel<<<g1(T * H, 256), 256, 0, st>>>(b->X, b->Y, T * H);
        rmsnorm_rows_kernel<<<static_cast<unsigned>(T), 256, 0, st>>>(b->X, nullptr, H, m->ffn_norm[l], 1e-5f, b->XN);
        if ((rc = gemm(b, b->XN, T, b->gu[l], b->GU)) != TIR_OK) return rc;
        silu_pairs_kernel<<<g1(T * F, 256), 256, 0, st>>>(b->GU, T, F, b->HH);
        if ((rc = gemm(b, b->HH, T, b->down[l], b->Y)) != TIR_OK) return rc;
        residual_add_kernel<<<g1(T * H, 256), 256, 0, st>>>(b->X, b->Y, T * H);
    }
    last_rows_kernel<<<(b->B + 127) / 128, 128, 0, st>>>(b->rows, b->B, tps);
    rmsnorm_rows_kernel<<<static_cast<unsigned>(b->B), 256, 0, st>>>(b->X, b->rows, H, m->out_norm, 1e-5f, b->XN);
    if ((rc = gemm(b, b->XN, b->B, b->lm, b->LG)) != TIR_OK) return rc;
    argmax_rows_kernel<<<static_cast<unsigned>(b->B), 256, 0, st>>>(b->LG, V, b->next);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return bfail(e, "batched forward");
    b->len += tps;
    return TIR_OK;
}

tir_status check_err(tir_batch* b) {
    cudaError_t e = cudaMemcpyAsync(b->h_err, b->err, 4, cudaMemcpyDeviceToHost, b->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(b->stream);
    if (e != cudaSuccess) return bfail(e, "batched forward");
    if (*b->h_err == kBErrBadToken) {
        b->len = 0;
        return fail(TIR_ERR_BAD_TOKEN, "a token id is not in the vocab; the batch was reset");
    }
    if (*b->h_err != 0) {
        b->len = 0;
        return fail(TIR_ERR_TIMEOUT, "device wait timed out; the batch was reset");
    }
    return TIR_OK;
}

}  // namespace

extern "C" {

tir_status tir_batch_create(tir_model* m, int32_t n_seqs, int32_t max_ctx, int32_t max_tokens_per_seq,
                            tir_batch** out) {
    clear_error();
    if (!m || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const tir_transformer& t = m->t;
    if (n_seqs <= 0 || max_ctx <= 0 || max_tokens_per_seq <= 0 || max_tokens_per_seq > max_ctx)
        return fail(TIR_ERR_INVALID_ARG, "need n_seqs, max_ctx > 0 and 0 < max_tokens_per_seq <= max_ctx");
    if (t.embed_dim % 64 != 0 || t.ffn_dim % 64 != 0 || t.q_heads / t.k_v_heads > 16)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "batched path needs embedding and FFN sizes that are multiples of 64 "
                                               "and at most 16 query heads per KV head");
    if (cudaSetDevice(m->device) != cudaSuccess) return fail(TIR_ERR_CUDA, "cudaSetDevice");
    tir_batch* b = new tir_batch;
    b->m = m;
    b->B = n_seqs;
    b->max_ctx = max_ctx;
    b->max_tps = max_tokens_per_seq;
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
    b->part_floats = static_cast<size_t>(b->sms) * 128 * 256;
    const size_t cache = static_cast<size_t>(L) * n_seqs * max_ctx * KVD;
    bool ok = balloc(b, cache * 4, &b->kc) && balloc(b, cache * 4, &b->vc) &&
              balloc(b, static_cast<size_t>(max_ctx) * 32 * 4, &b->rcos) &&
              balloc(b, static_cast<size_t>(max_ctx) * 32 * 4, &b->rsin) && balloc(b, T * H * 4, &b->X) &&
              balloc(b, T * H * 4, &b->XN) && balloc(b, T * (H + 2 * KVD) * 4, &b->QKV) &&
              balloc(b, T * H * 4, &b->ATT) && balloc(b, T * 2 * F * 4, &b->GU) && balloc(b, T * F * 4, &b->HH) &&
              balloc(b, T * H * 4, &b->Y) && balloc(b, static_cast<size_t>(n_seqs) * V * 4, &b->LG) &&
              balloc(b, static_cast<size_t>(gemm_x_plane_bytes(T, kmax)), &b->planes) &&
              balloc(b, static_cast<size_t>(gemm_tokens_padded(T)) * 4, &b->inv) &&
              balloc(b, b->part_floats * 4, &b->part) && balloc(b, T * 4, &b->ids) &&
              balloc(b, static_cast<size_t>(n_seqs) * 4, &b->rows) &&
              balloc(b, static_cast<size_t>(n_seqs) * 4, &b->next) && balloc(b, 16, &b->err);
    if (!ok || cudaMallocHost(&b->h_next, static_cast<size_t>(n_seqs) * 4) != cudaSuccess ||
        cudaMallocHost(&b->h_err, 16) != cudaSuccess) {
        delete b;
        return fail(TIR_ERR_OOM, "batch allocation failed");
    }
    std::vector<float> c, s;
    rope_table(t.base_freq, kHeadDim, max_ctx, c, s);
    if (cudaMemcpy(b->rcos, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(b->rsin, s.data(), s.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(b->err, 0, 16) != cudaSuccess) {
        delete b;
        return fail(TIR_ERR_CUDA, "batch initialisation failed");
    }
    // tensor-core copies of every projection (through one block staging buffer)
    uint8_t* staging = nullptr;
    const size_t sbytes = static_cast<size_t>(std::max(m->lm.n * (m->lm.k / 32), m->gu[0].n * (m->gu[0].k / 32))) * 34;
    if (cudaMalloc(&staging, sbytes) != cudaSuccess) {
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

void tir_batch_destroy(tir_batch* b) { delete b; }

tir_status tir_batch_reset(tir_batch* b) {
    if (!b) return fail(TIR_ERR_INVALID_ARG, "null argument");
    b->len = 0;
    return TIR_OK;
}

int32_t tir_batch_len(const tir_batch* b) { return b ? b->len : 0; }

void* tir_batch_stream(tir_batch* b) { return b ? static_cast<void*>(b->stream) : nullptr; }

tir_status tir_batch_step(tir_batch* b, const int32_t* ids_host, int32_t tokens_per_seq, int32_t* next_ids_host) {
    clear_error();
    if (!b || !ids_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (tokens_per_seq <= 0 || tokens_per_seq > b->max_tps)
        return fail(TIR_ERR_INVALID_ARG, "tokens_per_seq must be in [1, " + std::to_string(b->max_tps) + "]");
    if (b->len + tokens_per_seq > b->max_ctx) return fail(TIR_ERR_CTX_OVERFLOW, "batch context is full");
    cudaSetDevice(b->m->device);
    const size_t n = static_cast<size_t>(b->B) * tokens_per_seq;
    cudaError_t e = cudaMemcpyAsync(b->ids, ids_host, n * 4, cudaMemcpyHostToDevice, b->stream);
    if (e != cudaSuccess) return bfail(e, "id upload");
    tir_status rc = forward(b, tokens_per_seq);
    if (rc != TIR_OK) return rc;
    if (next_ids_host) {
        e = cudaMemcpyAsync(b->h_next, b->next, static_cast<size_t>(b->B) * 4, cudaMemcpyDeviceToHost, b->stream);
        if (e != cudaSuccess) return bfail(e, "id readback");
    }
    rc = check_err(b);
    if (rc == TIR_OK && next_ids_host) std::copy(b->h_next, b->h_next + b->B, next_ids_host);
    return rc;
}

// Per sequence: prefill n_prompt ids, then cap greedy steps (n_prompt + cap
// forwards, as generate_capped, src/lib.rs:239-314); out_ids [B][cap].
tir_status tir_batch_generate(tir_batch* b, const int32_t* prompts_host, int32_t n_prompt, int32_t cap,
                              int32_t* out_ids_host) {
    clear_error();
    if (!b || !prompts_host || (cap > 0 && !out_ids_host)) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (n_prompt <= 0 || n_prompt > b->max_tps || cap < 0)
        return fail(TIR_ERR_INVALID_ARG, "n_prompt must be in [1, " + std::to_string(b->max_tps) + "], cap >= 0");
    if (n_prompt + cap > b->max_ctx) return fail(TIR_ERR_CTX_OVERFLOW, "prompt + cap exceeds the batch context");
    cudaSetDevice(b->m->device);
    b->len = 0;
    const size_t n = static_cast<size_t>(b->B) * n_prompt;
    cudaError_t e = cudaMemcpyAsync(b->ids, prompts_host, n * 4, cudaMemcpyHostToDevice, b->stream);
    if (e != cudaSuccess) return bfail(e, "prompt upload");
    int32_t* gen = nullptr;  // [cap][B] on the device
    if (cap > 0 && cudaMallocAsync(reinterpret_cast<void**>(&gen), static_cast<size_t>(cap) * b->B * 4, b->stream) !=
                       cudaSuccess)
        return fail(TIR_ERR_OOM, "output allocation failed");
    tir_status rc = forward(b, n_prompt);
    for (int i = 0; rc == TIR_OK && i < cap; ++i) {
        // the sampled ids are both this step's output and its input
        cudaMemcpyAsync(gen + static_cast<size_t>(i) * b->B, b->next, static_cast<size_t>(b->B) * 4,
                        cudaMemcpyDeviceToDevice, b->stream);
        cudaMemcpyAsync(b->ids, b->next, static_cast<size_t>(b->B) * 4, cudaMemcpyDeviceToDevice, b->stream);
        rc = forward(b, 1);
    }
    std::vector<int32_t> host(static_cast<size_t>(cap) * b->B);
    if (rc == TIR_OK && cap > 0) {
        e = cudaMemcpyAsync(host.data(), gen, host.size() * 4, cudaMemcpyDeviceToHost, b->stream);
        if (e != cudaSuccess) rc = bfail(e, "id readback");
    }
    if (gen) cudaFreeAsync(gen, b->stream);
    const tir_status rc2 = check_err(b);
    if (rc == TIR_OK) rc = rc2;
    if (rc == TIR_OK)
        for (int s = 0; s < b->B; ++s)
            for (int i = 0; i < cap; ++i) out_ids_host[static_cast<size_t>(s) * cap + i] = host[static_cast<size_t>(i) * b->B + s];
    return rc;
}

}  // extern "C"
