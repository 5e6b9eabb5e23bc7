// ops.cu -- op-level sm_100a kernels behind the tir_* op entry points: one
// kernel per reference op (src/math.rs, src/kernels.rs, src/tokenizer.rs), plus
// the Q8_0 repack used at model upload.  The decode path itself runs in the
// persistent kernel of decode.cu; these serve the op-level ABI and tests.
//
// Exactness: dequantisation, embedding, activation quantisation and the
// integer block dots of q8_act_matmul (with the reference's block-order f32
// sum) are bit-exact.  rmsnorm/softmax reduce in parallel (fp32 within a few
// ulp of the sequential folds).  rope is bit-exact given the cos/sin the host
// evaluates with glibc, as the reference does.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "host.h"
#include "runtime.h"

namespace tir {

namespace {

constexpr uint32_t FULL = 0xffffffffu;

__device__ __forceinline__ float f16_at(const uint8_t* p) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

__device__ __forceinline__ uint32_t total_key(float v) {
    uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

// Rust `f32 as i8`: saturating, NaN -> 0.
__device__ __forceinline__ int8_t f32_as_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return static_cast<int8_t>(v);
}

// Q8_0 blocks -> split layout (signed int8 quants, f16 scales), optionally
// interleaving rows into the destination (dst row = r * step + off).
__global__ void repack_kernel(const uint8_t* __restrict__ blocks, int64_t rows, int64_t k,
                              uint8_t* __restrict__ quants, uint16_t* __restrict__ scales, int64_t sk,
                              int64_t step, int64_t off) {
    const int64_t nb = k / 32;
    const int64_t total = rows * nb;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / nb, b = i % nb;
        const uint8_t* src = blocks + i * 34;
        const int64_t dr = r * step + off;
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = static_cast<uint32_t>(src[2 + 4 * j]) | (static_cast<uint32_t>(src[3 + 4 * j]) << 8) |
                   (static_cast<uint32_t>(src[4 + 4 * j]) << 16) | (static_cast<uint32_t>(src[5 + 4 * j]) << 24);
        uint4* dst = reinterpret_cast<uint4*>(quants + dr * k + b * 32);
        dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
        dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
        scales[dr * sk + b] = static_cast<uint16_t>(src[0] | (src[1] << 8));
    }
}

// Q8_0 blocks -> warp-sliced tile-major layout (runtime.h q8_slice_offset):
// row r of the source lands in row dr = r * step + off of the matrix.
__global__ void repack_tiled_kernel(const uint8_t* __restrict__ blocks, int64_t rows, int64_t k,
                                    uint8_t* __restrict__ dst, int64_t tile_rows, int64_t step, int64_t off) {
    const int64_t nb = k / 32;
    const int rl_n = gemv_row_lanes(k);
    const int64_t total = rows * nb;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t r = i / nb, b = i % nb;
        const uint8_t* src = blocks + i * 34;
        const int64_t dr = r * step + off;
        const int64_t t = dr / tile_rows, rr = dr % tile_rows;
        const int rl = static_cast<int>(rr % rl_n), j = static_cast<int>(rr / rl_n);
        const int wi = static_cast<int>(b / 32), bl = static_cast<int>(b % 32);
        const int nbw = q8_slice_blocks(k, wi), nbwp = (nbw + 7) / 8 * 8;
        uint8_t* base = dst + q8_slice_offset(k, t, rl, wi);
        uint32_t w[8];
#pragma unroll
        for (int jj = 0; jj < 8; ++jj)
            w[jj] = static_cast<uint32_t>(src[2 + 4 * jj]) | (static_cast<uint32_t>(src[3 + 4 * jj]) << 8) |
                    (static_cast<uint32_t>(src[4 + 4 * jj]) << 16) | (static_cast<uint32_t>(src[5 + 4 * jj]) << 24);
        uint4* q = reinterpret_cast<uint4*>(base + (static_cast<int64_t>(j) * nbw + bl) * 32);
        q[0] = make_uint4(w[0], w[1], w[2], w[3]);
        q[1] = make_uint4(w[4], w[5], w[6], w[7]);
        reinterpret_cast<uint16_t*>(base + kTileMult * nbw * 32)[j * nbwp + bl] =
            static_cast<uint16_t>(src[0] | (src[1] << 8));
    }
}

// src/math.rs:117-137: f32(q) * f32(scale), exact.
__global__ void dequant_kernel(const uint8_t* __restrict__ blocks, int64_t n_blocks, float* __restrict__ out) {
    const int64_t total = n_blocks * 32;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const uint8_t* blk = blocks + (i / 32) * 34;
        out[i] = __fmul_rn(static_cast<float>(static_cast<int8_t>(blk[2 + i % 32])), f16_at(blk));
    }
}

__device__ float block_sum(float v, float* red) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(FULL, v, o);
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) t += red[w];
    __syncthreads();
    return t;
}

// src/math.rs:141-150
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ out,
                               int64_t n, float eps) {
    __shared__ float red[32];
    float ss = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) ss += x[i] * x[i];
    const float total = block_sum(ss, red);
    const float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(n)), eps));
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fdiv_rn(__fmul_rn(x[i], w[i]), rms);
}

// src/math.rs:153-161
__global__ void softmax_kernel(const float* __restrict__ x, float* __restrict__ out, int64_t n) {
    __shared__ float red[32];
    __shared__ uint32_t kmax;
    if (threadIdx.x == 0) kmax = 0u;
    __syncthreads();
    uint32_t km = 0u;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) km = max(km, total_key(x[i]));
    atomicMax(&kmax, km);
    __syncthreads();
    const uint32_t kb = kmax;
    const float mx = __uint_as_float((kb & 0x80000000u) ? (kb & 0x7fffffffu) : ~kb);
    float s = 0.f;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(x[i] - mx);
        out[i] = e;
        s += e;
    }
    const float total = block_sum(s, red);
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fdiv_rn(out[i], total);
}

struct RopeTable {
    float c[64], s[64];
};

// src/math.rs:196-228, adjacent pairs; no FMA contraction (Rust never fuses).
__global__ void rope_kernel(float* __restrict__ q, int64_t nq, float* __restrict__ k, int64_t nk,
                            const RopeTable tab, int64_t dim) {
    const int64_t half = dim / 2;
    const int64_t pq = nq / dim * half, pk = nk / dim * half;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < pq + pk;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float* v = i < pq ? q : k;
        const int64_t j = i < pq ? i : i - pq;
        const int64_t a = j % half;
        float* p = v + (j / half) * dim + 2 * a;
        const float c = tab.c[a], s = tab.s[a];
        const float p0 = p[0], p1 = p[1];
        p[0] = __fadd_rn(__fmul_rn(c, p0), __fmul_rn(-s, p1));
        p[1] = __fadd_rn(__fmul_rn(s, p0), __fmul_rn(c, p1));
    }
}

// f32 -> f16 bits, round to nearest even, in 32-bit integer arithmetic (the
// rule of the `half` crate's f16::from_f32; NaN stays a quiet NaN).
__device__ __forceinline__ uint32_t f32_to_f16_bits(float f) {
    const uint32_t x = __float_as_uint(f);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t exp = (x >> 23) & 0xffu;
    const uint32_t man = x & 0x7fffffu;
    if (exp == 0xffu) return sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0u);
    const int e = static_cast<int>(exp) - 127 + 15;
    if (e >= 0x1f) return sign | 0x7c00u;
    if (e <= 0) {
        const int s = 14 - e;
        if (s > 24) return sign;
        const uint32_t m = man | 0x800000u;
        uint32_t q = m >> s;
        const uint32_t r = m & ((1u << s) - 1u), half = 1u << (s - 1);
        if (r > half || (r == half && (q & 1u))) ++q;
        return sign | q;
    }
    uint32_t h = sign | (static_cast<uint32_t>(e) << 10) | (man >> 13);
    const uint32_t r = man & 0x1fffu;
    if (r > 0x1000u || (r == 0x1000u && (h & 1u))) ++h;
    return h;
}

// src/kernels.rs:8-31, one thread per 32-value block, bit-exact.
__global__ void activated_q8_kernel(const float* __restrict__ x, int64_t nb, uint8_t* __restrict__ out) {
    for (int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; b < nb;
         b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float* pre = x + b * 32;
        int best = 0;
        for (int i = 1; i < 32; ++i)
            if (!(total_key(fabsf(pre[best])) > total_key(fabsf(pre[i])))) best = i;
        const float scale = __fdiv_rn(pre[best], 127.0f);
        const uint32_t h = f32_to_f16_bits(scale);
        uint8_t* post = out + b * 34;
        post[0] = static_cast<uint8_t>(h & 0xffu);
        post[1] = static_cast<uint8_t>((h >> 8) & 0xffu);
        for (int i = 0; i < 32; ++i) post[2 + i] = static_cast<uint8_t>(f32_as_i8(roundf(__fdiv_rn(pre[i], scale))));
    }
}

// src/math.rs:101-112 / :39-50.  One warp per output row; integer block dots
// (exact), block value (isum * sa) * sw, then the reference's sequential f32
// sum over blocks in order, starting from -0.0 (Rust `Sum for f32`).
__global__ void q8_act_matmul_kernel(const uint8_t* __restrict__ xb, const uint8_t* __restrict__ quants,
                                     const uint16_t* __restrict__ scales, float* __restrict__ out, int64_t n,
                                     int64_t k, int64_t sk) {
    extern __shared__ uint8_t sm[];
    const int64_t nb = k / 32;
    int8_t* xq = reinterpret_cast<int8_t*>(sm);                               // [nb][32]
    float* xs = reinterpret_cast<float*>(sm + ((nb * 32 + 15) / 16) * 16);   // [nb]
    float* vals = xs + nb;                                                    // [warps][nb]
    for (int64_t i = threadIdx.x; i < nb * 32; i += blockDim.x) xq[i] = static_cast<int8_t>(xb[(i / 32) * 34 + 2 + i % 32]);
    for (int64_t i = threadIdx.x; i < nb; i += blockDim.x) xs[i] = f16_at(xb + i * 34);
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    float* my = vals + warp * nb;
    for (int64_t row = blockIdx.x * static_cast<int64_t>(nw) + warp; row < n; row += static_cast<int64_t>(gridDim.x) * nw) {
        const uint8_t* wr = quants + row * k;
        for (int64_t b = lane; b < nb; b += 32) {
            const uint4* w4 = reinterpret_cast<const uint4*>(wr + b * 32);
            const int* x4 = reinterpret_cast<const int*>(xq + b * 32);
            int isum = 0;
            bool neg_zero = true;  // all 32 products are -0.0
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint4 w = w4[h];
                const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int xv = x4[h * 4 + j];
                    isum = __dp4a(static_cast<int>(ws[j]), xv, isum);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const int a = static_cast<int8_t>(xv >> (8 * e));
                        const int c = static_cast<int8_t>(ws[j] >> (8 * e));
                        neg_zero = neg_zero && (a == 0 || c == 0) && ((a < 0) != (c < 0));
                    }
                }
            }
            const float bs = (isum == 0 && neg_zero) ? -0.0f : static_cast<float>(isum);
            const float sw = __half2float(__ushort_as_half(scales[row * sk + b]));
            my[b] = __fmul_rn(__fmul_rn(bs, xs[b]), sw);
        }
        __syncwarp();
        if (lane == 0) {
            float total = -0.0f;
            for (int64_t b = 0; b < nb; ++b) total = __fadd_rn(total, my[b]);
            out[row] = total;
        }
        __syncwarp();
    }
}

// src/tokenizer.rs:152-167: max by total order, ties -> last index.
__global__ void argmax_kernel(const float* __restrict__ x, int64_t n, int32_t* __restrict__ out) {
    __shared__ unsigned long long best_s;
    if (threadIdx.x == 0) best_s = 0ull;
    __syncthreads();
    unsigned long long best = 0ull;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x)
        best = max(best, (static_cast<unsigned long long>(total_key(x[i])) << 32) | static_cast<uint32_t>(i));
    atomicMax(&best_s, best);
    __syncthreads();
    if (threadIdx.x == 0) *out = n > 0 ? static_cast<int32_t>(best_s & 0xffffffffu) : 0;
}

// src/forward.rs:86-174 for one position: one warp per query head, online
// softmax over chunks of 32 positions; caches [kv][max_ctx][64].
__global__ void attention_kernel(const float* __restrict__ q, const float* __restrict__ kc,
                                 const float* __restrict__ vc, float* __restrict__ out, int64_t qh, int64_t kvh,
                                 int64_t n_ctx, int64_t max_ctx) {
    const int64_t h = blockIdx.x;
    const int lane = threadIdx.x;
    const int64_t g = h / (qh / kvh);
    const float* qv = q + h * 64;
    const float* K = kc + g * max_ctx * 64;
    const float* V = vc + g * max_ctx * 64;
    const float q0 = qv[lane], q1 = qv[lane + 32];
    float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
    for (int64_t c0 = 0; c0 < n_ctx; c0 += 32) {
        const int nc = static_cast<int>(n_ctx - c0 < 32 ? n_ctx - c0 : 32);
        float s = -INFINITY;
        for (int t = 0; t < nc; ++t) {
            const float* kr = K + (c0 + t) * 64;
            float d = q0 * kr[lane] + q1 * kr[lane + 32];
#pragma unroll
            for (int o = 16; o; o >>= 1) d += __shfl_xor_sync(FULL, d, o);
            if (lane == t) s = d / 8.0f;
        }
        float cm = s;
#pragma unroll
        for (int o = 16; o; o >>= 1) cm = fmaxf(cm, __shfl_xor_sync(FULL, cm, o));
        const float mn = fmaxf(m, cm);
        const float pr = lane < nc ? expf(s - mn) : 0.f;
        const float corr = expf(m - mn);
        float ps = pr;
#pragma unroll
        for (int o = 16; o; o >>= 1) ps += __shfl_xor_sync(FULL, ps, o);
        l = l * corr + ps;
        o0 *= corr;
        o1 *= corr;
        for (int t = 0; t < nc; ++t) {
            const float pt = __shfl_sync(FULL, pr, t);
            o0 = fmaf(pt, V[(c0 + t) * 64 + lane], o0);
            o1 = fmaf(pt, V[(c0 + t) * 64 + lane + 32], o1);
        }
        m = mn;
    }
    out[h * 64 + lane] = o0 / l;
    out[h * 64 + lane + 32] = o1 / l;
}

// src/math.rs:171-175: silu(g) * u with IEEE division, no contraction.
__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                                int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = __fmul_rn(__fdiv_rn(g[i], __fadd_rn(1.0f, expf(-g[i]))), u[i]);
}

__global__ void fill_kernel(float* out, float v, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = v;
}

int grid_for(int64_t n, int threads) {
    int64_t g = (n + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > 148 * 16) g = 148 * 16;
    return static_cast<int>(g);
}

int last_err() { return static_cast<int>(cudaGetLastError()); }

}  // namespace

int launch_repack(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* quants, uint16_t* scales, int64_t sk,
                  int64_t step, int64_t off, void* stream) {
    if (rows * (k / 32) == 0) return 0;
    repack_kernel<<<grid_for(rows * (k / 32), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        blocks, rows, k, quants, scales, sk, step, off);
    return last_err();
}

int launch_repack_tiled(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* dst, int64_t n_total,
                        int64_t tile_rows, int64_t step, int64_t off, void* stream) {
    (void)n_total;
    if (rows <= 0) return 0;
    repack_tiled_kernel<<<grid_for(rows * (k / 32), 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        blocks, rows, k, dst, tile_rows, step, off);
    return last_err();
}

int launch_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, void* stream) {
    if (n_blocks == 0) return 0;
    dequant_kernel<<<grid_for(n_blocks * 32, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(blocks, n_blocks, out);
    return last_err();
}

int launch_rmsnorm(const float* x, const float* w, float* out, int64_t n, float eps, void* stream) {
    rmsnorm_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, w, out, n, eps);
    return last_err();
}

int launch_softmax(const float* x, float* out, int64_t n, void* stream) {
    softmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, out, n);
    return last_err();
}

int launch_rope(float* q, int64_t nq, float* k, int64_t nk, const float* cs, int64_t dim, void* stream) {
    RopeTable tab{};
    for (int64_t i = 0; i < dim / 2 && i < 64; ++i) {
        tab.c[i] = cs[i];
        tab.s[i] = cs[dim / 2 + i];
    }
    const int64_t pairs = (nq / dim + nk / dim) * (dim / 2);
    if (pairs == 0) return 0;
    rope_kernel<<<grid_for(pairs, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(q, nq, k, nk, tab, dim);
    return last_err();
}

int launch_activated_q8(const float* x, int64_t k, uint8_t* out, void* stream) {
    const int64_t nb = k / 32;
    if (nb == 0) return 0;
    activated_q8_kernel<<<grid_for(nb, 128), 128, 0, static_cast<cudaStream_t>(stream)>>>(x, nb, out);
    return last_err();
}

int launch_q8_act_matmul(const uint8_t* xb, const uint8_t* quants, const uint16_t* scales, float* out, int64_t n,
                         int64_t k, void* stream) {
    const int64_t nb = k / 32;
    const int threads = 256;
    const size_t smem = ((nb * 32 + 15) / 16) * 16 + nb * 4 + static_cast<size_t>(threads / 32) * nb * 4;
    static thread_local size_t configured = 0;
    if (smem > 48 * 1024 && smem > configured) {
        cudaFuncSetAttribute(q8_act_matmul_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        configured = smem;
    }
    const int grid = static_cast<int>((n + 7) / 8 < 148 * 4 ? (n + 7) / 8 : 148 * 4);
    q8_act_matmul_kernel<<<grid, threads, smem, static_cast<cudaStream_t>(stream)>>>(xb, quants, scales, out, n, k,
                                                                                     scale_stride(k));
    return last_err();
}

int launch_argmax(const float* x, int64_t n, int32_t* out, void* stream) {
    argmax_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(x, n, out);
    return last_err();
}

int launch_attention(const float* q, const float* kc, const float* vc, float* out, int64_t qh, int64_t kvh,
                     int64_t n_ctx, int64_t max_ctx, void* stream) {
    attention_kernel<<<static_cast<unsigned>(qh), 32, 0, static_cast<cudaStream_t>(stream)>>>(q, kc, vc, out, qh, kvh,
                                                                                             n_ctx, max_ctx);
    return last_err();
}

int launch_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream) {
    silu_mul_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(gate, up, out, n);
    return last_err();
}

int launch_fill_f32(float* out, float v, int64_t n, void* stream) {
    fill_kernel<<<grid_for(n, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(out, v, n);
    return last_err();
}

}  // namespace tir
