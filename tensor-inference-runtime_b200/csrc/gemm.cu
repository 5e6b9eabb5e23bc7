// gemm.cu -- batched Q8_0 matmul on the sm_100a tensor cores:
//   Y[t][n] = sum_k X[t][k] * f32(q[n][k]) * f32(scale[n][k / 32])
// for many tokens t at once (batched decode, prefill).  The reference applies
// q8_matmul (src/math.rs:87-98) token by token; this computes the same sums
// in a different order, to within f32 rounding.
//
// Exactness.  Every weight q * scale (8 + 11 significant bits) times a per-row
// power of two 2^kw is split exactly into two f16 values, a_hi + a_lo.  Every
// activation row is scaled by a per-token power of two 2^kx (so its largest
// magnitude lies in [2^9, 2^10)) and split into x_hi + x_lo (22 bits).  Three
// f16 x f16 -> f32 tensor-core passes (a_hi x_hi + a_hi x_lo + a_lo x_hi)
// accumulate in TMEM; the dropped a_lo x_lo term is below 2^-21 of the
// product, and the powers of two are divided out exactly in the epilogue.
//
// Data flow per CTA (one 128-row weight tile x one NT-token tile, NT = 256,
// or 64 for small batches; K in steps of 64): warp 0 streams each step's raw
// Q8_0 block (8.5 KB) and the step's pre-split activation planes (NT x 256 B)
// with TMA bulk copies into a 2- or 3-stage ring (each SM's copy engine spends
// a fixed time per copy, so the copies are few and large); warps 2-5 expand the raw block into the 128B-swizzled f16 hi/lo A
// planes; one thread of warp 1 issues the 12 tcgen05.mma of the step (4 K
// sub-steps x 3 passes) and commits the stage back to the producer; after the
// last step warps 2-5 read the f32 accumulator out of TMEM.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <vector>

#include "host.h"
#include "ptx.cuh"
#include "runtime.h"

namespace tir {

namespace {

constexpr int kGM = 128;    // weight rows per tile (UMMA M)
constexpr int kGKS = 64;    // K per stage: one 128-byte f16 row
constexpr int kGThreads = 192;
constexpr int kGWBytes = kGM * kGKS + kGM * 2 * 2;  // quants + 2 f16 scales per row
constexpr int kGPlaneA = kGM * kGKS * 2;            // one f16 weight plane of a stage (16 KB)
constexpr uint32_t kGErrTimeout = 25;

template <int NT>
struct GemmCfg {
    static constexpr int kStages = NT >= 256 ? 2 : 3;
    static constexpr int kPlaneX = NT * kGKS * 2;  // one f16 activation plane of a stage
};

template <int NT>
struct GemmSmem {
    static constexpr int S = GemmCfg<NT>::kStages;
    uint8_t a[S][2 * kGPlaneA];                   // weight planes hi | lo (128B-swizzled, K-major)
    uint8_t x[S][2 * GemmCfg<NT>::kPlaneX];       // activation planes hi | lo, as laid out in global
    uint8_t w[S][kGWBytes];                       // raw Q8_0 block of the step (TMA target)
    uint64_t full_raw[S], full_a[S], empty[S], acc;
    uint32_t tmem_base;
    int32_t ok;
    float inv_x[NT];
};
static_assert(offsetof(GemmSmem<256>, x) % 1024 == 0 && offsetof(GemmSmem<64>, x) % 1024 == 0,
              "swizzle atoms need 1 KB");
static_assert(sizeof(GemmSmem<256>) + 1024 <= 227 * 1024 && sizeof(GemmSmem<64>) + 1024 <= 227 * 1024,
              "shared memory budget");

struct GemmParams {
    const uint8_t* w;        // tiled weights: [row tile][k step] blocks of kGWBytes
    const float* w_pow2;     // [n rounded up to 128]: 2^kw of each row
    const uint8_t* xp;       // activation planes: [token tile][k step][hi | lo]
    const float* x_inv;      // [tokens rounded up to 128]: 2^-kx of each token
    float* y;                // [splits][tokens][y_ld]
    int32_t n, k, tokens, y_ld, ks_per_split;
    uint32_t* err;
    unsigned long long timeout_ns;
};

// Byte offset of f16 element (row r, column c < 64) in a 128B-swizzled K-major
// plane: 8-row atoms of 1 KB, 16-byte chunk index XORed with r % 8.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
    return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + (c & 7) * 2);
}

__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr) {
    // start address, LBO 16 B (unused with swizzle), SBO 1 KB, version 1, SWIZZLE_128B
    return static_cast<uint64_t>((saddr >> 4) & 0x3FFFu) | (1ull << 16) | (static_cast<uint64_t>(1024 >> 4) << 32) |
           (1ull << 46) | (2ull << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Bounded wait on an mbarrier phase; false (error recorded) on expiry.
__device__ __forceinline__ bool gwait(const GemmParams& p, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 0;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63u) == 63u && globaltimer_ns() - t0 > p.timeout_ns) {
            atomicCAS(p.err, 0u, kGErrTimeout);
            return false;
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(kGThreads, 1) gemm_q8_kernel(const __grid_constant__ GemmParams p) {
    constexpr int kGStages = GemmCfg<NT>::kStages;
    constexpr int kGPlaneX = GemmCfg<NT>::kPlaneX;
    extern __shared__ uint8_t g_smem_raw[];
    GemmSmem<NT>& s =
        *reinterpret_cast<GemmSmem<NT>*>((reinterpret_cast<uintptr_t>(g_smem_raw) + 1023) & ~uintptr_t(1023));
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rt = blockIdx.x, tt = blockIdx.y, split = blockIdx.z;
    const int nks_all = p.k / kGKS;
    const int ks0 = split * p.ks_per_split;
    const int nks = min(nks_all, ks0 + p.ks_per_split) - ks0;
    if (tid == 0) {
        for (int i = 0; i < kGStages; ++i) {
            mbar_init(&s.full_raw[i], 1);
            mbar_init(&s.full_a[i], 4);
            mbar_init(&s.empty[i], 1);
        }
        mbar_init(&s.acc, 1);
        s.ok = 1;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem_base)),
                     "r"(static_cast<uint32_t>(NT)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    for (int i = tid; i < NT; i += kGThreads) s.inv_x[i] = p.x_inv[tt * NT + i];
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;

    if (warp == 0) {
        // ---- producer: raw weight block + activation planes of each K step
        if (lane == 0) {
            for (int i = 0; i < nks; ++i) {
                const int st = i % kGStages;
                if (i >= kGStages && !gwait(p, &s.empty[st], ((i / kGStages) - 1) & 1)) {
                    s.ok = 0;
                    break;
                }
                mbar_arrive_expect_tx(&s.full_raw[st], kGWBytes + 2 * kGPlaneX);
                bulk_g2s(s.w[st], p.w + (static_cast<size_t>(rt) * nks_all + ks0 + i) * kGWBytes, kGWBytes,
                         &s.full_raw[st]);
                bulk_g2s(s.x[st], p.xp + (static_cast<size_t>(tt) * nks_all + ks0 + i) * (2 * kGPlaneX), 2 * kGPlaneX,
                         &s.full_raw[st]);
            }
            // every copy issued lands before the CTA can leave
            for (int i = max(0, nks - kGStages); i < nks; ++i) gwait(p, &s.full_raw[i % kGStages], (i / kGStages) & 1);
        }
    } else if (warp == 1) {
        // ---- MMA issue (one thread)
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(NT >> 3) << 17) | (static_cast<uint32_t>(kGM >> 4) << 24);
            for (int i = 0; i < nks; ++i) {
                const int st = i % kGStages;
                if (!gwait(p, &s.full_raw[st], (i / kGStages) & 1) || !gwait(p, &s.full_a[st], (i / kGStages) & 1)) {
                    s.ok = 0;
                    break;
                }
                tc_fence_after();
                const uint32_t a_hi = smem_u32(s.a[st]), a_lo = a_hi + kGPlaneA;
                const uint32_t x_hi = smem_u32(s.x[st]), x_lo = x_hi + kGPlaneX;
#pragma unroll
                for (int kk = 0; kk < kGKS / 16; ++kk) {
                    const uint32_t o = kk * 32;
                    umma_f16(tmem, umma_desc(a_hi + o), umma_desc(x_hi + o), idesc, (i > 0 || kk > 0) ? 1u : 0u);
                    umma_f16(tmem, umma_desc(a_hi + o), umma_desc(x_lo + o), idesc, 1u);
                    umma_f16(tmem, umma_desc(a_lo + o), umma_desc(x_hi + o), idesc, 1u);
                }
                umma_commit(&s.empty[st]);  // the stage is free once these MMAs completed
            }
            umma_commit(&s.acc);
        }
    } else {
        // ---- converters: thread r expands weight row r of each step
        const int r = tid - 64;
        const float pw = p.w_pow2[rt * kGM + r];
        bool ok = true;
        for (int i = 0; i < nks && ok; ++i) {
            const int st = i % kGStages;
            ok = gwait(p, &s.full_raw[st], (i / kGStages) & 1);
            if (ok) {
                const uint8_t* wq = s.w[st] + r * kGKS;
                const __half* ws = reinterpret_cast<const __half*>(s.w[st] + kGM * kGKS) + r * 2;
                const float s0 = __half2float(ws[0]) * pw, s1 = __half2float(ws[1]) * pw;
                uint8_t* ahi = s.a[st];
                uint8_t* alo = s.a[st] + kGPlaneA;
#pragma unroll
                for (int ch = 0; ch < 8; ++ch) {  // 8 columns per 16-byte chunk
                    const uint2 qv = *reinterpret_cast<const uint2*>(wq + ch * 8);
                    const float sc = ch < 4 ? s0 : s1;
                    __align__(16) __half hi[8];
                    __align__(16) __half lo[8];
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const uint32_t word = e < 4 ? qv.x : qv.y;
                        const float a = static_cast<float>(static_cast<int8_t>((word >> (8 * (e & 3))) & 0xffu)) * sc;
                        hi[e] = __float2half_rn(a);
                        lo[e] = __float2half_rn(a - __half2float(hi[e]));
                    }
                    const uint32_t off = sw128_offset(r, ch * 8);
                    *reinterpret_cast<uint4*>(ahi + off) = *reinterpret_cast<const uint4*>(hi);
                    *reinterpret_cast<uint4*>(alo + off) = *reinterpret_cast<const uint4*>(lo);
                }
                fence_proxy_async_smem();  // generic-proxy writes, read by the tensor cores
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.full_a[st]);
        }
        // ---- epilogue: TMEM lane quarter (warp % 4) holds weight rows 32 q .. 32 q + 31
        const bool acc_ok = __all_sync(0xffffffffu, ok && gwait(p, &s.acc, 0));
        tc_fence_after();
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int n = rt * kGM + row;
        const float inv_w = 1.0f / p.w_pow2[rt * kGM + row];
        if (acc_ok) {
            for (int c0 = 0; c0 < NT; c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = tt * NT + c0 + j;
                    if (t < p.tokens && n < p.n)
                        p.y[(static_cast<size_t>(split) * p.tokens + t) * p.y_ld + n] =
                            __uint_as_float(v[j]) * s.inv_x[c0 + j] * inv_w;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                                "r"(static_cast<uint32_t>(NT)));
}

// ---- layouts -----------------------------------------------------------------

// Q8_0 blocks [n][k/32] -> [row tile][k step] blocks: 128 x 64 int8 quants
// (row-major), then 128 x 2 f16 scales; rows past n stay zero.  Also 2^kw per
// row: the power of two that brings 127 * (largest scale of the row) into
// [2^14, 2^15).
__global__ void gemm_repack_kernel(const uint8_t* __restrict__ blocks, int64_t n, int64_t k, uint8_t* __restrict__ out,
                                   float* __restrict__ pow2) {
    const int64_t nb = k / 32, nks = k / kGKS;
    const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (row >= n) return;
    const int64_t rtile = row / kGM, r = row % kGM;
    float mx = 0.f;
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* src = blocks + (row * nb + b) * 34;
        const uint16_t sb = static_cast<uint16_t>(src[0] | (src[1] << 8));
        mx = fmaxf(mx, fabsf(__half2float(__ushort_as_half(sb))));
        uint8_t* dst = out + (rtile * nks + b / 2) * kGWBytes;
        uint4* q = reinterpret_cast<uint4*>(dst + r * kGKS + (b & 1) * 32);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = static_cast<uint32_t>(src[2 + 4 * j]) | (static_cast<uint32_t>(src[3 + 4 * j]) << 8) |
                   (static_cast<uint32_t>(src[4 + 4 * j]) << 16) | (static_cast<uint32_t>(src[5 + 4 * j]) << 24);
        q[0] = make_uint4(w[0], w[1], w[2], w[3]);
        q[1] = make_uint4(w[4], w[5], w[6], w[7]);
        reinterpret_cast<uint16_t*>(dst + kGM * kGKS)[r * 2 + (b & 1)] = sb;
    }
    // 127 * mx < 2^E  ->  2^kw = 2^(15 - E); zero or non-finite rows: 1
    int e = 0;
    const float m = 127.0f * mx;
    float pw = 1.0f;
    if (m > 0.f && m < 3.0e38f) {
        frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1): 2^(e-1) <= m < 2^e
        pw = ldexpf(1.0f, 15 - e);
    }
    pow2[row] = pw;
}

// Activations X [tokens][k] f32 -> [token tile][k step] planes (hi | lo,
// 128B-swizzled, nt tokens x 64 columns each) and 2^-kx per token, one warp
// per token (tile rows past `tokens` are zero).
__global__ void gemm_x_planes_kernel(const float* __restrict__ x, int64_t tokens, int64_t k, int64_t tokens_pad,
                                     int nt, uint8_t* __restrict__ planes, float* __restrict__ inv) {
    const int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (t >= tokens_pad) return;
    const int64_t plane = static_cast<int64_t>(nt) * kGKS * 2;
    const int64_t nks = k / kGKS, ttile = t / nt, tr = t % nt;
    const float* row = x + t * k;
    float mx = 0.f;
    if (t < tokens)
        for (int64_t c = lane; c < k; c += 32) mx = fmaxf(mx, fabsf(row[c]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int e = 0;
    float sx = 0.f, isx = 0.f;
    if (mx > 0.f && mx < 3.0e38f) {
        frexpf(mx, &e);  // 2^(e-1) <= mx < 2^e
        sx = ldexpf(1.0f, 10 - e);
        isx = ldexpf(1.0f, e - 10);
    }
    for (int64_t ch = lane; ch < k / 8; ch += 32) {  // 8-column chunks
        const int64_t c0 = ch * 8, ks = c0 / kGKS, cc = c0 % kGKS;
        __align__(16) __half hi[8];
        __align__(16) __half lo[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float v = t < tokens ? row[c0 + j] * sx : 0.f;
            hi[j] = __float2half_rn(v);
            lo[j] = __float2half_rn(v - __half2float(hi[j]));
        }
        uint8_t* base = planes + (ttile * nks + ks) * (2 * plane);
        const uint32_t off = sw128_offset(static_cast<int>(tr), static_cast<int>(cc));
        *reinterpret_cast<uint4*>(base + off) = *reinterpret_cast<const uint4*>(hi);
        *reinterpret_cast<uint4*>(base + plane + off) = *reinterpret_cast<const uint4*>(lo);
    }
    if (lane == 0) inv[t] = isx;
}

// Sum of the split-K partial products, [splits][tokens][ld] -> [tokens][ld].
__global__ void gemm_reduce_kernel(const float* __restrict__ part, int splits, int64_t tokens, int64_t n, int64_t ld,
                                   float* __restrict__ y) {
    const int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
    if (i >= tokens * n) return;
    const int64_t t = i / n, c = i % n;
    float acc = 0.f;
    for (int sp = 0; sp < splits; ++sp) acc += part[(static_cast<int64_t>(sp) * tokens + t) * ld + c];
    y[t * ld + c] = acc;
}

}  // namespace

int64_t gemm_q8_weight_bytes(int64_t n, int64_t k) {
    return ((n + kGM - 1) / kGM) * (k / kGKS) * kGWBytes;
}
int64_t gemm_q8_rows_padded(int64_t n) { return (n + kGM - 1) / kGM * kGM; }
// Token tile of a matmul over `tokens` activation rows: 64 for small batches
// (decode), else 256.
int gemm_token_tile(int64_t tokens) { return tokens <= 64 ? 64 : 256; }
int64_t gemm_x_plane_bytes(int64_t tokens, int64_t k) {
    const int nt = gemm_token_tile(tokens);
    return ((tokens + nt - 1) / nt) * (k / kGKS) * 2 * (static_cast<int64_t>(nt) * kGKS * 2);
}
int64_t gemm_tokens_padded(int64_t tokens) {
    const int nt = gemm_token_tile(tokens);
    return (tokens + nt - 1) / nt * nt;
}

int launch_gemm_repack(const uint8_t* blocks, int64_t n, int64_t k, uint8_t* out, float* pow2, void* stream) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(out, 0, static_cast<size_t>(gemm_q8_weight_bytes(n, k)), st);
    if (e != cudaSuccess) return static_cast<int>(e);
    const int64_t np = gemm_q8_rows_padded(n);
    if (np > n) {
        // padded rows: scale 1 (their quants are zero)
        std::vector<float> ones(static_cast<size_t>(np - n), 1.0f);
        e = cudaMemcpyAsync(pow2 + n, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return static_cast<int>(e);
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    gemm_repack_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, st>>>(blocks, n, k, out, pow2);
    return static_cast<int>(cudaGetLastError());
}

int launch_gemm_x_planes(const float* x, int64_t tokens, int64_t k, uint8_t* planes, float* inv, void* stream) {
    const int64_t tp = gemm_tokens_padded(tokens);
    gemm_x_planes_kernel<<<static_cast<unsigned>((tp + 7) / 8), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        x, tokens, k, tp, gemm_token_tile(tokens), planes, inv);
    return static_cast<int>(cudaGetLastError());
}

// y[t][n] (row stride y_ld) for t < tokens, n < n_rows; `part` (splits x
// tokens x y_ld floats) is scratch for split-K, used when splits > 1.
int launch_gemm_q8(const uint8_t* w, const float* w_pow2, const uint8_t* planes, const float* x_inv, int64_t n,
                   int64_t k, int64_t tokens, float* y, int64_t y_ld, int splits, float* part, uint32_t* err,
                   unsigned long long timeout_ns, void* stream) {
    static thread_local int configured = -1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (configured != dev) {
        cudaError_t e = cudaFuncSetAttribute(gemm_q8_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(sizeof(GemmSmem<64>) + 1024));
        if (e == cudaSuccess)
            e = cudaFuncSetAttribute(gemm_q8_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(sizeof(GemmSmem<256>) + 1024));
        if (e != cudaSuccess) return static_cast<int>(e);
        configured = dev;
    }
    const int nt = gemm_token_tile(tokens);
    const int nks = static_cast<int>(k / kGKS);
    if (splits < 1) splits = 1;
    if (splits > nks) splits = nks;
    GemmParams p{};
    p.w = w;
    p.w_pow2 = w_pow2;
    p.xp = planes;
    p.x_inv = x_inv;
    p.n = static_cast<int32_t>(n);
    p.k = static_cast<int32_t>(k);
    p.tokens = static_cast<int32_t>(tokens);
    p.y_ld = static_cast<int32_t>(y_ld);
    p.ks_per_split = (nks + splits - 1) / splits;
    splits = (nks + p.ks_per_split - 1) / p.ks_per_split;
    p.y = splits > 1 ? part : y;
    p.err = err;
    p.timeout_ns = timeout_ns;
    const dim3 grid(static_cast<unsigned>((n + kGM - 1) / kGM), static_cast<unsigned>((tokens + nt - 1) / nt),
                    static_cast<unsigned>(splits));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (nt == 64)
        gemm_q8_kernel<64><<<grid, kGThreads, sizeof(GemmSmem<64>) + 1024, st>>>(p);
    else
        gemm_q8_kernel<256><<<grid, kGThreads, sizeof(GemmSmem<256>) + 1024, st>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || splits == 1) return static_cast<int>(e);
    const int64_t total = tokens * n;
    gemm_reduce_kernel<<<static_cast<unsigned>((total + 255) / 256), 256, 0, st>>>(part, splits, tokens, n, y_ld, y);
    return static_cast<int>(cudaGetLastError());
}

}  // namespace tir
