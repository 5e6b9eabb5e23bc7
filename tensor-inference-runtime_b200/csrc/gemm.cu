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
// or 64 for small batches; K in steps of 64): warp 0 streams each step's
// pre-split activation planes (NT x 256 B) with one TMA bulk copy into a ring
// of GemmCfg::kRaw stages; each of the kGConvWarps converter warps' threads
// copies its own 16 bytes of the step's raw Q8_0 block (and the row's scales)
// with cp.async into a private ring kWStages steps ahead (each SM's copy
// engine spends a fixed time per copy, so a step takes one TMA copy, not two)
// and expands them into the 128B-swizzled f16 hi/lo A planes of a separate
// ring of kConv stages, in packed f16 arithmetic (two instructions per
// weight); one thread of warp 1 issues the
// tcgen05.mma of the step (4 K sub-steps x 3 passes) and commits both stages
// back; after the last step the converter warps read the f32 accumulator out
// of TMEM.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <vector>

#include "host.h"
#include "launch.cuh"
#include "parts.cuh"
#include "planes.cuh"
#include "ptx.cuh"
#include "runtime.h"

namespace tir {

// The plane writers keep a whole activation row in one CTA's registers.
constexpr int64_t kPlaneMaxK = static_cast<int64_t>(kPlaneMaxChunks) * 8 * kPlaneThreads;
static_assert(kPlaneMaxK >= kMaxK, "the plane writers cover every row the runtime accepts");

namespace {

constexpr int kGM = 128;    // weight rows per tile (UMMA M)
constexpr int kGConvWarps = 16;  // weight converters, then the epilogue (kGRowThreads warps per TMEM lane quarter)
constexpr int kGThreads = 64 + 32 * kGConvWarps;
constexpr int kGRowThreads = kGConvWarps / 4;     // converter threads per weight row
constexpr int kGConvCols = kGKS / kGRowThreads;    // columns of a row one converter thread expands
static_assert(kGConvWarps % 4 == 0 && kGConvCols == 16, "a converter thread expands 16 columns (one 16-byte copy)");
constexpr int kGWBytes = kGM * kGKS + kGM * 2 * 2;  // quants + 2 f16 scales per row
constexpr int kGPlaneA = kGM * kGKS * 2;            // one f16 weight plane of a stage (16 KB)
constexpr uint32_t kGErrTimeout = 25;
constexpr int kGMaxSplits = 16;  // split-K CTAs per tile

template <int NT>
struct GemmCfg {
    // Small token tiles issue a_hi x [x_hi | x_lo] as one MMA of N = 2 NT
    // (the two activation planes are adjacent rows of one K-major operand),
    // accumulating into TMEM columns [0, 2 NT), and a_lo x x_hi into [0, NT);
    // the epilogue adds column c and c + NT.  Large tiles issue the three
    // passes separately (N is at most 256).
    static constexpr bool kMergeLo = 2 * NT <= 256;
    static constexpr int kTmemCols = kMergeLo ? 2 * NT : NT;
    // TMA ring of the steps' activation planes.
    static constexpr int kRaw = NT >= 256 ? 2 : 3;
    // Each converter thread's own ring of its raw weight bytes (cp.async),
    // kWStages steps ahead: the weights take no TMA copy (each SM's copy
    // engine spends a fixed time per copy, and a step then needs only one).
    static constexpr int kWStages = NT >= 256 ? 3 : 4;
    // Expanded weight-plane stages: a stage returns to the converters only
    // when its MMAs have completed, so short steps need more of them.
    static constexpr int kConv = NT >= 256 ? 2 : 4;
    static constexpr int kPlaneX = NT * kGKS * 2;  // one f16 activation plane of a stage
};

template <int NT>
struct GemmSmem {
    using C = GemmCfg<NT>;
    uint8_t a[C::kConv][2 * kGPlaneA];            // weight planes hi | lo (128B-swizzled, K-major)
    uint8_t x[C::kRaw][2 * C::kPlaneX];           // activation planes hi | lo, as laid out in global (TMA target)
    uint4 wq[C::kWStages][kGConvWarps * 32];      // each converter thread's 16 quants of a step
    uint32_t ws[C::kWStages][kGConvWarps * 32];   // ... and its row's two f16 scales
    uint64_t full_x[C::kRaw], empty_x[C::kRaw], full_a[C::kConv], empty_a[C::kConv], acc;
    uint32_t tmem_base;
    int32_t ok;
    float inv_x[NT];  // 2^-kx of the tile's tokens
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
    float* y;                // [splits][tokens][y_ld]: the partial products of the K splits
    int32_t n, k, tokens, y_ld, ks_per_split;
    uint32_t* err;
    unsigned long long timeout_ns;
};


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

__device__ __forceinline__ void cp_async4_ca(void* dst_smem, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst_smem)), "l"(src) : "memory");
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

// Bounded wait on an mbarrier phase; false (error recorded) on expiry, or
// at once when an earlier launch already recorded an error (so a failing
// launch sequence ends quickly instead of timing out kernel by kernel).
__device__ __forceinline__ bool gwait(const GemmParams& p, uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t n = 0;; ++n) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((n & 63u) == 63u) {
            if (ld_relaxed_gpu(p.err) != 0u) return false;
            if (globaltimer_ns() - t0 > p.timeout_ns) {
                if (atomicCAS(p.err, 0u, kGErrTimeout) == 0u) p.err[3] = kGErrTimeout;  // [3]: left for the host
                return false;
            }
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(kGThreads, 1) gemm_q8_kernel(const __grid_constant__ GemmParams p) {
    constexpr int kRaw = GemmCfg<NT>::kRaw;
    constexpr int kConv = GemmCfg<NT>::kConv;
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
        for (int i = 0; i < kRaw; ++i) {
            mbar_init(&s.full_x[i], 1);
            mbar_init(&s.empty_x[i], 1);  // the MMAs' commit
        }
        for (int i = 0; i < kConv; ++i) {
            mbar_init(&s.full_a[i], kGConvWarps);
            mbar_init(&s.empty_a[i], 1);
        }
        mbar_init(&s.acc, 1);
        s.ok = 1;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s.tmem_base)),
                     "r"(static_cast<uint32_t>(GemmCfg<NT>::kTmemCols)));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = s.tmem_base;
    if (tid == 0) griddep_launch_dependents();

    if (warp == 0) {
        // ---- producer: the activation planes of each K step (after the
        // earlier work of the stream that writes them)
        if (lane == 0) {
            const uint8_t* xsrc = p.xp + (static_cast<size_t>(tt) * nks_all + ks0) * (2 * kGPlaneX);
            const int pre = min(nks, kRaw);
            griddep_wait();
            for (int i = 0; i < pre; ++i) {
                mbar_arrive_expect_tx(&s.full_x[i], 2 * kGPlaneX);
                bulk_g2s(s.x[i], xsrc + static_cast<size_t>(i) * (2 * kGPlaneX), 2 * kGPlaneX, &s.full_x[i]);
            }
            int issued = pre;
            for (int i = pre; i < nks; ++i) {
                const int st = i % kRaw;
                if (!gwait(p, &s.empty_x[st], ((i / kRaw) - 1) & 1)) {
                    s.ok = 0;
                    break;
                }
                mbar_arrive_expect_tx(&s.full_x[st], 2 * kGPlaneX);
                bulk_g2s(s.x[st], xsrc + static_cast<size_t>(i) * (2 * kGPlaneX), 2 * kGPlaneX, &s.full_x[st]);
                issued = i + 1;
            }
            // every copy issued lands before the CTA can leave
            for (int i = max(0, issued - kRaw); i < issued; ++i) gwait(p, &s.full_x[i % kRaw], (i / kRaw) & 1);
        }
    } else if (warp == 1) {
        // ---- MMA issue (one thread)
        if (lane == 0) {
            const uint32_t idesc = (1u << 4) | (static_cast<uint32_t>(NT >> 3) << 17) | (static_cast<uint32_t>(kGM >> 4) << 24);
            const uint32_t idesc2 =
                (1u << 4) | (static_cast<uint32_t>((2 * NT) >> 3) << 17) | (static_cast<uint32_t>(kGM >> 4) << 24);
            for (int i = 0; i < nks; ++i) {
                const int st = i % kRaw, sa = i % kConv;
                if (!gwait(p, &s.full_x[st], (i / kRaw) & 1) || !gwait(p, &s.full_a[sa], (i / kConv) & 1)) {
                    s.ok = 0;
                    break;
                }
                tc_fence_after();
                const uint32_t a_hi = smem_u32(s.a[sa]), a_lo = a_hi + kGPlaneA;
                const uint32_t x_hi = smem_u32(s.x[st]), x_lo = x_hi + kGPlaneX;
#pragma unroll
                for (int kk = 0; kk < kGKS / 16; ++kk) {
                    const uint32_t o = kk * 32;
                    if constexpr (GemmCfg<NT>::kMergeLo) {
                        umma_f16(tmem, umma_desc(a_hi + o), umma_desc(x_hi + o), idesc2, (i > 0 || kk > 0) ? 1u : 0u);
                    } else {
                        umma_f16(tmem, umma_desc(a_hi + o), umma_desc(x_hi + o), idesc, (i > 0 || kk > 0) ? 1u : 0u);
                        umma_f16(tmem, umma_desc(a_hi + o), umma_desc(x_lo + o), idesc, 1u);
                    }
                    umma_f16(tmem, umma_desc(a_lo + o), umma_desc(x_hi + o), idesc, 1u);
                }
                // the weight planes and the activation planes are free once these MMAs completed
                umma_commit(&s.empty_a[sa]);
                umma_commit(&s.empty_x[st]);
            }
            umma_commit(&s.acc);
        }
    } else {
        // ---- converters: threads r + 128 j (j < kGRowThreads) expand weight
        // row r of each step, columns [kGConvCols j, kGConvCols (j + 1)),
        // copying their own 16 quant bytes and the row's scales into their
        // ring slot kWStages steps ahead (the weights do not depend on
        // earlier work of the stream, so the first copies go out at once).  The raw
        // block holds q + 128 as bytes and f16 scales already multiplied by
        // the row's 2^kw, so a = q * s' (at most 19 significant bits, below
        // 2^15) splits in packed f16 arithmetic: hi = RN(q * s'), and
        // lo = q * s' - hi, exact in one fused multiply-add (at most 8
        // significant bits, all at or above the last bit of s').  Bytes become
        // f16 by the magic-number route: 0x64 << 8 | b is the f16 1024 + b.
        constexpr int kCh = kGConvCols / 8;
        constexpr int kWS = GemmCfg<NT>::kWStages;
        const int ct = tid - 64;
        const int r = ct & (kGM - 1), hc = ct >> 7;  // row, column part
        uint32_t offs[kCh];
#pragma unroll
        for (int ch = 0; ch < kCh; ++ch) offs[ch] = sw128_offset(r, hc * kGConvCols + ch * 8);
        const __half2 bias = __float2half2_rn(1152.0f);  // 1024 + 128
        const uint8_t* wsrc = p.w + (static_cast<size_t>(rt) * nks_all + ks0) * kGWBytes + r * kGKS + hc * kGConvCols;
        const uint8_t* ssrc = p.w + (static_cast<size_t>(rt) * nks_all + ks0) * kGWBytes + kGM * kGKS + r * 4;
        auto wissue = [&](int i) {  // one commit group per step (empty past the last)
            if (i < nks) {
                cp_async16(&s.wq[i % kWS][ct], wsrc + static_cast<size_t>(i) * kGWBytes);
                cp_async4_ca(&s.ws[i % kWS][ct], ssrc + static_cast<size_t>(i) * kGWBytes);
            }
            cp_async_commit();
        };
#pragma unroll
        for (int i = 0; i < kWS; ++i) wissue(i);
        bool ok = true;
        for (int i = 0; i < nks && ok; ++i) {
            const int sa = i % kConv;
            cp_async_wait<kWS - 1>();  // this thread's copies of step i landed
            const uint4 q16 = s.wq[i % kWS][ct];
            const uint32_t s2 = s.ws[i % kWS][ct];
            wissue(i + kWS);  // into the slot just read
            if (i >= kConv) ok = gwait(p, &s.empty_a[sa], ((i / kConv) - 1) & 1);
            if (ok) {
                const __half2 sc2 = *reinterpret_cast<const __half2*>(&s2);
                const __half2 sc = hc * kGConvCols >= 32 ? __high2half2(sc2) : __low2half2(sc2);
                const uint32_t qw[4] = {q16.x, q16.y, q16.z, q16.w};
                uint8_t* ahi = s.a[sa];
                uint8_t* alo = s.a[sa] + kGPlaneA;
#pragma unroll
                for (int ch = 0; ch < kCh; ++ch) {  // 8 columns per 16-byte chunk
                    const uint2 qv = make_uint2(qw[2 * ch], qw[2 * ch + 1]);
                    uint4 hv, lv;
                    uint32_t* hp = &hv.x;
                    uint32_t* lp = &lv.x;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const uint32_t word = e < 2 ? qv.x : qv.y;
                        const uint32_t h = __byte_perm(word, 0x64646464u, (e & 1) ? 0x4342u : 0x4140u);
                        const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&h), bias);
                        const __half2 hi = __hmul2(q, sc);
                        const __half2 lo = __hfma2(q, sc, __hneg2(hi));
                        hp[e] = *reinterpret_cast<const uint32_t*>(&hi);
                        lp[e] = *reinterpret_cast<const uint32_t*>(&lo);
                    }
                    *reinterpret_cast<uint4*>(ahi + offs[ch]) = hv;
                    *reinterpret_cast<uint4*>(alo + offs[ch]) = lv;
                }
                fence_proxy_async_smem();  // generic-proxy writes, read by the tensor cores
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&s.full_a[sa]);
        }
        cp_async_wait_all();  // no copy lands after the CTA leaves
        // ---- epilogue: TMEM lane quarter (warp % 4) holds weight rows 32 q .. 32 q + 31,
        // read by kGRowThreads warps, each a share of the tile's tokens; it reads
        // 2^-kx per token and may add into y: after earlier work
        griddep_wait();
        for (int i = tid - 64; i < NT; i += 32 * kGConvWarps) s.inv_x[i] = p.x_inv[tt * NT + i];
        asm volatile("bar.sync 1, %0;" ::"n"(32 * kGConvWarps) : "memory");  // the epilogue warps
        const bool acc_ok = __all_sync(0xffffffffu, ok && gwait(p, &s.acc, 0));
        tc_fence_after();
        const int q = warp & 3;
        const int row = q * 32 + lane;
        const int n = rt * kGM + row;
        const float inv_w = 1.0f / p.w_pow2[rt * kGM + row];
        const float* inv_x = s.inv_x;
        // split-K: CTA `split` stores its partial product as partial tile
        // `split` of y ([splits][tokens][y_ld]); the reader adds them up
        float* y = p.y + static_cast<size_t>(split) * p.tokens * p.y_ld;
        if (acc_ok) {  // warp-uniform: the TMEM loads are warp-collective
            const int part = (warp - 2) >> 2;  // this warp's share of the tile's tokens
            for (int c0 = part * (NT / kGRowThreads); c0 < (part + 1) * (NT / kGRowThreads); c0 += 16) {
                uint32_t v[16];
                tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, v);
                if constexpr (GemmCfg<NT>::kMergeLo) {  // + a_hi x x_lo from columns NT..2 NT
                    uint32_t w[16];
                    tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + NT + c0, w);
#pragma unroll
                    for (int j = 0; j < 16; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(w[j]));
                }
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int t = tt * NT + c0 + j;
                    if (t < p.tokens && n < p.n)
                        y[static_cast<size_t>(t) * p.y_ld + n] = __uint_as_float(v[j]) * inv_x[c0 + j] * inv_w;
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                                "r"(static_cast<uint32_t>(GemmCfg<NT>::kTmemCols)));
}

// ---- layouts -----------------------------------------------------------------

// Q8_0 blocks [n][k/32] -> [row tile][k step] blocks: 128 x 64 quants as
// q + 128 bytes (row-major), then 128 x 2 f16 scales multiplied by the row's
// 2^kw; rows past n stay zero.  2^kw, kept per row for the epilogue, brings
// 127 * (largest scale of the row) into [2^14, 2^15), so every scaled scale
// and every q * scale stays inside the f16 range.
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
    }
    // 127 * mx < 2^E  ->  2^kw = 2^(15 - E); zero or non-finite rows: 1
    int e = 0;
    const float m = 127.0f * mx;
    float pw = 1.0f;
    if (m > 0.f && m < 3.0e38f) {
        frexpf(m, &e);  // m = f * 2^e, f in [0.5, 1): 2^(e-1) <= m < 2^e
        pw = ldexpf(1.0f, 15 - e);
    }
    for (int64_t b = 0; b < nb; ++b) {
        const uint8_t* src = blocks + (row * nb + b) * 34;
        const uint16_t sb = static_cast<uint16_t>(src[0] | (src[1] << 8));
        uint8_t* dst = out + (rtile * nks + b / 2) * kGWBytes;
        uint4* q = reinterpret_cast<uint4*>(dst + r * kGKS + (b & 1) * 32);
        uint32_t w[8];
#pragma unroll
        for (int j = 0; j < 8; ++j)
            w[j] = (static_cast<uint32_t>(src[2 + 4 * j]) | (static_cast<uint32_t>(src[3 + 4 * j]) << 8) |
                    (static_cast<uint32_t>(src[4 + 4 * j]) << 16) | (static_cast<uint32_t>(src[5 + 4 * j]) << 24)) ^
                   0x80808080u;
        q[0] = make_uint4(w[0], w[1], w[2], w[3]);
        q[1] = make_uint4(w[4], w[5], w[6], w[7]);
        const __half sc = __float2half_rn(__half2float(__ushort_as_half(sb)) * pw);
        reinterpret_cast<uint16_t*>(dst + kGM * kGKS)[r * 2 + (b & 1)] = __half_as_ushort(sc);
    }
    pow2[row] = pw;
}

// Activation rows -> [token tile][k step] planes (hi | lo, 128B-swizzled,
// nt tokens x 64 columns each) and 2^-kx per token.  One CTA of kPlaneThreads
// per token row (rows t >= tokens of the last tile are written as zeros);
// val(c) gives column c of the row, evaluated once for the row's largest
// magnitude and once for the split.

// Planes of X [tokens][k] as given.
__global__ void __launch_bounds__(kPlaneThreads) gemm_x_planes_kernel(const float* __restrict__ x, int64_t tokens,
                                                                      int64_t k, int nt, uint8_t* __restrict__ planes,
                                                                      float* __restrict__ inv) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t t = blockIdx.x;
    const bool live = t < tokens;
    const int nc = plane_chunks(k);
    float v[kPlaneMaxChunks * 8];
#pragma unroll
    for (int i = 0; i < kPlaneMaxChunks; ++i)
        if (i < nc && live) load8(x + t * k + (threadIdx.x + static_cast<int64_t>(i) * kPlaneThreads) * 8, v + 8 * i);
    planes_store(v, nc, live, t, k, nt, planes, inv);
}

// Planes of rmsnorm(h) * w (src/math.rs:141-150, the division as a
// multiplication by the correctly rounded reciprocal), h = row
// rows ? rows[t] : t of X -- after X += Y on that row when Y is given (the
// residual add of src/forward.rs, fused here so the matmul before it only
// stores; X keeps the sum), Y the sum of y_parts partial tiles y_part floats
// apart, added in partial order.  rows[t] < 0 marks an unused slot (zero
// planes).
__global__ void __launch_bounds__(kPlaneThreads) gemm_norm_planes_kernel(float* __restrict__ X,
                                                                         const float* __restrict__ Y, int y_parts,
                                                                         int64_t y_part,
                                                                         const int32_t* __restrict__ rows,
                                                                         int64_t tokens, int64_t k,
                                                                         const float* __restrict__ w, float eps, int nt,
                                                                         uint8_t* __restrict__ planes,
                                                                         float* __restrict__ inv) {
    __shared__ float part[kPlaneThreads / 32];
    griddep_launch_dependents();
    griddep_wait();
    const int64_t t = blockIdx.x;
    // a gathered row index < 0 (an idle sequence) is not live: zero planes
    const int64_t xg = t < tokens ? (rows ? static_cast<int64_t>(rows[t]) : t) : -1;
    const bool live = xg >= 0;
    const int nc = plane_chunks(k);
    float v[kPlaneMaxChunks * 8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < kPlaneMaxChunks; ++i) {
        if (i >= nc || !live) continue;
        const int64_t c0 = (threadIdx.x + static_cast<int64_t>(i) * kPlaneThreads) * 8;
        float* x = X + xg * k + c0;
        load8(x, v + 8 * i);
        if (Y) {
            float y[8], yj[8];
            load8(Y + xg * k + c0, y);
            for (int j = 1; j < y_parts; ++j) {
                load8(Y + j * y_part + xg * k + c0, yj);
#pragma unroll
                for (int u = 0; u < 8; ++u) y[u] = __fadd_rn(y[u], yj[u]);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) v[8 * i + u] = __fadd_rn(v[8 * i + u], y[u]);
            store8(x, v + 8 * i);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) ss = fmaf(v[8 * i + u], v[8 * i + u], ss);
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float total = 0.f;
    for (int i = 0; i < kPlaneThreads / 32; ++i) total += part[i];
    const float r = __frcp_rn(__fsqrt_rn(__fadd_rn(__fdiv_rn(total, static_cast<float>(k)), eps)));
#pragma unroll
    for (int i = 0; i < kPlaneMaxChunks; ++i) {
        if (i >= nc || !live) continue;
        float wv[8];
        load8(w + (threadIdx.x + static_cast<int64_t>(i) * kPlaneThreads) * 8, wv);
#pragma unroll
        for (int u = 0; u < 8; ++u) v[8 * i + u] = __fmul_rn(__fmul_rn(v[8 * i + u], wv[u]), r);
    }
    planes_store(v, nc, live, t, k, nt, planes, inv);
}

// Planes of h[t][j] = silu(gate) * up from interleaved (gate_j, up_j) columns
// of GU [tokens][2 f] (src/math.rs:171-175), GU the sum of `parts` partial
// tiles `part` floats apart, added in partial order.
__global__ void __launch_bounds__(kPlaneThreads) gemm_silu_planes_kernel(const float* __restrict__ gu, int parts,
                                                                         int64_t part, int64_t tokens, int64_t f,
                                                                         int nt,
                                                                         uint8_t* __restrict__ planes,
                                                                         float* __restrict__ inv) {
    griddep_launch_dependents();
    griddep_wait();
    const int64_t t = blockIdx.x;
    const bool live = t < tokens;
    const int nc = plane_chunks(f);
    float v[kPlaneMaxChunks * 8];
#pragma unroll
    for (int i = 0; i < kPlaneMaxChunks; ++i) {
        if (i >= nc || !live) continue;
        const float* row = gu + t * 2 * f + (threadIdx.x + static_cast<int64_t>(i) * kPlaneThreads) * 16;
        float a[16], b[16];
        load8(row, a);
        load8(row + 8, a + 8);
        for (int j = 1; j < parts; ++j) {
            load8(row + j * part, b);
            load8(row + j * part + 8, b + 8);
#pragma unroll
            for (int u = 0; u < 16; ++u) a[u] = __fadd_rn(a[u], b[u]);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u)
            v[8 * i + u] = __fmul_rn(__fdiv_rn(a[2 * u], __fadd_rn(1.0f, expf(-a[2 * u]))), a[2 * u + 1]);
    }
    planes_store(v, nc, live, t, f, nt, planes, inv);
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
        // padded rows: 2^kw = 1 (their scales are zero)
        std::vector<float> ones(static_cast<size_t>(np - n), 1.0f);
        e = cudaMemcpyAsync(pow2 + n, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice, st);
        if (e != cudaSuccess) return static_cast<int>(e);
        e = cudaStreamSynchronize(st);
        if (e != cudaSuccess) return static_cast<int>(e);
    }
    gemm_repack_kernel<<<static_cast<unsigned>((n + 127) / 128), 128, 0, st>>>(blocks, n, k, out, pow2);
    return static_cast<int>(cudaGetLastError());
}

int launch_gemm_x_planes(const float* x, int64_t tokens, int64_t k, uint8_t* planes, float* inv, void* stream,
                         bool pdl) {
    if (k > kPlaneMaxK) return static_cast<int>(cudaErrorInvalidValue);  // one CTA covers a row
    return static_cast<int>(launch_kernel(gemm_x_planes_kernel, dim3(static_cast<unsigned>(gemm_tokens_padded(tokens))),
                                          dim3(kPlaneThreads), 0, static_cast<cudaStream_t>(stream), pdl, x, tokens, k,
                                          gemm_token_tile(tokens), planes, inv));
}

int launch_gemm_norm_planes(float* X, float* Y, int y_parts, int64_t y_part, const int32_t* rows, int64_t tokens,
                            int64_t k, const float* w, float eps, uint8_t* planes, float* inv, void* stream, bool pdl) {
    if (k > kPlaneMaxK) return static_cast<int>(cudaErrorInvalidValue);  // one CTA covers a row
    return static_cast<int>(launch_kernel(gemm_norm_planes_kernel,
                                          dim3(static_cast<unsigned>(gemm_tokens_padded(tokens))), dim3(kPlaneThreads),
                                          0, static_cast<cudaStream_t>(stream), pdl, X, Y, y_parts, y_part, rows, tokens,
                                          k, w, eps,
                                          gemm_token_tile(tokens), planes, inv));
}

int launch_gemm_silu_planes(float* gu, int parts, int64_t part, int64_t tokens, int64_t f, uint8_t* planes,
                            float* inv, void* stream, bool pdl) {
    if (f > kPlaneMaxK) return static_cast<int>(cudaErrorInvalidValue);  // one CTA covers a row
    return static_cast<int>(launch_kernel(gemm_silu_planes_kernel,
                                          dim3(static_cast<unsigned>(gemm_tokens_padded(tokens))), dim3(kPlaneThreads),
                                          0, static_cast<cudaStream_t>(stream), pdl, gu, parts, part, tokens, f,
                                          gemm_token_tile(tokens), planes, inv));
}

int64_t gemm_tile_count(int64_t n, int64_t tokens) {
    const int nt = gemm_token_tile(tokens);
    return ((n + kGM - 1) / kGM) * ((tokens + nt - 1) / nt);
}

// Opt the matmul kernels into their shared memory on the current device
// (once per thread and device; call it before capturing a launch in a graph).
int gemm_configure() {
    static thread_local int configured = -1;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return static_cast<int>(e);
    if (configured == dev) return 0;
    e = cudaFuncSetAttribute(gemm_q8_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(GemmSmem<64>) + 1024));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(gemm_q8_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(GemmSmem<256>) + 1024));
    if (e != cudaSuccess) return static_cast<int>(e);
    configured = dev;
    return 0;
}

// K steps per split and the number of splits actually used when asking for
// `splits` over k columns (every split non-empty).
int gemm_real_splits(int64_t k, int splits) {
    const int nks = static_cast<int>(k / kGKS);
    splits = std::max(1, std::min({splits, nks, kGMaxSplits}));
    const int per = (nks + splits - 1) / splits;
    return (nks + per - 1) / per;
}

// Split-K factor for a matmul on `sms` multiprocessors (one CTA each): none
// when the tiles alone fill the GPU, else the fewest waves of the shortest
// CTAs, each CTA paying about three K steps of pipeline fill.
int gemm_splits(int64_t n, int64_t k, int64_t tokens, int sms) {
    const int64_t tiles = gemm_tile_count(n, tokens), nks = k / kGKS;
    if (tiles <= 0 || nks <= 0 || sms <= 0 || tiles >= sms) return 1;
    int best = 1;
    int64_t best_cost = (tiles + sms - 1) / sms * (nks + 3);
    for (int sp = 2; sp <= std::min<int64_t>(nks, kGMaxSplits); ++sp) {
        if (gemm_real_splits(k, sp) != sp) continue;
        const int64_t per = (nks + sp - 1) / sp;
        const int64_t cost = (tiles * sp + sms - 1) / sms * (per + 3);
        if (cost < best_cost) {
            best_cost = cost;
            best = sp;
        }
    }
    return best;
}

// Partial products of y[t][n] (row stride y_ld) for t < tokens, n < n_rows:
// with s = gemm_real_splits(k, splits), partial j (K steps of split j) goes
// to y + j * tokens * y_ld, and y is their sum in order j = 0 .. s - 1.
int launch_gemm_q8(const uint8_t* w, const float* w_pow2, const uint8_t* planes, const float* x_inv, int64_t n,
                   int64_t k, int64_t tokens, float* y, int64_t y_ld, int splits, uint32_t* err,
                   unsigned long long timeout_ns, void* stream, bool pdl) {
    const int cfg = gemm_configure();
    if (cfg != 0) return cfg;
    const int nt = gemm_token_tile(tokens);
    const int nks = static_cast<int>(k / kGKS);
    splits = gemm_real_splits(k, splits);
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
    p.y = y;
    p.err = err;
    p.timeout_ns = timeout_ns;
    const dim3 grid(static_cast<unsigned>((n + kGM - 1) / kGM), static_cast<unsigned>((tokens + nt - 1) / nt),
                    static_cast<unsigned>(splits));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e = nt == 64 ? launch_kernel(gemm_q8_kernel<64>, grid, dim3(kGThreads),
                                                    sizeof(GemmSmem<64>) + 1024, st, pdl, p)
                                   : launch_kernel(gemm_q8_kernel<256>, grid, dim3(kGThreads),
                                                   sizeof(GemmSmem<256>) + 1024, st, pdl, p);
    return static_cast<int>(e);
}

// y[i] = sum of the `splits` partial tiles (stride `part` floats) at i, i < n.
__global__ void gemm_sum_parts_kernel(const float* __restrict__ y_parts, int splits, int64_t part, int64_t n,
                                      float* __restrict__ y) {
    griddep_launch_dependents();
    griddep_wait();
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float acc = y_parts[i];
        for (int j = 1; j < splits; ++j) acc = __fadd_rn(acc, y_parts[j * part + i]);
        y[i] = acc;
    }
}

int launch_gemm_sum_parts(const float* y_parts, int splits, int64_t part, int64_t n, float* y, void* stream, bool pdl) {
    const unsigned grid = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 148 * 8));
    return static_cast<int>(launch_kernel(gemm_sum_parts_kernel, dim3(grid), dim3(256), 0,
                                          static_cast<cudaStream_t>(stream), pdl, y_parts, splits, part, n, y));
}

}  // namespace tir
