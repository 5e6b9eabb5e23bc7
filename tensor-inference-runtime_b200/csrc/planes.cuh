// planes.cuh -- the activation planes the tensor-core matmul reads
// (gemm.cu): per token row, every value scaled by a per-row power of two and
// split into f16 hi + lo, stored per (token tile, 64-column K step) as two
// 128B-swizzled K-major planes.  Shared by the plane-writer kernels (gemm.cu)
// and the batched decode attention (batch.cu), which writes the planes of a
// token row itself once the row's last kv head is done.
#pragma once
#include <cuda_fp16.h>

#include <cstdint>

namespace tir {

constexpr int kGKS = 64;            // K per matmul stage: one 128-byte f16 row
constexpr int kPlaneThreads = 256;  // threads of a plane-writing CTA (one token row)

// Byte offset of f16 element (row r, column c < 64) in a 128B-swizzled K-major
// plane: 8-row atoms of 1 KB, 16-byte chunk index XORed with r % 8.
__host__ __device__ __forceinline__ uint32_t sw128_offset(int r, int c) {
    return static_cast<uint32_t>((r >> 3) * 1024 + (r & 7) * 128 + ((((c >> 3) ^ (r & 7)) & 7) << 4) + (c & 7) * 2);
}

// Each plane-writer thread owns columns [8 ch, 8 ch + 8) for its chunks
// ch = tid + i * kPlaneThreads, i < plane_chunks(k), and keeps their values in
// registers from the first read to the last write.
constexpr int kPlaneMaxChunks = 3;  // k <= 3 x 8 x kPlaneThreads = 6144
__device__ __forceinline__ int plane_chunks(int64_t k) {
    const int64_t nch = k / 8;
    const int64_t tid = threadIdx.x;
    return tid < nch ? static_cast<int>((nch - 1 - tid) / kPlaneThreads + 1) : 0;
}

__device__ __forceinline__ void load8(const float* p, float* v) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

// load8 from L2 (data other CTAs of the same kernel wrote).
__device__ __forceinline__ void load8_cg(const float* p, float* v) {
    const float4 a = __ldcg(reinterpret_cast<const float4*>(p)), b = __ldcg(reinterpret_cast<const float4*>(p + 4));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ void store8(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// The planes of token row t from the thread's register values v (chunk i at
// v[8 i]): the row's largest magnitude m (a CTA reduction) sets 2^kx with
// m * 2^kx in [2^9, 2^10), then each value * 2^kx is split into f16 hi + lo
// and stored into the 128B-swizzled hi and lo planes of its (token tile,
// K step); inv[t] = 2^-kx.  A row that is not live gets zero planes.
__device__ __forceinline__ void planes_store(const float* v, int nc, bool live, int64_t t, int64_t k, int nt,
                                             uint8_t* __restrict__ planes, float* __restrict__ inv) {
    __shared__ float red[kPlaneThreads / 32];
    const int tid = threadIdx.x;
    float mx = 0.f;
    if (live)
#pragma unroll
        for (int i = 0; i < kPlaneMaxChunks * 8; ++i)
            if (i < nc * 8) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if ((tid & 31) == 0) red[tid >> 5] = mx;
    __syncthreads();
    mx = red[0];
#pragma unroll
    for (int i = 1; i < kPlaneThreads / 32; ++i) mx = fmaxf(mx, red[i]);
    int e = 0;
    float sx = 0.f, isx = 0.f;
    if (mx > 0.f && mx < 3.0e38f) {
        frexpf(mx, &e);  // 2^(e-1) <= mx < 2^e
        sx = ldexpf(1.0f, 10 - e);
        isx = ldexpf(1.0f, e - 10);
    }
    const int64_t plane = static_cast<int64_t>(nt) * kGKS * 2;
    const int64_t nks = k / kGKS, ttile = t / nt;
    const int tr = static_cast<int>(t % nt);
#pragma unroll
    for (int i = 0; i < kPlaneMaxChunks; ++i) {
        if (i >= nc) break;
        const int64_t c0 = (static_cast<int64_t>(tid) + static_cast<int64_t>(i) * kPlaneThreads) * 8, ks = c0 / kGKS;
        const int cc = static_cast<int>(c0 % kGKS);
        uint4 hv, lv;
        uint32_t* hp = &hv.x;
        uint32_t* lp = &lv.x;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float v0 = live ? v[8 * i + 2 * j] * sx : 0.f;
            const float v1 = live ? v[8 * i + 2 * j + 1] * sx : 0.f;
            const __half2 hi = __floats2half2_rn(v0, v1);
            const float2 hf = __half22float2(hi);
            const __half2 lo = __floats2half2_rn(v0 - hf.x, v1 - hf.y);
            hp[j] = *reinterpret_cast<const uint32_t*>(&hi);
            lp[j] = *reinterpret_cast<const uint32_t*>(&lo);
        }
        uint8_t* base = planes + (ttile * nks + ks) * (2 * plane);
        const uint32_t off = sw128_offset(tr, cc);
        *reinterpret_cast<uint4*>(base + off) = hv;
        *reinterpret_cast<uint4*>(base + plane + off) = lv;
    }
    if (tid == 0) inv[t] = isx;
}

}  // namespace tir
