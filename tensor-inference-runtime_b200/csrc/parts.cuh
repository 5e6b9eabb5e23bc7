// parts.cuh -- readers of split-K matmul outputs: the product is the sum of
// `parts` partial tiles `part` floats apart, added in partial order (so the
// result does not depend on scheduling).
#pragma once
#include <cstdint>

namespace tir {

// row[c] = sum over j < parts of row[j * part + c] for c < n, by the CTA's
// threads (each keeps 8 columns in flight per partial), then a CTA barrier.
// Every thread of the CTA must call it.
__device__ __forceinline__ void sum_parts_inplace(float* row, int parts, int64_t part, int n) {
    if (parts > 1) {
        const int nt = blockDim.x;
        for (int c0 = threadIdx.x; c0 < n; c0 += nt * 8) {
            float acc[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * nt;
                acc[u] = c < n ? row[c] : 0.f;
            }
            for (int j = 1; j < parts; ++j) {
                const float* pj = row + j * part;
#pragma unroll
                for (int u = 0; u < 8; ++u) {
                    const int c = c0 + u * nt;
                    if (c < n) acc[u] = __fadd_rn(acc[u], pj[c]);
                }
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                const int c = c0 + u * nt;
                if (c < n) row[c] = acc[u];
            }
        }
    }
    __syncthreads();
}

}  // namespace tir
