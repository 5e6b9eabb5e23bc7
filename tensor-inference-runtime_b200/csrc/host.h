// host.h -- host-side internals shared by the C ABI implementation files.
#pragma once
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/tir.h"

namespace tir {

// Thread-local error reporting (tir_last_error).
tir_status fail(tir_status st, const std::string& msg);
void clear_error();

// Limit of every bounded device-side wait: TIR_TIMEOUT_MS (default 2000 ms).
unsigned long long timeout_ns();

// The library's allocation calls (counted; failable on demand for tests,
// tir_debug_fail_alloc_after).
cudaError_t dev_malloc(void** p, size_t bytes);
cudaError_t dev_malloc_async(void** p, size_t bytes, cudaStream_t stream);
cudaError_t host_malloc_pinned(void** p, size_t bytes);
template <typename T>
cudaError_t dev_malloc(T** p, size_t bytes) {
    return dev_malloc(reinterpret_cast<void**>(p), bytes);
}
template <typename T>
cudaError_t host_malloc_pinned(T** p, size_t bytes) {
    return host_malloc_pinned(reinterpret_cast<void**>(p), bytes);
}

// The sticky error word of tir_swiglu_static's control block on `device`
// (0: none), cleared by the read.  Makes no allocation.
tir_status static_scratch_take_error(int device, uint32_t* code);

// ---- GGUF (src/state.rs, src/reader.rs) ------------------------------------
struct MetaValue {
    uint32_t vtype = 0;
    uint64_t u = 0;
    int64_t i = 0;
    double f = 0.0;
    std::string str;
    uint32_t array_type = 0;
    std::vector<MetaValue> items;
};

struct MetaField {
    std::string name;
    MetaValue value;
};

struct TensorInfo {
    std::string name;
    uint32_t n_dims = 0;
    std::vector<uint64_t> shape;
    uint32_t dtype = 0;
    uint64_t offset = 0;
    const uint8_t* data = nullptr;
    size_t data_bytes = 0;
};

}  // namespace tir

struct tir_gguf {
    std::vector<uint8_t> owned;
    void* map_base = nullptr;
    size_t map_len = 0;
    const uint8_t* data = nullptr;
    size_t len = 0;
    uint32_t version = 0;
    std::vector<tir::MetaField> fields;
    std::vector<tir::TensorInfo> tensors;
    std::unordered_map<std::string, size_t> index;
    bool has_transformer = false;
    tir_transformer transformer{};
    ~tir_gguf();
};

namespace tir {
// A weight matrix in HBM: tile-major (q = the tiled matrix, s unused, r rows
// per tile) for the streamed projections, split (q [n][k], s [n][sk]) for the
// embedding table, which is read one row at a time.
struct Mat {
    uint8_t* q = nullptr;
    uint16_t* s = nullptr;
    int64_t n = 0, k = 0, sk = 0, r = 0;
    bool tiled = false;
};

}  // namespace tir

struct tir_model {
    int device = 0;
    tir_transformer t{};
    uint8_t* dev = nullptr;
    size_t dev_bytes = 0;
    uint64_t weight_bytes = 0;  // quants + scales + norm weights
    std::vector<tir::Mat> qkv, o, gu, down;
    tir::Mat lm, embd;
    std::vector<float*> attn_norm, ffn_norm;
    float* out_norm = nullptr;
    ~tir_model();
};

namespace tir {

// Parses a complete file image held by `g` (g->data/len set): load_model's
// parse (src/lib.rs:29-138).
tir_status gguf_parse_all(tir_gguf* g);
// parse_general (src/reader.rs:98-169).
tir_status gguf_parse_general(const uint8_t* map, size_t len, size_t offset, uint64_t count,
                              std::vector<MetaField>& out, size_t& end);
const TensorInfo* gguf_find(const tir_gguf* g, const std::string& name);

// ---- op-level kernel launchers (ops.cu) -------------------------------------
int launch_repack(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* quants, uint16_t* scales,
                  int64_t sk, int64_t dst_row_step, int64_t dst_row_off, void* stream);
int launch_repack_tiled(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* dst, int64_t n_total,
                        int64_t tile_rows, int64_t dst_row_step, int64_t dst_row_off, void* stream);
int launch_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, void* stream);
int launch_rmsnorm(const float* x, const float* w, float* out, int64_t n, float eps, void* stream);
int launch_softmax(const float* x, float* out, int64_t n, void* stream);
int launch_rope(float* q, int64_t nq, float* k, int64_t nk, const float* cs, int64_t dim,
                void* stream);
int launch_activated_q8(const float* x, int64_t k, uint8_t* out, void* stream);
int launch_q8_act_matmul(const uint8_t* xb, const uint8_t* quants, const uint16_t* scales,
                         float* out, int64_t n, int64_t k, void* stream);
int launch_argmax(const float* x, int64_t n, int32_t* out, void* stream);
int launch_attention(const float* q, const float* kc, const float* vc, float* out, int64_t qh,
                     int64_t kvh, int64_t n_ctx, int64_t max_ctx, void* stream);
int launch_silu_mul(const float* gate, const float* up, float* out, int64_t n, void* stream);
int launch_fill_f32(float* out, float v, int64_t n, void* stream);

// Streaming Q8_0 matvec (decode.cu machinery, one phase) over the split
// layout (quants, scales) or, with scales == NULL, the tile-major layout.
tir_status q8_matmul_stream(const float* x, const uint8_t* quants, const uint16_t* scales, float* out,
                            int64_t n, int64_t k, void* stream, bool qact = false);

// Batched Q8_0 matmul on the tensor cores (gemm.cu).
int64_t gemm_q8_weight_bytes(int64_t n, int64_t k);
int64_t gemm_q8_rows_padded(int64_t n);
int64_t gemm_x_plane_bytes(int64_t tokens, int64_t k);
int64_t gemm_tokens_padded(int64_t tokens);
int gemm_token_tile(int64_t tokens);  // token rows per matmul tile (64 or 256)
int launch_gemm_repack(const uint8_t* blocks, int64_t n, int64_t k, uint8_t* out, float* pow2, void* stream);
// pdl: launched with a programmatic dependency on the stream's previous work.
int launch_gemm_x_planes(const float* x, int64_t tokens, int64_t k, uint8_t* planes, float* inv, void* stream,
                         bool pdl = false);
// Planes of rmsnorm(X[r]) * w, r = rows ? rows[t] : t for t < tokens, after
// X[r] += Y[r] when Y is not null (X keeps the sum), Y the sum of y_parts
// partial tiles y_part floats apart, added in partial order (Y is left as it
// is).  Gathered rows must be distinct; a negative rows[t] gives zero planes
// for t.
int launch_gemm_norm_planes(float* X, float* Y, int y_parts, int64_t y_part, const int32_t* rows, int64_t tokens,
                            int64_t k, const float* w, float eps, uint8_t* planes, float* inv, void* stream,
                            bool pdl = false);
// Planes of silu(gate) * up from interleaved (gate, up) columns of gu
// [tokens][2 f], the sum of `parts` partial tiles `part` floats apart, added
// in partial order (gu is left as it is).
int launch_gemm_silu_planes(float* gu, int parts, int64_t part, int64_t tokens, int64_t f, uint8_t* planes,
                            float* inv, void* stream, bool pdl = false);
// Shared-memory opt-in of the matmul kernels on the current device (0 or a cudaError_t).
int gemm_configure();
// Weight-row tiles x token tiles of a matmul of n rows over `tokens` rows.
int64_t gemm_tile_count(int64_t n, int64_t tokens);
// Split-K factor for a matmul on `sms` multiprocessors, and the number of
// splits (partial tiles) a request for `splits` yields.
int gemm_splits(int64_t n, int64_t k, int64_t tokens, int sms);
int gemm_real_splits(int64_t k, int splits);
// Partial products of y = the planes' rows x the prepared weights: partial j
// of s = gemm_real_splits(k, splits) at y + j * tokens * y_ld (y is their sum
// in order).
int launch_gemm_q8(const uint8_t* w, const float* w_pow2, const uint8_t* planes, const float* x_inv, int64_t n,
                   int64_t k, int64_t tokens, float* y, int64_t y_ld, int splits, uint32_t* err,
                   unsigned long long timeout_ns, void* stream, bool pdl = false);
// y[i] = sum of `splits` partial tiles (stride `part` floats), i < n.
int launch_gemm_sum_parts(const float* y_parts, int splits, int64_t part, int64_t n, float* y, void* stream,
                          bool pdl = false);

// Rows per weight tile of a matrix with k columns (0: unsupported k).
int tile_rows_for(int64_t k, bool pairs);

// glibc-evaluated RoPE table for positions [0, max_ctx): cos/sin of
// rope_angles (src/math.rs:181-193).
void rope_table(float base, int64_t dim, int64_t max_ctx, std::vector<float>& cos_out,
                std::vector<float>& sin_out);

}  // namespace tir
