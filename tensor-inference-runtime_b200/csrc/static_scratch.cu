// static_scratch.cu -- tir_swiglu_static: the SwiGLU FFN block with its
// intermediate vectors in a fixed, file-scope device array instead of memory
// allocated per call.  For callers that must not allocate device memory while
// they run (a serving loop that reserved all of its memory up front, or code
// running next to a memory-capped pool): this entry makes no cudaMalloc,
// cudaMallocAsync, cudaFree or allocating library call.
//
// The scratch holds gate, up and silu(gate)*up for f <= kSwigluStaticMaxF
// (3 x 6144 floats = 72 KB) plus the streaming matvec's control words.  Its
// address is looked up with cudaGetSymbolAddress on the first call on each
// device, with that device current; make that first call before any stream
// capture on the device.  There is one scratch per device, so calls on the
// same device must not overlap in time (issue them on one stream or order them
// explicitly); overlapping calls race on the scratch.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "host.h"
#include "runtime.h"

namespace tir {

constexpr int64_t kSwigluStaticMaxF = kMaxK;  // 6144

// gate | up | silu(gate)*up, each kSwigluStaticMaxF floats.  Fully written
// before being read on every call: no initial value needed.
static __device__ __align__(256) float g_swiglu_scratch[3 * kSwigluStaticMaxF];
// [0] phase counter (only ever incremented, any start value works);
// [4..6] error words: must be zero when a matvec starts, so every call
// clears them on its stream before its first launch; [7] the code of a
// failed wait, kept until tir_ops_check collects it; [8] the matvec's exit
// count (zero between launches: the last CTA to leave resets it).
static __device__ __align__(256) uint32_t g_swiglu_ctl[16];

namespace {

struct StaticBufs {
    float* scratch = nullptr;
    uint32_t* ctl = nullptr;
};

constexpr int kMaxDevices = 64;

// Symbol addresses, looked up once per device with that device current.
tir_status static_bufs(int dev, StaticBufs* out) {
    static std::mutex mu;
    static StaticBufs table[kMaxDevices];
    if (dev < 0 || dev >= kMaxDevices) return fail(TIR_ERR_INVALID_ARG, "device index out of range");
    std::lock_guard<std::mutex> lock(mu);
    StaticBufs& b = table[dev];
    if (!b.scratch) {
        void* s = nullptr;
        void* c = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&s, g_swiglu_scratch);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(&c, g_swiglu_ctl);
        if (e != cudaSuccess)
            return fail(TIR_ERR_CUDA, std::string("tir_swiglu_static: cudaGetSymbolAddress: ") + cudaGetErrorName(e));
        b.ctl = static_cast<uint32_t*>(c);
        b.scratch = static_cast<float*>(s);
    }
    *out = b;
    return TIR_OK;
}

// One streaming Q8_0 matvec phase (as q8_matmul_stream) on caller-given
// control words.
tir_status matvec(const float* x, const uint8_t* quants, const uint16_t* scales, float* out, int64_t n, int64_t k,
                  uint32_t* ctl, int sms, void* stream) {
    DecodeParams p{};
    PhaseDesc& d = p.single;
    d.kind = PH_GEMV;
    d.in_kind = IN_RAW;
    d.epi = EPI_STORE;
    d.n = static_cast<int32_t>(n);
    d.k = static_cast<int32_t>(k);
    d.sk = static_cast<int32_t>(scale_stride(k));
    d.rows_per_tile = tile_rows_for(k, false);
    d.n_tiles = static_cast<int32_t>((n + d.rows_per_tile - 1) / d.rows_per_tile);
    d.wq = quants;
    d.ws = scales;
    d.in = x;
    d.out = out;
    p.phases = nullptr;
    p.n_phases = 1;
    p.n_steps = 1;
    p.counters = ctl;
    p.error = ctl + 4;
    p.argmax_part = nullptr;  // EPI_STORE phases never touch it
    p.timeout_ns = timeout_ns();
    p.hold_phase = -1;
    const int grid = d.n_tiles < sms ? d.n_tiles : sms;
    const int rc = decode_launch(p, grid, stream, false);
    if (rc != 0)
        return fail(TIR_ERR_CUDA, std::string("tir_swiglu_static: matvec launch: ") +
                                      cudaGetErrorName(static_cast<cudaError_t>(rc)));
    return TIR_OK;
}

}  // namespace

tir_status static_scratch_take_error(int device, uint32_t* code) {
    *code = 0;
    StaticBufs b;
    const tir_status rc = static_bufs(device, &b);
    if (rc != TIR_OK) return rc;
    cudaError_t e = cudaMemcpy(code, b.ctl + 7, sizeof(uint32_t), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && *code != 0u) e = cudaMemset(b.ctl + 7, 0, sizeof(uint32_t));
    if (e != cudaSuccess)
        return fail(TIR_ERR_CUDA, std::string("tir_swiglu_static: error word readback: ") + cudaGetErrorName(e));
    return TIR_OK;
}

}  // namespace tir

using namespace tir;

extern "C" tir_status tir_swiglu_static(const float* x, const uint8_t* gate_q, const uint16_t* gate_s,
                                        const uint8_t* up_q, const uint16_t* up_s, const uint8_t* down_q,
                                        const uint16_t* down_s, float* out, int64_t k, int64_t f, void* stream) {
    clear_error();
    if (k <= 0 || f <= 0 || k % 32 || f % 32 || k > kMaxK)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE,
                    "tir_swiglu_static needs k, f positive multiples of 32 and k <= " + std::to_string(kMaxK));
    if (f > kSwigluStaticMaxF)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "tir_swiglu_static: f = " + std::to_string(f) +
                                                   " exceeds its static scratch of " +
                                                   std::to_string(kSwigluStaticMaxF) + " floats per vector");
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(TIR_ERR_CUDA, std::string("tir_swiglu_static: cudaGetDevice: ") + cudaGetErrorName(e));
    StaticBufs b;
    tir_status rc = static_bufs(dev, &b);
    if (rc != TIR_OK) return rc;
    const int sms = decode_grid_size(dev);
    if (sms <= 0) return fail(TIR_ERR_CUDA, "tir_swiglu_static: no multiprocessor count for the current device");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    e = cudaMemsetAsync(b.ctl + 4, 0, 3 * sizeof(uint32_t), st);
    if (e != cudaSuccess) return fail(TIR_ERR_CUDA, std::string("tir_swiglu_static: clear error words: ") + cudaGetErrorName(e));
    float* gate = b.scratch;
    float* up = b.scratch + kSwigluStaticMaxF;
    float* hid = b.scratch + 2 * kSwigluStaticMaxF;
    rc = matvec(x, gate_q, gate_s, gate, f, k, b.ctl, sms, stream);
    if (rc == TIR_OK) rc = matvec(x, up_q, up_s, up, f, k, b.ctl, sms, stream);
    if (rc == TIR_OK && launch_silu_mul(gate, up, hid, f, stream) != 0)
        rc = fail(TIR_ERR_CUDA, "tir_swiglu_static: silu launch failed");
    if (rc == TIR_OK) rc = matvec(hid, down_q, down_s, out, k, f, b.ctl, sms, stream);
    return rc;
}
