// api.cpp -- the extern "C" boundary (include/tir.h): GGUF handles, model
// upload to HBM, the KV-cache state, the forward/generate drivers and the
// op-level entry points.  No compute happens on the host except what the
// reference itself does on the host (rope_angles, src/math.rs:181-193, and the
// cos/sin of those angles, evaluated with the same glibc libm).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "host.h"
#include "runtime.h"

#define TIR_VERSION "0.1.0-sm100a"

namespace tir {

static thread_local std::string g_error;

tir_status fail(tir_status st, const std::string& msg) {
    g_error = msg;
    return st;
}

void clear_error() { g_error.clear(); }

static tir_status cuda_fail(cudaError_t e, const char* what) {
    return fail(e == cudaErrorMemoryAllocation ? TIR_ERR_OOM : TIR_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

#define CUDA_TRY(expr, what)                         \
    do {                                             \
        cudaError_t e_ = (expr);                     \
        if (e_ != cudaSuccess) return cuda_fail(e_, what); \
    } while (0)

// Every allocation the library makes (device, stream-ordered and pinned host)
// goes through these: they count the calls (tir_debug_alloc_count) and, when
// armed by tir_debug_fail_alloc_after(n), make the n-th next call fail once
// with cudaErrorMemoryAllocation, so the load / create paths' OOM branches can
// be driven without exhausting a GPU.
static std::atomic<long long> g_alloc_calls{0};
static std::atomic<long long> g_alloc_fail_in{-1};

static bool alloc_injected_failure() {
    g_alloc_calls.fetch_add(1);
    long long n = g_alloc_fail_in.load();
    while (n >= 0) {
        if (g_alloc_fail_in.compare_exchange_weak(n, n - 1)) return n == 0;
    }
    return false;
}

cudaError_t dev_malloc(void** p, size_t bytes) {
    if (alloc_injected_failure()) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMalloc(p, bytes);
}

cudaError_t dev_malloc_async(void** p, size_t bytes, cudaStream_t stream) {
    if (alloc_injected_failure()) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMallocAsync(p, bytes, stream);
}

cudaError_t host_malloc_pinned(void** p, size_t bytes) {
    if (alloc_injected_failure()) {
        *p = nullptr;
        return cudaErrorMemoryAllocation;
    }
    return cudaMallocHost(p, bytes);
}

// Rows per weight tile of a matrix with k columns (gemv_tile_rows, even, so
// fused pairs -- RoPE, gate|up -- never straddle tiles); 0 if k is not a
// positive multiple of 32 or longer than kMaxK.
int tile_rows_for(int64_t k, bool pairs) {
    (void)pairs;
    if (k <= 0 || k % 32 != 0 || k > kMaxK || gemv_wpr(k) > kWarps) return 0;
    return gemv_tile_rows(k);
}

// rope_angles (src/math.rs:181-193) and cosf/sinf of each angle, exactly as
// the reference evaluates them per token (src/math.rs:207-208, glibc libm).
void rope_table(float base, int64_t dim, int64_t max_ctx, std::vector<float>& c, std::vector<float>& s) {
    const int64_t half = dim / 2;
    c.assign(static_cast<size_t>(max_ctx * half), 0.f);
    s.assign(static_cast<size_t>(max_ctx * half), 0.f);
    std::vector<float> freq(static_cast<size_t>(half));
    for (int64_t i = 0; i < half; ++i)
        freq[i] = powf(base, (-2.0f * static_cast<float>(i)) / static_cast<float>(dim));
    for (int64_t pos = 0; pos < max_ctx; ++pos)
        for (int64_t i = 0; i < half; ++i) {
            const float theta = static_cast<float>(pos) * freq[i];
            c[pos * half + i] = cosf(theta);
            s[pos * half + i] = sinf(theta);
        }
}

// Small per-device buffers for the single-phase streaming matvec.
struct DevCtx {
    uint32_t* counters = nullptr;  // [1]
    uint32_t* error = nullptr;     // [4]
    unsigned long long* argmax = nullptr;
};

static DevCtx* dev_ctx(int device) {
    static std::mutex mu;
    static std::vector<DevCtx*> ctxs;
    std::lock_guard<std::mutex> lock(mu);
    if (device >= static_cast<int>(ctxs.size())) ctxs.resize(device + 1, nullptr);
    if (!ctxs[device]) {
        DevCtx* c = new DevCtx;
        if (dev_malloc(reinterpret_cast<void**>(&c->counters), 64) != cudaSuccess ||
            dev_malloc(reinterpret_cast<void**>(&c->error), 64) != cudaSuccess ||
            dev_malloc(reinterpret_cast<void**>(&c->argmax), 8 * 1024) != cudaSuccess) {
            cudaFree(c->counters);  // cudaFree(nullptr) is a no-op
            cudaFree(c->error);
            cudaFree(c->argmax);
            delete c;
            return nullptr;
        }
        cudaMemset(c->counters, 0, 64);
        cudaMemset(c->error, 0, 64);
        ctxs[device] = c;
    }
    return ctxs[device];
}

unsigned long long timeout_ns() {
    const char* e = std::getenv("TIR_TIMEOUT_MS");
    long long ms = e ? std::atoll(e) : 2000;
    if (ms <= 0) ms = 2000;
    return static_cast<unsigned long long>(ms) * 1000000ull;
}

// Words 0..2 of an op's error block make a launch's waits give up at once.
// The tensor-core ops clear them on the launch's stream before every launch;
// a single matvec of the decode kernel leaves them cleared itself (its last
// CTA to exit, counted in word 4), so back-to-back matvecs pay no extra
// stream operation.  Word 3 keeps the code of a failure until tir_ops_check
// collects it.
static cudaError_t clear_launch_error(uint32_t* err, void* stream) {
    return cudaMemsetAsync(err, 0, 3 * sizeof(uint32_t), static_cast<cudaStream_t>(stream));
}

// tir_debug_hold_next_op: microseconds of the held second pass of the next
// streaming matvec (0: none).
static std::atomic<int> g_hold_next_op_us{0};

tir_status q8_matmul_stream(const float* x, const uint8_t* quants, const uint16_t* scales, float* out, int64_t n,
                            int64_t k, void* stream, bool qact) {
    if (n == 0) return TIR_OK;
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    DevCtx* c = dev_ctx(dev);
    if (!c) return fail(TIR_ERR_OOM, "device context allocation failed");
    const int sms = decode_grid_size(dev);
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
    d.tiled = scales == nullptr ? 1 : 0;
    d.qact = qact ? 1 : 0;
    p.qact = d.qact;
    d.wq = quants;
    d.ws = scales;
    d.in = x;
    d.out = out;
    p.phases = nullptr;
    p.n_phases = 1;
    p.n_steps = 1;
    p.counters = c->counters;
    p.error = c->error;
    p.argmax_part = c->argmax;
    p.timeout_ns = timeout_ns();
    p.hold_phase = -1;
    if (const int us = g_hold_next_op_us.exchange(0); us > 0) {
        // a second pass of the same matvec whose start waits for one release
        // more than the grid makes (the counter, otherwise only ever
        // incremented, starts from zero): it gives up after `us` and records it
        p.n_steps = 2;
        p.hold_phase = 0;
        p.timeout_ns = static_cast<unsigned long long>(us) * 1000ull;
        CUDA_TRY(cudaMemsetAsync(c->counters, 0, sizeof(uint32_t), static_cast<cudaStream_t>(stream)),
                 "counter reset");
    }
    const int grid = d.n_tiles < sms ? d.n_tiles : sms;
    const int rc = decode_launch(p, grid, stream, false);  // words 0..2 are clear: the previous matvec cleared them
    if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "q8 matvec launch");
    return TIR_OK;
}

}  // namespace tir

using namespace tir;

// ---------------------------------------------------------------------------
// model / state objects
// ---------------------------------------------------------------------------
tir_model::~tir_model() {
    if (dev) {
        cudaSetDevice(device);
        cudaFree(dev);
    }
}

struct tir_state {
    tir_model* m = nullptr;
    int32_t max_ctx = 0;
    int grid = 0;
    int max_splits = 1;
    cudaStream_t stream = nullptr;
    std::vector<void*> allocs;
    float *x = nullptr, *x0 = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr;
    float *dump = nullptr, *kc = nullptr, *vc = nullptr, *rope_cos = nullptr, *rope_sin = nullptr;
    uint8_t* qdump = nullptr;  // Mode::Quantize inputs of the last forward, [(2 L + 1)][H / 32] blocks
    float* attn_part = nullptr;
    uint32_t *attn_cnt = nullptr, *counters = nullptr, *error = nullptr;
    unsigned long long* argmax_part = nullptr;
    int32_t *prompt = nullptr, *out_ids = nullptr, *tmp_id = nullptr;
    PhaseDesc* d_phases = nullptr;
    int n_phases = 0;
    int32_t mode = 0;  // the model's mode the phase table was built for
    int32_t len = 0;
    bool dump_on = false;
    unsigned long long* trace = nullptr;
    int32_t trace_step = -1;
    int32_t hold_phase = -1;                // tir_debug_hold_phase, next launch only
    unsigned long long hold_timeout_ns = 0;
    int32_t* h_ids = nullptr;  // pinned, max_ctx
    uint32_t* h_err = nullptr; // pinned, 4
    ~tir_state() {
        cudaSetDevice(m ? m->device : 0);
        if (stream) cudaStreamSynchronize(stream);
        for (void* p : allocs) cudaFree(p);
        if (h_ids) cudaFreeHost(h_ids);
        if (h_err) cudaFreeHost(h_err);
        if (stream) cudaStreamDestroy(stream);
    }
};

extern "C" {

const char* tir_last_error(void) { return g_error.c_str(); }
const char* tir_version(void) { return TIR_VERSION; }

// ---------------------------------------------------------------------------
// GGUF
// ---------------------------------------------------------------------------
tir_status tir_gguf_open(const char* path, tir_gguf** out) {
    clear_error();
    if (!path || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    const int fd = open(path, O_RDONLY);
    if (fd < 0) return fail(TIR_ERR_IO, std::string("cannot open ") + path + ": " + std::strerror(errno));
    struct stat st;
    if (fstat(fd, &st) != 0) {
        close(fd);
        return fail(TIR_ERR_IO, std::string("cannot stat ") + path);
    }
    tir_gguf* g = new tir_gguf;
    if (st.st_size > 0) {
        void* base = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
        if (base == MAP_FAILED) {
            close(fd);
            delete g;
            return fail(TIR_ERR_IO, std::string("cannot map ") + path);
        }
        g->map_base = base;
        g->map_len = static_cast<size_t>(st.st_size);
        g->data = static_cast<const uint8_t*>(base);
        g->len = g->map_len;
    }
    close(fd);
    const tir_status rc = gguf_parse_all(g);
    if (rc != TIR_OK) {
        delete g;
        return rc;
    }
    *out = g;
    return TIR_OK;
}

tir_status tir_gguf_open_bytes(const uint8_t* data, size_t len, tir_gguf** out) {
    clear_error();
    if ((!data && len) || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    tir_gguf* g = new tir_gguf;
    g->owned.assign(data, data + len);
    g->data = g->owned.data();
    g->len = len;
    const tir_status rc = gguf_parse_all(g);
    if (rc != TIR_OK) {
        delete g;
        return rc;
    }
    *out = g;
    return TIR_OK;
}

void tir_gguf_close(tir_gguf* g) { delete g; }

tir_status tir_gguf_parse_general(const uint8_t* data, size_t len, size_t offset, uint64_t count, tir_gguf** out,
                                  size_t* end_offset) {
    clear_error();
    if ((!data && len) || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    tir_gguf* g = new tir_gguf;
    g->owned.assign(data, data + len);
    g->data = g->owned.data();
    g->len = len;
    size_t end = 0;
    const tir_status rc = gguf_parse_general(g->data, len, offset, count, g->fields, end);
    if (rc != TIR_OK) {
        delete g;
        return rc;
    }
    if (end_offset) *end_offset = end;
    *out = g;
    return TIR_OK;
}

tir_status tir_gguf_parse_q8(uint64_t count, size_t byte_count, size_t map_len, size_t offset, size_t* out_len) {
    clear_error();
    // src/reader.rs:258-272
    if (count % 32 != 0)
        return fail(TIR_ERR_BAD_QUANT_BLOCK, "q8_0 tensor length " + std::to_string(count) + " is not a multiple of 32");
    const size_t total = static_cast<size_t>(count / 32) * byte_count;
    size_t end;
    if (__builtin_add_overflow(offset, total, &end) || end > map_len)
        return fail(TIR_ERR_UNEXPECTED_EOF, "unexpected end of file reading q8_0 tensor data at offset " + std::to_string(offset));
    if (out_len) *out_len = total;
    return TIR_OK;
}

uint32_t tir_gguf_version(const tir_gguf* g) { return g ? g->version : 0; }
int64_t tir_gguf_n_metadata(const tir_gguf* g) { return g ? static_cast<int64_t>(g->fields.size()) : 0; }

static void fill_field(const std::string* name, const MetaValue& v, tir_metadata_field* out) {
    std::memset(out, 0, sizeof(*out));
    out->name = name ? name->c_str() : nullptr;
    out->vtype = v.vtype;
    out->u = v.u;
    out->i = v.i;
    out->f = v.f;
    out->str = v.str.c_str();
    out->str_len = v.str.size();
    out->array_type = v.array_type;
    out->array_len = v.items.size();
}

tir_status tir_gguf_metadata(const tir_gguf* g, int64_t i, tir_metadata_field* out) {
    if (!g || !out || i < 0 || i >= static_cast<int64_t>(g->fields.size()))
        return fail(TIR_ERR_INVALID_ARG, "metadata index out of range");
    fill_field(&g->fields[i].name, g->fields[i].value, out);
    return TIR_OK;
}

tir_status tir_gguf_metadata_item(const tir_gguf* g, int64_t i, uint64_t j, tir_metadata_field* out) {
    if (!g || !out || i < 0 || i >= static_cast<int64_t>(g->fields.size()) ||
        j >= g->fields[i].value.items.size())
        return fail(TIR_ERR_INVALID_ARG, "metadata item out of range");
    fill_field(nullptr, g->fields[i].value.items[j], out);
    return TIR_OK;
}

int64_t tir_gguf_n_tensors(const tir_gguf* g) { return g ? static_cast<int64_t>(g->tensors.size()) : 0; }

tir_status tir_gguf_tensor_info(const tir_gguf* g, int64_t i, tir_tensor_info* out) {
    if (!g || !out || i < 0 || i >= static_cast<int64_t>(g->tensors.size()))
        return fail(TIR_ERR_INVALID_ARG, "tensor index out of range");
    const TensorInfo& t = g->tensors[i];
    std::memset(out, 0, sizeof(*out));
    out->name = t.name.c_str();
    out->n_dims = t.n_dims;
    for (size_t d = 0; d < t.shape.size() && d < 8; ++d) out->shape[d] = t.shape[d];
    out->dtype = t.dtype;
    out->offset = t.offset;
    out->data_bytes = t.data_bytes;
    return TIR_OK;
}

tir_status tir_gguf_tensor_data(const tir_gguf* g, const char* name, const uint8_t** data, size_t* len) {
    clear_error();
    if (!g || !name) return fail(TIR_ERR_INVALID_ARG, "null argument");
    const TensorInfo* t = gguf_find(g, name);
    if (!t) return fail(TIR_ERR_TENSOR_LOAD, std::string("unable to load tensor: ") + name);  // src/forward.rs:284
    if (data) *data = t->data;
    if (len) *len = t->data_bytes;
    return TIR_OK;
}

tir_status tir_gguf_transformer(const tir_gguf* g, tir_transformer* out) {
    if (!g || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (!g->has_transformer) return fail(TIR_ERR_MISSING_FIELD, "Metadata Load error: missing required field: Layers");
    *out = g->transformer;
    return TIR_OK;
}

// ---------------------------------------------------------------------------
// model
// ---------------------------------------------------------------------------
static tir_status need_tensor(const tir_gguf* g, const std::string& name, uint32_t dtype,
                              std::vector<uint64_t> shape, const TensorInfo** out) {
    const TensorInfo* t = gguf_find(g, name);
    if (!t) return fail(TIR_ERR_TENSOR_LOAD, "unable to load tensor: " + name);
    if (t->dtype != dtype || t->shape != shape) {
        std::string s = "tensor " + name + " has dtype " + std::to_string(t->dtype) + " shape [";
        for (size_t i = 0; i < t->shape.size(); ++i) s += (i ? "," : "") + std::to_string(t->shape[i]);
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, s + "], not the Llama-2 layout this runtime serves");
    }
    *out = t;
    return TIR_OK;
}

static size_t a256(size_t v) { return (v + 255) / 256 * 256; }

tir_status tir_model_load_gguf(const tir_gguf* g, int device, tir_model** out) {
    clear_error();
    if (!g || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = nullptr;
    if (!g->has_transformer) return fail(TIR_ERR_MISSING_FIELD, "Metadata Load error: missing required field: Layers");
    tir_transformer t = g->transformer;
    const uint64_t L = t.layers, H = t.embed_dim, hd = t.dim, nq = t.q_heads, nkv = t.k_v_heads;
    // Fused pairs (RoPE, gate|up) need tiles of an even number of rows of H
    // columns that fit one ring slot.  A step has 5 phases per layer + 1.
    if (hd != static_cast<uint64_t>(kHeadDim) || nq == 0 || nkv == 0 || nq % nkv != 0 || H != nq * hd ||
        H % 32 != 0 || H > static_cast<uint64_t>(kMaxK) || tile_rows_for(static_cast<int64_t>(H), true) == 0 ||
        5 * t.layers + 1 > kMaxPhases)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE,
                    "unsupported shape: head dim " + std::to_string(hd) + ", embedding " + std::to_string(H) +
                        ", heads " + std::to_string(nq) + "/" + std::to_string(nkv) + " (head dim must be 64)");
    const uint64_t KVD = nkv * hd;
    const TensorInfo *te, *to, *ton;
    tir_status rc;
    if ((rc = need_tensor(g, "token_embd.weight", TIR_DTYPE_Q8_0, {H, t.vocab}, &te)) != TIR_OK) {
        // vocab comes from output.weight; report whichever is missing.
        if (!gguf_find(g, "output.weight")) return fail(TIR_ERR_TENSOR_LOAD, "unable to load tensor: output.weight");
        return rc;
    }
    if ((rc = need_tensor(g, "output.weight", TIR_DTYPE_Q8_0, {H, t.vocab}, &to)) != TIR_OK) return rc;
    if ((rc = need_tensor(g, "output_norm.weight", TIR_DTYPE_F32, {H}, &ton)) != TIR_OK) return rc;
    const uint64_t F = t.ffn_dim, V = t.vocab;
    if (F == 0 || F % 32 != 0 || F > static_cast<uint64_t>(kMaxK) || V == 0 || V > (1u << 30))
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "unsupported ffn/vocab size");
    struct LT {
        const TensorInfo *an, *q, *k, *v, *o, *fn, *gt, *up, *dn;
    };
    std::vector<LT> lt(L);
    for (uint64_t l = 0; l < L; ++l) {
        const std::string p = "blk." + std::to_string(l) + ".";
        LT& x = lt[l];
        if ((rc = need_tensor(g, p + "attn_norm.weight", TIR_DTYPE_F32, {H}, &x.an)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "attn_q.weight", TIR_DTYPE_Q8_0, {H, H}, &x.q)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "attn_k.weight", TIR_DTYPE_Q8_0, {H, KVD}, &x.k)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "attn_v.weight", TIR_DTYPE_Q8_0, {H, KVD}, &x.v)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "attn_output.weight", TIR_DTYPE_Q8_0, {H, H}, &x.o)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "ffn_norm.weight", TIR_DTYPE_F32, {H}, &x.fn)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "ffn_gate.weight", TIR_DTYPE_Q8_0, {H, F}, &x.gt)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "ffn_up.weight", TIR_DTYPE_Q8_0, {H, F}, &x.up)) != TIR_OK) return rc;
        if ((rc = need_tensor(g, p + "ffn_down.weight", TIR_DTYPE_Q8_0, {F, H}, &x.dn)) != TIR_OK) return rc;
    }

    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) return fail(TIR_ERR_NO_DEVICE, "no CUDA device");
    if (device < 0 || device >= ndev) return fail(TIR_ERR_INVALID_ARG, "device index out of range");
    CUDA_TRY(cudaSetDevice(device), "cudaSetDevice");

    tir_model* m = new tir_model;
    m->device = device;
    m->t = t;
    // Layout: one allocation; each matrix = quants then scales, 256-B aligned.
    size_t off = 0;
    auto plan = [&](Mat& mt, int64_t n, int64_t k) {  // split layout
        mt.n = n;
        mt.k = k;
        mt.sk = scale_stride(k);
        mt.q = reinterpret_cast<uint8_t*>(off);
        off = a256(off + static_cast<size_t>(n * k));
        mt.s = reinterpret_cast<uint16_t*>(off);
        off = a256(off + static_cast<size_t>(n * mt.sk * 2));
    };
    auto plan_tiled = [&](Mat& mt, int64_t n, int64_t k, bool pairs) {
        mt.n = n;
        mt.k = k;
        mt.sk = scale_stride(k);
        mt.r = tile_rows_for(k, pairs);
        mt.tiled = true;
        mt.q = reinterpret_cast<uint8_t*>(off);
        off = a256(off + static_cast<size_t>(q8_tiled_matrix_bytes(n, k)));
    };
    auto plan_f32 = [&](int64_t n) {
        const size_t at = off;
        off = a256(off + static_cast<size_t>(n) * 4);
        return at;
    };
    m->qkv.resize(L);
    m->o.resize(L);
    m->gu.resize(L);
    m->down.resize(L);
    std::vector<size_t> an_off(L), fn_off(L);
    for (uint64_t l = 0; l < L; ++l) {
        plan_tiled(m->qkv[l], static_cast<int64_t>(H + 2 * KVD), static_cast<int64_t>(H), true);
        plan_tiled(m->o[l], static_cast<int64_t>(H), static_cast<int64_t>(H), false);
        plan_tiled(m->gu[l], static_cast<int64_t>(2 * F), static_cast<int64_t>(H), true);
        plan_tiled(m->down[l], static_cast<int64_t>(H), static_cast<int64_t>(F), false);
        an_off[l] = plan_f32(static_cast<int64_t>(H));
        fn_off[l] = plan_f32(static_cast<int64_t>(H));
    }
    plan_tiled(m->lm, static_cast<int64_t>(V), static_cast<int64_t>(H), false);
    plan(m->embd, static_cast<int64_t>(V), static_cast<int64_t>(H));
    const size_t on_off = plan_f32(static_cast<int64_t>(H));
    m->dev_bytes = off;
    cudaError_t e = dev_malloc(&m->dev, off);
    if (e != cudaSuccess) {
        delete m;
        return cuda_fail(e, "weight allocation");
    }
    auto fix = [&](Mat& mt) {
        mt.q = m->dev + reinterpret_cast<size_t>(mt.q);
        mt.s = mt.tiled ? nullptr : reinterpret_cast<uint16_t*>(m->dev + reinterpret_cast<size_t>(mt.s));
    };
    for (uint64_t l = 0; l < L; ++l) {
        fix(m->qkv[l]);
        fix(m->o[l]);
        fix(m->gu[l]);
        fix(m->down[l]);
        m->attn_norm.push_back(reinterpret_cast<float*>(m->dev + an_off[l]));
        m->ffn_norm.push_back(reinterpret_cast<float*>(m->dev + fn_off[l]));
    }
    fix(m->lm);
    fix(m->embd);
    m->out_norm = reinterpret_cast<float*>(m->dev + on_off);

    // Upload: raw Q8_0 bytes to a staging buffer, repacked on the device.
    size_t staging_bytes = te->data_bytes > to->data_bytes ? te->data_bytes : to->data_bytes;
    for (const LT& x : lt)
        for (const TensorInfo* ti : {x.q, x.k, x.v, x.o, x.gt, x.up, x.dn})
            if (ti->data_bytes > staging_bytes) staging_bytes = ti->data_bytes;
    uint8_t* staging = nullptr;
    e = dev_malloc(&staging, staging_bytes);
    if (e != cudaSuccess) {
        delete m;
        return cuda_fail(e, "staging allocation");
    }
    auto fail_upload = [&](cudaError_t er, const char* what) {
        cudaFree(staging);
        delete m;
        return cuda_fail(er, what);
    };
    if ((e = cudaMemset(m->dev, 0, off)) != cudaSuccess) return fail_upload(e, "memset");
    auto put_mat = [&](const TensorInfo* ti, const Mat& mt, int64_t row0, int64_t step, int64_t roff) -> cudaError_t {
        const int64_t k = static_cast<int64_t>(ti->shape[0]);
        const int64_t rows = static_cast<int64_t>(ti->shape[1]);
        cudaError_t er = cudaMemcpy(staging, ti->data, ti->data_bytes, cudaMemcpyHostToDevice);
        if (er != cudaSuccess) return er;
        const int rc2 = mt.tiled ? launch_repack_tiled(staging, rows, k, mt.q, mt.n, mt.r, step, row0 + roff, nullptr)
                                 : launch_repack(staging, rows, k, mt.q + row0 * mt.k, mt.s + row0 * mt.sk, mt.sk,
                                                 step, roff, nullptr);
        if (rc2 != 0) return static_cast<cudaError_t>(rc2);
        return cudaDeviceSynchronize();
    };
    auto put_f32 = [&](const TensorInfo* ti, float* dst) {
        return cudaMemcpy(dst, ti->data, ti->data_bytes, cudaMemcpyHostToDevice);
    };
    for (uint64_t l = 0; l < L; ++l) {
        const LT& x = lt[l];
        if ((e = put_mat(x.q, m->qkv[l], 0, 1, 0)) != cudaSuccess) return fail_upload(e, "upload attn_q");
        if ((e = put_mat(x.k, m->qkv[l], static_cast<int64_t>(H), 1, 0)) != cudaSuccess) return fail_upload(e, "upload attn_k");
        if ((e = put_mat(x.v, m->qkv[l], static_cast<int64_t>(H + KVD), 1, 0)) != cudaSuccess) return fail_upload(e, "upload attn_v");
        if ((e = put_mat(x.o, m->o[l], 0, 1, 0)) != cudaSuccess) return fail_upload(e, "upload attn_output");
        if ((e = put_mat(x.gt, m->gu[l], 0, 2, 0)) != cudaSuccess) return fail_upload(e, "upload ffn_gate");
        if ((e = put_mat(x.up, m->gu[l], 0, 2, 1)) != cudaSuccess) return fail_upload(e, "upload ffn_up");
        if ((e = put_mat(x.dn, m->down[l], 0, 1, 0)) != cudaSuccess) return fail_upload(e, "upload ffn_down");
        if ((e = put_f32(x.an, m->attn_norm[l])) != cudaSuccess) return fail_upload(e, "upload attn_norm");
        if ((e = put_f32(x.fn, m->ffn_norm[l])) != cudaSuccess) return fail_upload(e, "upload ffn_norm");
    }
    if ((e = put_mat(to, m->lm, 0, 1, 0)) != cudaSuccess) return fail_upload(e, "upload output");
    if ((e = put_mat(te, m->embd, 0, 1, 0)) != cudaSuccess) return fail_upload(e, "upload token_embd");
    if ((e = put_f32(ton, m->out_norm)) != cudaSuccess) return fail_upload(e, "upload output_norm");
    cudaFree(staging);
    uint64_t wb = 0;
    auto mb = [](const Mat& mt) { return static_cast<uint64_t>(mt.n * mt.k + mt.n * (mt.k / 32) * 2); };
    for (uint64_t l = 0; l < L; ++l) wb += mb(m->qkv[l]) + mb(m->o[l]) + mb(m->gu[l]) + mb(m->down[l]) + 8 * H;
    wb += mb(m->lm) + 4 * H;
    m->weight_bytes = wb;
    *out = m;
    return TIR_OK;
}

tir_status tir_model_load(const char* path, int device, tir_model** out) {
    tir_gguf* g = nullptr;
    tir_status rc = tir_gguf_open(path, &g);
    if (rc != TIR_OK) return rc;
    rc = tir_model_load_gguf(g, device, out);
    tir_gguf_close(g);
    return rc;
}

tir_status tir_model_info(const tir_model* m, tir_transformer* out) {
    if (!m || !out) return fail(TIR_ERR_INVALID_ARG, "null argument");
    *out = m->t;
    return TIR_OK;
}

tir_status tir_model_set_mode(tir_model* m, int32_t mode) {
    if (!m) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (mode != 0 && mode != 1) return fail(TIR_ERR_INVALID_ARG, "mode must be 0 (Normal) or 1 (Quantize)");
    m->t.mode = mode;
    return TIR_OK;
}

uint64_t tir_model_weight_bytes(const tir_model* m) { return m ? m->weight_bytes : 0; }

void tir_model_destroy(tir_model* m) { delete m; }

// ---------------------------------------------------------------------------
// state
// ---------------------------------------------------------------------------
static tir_status build_phases(tir_state* s) {
    tir_model* m = s->m;
    const tir_transformer& t = m->t;
    const int64_t L = t.layers, H = t.embed_dim, KVD = t.kv_dim;
    const size_t layer_cache = static_cast<size_t>(t.k_v_heads) * s->max_ctx * kHeadDim;
    std::vector<PhaseDesc> ph;
    auto gemv = [&](const Mat& mt, int layer, int32_t in_kind, const float* in, const float* norm_w, int32_t epi,
                    float* out) {
        PhaseDesc d{};
        d.kind = PH_GEMV;
        d.layer = layer;
        d.in_kind = in_kind;
        d.epi = epi;
        d.n = static_cast<int32_t>(mt.n);
        d.k = static_cast<int32_t>(mt.k);
        d.sk = static_cast<int32_t>(mt.sk);
        d.rows_per_tile = static_cast<int32_t>(mt.r);
        d.n_tiles = static_cast<int32_t>((mt.n + d.rows_per_tile - 1) / d.rows_per_tile);
        d.tiled = 1;
        d.wq = mt.q;
        d.ws = nullptr;
        d.in = in;
        d.norm_w = norm_w;
        d.out = out;
        return d;
    };
    // Mode::Quantize (src/forward.rs:261-275) quantises the input of the
    // q, k, v, o and lm_head matmuls; the FFN always runs q8_matmul.
    const int32_t qact = t.mode == 1 ? 1 : 0;
    for (int64_t l = 0; l < L; ++l) {
        PhaseDesc q = gemv(m->qkv[l], static_cast<int>(l), l == 0 ? IN_X0_NORM : IN_X_NORM, s->x, m->attn_norm[l],
                           EPI_QKV, s->q);
        q.qact = qact;
        q.kc = s->kc + l * layer_cache;
        q.vc = s->vc + l * layer_cache;
        ph.push_back(q);
        PhaseDesc a{};
        a.kind = PH_ATTN;
        a.layer = static_cast<int>(l);
        a.kc = q.kc;
        a.vc = q.vc;
        ph.push_back(a);
        PhaseDesc o = gemv(m->o[l], static_cast<int>(l), IN_ATTN, s->attn, nullptr, EPI_RESID, s->x);
        o.qact = qact;
        ph.push_back(o);
        ph.push_back(gemv(m->gu[l], static_cast<int>(l), IN_X_NORM, s->x, m->ffn_norm[l], EPI_GU, s->h));
        PhaseDesc dn = gemv(m->down[l], static_cast<int>(l), IN_RAW, s->h, nullptr, EPI_RESID, s->x);
        dn.dump = 1;
        ph.push_back(dn);
    }
    PhaseDesc lm = gemv(m->lm, -1, L == 0 ? IN_X0_NORM : IN_X_NORM, s->x, m->out_norm, EPI_LOGITS, s->logits);
    lm.qact = qact;
    ph.push_back(lm);
    (void)H;
    (void)KVD;
    if (s->d_phases) {  // the model's mode changed since: same shapes, new table
        CUDA_TRY(cudaStreamSynchronize(s->stream), "phase table update");
        CUDA_TRY(cudaMemcpy(s->d_phases, ph.data(), ph.size() * sizeof(PhaseDesc), cudaMemcpyHostToDevice),
                 "phase table upload");
        s->mode = t.mode;
        return TIR_OK;
    }
    s->n_phases = static_cast<int>(ph.size());
    s->mode = t.mode;
    void* p = nullptr;
    CUDA_TRY(dev_malloc(&p, ph.size() * sizeof(PhaseDesc)), "phase table");
    s->allocs.push_back(p);
    s->d_phases = static_cast<PhaseDesc*>(p);
    CUDA_TRY(cudaMemcpy(p, ph.data(), ph.size() * sizeof(PhaseDesc), cudaMemcpyHostToDevice), "phase table upload");
    void* c = nullptr;
    CUDA_TRY(dev_malloc(&c, ph.size() * sizeof(uint32_t)), "phase counters");
    s->allocs.push_back(c);
    s->counters = static_cast<uint32_t*>(c);
    return TIR_OK;
}

tir_status tir_state_create(tir_model* m, int32_t max_ctx, tir_state** out) {
    clear_error();
    if (!m || !out || max_ctx <= 0) return fail(TIR_ERR_INVALID_ARG, "invalid argument");
    *out = nullptr;
    CUDA_TRY(cudaSetDevice(m->device), "cudaSetDevice");
    const tir_transformer& t = m->t;
    tir_state* s = new tir_state;
    s->m = m;
    s->max_ctx = max_ctx;
    s->grid = decode_grid_size(m->device);
    int occ = 0;
    cudaError_t e = cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking);
    if (e != cudaSuccess) {
        delete s;
        return cuda_fail(e, "stream");
    }
    const int64_t H = t.embed_dim, V = t.vocab, F = t.ffn_dim, L = t.layers;
    const int64_t group = t.q_heads / t.k_v_heads;
    int64_t ms = static_cast<int64_t>(s->grid) / static_cast<int64_t>(t.k_v_heads);
    const int64_t need = (max_ctx + kAttnChunk - 1) / kAttnChunk;
    if (ms > need) ms = need;
    if (ms < 1) ms = 1;
    s->max_splits = static_cast<int>(ms);
    auto alloc = [&](size_t bytes, void** p) -> bool {
        if (dev_malloc(p, bytes ? bytes : 16) != cudaSuccess) return false;
        s->allocs.push_back(*p);
        return true;
    };
    const size_t cache_f = static_cast<size_t>(L) * t.k_v_heads * max_ctx * kHeadDim;
    bool ok = alloc(H * 4, reinterpret_cast<void**>(&s->x)) && alloc(H * 4, reinterpret_cast<void**>(&s->x0)) &&
              alloc(H * 4, reinterpret_cast<void**>(&s->q)) && alloc(H * 4, reinterpret_cast<void**>(&s->attn)) &&
              alloc(F * 4, reinterpret_cast<void**>(&s->h)) && alloc(V * 4, reinterpret_cast<void**>(&s->logits)) &&
              alloc((L + 1) * H * 4, reinterpret_cast<void**>(&s->dump)) &&
              alloc((2 * L + 1) * (H / 32) * 34, reinterpret_cast<void**>(&s->qdump)) &&
              alloc(cache_f * 4, reinterpret_cast<void**>(&s->kc)) && alloc(cache_f * 4, reinterpret_cast<void**>(&s->vc)) &&
              alloc(static_cast<size_t>(max_ctx) * 32 * 4, reinterpret_cast<void**>(&s->rope_cos)) &&
              alloc(static_cast<size_t>(max_ctx) * 32 * 4, reinterpret_cast<void**>(&s->rope_sin)) &&
              alloc(static_cast<size_t>(t.k_v_heads) * ms * group * kAttnRec * 4,
                    reinterpret_cast<void**>(&s->attn_part)) &&
              alloc(static_cast<size_t>(L) * t.k_v_heads * 4, reinterpret_cast<void**>(&s->attn_cnt)) &&
              alloc(16, reinterpret_cast<void**>(&s->error)) &&
              alloc(static_cast<size_t>(s->grid) * 8, reinterpret_cast<void**>(&s->argmax_part)) &&
              alloc(static_cast<size_t>(max_ctx) * 4, reinterpret_cast<void**>(&s->prompt)) &&
              alloc(static_cast<size_t>(max_ctx) * 4, reinterpret_cast<void**>(&s->out_ids)) &&
              alloc(16, reinterpret_cast<void**>(&s->tmp_id));
    if (!ok) {
        delete s;
        return fail(TIR_ERR_OOM, "state allocation failed (KV cache of " + std::to_string(max_ctx) + " positions)");
    }
    if (host_malloc_pinned(&s->h_ids, static_cast<size_t>(max_ctx) * 4) != cudaSuccess ||
        host_malloc_pinned(&s->h_err, 16) != cudaSuccess) {
        delete s;
        return fail(TIR_ERR_OOM, "pinned host allocation failed");
    }
    std::vector<float> c, sn;
    rope_table(t.base_freq, static_cast<int64_t>(t.dim), max_ctx, c, sn);
    if (cudaMemcpy(s->rope_cos, c.data(), c.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(s->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(s->attn_cnt, 0, static_cast<size_t>(L) * t.k_v_heads * 4) != cudaSuccess ||
        cudaMemset(s->argmax_part, 0, static_cast<size_t>(s->grid) * 8) != cudaSuccess) {
        delete s;
        return fail(TIR_ERR_CUDA, "state initialisation failed");
    }
    tir_status rc = build_phases(s);
    if (rc != TIR_OK) {
        delete s;
        return rc;
    }
    // The persistent kernel needs one CTA per SM resident at once.
    occ = decode_blocks_per_sm();
    if (occ < 1) {
        delete s;
        return fail(TIR_ERR_CUDA, "the decode kernel cannot be resident on this device (" +
                                      std::to_string(decode_smem_bytes()) + " B shared memory per CTA)");
    }
    *out = s;
    return TIR_OK;
}

tir_status tir_state_reset(tir_state* s) {
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    s->len = 0;
    return TIR_OK;
}

int32_t tir_state_len(const tir_state* s) { return s ? s->len : 0; }
void* tir_state_stream(tir_state* s) { return s ? static_cast<void*>(s->stream) : nullptr; }
void tir_state_destroy(tir_state* s) { delete s; }

static tir_status launch_steps(tir_state* s, int n_steps, int pos0, const float* x0, const int32_t* prompt,
                               int n_prompt, int32_t* out_ids) {
    const tir_transformer& t = s->m->t;
    if (s->mode != t.mode) {  // tir_model_set_mode since the table was built
        const tir_status rc = build_phases(s);
        if (rc != TIR_OK) return rc;
    }
    DecodeParams p{};
    p.phases = s->d_phases;
    p.n_phases = s->n_phases;
    p.n_steps = n_steps;
    p.pos0 = pos0;
    p.H = static_cast<int32_t>(t.embed_dim);
    p.q_heads = static_cast<int32_t>(t.q_heads);
    p.kv_heads = static_cast<int32_t>(t.k_v_heads);
    p.group = static_cast<int32_t>(t.q_heads / t.k_v_heads);
    p.kvd = static_cast<int32_t>(t.kv_dim);
    p.max_ctx = s->max_ctx;
    p.vocab = static_cast<int32_t>(t.vocab);
    p.max_splits = s->max_splits;
    p.qact = t.mode == 1 ? 1 : 0;
    p.x0 = x0;
    p.prompt = prompt;
    p.n_prompt = n_prompt;
    p.out_ids = out_ids;
    p.embd_q = s->m->embd.q;
    p.embd_s = s->m->embd.s;
    p.embd_sk = static_cast<int32_t>(s->m->embd.sk);
    p.rms_eps = 1e-5f;  // src/math.rs:144, whatever the file says
    p.x = s->x;
    p.dump = s->dump_on ? s->dump : nullptr;
    p.qdump = s->dump_on && t.mode == 1 ? s->qdump : nullptr;
    p.n_layers = static_cast<int32_t>(t.layers);
    p.rope_cos = s->rope_cos;
    p.rope_sin = s->rope_sin;
    p.attn_part = s->attn_part;
    p.attn_cnt = s->attn_cnt;
    p.attn_out = s->attn;
    p.q = s->q;
    p.counters = s->counters;
    p.argmax_part = s->argmax_part;
    p.error = s->error;
    p.timeout_ns = s->hold_phase >= 0 ? s->hold_timeout_ns : timeout_ns();
    p.hold_phase = s->hold_phase;
    s->hold_phase = -1;
    p.trace = s->trace_step >= 0 ? s->trace : nullptr;
    p.trace_step = s->trace_step;
    CUDA_TRY(cudaMemsetAsync(s->counters, 0, static_cast<size_t>(s->n_phases) * 4, s->stream), "counter reset");
    CUDA_TRY(cudaMemsetAsync(s->error, 0, 16, s->stream), "error reset");
    CUDA_TRY(cudaMemsetAsync(s->attn_cnt, 0, static_cast<size_t>(t.layers) * t.k_v_heads * 4, s->stream),
             "attention counter reset");
    const int rc = decode_launch(p, s->grid, s->stream, true);
    if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "decode launch");
    return TIR_OK;
}

static tir_status finish(tir_state* s) {
    CUDA_TRY(cudaMemcpyAsync(s->h_err, s->error, 12, cudaMemcpyDeviceToHost, s->stream), "error readback");
    CUDA_TRY(cudaStreamSynchronize(s->stream), "decode");
    if (s->h_err[0] == TIR_ERR_BAD_TOKEN) {
        s->len = 0;
        return fail(TIR_ERR_BAD_TOKEN, "a token id read on the device (step " +
                                           std::to_string(static_cast<int>(s->h_err[2])) +
                                           ") is not in the vocab; the cache was reset");
    }
    if (s->h_err[0] != 0) {
        s->len = 0;
        return fail(TIR_ERR_TIMEOUT, "device wait timed out (phase " + std::to_string(static_cast<int>(s->h_err[1])) +
                                         ", step " + std::to_string(static_cast<int>(s->h_err[2])) +
                                         "); the cache was reset");
    }
    return TIR_OK;
}

tir_status tir_forward_embedded(tir_state* s, const float* x_host, int32_t pos, float* logits_host) {
    clear_error();
    if (!s || !x_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (pos != s->len) return fail(TIR_ERR_INVALID_ARG, "pos " + std::to_string(pos) + " does not match the cache length " + std::to_string(s->len));
    if (pos >= s->max_ctx) return fail(TIR_ERR_CTX_OVERFLOW, "pos " + std::to_string(pos) + " >= max_ctx " + std::to_string(s->max_ctx));
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    const size_t H = s->m->t.embed_dim;
    CUDA_TRY(cudaMemcpyAsync(s->x0, x_host, H * 4, cudaMemcpyHostToDevice, s->stream), "input upload");
    tir_status rc = launch_steps(s, 1, pos, s->x0, nullptr, 1, nullptr);
    if (rc != TIR_OK) return rc;
    if (logits_host)
        CUDA_TRY(cudaMemcpyAsync(logits_host, s->logits, s->m->t.vocab * 4, cudaMemcpyDeviceToHost, s->stream),
                 "logits readback");
    rc = finish(s);
    if (rc == TIR_OK) s->len = pos + 1;
    return rc;
}

tir_status tir_forward(tir_state* s, int32_t token_id, int32_t pos, float* logits_host) {
    clear_error();
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (token_id < 0 || static_cast<uint64_t>(token_id) >= s->m->t.vocab)
        return fail(TIR_ERR_BAD_TOKEN, "token id " + std::to_string(token_id) + " is not in the vocab");
    if (pos != s->len) return fail(TIR_ERR_INVALID_ARG, "pos " + std::to_string(pos) + " does not match the cache length " + std::to_string(s->len));
    if (pos >= s->max_ctx) return fail(TIR_ERR_CTX_OVERFLOW, "pos " + std::to_string(pos) + " >= max_ctx " + std::to_string(s->max_ctx));
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    s->h_ids[0] = token_id;
    CUDA_TRY(cudaMemcpyAsync(s->prompt, s->h_ids, 4, cudaMemcpyHostToDevice, s->stream), "token upload");
    tir_status rc = launch_steps(s, 1, pos, nullptr, s->prompt, 1, nullptr);
    if (rc != TIR_OK) return rc;
    if (logits_host)
        CUDA_TRY(cudaMemcpyAsync(logits_host, s->logits, s->m->t.vocab * 4, cudaMemcpyDeviceToHost, s->stream),
                 "logits readback");
    rc = finish(s);
    if (rc == TIR_OK) s->len = pos + 1;
    return rc;
}

static tir_status check_generate(tir_state* s, int32_t n_prompt, int32_t cap) {
    if (n_prompt < 0 || cap < 0) return fail(TIR_ERR_INVALID_ARG, "negative length");
    if (static_cast<int64_t>(n_prompt) + cap > s->max_ctx)
        return fail(TIR_ERR_CTX_OVERFLOW, "prompt + cap = " + std::to_string(static_cast<int64_t>(n_prompt) + cap) +
                                              " positions > max_ctx " + std::to_string(s->max_ctx));
    return TIR_OK;
}

tir_status tir_generate_capped_device(tir_state* s, const int32_t* prompt_dev, int32_t n_prompt, int32_t cap,
                                      int32_t* out_ids_dev) {
    clear_error();
    if (!s || (n_prompt > 0 && !prompt_dev) || (cap > 0 && !out_ids_dev)) return fail(TIR_ERR_INVALID_ARG, "null argument");
    tir_status rc = check_generate(s, n_prompt, cap);
    if (rc != TIR_OK) return rc;
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    s->len = 0;
    const int n_steps = n_prompt + cap;
    if (n_steps == 0) return TIR_OK;
    rc = launch_steps(s, n_steps, 0, nullptr, prompt_dev, n_prompt, out_ids_dev);
    if (rc == TIR_OK) s->len = n_steps;
    return rc;
}

tir_status tir_generate_capped(tir_state* s, const int32_t* prompt_host, int32_t n_prompt, int32_t cap,
                               int32_t* out_ids_host, float* last_logits_host) {
    clear_error();
    if (!s || (n_prompt > 0 && !prompt_host) || (cap > 0 && !out_ids_host)) return fail(TIR_ERR_INVALID_ARG, "null argument");
    tir_status rc = check_generate(s, n_prompt, cap);
    if (rc != TIR_OK) return rc;
    for (int32_t i = 0; i < n_prompt; ++i)
        if (prompt_host[i] < 0 || static_cast<uint64_t>(prompt_host[i]) >= s->m->t.vocab)
            return fail(TIR_ERR_BAD_TOKEN, "token id " + std::to_string(prompt_host[i]) + " is not in the vocab");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    s->len = 0;
    const int n_steps = n_prompt + cap;
    if (n_steps == 0) return TIR_OK;
    std::memcpy(s->h_ids, prompt_host, static_cast<size_t>(n_prompt) * 4);
    if (n_prompt > 0)
        CUDA_TRY(cudaMemcpyAsync(s->prompt, s->h_ids, static_cast<size_t>(n_prompt) * 4, cudaMemcpyHostToDevice, s->stream),
                 "prompt upload");
    rc = launch_steps(s, n_steps, 0, nullptr, s->prompt, n_prompt, s->out_ids);
    if (rc != TIR_OK) return rc;
    if (cap > 0)
        CUDA_TRY(cudaMemcpyAsync(s->h_ids, s->out_ids, static_cast<size_t>(cap) * 4, cudaMemcpyDeviceToHost, s->stream),
                 "ids readback");
    if (last_logits_host)
        CUDA_TRY(cudaMemcpyAsync(last_logits_host, s->logits, s->m->t.vocab * 4, cudaMemcpyDeviceToHost, s->stream),
                 "logits readback");
    rc = finish(s);
    if (rc != TIR_OK) return rc;
    if (cap > 0) std::memcpy(out_ids_host, s->h_ids, static_cast<size_t>(cap) * 4);
    s->len = n_steps;
    return TIR_OK;
}

// The prompt phase of generate_capped (src/lib.rs:239-314, token by token
// from position 0) without greedy steps: the state then holds the prompt's
// KV cache and last_logits_host (optional) the last position's logits.  A
// tir_state holds one sequence; n_seqs sequences prefill through
// tir_batch_step (tokens_per_seq = seq_len).
tir_status tir_prefill(tir_state* s, const int32_t* ids_host, int32_t n_seqs, int32_t seq_len, float* last_logits_host) {
    clear_error();
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (n_seqs != 1)
        return fail(TIR_ERR_INVALID_ARG, "a tir_state holds one sequence: prefill n_seqs sequences with tir_batch_step");
    if (seq_len <= 0) return fail(TIR_ERR_INVALID_ARG, "seq_len must be positive");
    return tir_generate_capped(s, ids_host, seq_len, 0, nullptr, last_logits_host);
}

// generate_capped on text (src/lib.rs:239-314): encode (BOS + BPE ids), the
// prompt fed token by token, then cap greedy ids.
tir_status tir_generate_capped_text(tir_state* s, const tir_tokenizer* tk, const char* text, int64_t text_len,
                                    int32_t cap, int32_t* out_ids_host) {
    clear_error();
    if (!s || !tk) return fail(TIR_ERR_INVALID_ARG, "null argument");
    int64_t n = 0;
    tir_status rc = tir_encode(tk, text, text_len, nullptr, 0, &n);
    if (rc != TIR_OK) return rc;
    std::vector<int32_t> ids(static_cast<size_t>(n));
    rc = tir_encode(tk, text, text_len, ids.data(), n, &n);
    if (rc != TIR_OK) return rc;
    return tir_generate_capped(s, ids.data(), static_cast<int32_t>(n), cap, out_ids_host, nullptr);
}

// generate (src/lib.rs:140-236): encode, the prompt token by token, then
// greedy ids until id 13 (newline) or 2 (EOS), which is not kept; the ids
// before it decoded to text.  The reference loops without bound; here at
// most max_new ids are generated (one device launch of max_new steps, cut at
// the first stop id).  *n_ids gets the number of ids kept.
tir_status tir_generate_text(tir_state* s, const tir_tokenizer* tk, const char* text, int64_t text_len,
                             int32_t max_new, char* out_text, int64_t cap, int64_t* out_len, int32_t* n_ids) {
    clear_error();
    if (!s || !tk || max_new < 0) return fail(TIR_ERR_INVALID_ARG, "null argument or negative max_new");
    int64_t n = 0;
    tir_status rc = tir_encode(tk, text, text_len, nullptr, 0, &n);
    if (rc != TIR_OK) return rc;
    std::vector<int32_t> prompt(static_cast<size_t>(n));
    rc = tir_encode(tk, text, text_len, prompt.data(), n, &n);
    if (rc != TIR_OK) return rc;
    std::vector<int32_t> gen(static_cast<size_t>(std::max(max_new, 1)));
    rc = tir_generate_capped(s, prompt.data(), static_cast<int32_t>(n), max_new, gen.data(), nullptr);
    if (rc != TIR_OK) return rc;
    int32_t kept = 0;
    while (kept < max_new && gen[static_cast<size_t>(kept)] != 13 && gen[static_cast<size_t>(kept)] != 2) ++kept;
    if (n_ids) *n_ids = kept;
    return tir_decode(tk, gen.data(), kept, out_text, cap, out_len);
}

tir_status tir_state_sync(tir_state* s) {
    clear_error();
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    return finish(s);
}

tir_status tir_test_forward(tir_state* s, int32_t* out_id) {
    clear_error();
    if (!s || !out_id) return fail(TIR_ERR_INVALID_ARG, "null argument");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    s->len = 0;
    const int64_t H = s->m->t.embed_dim;
    if (launch_fill_f32(s->x0, 1.0f, H, s->stream) != 0) return fail(TIR_ERR_CUDA, "fill launch");
    tir_status rc = launch_steps(s, 1, 0, s->x0, nullptr, 1, nullptr);
    if (rc != TIR_OK) return rc;
    if (launch_argmax(s->logits, static_cast<int64_t>(s->m->t.vocab), s->tmp_id, s->stream) != 0)
        return fail(TIR_ERR_CUDA, "argmax launch");
    CUDA_TRY(cudaMemcpyAsync(s->h_ids, s->tmp_id, 4, cudaMemcpyDeviceToHost, s->stream), "id readback");
    rc = finish(s);
    if (rc != TIR_OK) return rc;
    *out_id = s->h_ids[0];
    s->len = 1;
    return TIR_OK;
}

tir_status tir_state_enable_dump(tir_state* s, int32_t enable) {
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    s->dump_on = enable != 0;
    return TIR_OK;
}

tir_status tir_state_dump(tir_state* s, float* out_host) {
    clear_error();
    if (!s || !out_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (!s->dump_on) return fail(TIR_ERR_INVALID_ARG, "dump not enabled");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    const size_t n = static_cast<size_t>(s->m->t.layers + 1) * s->m->t.embed_dim;
    CUDA_TRY(cudaMemcpyAsync(out_host, s->dump, n * 4, cudaMemcpyDeviceToHost, s->stream), "dump readback");
    CUDA_TRY(cudaStreamSynchronize(s->stream), "dump readback");
    return TIR_OK;
}

// The per-layer outputs [L][H] of the last forward (rows 1..L of the dump),
// for layer-by-layer comparison with the reference's forward
// (src/forward.rs:13-258); the dump must be on (tir_state_enable_dump).
tir_status tir_debug_dump_layers(tir_state* s, float* out_host) {
    clear_error();
    if (!s || !out_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (!s->dump_on) return fail(TIR_ERR_INVALID_ARG, "dump not enabled");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    const size_t h = s->m->t.embed_dim;
    CUDA_TRY(cudaMemcpyAsync(out_host, s->dump + h, static_cast<size_t>(s->m->t.layers) * h * 4, cudaMemcpyDeviceToHost,
                             s->stream),
             "dump readback");
    CUDA_TRY(cudaStreamSynchronize(s->stream), "dump readback");
    return TIR_OK;
}

// The Q8_0 blocks Mode::Quantize made of the q|k|v, o and lm_head inputs in
// the last forward (activated_q8, src/kernels.rs:8-31): [2 l] q|k|v of layer
// l, [2 l + 1] o of layer l, [2 L] lm_head; needs the dump on and Mode 1.
tir_status tir_debug_dump_qact(tir_state* s, uint8_t* out_host) {
    clear_error();
    if (!s || !out_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (!s->dump_on || s->m->t.mode != 1) return fail(TIR_ERR_INVALID_ARG, "needs the dump on and Mode::Quantize");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    const size_t n = static_cast<size_t>(2 * s->m->t.layers + 1) * (s->m->t.embed_dim / 32) * 34;
    CUDA_TRY(cudaMemcpyAsync(out_host, s->qdump, n, cudaMemcpyDeviceToHost, s->stream), "qact dump readback");
    CUDA_TRY(cudaStreamSynchronize(s->stream), "qact dump readback");
    return TIR_OK;
}

tir_status tir_state_enable_trace(tir_state* s, int32_t step) {
    clear_error();
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    if (step >= 0 && !s->trace) {
        void* p = nullptr;
        const size_t bytes = static_cast<size_t>(s->n_phases) * s->grid * kTraceFields * 8;
        CUDA_TRY(dev_malloc(&p, bytes), "trace buffer");
        s->allocs.push_back(p);
        s->trace = static_cast<unsigned long long*>(p);
        CUDA_TRY(cudaMemset(p, 0, bytes), "trace buffer");
    }
    s->trace_step = step < 0 ? -1 : step;
    return TIR_OK;
}

tir_status tir_state_trace_dims(const tir_state* s, int32_t* n_phases, int32_t* grid) {
    if (!s) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (n_phases) *n_phases = s->n_phases;
    if (grid) *grid = s->grid;
    return TIR_OK;
}

tir_status tir_state_trace(tir_state* s, uint64_t* out_host) {
    clear_error();
    if (!s || !out_host) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (!s->trace) return fail(TIR_ERR_INVALID_ARG, "trace not enabled");
    CUDA_TRY(cudaSetDevice(s->m->device), "cudaSetDevice");
    CUDA_TRY(cudaStreamSynchronize(s->stream), "trace readback");
    CUDA_TRY(cudaMemcpy(out_host, s->trace, static_cast<size_t>(s->n_phases) * s->grid * kTraceFields * 8,
                        cudaMemcpyDeviceToHost),
             "trace readback");
    return TIR_OK;
}

// ---------------------------------------------------------------------------
// op-level entry points
// ---------------------------------------------------------------------------
static tir_status op_rc(int rc, const char* what) {
    if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), what);
    return TIR_OK;
}

int64_t tir_q8_scale_stride(int64_t k) { return scale_stride(k); }

tir_status tir_q8_repack(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* quants, uint16_t* scales,
                         void* stream) {
    clear_error();
    if (rows < 0 || k < 0 || k % 32 != 0) return fail(TIR_ERR_BAD_QUANT_BLOCK, "q8_0 tensor length " + std::to_string(k) + " is not a multiple of 32");
    const int64_t sk = scale_stride(k);
    if (rows > 0 && cudaMemsetAsync(scales, 0, static_cast<size_t>(rows * sk * 2), static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return fail(TIR_ERR_CUDA, "scale memset");
    return op_rc(launch_repack(blocks, rows, k, quants, scales, sk, 1, 0, stream), "repack");
}

tir_status tir_q8_matmul(const float* x, const uint8_t* quants, const uint16_t* scales, float* out, int64_t n,
                         int64_t k, void* stream) {
    clear_error();
    if (n < 0 || k <= 0 || k % 32 != 0 || k > kMaxK)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "q8 matvec needs 0 < k <= " + std::to_string(kMaxK) + ", k % 32 == 0");
    if (n > INT32_MAX / 2) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "too many rows");
    if (!quants || !scales) return fail(TIR_ERR_INVALID_ARG, "null weights");
    return q8_matmul_stream(x, quants, scales, out, n, k, stream);
}

tir_status tir_q8_matmul_qact(const float* x, const uint8_t* quants, const uint16_t* scales, float* out, int64_t n,
                              int64_t k, void* stream) {
    clear_error();
    if (n < 0 || k <= 0 || k % 32 != 0 || k > kMaxK)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "q8 matvec needs 0 < k <= " + std::to_string(kMaxK) + ", k % 32 == 0");
    if (n > INT32_MAX / 2) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "too many rows");
    if (!quants || !scales) return fail(TIR_ERR_INVALID_ARG, "null weights");
    return q8_matmul_stream(x, quants, scales, out, n, k, stream, true);
}

int64_t tir_q8_tile_rows(int64_t k) { return tile_rows_for(k, false); }

int64_t tir_q8_tiled_bytes(int64_t n, int64_t k) {
    if (n < 0 || tile_rows_for(k, false) == 0) return -1;
    return q8_tiled_matrix_bytes(n, k);
}

tir_status tir_q8_repack_tiled(const uint8_t* blocks, int64_t rows, int64_t k, uint8_t* out, void* stream) {
    clear_error();
    if (rows < 0 || k <= 0 || k % 32 != 0) return fail(TIR_ERR_BAD_QUANT_BLOCK, "q8_0 tensor length " + std::to_string(k) + " is not a multiple of 32");
    const int r = tile_rows_for(k, false);
    if (r == 0 || k > kMaxK) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "tiled layout needs k <= " + std::to_string(kMaxK));
    if (rows > 0 && cudaMemsetAsync(out, 0, static_cast<size_t>(q8_tiled_matrix_bytes(rows, k)), static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return fail(TIR_ERR_CUDA, "tiled memset");
    return op_rc(launch_repack_tiled(blocks, rows, k, out, rows, r, 1, 0, stream), "repack");
}

tir_status tir_q8_matmul_tiled(const float* x, const uint8_t* w, float* out, int64_t n, int64_t k, void* stream) {
    clear_error();
    if (n < 0 || k <= 0 || k % 32 != 0 || k > kMaxK)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "q8 matvec needs 0 < k <= " + std::to_string(kMaxK) + ", k % 32 == 0");
    if (n > INT32_MAX / 2) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "too many rows");
    if (!w) return fail(TIR_ERR_INVALID_ARG, "null weights");
    return q8_matmul_stream(x, w, nullptr, out, n, k, stream);
}

int64_t tir_q8_gemm_bytes(int64_t n, int64_t k) {
    if (n <= 0 || k <= 0 || k % 64 != 0) return -1;
    return gemm_q8_weight_bytes(n, k);
}

int64_t tir_q8_gemm_rows(int64_t n) { return n <= 0 ? 0 : gemm_q8_rows_padded(n); }

tir_status tir_q8_gemm_prepare(const uint8_t* blocks, int64_t n, int64_t k, uint8_t* w, float* w_pow2, void* stream) {
    clear_error();
    if (n <= 0 || k <= 0 || k % 64 != 0)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "tensor-core layout needs n > 0 and k a positive multiple of 64");
    if (!blocks || !w || !w_pow2) return fail(TIR_ERR_INVALID_ARG, "null argument");
    return op_rc(launch_gemm_repack(blocks, n, k, w, w_pow2, stream), "gemm repack");
}

tir_status tir_q8_matmul_batch(const float* x, int64_t tokens, const uint8_t* w, const float* w_pow2, float* y,
                               int64_t n, int64_t k, void* stream) {
    clear_error();
    if (tokens < 0 || n <= 0 || k <= 0 || k % 64 != 0 || k > kMaxK || n > INT32_MAX / 2 || tokens > INT32_MAX / 2)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE,
                    "batched q8 matmul needs n > 0 and k a positive multiple of 64, at most " + std::to_string(kMaxK));
    if (!x || !w || !w_pow2 || !y) return fail(TIR_ERR_INVALID_ARG, "null argument");
    if (tokens == 0) return TIR_OK;
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    DevCtx* c = dev_ctx(dev);
    if (!c) return fail(TIR_ERR_OOM, "device context allocation failed");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const int sms = decode_grid_size(dev);
    const int splits = gemm_real_splits(k, gemm_splits(n, k, tokens, sms));
    uint8_t* planes = nullptr;
    const size_t pbytes = static_cast<size_t>(gemm_x_plane_bytes(tokens, k));
    const size_t ibytes = static_cast<size_t>(gemm_tokens_padded(tokens)) * 4;
    const size_t sbytes = splits > 1 ? static_cast<size_t>(splits) * tokens * n * 4 : 0;
    CUDA_TRY(dev_malloc_async(reinterpret_cast<void**>(&planes), pbytes + ibytes + sbytes, st),
             "batched matmul scratch");
    float* inv = reinterpret_cast<float*>(planes + pbytes);
    float* part = splits > 1 ? reinterpret_cast<float*>(planes + pbytes + ibytes) : y;
    int rc = static_cast<int>(clear_launch_error(c->error, stream));
    if (rc == 0) rc = launch_gemm_x_planes(x, tokens, k, planes, inv, stream);
    if (rc == 0) rc = launch_gemm_q8(w, w_pow2, planes, inv, n, k, tokens, part, n, splits, c->error, timeout_ns(), stream);
    if (rc == 0 && splits > 1) rc = launch_gemm_sum_parts(part, splits, tokens * n, tokens * n, y, stream);
    cudaFreeAsync(planes, st);
    if (rc != 0) return cuda_fail(static_cast<cudaError_t>(rc), "batched q8 matmul");
    return TIR_OK;
}

tir_status tir_q8_dequant(const uint8_t* blocks, int64_t n_blocks, float* out, void* stream) {
    clear_error();
    if (n_blocks < 0) return fail(TIR_ERR_INVALID_ARG, "negative size");
    return op_rc(launch_dequant(blocks, n_blocks, out, stream), "dequant");
}

tir_status tir_embed(const uint8_t* blocks, int64_t vocab, int64_t id, int64_t dim, float* out, void* stream) {
    clear_error();
    if (dim % 32 != 0) return fail(TIR_ERR_BAD_QUANT_BLOCK, "q8_0 tensor length " + std::to_string(dim) + " is not a multiple of 32");
    if (id < 0 || id >= vocab) return fail(TIR_ERR_BAD_TOKEN, "token id " + std::to_string(id) + " is not in the vocab");
    const int64_t row_blocks = dim / 32;
    return op_rc(launch_dequant(blocks + id * row_blocks * 34, row_blocks, out, stream), "embed");
}

tir_status tir_rmsnorm(const float* x, const float* w, float* out, int64_t n, void* stream) {
    clear_error();
    if (n <= 0) return fail(TIR_ERR_INVALID_ARG, "empty input");
    return op_rc(launch_rmsnorm(x, w, out, n, 1e-5f, stream), "rmsnorm");
}

tir_status tir_softmax(const float* x, float* out, int64_t n, void* stream) {
    clear_error();
    if (n <= 0) return fail(TIR_ERR_INVALID_ARG, "empty input (the reference unwraps on it)");
    return op_rc(launch_softmax(x, out, n, stream), "softmax");
}

void tir_rope_angles(float base, int64_t pos, int64_t dim, float* out_host) {
    for (int64_t i = 0; i < dim / 2; ++i) {
        const float frequency = powf(base, (-2.0f * static_cast<float>(i)) / static_cast<float>(dim));
        out_host[i] = static_cast<float>(pos) * frequency;
    }
}

tir_status tir_rope(float* q, int64_t nq, float* k, int64_t nk, const float* thetas_host, int64_t dim,
                    void* stream) {
    clear_error();
    if (dim <= 0 || dim % 2 != 0 || dim > 128 || !thetas_host) return fail(TIR_ERR_INVALID_ARG, "rope dim must be even and <= 128");
    std::vector<float> cs(static_cast<size_t>(dim));
    for (int64_t i = 0; i < dim / 2; ++i) {
        cs[i] = cosf(thetas_host[i]);
        cs[dim / 2 + i] = sinf(thetas_host[i]);
    }
    return op_rc(launch_rope(q, nq, k, nk, cs.data(), dim, stream), "rope");
}

tir_status tir_swiglu(const float* x, const uint8_t* gate_q, const uint16_t* gate_s, const uint8_t* up_q,
                      const uint16_t* up_s, const uint8_t* down_q, const uint16_t* down_s, float* out, int64_t k,
                      int64_t f, void* stream) {
    clear_error();
    if (k <= 0 || f <= 0 || k % 32 || f % 32 || k > kMaxK || f > kMaxK)
        return fail(TIR_ERR_UNSUPPORTED_SHAPE, "swiglu needs k, f multiples of 32 and <= " + std::to_string(kMaxK));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float* tmp = nullptr;
    CUDA_TRY(dev_malloc_async(reinterpret_cast<void**>(&tmp), static_cast<size_t>(3 * f) * 4, st), "swiglu scratch");
    tir_status rc = q8_matmul_stream(x, gate_q, gate_s, tmp, f, k, stream);
    if (rc == TIR_OK) rc = q8_matmul_stream(x, up_q, up_s, tmp + f, f, k, stream);
    if (rc == TIR_OK) rc = op_rc(launch_silu_mul(tmp, tmp + f, tmp + 2 * f, f, stream), "silu");
    if (rc == TIR_OK) rc = q8_matmul_stream(tmp + 2 * f, down_q, down_s, out, k, f, stream);
    cudaFreeAsync(tmp, st);
    return rc;
}

tir_status tir_activated_q8(const float* x, int64_t k, uint8_t* out_blocks, void* stream) {
    clear_error();
    if (k < 0 || k % 32 != 0) return fail(TIR_ERR_BAD_QUANT_BLOCK, "q8_0 tensor length " + std::to_string(k) + " is not a multiple of 32");
    return op_rc(launch_activated_q8(x, k, out_blocks, stream), "activated_q8");
}

tir_status tir_q8_act_matmul(const uint8_t* x_blocks, const uint8_t* quants, const uint16_t* scales, float* out,
                             int64_t n, int64_t k, void* stream) {
    clear_error();
    if (k <= 0 || k % 32 != 0 || k > 65536) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "k must be a positive multiple of 32");
    if (n == 0) return TIR_OK;
    return op_rc(launch_q8_act_matmul(x_blocks, quants, scales, out, n, k, stream), "q8_act_matmul");
}

tir_status tir_argmax(const float* x, int64_t n, int32_t* out_id, void* stream) {
    clear_error();
    if (n < 0) return fail(TIR_ERR_INVALID_ARG, "negative size");
    return op_rc(launch_argmax(x, n, out_id, stream), "argmax");
}

tir_status tir_ops_check(void* stream) {
    clear_error();
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev), "cudaGetDevice");
    CUDA_TRY(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "stream synchronize");
    uint32_t code = 0;
    DevCtx* c = dev_ctx(dev);
    if (!c) return fail(TIR_ERR_OOM, "device context allocation failed");
    CUDA_TRY(cudaMemcpy(&code, c->error + 3, sizeof(uint32_t), cudaMemcpyDeviceToHost), "op error readback");
    if (code != 0u) CUDA_TRY(cudaMemset(c->error + 3, 0, sizeof(uint32_t)), "op error reset");
    uint32_t scode = 0;
    const tir_status rc = static_scratch_take_error(dev, &scode);
    if (rc != TIR_OK) return rc;
    if (code != 0u || scode != 0u)
        return fail(TIR_ERR_TIMEOUT, "a device-side wait of an op launched on device " + std::to_string(dev) +
                                         " gave up (TIR_TIMEOUT_MS); its outputs are incomplete");
    return TIR_OK;
}

void tir_debug_fail_alloc_after(int64_t n) { g_alloc_fail_in.store(n < 0 ? -1 : static_cast<long long>(n)); }

int64_t tir_debug_alloc_count(void) { return static_cast<int64_t>(g_alloc_calls.load()); }

tir_status tir_debug_hold_next_op(int32_t timeout_us) {
    clear_error();
    if (timeout_us <= 0) return fail(TIR_ERR_INVALID_ARG, "the hold needs a positive limit");
    g_hold_next_op_us.store(timeout_us);
    return TIR_OK;
}

tir_status tir_debug_hold_phase(tir_state* s, int32_t phase, int32_t timeout_us) {
    clear_error();
    if (!s || phase < 0 || phase >= s->n_phases || timeout_us <= 0)
        return fail(TIR_ERR_INVALID_ARG, "hold needs a phase in [0, n_phases) and a positive limit");
    s->hold_phase = phase;
    s->hold_timeout_ns = static_cast<unsigned long long>(timeout_us) * 1000ull;
    return TIR_OK;
}

tir_status tir_attention(const float* q, const float* k_cache, const float* v_cache, float* out, int64_t q_heads,
                         int64_t k_v_heads, int64_t dim, int64_t n_ctx, int64_t max_ctx, void* stream) {
    clear_error();
    if (dim != kHeadDim) return fail(TIR_ERR_UNSUPPORTED_SHAPE, "attention head dim must be 64");
    if (q_heads <= 0 || k_v_heads <= 0 || q_heads % k_v_heads != 0 || n_ctx <= 0 || n_ctx > max_ctx)
        return fail(TIR_ERR_INVALID_ARG, "bad attention shape");
    return op_rc(launch_attention(q, k_cache, v_cache, out, q_heads, k_v_heads, n_ctx, max_ctx, stream), "attention");
}

}  // extern "C"
