/*
 * tir.h -- C ABI of the B200 (sm_100a) decode runtime for the Q8_0 Llama-2
 * path of ZeroR0R/tensor-inference-runtime.
 *
 * The reference is an in-process Rust crate; every entry point below names the
 * reference function (path:line within that crate) it replaces.  Plain
 * pointers and sizes only.  Unless stated otherwise:
 *   - "host" pointers are ordinary CPU memory, "device" pointers are CUDA
 *     global memory on the device the object was created on;
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default);
 *   - functions return tir_status; on failure tir_last_error() returns a
 *     thread-local message formatted like the reference's thiserror Display.
 * The library owns all memory it allocates.  A tir_state is not thread-safe;
 * distinct states may be driven from distinct host threads.
 */
#ifndef TIR_H
#define TIR_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (src/error.rs) ----------------------------------------- */
typedef enum tir_status {
    TIR_OK = 0,
    /* ReaderError, src/error.rs:5-24 */
    TIR_ERR_UNEXPECTED_EOF = 1,
    TIR_ERR_INVALID_UTF8 = 2,
    TIR_ERR_BAD_MAGIC = 3,
    TIR_ERR_BAD_VERSION = 4,
    TIR_ERR_UNSUPPORTED_TYPE = 5,
    TIR_ERR_UNSUPPORTED_DTYPE = 6,
    TIR_ERR_BAD_QUANT_BLOCK = 7,
    /* MetaDataError, src/error.rs:27-36 */
    TIR_ERR_MISSING_FIELD = 8,
    TIR_ERR_WRONG_TYPE = 9,
    /* ModelLoadError::TensorDataError, src/error.rs:52-53 */
    TIR_ERR_TENSOR_DATA = 10,
    /* ForwardPassError::TensorLoadError, src/error.rs:60-61 */
    TIR_ERR_TENSOR_LOAD = 11,
    /* TokenizerError::UnknownId (src/error.rs:44-45); also an out-of-range id
     * that the reference's embed() would panic on (src/tokenizer.rs:15) */
    TIR_ERR_BAD_TOKEN = 12,
    /* std::io::Error from read_gguf (src/reader.rs:15-21) */
    TIR_ERR_IO = 13,
    /* runtime conditions with no reference counterpart */
    TIR_ERR_CUDA = 20,
    TIR_ERR_OOM = 21,
    TIR_ERR_CTX_OVERFLOW = 22,  /* pos >= the state's max_ctx */
    TIR_ERR_INVALID_ARG = 23,
    TIR_ERR_UNSUPPORTED_SHAPE = 24,
    TIR_ERR_TIMEOUT = 25,       /* a bounded device-side wait gave up */
    TIR_ERR_NO_DEVICE = 26
} tir_status;

/* Thread-local message of the last failing call on this thread. */
const char *tir_last_error(void);
/* Version string of this library. */
const char *tir_version(void);

/* ---- GGUF reader (src/reader.rs, src/lib.rs:29-138, src/state.rs) -------- */

/* GgufMetadataValueType, src/state.rs:28-56 */
enum {
    TIR_GGUF_U8 = 0, TIR_GGUF_I8 = 1, TIR_GGUF_U16 = 2, TIR_GGUF_I16 = 3,
    TIR_GGUF_U32 = 4, TIR_GGUF_I32 = 5, TIR_GGUF_F32 = 6, TIR_GGUF_BOOL = 7,
    TIR_GGUF_STRING = 8, TIR_GGUF_ARRAY = 9, TIR_GGUF_U64 = 10, TIR_GGUF_I64 = 11,
    TIR_GGUF_F64 = 12
};
/* Tensor dtypes the reference accepts (src/reader.rs:247-253). */
enum { TIR_DTYPE_F32 = 0, TIR_DTYPE_Q8_0 = 8 };

typedef struct tir_gguf tir_gguf;

/* MetaDataField (src/state.rs:9-14) with the value widened: `u` holds
 * U8/U16/U32/U64/BOOL, `i` holds I8/I16/I32/I64, `f` holds F32/F64 (F32
 * exactly), `str`/`str_len` hold STRING (not NUL-terminated), and
 * `array_type`/`array_len` describe ARRAY (items via tir_gguf_metadata_item). */
typedef struct tir_metadata_field {
    const char *name;
    uint32_t vtype;
    uint64_t u;
    int64_t i;
    double f;
    const char *str;
    uint64_t str_len;
    uint32_t array_type;
    uint64_t array_len;
} tir_metadata_field;

/* Tensor (src/data.rs:3-9): `n_dims` is the reference's `n_elements` field. */
typedef struct tir_tensor_info {
    const char *name;
    uint32_t n_dims;
    uint64_t shape[8];
    uint32_t dtype;
    uint64_t offset;      /* relative to the aligned data start */
    uint64_t data_bytes;  /* parse_tensor_data's slice length */
} tir_tensor_info;

/* Transformer (src/data.rs:25-33) plus the sizes the reference hard-codes
 * (src/forward.rs:46,54,250; src/math.rs:165), read from tensor shapes. */
typedef struct tir_transformer {
    uint32_t layers;
    uint64_t dim;        /* head / rope dimension (llama.rope.dimension_count) */
    uint64_t embed_dim;
    uint64_t q_heads;
    uint64_t k_v_heads;
    float base_freq;
    int32_t mode;        /* Mode, src/data.rs:16-20: 0 Normal, 1 Quantize */
    uint64_t kv_dim;     /* k_v_heads * dim */
    uint64_t ffn_dim;
    uint64_t vocab;
} tir_transformer;

/* read_gguf + load_model's parse (src/reader.rs:15, src/lib.rs:29-138):
 * checks magic/version, parses metadata, the Transformer fields, tensor infos
 * and every tensor's data bounds.  The file is read into host memory. */
tir_status tir_gguf_open(const char *path, tir_gguf **out);
/* Same over a caller buffer; the bytes are copied. */
tir_status tir_gguf_open_bytes(const uint8_t *data, size_t len, tir_gguf **out);
void tir_gguf_close(tir_gguf *g);
/* parse_general (src/reader.rs:98-169) alone, over `count` fields starting at
 * `offset` of `data`; returns a handle holding only metadata and the offset
 * just past the last field. */
tir_status tir_gguf_parse_general(const uint8_t *data, size_t len, size_t offset,
                                  uint64_t count, tir_gguf **out, size_t *end_offset);
/* parse_q8 (src/reader.rs:258-272): byte length of `count` Q8_0 weights. */
tir_status tir_gguf_parse_q8(uint64_t count, size_t byte_count, size_t map_len, size_t offset,
                             size_t *out_len);
uint32_t tir_gguf_version(const tir_gguf *g);
int64_t tir_gguf_n_metadata(const tir_gguf *g);
tir_status tir_gguf_metadata(const tir_gguf *g, int64_t i, tir_metadata_field *out);
tir_status tir_gguf_metadata_item(const tir_gguf *g, int64_t i, uint64_t j,
                                  tir_metadata_field *out);
int64_t tir_gguf_n_tensors(const tir_gguf *g);
tir_status tir_gguf_tensor_info(const tir_gguf *g, int64_t i, tir_tensor_info *out);
/* The HashMap<String,&[u8]> lookup of get_tensor (src/forward.rs:277-285):
 * TIR_ERR_TENSOR_LOAD if `name` is absent.  Host pointer into the handle. */
tir_status tir_gguf_tensor_data(const tir_gguf *g, const char *name, const uint8_t **data,
                                size_t *len);
/* load_model's Transformer extraction (src/lib.rs:70-115). */
tir_status tir_gguf_transformer(const tir_gguf *g, tir_transformer *out);

/* ---- model: weights resident in HBM --------------------------------------- */
typedef struct tir_model tir_model;

/* read_gguf + load_model (src/reader.rs:15, src/lib.rs:29): parse, repack
 * Q8_0 into the runtime's split layout and upload once to HBM on `device`. */
tir_status tir_model_load(const char *path, int device, tir_model **out);
tir_status tir_model_load_gguf(const tir_gguf *g, int device, tir_model **out);
tir_status tir_model_info(const tir_model *m, tir_transformer *out);
/* Mode switch (the q_act cargo feature, src/lib.rs:99-103). */
tir_status tir_model_set_mode(tir_model *m, int32_t mode);
/* Device bytes held by the model's weights. */
uint64_t tir_model_weight_bytes(const tir_model *m);
void tir_model_destroy(tir_model *m);

/* ---- state: the KV cache (src/data.rs:41-51 Cache) ----------------------- */
typedef struct tir_state tir_state;

/* Cache::new (src/data.rs:48), bounded: one sequence, positions < max_ctx. */
tir_status tir_state_create(tir_model *m, int32_t max_ctx, tir_state **out);
/* Empties the cache (next forward is pos 0). */
tir_status tir_state_reset(tir_state *s);
/* Number of cached positions. */
int32_t tir_state_len(const tir_state *s);
/* The CUDA stream (cudaStream_t) every call on this state is ordered on. */
void *tir_state_stream(tir_state *s);
void tir_state_destroy(tir_state *s);

/* forward (src/forward.rs:13-258) with the input already embedded:
 * x_host = embed_dim floats, pos must equal tir_state_len(s).
 * logits_host (optional) receives vocab floats. */
tir_status tir_forward_embedded(tir_state *s, const float *x_host, int32_t pos,
                                float *logits_host);
/* embed (src/tokenizer.rs:10) + forward: token id in, logits out. */
tir_status tir_forward(tir_state *s, int32_t token_id, int32_t pos, float *logits_host);
/* generate_capped (src/lib.rs:239-314) on token ids: token-by-token prompt
 * pass then greedy decode of `cap` ids into out_ids_host.  The whole loop runs
 * on the device in one launch; only ids cross the boundary.  Starts from an
 * empty cache.  last_logits_host (optional): logits of the final forward. */
tir_status tir_generate_capped(tir_state *s, const int32_t *prompt_host, int32_t n_prompt,
                               int32_t cap, int32_t *out_ids_host, float *last_logits_host);
/* The prompt pass of generate_capped alone: seq_len ids from position 0 of an
 * empty cache; last_logits_host (optional) gets the last position's logits.
 * n_seqs must be 1 (a tir_state holds one sequence; n_seqs sequences prefill
 * with tir_batch_step, tokens_per_seq = seq_len). */
tir_status tir_prefill(tir_state *s, const int32_t *ids_host, int32_t n_seqs, int32_t seq_len,
                       float *last_logits_host);
/* Same with device buffers, asynchronous on tir_state_stream(s). */
tir_status tir_generate_capped_device(tir_state *s, const int32_t *prompt_dev, int32_t n_prompt,
                                      int32_t cap, int32_t *out_ids_dev);
/* Waits for the state's stream and reports a device-side timeout, if any
 * (use after tir_generate_capped_device). */
tir_status tir_state_sync(tir_state *s);
/* test_forward (src/lib.rs:316-328): all-ones embedding at pos 0 on an empty
 * cache, argmax of the logits. */
tir_status tir_test_forward(tir_state *s, int32_t *out_id);
/* Residual stream of the last forward: (layers+1) x embed_dim floats, the
 * input and the output of every layer (the per-layer dump of
 * save_intermediate, src/forward.rs:287-308).  Enable before the forward. */
tir_status tir_state_enable_dump(tir_state *s, int32_t enable);
tir_status tir_state_dump(tir_state *s, float *out_host);
/* The layer outputs alone: layers x embed_dim floats (rows 1.. of the dump). */
tir_status tir_debug_dump_layers(tir_state *s, float *out_host);
/* Mode::Quantize: the Q8_0 blocks activated_q8 (src/kernels.rs:8-31) made of
 * the q|k|v, o and lm_head inputs in the last forward, as the fused kernel
 * staged them: [(2 L + 1)][embed_dim / 32] blocks of 34 bytes ([2 l] q|k|v of
 * layer l, [2 l + 1] o of layer l, [2 L] lm_head).  Needs the dump on
 * (tir_state_enable_dump) and the model in Mode 1; runtime extension for
 * parity tests. */
tir_status tir_debug_dump_qact(tir_state *s, uint8_t *out_host);
/* Phase timeline (profiling; the reference's tracing is the debug-build
 * save_intermediate, src/forward.rs:287-308): with step >= 0, every later
 * launch records, for forward step `step`, eight values per phase per CTA:
 * globaltimer stamps (ns) at start, inputs ready, input staged and release,
 * then ns spent waiting for streamed weights, tiles processed, ns spent
 * waiting for the previous phase, 0.  step < 0 turns it off.
 * tir_state_trace copies n_phases x grid x 8 uint64 values. */
tir_status tir_state_enable_trace(tir_state *s, int32_t step);
tir_status tir_state_trace_dims(const tir_state *s, int32_t *n_phases, int32_t *grid);
tir_status tir_state_trace(tir_state *s, uint64_t *out_host);

/* ---- text: tokenizer and text drivers (src/tokenizer.rs:37-150, src/lib.rs:140-314)
 * Host-side BPE over the GGUF's tokenizer.ggml.tokens / tokenizer.ggml.merges. */
typedef struct tir_tokenizer tir_tokenizer;
/* MissingField / WrongType as the drivers report them (src/lib.rs:149-160,
 * src/tokenizer.rs:42-48). */
tir_status tir_tokenizer_create(const tir_gguf *g, tir_tokenizer **out);
/* From caller arrays (token / merge strings with their byte lengths). */
tir_status tir_tokenizer_create_from(const char *const *tokens, const uint64_t *token_lens, int64_t n_tokens,
                                     const char *const *merges, const uint64_t *merge_lens, int64_t n_merges,
                                     tir_tokenizer **out);
void tir_tokenizer_destroy(tir_tokenizer *t);
int64_t tir_tokenizer_vocab_size(const tir_tokenizer *t);
/* encode (src/tokenizer.rs:37-120): BOS 1, then the BPE ids of `text`
 * (UTF-8, text_len bytes).  *n gets the id count; up to cap ids are written. */
tir_status tir_encode(const tir_tokenizer *t, const char *text, int64_t text_len, int32_t *ids, int64_t cap,
                      int64_t *n);
/* decode (src/tokenizer.rs:122-143): TIR_ERR_BAD_TOKEN on an id outside the
 * vocab (UnknownId).  *len gets the byte length; up to cap - 1 bytes and a NUL
 * are written. */
tir_status tir_decode(const tir_tokenizer *t, const int32_t *ids, int64_t n_ids, char *out, int64_t cap,
                      int64_t *len);
/* generate_capped on text (src/lib.rs:239-314): out_ids_host [cap]. */
tir_status tir_generate_capped_text(tir_state *s, const tir_tokenizer *tk, const char *text, int64_t text_len,
                                    int32_t cap, int32_t *out_ids_host);
/* generate (src/lib.rs:140-236): greedy until id 13 or 2 (not kept), at most
 * max_new ids; the kept ids decoded into out_text. */
tir_status tir_generate_text(tir_state *s, const tir_tokenizer *tk, const char *text, int64_t text_len,
                             int32_t max_new, char *out_text, int64_t cap, int64_t *out_len, int32_t *n_ids);

/* ---- batched sequences: many tokens per forward --------------------------- */
/* n_seqs sequences, each computing what generate_capped (src/lib.rs:239-314)
 * computes for it alone, with every projection on the tensor cores
 * (tir_q8_matmul_batch).  The KV cache (replacing the unbounded Cache,
 * src/data.rs:41-51) is paged: positions in pages of 16 from a pool shared by
 * the sequences, taken as a sequence grows and returned when it is reset, so
 * sequences of different lengths share the memory (continuous batching).
 * The batch keeps a tensor-core copy of the model's weights. */
typedef struct tir_batch tir_batch;
/* A pool of n_pages pages (16 positions each, all layers). */
tir_status tir_batch_create_paged(tir_model *m, int32_t n_seqs, int32_t max_ctx, int32_t max_tokens_per_seq,
                                  int32_t n_pages, tir_batch **out);
/* The pool every sequence can fill to max_ctx at once. */
tir_status tir_batch_create(tir_model *m, int32_t n_seqs, int32_t max_ctx, int32_t max_tokens_per_seq,
                            tir_batch **out);
void tir_batch_destroy(tir_batch *b);
/* Every sequence / sequence `seq` empty again (its pages back in the pool). */
tir_status tir_batch_reset(tir_batch *b);
tir_status tir_batch_reset_seq(tir_batch *b, int32_t seq);
/* The longest sequence's length; sequence `seq`'s length; free pool pages. */
int32_t tir_batch_len(const tir_batch *b);
int32_t tir_batch_seq_len(const tir_batch *b, int32_t seq);
int32_t tir_batch_free_pages(const tir_batch *b);
void *tir_batch_stream(tir_batch *b);
/* counts_host[s] new ids for sequence s (0: idle this step, > 1: a prompt
 * chunk, mixed freely), ids_host their concatenation in sequence order;
 * next_ids_host [n_seqs] (may be NULL) gets each sequence's greedy next id
 * (meaningless for idle ones).  TIR_ERR_CTX_OVERFLOW past max_ctx, TIR_ERR_OOM
 * when the pool runs short (nothing changes then). */
tir_status tir_batch_step_ragged(tir_batch *b, const int32_t *ids_host, const int32_t *counts_host,
                                 int32_t *next_ids_host);
/* tokens_per_seq ids for every sequence (ids_host [n_seqs][tokens_per_seq]). */
tir_status tir_batch_step(tir_batch *b, const int32_t *ids_host, int32_t tokens_per_seq,
                          int32_t *next_ids_host);
/* Per sequence from empty: prompt (prompts_host [n_seqs][n_prompt]) then cap
 * greedy steps, n_prompt + cap forwards as generate_capped; out_ids_host
 * [n_seqs][cap]. */
tir_status tir_batch_generate(tir_batch *b, const int32_t *prompts_host, int32_t n_prompt, int32_t cap,
                              int32_t *out_ids_host);
/* Logits of every sequence's last row in the last forward, logits_host
 * [n_seqs][vocab] (forward's return value, src/forward.rs:242-252, per
 * sequence; a sequence idle in that step gets zeros). */
tir_status tir_batch_logits(tir_batch *b, float *logits_host);
/* Per-layer outputs of chosen step rows, for layer-by-layer comparison with
 * the reference's forward (src/forward.rs:13-258; the batched counterpart of
 * tir_debug_dump_layers).  tir_batch_dump_rows arms a dump of rows_host[i]
 * (indices into the step's rows, sequence-major) for every later forward run
 * outside the captured decode graph (prefill and ragged steps; n_rows = 0
 * disarms); tir_batch_dump copies [n_rows][layers][embed_dim] of the last
 * such forward to out_host. */
tir_status tir_batch_dump_rows(tir_batch *b, const int32_t *rows_host, int32_t n_rows);
tir_status tir_batch_dump(tir_batch *b, float *out_host);

/* ---- op-level kernels (device pointers, asynchronous on `stream`) --------- */

/* Q8_0 blocks (34 B: f16 scale LE + 32 int8) of a [rows][k] tensor into the
 * runtime's split layout: quants [rows][k] signed int8 q, scales
 * [rows][scale_stride] f16 with scale_stride = tir_q8_scale_stride(k). */
int64_t tir_q8_scale_stride(int64_t k);
tir_status tir_q8_repack(const uint8_t *blocks, int64_t rows, int64_t k, uint8_t *quants,
                         uint16_t *scales, void *stream);
/* Tile-major Q8_0 layout (the layout the decode kernel streams): tiles of
 * tir_q8_tile_rows(k) rows, each holding its rows' int8 quants followed by
 * their f16 scales (scale_stride per row), so one bulk copy moves a tile.
 * tir_q8_tiled_bytes gives the buffer size (-1 for an unsupported k). */
int64_t tir_q8_tile_rows(int64_t k);
int64_t tir_q8_tiled_bytes(int64_t n, int64_t k);
tir_status tir_q8_repack_tiled(const uint8_t *blocks, int64_t rows, int64_t k, uint8_t *out,
                               void *stream);
/* q8_matmul (src/math.rs:87-98) over the tile-major layout. */
tir_status tir_q8_matmul_tiled(const float *x, const uint8_t *w, float *out, int64_t n, int64_t k,
                               void *stream);
/* Batched q8_matmul: the reference's q8_matmul (src/math.rs:87-98) applied to
 * many tokens at once (its forward, src/forward.rs:261-275, does it token by
 * token), on the sm_100a tensor cores.  The weights first go into the
 * tensor-core layout: tir_q8_gemm_bytes(n, k) bytes plus tir_q8_gemm_rows(n)
 * floats (a power of two per row), prepared once from Q8_0 blocks on the
 * device.  Then y[t][j] = sum_c x[t][c] * W[j][c] (f32, y row stride n) for
 * t < tokens; k must be a multiple of 64 and at most 6144 (one activation
 * row is split into the matmul's f16 planes by one CTA, 24 values per
 * thread); larger k returns TIR_ERR_UNSUPPORTED_SHAPE. */
int64_t tir_q8_gemm_bytes(int64_t n, int64_t k);
int64_t tir_q8_gemm_rows(int64_t n);
tir_status tir_q8_gemm_prepare(const uint8_t *blocks, int64_t n, int64_t k, uint8_t *w, float *w_pow2,
                               void *stream);
tir_status tir_q8_matmul_batch(const float *x, int64_t tokens, const uint8_t *w, const float *w_pow2,
                               float *y, int64_t n, int64_t k, void *stream);
/* q8_matmul (src/math.rs:87-98): out[n] = sum_b f32(s[n,b]) * sum_i x[32b+i]*q[n,b,i].
 * Streaming sm_100a GEMV over the split layout. */
tir_status tir_q8_matmul(const float *x, const uint8_t *quants, const uint16_t *scales,
                         float *out, int64_t n, int64_t k, void *stream);
/* matmul in Mode::Quantize (src/forward.rs:266-273): the f32 input quantised
 * per 32 values by activated_q8 (src/kernels.rs:8-31), then q8_act_matmul
 * (src/math.rs:101-112) -- exact integer block dots times the f16 activation
 * scale and the weight scale -- on the split layout; the same input staging
 * and block dot as the fused decode kernel's Mode::Quantize phases. */
tir_status tir_q8_matmul_qact(const float *x, const uint8_t *quants, const uint16_t *scales, float *out,
                              int64_t n, int64_t k, void *stream);
/* q8_full_dequant / q8_dequant_block (src/math.rs:117-137): bit-exact. */
tir_status tir_q8_dequant(const uint8_t *blocks, int64_t n_blocks, float *out, void *stream);
/* embed (src/tokenizer.rs:10-32): row `id` of a Q8_0 [vocab][dim] table. */
tir_status tir_embed(const uint8_t *blocks, int64_t vocab, int64_t id, int64_t dim, float *out,
                     void *stream);
/* rmsnorm (src/math.rs:141-150). */
tir_status tir_rmsnorm(const float *x, const float *w, float *out, int64_t n, void *stream);
/* softmax (src/math.rs:153-161). */
tir_status tir_softmax(const float *x, float *out, int64_t n, void *stream);
/* rope (src/math.rs:196-228) in place; thetas = dim/2 angles (rope_angles). */
tir_status tir_rope(float *q, int64_t nq, float *k, int64_t nk, const float *thetas, int64_t dim,
                    void *stream);
/* rope_angles (src/math.rs:181-193), host: dim/2 floats into out_host. */
void tir_rope_angles(float base, int64_t pos, int64_t dim, float *out_host);
/* swiglu (src/math.rs:164-178) over split-layout gate/up ([f][k]) and down
 * ([k][f]) matrices. */
tir_status tir_swiglu(const float *x, const uint8_t *gate_q, const uint16_t *gate_s,
                      const uint8_t *up_q, const uint16_t *up_s, const uint8_t *down_q,
                      const uint16_t *down_s, float *out, int64_t k, int64_t f, void *stream);
/* tir_swiglu without device allocation.  No counterpart in the reference; this
 * is for callers that must not allocate device memory while they run.  Same inputs
 * and results as tir_swiglu, but gate, up and silu(gate)*up live in a fixed
 * per-device static array, so f <= 6144 (k <= 6144 as for tir_swiglu); larger
 * sizes return TIR_ERR_UNSUPPORTED_SHAPE.  Makes no cudaMalloc/cudaFree call.
 * The first call on a device looks the array's address up (cudaGetSymbolAddress)
 * with that device current; make it before any stream capture on the device.
 * Calls on the same device must not overlap in time: they share the array.
 * A device-side wait that runs out is reported by tir_ops_check. */
tir_status tir_swiglu_static(const float *x, const uint8_t *gate_q, const uint16_t *gate_s,
                             const uint8_t *up_q, const uint16_t *up_s, const uint8_t *down_q,
                             const uint16_t *down_s, float *out, int64_t k, int64_t f,
                             void *stream);
/* activated_q8 (src/kernels.rs:8-31): k floats -> k/32 Q8_0 blocks, bit-exact. */
tir_status tir_activated_q8(const float *x, int64_t k, uint8_t *out_blocks, void *stream);
/* q8_act_matmul (src/math.rs:101-112): quantised activation (Q8_0 blocks) x
 * split-layout weights; exact integer block dots, reference block order. */
tir_status tir_q8_act_matmul(const uint8_t *x_blocks, const uint8_t *quants,
                             const uint16_t *scales, float *out, int64_t n, int64_t k,
                             void *stream);
/* sample (src/tokenizer.rs:152-167): argmax by total order, last of equal
 * maxima; n == 0 gives 0. */
tir_status tir_argmax(const float *x, int64_t n, int32_t *out_id, void *stream);
/* Grouped-query decode attention (src/forward.rs:86-174) for one position:
 * q [q_heads*dim], caches [k_v_heads][max_ctx][dim] holding n_ctx positions,
 * out [q_heads*dim]. */
tir_status tir_attention(const float *q, const float *k_cache, const float *v_cache,
                         float *out, int64_t q_heads, int64_t k_v_heads, int64_t dim,
                         int64_t n_ctx, int64_t max_ctx, void *stream);

/* The op entry points above run asynchronously on the caller's stream, so a
 * bounded device-side wait that gave up (TIR_TIMEOUT_MS) inside one of them
 * cannot be returned by the call itself.  tir_ops_check synchronises `stream`
 * and returns TIR_ERR_TIMEOUT if any op launched on the current device since
 * the last check recorded one (tir_q8_matmul*, tir_swiglu*,
 * tir_q8_matmul_batch), clearing the record; TIR_OK otherwise.  No launch
 * starts with an earlier launch's failure in its error words (a matvec's
 * last CTA to exit clears them; the tensor-core op clears them before it
 * starts), so one failure does not make later calls skip their work.  Runtime extension; no counterpart in the
 * reference, whose ops are synchronous CPU code. */
tir_status tir_ops_check(void *stream);

/* ---- test hooks (runtime extensions; no counterpart in the reference) ----
 * tir_debug_fail_alloc_after(n): the n-th next allocation the library makes
 * (device, stream-ordered or pinned host; n = 0 is the next one) fails once
 * with TIR_ERR_OOM, driving the failure branches of model load and
 * state/batch creation (the reference's ModelLoadError, src/error.rs:49-59,
 * covers the same load step).  n < 0 disarms.
 * tir_debug_alloc_count: allocations attempted so far (all kinds).
 * tir_debug_hold_phase(s, phase, timeout_us): in the next decode launch of
 * `s`, the dependency wait at the start of `phase` (in [0, n_phases); phase 0
 * waits from the launch's second step on) expects one release more than the
 * grid makes, with a limit of timeout_us, so that wait runs out on purpose:
 * the launch returns TIR_ERR_TIMEOUT and resets the state, whose next call
 * decodes normally.
 * tir_debug_hold_next_op(timeout_us): the next streaming Q8_0 matvec
 * (tir_q8_matmul, _qact, _tiled, or one inside tir_swiglu) completes its
 * output, then runs a second pass whose start waits for a release that never
 * comes and gives up after timeout_us; tir_ops_check then reports it. */
void tir_debug_fail_alloc_after(int64_t n);
tir_status tir_debug_hold_next_op(int32_t timeout_us);
int64_t tir_debug_alloc_count(void);
tir_status tir_debug_hold_phase(tir_state *s, int32_t phase, int32_t timeout_us);

#ifdef __cplusplus
}
#endif
#endif
