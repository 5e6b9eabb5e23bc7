/*
 * oracle.h -- CPU restatement of the reference's Q8_0 Llama-2 decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path in
 * tensor-inference-runtime_b200/: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / --impl reference legs of bench.py may load it.  The product
 * never links, calls or falls back to it.
 *
 * Every function restates one function of ZeroR0R/tensor-inference-runtime
 * (Rust, CPU-only) with the same arithmetic order: sequential left folds,
 * no FMA contraction (build with -ffp-contract=off), glibc libm for
 * exp/pow/sin/cos, correctly rounded sqrt and division, RNE f32->f16, and
 * Rust's `Sum for f32`, which folds from -0.0.  The file:line in each comment
 * is the reference function restated.
 *
 * Pinning: the reference crate cannot be built here (no Rust toolchain), so
 * the oracle is pinned against the reference's own known-answer unit tests
 * (src/kernels.rs:37-55, src/math.rs:248-430, src/reader.rs:308-359); see
 * tests/test_oracle_kat.py.  Whole-model outputs are not pinned by executing
 * the reference.
 *
 * Generalisation: the reference hard-codes the TinyLlama sizes (q buffer 2048,
 * k/v 256, FFN 5632, vocab 32000, activation buffer 2176).  The oracle takes
 * those sizes from the model; at the TinyLlama shape it is the same code.
 */
#ifndef TIR_ORACLE_H
#define TIR_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* f16 <-> f32 (the `half` 2.7.1 crate: from_f32 is round-to-nearest-even). */
float orc_f16_to_f32(uint16_t h);
uint16_t orc_f32_to_f16(float f);

/* src/math.rs:7 dot_prod_f32 */
float orc_dot_prod_f32(const float *a, const float *b, size_t n);
/* src/math.rs:18 dot_prod_q8: a has k floats, b has k/32 blocks of 34 bytes */
float orc_dot_prod_q8(const float *a, const uint8_t *b, size_t k);
/* src/math.rs:39 dot_prod_act_q8: both sides are k/32 blocks of 34 bytes */
float orc_dot_prod_act_q8(const uint8_t *a, const uint8_t *b, size_t k);
/* src/math.rs:87 q8_matmul: out[n] = dot_prod_q8(a, row n of b) */
void orc_q8_matmul(const float *a, const uint8_t *b, float *out, size_t n, size_t k);
/* src/math.rs:101 q8_act_matmul */
void orc_q8_act_matmul(const uint8_t *a, const uint8_t *b, float *out, size_t n, size_t k);
/* src/kernels.rs:8 activated_q8: k floats -> k/32 blocks of 34 bytes */
void orc_activated_q8(const float *x, size_t k, uint8_t *out);
/* src/math.rs:117-137 q8_dequant_block / q8_full_dequant */
void orc_q8_dequant(const uint8_t *blocks, size_t n_blocks, float *out);
/* src/math.rs:141 rmsnorm */
void orc_rmsnorm(const float *a, const float *w, float *out, size_t n);
/* src/math.rs:153 softmax */
void orc_softmax(const float *x, float *out, size_t n);
/* src/math.rs:164 swiglu (gate/up: f rows of k; down: k rows of f) */
void orc_swiglu(const float *x, const uint8_t *w_gate, const uint8_t *w_up,
                const uint8_t *w_down, float *out, size_t k, size_t f);
/* src/math.rs:181 rope_angles: dim/2 thetas */
void orc_rope_angles(float base, size_t pos, size_t dim, float *out);
/* src/math.rs:196 rope, in place on nq query floats and nk key floats */
void orc_rope(float *q, size_t nq, float *k, size_t nk, const float *thetas, size_t dim);
/* src/tokenizer.rs:10 embed: dequantise row `id` of a Q8_0 [vocab][dim] table */
void orc_embed(size_t id, const uint8_t *embed_tensor, size_t dim, float *out);
/* src/tokenizer.rs:152 sample: argmax by total_cmp, the last of equal maxima */
size_t orc_sample(const float *logits, size_t n);

/* Model shape: the Transformer struct of src/data.rs:25-33 plus the sizes the
 * reference hard-codes.  `mode` is src/data.rs:16-20 (0 Normal, 1 Quantize). */
typedef struct {
    int32_t n_layers, embed_dim, head_dim, q_heads, kv_heads, ffn_dim, vocab;
    float base_freq;
    int32_t mode;
} orc_dims;

/* Tensor table: raw GGUF bytes, in this order:
 *   [0] token_embd.weight  [1] output_norm.weight  [2] output.weight
 *   then per layer l, at 3 + 9*l: attn_norm, attn_q, attn_k, attn_v,
 *   attn_output, ffn_norm, ffn_gate, ffn_up, ffn_down. */
#define ORC_LAYER_TENSORS 9

/* src/data.rs:41-51 Cache: unbounded key/value arrays, layout [pos][layer][kvd]. */
typedef struct orc_cache orc_cache;
orc_cache *orc_cache_new(void);
void orc_cache_free(orc_cache *c);
size_t orc_cache_len(const orc_cache *c);

/* src/forward.rs:13-258 forward.  `token` is the embedded input (embed_dim
 * floats), `angles` the head_dim/2 rope thetas of `pos`.  logits: vocab floats.
 * dump (optional): (n_layers+1) x embed_dim floats, the residual stream before
 * layer 0 and after every layer.  Returns 0, or -1 if `pos` does not match the
 * cache length (the reference would read garbage or panic). */
int orc_forward(const orc_dims *d, const void *const *tensors, orc_cache *cache,
                const float *token, size_t pos, const float *angles,
                float *logits, float *dump);

/* src/lib.rs:239-314 generate_capped, restated on token ids (no tokenizer):
 * token-by-token prompt pass, then greedy decode until `cap` ids.
 * last_logits (optional) receives the logits of the final forward. */
int orc_generate_capped(const orc_dims *d, const void *const *tensors,
                        const int32_t *prompt, size_t n_prompt, size_t cap,
                        int32_t *out_ids, float *last_logits);

/* Thread count used by the parallel matvecs (Rayon's pool in the reference). */
void orc_set_threads(int n);
/* Test aid: buf (n_layers x embed_dim floats) receives each layer's attention
 * output from the next orc_forward calls on; NULL stops it. */
void orc_set_attn_dump(float *buf);
/* 1: eight matrix rows per pass and attention heads in parallel (same bits,
 * faster; for the tests); 0 (default): the reference's loop order. */
void orc_set_fast(int on);
int orc_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
