/*
 * oracle.c -- CPU restatement of the reference decode path (test
 * infrastructure only; see oracle.h for the rules this file follows).
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off -fopenmp).  No FMA
 * contraction and no -ffast-math, so every float operation below is one IEEE
 * single-precision operation in source order, as in the Rust reference.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Rust's `impl Sum for f32` folds from -0.0 (core::iter accum.rs). */
#define RUST_SUM_INIT (-0.0f)

static int g_threads = 0;
/* 0: one matrix row at a time and attention heads in order, as the reference
 * loops (the CPU baseline times this); 1: eight rows per pass and attention
 * heads in parallel, for the tests.  Every row and every head performs the
 * same operations in the same order either way, so the results are
 * bit-identical (tests/test_oracle_kat.py checks it). */
static int g_fast = 0;

void orc_set_threads(int n) { g_threads = n; }

void orc_set_fast(int on) { g_fast = on ? 1 : 0; }

/* When set, orc_forward also copies each layer's attention output (the input
 * of the output projection, src/forward.rs:176) to attn_dump + l * embed_dim. */
static float *g_attn_dump = NULL;

void orc_set_attn_dump(float *buf) { g_attn_dump = buf; }

int orc_get_threads(void) {
#ifdef _OPENMP
    return g_threads > 0 ? g_threads : omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- f16 <-> f32 ---------------------------------------------------------- */

float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: normalise */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400u) == 0);
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xffu;
    uint32_t man = x & 0x7fffffu;
    if (exp == 0xff) {
        if (man == 0) return (uint16_t)(sign | 0x7c00u);
        return (uint16_t)(sign | 0x7e00u | (man >> 13)); /* quiet NaN */
    }
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 0x1f) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        /* f16 subnormal: value in units of 2^-24 is M >> s */
        int32_t s = 14 - e;
        if (s > 24) return (uint16_t)sign;
        uint32_t M = man | 0x800000u;
        uint32_t q = M >> s;
        uint32_t r = M & ((1u << s) - 1u);
        uint32_t half = 1u << (s - 1);
        if (r > half || (r == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t h = sign | ((uint32_t)e << 10) | (man >> 13);
    uint32_t r = man & 0x1fffu;
    if (r > 0x1000u || (r == 0x1000u && (h & 1u))) h++; /* carry may reach inf */
    return (uint16_t)h;
}

static inline float block_scale(const uint8_t *blk) {
    return orc_f16_to_f32((uint16_t)(blk[0] | (blk[1] << 8)));
}

/* Rust `f32 as i8`: saturating, NaN -> 0. */
static inline int8_t f32_as_i8(float v) {
    if (v != v) return 0;
    if (v >= 127.0f) return 127;
    if (v <= -128.0f) return -128;
    return (int8_t)v; /* truncation toward zero, as `as` does */
}

/* Key whose unsigned order is f32::total_cmp's order. */
static inline uint32_t total_key(float v) {
    uint32_t b;
    memcpy(&b, &v, 4);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

/* ---- src/math.rs ----------------------------------------------------------- */

/* src/math.rs:7-15 */
float orc_dot_prod_f32(const float *a, const float *b, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) sum += a[i] * b[i];
    return sum;
}

/* src/math.rs:18-36: per block, a sequential 32-term sum of x*(i8 as f32),
 * then `sum += block_sum * f32(scale)`. */
float orc_dot_prod_q8(const float *a, const uint8_t *b, size_t k) {
    float sum = 0.0f;
    for (size_t blk = 0; blk < k / 32; blk++) {
        const uint8_t *bb = b + blk * 34;
        const float *ab = a + blk * 32;
        float scale = block_scale(bb);
        float block_sum = RUST_SUM_INIT;
        for (int i = 0; i < 32; i++) block_sum += ab[i] * (float)(int8_t)bb[2 + i];
        sum += block_sum * scale;
    }
    return sum;
}

/* src/math.rs:39-50 */
float orc_dot_prod_act_q8(const uint8_t *a, const uint8_t *b, size_t k) {
    float total = RUST_SUM_INIT;
    for (size_t blk = 0; blk < k / 32; blk++) {
        const uint8_t *ab = a + blk * 34;
        const uint8_t *bb = b + blk * 34;
        float scale_a = block_scale(ab);
        float scale_b = block_scale(bb);
        float block_sum = RUST_SUM_INIT;
        for (int i = 0; i < 32; i++)
            block_sum += (float)(int8_t)ab[2 + i] * (float)(int8_t)bb[2 + i];
        total += block_sum * scale_a * scale_b;
    }
    return total;
}

/* orc_dot_prod_q8 of eight consecutive rows at once: each row's sums take the
 * same operations in the same order as orc_dot_prod_q8's (the eight chains
 * are independent, so they only overlap in time). */
static void dot_prod_q8_x8(const float *a, const uint8_t *b, size_t row_bytes, size_t k, float *out) {
    float sum[8], block_sum[8], scale[8];
    for (int r = 0; r < 8; r++) sum[r] = 0.0f;
    for (size_t blk = 0; blk < k / 32; blk++) {
        const float *ab = a + blk * 32;
        for (int r = 0; r < 8; r++) {
            scale[r] = block_scale(b + r * row_bytes + blk * 34);
            block_sum[r] = RUST_SUM_INIT;
        }
        float qf[32][8]; /* the block's weights, row-interleaved */
        for (int r = 0; r < 8; r++)
            for (int i = 0; i < 32; i++) qf[i][r] = (float)(int8_t)b[r * row_bytes + blk * 34 + 2 + i];
        for (int i = 0; i < 32; i++)
            for (int r = 0; r < 8; r++) block_sum[r] += ab[i] * qf[i][r];
        for (int r = 0; r < 8; r++) sum[r] += block_sum[r] * scale[r];
    }
    for (int r = 0; r < 8; r++) out[r] = sum[r];
}

/* src/math.rs:87-98: 64-row chunks in parallel; each row is one sequential
 * dot, so the result does not depend on the thread count. */
void orc_q8_matmul(const float *a, const uint8_t *b, float *out, size_t n, size_t k) {
    size_t row_bytes = k / 32 * 34;
    int nt = orc_get_threads();
    (void)nt;
    if (g_fast) {
        long n8 = (long)(n / 8);
#pragma omp parallel for schedule(static, 8) num_threads(nt)
        for (long g = 0; g < n8; g++) dot_prod_q8_x8(a, b + (size_t)g * 8 * row_bytes, row_bytes, k, out + g * 8);
        for (size_t r = (size_t)n8 * 8; r < n; r++) out[r] = orc_dot_prod_q8(a, b + r * row_bytes, k);
        return;
    }
#pragma omp parallel for schedule(static, 64) num_threads(nt)
    for (long r = 0; r < (long)n; r++) out[r] = orc_dot_prod_q8(a, b + (size_t)r * row_bytes, k);
}

/* src/math.rs:101-112 */
void orc_q8_act_matmul(const uint8_t *a, const uint8_t *b, float *out, size_t n, size_t k) {
    size_t row_bytes = k / 32 * 34;
    int nt = orc_get_threads();
    (void)nt;
#pragma omp parallel for schedule(static, 64) num_threads(nt)
    for (long r = 0; r < (long)n; r++) out[r] = orc_dot_prod_act_q8(a, b + (size_t)r * row_bytes, k);
}

/* src/kernels.rs:8-31: the scale is the signed element of largest |x| (ties:
 * the later element) divided by 127; the stored scale is f16(scale) but the
 * quantisation divides by the f32 scale; q = round-half-away, saturating. */
void orc_activated_q8(const float *x, size_t k, uint8_t *out) {
    for (size_t blk = 0; blk < k / 32; blk++) {
        const float *pre = x + blk * 32;
        uint8_t *post = out + blk * 34;
        size_t best = 0;
        for (size_t i = 1; i < 32; i++)
            if (!(total_key(fabsf(pre[best])) > total_key(fabsf(pre[i])))) best = i;
        float scale = pre[best] / 127.0f;
        uint16_t h = orc_f32_to_f16(scale);
        post[0] = (uint8_t)(h & 0xff);
        post[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 32; i++) post[2 + i] = (uint8_t)f32_as_i8(roundf(pre[i] / scale));
    }
}

/* src/math.rs:117-137 (and src/reader.rs:285-299 convert_q8) */
void orc_q8_dequant(const uint8_t *blocks, size_t n_blocks, float *out) {
    for (size_t blk = 0; blk < n_blocks; blk++) {
        const uint8_t *bb = blocks + blk * 34;
        float scale = block_scale(bb);
        for (int i = 0; i < 32; i++) out[blk * 32 + i] = (float)(int8_t)bb[2 + i] * scale;
    }
}

/* src/math.rs:141-150 */
void orc_rmsnorm(const float *a, const float *w, float *out, size_t n) {
    float total = RUST_SUM_INIT;
    for (size_t i = 0; i < n; i++) total += a[i] * a[i];
    float rms_value = sqrtf((total / (float)n) + 1e-5f);
    for (size_t i = 0; i < n; i++) out[i] = (a[i] * w[i]) / rms_value;
}

/* src/math.rs:153-161 */
void orc_softmax(const float *x, float *out, size_t n) {
    if (n == 0) return; /* the reference unwraps (panics) on empty input */
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (!(total_key(x[best]) > total_key(x[i]))) best = i;
    float max = x[best];
    for (size_t i = 0; i < n; i++) out[i] = expf(x[i] - max);
    float total = RUST_SUM_INIT;
    for (size_t i = 0; i < n; i++) total += out[i];
    for (size_t i = 0; i < n; i++) out[i] = out[i] / total;
}

/* src/math.rs:164-178 */
void orc_swiglu(const float *x, const uint8_t *w_gate, const uint8_t *w_up,
                const uint8_t *w_down, float *out, size_t k, size_t f) {
    float *gate = (float *)malloc(f * sizeof(float));
    float *up = (float *)malloc(f * sizeof(float));
    float *hidden = (float *)malloc(f * sizeof(float));
    orc_q8_matmul(x, w_gate, gate, f, k);
    orc_q8_matmul(x, w_up, up, f, k);
    for (size_t i = 0; i < f; i++) hidden[i] = (gate[i] / (1.0f + expf(-gate[i]))) * up[i];
    orc_q8_matmul(hidden, w_down, out, k, f);
    free(gate);
    free(up);
    free(hidden);
}

/* src/math.rs:181-193 */
void orc_rope_angles(float base, size_t pos, size_t dim, float *out) {
    for (size_t i = 0; i < dim / 2; i++) {
        float frequency = powf(base, (-2.0f * (float)i) / (float)dim);
        out[i] = (float)pos * frequency;
    }
}

static void rope_chunks(float *v, size_t n, const float *thetas, size_t dim) {
    for (size_t c = 0; c + dim <= n; c += dim) {
        for (size_t i = 0; i < dim / 2; i++) {
            float angle = thetas[i];
            float *p = v + c + 2 * i;
            float e0 = cosf(angle) * p[0] + -sinf(angle) * p[1];
            float e1 = sinf(angle) * p[0] + cosf(angle) * p[1];
            p[0] = e0;
            p[1] = e1;
        }
    }
}

/* src/math.rs:196-228: adjacent pairs (2i, 2i+1) of every dim-wide head. */
void orc_rope(float *q, size_t nq, float *k, size_t nk, const float *thetas, size_t dim) {
    rope_chunks(q, nq, thetas, dim);
    rope_chunks(k, nk, thetas, dim);
}

/* ---- src/tokenizer.rs ------------------------------------------------------ */

/* src/tokenizer.rs:10-32 */
void orc_embed(size_t id, const uint8_t *embed_tensor, size_t dim, float *out) {
    size_t row_bytes = dim + dim / 32 * 2;
    orc_q8_dequant(embed_tensor + row_bytes * id, dim / 32, out);
}

/* src/tokenizer.rs:152-167 */
size_t orc_sample(const float *logits, size_t n) {
    if (n == 0) return 0;
    size_t best = 0;
    for (size_t i = 1; i < n; i++)
        if (!(total_key(logits[best]) > total_key(logits[i]))) best = i;
    return best;
}

/* ---- src/data.rs Cache ----------------------------------------------------- */

struct orc_cache {
    float *key_cache, *value_cache;
    size_t len, cap;
};

orc_cache *orc_cache_new(void) { return (orc_cache *)calloc(1, sizeof(orc_cache)); }

void orc_cache_free(orc_cache *c) {
    if (!c) return;
    free(c->key_cache);
    free(c->value_cache);
    free(c);
}

size_t orc_cache_len(const orc_cache *c) { return c->len; }

static void cache_extend(orc_cache *c, const float *k, const float *v, size_t n) {
    if (c->len + n > c->cap) {
        size_t cap = c->cap ? c->cap * 2 : 4096;
        while (cap < c->len + n) cap *= 2;
        c->key_cache = (float *)realloc(c->key_cache, cap * sizeof(float));
        c->value_cache = (float *)realloc(c->value_cache, cap * sizeof(float));
        c->cap = cap;
    }
    memcpy(c->key_cache + c->len, k, n * sizeof(float));
    memcpy(c->value_cache + c->len, v, n * sizeof(float));
    c->len += n;
}

/* ---- src/forward.rs -------------------------------------------------------- */

/* src/forward.rs:261-275 matmul: Normal -> q8_matmul; Quantize ->
 * activated_q8 then q8_act_matmul. */
static void mode_matmul(const orc_dims *d, const float *act, const uint8_t *w, float *out,
                        size_t n, size_t k) {
    if (d->mode == 1) {
        uint8_t *quantized = (uint8_t *)calloc(k / 32 * 34, 1);
        orc_activated_q8(act, k, quantized);
        orc_q8_act_matmul(quantized, w, out, n, k);
        free(quantized);
    } else {
        orc_q8_matmul(act, w, out, n, k);
    }
}

#define TENSOR(i) ((const uint8_t *)T[(i)])
#define LAYER_T(l, j) ((const uint8_t *)T[3 + ORC_LAYER_TENSORS * (l) + (j)])

/* src/forward.rs:13-258 */
int orc_forward(const orc_dims *d, const void *const *T, orc_cache *cache,
                const float *token_in, size_t pos, const float *angles,
                float *logits, float *dump) {
    const size_t H = (size_t)d->embed_dim, L = (size_t)d->n_layers;
    const size_t hd = (size_t)d->head_dim, nq = (size_t)d->q_heads, nkv = (size_t)d->kv_heads;
    const size_t KVD = nkv * hd, F = (size_t)d->ffn_dim, V = (size_t)d->vocab;
    const size_t group = nq / nkv;
    if (cache->len != pos * L * KVD) return -1;

    float *token = (float *)malloc(H * sizeof(float));
    float *o = (float *)malloc(H * sizeof(float));
    float *query = (float *)malloc(H * sizeof(float));
    float *key = (float *)malloc(KVD * sizeof(float));
    float *value = (float *)malloc(KVD * sizeof(float));
    float *weighted_values = (float *)malloc(H * sizeof(float));
    float *f_out = (float *)malloc(H * sizeof(float));
    float *activated = (float *)malloc(H * sizeof(float));
    float *scores = (float *)malloc((pos + 1) * sizeof(float));
    float *probs = (float *)malloc((pos + 1) * sizeof(float));
    memcpy(token, token_in, H * sizeof(float));
    if (dump) memcpy(dump, token, H * sizeof(float));

    for (size_t l = 0; l < L; l++) {
        /* :31-36 attention rmsnorm */
        orc_rmsnorm(token, (const float *)LAYER_T(l, 0), o, H);
        /* :41-58 q, k, v */
        mode_matmul(d, o, LAYER_T(l, 1), query, H, H);
        mode_matmul(d, o, LAYER_T(l, 2), key, KVD, H);
        mode_matmul(d, o, LAYER_T(l, 3), value, KVD, H);
        /* :71 rope */
        orc_rope(query, H, key, KVD, angles, hd);
        /* :83-84 append to the cache */
        cache_extend(cache, key, value, KVD);

        /* :86-174 grouped-query attention over positions pos, pos-1, ..., 0;
         * query head h uses kv head h / group.  Heads are independent: in
         * fast mode they run in parallel, each on its own score buffers. */
        float sq = sqrtf((float)hd);
        int nt_attn = g_fast ? orc_get_threads() : 1;
        (void)nt_attn;
#pragma omp parallel for schedule(dynamic, 1) num_threads(nt_attn)
        for (long hl = 0; hl < (long)nq; hl++) {
            size_t h = (size_t)hl, g = h / group;
            float *sc = g_fast ? (float *)malloc((pos + 1) * sizeof(float)) : scores;
            float *pr = g_fast ? (float *)malloc((pos + 1) * sizeof(float)) : probs;
            const float *qv = query + h * hd;
            for (size_t j = 0; j <= pos; j++) {
                size_t t = pos - j;
                const float *kv = cache->key_cache + t * L * KVD + l * KVD + g * hd;
                sc[j] = orc_dot_prod_f32(qv, kv, hd) / sq;
            }
            orc_softmax(sc, pr, pos + 1);
            float *w = weighted_values + h * hd;
            for (size_t e = 0; e < hd; e++) w[e] = 0.0f;
            for (size_t j = 0; j <= pos; j++) {
                size_t t = pos - j;
                const float *vv = cache->value_cache + t * L * KVD + l * KVD + g * hd;
                for (size_t e = 0; e < hd; e++) w[e] = w[e] + vv[e] * pr[j];
            }
            if (g_fast) {
                free(sc);
                free(pr);
            }
        }

        if (g_attn_dump) memcpy(g_attn_dump + l * H, weighted_values, H * sizeof(float));
        /* :176-192 output projection and residual */
        mode_matmul(d, weighted_values, LAYER_T(l, 4), f_out, H, H);
        for (size_t i = 0; i < H; i++) token[i] = token[i] + f_out[i];

        /* :194-236 ffn rmsnorm, SwiGLU (always the f32 path), residual */
        orc_rmsnorm(token, (const float *)LAYER_T(l, 5), o, H);
        orc_swiglu(o, LAYER_T(l, 6), LAYER_T(l, 7), LAYER_T(l, 8), activated, H, F);
        for (size_t i = 0; i < H; i++) token[i] = token[i] + activated[i];
        if (dump) memcpy(dump + (l + 1) * H, token, H * sizeof(float));
    }

    /* :241-252 final norm and classifier */
    orc_rmsnorm(token, (const float *)TENSOR(1), o, H);
    mode_matmul(d, o, TENSOR(2), logits, V, H);

    free(token); free(o); free(query); free(key); free(value);
    free(weighted_values); free(f_out); free(activated); free(scores); free(probs);
    return 0;
}

/* src/lib.rs:239-314 generate_capped, by token id. */
int orc_generate_capped(const orc_dims *d, const void *const *T,
                        const int32_t *prompt, size_t n_prompt, size_t cap,
                        int32_t *out_ids, float *last_logits) {
    const size_t H = (size_t)d->embed_dim, V = (size_t)d->vocab, hd = (size_t)d->head_dim;
    orc_cache *cache = orc_cache_new();
    float *embedded = (float *)malloc(H * sizeof(float));
    float *angles = (float *)malloc(hd / 2 * sizeof(float));
    float *logits = (float *)malloc(V * sizeof(float));
    size_t n_logits = 0; /* `let mut logits = vec![]` */
    size_t pos = 0;
    int rc = 0;
    for (size_t i = 0; i < n_prompt && rc == 0; i++) {
        orc_embed((size_t)prompt[i], TENSOR(0), H, embedded);
        orc_rope_angles(d->base_freq, pos, hd, angles);
        rc = orc_forward(d, T, cache, embedded, pos, angles, logits, NULL);
        n_logits = V;
        pos++;
    }
    size_t n_out = 0;
    while (rc == 0 && n_out < cap) {
        size_t id = orc_sample(logits, n_logits);
        out_ids[n_out++] = (int32_t)id;
        orc_embed(id, TENSOR(0), H, embedded);
        orc_rope_angles(d->base_freq, pos, hd, angles);
        rc = orc_forward(d, T, cache, embedded, pos, angles, logits, NULL);
        n_logits = V;
        pos++;
    }
    if (last_logits && n_logits) memcpy(last_logits, logits, V * sizeof(float));
    free(embedded); free(angles); free(logits);
    orc_cache_free(cache);
    return rc;
}
