/*
 * CPU ORACLE — test infrastructure only.
 *
 * A plain-C restatement of the reference CPU path of convo-lang/defer
 * (a pure-Rust crate), used as the checker for the B200 product path.
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may
 * load this library; the product (defer_b200/) never links or calls it.
 *
 * Arithmetic follows the reference exactly: every reduction is one
 * accumulator walked in index order, `a * b + c` is never contracted
 * (compile with -ffp-contract=off, no -ffast-math), transcendental
 * functions come from the platform libm (expf/cosf/sinf/tanhf/pow), which
 * is what Rust's std calls on Linux.
 *
 * Parity status: the reference cannot be compiled in this environment
 * (no cargo/rustc, no vendored rand crates), so this restatement is pinned
 * against the reference's own known-answer unit tests (ops.rs:189-252,
 * sampler.rs:116-162, safetensors.rs:305-313, crc32.rs:33-35) and the
 * ChaCha block function against an independent ChaCha20 implementation and
 * the published ChaCha8 test vector. Forward-pass bits against the real
 * Rust binary are unpinned.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FP_FAST_FMAF) || defined(__FAST_MATH__)
#error "oracle must be compiled without fast-math / FMA contraction"
#endif

#define OR_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------ ops.rs */

/* ops.rs:9-22 */
OR_EXPORT void or_matmul_sequential(float *out, const float *a, const float *b, size_t m, size_t n, size_t k) {
    for (size_t i = 0; i < m; i++)
        for (size_t j = 0; j < n; j++) {
            float sum = 0.0f;
            for (size_t p = 0; p < k; p++) sum += a[i * k + p] * b[p * n + j];
            out[i * n + j] = sum;
        }
}

/* ops.rs:26-71 — four independent rows per pass, one accumulator per row in
 * index order, bias added after the sum. */
OR_EXPORT void or_linear(float *out, const float *x, const float *w, const float *bias, size_t in_dim,
                         size_t out_dim) {
    size_t blocks = out_dim / 4;
    for (size_t blk = 0; blk < blocks; blk++) {
        size_t o = blk * 4;
        const float *r0 = w + o * in_dim;
        const float *r1 = r0 + in_dim;
        const float *r2 = r1 + in_dim;
        const float *r3 = r2 + in_dim;
        float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
        for (size_t i = 0; i < in_dim; i++) {
            float xi = x[i];
            s0 += r0[i] * xi;
            s1 += r1[i] * xi;
            s2 += r2[i] * xi;
            s3 += r3[i] * xi;
        }
        if (bias) {
            s0 += bias[o];
            s1 += bias[o + 1];
            s2 += bias[o + 2];
            s3 += bias[o + 3];
        }
        out[o] = s0;
        out[o + 1] = s1;
        out[o + 2] = s2;
        out[o + 3] = s3;
    }
    for (size_t o = blocks * 4; o < out_dim; o++) {
        const float *row = w + o * in_dim;
        float sum = 0.0f;
        for (size_t i = 0; i < in_dim; i++) sum += row[i] * x[i];
        if (bias) sum += bias[o];
        out[o] = sum;
    }
}

/* ops.rs:74-81 */
OR_EXPORT float or_dot(const float *a, const float *b, size_t n) {
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) sum += a[i] * b[i];
    return sum;
}

/* ops.rs:84-95 — out = (x * inv) * w */
OR_EXPORT void or_rmsnorm(float *out, const float *x, const float *w, size_t n, float eps) {
    float ss = 0.0f;
    for (size_t i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (size_t i = 0; i < n; i++) out[i] = x[i] * inv * w[i];
}

/* ops.rs:98-118 */
OR_EXPORT void or_layernorm(float *out, const float *x, const float *w, const float *b, size_t len, float eps) {
    float n = (float)len;
    float mean = 0.0f;
    for (size_t i = 0; i < len; i++) mean += x[i];
    mean /= n;
    float var = 0.0f;
    for (size_t i = 0; i < len; i++) {
        float d = x[i] - mean;
        var += d * d;
    }
    var /= n;
    float inv = 1.0f / sqrtf(var + eps);
    for (size_t i = 0; i < len; i++) out[i] = (x[i] - mean) * inv * w[i] + b[i];
}

/* ops.rs:120-122 */
OR_EXPORT float or_silu(float x) { return x / (1.0f + expf(-x)); }

/* ops.rs:125-128 */
OR_EXPORT float or_gelu(float x) {
    const float C = 0.7978846f; /* sqrt(2/pi) as written in the reference */
    return 0.5f * x * (1.0f + tanhf(C * (x + 0.044715f * x * x * x)));
}

/* ops.rs:159-178 */
OR_EXPORT void or_softmax_inplace(float *x, size_t n) {
    if (n == 0) return;
    float max = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if (x[i] > max) max = x[i];
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        x[i] = expf(x[i] - max);
        sum += x[i];
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) x[i] *= inv;
}

/* ------------------------------------------------------- ChaCha8 (rand_*) */
/*
 * Third-party arithmetic restated from published algorithms (not vendored in
 * the reference): rand_chacha 0.3.1 ChaCha8Rng (DJB ChaCha, 8 rounds, 64-bit
 * block counter in state words 12-13 starting at 0, stream id 0 in words
 * 14-15, keystream consumed as little-endian u32 words in order);
 * rand_core 0.6.4 SeedableRng::seed_from_u64 (PCG32 output function filling
 * the 32-byte seed 4 bytes at a time); rand 0.8 Standard f32 (one u32,
 * top 24 bits times 2^-24) and UniformFloat::sample_single for f32.
 * Call sites: engine.rs:19-21, engine.rs:51, sampler.rs:92, synthetic.rs:33-35.
 */
#define ROTL(v, n) (((v) << (n)) | ((v) >> (32 - (n))))
#define QR(a, b, c, d)                                                                                            \
    a += b; d ^= a; d = ROTL(d, 16);                                                                              \
    c += d; b ^= c; b = ROTL(b, 12);                                                                              \
    a += b; d ^= a; d = ROTL(d, 8);                                                                               \
    c += d; b ^= c; b = ROTL(b, 7);

OR_EXPORT void or_chacha_block(const uint32_t in[16], uint32_t out[16], int rounds) {
    uint32_t x[16];
    memcpy(x, in, sizeof(x));
    for (int i = 0; i < rounds; i += 2) {
        QR(x[0], x[4], x[8], x[12]);
        QR(x[1], x[5], x[9], x[13]);
        QR(x[2], x[6], x[10], x[14]);
        QR(x[3], x[7], x[11], x[15]);
        QR(x[0], x[5], x[10], x[15]);
        QR(x[1], x[6], x[11], x[12]);
        QR(x[2], x[7], x[8], x[13]);
        QR(x[3], x[4], x[9], x[14]);
    }
    for (int i = 0; i < 16; i++) out[i] = x[i] + in[i];
}

typedef struct {
    uint32_t key[8];
    uint64_t word_pos; /* words consumed so far (ChaCha8Rng::get_word_pos) */
    uint64_t buf_block; /* block index held in buf, or UINT64_MAX */
    uint32_t buf[16];
} or_chacha;

OR_EXPORT size_t or_chacha_sizeof(void) { return sizeof(or_chacha); }

OR_EXPORT void or_chacha_init(or_chacha *c, const uint8_t seed[32]) {
    for (int i = 0; i < 8; i++)
        c->key[i] = (uint32_t)seed[4 * i] | ((uint32_t)seed[4 * i + 1] << 8) | ((uint32_t)seed[4 * i + 2] << 16) |
                    ((uint32_t)seed[4 * i + 3] << 24);
    c->word_pos = 0;
    c->buf_block = UINT64_MAX;
}

static void chacha_fill(or_chacha *c, uint64_t block) {
    uint32_t st[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u};
    memcpy(st + 4, c->key, 32);
    st[12] = (uint32_t)block;
    st[13] = (uint32_t)(block >> 32);
    st[14] = 0;
    st[15] = 0;
    or_chacha_block(st, c->buf, 8);
    c->buf_block = block;
}

OR_EXPORT uint32_t or_chacha_next_u32(or_chacha *c) {
    uint64_t block = c->word_pos / 16;
    if (c->buf_block != block) chacha_fill(c, block);
    uint32_t v = c->buf[c->word_pos % 16];
    c->word_pos++;
    return v;
}

OR_EXPORT uint64_t or_chacha_word_pos(const or_chacha *c) { return c->word_pos; }

/* rand 0.8 `Standard` for f32: 24 high bits scaled by 2^-24 (sampler.rs:92). */
OR_EXPORT float or_u32_to_unit_f32(uint32_t v) { return (float)(v >> 8) * (1.0f / 16777216.0f); }

OR_EXPORT float or_chacha_gen_f32(or_chacha *c) { return or_u32_to_unit_f32(or_chacha_next_u32(c)); }

/* rand 0.8 UniformFloat<f32>::sample_single (synthetic.rs:34). */
OR_EXPORT float or_chacha_gen_range_f32(or_chacha *c, float low, float high) {
    float scale = high - low;
    for (;;) {
        uint32_t bits = (or_chacha_next_u32(c) >> 9) | 0x3F800000u;
        float v12;
        memcpy(&v12, &bits, 4);
        float v01 = v12 - 1.0f;
        float res = v01 * scale + low;
        if (res < high) return res;
        uint32_t sb;
        memcpy(&sb, &scale, 4);
        sb -= 1;
        memcpy(&scale, &sb, 4);
    }
}

/* rand_core 0.6.4 SeedableRng::seed_from_u64 (engine.rs:19-21). */
OR_EXPORT void or_seed_from_u64(uint64_t state, uint8_t out[32]) {
    const uint64_t MUL = 6364136223846793005ull;
    const uint64_t INC = 11634580027462260723ull;
    for (int i = 0; i < 8; i++) {
        state = state * MUL + INC;
        uint64_t s = state;
        uint32_t xorshifted = (uint32_t)(((s >> 18) ^ s) >> 27);
        uint32_t rot = (uint32_t)(s >> 59);
        uint32_t x = (xorshifted >> rot) | (xorshifted << ((32 - rot) & 31));
        out[4 * i] = (uint8_t)x;
        out[4 * i + 1] = (uint8_t)(x >> 8);
        out[4 * i + 2] = (uint8_t)(x >> 16);
        out[4 * i + 3] = (uint8_t)(x >> 24);
    }
}

/* -------------------------------------------------------------- sampler.rs */

/* sampler.rs:24-40 — strict `>`, NaN skipped, lowest index wins. */
OR_EXPORT size_t or_argmax(const float *l, size_t n) {
    size_t best = 0;
    float best_val = -INFINITY;
    int found = 0;
    for (size_t i = 0; i < n; i++) {
        float v = l[i];
        if (isnan(v)) continue;
        if (!found || v > best_val) {
            best = i;
            best_val = v;
            found = 1;
        }
    }
    return best;
}

/* sampler.rs:43-75 */
OR_EXPORT void or_softmax_with_temperature(const float *logits, size_t n, float t, float *probs) {
    float max = -INFINITY;
    for (size_t i = 0; i < n; i++) {
        float s = logits[i] / t;
        if (s > max) max = s;
    }
    float sum = 0.0f;
    for (size_t i = 0; i < n; i++) {
        float s = logits[i] / t;
        float p = isnan(s) ? 0.0f : expf(s - max);
        probs[i] = p;
        sum += p;
    }
    if (!(sum > 0.0f) || !isfinite(sum)) {
        size_t best = or_argmax(logits, n);
        for (size_t i = 0; i < n; i++) probs[i] = 0.0f;
        if (n) probs[best] = 1.0f;
        return;
    }
    float inv = 1.0f / sum;
    for (size_t i = 0; i < n; i++) probs[i] *= inv;
}

/* sampler.rs:94-108 — CDF scan with an already drawn r. */
OR_EXPORT size_t or_cdf_scan(const float *probs, size_t n, float r) {
    float cumulative = 0.0f;
    size_t last_nonzero = 0;
    for (size_t i = 0; i < n; i++) {
        float p = probs[i];
        if (p > 0.0f) {
            last_nonzero = i;
            cumulative += p;
            if (r < cumulative) return i;
        }
    }
    return last_nonzero;
}

/* sampler.rs:78-109 with the PRNG word passed in (temperature > 0 draws
 * exactly one word; temperature == 0 ignores it). `probs` is scratch of n. */
OR_EXPORT size_t or_sample_token_word(const float *logits, size_t n, float t, uint32_t word, float *probs) {
    if (t == 0.0f) return or_argmax(logits, n);
    or_softmax_with_temperature(logits, n, t, probs);
    return or_cdf_scan(probs, n, or_u32_to_unit_f32(word));
}

/* ---------------------------------------------------------------- model.rs */

typedef struct {
    const float *attn_norm, *wq, *bq, *wk, *bk, *wv, *bv, *wo, *ffn_norm, *w_gate, *w_up, *w_down;
} or_layer;

typedef struct {
    size_t vocab, hidden, inter, layers, heads, kv_heads, head_dim, max_seq;
    float eps, theta;
    int gelu;
    const float *embed, *norm, *lm_head; /* lm_head NULL when tied */
    or_layer *layer;
    float *inv_freq;
} or_model;

typedef struct {
    size_t kv_dim, layers, len, cap;
    float **keys, **values;
} or_cache;

/* model.rs:301-363 (the tensors are already converted to f32 by the loader;
 * inv_freq in f64 then rounded to f32, model.rs:348-353). */
OR_EXPORT or_model *or_model_new(size_t vocab, size_t hidden, size_t inter, size_t layers, size_t heads,
                                 size_t kv_heads, size_t head_dim, size_t max_seq, float eps, float theta, int gelu) {
    or_model *m = (or_model *)calloc(1, sizeof(or_model));
    m->vocab = vocab;
    m->hidden = hidden;
    m->inter = inter;
    m->layers = layers;
    m->heads = heads;
    m->kv_heads = kv_heads;
    m->head_dim = head_dim;
    m->max_seq = max_seq;
    m->eps = eps;
    m->theta = theta;
    m->gelu = gelu;
    m->layer = (or_layer *)calloc(layers ? layers : 1, sizeof(or_layer));
    size_t half = head_dim / 2;
    m->inv_freq = (float *)calloc(half ? half : 1, sizeof(float));
    for (size_t i = 0; i < half; i++) {
        double exponent = (double)(2 * i) / (double)head_dim;
        m->inv_freq[i] = (float)(1.0 / pow((double)theta, exponent));
    }
    return m;
}

OR_EXPORT void or_model_set_globals(or_model *m, const float *embed, const float *norm, const float *lm_head) {
    m->embed = embed;
    m->norm = norm;
    m->lm_head = lm_head;
}

OR_EXPORT void or_model_set_layer(or_model *m, size_t l, const float *attn_norm, const float *wq, const float *bq,
                                  const float *wk, const float *bk, const float *wv, const float *bv, const float *wo,
                                  const float *ffn_norm, const float *w_gate, const float *w_up, const float *w_down) {
    or_layer *L = &m->layer[l];
    L->attn_norm = attn_norm;
    L->wq = wq;
    L->bq = bq;
    L->wk = wk;
    L->bk = bk;
    L->wv = wv;
    L->bv = bv;
    L->wo = wo;
    L->ffn_norm = ffn_norm;
    L->w_gate = w_gate;
    L->w_up = w_up;
    L->w_down = w_down;
}

OR_EXPORT void or_model_free(or_model *m) {
    if (!m) return;
    free(m->layer);
    free(m->inv_freq);
    free(m);
}

OR_EXPORT const float *or_model_inv_freq(const or_model *m) { return m->inv_freq; }

/* model.rs:184-243 — append-only cache, keys[l] is [len, kv_dim]. */
OR_EXPORT or_cache *or_cache_new(const or_model *m, size_t cap) {
    or_cache *c = (or_cache *)calloc(1, sizeof(or_cache));
    c->kv_dim = m->kv_heads * m->head_dim;
    c->layers = m->layers;
    c->cap = cap;
    c->keys = (float **)calloc(m->layers ? m->layers : 1, sizeof(float *));
    c->values = (float **)calloc(m->layers ? m->layers : 1, sizeof(float *));
    for (size_t l = 0; l < m->layers; l++) {
        c->keys[l] = (float *)calloc(cap * c->kv_dim + 1, sizeof(float));
        c->values[l] = (float *)calloc(cap * c->kv_dim + 1, sizeof(float));
    }
    return c;
}

OR_EXPORT void or_cache_free(or_cache *c) {
    if (!c) return;
    for (size_t l = 0; l < c->layers; l++) {
        free(c->keys[l]);
        free(c->values[l]);
    }
    free(c->keys);
    free(c->values);
    free(c);
}

OR_EXPORT size_t or_cache_len(const or_cache *c) { return c->len; }
OR_EXPORT size_t or_cache_cap(const or_cache *c) { return c->cap; }
OR_EXPORT const float *or_cache_keys(const or_cache *c, size_t l) { return c->keys[l]; }
OR_EXPORT const float *or_cache_values(const or_cache *c, size_t l) { return c->values[l]; }

/* model.rs:211-220 */
OR_EXPORT void or_cache_truncate(or_cache *c, size_t n) {
    if (n < c->len) c->len = n;
}

/* Timing samples only (bench.py's CPU legs): sets the length to n <= cap
 * without computing the rows in between, which keep what they hold (zeros
 * in a new cache). The CPU cost of a forward at position p does not depend
 * on the cached values, so a forward at any position of a workload can be
 * timed without first running every position before it. */
OR_EXPORT void or_cache_set_len(or_cache *c, size_t n) {
    if (n <= c->cap) c->len = n;
}

/* KvCache::clone (attribution.rs:254). */
OR_EXPORT void or_cache_copy(or_cache *dst, const or_cache *src) {
    size_t n = src->len < dst->cap ? src->len : dst->cap;
    for (size_t l = 0; l < src->layers; l++) {
        memcpy(dst->keys[l], src->keys[l], n * src->kv_dim * sizeof(float));
        memcpy(dst->values[l], src->values[l], n * src->kv_dim * sizeof(float));
    }
    dst->len = n;
}

static void rope_apply(float *vec, size_t n_heads, size_t hd, const float *cs, const float *sn) {
    size_t half = hd / 2;
    for (size_t h = 0; h < n_heads; h++) {
        size_t base = h * hd;
        for (size_t i = 0; i < half; i++) {
            float x0 = vec[base + i];
            float x1 = vec[base + i + half];
            vec[base + i] = x0 * cs[i] - x1 * sn[i];
            vec[base + i + half] = x1 * cs[i] + x0 * sn[i];
        }
    }
}

/* The RoPE tables of one position exactly as model.rs:438-445 builds them. */
OR_EXPORT void or_rope_tables(const or_model *m, size_t pos, float *cs, float *sn) {
    size_t half = m->head_dim / 2;
    for (size_t i = 0; i < half; i++) {
        float angle = (float)pos * m->inv_freq[i];
        cs[i] = cosf(angle);
        sn[i] = sinf(angle);
    }
}

/*
 * model.rs:394-520 — one token at position cache.len(). Returns 0 on
 * success, 3 (Model error) on a bad token / exceeded context / full cache,
 * with a message in `err`.
 */
OR_EXPORT int or_forward(const or_model *m, or_cache *c, uint32_t token, const size_t *masked, size_t n_masked,
                         float *logits, char *err, size_t errlen) {
    size_t pos = c->len;
    if ((size_t)token >= m->vocab) {
        if (err) snprintf(err, errlen, "token id %u out of range", token);
        return 3;
    }
    if (pos >= m->max_seq) {
        if (err) snprintf(err, errlen, "context length %zu exceeded", m->max_seq);
        return 3;
    }
    if (pos >= c->cap) {
        if (err) snprintf(err, errlen, "oracle cache capacity %zu exceeded", c->cap);
        return 3;
    }
    size_t hd = m->head_dim, half = hd / 2;
    size_t group = m->heads / m->kv_heads;
    size_t kv_dim = m->kv_heads * hd, q_dim = m->heads * hd;
    float scale = 1.0f / sqrtf((float)hd);
    size_t H = m->hidden, FF = m->inter;

    unsigned char *skip = NULL;
    if (n_masked) {
        skip = (unsigned char *)calloc(pos + 1, 1);
        for (size_t i = 0; i < n_masked; i++)
            if (masked[i] < pos) skip[masked[i]] = 1;
    }

    float *x = (float *)malloc(H * sizeof(float));
    float *xb = (float *)calloc(H, sizeof(float));
    float *q = (float *)calloc(q_dim, sizeof(float));
    float *k = (float *)calloc(kv_dim, sizeof(float));
    float *v = (float *)calloc(kv_dim, sizeof(float));
    float *att = (float *)calloc(q_dim, sizeof(float));
    float *scores = (float *)calloc(pos + 1, sizeof(float));
    float *gate = (float *)calloc(FF, sizeof(float));
    float *up = (float *)calloc(FF, sizeof(float));
    float *cs = (float *)calloc(half ? half : 1, sizeof(float));
    float *sn = (float *)calloc(half ? half : 1, sizeof(float));
    memcpy(x, m->embed + (size_t)token * H, H * sizeof(float));
    or_rope_tables(m, pos, cs, sn);

    for (size_t l = 0; l < m->layers; l++) {
        const or_layer *L = &m->layer[l];
        or_rmsnorm(xb, x, L->attn_norm, H, m->eps);
        or_linear(q, xb, L->wq, L->bq, H, q_dim);
        or_linear(k, xb, L->wk, L->bk, H, kv_dim);
        or_linear(v, xb, L->wv, L->bv, H, kv_dim);
        rope_apply(q, m->heads, hd, cs, sn);
        rope_apply(k, m->kv_heads, hd, cs, sn);
        memcpy(c->keys[l] + pos * kv_dim, k, kv_dim * sizeof(float));
        memcpy(c->values[l] + pos * kv_dim, v, kv_dim * sizeof(float));
        const float *keys = c->keys[l], *vals = c->values[l];
        for (size_t h = 0; h < m->heads; h++) {
            size_t kvh = h / group;
            const float *qh = q + h * hd;
            for (size_t t = 0; t <= pos; t++) scores[t] = or_dot(qh, keys + t * kv_dim + kvh * hd, hd) * scale;
            if (skip)
                for (size_t t = 0; t < pos; t++)
                    if (skip[t]) scores[t] = -INFINITY;
            or_softmax_inplace(scores, pos + 1);
            float *out = att + h * hd;
            for (size_t d = 0; d < hd; d++) {
                float acc = 0.0f;
                for (size_t t = 0; t <= pos; t++) acc += scores[t] * vals[t * kv_dim + kvh * hd + d];
                out[d] = acc;
            }
        }
        or_linear(xb, att, L->wo, NULL, q_dim, H);
        for (size_t i = 0; i < H; i++) x[i] += xb[i];
        or_rmsnorm(xb, x, L->ffn_norm, H, m->eps);
        or_linear(gate, xb, L->w_gate, NULL, H, FF);
        or_linear(up, xb, L->w_up, NULL, H, FF);
        if (m->gelu)
            for (size_t i = 0; i < FF; i++) gate[i] = or_gelu(gate[i]);
        else
            for (size_t i = 0; i < FF; i++) gate[i] = or_silu(gate[i]);
        for (size_t i = 0; i < FF; i++) gate[i] *= up[i];
        or_linear(xb, gate, L->w_down, NULL, FF, H);
        for (size_t i = 0; i < H; i++) x[i] += xb[i];
    }
    c->len += 1;
    or_rmsnorm(xb, x, m->norm, H, m->eps);
    const float *head = m->lm_head ? m->lm_head : m->embed;
    or_linear(logits, xb, head, NULL, H, m->vocab);

    free(skip);
    free(x);
    free(xb);
    free(q);
    free(k);
    free(v);
    free(att);
    free(scores);
    free(gate);
    free(up);
    free(cs);
    free(sn);
    return 0;
}

/* ---------------------------------------------------------- attribution.rs */

/* attribution.rs:71-85 — log softmax at idx in f64, sequential. */
OR_EXPORT double or_log_softmax_at(const float *logits, size_t n, size_t idx) {
    double max = -INFINITY;
    for (size_t i = 0; i < n; i++)
        if ((double)logits[i] > max) max = (double)logits[i];
    double sum = 0.0;
    for (size_t i = 0; i < n; i++)
        if (!isnan(logits[i])) sum += exp((double)logits[i] - max);
    return ((double)logits[idx] - max) - log(sum);
}

/* ------------------------------------------------------------------ crc32 */

/* crc32.rs:4-28 — IEEE reflected CRC-32, poly 0xEDB88320. */
OR_EXPORT uint32_t or_crc32(const uint8_t *data, size_t n) {
    static uint32_t table[256];
    static int init = 0;
    if (!init) {
        for (uint32_t i = 0; i < 256; i++) {
            uint32_t c = i;
            for (int k = 0; k < 8; k++) c = (c & 1) ? (0xEDB88320u ^ (c >> 1)) : (c >> 1);
            table[i] = c;
        }
        init = 1;
    }
    uint32_t c = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; i++) c = table[(c ^ data[i]) & 0xFF] ^ (c >> 8);
    return c ^ 0xFFFFFFFFu;
}
