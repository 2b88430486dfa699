/* C oracle: a CPU restatement of the reference's PLaMo-3 token loop.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product library links or calls this
 * file; it is the checker that the CUDA path is compared against (tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference leg).
 *
 * The reference's CPU path is hand-written AArch64 assembly for Darwin
 * (reference src/ *.s files). It cannot be assembled or run on this x86-64 host, so
 * every function below restates one assembly routine operation for operation:
 * the same FP32 rounding points, the same fused multiply-adds (fmla/fmadd ->
 * fmaf) and the same summation order. It is compiled with -ffp-contract=off so
 * that the compiler adds no fusion of its own. Symbol names are the
 * reference's, which lets the reference's own known-answer tests
 * (reference tests/{math,activation,token,qkv,rope,cache,cache_rope,
 * rope_table,trig,attention,model,mixer,matmul,prefill,cache_rope_cached}.c)
 * be compiled unchanged against this file (see oracle/Makefile).
 *
 * Parity pin: those reference tests pass against this restatement (the
 * `make -C oracle ref-tests` recipe, run by tests/test_oracle_pins.py).
 */
#include "plamo_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

/* ---------------------------------------------------------------- helpers */

static inline float bf16(uint16_t bits) {
    uint32_t word = (uint32_t)bits << 16;
    float value;
    memcpy(&value, &word, 4);
    return value;
}

static inline uint32_t float_bits(float value) {
    uint32_t word;
    memcpy(&word, &value, 4);
    return word;
}

/* Row-split worker count for the timed CPU baseline. Each output row keeps
   its own accumulation order, so the result is independent of this value
   (the reference splits the same way: runtime/parallel.c:35-92). */
static int oracle_thread_count = 1;
void oracle_set_threads(int threads) {
    oracle_thread_count = threads > 0 ? threads : 1;
}
int oracle_threads(void) {
    return oracle_thread_count;
}

/* Row windows of the reference's weight provider (src/math.s:5-70). They
   bound I/O lifetimes and never change arithmetic; kept as a symbol because
   the reference's matmul test sets it. */
uint64_t plamo_weight_chunk_bytes = 0;

/* ----------------------------------------------------------- src/math.s */

/* One output row: four FMA lanes over columns c = j (mod 4), reduced as
   (l0 + l1) + (l2 + l3), then a scalar FMA tail (src/math.s:86-344; the 8-row,
   4-row and 1-row loops all keep this per-row order). */
static inline float matvec_row4(const uint16_t *w, const float *x, uint64_t cols) {
    float l0 = 0, l1 = 0, l2 = 0, l3 = 0;
    uint64_t body = cols & ~(uint64_t)3, c = 0;
    for (; c < body; c += 4) {
        l0 = fmaf(bf16(w[c]), x[c], l0);
        l1 = fmaf(bf16(w[c + 1]), x[c + 1], l1);
        l2 = fmaf(bf16(w[c + 2]), x[c + 2], l2);
        l3 = fmaf(bf16(w[c + 3]), x[c + 3], l3);
    }
    float s = (l0 + l1) + (l2 + l3);
    for (; c < cols; ++c)
        s = fmaf(bf16(w[c]), x[c], s);
    return s;
}

/* NOT the reference's order: eight FMA lanes reduced pairwise. Only for
   measuring how far an equally valid FP32 summation order moves a whole
   model's outputs (the spread a GPU's own order is held to in the
   whole-model fixtures); off unless oracle_set_matvec_lanes(8) is called. */
static inline float matvec_row8(const uint16_t *w, const float *x, uint64_t cols) {
    float l[8] = {0};
    uint64_t body = cols & ~(uint64_t)7, c = 0;
    for (; c < body; c += 8)
        for (int j = 0; j < 8; ++j)
            l[j] = fmaf(bf16(w[c + j]), x[c + j], l[j]);
    float s = ((l[0] + l[1]) + (l[2] + l[3])) + ((l[4] + l[5]) + (l[6] + l[7]));
    for (; c < cols; ++c)
        s = fmaf(bf16(w[c]), x[c], s);
    return s;
}

static int oracle_matvec_lanes = 4;
void oracle_set_matvec_lanes(int lanes) {
    oracle_matvec_lanes = lanes == 8 ? 8 : 4;
}

static inline float matvec_row(const uint16_t *w, const float *x, uint64_t cols) {
    return oracle_matvec_lanes == 8 ? matvec_row8(w, x, cols) : matvec_row4(w, x, cols);
}

struct matvec_job {
    const uint16_t *w;
    const float *x;
    float *y;
    uint64_t cols, group0, group1, rows;
};

static void *matvec_worker(void *argument) {
    const struct matvec_job *job = argument;
    for (uint64_t g = job->group0; g < job->group1; ++g) {
        uint64_t r0 = g * 24, r1 = r0 + 24 < job->rows ? r0 + 24 : job->rows;
        for (uint64_t r = r0; r < r1; ++r)
            job->y[r] = matvec_row(job->w + r * job->cols, job->x, job->cols);
    }
    return NULL;
}

void plamo_bf16_matvec_serial(const uint16_t *w, const float *x, float *y, uint64_t rows,
                              uint64_t cols) {
    if (oracle_thread_count > 1 && rows >= 48 && rows * cols >= (1u << 18)) {
        /* Contiguous ranges of 24-row groups, as runtime/parallel.c:35-48
           assigns them to workers. */
        enum { MAX_WORKERS = 256 };
        uint64_t groups = (rows + 23) / 24;
        uint64_t workers = (uint64_t)oracle_thread_count;
        if (workers > MAX_WORKERS)
            workers = MAX_WORKERS;
        if (workers > groups)
            workers = groups;
        struct matvec_job jobs[MAX_WORKERS];
        pthread_t threads[MAX_WORKERS];
        for (uint64_t i = 0; i < workers; ++i)
            jobs[i] = (struct matvec_job){w, x, y, cols, groups * i / workers,
                                          groups * (i + 1) / workers, rows};
        uint64_t started = 1;
        for (uint64_t i = 1; i < workers; ++i, ++started)
            if (pthread_create(&threads[i], NULL, matvec_worker, &jobs[i]))
                break;
        matvec_worker(&jobs[0]);
        for (uint64_t i = started; i < workers; ++i)
            matvec_worker(&jobs[i]);
        for (uint64_t i = 1; i < started; ++i)
            pthread_join(threads[i], NULL);
        return;
    }
    for (uint64_t r = 0; r < rows; ++r)
        y[r] = matvec_row(w + r * cols, x, cols);
}

void plamo_bf16_matvec_core(const uint16_t *w, const float *x, float *y, uint64_t rows,
                            uint64_t cols) {
    plamo_bf16_matvec_serial(w, x, y, rows, cols);
}

void plamo_bf16_matvec(const uint16_t *w, const float *x, float *y, uint64_t rows,
                       uint64_t cols) {
    plamo_bf16_matvec_serial(w, x, y, rows, cols);
}

/* Sequential FP32 sum of squares, 1/sqrt(mean + eps), then
   (x * inverse) * (w + offset) (src/math.s:349-397). In-place allowed. */
void plamo_rmsnorm(const float *x, const uint16_t *w, float *y, uint64_t n, float eps,
                   float offset) {
    if (!n)
        return;
    float sum = 0;
    for (uint64_t i = 0; i < n; ++i) {
        float square = x[i] * x[i];
        sum = sum + square;
    }
    sum = sum / (float)n;
    sum = sum + eps;
    sum = sqrtf(sum);
    float inverse = 1.0f / sum;
    for (uint64_t i = 0; i < n; ++i) {
        float scaled = x[i] * inverse;
        y[i] = scaled * (bf16(w[i]) + offset);
    }
}

/* ------------------------------------------------ src/matmul*.s (batched) */

/* Every batched kernel is bitwise equal to the per-token matvec
   (reference tests/matmul.c:20-77 checks exactly that), so the restatement is
   the per-token matvec with the descriptor's strides. */
void plamo_bf16_matmul_core(const struct plamo_matmul *m) {
    for (uint64_t t = 0; t < m->tokens; ++t)
        plamo_bf16_matvec_serial(m->weights, m->input + t * m->input_stride,
                                 m->output + t * m->output_stride, m->rows, m->columns);
}
void plamo_bf16_matmul(const struct plamo_matmul *m) {
    plamo_bf16_matmul_core(m);
}
void plamo_bf16_matmul8x3(const struct plamo_matmul *m) {
    plamo_bf16_matmul_core(m);
}
void plamo_bf16_linear(const uint16_t *w, const float *x, float *y, uint64_t rows, uint64_t cols,
                       uint64_t tokens, uint64_t xstride, uint64_t ystride) {
    struct plamo_matmul m = {w, x, y, rows, cols, tokens, xstride, ystride};
    plamo_bf16_matmul_core(&m);
}

/* ------------------------------------------------------ src/activation.s */

static const float exp_low = -87.0f, exp_high = 88.0f, exp_log2e = 1.4426950408889634f,
                   exp_ln2 = 0.6931471805599453f;
/* Taylor coefficients 1/7! .. 1/2! of the degree-7 polynomial on
   [-ln2/2, ln2/2] (src/activation.s:229-232). */
static const float exp_poly[6] = {0.0001984126984126984f, 0.001388888888888889f,
                                  0.008333333333333333f,  0.041666666666666664f,
                                  0.16666666666666666f,   0.5f};

/* exp(x): x < -87 -> 0, x > 88 -> +inf, else n = rint(x*log2e),
   r = fma(-n, ln2, x), Horner in FMA, times 2^n (src/activation.s:6-46). */
float plamo_exp(float x) {
    if (!(x >= exp_low))
        return 0.0f;
    if (x > exp_high)
        return INFINITY;
    float n = rintf(x * exp_log2e);
    int32_t e = (int32_t)n;
    float r = fmaf(-n, exp_ln2, x);
    float p = exp_poly[0];
    for (int k = 1; k < 6; ++k)
        p = fmaf(p, r, exp_poly[k]);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    uint32_t bits = (uint32_t)(e + 127) << 23;
    float scale;
    memcpy(&scale, &bits, 4);
    return p * scale;
}

/* In-place softmax: sequential max, exp(x - max), sequential sum, divide
   (src/activation.s:88-178). */
void plamo_softmax(float *x, uint64_t n) {
    if (!n)
        return;
    float maximum = x[0];
    for (uint64_t i = 1; i < n; ++i)
        maximum = fmaxf(maximum, x[i]);
    float sum = 0;
    for (uint64_t i = 0; i < n; ++i) {
        x[i] = plamo_exp(x[i] - maximum);
        sum = sum + x[i];
    }
    for (uint64_t i = 0; i < n; ++i)
        x[i] = x[i] / sum;
}

/* out[i] = (g / (exp(-g) + 1)) * u with g = in[i], u = in[n + i]
   (src/activation.s:182-226). out may alias the gate half. */
void plamo_swiglu(const float *in, float *out, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i) {
        float g = in[i], u = in[n + i];
        float d = plamo_exp(-g) + 1.0f;
        out[i] = (g / d) * u;
    }
}

/* ------------------------------------------------------------ src/token.s */

int plamo_embedding(const uint16_t *table, uint64_t token, uint64_t vocab, uint64_t hidden,
                    float *out) {
    if (token >= vocab)
        return 0;
    const uint16_t *row = table + token * hidden;
    for (uint64_t i = 0; i < hidden; ++i)
        out[i] = bf16(row[i]);
    return 1;
}

/* First maximal index; empty input or any NaN gives UINT64_MAX
   (src/token.s:35-63). */
uint64_t plamo_argmax(const float *x, uint64_t n) {
    if (!n || isnan(x[0]))
        return UINT64_MAX;
    float best = x[0];
    uint64_t index = 0;
    for (uint64_t i = 1; i < n; ++i) {
        if (isnan(x[i]))
            return UINT64_MAX;
        if (x[i] > best) {
            best = x[i];
            index = i;
        }
    }
    return index;
}

/* -------------------------------------------------------------- src/qkv.s */

void plamo_qk_norm(float *qkv, const uint16_t *qn, const uint16_t *kn, uint64_t qh, uint64_t kh,
                   uint64_t dim) {
    for (uint64_t head = 0; head < qh + kh; ++head)
        plamo_rmsnorm(qkv + head * dim, head < qh ? qn : kn, qkv + head * dim, dim, 1e-6f, 1.0f);
}

void plamo_qkv(const struct qkv *d) {
    plamo_bf16_matvec(d->weight, d->input, d->out, (d->qh + 2 * d->kh) * d->dim, d->hidden);
    plamo_qk_norm(d->out, d->qn, d->kn, d->qh, d->kh, d->dim);
}

/* ------------------------------------------------------------ src/cache.s */

int plamo_cache_append(struct cache *c, const float *k, const float *v) {
    if (!c->capacity || !c->width || c->count > c->capacity)
        return 0;
    if (c->count == c->capacity) {
        if (!c->sliding)
            return 0;
        uint64_t words = (c->capacity - 1) * c->width;
        memmove(c->k, c->k + c->width, words * 4);
        memmove(c->v, c->v + c->width, words * 4);
        c->count--;
    }
    memcpy(c->k + c->count * c->width, k, c->width * 4);
    memcpy(c->v + c->count * c->width, v, c->width * 4);
    c->count++;
    return 1;
}

/* ------------------------------------------------------------- src/trig.s */

static const double two_pi = 6.283185307179586;
/* Taylor series of sin(r)/r and cos(r) in r^2, highest order first:
   1/17!, -1/15!, ..., -1/3! and 1/16!, ..., -1/2! (src/trig.s:41-44). */
static const double sin_poly[8] = {2.8114572543455206e-15, -7.647163731819816e-13,
                                   1.6059043836821613e-10, -2.505210838544172e-08,
                                   2.7557319223985893e-06, -0.0001984126984126984,
                                   0.008333333333333333,   -0.16666666666666666};
static const double cos_poly[8] = {4.779477332387385e-14, -1.1470745597729725e-11,
                                   2.08767569878681e-09,  -2.755731922398589e-07,
                                   2.48015873015873e-05,  -0.001388888888888889,
                                   0.041666666666666664,  -0.5};

/* out = {sin, cos} in FP32 of a double angle: reduce by 2*pi with a fused
   multiply-subtract, then Horner in r^2 (src/trig.s:5-39). */
void plamo_sincos(double angle, float *out) {
    double n = rint(angle / two_pi);
    double r = fma(-n, two_pi, angle);
    double r2 = r * r;
    double p = sin_poly[0];
    for (int k = 1; k < 8; ++k)
        p = fma(p, r2, sin_poly[k]);
    p = fma(p, r2, 1.0);
    p = p * r;
    out[0] = (float)p;
    p = cos_poly[0];
    for (int k = 1; k < 8; ++k)
        p = fma(p, r2, cos_poly[k]);
    p = fma(p, r2, 1.0);
    out[1] = (float)p;
}

/* -------------------------------------------------------- src/rope_table.s */

void plamo_rope_table(const float *freq, uint64_t position, uint64_t half, float *cos_out,
                      float *sin_out, float scale) {
    float p = (float)position;
    for (uint64_t j = 0; j < half; ++j) {
        float angle = freq[j] * p;
        float sc[2];
        plamo_sincos((double)angle, sc);
        sin_out[j] = sc[0] * scale;
        cos_out[j] = sc[1] * scale;
    }
}

/* ------------------------------------------------------------- src/rope.s */

/* Split-half rotation, separate multiplies (no FMA) (src/rope.s:15-67). */
void plamo_rope_copy(const float *src, float *dst, const float *c, const float *s, uint64_t heads,
                     uint64_t half) {
    if (!heads || !half)
        return;
    for (uint64_t h = 0; h < heads; ++h) {
        const float *a = src + h * 2 * half;
        float *o = dst + h * 2 * half;
        for (uint64_t i = 0; i < half; ++i) {
            float x1 = a[i], x2 = a[i + half];
            float p = x1 * c[i], q = x2 * s[i];
            float r = x2 * c[i], t = x1 * s[i];
            o[i] = p - q;
            o[i + half] = r + t;
        }
    }
}

void plamo_rope_apply(float *x, const float *c, const float *s, uint64_t heads, uint64_t half) {
    plamo_rope_copy(x, x, c, s, heads, half);
}

/* ------------------------------------------------------- src/cache_rope.s */

static void cache_rope_from(struct rotation *r, uint64_t from, float scale) {
    const struct cache *c = r->cache;
    for (uint64_t t = from; t < c->count; ++t) {
        plamo_rope_table(r->freq, t, r->dim / 2, r->cos, r->sin, scale);
        plamo_rope_copy(c->k + t * c->width, r->out + t * c->width, r->cos, r->sin, r->heads,
                        r->dim / 2);
    }
}

/* Rotate every cached key at its local position 0..count-1. */
void plamo_cache_rope(struct rotation *r, float scale) {
    cache_rope_from(r, 0, scale);
}

/* Rotate only the newest row when exactly one row was appended since the
   last call with the same concentration; otherwise (eviction, reset, several
   rows, scale change) rotate all rows again (src/cache_rope.s:15-37). */
void plamo_cache_rope_cached(struct rotation *r, float scale) {
    uint64_t count = r->cache->count;
    uint64_t bits = float_bits(scale);
    if (count) {
        uint64_t from = 0;
        if (r->scale_bits == bits && r->processed_count + 1 == count)
            from = r->processed_count;
        cache_rope_from(r, from, scale);
    }
    r->processed_count = count;
    r->scale_bits = bits;
}

/* -------------------------------------------------------- src/attention.s */

/* One query head over n KV rows of token stride `stride` floats: sequential
   FMA dot products times 1/sqrt(d), softmax, sequential weighted values
   (src/attention.s:8-139). */
void plamo_attention_head(const float *q, const float *k, const float *v, float *out,
                          float *scores, uint64_t n, uint64_t d, uint64_t stride) {
    float scale = 1.0f / sqrtf((float)d);
    for (uint64_t i = 0; i < n; ++i) {
        float acc = 0;
        const float *key = k + i * stride;
        for (uint64_t j = 0; j < d; ++j)
            acc = fmaf(q[j], key[j], acc);
        scores[i] = acc * scale;
    }
    plamo_softmax(scores, n);
    for (uint64_t j = 0; j < d; ++j) {
        float acc = 0;
        for (uint64_t i = 0; i < n; ++i)
            acc = fmaf(scores[i], v[i * stride + j], acc);
        out[j] = acc;
    }
}

void plamo_gqa(const struct gqa *g) {
    uint64_t group = g->qh / g->kh;
    for (uint64_t h = 0; h < g->qh; ++h) {
        uint64_t kv = h / group;
        plamo_attention_head(g->q + h * g->dim, g->k + kv * g->dim, g->v + kv * g->dim,
                             g->out + h * g->dim, g->scores, g->tokens, g->dim, g->kh * g->dim);
    }
}

/* ------------------------------------------------------------ src/model.s */

void plamo_mlp(const uint16_t *gu, const uint16_t *down, const float *in, float *out,
               float *scratch, uint64_t hidden, uint64_t inter) {
    plamo_bf16_matvec(gu, in, scratch, 2 * inter, hidden);
    plamo_swiglu(scratch, scratch, inter);
    plamo_bf16_matvec(down, scratch, out, hidden, inter);
}

void plamo_residual(float *dst, const float *branch, uint64_t n) {
    for (uint64_t i = 0; i < n; ++i)
        dst[i] = dst[i] + branch[i];
}

/* Post-MLP norm offset 1/5^1.5 (src/model.s:112). */
static const float mlp_post_offset = 0.08944271909999159f;
/* Post-mixer norm offset (src/layer.s:51). */
static const float mixer_post_offset = 0.2f;

void plamo_mlp_branch(const struct mlp *m) {
    plamo_rmsnorm(m->state, m->pre, m->normalized, m->hidden, 1e-6f, 1.0f);
    plamo_mlp(m->gu, m->down, m->normalized, m->branch, m->scratch, m->hidden, m->intermediate);
    plamo_rmsnorm(m->branch, m->post, m->branch, m->hidden, 1e-6f, mlp_post_offset);
    plamo_residual(m->state, m->branch, m->hidden);
}

/* ------------------------------------------------------------ src/mixer.s */

int plamo_mixer_attention(const struct mixer *m, float *qkv, float *out, float scale) {
    const struct qkv *q = m->qkv;
    struct cache *c = m->cache;
    struct rotation *r = m->rotation;
    const float *k_new = qkv + q->qh * q->dim, *v_new = k_new + c->width;
    if (!plamo_cache_append(c, k_new, v_new))
        return 0;
    plamo_cache_rope_cached(r, scale);
    plamo_rope_apply(qkv, r->cos, r->sin, q->qh, q->dim / 2);
    struct gqa g = {qkv,        r->out,        c->v,        out,       m->gqa->scores,
                    c->count,   m->gqa->dim,   m->gqa->qh,  m->gqa->kh};
    plamo_gqa(&g);
    return 1;
}

int plamo_mixer(const struct mixer *m, float scale) {
    plamo_qkv(m->qkv);
    if (!plamo_mixer_attention(m, m->qkv->out, m->gqa->out, scale))
        return 0;
    plamo_bf16_matvec(m->weight, m->gqa->out, m->out, m->hidden, m->gqa->dim * m->gqa->qh);
    return 1;
}

/* ------------------------------------------------------------ src/layer.s */

int plamo_layer(const struct layer *l, float scale) {
    plamo_rmsnorm(l->state, l->pre, l->normalized, l->hidden, 1e-6f, 1.0f);
    l->mixer->qkv->input = l->normalized;
    l->mixer->out = l->branch;
    if (!plamo_mixer(l->mixer, scale))
        return 0;
    plamo_rmsnorm(l->branch, l->post, l->branch, l->hidden, 1e-6f, mixer_post_offset);
    plamo_residual(l->state, l->branch, l->hidden);
    l->mlp->state = l->state;
    plamo_mlp_branch(l->mlp);
    return 1;
}

/* ---------------------------------------------------------- src/forward.s */

static int forward_common(struct model *m, uint64_t token, int logits) {
    if (!plamo_embedding(m->embedding, token, m->vocab, m->hidden, m->state))
        return 0;
    for (uint64_t i = 0; i < m->count; ++i) {
        struct layer *l = m->layers[i];
        l->state = m->state;
        if (!plamo_layer(l, m->scales[i]))
            return 0;
    }
    if (logits) {
        plamo_rmsnorm(m->state, m->norm, m->normalized, m->hidden, 1e-6f, 1.0f);
        plamo_bf16_matvec(m->head, m->normalized, m->logits, m->vocab, m->hidden);
    }
    return 1;
}

int plamo_forward(struct model *m, uint64_t token) {
    return forward_common(m, token, 1);
}

int plamo_forward_hidden(struct model *m, uint64_t token) {
    return forward_common(m, token, 0);
}

/* ------------------------------------------------------------ src/batch.s */

void plamo_rmsnorm_rows(const float *x, const uint16_t *w, float *y, uint64_t width, uint64_t rows,
                        float eps, float offset) {
    for (uint64_t r = 0; r < rows; ++r)
        plamo_rmsnorm(x + r * width, w, y + r * width, width, eps, offset);
}

void plamo_swiglu_rows(float *gu, uint64_t width, uint64_t rows) {
    for (uint64_t r = 0; r < rows; ++r)
        plamo_swiglu(gu + r * 2 * width, gu + r * 2 * width, width);
}

/* Layer-major batch: projections over all tokens, attention and cache
   updates in token order (src/batch.s:61-223). */
int plamo_layer_batch(const struct layer *l, float *states, uint64_t tokens,
                      const struct plamo_prefill_workspace *ws, float scale) {
    if (!tokens)
        return 1;
    const struct mixer *mix = l->mixer;
    const struct qkv *q = mix->qkv;
    const struct mlp *p = l->mlp;
    uint64_t h = l->hidden, aw = q->qh * q->dim, qw = (q->qh + 2 * q->kh) * q->dim;
    uint64_t inter = p->intermediate;
    plamo_rmsnorm_rows(states, l->pre, ws->normalized, h, tokens, 1e-6f, 1.0f);
    plamo_bf16_linear(q->weight, ws->normalized, ws->qkv, qw, h, tokens, h, qw);
    for (uint64_t t = 0; t < tokens; ++t) {
        plamo_qk_norm(ws->qkv + t * qw, q->qn, q->kn, q->qh, q->kh, q->dim);
        if (!plamo_mixer_attention(mix, ws->qkv + t * qw, ws->attention + t * aw, scale))
            return 0;
    }
    plamo_bf16_linear(mix->weight, ws->attention, ws->branch, h, aw, tokens, aw, h);
    plamo_rmsnorm_rows(ws->branch, l->post, ws->branch, h, tokens, 1e-6f, mixer_post_offset);
    plamo_residual(states, ws->branch, tokens * h);
    plamo_rmsnorm_rows(states, p->pre, ws->normalized, h, tokens, 1e-6f, 1.0f);
    plamo_bf16_linear(p->gu, ws->normalized, ws->gate_up, 2 * inter, h, tokens, h, 2 * inter);
    plamo_swiglu_rows(ws->gate_up, inter, tokens);
    plamo_bf16_linear(p->down, ws->gate_up, ws->branch, h, inter, tokens, 2 * inter, h);
    plamo_rmsnorm_rows(ws->branch, p->post, ws->branch, h, tokens, 1e-6f, mlp_post_offset);
    plamo_residual(states, ws->branch, tokens * h);
    return 1;
}

/* ---------------------------------------------------------- src/prefill.s */

static void prefill_final(struct model *m, const float *states, uint64_t n) {
    memcpy(m->state, states + (n - 1) * m->hidden, m->hidden * 4);
    plamo_rmsnorm(m->state, m->norm, m->normalized, m->hidden, 1e-6f, 1.0f);
    plamo_bf16_matvec(m->head, m->normalized, m->logits, m->vocab, m->hidden);
}

/* Layer-major prompt: all embeddings, then every layer over every token,
   then final norm + head for the last token only (src/prefill.s:7-178). */
int plamo_prefill(struct model *m, const uint32_t *ids, uint64_t n, float *states) {
    if (!n)
        return 0;
    uint64_t h = m->hidden;
    for (uint64_t t = 0; t < n; ++t)
        if (!plamo_embedding(m->embedding, ids[t], m->vocab, h, states + t * h))
            return 0;
    int ok = 1;
    if (m->count && n >= 2) {
        const struct qkv *q = m->layers[0]->mixer->qkv;
        uint64_t aw = q->qh * q->dim, qw = (q->qh + 2 * q->kh) * q->dim;
        uint64_t gw = 2 * m->layers[0]->mlp->intermediate;
        float *work = malloc((size_t)((gw + aw + qw + 2 * h) * n * 4));
        if (!work)
            return 0;
        struct plamo_prefill_workspace ws;
        ws.normalized = work;
        ws.qkv = ws.normalized + n * h;
        ws.attention = ws.qkv + n * qw;
        ws.branch = ws.attention + n * aw;
        ws.gate_up = ws.branch + n * h;
        for (uint64_t i = 0; i < m->count && ok; ++i)
            ok = plamo_layer_batch(m->layers[i], states, n, &ws, m->scales[i]);
        free(work);
    } else {
        for (uint64_t i = 0; i < m->count && ok; ++i)
            for (uint64_t t = 0; t < n && ok; ++t) {
                m->layers[i]->state = states + t * h;
                ok = plamo_layer(m->layers[i], m->scales[i]);
            }
    }
    if (!ok)
        return 0;
    prefill_final(m, states, n);
    return 1;
}

/* Token-by-token layer-major prompt (reference tests/prefill_reference.s),
   used by the reference's prefill test as the sequential baseline. */
int plamo_prefill_reference(struct model *m, const uint32_t *ids, uint64_t n, float *states) {
    if (!n)
        return 0;
    uint64_t h = m->hidden;
    for (uint64_t t = 0; t < n; ++t)
        if (!plamo_embedding(m->embedding, ids[t], m->vocab, h, states + t * h))
            return 0;
    for (uint64_t i = 0; i < m->count; ++i)
        for (uint64_t t = 0; t < n; ++t) {
            m->layers[i]->state = states + t * h;
            if (!plamo_layer(m->layers[i], m->scales[i]))
                return 0;
        }
    prefill_final(m, states, n);
    return 1;
}

/* ----------------------------------------------- tools/rope_constants.py */

static float fp(double value) {
    return (float)value;
}

/* Inverse frequencies of one RoPE variant with FP32 rounding after every
   step, as tools/rope_constants.py:21-52 forms them. */
void oracle_rope_frequencies(double base, int yarn, double factor, double original,
                             double beta_fast, double beta_slow, uint64_t half, float *out) {
    const double pi = 3.141592653589793;
    double low = 0, high = 0;
    if (yarn) {
        low = half * log(original / (beta_fast * 2 * pi)) / log(base);
        high = half * log(original / (beta_slow * 2 * pi)) / log(base);
    }
    for (uint64_t index = 0; index < half; ++index) {
        float frequency = fp(pow(base, (double)index / (double)half));
        float extrapolated = fp(1.0 / (double)frequency);
        if (yarn) {
            float ramp = fp((double)fp((double)index - (double)fp(low)) / (double)fp(high - low));
            double clipped = ramp < 0 ? 0 : (ramp > 1 ? 1 : ramp);
            float mask = fp(1.0 - clipped);
            float interpolated = fp(1.0 / (double)fp(factor * (double)frequency));
            extrapolated = fp((double)fp((double)interpolated * (double)fp(1.0 - (double)mask)) +
                              (double)fp((double)extrapolated * (double)mask));
        }
        out[index] = extrapolated;
    }
}

/* The pinned checkpoints' two variants (tools/profiles/<model>/config.json
   rope_parameters): sliding layers default theta 1e4; full layers YaRN theta
   1e6, factor 256, original 4096, beta 32/1. Concentration 1 + 0.1 ln 256. */
float plamo_rope_local[64], plamo_rope_global[64];
float plamo_rope_local_scale = 1.0f, plamo_rope_global_scale = 1.0f;

__attribute__((constructor)) static void oracle_rope_constants(void) {
    oracle_rope_frequencies(10000.0, 0, 1, 1, 1, 1, 64, plamo_rope_local);
    oracle_rope_frequencies(1000000.0, 1, 256.0, 4096.0, 32.0, 1.0, 64, plamo_rope_global);
    plamo_rope_local_scale = 1.0f;
    plamo_rope_global_scale = fp(1 + 0.1 * log(256.0));
}

/* ------------------------------------------------ synthetic test inputs */

#include "../include/plamo_synthetic.h"

struct synthetic_job {
    uint16_t *dst;
    uint64_t begin, end, seed;
    float mean, std;
};

static void *synthetic_worker(void *argument) {
    const struct synthetic_job *job = argument;
    for (uint64_t i = job->begin; i < job->end; ++i)
        job->dst[i] = plamo_synthetic_bf16(job->seed, i, job->mean, job->std);
    return NULL;
}

/* Host copy of the seeded BF16 tensor the benchmark generates in HBM
   (same generator definition, include/plamo_synthetic.h), split across
   `threads` workers. Lets the CPU baseline build its model without the GPU. */
void oracle_synthetic_bf16(uint16_t *dst, uint64_t count, uint64_t seed, float mean, float std,
                           int threads) {
    enum { MAX_WORKERS = 256 };
    if (threads < 1)
        threads = 1;
    if (threads > MAX_WORKERS)
        threads = MAX_WORKERS;
    struct synthetic_job jobs[MAX_WORKERS];
    pthread_t ids[MAX_WORKERS];
    int created[MAX_WORKERS] = {0};
    for (int t = 0; t < threads; ++t)
        jobs[t] = (struct synthetic_job){dst, count * (uint64_t)t / (uint64_t)threads,
                                         count * (uint64_t)(t + 1) / (uint64_t)threads, seed, mean,
                                         std};
    for (int t = 1; t < threads; ++t)
        created[t] = !pthread_create(&ids[t], NULL, synthetic_worker, &jobs[t]);
    synthetic_worker(&jobs[0]);
    for (int t = 1; t < threads; ++t) {
        if (created[t])
            pthread_join(ids[t], NULL);
        else
            synthetic_worker(&jobs[t]);
    }
}
