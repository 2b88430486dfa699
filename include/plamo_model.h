/* Model descriptor ABI of the PLaMo-3 token loop.
 *
 * These records are the interface between a host engine, the CUDA backend
 * (plamo_cuda.h) and the C oracle used by the tests. Their byte layout is the
 * one the reference's assembly kernels and engine agree on
 * (reference runtime/model.h:7-86, runtime/parallel.h:5-12), so that a model
 * descriptor built by the reference's loader, its prompt cache or its tests
 * can be handed to this backend without translation. Every record is plain
 * data: host pointers and 64-bit sizes.
 *
 * Units: all activations are FP32, all weights are BF16 bit patterns
 * (uint16_t, the upper half of an IEEE binary32), row-major exactly as they
 * are stored in the safetensors checkpoint.
 */
#ifndef PLAMO_MODEL_H
#define PLAMO_MODEL_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The records are the reference's, under the reference's own include guards
   (runtime/model.h: PLAMO_RUNTIME_MODEL_H, runtime/parallel.h:
   PLAMO_PARALLEL_H): a translation unit that includes the reference's
   headers first and this one after (an adapter such as
   integration/metal_cuda.c) sees each record once. This header does not
   define those guards itself. */
#ifndef PLAMO_RUNTIME_MODEL_H
/* Fused Q|K|V projection followed by per-head RMSNorm(+1) of Q and K.
   out = [(qh + 2*kh) * dim], Q heads, then K heads, then V heads. */
struct qkv {
    const float *input;
    const uint16_t *weight, *qn, *kn;
    float *out;
    uint64_t hidden, qh, kh, dim;
};
/* Token-major KV rows [capacity, width] holding normalised, unrotated keys and
   values. `count` rows are valid. A sliding cache drops its oldest row when
   full; a global cache refuses to grow past capacity. */
struct cache {
    float *k, *v;
    uint64_t capacity, count, width, sliding;
};
/* Rotated copy of the cached keys at local positions 0..count-1, its
   frequency table (dim/2 FP32) and the cos/sin scratch left at count-1.
   processed_count/scale_bits record which rows are up to date. */
struct rotation {
    struct cache *cache;
    float *out;
    const float *freq;
    float *cos, *sin;
    uint64_t heads, dim, processed_count, scale_bits;
};
/* Grouped-query attention of one query token over `tokens` KV rows. */
struct gqa {
    float *q, *k, *v, *out, *scores;
    uint64_t tokens, dim, qh, kh;
};
struct mixer {
    struct qkv *qkv;
    struct cache *cache;
    struct rotation *rotation;
    struct gqa *gqa;
    const uint16_t *weight; /* o_proj [hidden, qh*dim] */
    float *out;
    uint64_t hidden;
};
/* Only state is a result; normalized/branch/scratch are CPU workspace. */
struct mlp {
    float *state;
    const uint16_t *pre, *post, *gu, *down;
    float *normalized, *branch, *scratch;
    uint64_t hidden, intermediate;
};
struct layer {
    float *state;
    const uint16_t *pre, *post;
    float *normalized, *branch;
    struct mixer *mixer;
    struct mlp *mlp;
    uint64_t hidden;
};
struct model {
    const uint16_t *embedding;
    uint64_t vocab, hidden;
    float *state;
    struct layer **layers;
    uint64_t count;
    float *scales; /* RoPE concentration per layer */
    const uint16_t *norm;
    float *normalized;
    const uint16_t *head;
    float *logits;
};
/* Checkpoint mapping and weight schema records (reference runtime/model.h:65-74). */
struct plamo_mapping {
    void *base;
    uint64_t bytes;
};
struct plamo_weight_spec {
    const char *name;
    uint64_t rank;
    const uint64_t *shape;
    void **slot;
};
#endif
#ifndef PLAMO_PARALLEL_H
/* Y[token, row] = W[row, :] . X[token, :], strides in FP32 elements. */
struct plamo_matmul {
    const uint16_t *weights;
    const float *input;
    float *output;
    uint64_t rows, columns, tokens, input_stride, output_stride;
};
#endif

#ifdef __cplusplus
#define PLAMO_STATIC_ASSERT static_assert
#else
#define PLAMO_STATIC_ASSERT _Static_assert
#endif
PLAMO_STATIC_ASSERT(sizeof(struct model) == 88, "model ABI");
PLAMO_STATIC_ASSERT(sizeof(struct qkv) == 72, "QKV ABI");
PLAMO_STATIC_ASSERT(sizeof(struct cache) == 48, "cache ABI");
PLAMO_STATIC_ASSERT(sizeof(struct rotation) == 72, "rotation ABI");
PLAMO_STATIC_ASSERT(sizeof(struct gqa) == 72, "GQA ABI");
PLAMO_STATIC_ASSERT(sizeof(struct mixer) == 56, "mixer ABI");
PLAMO_STATIC_ASSERT(sizeof(struct mlp) == 80, "MLP ABI");
PLAMO_STATIC_ASSERT(sizeof(struct layer) == 64, "layer ABI");
PLAMO_STATIC_ASSERT(sizeof(struct plamo_matmul) == 64, "matmul ABI");
PLAMO_STATIC_ASSERT(sizeof(struct plamo_mapping) == 16, "mapping ABI");
PLAMO_STATIC_ASSERT(sizeof(struct plamo_weight_spec) == 32, "weight schema ABI");
PLAMO_STATIC_ASSERT(offsetof(struct layer, mixer) == 40, "layer ABI");
PLAMO_STATIC_ASSERT(offsetof(struct cache, count) == 24, "cache ABI");
PLAMO_STATIC_ASSERT(offsetof(struct rotation, processed_count) == 56, "rotation ABI");

#ifdef __cplusplus
}
#endif
#endif
