/* C oracle of the PLaMo-3 token loop: declarations.
 *
 * TEST INFRASTRUCTURE ONLY (checker for the CUDA path; never linked into the
 * product library). Each function restates the reference assembly routine of
 * the same name; plamo_oracle.c cites the file and lines it follows.
 */
#ifndef PLAMO_ORACLE_H
#define PLAMO_ORACLE_H
#include "../include/plamo_model.h"

#ifdef __cplusplus
extern "C" {
#endif

void oracle_set_threads(int threads);
int oracle_threads(void);
/* 4 (default): the reference's matvec order. 8: an equally valid FP32 order
   that is not the reference's, for measuring a whole model's sensitivity to
   summation order. */
void oracle_set_matvec_lanes(int lanes);
extern uint64_t plamo_weight_chunk_bytes;

void plamo_bf16_matvec(const uint16_t *, const float *, float *, uint64_t rows, uint64_t cols);
void plamo_bf16_matvec_serial(const uint16_t *, const float *, float *, uint64_t, uint64_t);
void plamo_bf16_matvec_core(const uint16_t *, const float *, float *, uint64_t, uint64_t);
void plamo_bf16_matmul(const struct plamo_matmul *);
void plamo_bf16_matmul_core(const struct plamo_matmul *);
void plamo_bf16_matmul8x3(const struct plamo_matmul *);
void plamo_bf16_linear(const uint16_t *, const float *, float *, uint64_t rows, uint64_t cols,
                       uint64_t tokens, uint64_t xstride, uint64_t ystride);
void plamo_rmsnorm(const float *, const uint16_t *, float *, uint64_t, float eps, float offset);
void plamo_rmsnorm_rows(const float *, const uint16_t *, float *, uint64_t width, uint64_t rows,
                        float eps, float offset);

float plamo_exp(float);
void plamo_softmax(float *, uint64_t);
void plamo_swiglu(const float *, float *, uint64_t);
void plamo_swiglu_rows(float *, uint64_t width, uint64_t rows);

int plamo_embedding(const uint16_t *, uint64_t token, uint64_t vocab, uint64_t hidden, float *);
uint64_t plamo_argmax(const float *, uint64_t);

void plamo_qkv(const struct qkv *);
void plamo_qk_norm(float *, const uint16_t *, const uint16_t *, uint64_t qh, uint64_t kh,
                   uint64_t dim);
int plamo_cache_append(struct cache *, const float *, const float *);

void plamo_sincos(double, float *);
void plamo_rope_table(const float *freq, uint64_t position, uint64_t half, float *cos_out,
                      float *sin_out, float scale);
void plamo_rope_copy(const float *, float *, const float *, const float *, uint64_t heads,
                     uint64_t half);
void plamo_rope_apply(float *, const float *, const float *, uint64_t heads, uint64_t half);
void plamo_cache_rope(struct rotation *, float);
void plamo_cache_rope_cached(struct rotation *, float);
void oracle_rope_frequencies(double base, int yarn, double factor, double original,
                             double beta_fast, double beta_slow, uint64_t half, float *out);
extern float plamo_rope_local[64], plamo_rope_global[64];
extern float plamo_rope_local_scale, plamo_rope_global_scale;

void plamo_attention_head(const float *q, const float *k, const float *v, float *out,
                          float *scores, uint64_t n, uint64_t d, uint64_t stride);
void plamo_gqa(const struct gqa *);

void plamo_mlp(const uint16_t *, const uint16_t *, const float *, float *, float *,
               uint64_t hidden, uint64_t inter);
void plamo_residual(float *, const float *, uint64_t);
void plamo_mlp_branch(const struct mlp *);
int plamo_mixer_attention(const struct mixer *, float *qkv, float *out, float scale);
int plamo_mixer(const struct mixer *, float);
int plamo_layer(const struct layer *, float);

struct plamo_prefill_workspace {
    float *normalized, *qkv, *attention, *branch, *gate_up;
};
int plamo_layer_batch(const struct layer *, float *states, uint64_t tokens,
                      const struct plamo_prefill_workspace *, float scale);
int plamo_forward(struct model *, uint64_t);
int plamo_forward_hidden(struct model *, uint64_t);
int plamo_prefill(struct model *, const uint32_t *, uint64_t, float *);
int plamo_prefill_reference(struct model *, const uint32_t *, uint64_t, float *);

#ifdef __cplusplus
}
#endif
#endif
