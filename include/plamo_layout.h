/* Model descriptor builder for C hosts on Linux.
 *
 * The reference generates its `struct model` records, work buffers and weight
 * schema at build time as Darwin assembly (reference tools/model_layout.py,
 * tools/weight_schema.py, tools/rope_constants.py -> src/model_layout.s,
 * src/weight_schema.s, src/rope_constants.s). This builder makes the same
 * records at run time from a profile's parameters, with the same wiring:
 *
 *   * every layer shares the work buffers (state, normalized, branch, QKV
 *     output, attention output, MLP scratch, scores, cos/sin); each layer has
 *     its own K, V and rotated-K rows of `capacity` rows (window + 1 for
 *     sliding layers, the full-attention capacity otherwise);
 *   * layer i is full attention iff (i + 1) % pattern == 0, rotating with the
 *     YaRN frequency table and concentration 1 + 0.1 ln(factor); sliding
 *     layers use the local table and concentration 1;
 *   * the weight schema lists every tensor in the reference's slot order
 *     (embed_tokens, norm, lm_head unless tied, then per layer qkv_proj,
 *     o_proj, q_norm, k_norm, gate_up_proj, down_proj, pre/post mixer norms,
 *     pre/post MLP norms); each entry's slot is the descriptor field the
 *     tensor belongs in, so plamo_bind_weights (plamo_safetensors.h) fills
 *     the records directly.
 *
 * Typical use:
 *   struct plamo_model_config cfg;
 *   plamo_model_config_profile("8b", &cfg);
 *   struct plamo_model_layout *lay = plamo_model_layout_create(&cfg, 8192, err, sizeof err);
 *   plamo_bind_weights(maps, files, plamo_model_layout_schema(lay));
 *   plamo_model_layout_finish(lay);           // ties the head, checks every slot
 *   struct model *m = plamo_model_layout_model(lay);
 *   ... plamo_cuda_preload / plamo_cuda_prepare_model(cuda, m) ...
 *   plamo_model_layout_destroy(lay);
 */
#ifndef PLAMO_LAYOUT_H
#define PLAMO_LAYOUT_H
#include <stddef.h>
#include <stdint.h>

#include "plamo_model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* The fields of a PLaMo-3 config.json that shape the descriptors. */
struct plamo_model_config {
    uint64_t hidden, layers, query_heads, kv_heads, head_dim, intermediate, vocab;
    uint64_t window;       /* window_size: sliding layers keep window + 1 rows */
    uint64_t pattern;      /* sliding_window_pattern */
    uint64_t max_position; /* max_position_embeddings: full-attention rows */
    uint64_t tied;         /* tie_word_embeddings */
    double local_theta;    /* rope_parameters.sliding_attention.rope_theta */
    double global_theta;   /* rope_parameters.full_attention.rope_theta (YaRN) */
    double yarn_factor, yarn_original, beta_fast, beta_slow;
};

#ifdef __cplusplus
static_assert(sizeof(struct plamo_model_config) == 136, "model config ABI");
#else
_Static_assert(sizeof(struct plamo_model_config) == 136, "model config ABI");
#endif

struct plamo_model_layout;

/* The parameters of a pinned profile ("0.8b", "2b", "8b", "31b"); 0 if unknown. */
int plamo_model_config_profile(const char *name, struct plamo_model_config *cfg);

/* Records, work buffers (zeroed) and schema for `cfg`. full_capacity bounds
   the rows of full-attention layers (0: max_position). NULL with a message
   on invalid parameters or allocation failure. */
struct plamo_model_layout *plamo_model_layout_create(const struct plamo_model_config *cfg, uint64_t full_capacity,
                                                     char *error, size_t cap);

/* NULL-name-terminated schema whose slots point into the layout's records. */
const struct plamo_weight_spec *plamo_model_layout_schema(const struct plamo_model_layout *layout);

/* After binding: points a tied head at the embedding; 1 when every weight
   field is set, else 0. */
int plamo_model_layout_finish(struct plamo_model_layout *layout);

struct model *plamo_model_layout_model(struct plamo_model_layout *layout);

/* Bytes of FP32 work buffers and KV rows the layout holds. */
uint64_t plamo_model_layout_buffer_bytes(const struct plamo_model_layout *layout);

/* The FP32 frequency table of one RoPE kind (dim/2 entries): FP32 rounding
   after every step as reference tools/rope_constants.py:21-52; YaRN when
   `yarn` is nonzero. */
void plamo_rope_frequencies(const struct plamo_model_config *cfg, int yarn, float *out);

void plamo_model_layout_destroy(struct plamo_model_layout *layout);

#ifdef __cplusplus
}
#endif
#endif
