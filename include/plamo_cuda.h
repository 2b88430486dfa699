/* B200 (sm_100a) backend of the PLaMo-3 token loop: C ABI.
 *
 * Drop-in for the reference's GPU backend interface (reference
 * runtime/metal.h:48-88). Each plamo_cuda_* entry replaces the plamo_metal_*
 * entry of the same suffix with the same arguments, return convention and
 * ownership rules, so the reference's engine (runtime/engine.c call sites
 * :180,187,234,243,264,302,304,369,462,481,495,540,562,597) binds to it by a
 * rename. The remaining entries are additions a CUDA device needs (explicit
 * host/device KV synchronisation, on-device greedy selection, the request
 * loop over token ids, timing and synthetic weights for benchmarks).
 *
 * Return convention of forward/prefill/verify/commit/linear/mlp, as
 * reference runtime/metal.h:63-74: 1 success; 0 declined with no state
 * changed (the caller may use another path); -1 executed and failed (do not
 * retry: KV may have advanced).
 *
 * Threading: one context is owned by one host thread; calls are serialised.
 */
#ifndef PLAMO_CUDA_H
#define PLAMO_CUDA_H
#include "plamo_model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Largest candidate block of one verification (reference runtime/metal.h:75). */
enum { PLAMO_CUDA_VERIFY_MAX = 16 };

struct plamo_cuda_config {
    int device;               /* CUDA device ordinal */
    uint64_t max_context;     /* KV rows kept per full-attention layer; 0 = 8192 + 16 */
    uint64_t max_prefill;     /* largest prompt of one prefill call; 0 = 4096 */
    uint64_t reserve;         /* HBM bytes left unallocated; 0 = 1 GiB */
    unsigned copy_kv_to_host; /* 1: keep the host K/V/rotated-K arrays current after
                                 every call (reference semantics, slower); 0: device
                                 KV is canonical and plamo_cuda_sync_host copies it */
};

struct plamo_cuda_info {
    char device[128], note[256];
    uint64_t launches, graph_launches, forwards, prefills, verification_batches,
        verified_tokens, committed_tokens, declines, errors;
    uint64_t weight_bytes, kv_bytes, workspace_bytes, allocated_bytes;
    uint64_t sm_count;
    double gpu_seconds; /* device time of completed forward/prefill/verify calls */
    /* KV page pool: pages mapped into requests' page tables, and pages
       allocated in all (kv_bytes counts the latter); a page holds 64 rows of
       keys and values of one layer. */
    uint64_t kv_pages_used, kv_pages_allocated;
};

struct plamo_cuda;

/* reference runtime/metal.h:48: NULL + message in error[cap] on failure. */
struct plamo_cuda *plamo_cuda_open(const struct plamo_cuda_config *, char *error, size_t cap);
/* reference runtime/metal.h:49 */
void plamo_cuda_close(struct plamo_cuda *);
/* reference runtime/metal.h:50: releases scratch not needed by prepared models,
   including the KV page chunks of a pool none of whose pages is mapped. */
void plamo_cuda_maintain(struct plamo_cuda *);
/* reference runtime/metal.h:51 */
void plamo_cuda_get_info(const struct plamo_cuda *, struct plamo_cuda_info *);
/* reference runtime/metal.h:55: copy host BF16 bytes [src, src+bytes) into HBM
   and remember the mapping. 0 on allocation or copy failure. */
int plamo_cuda_preload(struct plamo_cuda *, const void *src, uint64_t bytes);
/* reference runtime/metal.h:58: touch every resident byte once on the device. */
int plamo_cuda_warm_cache(struct plamo_cuda *);
/* reference runtime/metal.h:62: allocate device KV, RoPE tables and workspace for
   `model` and resolve each weight pointer to its HBM copy (uploading any weight
   not preloaded). Must precede forward/prefill/verify on that model. */
int plamo_cuda_prepare_model(struct plamo_cuda *, struct model *);
/* reference runtime/metal.h:67: one complete decode step of `token`. On success
   model->state, ->normalized and ->logits are current on the host. */
int plamo_cuda_forward(struct plamo_cuda *, struct model *, uint64_t token);
/* reference runtime/metal.h:73: layer-major prompt. states (tokens x hidden, may
   be NULL) receives every prompt state; model state/logits are for the last. */
int plamo_cuda_prefill(struct plamo_cuda *, struct model *, const uint32_t *ids,
                       uint64_t tokens, float *states);
/* reference runtime/metal.h:79: run candidates ids[0..tokens) without changing
   the committed state; next[j] = greedy token after ids[0..j]. */
int plamo_cuda_verify(struct plamo_cuda *, struct model *, const uint32_t *ids,
                      uint64_t tokens, uint32_t *next);
/* reference runtime/metal.h:81: commit candidate `index` of the last verify; indices
   must be committed in order 0,1,2,... */
int plamo_cuda_commit(struct plamo_cuda *, struct model *, uint64_t index);
/* reference runtime/metal.h:85: synchronous dense projection of host buffers. */
int plamo_cuda_linear(struct plamo_cuda *, const struct plamo_matmul *);
/* Size of the static device staging used by plamo_cuda_linear_static, in
   FP32 elements (16 MiB): tokens * (columns + rows) must not exceed it. */
#define PLAMO_CUDA_LINEAR_STATIC_FLOATS (4ull << 20)
/* No counterpart in the reference. Same projection as plamo_cuda_linear, for
   callers that cannot allocate device memory: it stages the host input and
   output rows in one fixed array compiled into this library (every GPU that
   loads it holds 16 MiB until the process exits) and calls no cudaMalloc,
   cudaFree or allocating library routine. Weights must already be preloaded
   (0 otherwise). A request needing more than PLAMO_CUDA_LINEAR_STATIC_FLOATS
   staging floats is declined (0) with the reason in plamo_cuda_info.note.
   The first call on a device looks up the array's device address; make that
   first call before any stream capture. All calls share the array, so calls
   that overlap on the GPU (several host threads, several contexts on one
   device) race; serialise them. */
int plamo_cuda_linear_static(struct plamo_cuda *, const struct plamo_matmul *);
/* reference runtime/metal.h:88: complete MLP branch (norm, gate_up, SwiGLU, down,
   norm, residual) applied in place to states[tokens x hidden]. */
int plamo_cuda_mlp(struct plamo_cuda *, const struct mlp *, float *states, uint64_t tokens);

/* ---- additions a discrete GPU needs ---- */

/* Copy the device-canonical KV rows, rotated keys (local positions, as the
   reference's rotation cache holds them), state, normalized and logits of
   `model` into its host arrays, and set the host counters. */
int plamo_cuda_sync_host(struct plamo_cuda *, struct model *);
/* Copy only state, normalized and logits of the last step into the host
   descriptors of `model` (what plamo_cuda_forward leaves there; the greedy
   entry points leave them on the device). */
int plamo_cuda_read_outputs(struct plamo_cuda *, struct model *);
/* Free the device state prepared for `model` (KV, workspace, graph). */
int plamo_cuda_release_model(struct plamo_cuda *, struct model *);
/* Unregister and free every preloaded range inside [src, src+bytes) (weights
   whose host memory is about to be reused); prepared models are released too.
   Returns the number of ranges freed. */
int plamo_cuda_release_weights(struct plamo_cuda *, const void *src, uint64_t bytes);
/* Declare the host K/V arrays of `model` canonical: the next call uploads
   rows [0, count) of every layer (use after writing host KV directly, e.g. by
   a CPU path or a prompt-cache restore that kept the same counts). A host
   count that differs from the device's is detected without this call. */
int plamo_cuda_invalidate(struct plamo_cuda *, struct model *);
/* Decode `token` and select the next token on the device (first maximal
   logit, reference src/token.s:35-63). Host state/logits are not copied.
   *next = UINT32_MAX when a logit is NaN. */
int plamo_cuda_forward_greedy(struct plamo_cuda *, struct model *, uint64_t token,
                              uint32_t *next);
/* forward_greedy that also returns the top-2 logit margin of the step (best
   minus the largest value at any other index): the draft proposer's
   confidence (reference runtime/worker.c:268-286). */
int plamo_cuda_forward_greedy_margin(struct plamo_cuda *, struct model *, uint64_t token, uint32_t *next,
                                     float *margin);
/* Prefill and select the first generated token on the device. */
int plamo_cuda_prefill_greedy(struct plamo_cuda *, struct model *, const uint32_t *ids,
                              uint64_t tokens, uint32_t *next);
/* Greedy request loop over token ids (reference runtime/engine.c:428-617 without
   the tokenizer): reset the request, prefill, then decode until max_tokens or a
   stop id (1, 16).
   out[] receives the emitted ids; returns their count, or -1 on failure.
   on_token (may be NULL) sees each id as soon as it is on the host; a zero
   return cancels. */
struct plamo_cuda_timing {
    double prefill_seconds, decode_seconds, first_token_seconds;
    uint64_t prompt_tokens, completion_tokens, decode_steps;
    const char *finish_reason;
};
int64_t plamo_cuda_generate(struct plamo_cuda *, struct model *, const uint32_t *ids,
                            uint64_t tokens, uint64_t max_tokens, uint32_t *out,
                            int (*on_token)(uint32_t id, void *context), void *context,
                            struct plamo_cuda_timing *timing);
/* One decoder layer of one decode step on a host hidden vector, in place
   (reference src/layer.s:8-48 plamo_layer): appends one KV row to layer
   `index` and advances only that layer. The layer's launches are recorded
   as a CUDA graph on its first call and replayed after (positions and KV
   pages are read on the device). */
int plamo_cuda_layer(struct plamo_cuda *, struct model *, uint64_t index, float *state);
/* Drop the newest `rows` committed rows of every layer of `model` (at most
   PLAMO_CUDA_VERIFY_MAX + 1): the draft model's rollback after a partially
   accepted proposal (reference runtime/draft.c:258-297). */
int plamo_cuda_rollback(struct plamo_cuda *, struct model *, uint64_t rows);
/* Speculative greedy request loop (reference runtime/engine.c:523-586, draft
   proposer runtime/worker.c:198-318): `draft` (a smaller model prepared in the
   same context) proposes up to `block` tokens (<= PLAMO_CUDA_VERIFY_MAX, with
   the reference's adaptive 2/8/16 horizon), `target` verifies them in one pass
   and commits the agreeing prefix. The emitted ids are exactly the target's
   greedy tokens. Returns their count or -1. */
struct plamo_cuda_speculation {
    double prefill_seconds, decode_seconds;
    uint64_t completion_tokens, decode_steps, verify_batches, proposed_tokens, accepted_tokens;
    const char *finish_reason;
};
int64_t plamo_cuda_generate_speculative(struct plamo_cuda *, struct model *target, struct model *draft,
                                        const uint32_t *ids, uint64_t tokens, uint64_t max_tokens, unsigned block,
                                        uint32_t *out, int (*on_token)(uint32_t id, void *context), void *context,
                                        struct plamo_cuda_speculation *stats);
/* Reset the request state of `model` (all KV counts to zero) on host and device,
   like the reference's plamo_reset_request (runtime/engine.c:46-55). */
void plamo_cuda_reset_request(struct plamo_cuda *, struct model *);

/* Multi-request decode (no counterpart in the reference, which serves one
   request at a time): `count` (1..PLAMO_CUDA_VERIFY_MAX) prepared models with
   identical shapes over the same preloaded weights - each its own descriptor
   tree and KV cache, one per request - advance one token each per step and
   share one pass over the weights: the projections run as tcgen05 GEMMs over
   the `count` rows, attention runs per request on its own cache (head dim
   128). step() appends tokens[i] to request i and writes its greedy next token
   to next[i], like plamo_cuda_forward_greedy on each model (host state and
   logits are not copied; host KV counts are). One CUDA graph per step.
   Returns 1, 0 (declined: a cache is full or a token is outside the
   vocabulary; nothing changed) or -1. time_batch runs `steps` steps feeding
   each step's tokens into the next on the device and returns the device
   milliseconds. */
struct plamo_cuda_batch;
struct plamo_cuda_batch *plamo_cuda_batch_open(struct plamo_cuda *, struct model *const *models, unsigned count);
int plamo_cuda_batch_step(struct plamo_cuda_batch *, const uint32_t *tokens, uint32_t *next);
double plamo_cuda_time_batch(struct plamo_cuda_batch *, uint64_t steps);
void plamo_cuda_batch_close(struct plamo_cuda_batch *);

/* Device prompt (template prefix) cache: the snapshots of reference
   runtime/prompt_cache.h:8-16, held in device memory. Capture copies the
   committed KV rows [0, tokens) of every layer of a prepared model after a
   fresh prefill of exactly `tokens` ids (1..PLAMO_CUDA_PREFIX_LIMIT); restore
   writes them back into the device rings of the same model, sets every layer's
   count (host and device) to the snapshot's tokens and returns that count, so a
   following prefill of ids[tokens...] continues the prompt. The acceptance
   rules are the reference's (runtime/prompt_cache.c:15-81): capture returns
   NULL unless every layer holds exactly `tokens` rows and the reference's
   16 MiB snapshot bound admits the model; restore returns 0 (touching nothing)
   unless `model` is the captured one, `tokens` exceeds the snapshot's, the
   snapshot ids are a prefix of `ids`, and every layer's width and capacity fit
   (all layers are checked before any is written). A snapshot is immutable,
   independent of later requests and owned by the caller; free it with
   plamo_cuda_prompt_cache_free before closing its context. bytes() counts the
   device memory it holds (K and V rows; rotated keys are derived on the fly). */
#define PLAMO_CUDA_PREFIX_LIMIT 64
struct plamo_cuda_prompt_cache;
struct plamo_cuda_prompt_cache *plamo_cuda_prompt_cache_capture(struct plamo_cuda *, const struct model *,
                                                                const uint32_t *ids, uint64_t tokens);
uint64_t plamo_cuda_prompt_cache_restore(struct plamo_cuda *, const struct plamo_cuda_prompt_cache *,
                                         struct model *, const uint32_t *ids, uint64_t tokens);
uint64_t plamo_cuda_prompt_cache_tokens(const struct plamo_cuda_prompt_cache *);
uint64_t plamo_cuda_prompt_cache_bytes(const struct plamo_cuda_prompt_cache *);
void plamo_cuda_prompt_cache_free(struct plamo_cuda_prompt_cache *);

/* Standalone BF16 GEMV on device buffers: y[rows] = W[rows, cols] . x[cols]
   with FP32 accumulation (the decode projection kernel). Asynchronous on the
   context's stream. */
int plamo_cuda_gemv_device(struct plamo_cuda *, const uint16_t *w, const float *x, float *y,
                           uint64_t rows, uint64_t cols);

/* Prompt projection on device buffers: y[t][r] (row stride ys) =
   sum_k W[r][k] x[t][k] (x row stride xs, FP32). Tensor cores (tcgen05, x split
   into three BF16 terms, FP32 accumulation) when rows are 16-byte aligned and
   cols % 8 == 0, the FP32 CUDA-core kernel otherwise. Synchronous. */
int plamo_cuda_gemm_device(struct plamo_cuda *, const float *x, uint64_t xs, const uint16_t *w, float *y,
                           uint64_t ys, uint64_t tokens, uint64_t rows, uint64_t cols);

/* ---- device memory and timing helpers for tests and benchmarks ---- */
void *plamo_cuda_device_alloc(struct plamo_cuda *, uint64_t bytes);
void plamo_cuda_device_free(struct plamo_cuda *, void *);
int plamo_cuda_copy_to_device(struct plamo_cuda *, void *dst, const void *src, uint64_t bytes);
int plamo_cuda_copy_to_host(struct plamo_cuda *, void *dst, const void *src, uint64_t bytes);
int plamo_cuda_synchronize(struct plamo_cuda *);
/* Device time in milliseconds of `repeats` launches of the decode step graph
   of `model` (tokens fed back from the on-device argmax), measured with CUDA
   events on the launching stream. */
double plamo_cuda_time_decode(struct plamo_cuda *, struct model *, uint64_t repeats);
/* Same for the standalone GEMV over `repeats` launches. */
double plamo_cuda_time_gemv(struct plamo_cuda *, const uint16_t *w, const float *x, float *y,
                            uint64_t rows, uint64_t cols, uint64_t repeats);
/* Same, launch i reading the weights of copy i % copies (copies consecutive
   [rows, cols] matrices at w): rotating through more bytes than L2 holds
   makes each launch stream its weights from HBM. */
double plamo_cuda_time_gemv_copies(struct plamo_cuda *, const uint16_t *w, uint64_t copies, const float *x, float *y,
                                   uint64_t rows, uint64_t cols, uint64_t repeats);
/* Same for `repeats` back-to-back prompt projections (split + GEMM). */
double plamo_cuda_time_gemm(struct plamo_cuda *, const float *x, const uint16_t *w, float *y, uint64_t tokens,
                            uint64_t rows, uint64_t cols, uint64_t repeats);
/* Kernels launched by the library since open (counts every launch and every
   kernel node of a launched graph). */
uint64_t plamo_cuda_kernel_launches(const struct plamo_cuda *);
/* How a decode step of `model` runs, preparing it if needed: "persistent" (one
   launch per token: every projection, attention and the greedy choice in one
   kernel with one CTA per SM) or "graph: <reason>" (one CUDA graph of
   per-projection kernels, with the reason the one-launch step does not
   apply). NULL when the model is not prepared. Valid until the next call. */
const char *plamo_cuda_decode_path(struct plamo_cuda *, struct model *);
/* One persistent decode step of `token` (as plamo_cuda_forward_greedy, the
   step is committed) that also records device timestamps (ns, %globaltimer)
   of CTA 0 into stamps: [0] kernel start; [1 + b] when its consumer warps
   passed grid barrier b, b < B = 5 * layers + 1 (per layer: after qkv, after
   attention, after o_proj, after gate_up, after down_proj; last: after the
   head); [1 + B + p] when its producer warp issued the first weight chunk of
   projection p, p < 4 * layers + 1 (qkv, o_proj, gate_up, down_proj per
   layer, then the head).
   On the graph path (per-projection kernels) a graph of the same step with
   timestamping launches is captured and run once instead: six stamps per
   launch, 5 * layers + 1 launches in step order (per layer qkv, attention,
   o_proj, gate_up, down_proj; then the head): [0] the first CTA's entry,
   [1] the last CTA past its dependency wait and prologue, [2] the first CTA
   done with its weight stream (attention: done), [3] the last one, [4] the
   last CTA past its dependency wait alone, [5] the last CTA's entry.
   Returns the number of stamps, or -1 when capacity is too small. */
double plamo_cuda_decode_trace(struct plamo_cuda *, struct model *, uint64_t token, uint64_t *stamps,
                               uint64_t capacity);

/* Synthetic BF16 weights generated on the device: value(i) =
   mean + std * z(seed, i), z = (sum of 12 hash bytes - 1530) / 256, rounded to
   BF16 (plamo_synthetic.h restates it for the host). Registers the range
   [host_key, host_key + count*2) like plamo_cuda_preload without reading it. */
int plamo_cuda_preload_synthetic(struct plamo_cuda *, const void *host_key, uint64_t count,
                                 uint64_t seed, float mean, float std);
/* Copy the HBM bytes registered under host key range [key, key+bytes) to dst. */
int plamo_cuda_read_weights(struct plamo_cuda *, const void *key, void *dst, uint64_t bytes);
int plamo_cuda_fill_synthetic_bf16(struct plamo_cuda *, uint16_t *device_dst, uint64_t count,
                                   uint64_t seed, float mean, float std);
int plamo_cuda_fill_synthetic_f32(struct plamo_cuda *, float *device_dst, uint64_t count,
                                  uint64_t seed, float mean, float std);
/* A shard of a synthetic [*, full_cols] tensor: registers under host_key the
   rows row_start[i] .. row_start[i]+row_count[i]-1 (segments in order) and
   columns col0 .. col0+cols-1 of the tensor plamo_cuda_preload_synthetic
   would generate with the same seed, bit for bit. */
int plamo_cuda_preload_synthetic_rows(struct plamo_cuda *, const void *host_key, uint64_t cols,
                                      uint64_t full_cols, uint64_t col0, const uint64_t *row_start,
                                      const uint64_t *row_count, unsigned segments, uint64_t seed,
                                      float mean, float std);

/* Tensor parallelism (no counterpart in the reference, which runs on one
   GPU): one process and one context per GPU, `size` ranks (2..8). Each rank
   prepares its shard of the model: the descriptor tree of the full model with
   qh/size query heads, kh/size KV heads and intermediate/size MLP rows (rank
   r holds query heads [r*qh/size, ...), KV heads [r*kh/size, ...), gate and
   up rows [r*I/size, ...) and the matching o_proj and down_proj columns), the
   full embedding, `vocab` = the full vocabulary, and `head` pointing at the
   rank's `vocab_rows` head rows starting at global row `vocab_offset`.
   tp_prepare prepares that shard, allocates this rank's exchange buffer and
   returns its CUDA IPC handle; after every rank has called it, tp_connect
   maps the peers' buffers (handles indexed by rank, `size` entries). From then
   on forward / prefill / verify / generate of the shard run tensor-parallel:
   the o_proj and down_proj partial sums are pushed into every peer's buffer
   by the projection kernels themselves and summed in rank order by the
   consumer's prologue (one exchange per attention block and per MLP block,
   P2P stores over NVLink, no multicast), and the greedy token is the first
   maximum over the ranks' head slices. Every rank must make the same calls
   in the same order; a peer that does not arrive within 2 s makes the call
   fail (-1). The host logits hold only this rank's slice
   [vocab_offset, vocab_offset + vocab_rows). */
#define PLAMO_CUDA_TP_MAX 8
struct plamo_cuda_tp_handle {
    unsigned char bytes[64];
};
int plamo_cuda_tp_prepare(struct plamo_cuda *, struct model *shard, unsigned rank, unsigned size,
                          uint64_t vocab_offset, uint64_t vocab_rows, struct plamo_cuda_tp_handle *handle);
int plamo_cuda_tp_connect(struct plamo_cuda *, struct model *shard, const struct plamo_cuda_tp_handle *handles);

#ifdef __cplusplus
}
#endif
#endif
