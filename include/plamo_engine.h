/* PLaMo-3 translation engine on Linux over the CUDA backend: the request path
 * of reference runtime/engine.h:48-62 (open, prepare, tokenize, translate with
 * streamed token callbacks), so a CLI or worker written against that header
 * drives the B200 backend.
 *
 * Composition: the tokenizer (plamo_tokenizer.h) wraps the text in the
 * translation template and encodes it; the checkpoint shards are mapped and
 * bound into run-time descriptors (plamo_safetensors.h, plamo_layout.h); the
 * CUDA backend (plamo_cuda.h) holds the weights in HBM, prefills the prompt
 * and decodes greedily on the device; the fixed template prefix of each
 * direction is snapshotted on the device once (plamo_engine_prepare) and
 * restored for every request that starts with it.
 *
 * Differences from the reference, all following from the platform:
 *   - the reference compiles the model name and file paths into the binary;
 *     here plamo_engine_open_files takes them, and plamo_engine_open (the
 *     reference's signature) reads them from PLAMO_MODEL_DIR (tokenizer.jsonl
 *     and *.safetensors shards) and PLAMO_MODEL_PROFILE ("0.8b", "2b", "8b",
 *     "31b"; default "8b");
 *   - struct plamo_engine_info carries the CUDA backend's counters where the
 *     reference carries Metal's and its weight cache's;
 *   - there is no CPU path: the token loop runs on the GPU or the call fails
 *     (PLAMO_BACKEND_CPU is refused at open);
 *   - plamo_engine_close exists (the reference keeps one engine per process).
 * Requests are serialised: one engine, one request at a time, not thread-safe.
 */
#ifndef PLAMO_ENGINE_H
#define PLAMO_ENGINE_H
#include <stddef.h>
#include <stdint.h>

#include "plamo_cuda.h"
#include "plamo_layout.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference runtime/engine.h:8. RESIDENT uploads every shard at open; AUTO and
   STREAM upload at the first prepare or request (HBM holds the weights either
   way). */
enum plamo_memory_mode { PLAMO_MEMORY_AUTO, PLAMO_MEMORY_RESIDENT, PLAMO_MEMORY_STREAM };
/* reference runtime/engine.h:9-14 with the GPU backend renamed. */
enum plamo_backend { PLAMO_BACKEND_AUTO, PLAMO_BACKEND_CPU, PLAMO_BACKEND_CUDA };

/* reference runtime/engine.h:16-27 (gpu: the CUDA backend's counters). */
struct plamo_engine_info {
    const char *memory_mode;
    const char *backend;
    char memory_note[256];
    uint64_t weight_bytes, preloaded_weight_bytes, reclaimable_bytes, physical_bytes;
    uint64_t prefix_tokens[2], prefix_bytes;
    struct plamo_cuda_info gpu;
    unsigned threads, speculative_tokens;
    double load_seconds, preload_seconds, prefix_seconds;
};

/* reference runtime/engine.h:28-40; fields with no meaning on this backend
   (staged/read/cache/mapped counters of the reference's streaming weights)
   stay zero. */
struct plamo_result {
    uint64_t prompt_tokens, completion_tokens, decode_steps, staged_bytes, read_calls;
    uint64_t cache_hits, cache_hit_bytes, cache_misses;
    uint64_t decode_staged_bytes, decode_read_calls, decode_command_buffers, decode_gpu_dispatches;
    uint64_t decode_mapped_bytes;
    uint64_t prefill_command_buffers, prefill_gpu_dispatches;
    uint64_t cached_prompt_tokens;
    uint64_t prefill_logits_hash, prefill_state_hash, logits_hash, state_hash;
    uint64_t speculative_batches, speculative_tokens, proposed_tokens, accepted_tokens;
    double tokenize_seconds, prefill_seconds, decode_seconds, first_token_seconds, total_seconds;
    double decode_gpu_seconds, prefill_gpu_seconds;
    double draft_seconds;
    const char *finish_reason;
};

/* reference runtime/engine.h:41-45: prefill(prompt tokens) once, then
   token(id, its bytes) per emitted token; returning 0 cancels. */
struct plamo_callbacks {
    void (*prefill)(uint64_t prompt_tokens, void *context);
    int (*token)(uint32_t id, const char *bytes, size_t count, void *context);
    void *context;
};

/* Where the model is (no counterpart in the reference, which compiles these
   in). `config` is used when `profile` is NULL. max_context bounds the rows
   of full-attention layers (0: 8192 + 16); device is the CUDA ordinal. */
struct plamo_engine_files {
    const char *tokenizer;
    const char *const *weights;
    unsigned weight_count;
    const char *profile;
    const struct plamo_model_config *config;
    uint64_t max_context;
    int device;
};

struct plamo_engine;

/* Open from explicit files. NULL with a message on failure. */
struct plamo_engine *plamo_engine_open_files(const struct plamo_engine_files *, enum plamo_memory_mode,
                                             int tokenizer_only, unsigned threads, enum plamo_backend,
                                             struct plamo_engine_info *, char *error, size_t cap);
/* reference runtime/engine.h:48-50; files from PLAMO_MODEL_DIR / PLAMO_MODEL_PROFILE. */
struct plamo_engine *plamo_engine_open(enum plamo_memory_mode, int tokenizer_only, unsigned threads,
                                       enum plamo_backend, struct plamo_engine_info *, char *error, size_t cap);
void plamo_engine_close(struct plamo_engine *);
/* reference runtime/engine.h:51 */
void plamo_engine_get_info(struct plamo_engine *, struct plamo_engine_info *);
/* reference runtime/engine.h:52 */
void plamo_engine_maintain_memory(struct plamo_engine *);
/* reference runtime/engine.h:53-57: upload and prepare the model, then prefill
   and snapshot on the device the fixed template prefix of both directions
   (PLAMO_PREFIX_CACHE=0 skips the snapshots). Idempotent; the request state
   is reset afterwards. 1, or 0 with a message. */
int plamo_engine_prepare(struct plamo_engine *, char *error, size_t cap);
/* reference runtime/engine.h:58-59: ids borrowed until the next call; UINT64_MAX on error. */
uint64_t plamo_engine_tokenize(struct plamo_engine *, const char *text, unsigned direction, const uint32_t **ids,
                               char *error, size_t cap);
/* reference runtime/engine.h:60-62: greedy translation of `text` (direction 1:
   English to Japanese, 2: Japanese to English, 0: raw continuation), at most
   max_tokens (1..4096) tokens, stopping at the end-of-text ids 1 and 16. 1 on
   success (result->finish_reason "stop", "length" or "cancelled"), or 0 with
   a message. */
int plamo_engine_translate(struct plamo_engine *, const char *text, unsigned direction, unsigned max_tokens,
                           const struct plamo_callbacks *, struct plamo_result *, char *error, size_t cap);

/* The worker's per-request telemetry (reference runtime/worker.c:84-184,
   report_result and report_compute) as one JSON object: {"event":"done",
   "finish_reason", "usage", "timings", "weight_io", "process_peak_rss_bytes",
   "verification" (the result hashes), "speculative", "compute"}, with the
   reference's keys; "compute" carries this backend's counters (launches as
   gpu_dispatches, graph launches as command_buffers, forwards, prefills,
   verification and commit counts, errors, device seconds, allocated, weight,
   KV and workspace bytes, the decode path and the last note). `result` may be
   NULL (the compute object alone, as the worker's readiness report). Writes
   at most cap bytes including the terminating NUL and returns the length the
   whole object needs (snprintf's rule), or 0 on a NULL engine. */
size_t plamo_engine_report_json(struct plamo_engine *, const struct plamo_result *result, char *out, size_t cap);

#ifdef __cplusplus
}
#endif
#endif
