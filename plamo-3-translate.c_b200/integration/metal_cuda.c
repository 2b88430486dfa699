/* The reference's GPU backend interface (runtime/metal.h) implemented over
 * this library's CUDA backend (include/plamo_cuda.h).
 *
 * A maintainer builds the reference engine with this file in place of
 * runtime/metal*.m and links libplamo_cuda.so:
 *
 *   cc -c integration/metal_cuda.c -I<reference>/runtime -I<this repo>/include
 *   cc ... metal_cuda.o -L<this repo>/plamo-3-translate.c_b200/lib -lplamo_cuda -lstdc++
 *
 * Every plamo_metal_* entry forwards to the plamo_cuda_* entry of the same
 * name with the same arguments and tri-state result (1 done, 0 declined with
 * nothing changed so the caller may use its CPU path, -1 failed). As the
 * reference's Metal module does (runtime/metal.m:901-946), a successful open
 * installs the compute hooks of runtime/compute.h, so the engine's assembly
 * entry points (plamo_forward, plamo_prefill, plamo_mlp_branch, batched
 * projections) run on the GPU, and close removes them. A projection the GPU
 * declines runs on the reference's own CPU kernel, as in the Metal module.
 *
 * The host KV arrays are kept current after every call (copy_kv_to_host),
 * because the reference's engine, prompt cache and CPU fallback read them.
 *
 * The reference's headers come first: include/plamo_model.h then sees their
 * include guards and does not define the shared records a second time.
 */
#include "compute.h"
#include "metal.h"

#include "plamo_cuda.h"

#include <stdio.h>
#include <string.h>

static struct plamo_cuda *as_cuda(const struct plamo_metal *b) { return (struct plamo_cuda *)(uintptr_t)b; }

static void hook_matmul(const struct plamo_matmul *p, void *context) {
    if (plamo_cuda_linear(context, p) != 1) plamo_bf16_matmul_core(p);
}
static void hook_matvec(const uint16_t *w, const float *x, float *y, uint64_t rows, uint64_t columns,
                        void *context) {
    const struct plamo_matmul p = {w, x, y, rows, columns, 1, columns, rows};
    hook_matmul(&p, context);
}
static int hook_mlp(const struct mlp *p, float *states, uint64_t tokens, void *context) {
    return plamo_cuda_mlp(context, p, states, tokens);
}
static int hook_forward(struct model *m, uint64_t token, void *context) {
    return plamo_cuda_forward(context, m, token);
}
static int hook_prefill(struct model *m, const uint32_t *ids, uint64_t tokens, float *states, void *context) {
    return plamo_cuda_prefill(context, m, ids, tokens, states);
}

struct plamo_metal *plamo_metal_open(const struct plamo_metal_config *config, char *error, size_t cap) {
    if (!config || plamo_compute_context) {
        if (error && cap) snprintf(error, cap, "a GPU backend is already installed or the configuration is missing");
        return NULL;
    }
    struct plamo_cuda_config c;
    memset(&c, 0, sizeof c);
    c.reserve = config->reserve;
    c.copy_kv_to_host = 1;
    struct plamo_cuda *cuda = plamo_cuda_open(&c, error, cap);
    if (!cuda) return NULL;
    if (config->memory == PLAMO_METAL_RESIDENT)
        for (size_t i = 0; i < config->count; ++i)
            if (!plamo_cuda_preload(cuda, config->maps[i].base, config->maps[i].bytes)) {
                struct plamo_cuda_info info;
                plamo_cuda_get_info(cuda, &info);
                if (error && cap) snprintf(error, cap, "%s", info.note);
                plamo_cuda_close(cuda);
                return NULL;
            }
    plamo_compute_context = cuda;
    plamo_matvec_kernel = hook_matvec;
    plamo_matmul_kernel = hook_matmul;
    plamo_mlp_kernel = hook_mlp;
    plamo_forward_kernel = hook_forward;
    plamo_prefill_kernel = hook_prefill;
    return (struct plamo_metal *)(void *)cuda;
}

void plamo_metal_close(struct plamo_metal *b) {
    if (!b) return;
    if (plamo_compute_context == (void *)b) {
        plamo_matvec_kernel = NULL;
        plamo_matmul_kernel = NULL;
        plamo_mlp_kernel = NULL;
        plamo_forward_kernel = NULL;
        plamo_prefill_kernel = NULL;
        plamo_compute_context = NULL;
    }
    plamo_cuda_close(as_cuda(b));
}

void plamo_metal_maintain(struct plamo_metal *b) { plamo_cuda_maintain(as_cuda(b)); }

void plamo_metal_get_info(const struct plamo_metal *b, struct plamo_metal_info *out) {
    struct plamo_cuda_info i;
    plamo_cuda_get_info(as_cuda(b), &i);
    memset(out, 0, sizeof *out);
    snprintf(out->device, sizeof out->device, "%s", i.device);
    snprintf(out->precision, sizeof out->precision, "fp32");
    snprintf(out->weight_storage, sizeof out->weight_storage, "bf16");
    snprintf(out->note, sizeof out->note, "%s", i.note);
    out->dispatches = i.launches;
    out->command_buffers = i.graph_launches;
    out->fused_decodes = i.forwards;
    out->fused_prefills = i.prefills;
    out->errors = i.errors;
    out->allocated_bytes = i.allocated_bytes;
    out->verification_batches = i.verification_batches;
    out->verified_tokens = i.verified_tokens;
    out->committed_tokens = i.committed_tokens;
    out->gpu_seconds = i.gpu_seconds;
}

int plamo_metal_preload(struct plamo_metal *b, const void *p, uint64_t n) { return plamo_cuda_preload(as_cuda(b), p, n); }
int plamo_metal_warm_cache(struct plamo_metal *b) { return plamo_cuda_warm_cache(as_cuda(b)); }
int plamo_metal_prepare_model(struct plamo_metal *b, struct model *m) {
    return plamo_cuda_prepare_model(as_cuda(b), m);
}
int plamo_metal_forward(struct plamo_metal *b, struct model *m, uint64_t token) {
    return plamo_cuda_forward(as_cuda(b), m, token);
}
int plamo_metal_prefill(struct plamo_metal *b, struct model *m, const uint32_t *ids, uint64_t tokens, float *states) {
    return plamo_cuda_prefill(as_cuda(b), m, ids, tokens, states);
}
int plamo_metal_verify(struct plamo_metal *b, struct model *m, const uint32_t *ids, uint64_t tokens, uint32_t *next) {
    return plamo_cuda_verify(as_cuda(b), m, ids, tokens, next);
}
int plamo_metal_commit(struct plamo_metal *b, struct model *m, uint64_t index) {
    return plamo_cuda_commit(as_cuda(b), m, index);
}
int plamo_metal_linear(struct plamo_metal *b, const struct plamo_matmul *p) { return plamo_cuda_linear(as_cuda(b), p); }
int plamo_metal_mlp(struct plamo_metal *b, const struct mlp *p, float *states, uint64_t tokens) {
    return plamo_cuda_mlp(as_cuda(b), p, states, tokens);
}
