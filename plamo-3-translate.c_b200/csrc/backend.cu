// Host side of the B200 backend: context, HBM weight registry, per-model
// device state, the decode step as one CUDA graph, the layer-major prompt,
// speculative verification/commit and the greedy request loop.
//
// Interface: include/plamo_cuda.h (drop-in for reference runtime/metal.h).
#include "../../include/plamo_cuda.h"
#include "../../include/plamo_synthetic.h"
#include "common.cuh"
#include "gemv.cuh"
#include "attention.cuh"
#include "rows.cuh"
#include "gemm_tc.cuh"
#include "persist.cuh"
#include "tp.cuh"

#include <cudaTypedefs.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <vector>

using namespace plamo;

namespace {

constexpr float kPostMixerOffset = 0.2f;                 // reference src/layer.s:51
constexpr float kPostMlpOffset = 0.08944271909999159f;   // reference src/model.s:112
constexpr uint64_t kVerifyMax = PLAMO_CUDA_VERIFY_MAX;
// Split-K scratch per model: splits x tokens x rows of the small-token
// projections (<= 16 tokens, fewer row tiles than SMs: at most
// 2 x 148 x 128 rows' worth per token).
constexpr uint64_t kSplitkFloats = 16ull * 40960;

// Device staging of plamo_cuda_linear_static: a fixed array in the module
// instead of cudaMalloc'd buffers. Every GPU that loads this library holds it
// (16 MiB) until the process exits; the input rows are staged at its start,
// the output rows right after them.
constexpr uint64_t kStaticLinearFloats = PLAMO_CUDA_LINEAR_STATIC_FLOATS;

struct Range {
    uintptr_t host;
    uint64_t bytes;
    char *dev;
};

// cos|sin table of one (frequency set, dim, concentration), positions rows.
struct Rope {
    std::vector<float> freq;
    uint64_t dim;
    uint32_t scale_bits;
    uint64_t positions;
    float *dev;
};

struct DLayer {
    struct layer *host;
    const uint16_t *qkv_w, *qn, *kn, *o_w, *pre, *post, *mpre, *mpost, *gu, *down;
    // KV slots [0, ring) in pages of kKvPageRows rows from the context's pool:
    // pages[i] (host mirror) and d_pages[i] (device table) hold page i's base,
    // the first `mapped` of them taken from the pool, the rest the pool's
    // zeroed spare page.
    std::vector<float *> pages;
    float **d_pages;
    uint64_t mapped;
    uint64_t ring, capacity;
    int sliding;
    Rope *rope;
    float scale;
    uint64_t appended;  // committed rows of the request (host mirror of d_appended)
    bool stale;         // host rows are canonical: upload before the next use
    uint64_t host_hash; // FNV-1a of the newest host K row written by this backend
};

// Tensor-parallel state of a shard (see tp.cuh). The exchange buffer has the
// same layout on every rank:
//   decode partials [2L][tp][H] {f32 value, u32 tag} pairs (tagged, no flags
//   needed), decode flags [2L][tp] u32 (unused by the tagged points) (point 2l after
//   o_proj of layer l, 2l+1 after its down_proj); prompt partials
//   [2][tp][tmax*H] f32 (alternating points), prompt flags [2L][tp] u32;
//   argmax slots [verify max][tp][4] u32.
struct TpState {
    bool active = false;
    uint32_t rank = 0, size = 0;
    uint64_t voff = 0;
    char *xbuf = nullptr;
    char *peer[kTpMax] = {};
    uint64_t off_dparts = 0, off_dflags = 0, off_pparts = 0, off_pflags = 0, off_args = 0, bytes = 0;
    uint32_t *tickets = nullptr;  // [4L] local: decode points, then prompt points
    uint32_t *epoch = nullptr;
    float *lval = nullptr;        // this rank's per-row best value [verify max]
    uint32_t *lidx = nullptr;     // and local index
};

struct DModel {
    struct model *host;
    uint64_t H, QH, KH, D, I, V, L, QW, AW, KVW;
    uint64_t Vh;  // head rows held here: V, or the rank's slice of a tensor-parallel shard
    TpState tp;
    const uint16_t *emb, *norm, *head;
    std::vector<DLayer> layers;
    uint64_t *d_appended;
    // decode step
    float *state[2], *final_state, *normalized, *logits;
    float *qkv, *q, *attn, *branch, *mid, *part;
    uint32_t *tickets, *arg_idx, *arg_nan, *d_token, *d_next, *d_error;
    float *arg_val, *arg_val2;
    uint32_t splits, gemv_grid;
    float last_margin = 0.0f;  // top-2 logit margin of the last greedy decode step
    // prompt / verification
    uint64_t tmax;
    float *p_states, *p_norm, *p_qkv, *p_q, *p_attn, *p_branch, *p_gu, *p_logits, *p_part;
    float *p_rotk;  // rotated keys of the blocked prompt attention [max capacity][KVW]
    uint32_t *p_ids, *p_next, *p_tickets;
    uint16_t *p_split;  // BF16 hi/mid/lo terms of a projection input, 3 x [T][K]
    uint16_t *p_glu;    // BF16 terms of the SwiGLU output of a fused gate/up projection, 3 x [T][I]
    float *p_splitk;    // split-K partial tiles of small-token projections
    float *v_kv;  // [L][kVerifyMax][2][KVW]
    uint64_t verify_count = 0, verify_committed = 0;
    bool verify_valid = false;
    // graph
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t graph_exec = nullptr;
    std::vector<cudaGraphExec_t> layer_exec;  // plamo_cuda_layer: one recorded step per layer
    std::vector<uint64_t> layer_nodes;
    uint64_t graph_nodes = 0;
    // persistent decode (one launch per token, single GPU)
    bool pt_ready = false;
    PtParams pt{};
    uint32_t pt_grid = 0;
    size_t pt_smem = 0;
    char pt_reason[96] = "";  // why the persistent step is not used
    unsigned long long *trace = nullptr;  // timeline records of a traced graph step (plamo_cuda_decode_trace)
    uint32_t trace_slot = 0;
    std::vector<void *> allocations;
    std::vector<uintptr_t> signature;  // host descriptor identity at prepare time
};

}  // namespace

// File scope: the device array itself. Host code only ever uses the address
// returned by cudaGetSymbolAddress (the name is a host-side stand-in).
static __device__ __align__(256) float g_linear_static_scratch[kStaticLinearFloats];

// Pages of KV rows shared by every request of a context with the same row
// width: chunks of kKvChunkPages pages are allocated as requests need them
// and stay with the context; pages return to `free` when a request resets or
// is released.
constexpr uint64_t kKvChunkPages = 16;
struct KvPool {
    std::vector<float *> chunks;
    std::vector<float *> free;
    float *spare = nullptr;  // zeroed page for the unmapped entries of page tables
    uint64_t used = 0;
};

struct plamo_cuda {
    int device;
    cudaStream_t stream;
    cudaEvent_t ev0, ev1;
    plamo_cuda_config config;
    plamo_cuda_info info;
    std::vector<Range> ranges;
    std::vector<std::unique_ptr<Rope>> ropes;
    std::map<struct model *, std::unique_ptr<DModel>> models;
    uint32_t *pinned_u32;  // small pinned staging (tokens, ids)
    uint64_t pinned_capacity;
    int sm_count;
    int smem_optin;
    int smem_per_sm;
    bool pdl;
    bool bulk_gemv;
    int gemv_ring_kb;
    int tc_stages;  // tcgen05 projection ring depth (0: as many as shared memory holds)
    int tc_tokm;    // token-major tcgen05 tiles for prompts: -1 by waves, 0 never, 1 always (PLAMO_CUDA_TC_TOKM)
    int tc_tokn;    // token-major tile width: 0 by waves, else 144, 160 or 192 (PLAMO_CUDA_TC_TOKN)
    int tc_glu;     // prompt gate/up projection fused with SwiGLU (PLAMO_CUDA_TC_GLU, default 1)
    float draft_margin;         // PLAMO_DRAFT_MIN_MARGIN, or -1: the reference's default rule
    unsigned draft_min_tokens;  // PLAMO_DRAFT_MIN_TOKENS, or 0: the reference's default rule
    bool tc_gemm;
    bool prompt_attn;  // blocked prompt attention (PLAMO_CUDA_PROMPT_ATTN=0 disables)
    int prompt_rows;   // its query rows per CTA: 64, 32, or 0 to choose by size (PLAMO_CUDA_PROMPT_ROWS)
    int prompt_bufs;   // key/value tile buffers of the 32-row kernel (PLAMO_CUDA_PROMPT_BUFS: 1, or 2)
    bool persistent;   // one-launch decode step where the shapes allow (opt-in: PLAMO_CUDA_PERSISTENT=1)
    bool cooperative;  // the device supports cooperative launches
    uint32_t pt_piece;  // bytes per bulk copy of the persistent step (PLAMO_CUDA_PT_PIECE_KB)
    int pt_stages;      // ring stages of the persistent step (PLAMO_CUDA_PT_STAGES; 0: as many as fit)
    int gemv_ctas;
    uint32_t *sink;
    float *static_scratch;  // device address of g_linear_static_scratch (set on first use)
    std::map<uint64_t, KvPool> kv_pools;  // by floats per K row (kv heads x head dim)
    char *staging = nullptr;   // grow-only device staging of linear / mlp (host buffers in and out)
    uint64_t staging_bytes = 0;
};

// A template-prefix snapshot (reference runtime/prompt_cache.c:5-13 keeps the
// model, the ids and each layer's width and RoPE scale beside the rows). The
// rows live in HBM as [layer][K|V][tokens][kv width]: the device rings hold
// unrotated keys, so the rotated copy the reference also stores is not needed.
struct plamo_cuda_prompt_cache {
    const struct model *model;
    const plamo_cuda *owner;
    int device;
    uint64_t tokens, layers, kvw, bytes;
    uint32_t ids[PLAMO_CUDA_PREFIX_LIMIT];
    std::vector<uint64_t> width;
    std::vector<uint32_t> scale_bits;
    float *rows;
};

// Requests decoded together (plamo_cuda_batch_*): model 0 lends its weights
// and prompt workspace, every model keeps its own KV.
struct plamo_cuda_batch {
    plamo_cuda *c;
    std::vector<struct model *> hosts;
    uint32_t B;
    DecodeAttnParams *d_attn;  // [L][B]
    uint64_t **d_counters;     // [B] each model's per-layer row counters
    uint32_t *d_tokens;        // [B] this step's tokens, then the greedy next ones
    cudaGraph_t graph;
    cudaGraphExec_t exec;
    uint64_t nodes;
};

namespace {

bool note(plamo_cuda *c, const char *what, cudaError_t e) {
    if (e == cudaSuccess) return true;
    c->info.errors++;
    snprintf(c->info.note, sizeof c->info.note, "%s: %s", what, cudaGetErrorString(e));
    return false;
}

uint32_t float_to_bits(float f) {
    uint32_t b;
    memcpy(&b, &f, 4);
    return b;
}

// ---- exact RoPE tables (host) ------------------------------------------
// The reference builds its GPU tables on the CPU with its own sin/cos
// (runtime/metal_model.m:145-175 -> src/rope_table.s, src/trig.s): angle =
// fp32(position) * freq[j] in FP32, then sin/cos in double by reduction modulo
// 2*pi and the Taylor series of sin(r)/r and cos(r) to r^16, each rounded to
// FP32 and multiplied by the concentration in FP32. Restated here so the
// device tables hold the same bits.
const double kTwoPi = 6.283185307179586;
const double kSinSeries[8] = {1.0 / 355687428096000.0, -1.0 / 1307674368000.0,
                              1.0 / 6227020800.0,      -1.0 / 39916800.0,
                              1.0 / 362880.0,          -1.0 / 5040.0,
                              1.0 / 120.0,             -1.0 / 6.0};
const double kCosSeries[8] = {1.0 / 20922789888000.0, -1.0 / 87178291200.0,
                              1.0 / 479001600.0,      -1.0 / 3628800.0,
                              1.0 / 40320.0,          -1.0 / 720.0,
                              1.0 / 24.0,             -1.0 / 2.0};

void sincos_exact(double angle, float *s, float *c) {
    double n = std::rint(angle / kTwoPi);
    double r = std::fma(-n, kTwoPi, angle);
    double r2 = r * r;
    double p = kSinSeries[0];
    for (int k = 1; k < 8; ++k) p = std::fma(p, r2, kSinSeries[k]);
    p = std::fma(p, r2, 1.0);
    volatile double sp = p * r;
    *s = static_cast<float>(sp);
    p = kCosSeries[0];
    for (int k = 1; k < 8; ++k) p = std::fma(p, r2, kCosSeries[k]);
    p = std::fma(p, r2, 1.0);
    *c = static_cast<float>(p);
}

void build_rope_rows(const float *freq, uint64_t dim, float scale, uint64_t from, uint64_t to,
                     float *out) {
    const uint64_t half = dim / 2;
    for (uint64_t pos = from; pos < to; ++pos) {
        float *row = out + (pos - from) * dim;
        const float p = static_cast<float>(pos);
        for (uint64_t j = 0; j < half; ++j) {
            volatile float angle = freq[j] * p;
            float s, c;
            sincos_exact(static_cast<double>(angle), &s, &c);
            volatile float cs = c * scale, ss = s * scale;
            row[j] = cs;
            row[half + j] = ss;
        }
    }
}

Rope *get_rope(plamo_cuda *c, const float *freq, uint64_t dim, float scale, uint64_t positions) {
    const uint32_t bits = float_to_bits(scale);
    for (auto &r : c->ropes)
        if (r->dim == dim && r->scale_bits == bits && r->positions >= positions &&
            !memcmp(r->freq.data(), freq, dim / 2 * sizeof(float)))
            return r.get();
    auto r = std::make_unique<Rope>();
    r->freq.assign(freq, freq + dim / 2);
    r->dim = dim;
    r->scale_bits = bits;
    r->positions = positions;
    std::vector<float> host(positions * dim);
    build_rope_rows(freq, dim, scale, 0, positions, host.data());
    if (!note(c, "rope alloc", cudaMalloc(&r->dev, host.size() * 4))) return nullptr;
    if (!note(c, "rope copy", cudaMemcpy(r->dev, host.data(), host.size() * 4, cudaMemcpyHostToDevice))) {
        cudaFree(r->dev);
        return nullptr;
    }
    c->info.allocated_bytes += host.size() * 4;
    c->ropes.push_back(std::move(r));
    return c->ropes.back().get();
}

// ---- weight registry -----------------------------------------------------
const Range *find_range(plamo_cuda *c, const void *p, uint64_t bytes) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    for (const Range &r : c->ranges)
        if (a >= r.host && a + bytes <= r.host + r.bytes) return &r;
    return nullptr;
}
const uint16_t *resolve(plamo_cuda *c, const void *p, uint64_t bytes, bool upload) {
    if (!p) return nullptr;
    const Range *r = find_range(c, p, bytes);
    if (!r && upload) {
        if (!plamo_cuda_preload(c, p, bytes)) return nullptr;
        r = find_range(c, p, bytes);
    }
    if (!r) return nullptr;
    return reinterpret_cast<const uint16_t *>(r->dev + (reinterpret_cast<uintptr_t>(p) - r->host));
}

// ---- launches ------------------------------------------------------------
template <typename... KArgs, typename... Args>
bool launch(plamo_cuda *c, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
            Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    if (c->pdl) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    c->info.launches++;
    return note(c, "launch", cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...));
}

template <int PRO, int EPI>
bool launch_gemv_shape(plamo_cuda *c, const GemvParams &p, int U, uint32_t grid, size_t smem) {
    switch (U) {
    case 4: return launch(c, gemv_kernel<PRO, EPI, 4>, dim3(grid), dim3(kGemvThreads), smem, p);
    case 2: return launch(c, gemv_kernel<PRO, EPI, 2>, dim3(grid), dim3(kGemvThreads), smem, p);
    case 1: return launch(c, gemv_kernel<PRO, EPI, 1>, dim3(grid), dim3(kGemvThreads), smem, p);
    default: return launch(c, gemv_kernel<PRO, EPI, 0>, dim3(grid), dim3(kGemvThreads), smem, p);
    }
}

// Shared-memory carveout preference (percent of the unified L1/shared
// array, -1: the driver's choice). Kernels whose CTAs are to share an SM
// must run with the same carveout: an SM only changes its split when idle.
template <typename K>
void prefer_carveout(K kernel, int carveout) {
    if (carveout >= 0) cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, carveout);
}

// Allow each kernel the device's opt-in shared memory minus its static part.
template <typename K>
void allow_smem(K kernel, int optin, int carveout) {
    cudaFuncAttributes a{};
    if (cudaFuncGetAttributes(&a, kernel) == cudaSuccess)
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             optin - static_cast<int>(a.sharedSizeBytes));
    prefer_carveout(kernel, carveout);
}

template <int PRO, int EPI>
void set_gemv_smem_limits(int optin, int carveout) {
    allow_smem(gemv_bulk_kernel<PRO, EPI, 1, false>, optin, carveout);
    allow_smem(gemv_bulk_kernel<PRO, EPI, 2, false>, optin, carveout);
    allow_smem(gemv_bulk_kernel<PRO, EPI, 4, false>, optin, carveout);
    allow_smem(gemv_bulk_kernel<PRO, EPI, 1, true>, optin, carveout);
    allow_smem(gemv_bulk_kernel<PRO, EPI, 2, true>, optin, carveout);
    allow_smem(gemv_bulk_kernel<PRO, EPI, 4, true>, optin, carveout);
    allow_smem(gemv_kernel<PRO, EPI, 4>, optin, carveout);
    allow_smem(gemv_kernel<PRO, EPI, 2>, optin, carveout);
    allow_smem(gemv_kernel<PRO, EPI, 1>, optin, carveout);
    allow_smem(gemv_kernel<PRO, EPI, 0>, optin, carveout);
}

// Grid of a projection: one CTA per SM (times the configured factor), fewer
// when there are fewer output units, more when the per-block partials would
// not fit in shared memory.
uint32_t gemv_grid(plamo_cuda *c, uint64_t units, uint64_t cols, int U, int pair, size_t *smem) {
    uint64_t grid = std::min<uint64_t>(units, static_cast<uint64_t>(c->sm_count) * c->gemv_ctas);
    if (!grid) grid = 1;
    const uint64_t segs = U ? cols / (256ull * U) : 1;
    const uint64_t cols_pad = (cols + 3) & ~3ull;
    for (;;) {
        const uint64_t per = (units + grid - 1) / grid;
        const size_t bytes = (cols_pad + per * segs * pair) * sizeof(float);
        if (bytes + 1024 <= static_cast<size_t>(c->smem_optin) || grid >= units) {
            *smem = bytes;
            return static_cast<uint32_t>(grid);
        }
        grid *= 2;
        if (grid > units) grid = units;
    }
}

int gemv_chunks(const void *w, uint64_t cols) {
    if (reinterpret_cast<uintptr_t>(w) % 16) return 0;
    if (cols % 1024 == 0) return 4;
    if (cols % 512 == 0) return 2;
    if (cols % 256 == 0) return 1;
    return 0;
}

template <int PRO, int EPI>
bool gemv(plamo_cuda *c, GemvParams p, uint32_t *grid_out = nullptr) {
    if constexpr (PRO == PRO_RESID_NORM)
        if (p.tp_role == 1) return gemv<PRO_RESID_NORM_TP, EPI>(c, p, grid_out);
    const int pair = EPI == EPI_SWIGLU ? 2 : 1;
    const uint64_t units = p.rows / pair;
    if (c->bulk_gemv && gemv_bulk_shape(p.cols) && reinterpret_cast<uintptr_t>(p.w) % 16 == 0 && units) {
        uint64_t grid = std::min<uint64_t>(units, static_cast<uint64_t>(c->sm_count) * c->gemv_ctas);
        // Ring depth: about gemv_ring_kb of chunks, at least two.
        const uint32_t chunk = gemv_bulk_chunk_bytes(p.cols);
        int stages = std::max(2, std::min<int>(kMaxStages, c->gemv_ring_kb * 1024 / static_cast<int>(chunk)));
        size_t smem = 0;
        for (;;) {
            smem = gemv_bulk_smem(p.cols, (units + grid - 1) / grid, pair, stages);
            if (smem + 2048 <= static_cast<size_t>(c->smem_optin)) break;
            if (stages > 2) --stages;
            else if (grid < units) grid = std::min<uint64_t>(units, grid * 2);
            else return false;
        }
        // The grid is one CTA per SM: two of its CTAs on one SM (possible for
        // narrow rows and few registers) would give that SM a double share of
        // the stream while another SM idles, so the request is more than half
        // an SM's shared memory. A smaller kernel (decode attention) still fits
        // beside it.
        if (c->gemv_ctas == 1)
            smem = std::max<size_t>(smem, static_cast<size_t>(c->smem_per_sm) / 2 - 1024 + 16);
        if (grid_out) *grid_out = static_cast<uint32_t>(grid);
        const dim3 g(static_cast<uint32_t>(grid)), b(kBulkThreads);
        if (p.cols % kSubElems) {
            switch (gemv_bulk_sets(p.cols)) {
            case 1: return launch(c, gemv_bulk_kernel<PRO, EPI, 1, true>, g, b, smem, p, stages);
            case 2: return launch(c, gemv_bulk_kernel<PRO, EPI, 2, true>, g, b, smem, p, stages);
            default: return launch(c, gemv_bulk_kernel<PRO, EPI, 4, true>, g, b, smem, p, stages);
            }
        }
        switch (gemv_bulk_sets(p.cols)) {
        case 1: return launch(c, gemv_bulk_kernel<PRO, EPI, 1, false>, g, b, smem, p, stages);
        case 2: return launch(c, gemv_bulk_kernel<PRO, EPI, 2, false>, g, b, smem, p, stages);
        default: return launch(c, gemv_bulk_kernel<PRO, EPI, 4, false>, g, b, smem, p, stages);
        }
    }
    const int U = gemv_chunks(p.w, p.cols);
    size_t smem = 0;
    const uint32_t grid = gemv_grid(c, units, p.cols, U, pair, &smem);
    if (grid_out) *grid_out = grid;
    return launch_gemv_shape<PRO, EPI>(c, p, U, grid, smem);
}

// SwiGLU of T rows of [gate | up] in place (and the split terms of `f`).
bool swiglu_rows(plamo_cuda *c, float *gu, uint64_t I, uint64_t T, const RowFuse &f) {
    if (I % 4 == 0)
        return launch(c, swiglu_rows4_kernel, dim3(static_cast<uint32_t>((I / 4 + 255) / 256), static_cast<uint32_t>(T)),
                      dim3(256), 0, gu, I, T, f);
    return launch(c, swiglu_rows_kernel, dim3(std::min<uint64_t>((I * T + 255) / 256, 4096)), dim3(256), 0, gu, I, T,
                  f);
}

bool gemm(plamo_cuda *c, const float *X, uint64_t xs, const uint16_t *W, float *Y, uint64_t ys,
          uint64_t T, uint64_t R, uint64_t K) {
    if (!T || !R) return true;
    dim3 grid((R + kGemmBN - 1) / kGemmBN, (T + kGemmBM - 1) / kGemmBM);
    return launch(c, gemm_simt_kernel, grid, dim3(256), 0, X, xs, W, Y, ys, T, R, K);
}

// ---- tcgen05 projections ---------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;

bool tensor_maps_available() {
    if (g_encode_tiled) return true;
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
        return false;
    g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    return true;
}

// 2-D BF16 row-major [rows][cols] map with a {64 x box_rows} box, 128-byte swizzle.
bool bf16_map(CUtensorMap *map, const void *ptr, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    cuuint64_t dims[2] = {cols, rows};
    cuuint64_t strides[1] = {cols * 2};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kTcK), box_rows};
    cuuint32_t elem[2] = {1, 1};
    return g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(ptr), dims, strides, box, elem,
                          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int N>
bool launch_tc(plamo_cuda *c, const CUtensorMap &mw, const CUtensorMap &mh, const CUtensorMap &mm,
               const CUtensorMap &ml, const TcGemmParams &p, uint32_t R, uint32_t T, uint32_t splits) {
    // Up to 32 tokens a tile streams weights with little math per byte: two
    // CTAs share each SM (half the shared memory each; their accumulator rings
    // take 256 of the 512 TMEM columns each), so two weight pipelines are in
    // flight per SM and a grid of up to 2 x 148 tiles is resident at once.
    const size_t budget = N <= 32 ? static_cast<size_t>(c->smem_per_sm) / 2 - 8192
                                  : static_cast<size_t>(c->smem_optin) - 2048;
    int stages = static_cast<int>(std::min<size_t>(kTcMaxStages, budget / tc_stage_bytes(N)));
    if (c->tc_stages) stages = std::min(stages, c->tc_stages);
    const dim3 grid((T + N - 1) / N, (R + kTcM - 1) / kTcM, splits);
    return launch(c, gemm_tc_kernel<N>, grid, dim3(tc_threads<N>()), tc_smem_bytes(N, stages), mw, mw, mh, mm, ml,
                  p, stages);
}

// Token-major tiles (128 tokens x 144, 160 or 192 weight rows) or weight-major
// ones (128 weight rows x 128 tokens) for a prompt of more than 64 tokens: one
// CTA per SM either way, so the choice compares waves of tiles times a wave's
// cost, measured on the 8B projections of a 455-token prompt (CUDA events,
// B200) relative to a weight-major wave: 1.06 for 144 rows, 1.11 for 160,
// 1.18 for 192. That sends qkv (5120 rows) to one wave of 144-row tiles
// (66.5 us; 192 rows 73.3, weight-major 108.2), gate_up (32768 rows) to five
// waves of 192-row tiles (316.4 us; 160 rows 352.9, weight-major 361.1) and
// keeps o_proj and down_proj (4096 rows) weight-major (215.3 us against 224.7
// for 144 rows). Ties go to the weight-major, then to the wider tile.
// PLAMO_CUDA_TC_TOKM=0 / 1 forces weight-major / token-major tiles,
// PLAMO_CUDA_TC_TOKN=144 / 160 / 192 the token-major width.
constexpr uint32_t kTcTokWidths[3] = {192, 160, 144};
constexpr uint64_t kTcTokCost[3] = {118, 111, 106};  // per wave, weight-major = 100
uint32_t tc_token_cols(plamo_cuda *c, uint64_t T, uint64_t R) {
    if (T <= 64 || c->tc_tokm == 0) return 0;
    const uint64_t sms = static_cast<uint64_t>(c->sm_count), tt = (T + kTcM - 1) / kTcM;
    auto waves = [&](uint64_t tiles) { return (tiles + sms - 1) / sms; };
    uint64_t best_cost = c->tc_tokm == 1 ? ~0ull : waves(tt * ((R + kTcM - 1) / kTcM)) * 100;
    uint32_t best = 0;
    for (int i = 0; i < 3; ++i) {
        const uint32_t n = kTcTokWidths[i];
        if (c->tc_tokn && n != static_cast<uint32_t>(c->tc_tokn)) continue;
        const uint64_t cost = waves(tt * ((R + n - 1) / n)) * kTcTokCost[i];
        if (cost < best_cost) {
            best_cost = cost;
            best = n;
        }
    }
    return best;
}

// mu: the up rows' map of a gate/up-paired launch (p.glu), else mw again.
template <int N>
bool launch_tc_tokm(plamo_cuda *c, const CUtensorMap &mw, const CUtensorMap &mu, const CUtensorMap &mh,
                    const CUtensorMap &mm, const CUtensorMap &ml, const TcGemmParams &p, uint32_t R, uint32_t T) {
    const size_t budget = static_cast<size_t>(c->smem_optin) - 2048;
    int stages = static_cast<int>(std::min<size_t>(kTcMaxStages, budget / tc_stage_bytes(N, true)));
    if (c->tc_stages) stages = std::min(stages, c->tc_stages);
    const dim3 grid((T + kTcM - 1) / kTcM, (R + N - 1) / N, 1);
    return launch(c, gemm_tc_kernel<N, true>, grid, dim3(tc_threads<N>()), tc_smem_bytes(N, stages, true), mw, mu,
                  mh, mm, ml, p, stages);
}

// Y[T][R] (row stride ys) = X[T][K] (row stride xs, FP32) . W[R][K]^T on the
// tensor cores when the shapes allow TMA (16-byte aligned rows), else on the
// FP32 CUDA-core kernel otherwise. split: BF16 scratch of 3*T*K elements
// (the hi, mid and lo terms).
// part/part_floats: scratch for split-K partial tiles (nullptr: no split K).
// presplit: `split` already holds the BF16 terms of X (written by the kernel
// that produced X), so no split pass runs. defer: when the projection splits
// K, leave the partial planes for the consumer to sum (RowFuse.bparts) and
// describe them here instead of summing into Y; defer->splits = 1 otherwise.
struct Deferred {
    uint32_t splits = 1;
    const float *part = nullptr;
    uint64_t plane = 0;
};

// Whether projection_with takes the tensor-core path for this weight.
bool tc_projection(plamo_cuda *c, const uint16_t *W, uint64_t T, uint64_t R, uint64_t K) {
    return c->tc_gemm && K % 8 == 0 && K >= kTcK && reinterpret_cast<uintptr_t>(W) % 16 == 0 && T < (1ull << 31) &&
           R < (1ull << 31) && tensor_maps_available();
}

bool projection_with(plamo_cuda *c, const float *X, uint64_t xs, const uint16_t *W, float *Y, uint64_t ys, uint64_t T,
                     uint64_t R, uint64_t K, uint16_t *split, uint32_t *error, float *part = nullptr,
                     uint64_t part_floats = 0, bool presplit = false, Deferred *defer = nullptr) {
    if (defer) *defer = Deferred{};
    if (!T || !R) return true;
    const bool tc = split && tc_projection(c, W, T, R, K);
    if (!tc && !X) return false;  // only BF16 terms of the input exist
    if (!tc) return gemm(c, X, xs, W, Y, ys, T, R, K);
    uint16_t *hi = split, *mid = split + T * K, *lo = split + 2 * T * K;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((T * K + 255) / 256, 8192));
    if (!presplit && !launch(c, split_hilo_kernel, dim3(blocks), dim3(256), 0, X, xs, static_cast<uint32_t>(T),
                             static_cast<uint32_t>(K), hi, mid, lo))
        return false;
    if (const uint32_t tn = tc_token_cols(c, T, R)) {
        CUtensorMap mw, mh, mm, ml;
        if (bf16_map(&mw, W, R, K, tn) && bf16_map(&mh, hi, T, K, kTcM) && bf16_map(&mm, mid, T, K, kTcM) &&
            bf16_map(&ml, lo, T, K, kTcM)) {
            TcGemmParams p{Y, ys, static_cast<uint32_t>(T), static_cast<uint32_t>(R), static_cast<uint32_t>(K),
                           error, part};
            const uint32_t r32 = static_cast<uint32_t>(R), t32 = static_cast<uint32_t>(T);
            return tn == 144   ? launch_tc_tokm<144>(c, mw, mw, mh, mm, ml, p, r32, t32)
                   : tn == 160 ? launch_tc_tokm<160>(c, mw, mw, mh, mm, ml, p, r32, t32)
                               : launch_tc_tokm<192>(c, mw, mw, mh, mm, ml, p, r32, t32);
        }
    }
    const uint32_t N = T <= 16 ? 16 : T <= 32 ? 32 : T <= 64 ? 64 : 128;
    CUtensorMap mw, mh, mm, ml;
    if (!bf16_map(&mw, W, R, K, kTcM) || !bf16_map(&mh, hi, T, K, N) || !bf16_map(&mm, mid, T, K, N) ||
        !bf16_map(&ml, lo, T, K, N)) {
        snprintf(c->info.note, sizeof c->info.note, "tensor map encode failed");
        return X && gemm(c, X, xs, W, Y, ys, T, R, K);
    }
    TcGemmParams p{Y, ys, static_cast<uint32_t>(T), static_cast<uint32_t>(R), static_cast<uint32_t>(K), error, part};
    const uint32_t r32 = static_cast<uint32_t>(R), t32 = static_cast<uint32_t>(T);
    // Split K when a handful of tokens leaves SMs without a row tile: as many
    // splits as keep every CTA resident at two per SM (one wave), at least 4
    // K blocks per split.
    uint32_t splits = 1;
    const uint64_t tiles = ((T + N - 1) / N) * ((R + kTcM - 1) / kTcM);
    const uint64_t kall = (K + kTcK - 1) / kTcK;
    if (part && T <= 16 && tiles < static_cast<uint64_t>(c->sm_count)) {
        uint64_t want = 2ull * c->sm_count / tiles;
        want = std::min<uint64_t>({want, kall / 4, 16});
        while (want > 1 && want * T * R > part_floats) --want;
        splits = static_cast<uint32_t>(std::max<uint64_t>(want, 1));
    }
    bool ok;
    switch (N) {
    case 16: ok = launch_tc<16>(c, mw, mh, mm, ml, p, r32, t32, splits); break;
    case 32: ok = launch_tc<32>(c, mw, mh, mm, ml, p, r32, t32, splits); break;
    case 64: ok = launch_tc<64>(c, mw, mh, mm, ml, p, r32, t32, splits); break;
    default: ok = launch_tc<128>(c, mw, mh, mm, ml, p, r32, t32, splits); break;
    }
    if (!ok || splits == 1) return ok;
    if (defer) {
        *defer = Deferred{splits, part, T * R};
        return true;
    }
    const uint32_t sum_blocks = static_cast<uint32_t>(std::min<uint64_t>((T * R + 255) / 256, 4096));
    return launch(c, splitk_sum_kernel, dim3(sum_blocks), dim3(256), 0, static_cast<const float *>(part), splits, t32,
                  r32, Y, ys);
}

bool projection(plamo_cuda *c, DModel *m, const float *X, uint64_t xs, const uint16_t *W, float *Y, uint64_t ys,
                uint64_t T, uint64_t R, uint64_t K, bool presplit = false, Deferred *defer = nullptr) {
    return projection_with(c, X, xs, W, Y, ys, T, R, K, T <= m->tmax ? m->p_split : nullptr, m->d_error,
                           m->p_splitk, kSplitkFloats, presplit, defer);
}

// The MLP's gate/up projection of a prompt fused with SwiGLU: token-major
// tiles of 96 gate rows and the same 96 up rows (two tensor maps over the
// halves of the [2I][K] weight), whose epilogue writes the BF16 terms of
// SwiGLU(gate, up) for the down projection into `terms` ([3][T][I]) - the
// same values swiglu_rows and its split would write, with no [T][2I]
// round trip through HBM and no launch. The input's terms are in m->p_split.
// Taken when the tile choice for the [2I][K] projection is 192-row
// token-major tiles (PLAMO_CUDA_TC_GLU=0 turns it off).
bool glu_fusable(plamo_cuda *c, DModel *m, const uint16_t *gu, const uint16_t *down, uint64_t T) {
    return c->tc_glu && m->p_glu && T <= m->tmax && tc_projection(c, gu, T, 2 * m->I, m->H) &&
           tc_projection(c, down, T, m->H, m->I) && tc_token_cols(c, T, 2 * m->I) == 192;
}

bool projection_glu(plamo_cuda *c, DModel *m, const uint16_t *gu, uint64_t T) {
    const uint64_t I = m->I, K = m->H;
    uint16_t *hi = m->p_split, *mid = hi + T * K, *lo = hi + 2 * T * K;
    CUtensorMap mw, mu, mh, mm, ml;
    if (!bf16_map(&mw, gu, I, K, 96) || !bf16_map(&mu, gu + I * K, I, K, 96) || !bf16_map(&mh, hi, T, K, kTcM) ||
        !bf16_map(&mm, mid, T, K, kTcM) || !bf16_map(&ml, lo, T, K, kTcM)) {
        snprintf(c->info.note, sizeof c->info.note, "tensor map encode failed");
        return false;
    }
    TcGemmParams p{};
    p.T = static_cast<uint32_t>(T);
    p.R = static_cast<uint32_t>(2 * I);
    p.K = static_cast<uint32_t>(K);
    p.error = m->d_error;
    p.glu = m->p_glu;
    p.glu_plane = T * I;
    p.glu_inter = static_cast<uint32_t>(I);
    return launch_tc_tokm<192>(c, mw, mu, mh, mm, ml, p, static_cast<uint32_t>(2 * I), static_cast<uint32_t>(T));
}

// The RowFuse of a row kernel whose output feeds projection W next (split
// terms when that projection runs on the tensor cores) and whose branch input
// may be the deferred partials of the previous projection.
RowFuse row_fuse(plamo_cuda *c, DModel *m, const uint16_t *next_w, uint64_t T, uint64_t R, uint64_t K,
                 const Deferred &in) {
    RowFuse f{};
    if (next_w && T <= m->tmax && tc_projection(c, next_w, T, R, K)) f.split = m->p_split;
    if (in.splits > 1) {
        f.bparts = in.part;
        f.bsplits = in.splits;
        f.bplane = in.plane;
    }
    return f;
}

AttnLayer attn_layer(const DModel *m, uint64_t l) {
    const DLayer &L = m->layers[l];
    AttnLayer a;
    a.pages = L.d_pages;
    a.kvw = m->KVW;
    a.appended = m->d_appended + l;
    a.ring = L.ring;
    a.capacity = L.capacity;
    a.sliding = L.sliding;
    a.table = L.rope->dev;
    a.positions = L.rope->positions;
    a.qn = L.qn;
    a.kn = L.kn;
    return a;
}

uint64_t layer_count(const DLayer &L) {
    return L.sliding ? std::min(L.appended, L.capacity) : L.appended;
}

void *dalloc(plamo_cuda *c, DModel *m, uint64_t bytes) {
    void *p = nullptr;
    if (!bytes) bytes = 16;
    if (!note(c, "cudaMalloc", cudaMalloc(&p, bytes))) return nullptr;
    cudaMemset(p, 0, bytes);
    m->allocations.push_back(p);
    c->info.allocated_bytes += bytes;
    return p;
}

// ---- KV pages -----------------------------------------------------------------
uint64_t kv_page_floats(uint64_t kvw) { return 2 * kKvPageRows * kvw; }

// The pool of row width kvw, with its zeroed spare page (0 if it cannot be made).
KvPool *kv_pool(plamo_cuda *c, uint64_t kvw) {
    KvPool &pool = c->kv_pools[kvw];
    if (!pool.spare) {
        const uint64_t bytes = kv_page_floats(kvw) * 4;
        if (!note(c, "kv spare page", cudaMalloc(&pool.spare, bytes))) {
            pool.spare = nullptr;
            return nullptr;
        }
        cudaMemset(pool.spare, 0, bytes);
        c->info.kv_bytes += bytes;
        c->info.allocated_bytes += bytes;
    }
    return &pool;
}

// One page from the pool, growing it by a chunk when it is empty.
float *kv_page_take(plamo_cuda *c, uint64_t kvw) {
    KvPool *pool = kv_pool(c, kvw);
    if (!pool) return nullptr;
    if (pool->free.empty()) {
        const uint64_t floats = kv_page_floats(kvw);
        float *chunk = nullptr;
        if (!note(c, "kv page chunk", cudaMalloc(&chunk, kKvChunkPages * floats * 4))) return nullptr;
        pool->chunks.push_back(chunk);
        c->info.kv_bytes += kKvChunkPages * floats * 4;
        c->info.allocated_bytes += kKvChunkPages * floats * 4;
        c->info.kv_pages_allocated += kKvChunkPages;
        for (uint64_t i = kKvChunkPages; i-- > 0;) pool->free.push_back(chunk + i * floats);
    }
    float *page = pool->free.back();
    pool->free.pop_back();
    ++pool->used;
    ++c->info.kv_pages_used;
    return page;
}

void kv_page_give(plamo_cuda *c, uint64_t kvw, float *page) {
    KvPool &pool = c->kv_pools[kvw];
    pool.free.push_back(page);
    --pool.used;
    --c->info.kv_pages_used;
}

// Map the pages of slots [0, min(rows, ring)) of layer L and upload the new
// page-table entries. False (nothing changed) when the pool cannot grow.
bool kv_map(plamo_cuda *c, const DModel *m, DLayer &L, uint64_t rows) {
    const uint64_t need = (std::min(rows, L.ring) + kKvPageRows - 1) / kKvPageRows;
    const uint64_t first = L.mapped;
    if (need <= first) return true;
    for (uint64_t i = first; i < need; ++i) {
        float *page = kv_page_take(c, m->KVW);
        if (!page) {
            for (uint64_t j = first; j < i; ++j) {
                kv_page_give(c, m->KVW, L.pages[j]);
                L.pages[j] = c->kv_pools[m->KVW].spare;
            }
            snprintf(c->info.note, sizeof c->info.note, "KV page pool cannot grow (device memory)");
            return false;
        }
        L.pages[i] = page;
    }
    if (!note(c, "kv page table", cudaMemcpyAsync(L.d_pages + first, L.pages.data() + first,
                                                  (need - first) * sizeof(float *), cudaMemcpyHostToDevice,
                                                  c->stream)))
        return false;
    L.mapped = need;
    return true;
}

// Return the pages of layer L past the first `keep` to the pool (their table
// entries point at the spare page again).
bool kv_unmap(plamo_cuda *c, const DModel *m, DLayer &L, uint64_t keep) {
    if (L.mapped <= keep) return true;
    KvPool &pool = c->kv_pools[m->KVW];
    for (uint64_t i = keep; i < L.mapped; ++i) {
        kv_page_give(c, m->KVW, L.pages[i]);
        L.pages[i] = pool.spare;
    }
    const uint64_t first = keep;
    const bool ok = note(c, "kv page table", cudaMemcpyAsync(L.d_pages + first, L.pages.data() + first,
                                                             (L.mapped - first) * sizeof(float *),
                                                             cudaMemcpyHostToDevice, c->stream));
    L.mapped = keep;
    return ok;
}

// Copy rows [0, rows) of layer L between its pages and row-major K and V
// arrays ([rows][kvw] each), toward the pages when `to_pages`.
bool kv_copy_rows(plamo_cuda *c, const DModel *m, const DLayer &L, uint64_t rows, float *k, float *v,
                  bool to_pages, cudaMemcpyKind kind) {
    const uint64_t kvw = m->KVW;
    for (uint64_t p = 0; p * kKvPageRows < rows; ++p) {
        const uint64_t n = std::min(kKvPageRows, rows - p * kKvPageRows);
        float *pk = L.pages[p], *pv = L.pages[p] + kKvPageRows * kvw;
        float *lk = k + p * kKvPageRows * kvw, *lv = v + p * kKvPageRows * kvw;
        const uint64_t bytes = n * kvw * 4;
        if (!note(c, "kv rows", cudaMemcpyAsync(to_pages ? pk : lk, to_pages ? lk : pk, bytes, kind, c->stream)) ||
            !note(c, "kv rows", cudaMemcpyAsync(to_pages ? pv : lv, to_pages ? lv : pv, bytes, kind, c->stream)))
            return false;
    }
    return true;
}

void free_model(plamo_cuda *c, DModel *m) {
    if (m->graph_exec) cudaGraphExecDestroy(m->graph_exec);
    for (cudaGraphExec_t e : m->layer_exec)
        if (e) cudaGraphExecDestroy(e);
    m->layer_exec.clear();
    if (m->graph) cudaGraphDestroy(m->graph);
    for (uint32_t r = 0; r < m->tp.size; ++r)
        if (r != m->tp.rank && m->tp.peer[r]) cudaIpcCloseMemHandle(m->tp.peer[r]);
    for (DLayer &L : m->layers) {
        for (uint64_t i = 0; i < L.mapped; ++i) kv_page_give(c, m->KVW, L.pages[i]);
        L.mapped = 0;
    }
    for (void *p : m->allocations) cudaFree(p);
    m->allocations.clear();
}

// Identity of a host descriptor tree: dimensions, every weight and KV pointer.
std::vector<uintptr_t> model_signature(const struct model *model) {
    std::vector<uintptr_t> sig;
    auto add = [&](const void *p) { sig.push_back(reinterpret_cast<uintptr_t>(p)); };
    sig.push_back(model->vocab);
    sig.push_back(model->hidden);
    sig.push_back(model->count);
    add(model->embedding);
    add(model->norm);
    add(model->head);
    add(model->state);
    add(model->logits);
    for (uint64_t i = 0; i < model->count; ++i) {
        const struct layer *l = model->layers[i];
        const struct qkv *q = l->mixer->qkv;
        const struct cache *k = l->mixer->cache;
        add(l);
        add(q->weight);
        add(l->mixer->weight);
        add(l->mlp->gu);
        add(l->mlp->down);
        add(k->k);
        sig.push_back(k->capacity);
        sig.push_back(q->dim);
        sig.push_back(l->mlp->intermediate);
    }
    return sig;
}

DModel *find_model(plamo_cuda *c, struct model *model) {
    auto it = c->models.find(model);
    return it == c->models.end() ? nullptr : it->second.get();
}

// Bring the device KV in line with the host descriptors: a host count of
// zero resets the layer (the engine's plamo_reset_request); any other count
// the device does not hold means the host wrote the rows itself (for example
// a prompt-cache restore), so they are uploaded as rows 0..count-1.
uint64_t row_hash(const float *row, uint64_t n) {
    const unsigned char *p = reinterpret_cast<const unsigned char *>(row);
    uint64_t h = 14695981039346656037ull;
    for (uint64_t i = 0; i < n * 4; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

uint64_t newest_row_hash(const DModel *m, const DLayer &L) {
    const struct cache *hc = L.host->mixer->cache;
    if (!hc->count) return 0;
    return row_hash(hc->k + (hc->count - 1) * m->KVW, m->KVW);
}

bool reconcile(plamo_cuda *c, DModel *m) {
    bool changed = false;
    for (uint64_t l = 0; l < m->L; ++l) {
        DLayer &L = m->layers[l];
        const struct cache *hc = L.host->mixer->cache;
        const uint64_t dc = layer_count(L);
        // With host copies enabled, a host write that kept the count is seen
        // through the newest row's hash.
        if (!L.stale && c->config.copy_kv_to_host && hc->count && hc->count == dc &&
            newest_row_hash(m, L) != L.host_hash)
            L.stale = true;
        if (hc->count == dc && !L.stale) continue;
        changed = true;
        L.stale = false;
        if (hc->count > L.ring || hc->count > L.capacity) return false;
        // A full layer keeps pages for the rows it holds; the others go back
        // to the pool (a reset returns all of them).
        if (!L.sliding && !kv_unmap(c, m, L, (hc->count + kKvPageRows - 1) / kKvPageRows)) return false;
        if (hc->count && (!kv_map(c, m, L, hc->count) ||
                          !kv_copy_rows(c, m, L, hc->count, hc->k, hc->v, true, cudaMemcpyHostToDevice)))
            return false;
        L.appended = hc->count;
    }
    if (changed) {
        std::vector<uint64_t> counts(m->L);
        for (uint64_t l = 0; l < m->L; ++l) counts[l] = m->layers[l].appended;
        if (!note(c, "counter upload", cudaMemcpyAsync(m->d_appended, counts.data(), m->L * 8,
                                                       cudaMemcpyHostToDevice, c->stream)))
            return false;
        if (!note(c, "sync", cudaStreamSynchronize(c->stream))) return false;
    }
    return true;
}

// Mirror the CPU path's descriptor updates after `rows` committed rows.
void publish_counts(DModel *m, uint64_t rows) {
    for (uint64_t l = 0; l < m->L; ++l) {
        DLayer &L = m->layers[l];
        L.appended += rows;
        struct cache *hc = L.host->mixer->cache;
        struct rotation *r = L.host->mixer->rotation;
        hc->count = layer_count(L);
        r->processed_count = hc->count;
        r->scale_bits = float_to_bits(L.scale);
    }
}

// Rows a decode/prefill of `tokens` would need; false when a full-attention
// cache cannot take them (the reference declines: src/cache.s global full) or
// the KV pages for them cannot be mapped. Maps those pages otherwise.
bool fits(plamo_cuda *c, DModel *m, uint64_t tokens) {
    for (const DLayer &L : m->layers) {
        if (!L.sliding && L.appended + tokens > L.capacity) return false;
        if (!L.sliding && L.appended + tokens > L.ring) return false;
        if (L.sliding && std::min(L.appended + tokens, L.capacity) > L.rope->positions) return false;
        if (!L.sliding && L.appended + tokens > L.rope->positions) return false;
    }
    for (DLayer &L : m->layers)
        if (!L.sliding && !kv_map(c, m, L, L.appended + tokens)) return false;
    return true;
}

// ---- decode step -----------------------------------------------------------
// The next launch's timeline record while a traced step is recorded, else null.
unsigned long long *next_trace(DModel *m) {
    return m->trace ? m->trace + kTraceWords * m->trace_slot++ : nullptr;
}

bool launch_decode_attention(plamo_cuda *c, DModel *m, uint64_t l) {
    DecodeAttnParams dp{attn_layer(m, l), static_cast<uint32_t>(m->QH), static_cast<uint32_t>(m->KH),
                        static_cast<uint32_t>(m->D), m->qkv, m->attn};
    dp.trace = next_trace(m);
    const size_t smem = decode_attention_smem(static_cast<uint32_t>(m->QH / m->KH), static_cast<uint32_t>(m->D));
    const dim3 block(kDecThreads);
    if (m->D == 128 && m->QH / m->KH <= 32)
        return launch(c, decode_attention128_kernel, dim3(static_cast<uint32_t>(m->KH), kDec128Splits), block,
                      decode_attention128_smem(static_cast<uint32_t>(m->QH / m->KH)), dp);
    return launch(c, decode_attention_kernel<0>, dim3(static_cast<uint32_t>(m->KH), kDecSplits), block, smem, dp);
}

// Exchange point `index` of the decode step (0..2L-1) or of a prompt.
TpPoint tp_point(DModel *m, bool prompt, uint64_t index) {
    const TpState &t = m->tp;
    TpPoint p{};
    p.tp = t.size;
    p.ll = prompt ? 0 : 1;  // decode points: {value, tag} pairs (8 bytes per element)
    p.stride = prompt ? m->tmax * m->H : m->H;
    const uint64_t parts = prompt ? t.off_pparts + (index % 2) * t.size * p.stride * 4
                                  : t.off_dparts + index * t.size * p.stride * 8;
    const uint64_t flags = (prompt ? t.off_pflags : t.off_dflags) + index * t.size * 4;
    p.parts = reinterpret_cast<const float *>(t.xbuf + parts);
    p.flags = reinterpret_cast<const uint32_t *>(t.xbuf + flags);
    for (uint32_t r = 0; r < t.size; ++r) {
        p.peer_parts[r] = reinterpret_cast<float *>(t.peer[r] + parts + t.rank * p.stride * (p.ll ? 8 : 4));
        p.peer_flags[r] = reinterpret_cast<uint32_t *>(t.peer[r] + flags) + t.rank;
    }
    p.ticket = t.tickets + (prompt ? 2 * m->L : 0) + index;
    p.epoch = t.epoch;
    p.error = m->d_error;
    return p;
}

TpArg tp_arg(DModel *m) {
    const TpState &t = m->tp;
    TpArg a{};
    a.tp = t.size;
    a.rank = t.rank;
    a.slots = reinterpret_cast<uint32_t *>(t.xbuf + t.off_args);
    for (uint32_t r = 0; r < t.size; ++r) a.peer_slots[r] = reinterpret_cast<uint32_t *>(t.peer[r] + t.off_args);
    a.epoch = t.epoch;
    a.error = m->d_error;
    return a;
}

// Greedy choice of every row of a [rows][V] logits block (per-chunk
// candidates in the head GEMV's candidate buffers, then a merge per row).
bool rows_argmax(plamo_cuda *c, DModel *m, const float *logits, uint64_t n, uint32_t rows, uint32_t *out,
                 float *out_val) {
    const uint32_t chunks = std::max<uint32_t>(1, std::min<uint32_t>(64, static_cast<uint32_t>(
                                                                          static_cast<uint64_t>(c->sm_count) * 64 / rows)));
    return launch(c, rows_argmax_partial_kernel, dim3(chunks, rows), dim3(256), 0, logits, n, m->arg_val,
                  m->arg_idx, m->arg_nan) &&
           launch(c, rows_argmax_merge_kernel, dim3(rows), dim3(32), 0, static_cast<const float *>(m->arg_val),
                  static_cast<const uint32_t *>(m->arg_idx), static_cast<const uint32_t *>(m->arg_nan), chunks, out,
                  out_val);
}

// Greedy token of one row from the head's per-block candidates: the local
// merge, then (tensor-parallel) the first maximum over the ranks' slices.
bool greedy_choice(plamo_cuda *c, DModel *m, uint32_t grid) {
    const bool tp = m->tp.active;
    if (!launch(c, argmax_merge_kernel, dim3(1), dim3(256), 0, static_cast<const float *>(m->arg_val),
                static_cast<const uint32_t *>(m->arg_idx), static_cast<const uint32_t *>(m->arg_nan), grid,
                tp ? m->tp.lidx : m->d_next, tp ? nullptr : m->d_token, tp ? m->tp.lval : nullptr,
                static_cast<const float *>(tp ? nullptr : m->arg_val2),
                tp ? nullptr : reinterpret_cast<float *>(m->d_next + 2)))
        return false;
    if (!tp) return true;
    return launch(c, tp_argmax_kernel, dim3(1), dim3(128), 0, static_cast<const float *>(m->tp.lval),
                  static_cast<const uint32_t *>(m->tp.lidx), 1u, static_cast<uint32_t>(m->tp.voff), tp_arg(m),
                  m->d_next, m->d_token);
}

// Prompt all-reduce of a [T][H] partial block in place.
bool tp_allreduce_rows(plamo_cuda *c, DModel *m, float *rows, uint64_t T, uint64_t index) {
    const TpPoint t = tp_point(m, true, index);
    const uint32_t grid = static_cast<uint32_t>(std::min<uint64_t>((T * m->H / 4 + 255) / 256, c->sm_count * 2ull));
    return launch(c, tp_push_kernel, dim3(grid), dim3(256), 0, static_cast<const float *>(rows), T * m->H, t) &&
           launch(c, tp_sum_kernel, dim3(grid), dim3(256), 0, rows, T * m->H, t);
}

bool record_decode(plamo_cuda *c, DModel *m) {
    int s = 0;
    for (uint64_t l = 0; l < m->L; ++l) {
        const DLayer &L = m->layers[l];
        GemvParams p{};
        p.w = L.qkv_w;
        p.rows = m->QW;
        p.cols = m->H;
        p.norm2 = L.pre;
        p.off2 = 1.0f;
        p.y = m->qkv;
        p.error = m->d_error;
        p.trace = next_trace(m);
        bool ok;
        if (l == 0) {
            p.embedding = m->emb;
            p.token = m->d_token;
            p.vocab = m->V;
            p.state_out = m->state[s];
            ok = gemv<PRO_EMBED_NORM, EPI_STORE>(c, p);
        } else {
            p.state_in = m->state[s];
            p.branch = m->branch;
            p.norm1 = m->layers[l - 1].mpost;
            p.off1 = kPostMlpOffset;
            p.state_out = m->state[s ^ 1];
            s ^= 1;
            if (m->tp.active) {
                p.tp_role = 1;
                p.tp = tp_point(m, false, 2 * (l - 1) + 1);
            }
            ok = gemv<PRO_RESID_NORM, EPI_STORE>(c, p);
        }
        if (!ok) return false;
        if (!launch_decode_attention(c, m, l)) return false;
        GemvParams o{};
        o.w = L.o_w;
        o.rows = m->H;
        o.cols = m->AW;
        o.x = m->attn;
        o.y = m->branch;
        o.trace = next_trace(m);
        if (m->tp.active) {
            o.tp_role = 2;
            o.tp = tp_point(m, false, 2 * l);
        }
        if (!gemv<PRO_X, EPI_STORE>(c, o)) return false;
        GemvParams g{};
        g.w = L.gu;
        g.rows = 2 * m->I;
        g.cols = m->H;
        g.state_in = m->state[s];
        g.branch = m->branch;
        g.norm1 = L.post;
        g.off1 = kPostMixerOffset;
        g.norm2 = L.mpre;
        g.off2 = 1.0f;
        g.state_out = m->state[s ^ 1];
        s ^= 1;
        g.y = m->mid;
        g.trace = next_trace(m);
        if (m->tp.active) {
            g.tp_role = 1;
            g.tp = tp_point(m, false, 2 * l);
        }
        if (!gemv<PRO_RESID_NORM, EPI_SWIGLU>(c, g)) return false;
        GemvParams d{};
        d.w = L.down;
        d.rows = m->H;
        d.cols = m->I;
        d.x = m->mid;
        d.y = m->branch;
        d.trace = next_trace(m);
        if (m->tp.active) {
            d.tp_role = 2;
            d.tp = tp_point(m, false, 2 * l + 1);
        }
        if (!gemv<PRO_X, EPI_STORE>(c, d)) return false;
    }
    GemvParams h{};
    h.w = m->head;
    h.rows = m->Vh;
    h.cols = m->H;
    h.state_in = m->state[s];
    h.branch = m->branch;
    h.norm1 = m->layers[m->L - 1].mpost;
    h.off1 = kPostMlpOffset;
    h.norm2 = m->norm;
    h.off2 = 1.0f;
    h.state_out = m->state[s ^ 1];
    h.trace = next_trace(m);
    m->final_state = m->state[s ^ 1];
    h.norm_out = m->normalized;
    h.y = m->logits;
    h.arg_val = m->arg_val;
    h.arg_val2 = m->arg_val2;
    h.arg_idx = m->arg_idx;
    h.arg_nan = m->arg_nan;
    if (m->tp.active) {
        h.tp_role = 1;
        h.tp = tp_point(m, false, 2 * m->L - 1);
    }
    uint32_t grid = 0;
    if (!gemv<PRO_RESID_NORM, EPI_ARGMAX>(c, h, &grid)) return false;
    if (!greedy_choice(c, m, grid)) return false;
    if (!launch(c, advance_kernel, dim3(1), dim3(32), 0, m->d_appended, m->L, uint64_t{1})) return false;
    return !m->tp.active || launch(c, tp_epoch_kernel, dim3(1), dim3(32), 0, m->tp.epoch);
}

// Advance the row counters of every request of a batch by one.
__global__ void batch_advance_kernel(uint64_t *const *counters, uint64_t layers, uint32_t requests) {
    pdl_wait();
    for (uint32_t i = threadIdx.x; i < layers * requests; i += blockDim.x) counters[i / layers][i % layers] += 1;
}

// One decode step of every request of a batch, layer-major over B rows: the
// prompt kernels for the norms and the (tcgen05, split-K) projections, the
// fused decode attention per request on its own cache, the head over all
// rows and a greedy choice per row into the token buffer.
bool record_batch(plamo_cuda *c, plamo_cuda_batch *b, DModel *m) {
    const uint64_t T = b->B, H = m->H;
    const uint32_t G = static_cast<uint32_t>(m->QH / m->KH);
    if (!launch(c, embed_rows_kernel, dim3(T), dim3(256), 0, m->emb, static_cast<const uint32_t *>(b->d_tokens), m->V,
                H, m->p_states, m->d_error))
        return false;
    // As record_prompt: row kernels write the next projection's BF16 terms and
    // sum the previous projection's split-K partials.
    Deferred down_parts;
    for (uint64_t l = 0; l < m->L; ++l) {
        const DLayer &L = m->layers[l];
        bool ok;
        RowFuse f = row_fuse(c, m, L.qkv_w, T, m->QW, H, down_parts);
        if (l == 0)
            ok = launch(c, norm_rows_kernel<ROW_NORM>, dim3(T), dim3(512), 0, m->p_states,
                        static_cast<const float *>(nullptr), static_cast<const uint16_t *>(nullptr), 0.0f, L.pre,
                        1.0f, m->p_norm, H, f);
        else
            ok = launch(c, norm_rows_kernel<ROW_RESID_NORM>, dim3(T), dim3(512), 0, m->p_states,
                        static_cast<const float *>(m->p_branch), m->layers[l - 1].mpost, kPostMlpOffset, L.pre,
                        1.0f, m->p_norm, H, f);
        if (!ok || !projection(c, m, m->p_norm, H, L.qkv_w, m->p_qkv, m->QW, T, m->QW, H, f.split != nullptr))
            return false;
        if (!launch(c, decode_attention128_batch_kernel, dim3(static_cast<uint32_t>(m->KH), kDec128BatchSplits, b->B),
                    dim3(kDecThreads), decode_attention128_smem(G),
                    static_cast<const DecodeAttnParams *>(b->d_attn + l * b->B)))
            return false;
        Deferred o_parts;
        if (!projection(c, m, m->p_attn, m->AW, L.o_w, m->p_branch, H, T, H, m->AW, false, &o_parts)) return false;
        f = row_fuse(c, m, L.gu, T, 2 * m->I, H, o_parts);
        if (!launch(c, norm_rows_kernel<ROW_RESID_NORM>, dim3(T), dim3(512), 0, m->p_states,
                    static_cast<const float *>(m->p_branch), L.post, kPostMixerOffset, L.mpre, 1.0f, m->p_norm, H, f))
            return false;
        if (!projection(c, m, m->p_norm, H, L.gu, m->p_gu, 2 * m->I, T, 2 * m->I, H, f.split != nullptr)) return false;
        f = row_fuse(c, m, L.down, T, H, m->I, Deferred{});
        if (!swiglu_rows(c, m->p_gu, m->I, T, f)) return false;
        if (!projection(c, m, m->p_gu, 2 * m->I, L.down, m->p_branch, H, T, H, m->I, f.split != nullptr,
                        &down_parts))
            return false;
    }
    const RowFuse fh = row_fuse(c, m, m->head, T, m->V, H, Deferred{});
    if (!launch(c, norm_rows_kernel<ROW_RESID>, dim3(T), dim3(512), 0, m->p_states,
                static_cast<const float *>(m->p_branch), m->layers[m->L - 1].mpost, kPostMlpOffset,
                static_cast<const uint16_t *>(nullptr), 0.0f, static_cast<float *>(nullptr), H,
                row_fuse(c, m, nullptr, T, 0, 0, down_parts)) ||
        !launch(c, norm_rows_kernel<ROW_NORM>, dim3(T), dim3(512), 0, m->p_states,
                static_cast<const float *>(nullptr), static_cast<const uint16_t *>(nullptr), 0.0f, m->norm, 1.0f,
                m->p_norm, H, fh) ||
        !projection(c, m, m->p_norm, H, m->head, m->p_logits, m->V, T, m->V, H, fh.split != nullptr) ||
        !rows_argmax(c, m, m->p_logits, m->V, static_cast<uint32_t>(T), b->d_tokens, nullptr))
        return false;
    return launch(c, batch_advance_kernel, dim3(1), dim3(256), 0, static_cast<uint64_t *const *>(b->d_counters), m->L,
                  b->B);
}

// ---- persistent decode step --------------------------------------------------
// Shapes the one-launch step takes: head dim 128, at most 16 query heads per
// KV head, every projection's columns a whole number (<= 32) of 512-column
// slots, a hidden size the prologue holds in registers, and a grid of one
// co-resident CTA per SM with at least three ring stages.
const char *persistent_plan(plamo_cuda *c, DModel *m, uint32_t *grid, size_t *smem, uint32_t *stages,
                            uint32_t *splits) {
    if (!c->persistent) return "one-launch step not enabled (PLAMO_CUDA_PERSISTENT=1)";
    if (!c->cooperative) return "no cooperative launch on this device";
    if (m->tp.active) return "tensor-parallel shard";
    if (m->D != 128 || m->QH % m->KH) return "head shape";
    const uint64_t G = m->QH / m->KH;
    if (G > kPtMaxG || m->H % 512 || m->AW % 512 || m->I % 512 || m->H > kPtMaxHidden) return "projection shape";
    if (m->H / 512 > kPtMaxSlots || m->AW / 512 > kPtMaxSlots || m->I / 512 > kPtMaxSlots) return "row width";
    if (m->L > 0xffff || m->Vh > 0xffffffffull || m->QW > 0xffffffffull) return "model size";
    // Bulk copies and vector loads of every weight need 16-byte alignment
    // (a mapped checkpoint can place a tensor anywhere).
    auto aligned = [](const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15) == 0; };
    if (!aligned(m->emb) || !aligned(m->norm) || !aligned(m->head)) return "unaligned weights";
    for (const DLayer &L : m->layers)
        for (const void *w : {static_cast<const void *>(L.qkv_w), static_cast<const void *>(L.o_w),
                              static_cast<const void *>(L.gu), static_cast<const void *>(L.down),
                              static_cast<const void *>(L.pre), static_cast<const void *>(L.post),
                              static_cast<const void *>(L.mpre), static_cast<const void *>(L.mpost),
                              static_cast<const void *>(L.qn), static_cast<const void *>(L.kn)})
            if (!aligned(w)) return "unaligned weights";
    const uint32_t g = static_cast<uint32_t>(c->sm_count);
    const uint32_t S = static_cast<uint32_t>(std::max<uint64_t>(
        1, std::min<uint64_t>({g / m->KH, kPtMaxSplits, 384 / G})));
    // Largest per-CTA partial block of any projection: rows x slots x pair.
    uint64_t part = 0;
    const uint64_t shapes[5][3] = {{m->QW, m->H, 1}, {m->H, m->AW, 1}, {m->I, m->H, 2}, {m->H, m->I, 1},
                                   {m->Vh, m->H, 1}};
    for (const auto &sh : shapes) part = std::max<uint64_t>(part, (sh[0] + g - 1) / g * (sh[1] / 512) * sh[2]);
    const uint64_t work =
        std::max<uint64_t>(((m->H + 3) & ~3ull) + part, pt_attention_floats(static_cast<uint32_t>(G), S)) * 4;
    cudaFuncAttributes attr{};
    if (cudaFuncGetAttributes(&attr, decode_token_kernel) != cudaSuccess) return "kernel attributes";
    const int64_t room = static_cast<int64_t>(c->smem_optin) - static_cast<int64_t>(attr.sharedSizeBytes) -
                         static_cast<int64_t>(work);
    const int64_t st = std::min<int64_t>(c->pt_stages ? c->pt_stages : kPtDefaultStages, room / kPtStageBytes);
    if (st < 3) return "shared memory";
    const size_t bytes = static_cast<size_t>(st) * kPtStageBytes + work;
    int per_sm = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_token_kernel, kPtThreads, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return cudaGetErrorString(e);
    }
    if (per_sm < 1) return "no resident CTA per SM";
    *grid = g;
    *smem = bytes;
    *stages = static_cast<uint32_t>(st);
    *splits = S;
    return nullptr;
}

bool persistent_init(plamo_cuda *c, DModel *m) {
    uint32_t grid = 0, stages = 0, S = 0;
    size_t smem = 0;
    if (const char *why = persistent_plan(c, m, &grid, &smem, &stages, &S)) {
        snprintf(m->pt_reason, sizeof m->pt_reason, "%s", why);
        return false;
    }
    std::vector<PtLayer> layers(m->L);
    for (uint64_t l = 0; l < m->L; ++l) {
        const DLayer &L = m->layers[l];
        layers[l] = PtLayer{L.qkv_w, L.o_w, L.gu, L.down, L.pre, L.post, L.mpre, L.mpost, attn_layer(m, l)};
    }
    const uint64_t G = m->QH / m->KH;
    auto *d_layers = static_cast<PtLayer *>(dalloc(c, m, m->L * sizeof(PtLayer)));
    auto *apart = static_cast<float *>(dalloc(c, m, m->KH * S * G * (128 + 2) * 4));
    auto *arrive = static_cast<uint32_t *>(dalloc(c, m, std::max<uint64_t>(m->KH, 4) * 4));
    auto *counters = static_cast<unsigned long long *>(dalloc(c, m, 16));
    if (!d_layers || !apart || !arrive || !counters) return false;
    if (!note(c, "persistent layers", cudaMemcpyAsync(d_layers, layers.data(), m->L * sizeof(PtLayer),
                                                      cudaMemcpyHostToDevice, c->stream)) ||
        !note(c, "persistent counters", cudaMemsetAsync(arrive, 0, std::max<uint64_t>(m->KH, 4) * 4, c->stream)) ||
        !note(c, "persistent counters", cudaMemsetAsync(counters, 0, 16, c->stream)) ||
        !note(c, "persistent init", cudaStreamSynchronize(c->stream)))
        return false;
    PtParams &p = m->pt;
    p.layers = d_layers;
    p.L = static_cast<uint32_t>(m->L);
    p.H = static_cast<uint32_t>(m->H);
    p.QH = static_cast<uint32_t>(m->QH);
    p.KH = static_cast<uint32_t>(m->KH);
    p.AW = static_cast<uint32_t>(m->AW);
    p.I = static_cast<uint32_t>(m->I);
    p.QW = static_cast<uint32_t>(m->QW);
    p.head_rows = static_cast<uint32_t>(m->Vh);
    p.vocab = m->V;
    p.emb = m->emb;
    p.norm = m->norm;
    p.head = m->head;
    p.token = m->d_token;
    p.next = m->d_next;
    p.state[0] = m->state[0];
    p.state[1] = m->state[1];
    p.normalized = m->normalized;
    p.logits = m->logits;
    p.qkv = m->qkv;
    p.attn = m->attn;
    p.branch = m->branch;
    p.mid = m->mid;
    p.apart = apart;
    p.head_arrive = arrive;
    p.bar = counters;
    p.gen = counters + 1;
    p.arg_val = m->arg_val;
    p.arg_val2 = m->arg_val2;
    p.arg_idx = m->arg_idx;
    p.arg_nan = m->arg_nan;
    p.appended = m->d_appended;
    p.S = S;
    p.stages = stages;
    p.piece = c->pt_piece;
    m->pt_grid = grid;
    m->pt_smem = smem;
    // The step leaves its final state where the graph's does: the layers flip
    // the ping-pong 2L - 1 times after layer 0 wrote state[0], the head once
    // more, so the head writes state[0].
    m->final_state = m->state[0];
    m->pt_ready = true;
    return true;
}

// Counters back to zero after a failed step (a CTA that stopped early left
// arrivals behind); the next launch starts from generation 0.
bool persistent_reset(plamo_cuda *c, DModel *m) {
    return note(c, "persistent reset",
                cudaMemsetAsync(m->pt.head_arrive, 0, std::max<uint64_t>(m->KH, 4) * 4, c->stream)) &&
           note(c, "persistent reset", cudaMemsetAsync(m->pt.bar, 0, 16, c->stream)) &&
           note(c, "persistent reset", cudaStreamSynchronize(c->stream));
}

bool launch_persistent(plamo_cuda *c, DModel *m) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(m->pt_grid);
    cfg.blockDim = dim3(kPtThreads);
    cfg.dynamicSmemBytes = m->pt_smem;
    cfg.stream = c->stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!note(c, "persistent decode", cudaLaunchKernelEx(&cfg, decode_token_kernel, m->pt))) return false;
    c->info.launches++;
    return true;
}

bool ensure_graph(plamo_cuda *c, DModel *m) {
    if (m->graph_exec || m->pt_ready) return true;
    if (persistent_init(c, m)) return true;
    if (!note(c, "capture", cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal)))
        return false;
    const uint64_t before = c->info.launches;
    const bool ok = record_decode(c, m);
    cudaGraph_t graph = nullptr;
    const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
    if (!ok || !note(c, "capture end", e)) {
        if (graph) cudaGraphDestroy(graph);
        return false;
    }
    m->graph_nodes = c->info.launches - before;
    c->info.launches = before;
    m->graph = graph;
    return note(c, "instantiate", cudaGraphInstantiate(&m->graph_exec, graph, 0));
}

bool launch_decode(plamo_cuda *c, DModel *m) {
    if (m->pt_ready) {
        if (!launch_persistent(c, m)) return false;
        c->info.graph_launches++;
        return true;
    }
    if (!note(c, "graph launch", cudaGraphLaunch(m->graph_exec, c->stream))) return false;
    c->info.graph_launches++;
    c->info.launches += m->graph_nodes;
    return true;
}

bool check_device_error(plamo_cuda *c, DModel *m) {
    uint32_t err = 0;
    if (!note(c, "error flag", cudaMemcpy(&err, m->d_error, 4, cudaMemcpyDeviceToHost))) return false;
    if (err) {
        cudaMemset(m->d_error, 0, 4);
        if (m->pt_ready) persistent_reset(c, m);
        c->info.errors++;
        snprintf(c->info.note, sizeof c->info.note, "%s",
                 err == 1   ? "device rejected a token id"
                 : err == 4 ? "a tensor-parallel peer did not arrive within 2 s"
                 : err == 5 ? "a decode grid barrier did not complete within 2 s"
                            : "a weight stream stalled for 2 s");
        return false;
    }
    return true;
}

// ---- layer-major prompt / verification ------------------------------------
// Attention of T prompt (or candidate) tokens of layer l. From 16 tokens on,
// queries whose window starts at row 0 (all of a full layer; a sliding
// layer's until its window fills) go to the blocked kernel, the rest to the
// per-token kernel; both give the same bits.
bool prompt_attention(plamo_cuda *c, DModel *m, uint64_t l, uint64_t T, size_t attn_smem) {
    const DLayer &L = m->layers[l];
    // The o projection's BF16 input terms, written by the attention kernels
    // themselves when that projection runs on the tensor cores.
    uint16_t *const o_terms = row_fuse(c, m, L.o_w, T, m->H, m->AW, Deferred{}).split;
    const uint64_t o_plane = T * m->AW;
    const AttnLayer al = attn_layer(m, l);
    const AttnShape shape{T, m->QH, m->KH, m->D, m->QW};
    const uint64_t G = m->QH / m->KH;
    uint64_t blocked = 0;
    if (c->prompt_attn && T >= 16 && m->D == kPaD && G <= kPaRows)
        blocked = L.sliding ? (L.capacity > L.appended ? std::min(T, L.capacity - L.appended) : 0) : T;
    if (blocked) {
        // Every key the blocked queries see, rotated once: rows [0, P + blocked).
        const uint64_t keys = L.appended + blocked;
        const uint32_t kgrid = static_cast<uint32_t>(
            std::min<uint64_t>((keys * m->KH * (kPaD / 2) + 255) / 256, static_cast<uint64_t>(c->sm_count) * 8));
        if (!launch(c, prompt_keys_kernel, dim3(kgrid), dim3(256), 0, al, static_cast<const float *>(m->p_qkv),
                    static_cast<uint32_t>(m->QW), static_cast<uint32_t>(m->QH), static_cast<uint32_t>(m->KH),
                    m->p_rotk, static_cast<uint32_t>(keys)))
            return false;
        // 32 query rows per CTA while 64-row blocks would not fill two waves
        // of two CTAs per SM (the longest blocks would set the launch time).
        const bool narrow = G <= 32 && (c->prompt_rows ? c->prompt_rows == 32
                                                       : ((blocked + kPaRows / G - 1) / (kPaRows / G)) * m->KH <
                                                             4ull * static_cast<uint64_t>(c->sm_count));
        const uint32_t per_block = static_cast<uint32_t>((narrow ? 32 : kPaRows) / G);
        PromptAttnParams pp{al,
                            m->p_q,
                            m->p_qkv,
                            m->p_rotk,
                            m->p_attn,
                            static_cast<uint32_t>(m->QH),
                            static_cast<uint32_t>(m->KH),
                            static_cast<uint32_t>(m->QW),
                            static_cast<uint32_t>(blocked),
                            per_block,
                            o_terms,
                            o_plane};
        const dim3 grid(static_cast<uint32_t>((blocked + per_block - 1) / per_block), static_cast<uint32_t>(m->KH));
        if (!(narrow ? (c->prompt_bufs == 1 ? launch(c, prompt_attention_kernel<32, 1>, grid, dim3(kPaThreads),
                                                     prompt_attention_smem_bytes<32, 1>(), pp)
                                            : launch(c, prompt_attention_kernel<32>, grid, dim3(kPaThreads),
                                                     prompt_attention_smem_bytes<32>(), pp))
                     : launch(c, prompt_attention_kernel<64>, grid, dim3(kPaThreads),
                              prompt_attention_smem_bytes<64>(), pp)))
            return false;
    }
    if (blocked == T) return true;
    const uint32_t splits = T >= 16 ? 1u : m->splits;
    AttnParams ap{al, shape, m->p_q, m->p_qkv, m->p_attn, m->p_part, m->p_tickets, splits,
                  static_cast<uint32_t>(blocked), o_terms, o_plane};
    return launch(c, attention_kernel, dim3(m->KH, T - blocked, splits), dim3(kAttnThreads), attn_smem, ap);
}

// mode 0: prefill (rows stored into the rings); 1: verification (rows kept
// per layer in v_kv, nothing committed).
bool record_prompt(plamo_cuda *c, DModel *m, uint64_t T, int mode, bool need_all_logits) {
    const uint64_t H = m->H;
    AttnShape shape{T, m->QH, m->KH, m->D, m->QW};
    const uint64_t G = m->QH / m->KH;
    const size_t attn_smem = attention_smem_bytes(G, m->D);
    if (!launch(c, embed_rows_kernel, dim3(T), dim3(256), 0, m->emb, static_cast<const uint32_t *>(m->p_ids),
                m->V, H, m->p_states, m->d_error))
        return false;
    // The row kernels write the BF16 terms of the next projection's input and
    // take the previous projection's split-K partials directly (RowFuse);
    // tensor-parallel branches are all-reduced in place, so nothing is
    // deferred across an exchange.
    const bool tp = m->tp.active;
    Deferred down_parts;
    for (uint64_t l = 0; l < m->L; ++l) {
        const DLayer &L = m->layers[l];
        bool ok;
        RowFuse f = row_fuse(c, m, L.qkv_w, T, m->QW, H, down_parts);
        if (l == 0)
            ok = launch(c, norm_rows_kernel<ROW_NORM>, dim3(T), dim3(512), 0, m->p_states,
                        static_cast<const float *>(nullptr), static_cast<const uint16_t *>(nullptr), 0.0f, L.pre,
                        1.0f, m->p_norm, H, f);
        else
            ok = launch(c, norm_rows_kernel<ROW_RESID_NORM>, dim3(T), dim3(512), 0, m->p_states,
                        static_cast<const float *>(m->p_branch), m->layers[l - 1].mpost, kPostMlpOffset, L.pre,
                        1.0f, m->p_norm, H, f);
        if (!ok || !projection(c, m, m->p_norm, H, L.qkv_w, m->p_qkv, m->QW, T, m->QW, H, f.split != nullptr))
            return false;
        AttnLayer al = attn_layer(m, l);
        if (!(m->D == 128 ? launch(c, qk_prep128_kernel, dim3(static_cast<uint32_t>((m->QH + m->KH + 7) / 8), T),
                                   dim3(256), 0, m->p_qkv, m->p_q, al, shape)
                          : launch(c, qk_prep_kernel, dim3(m->QH + m->KH, T), dim3(128), 0, m->p_qkv, m->p_q, al,
                                   shape)))
            return false;
        if (!prompt_attention(c, m, l, T, attn_smem)) return false;
        if (mode == 0) {
            const uint64_t first = T > L.ring ? T - L.ring : 0;
            if (!launch(c, kv_store_kernel, dim3(T - first), dim3(256), 0, al, shape,
                        static_cast<const float *>(m->p_qkv), first))
                return false;
        } else {
            // K and V of every candidate, per layer: [T][2][KVW]
            float *dst = m->v_kv + l * kVerifyMax * 2 * m->KVW;
            if (!note(c, "verify kv", cudaMemcpy2DAsync(dst, 2 * m->KVW * 4, m->p_qkv + m->QH * m->D,
                                                        m->QW * 4, 2 * m->KVW * 4, T, cudaMemcpyDeviceToDevice,
                                                        c->stream)))
                return false;
        }
        Deferred o_parts;
        const bool o_terms = row_fuse(c, m, L.o_w, T, H, m->AW, Deferred{}).split != nullptr;
        if (!projection(c, m, m->p_attn, m->AW, L.o_w, m->p_branch, H, T, H, m->AW, o_terms,
                        tp ? nullptr : &o_parts))
            return false;
        if (tp && !tp_allreduce_rows(c, m, m->p_branch, T, 2 * l)) return false;
        f = row_fuse(c, m, L.gu, T, 2 * m->I, H, o_parts);
        if (!launch(c, norm_rows_kernel<ROW_RESID_NORM>, dim3(T), dim3(512), 0, m->p_states,
                    static_cast<const float *>(m->p_branch), L.post, kPostMixerOffset, L.mpre, 1.0f, m->p_norm, H, f))
            return false;
        if (f.split && glu_fusable(c, m, L.gu, L.down, T)) {
            // gate/up + SwiGLU in one launch; down reads the terms it wrote.
            if (!projection_glu(c, m, L.gu, T) ||
                !projection_with(c, nullptr, 0, L.down, m->p_branch, H, T, H, m->I, m->p_glu, m->d_error,
                                 m->p_splitk, kSplitkFloats, true, tp ? nullptr : &down_parts))
                return false;
        } else {
            if (!projection(c, m, m->p_norm, H, L.gu, m->p_gu, 2 * m->I, T, 2 * m->I, H, f.split != nullptr))
                return false;
            f = row_fuse(c, m, L.down, T, H, m->I, Deferred{});
            if (!swiglu_rows(c, m->p_gu, m->I, T, f)) return false;
            if (!projection(c, m, m->p_gu, 2 * m->I, L.down, m->p_branch, H, T, H, m->I, f.split != nullptr,
                            tp ? nullptr : &down_parts))
                return false;
        }
        if (tp && !tp_allreduce_rows(c, m, m->p_branch, T, 2 * l + 1)) return false;
    }
    if (!launch(c, norm_rows_kernel<ROW_RESID>, dim3(T), dim3(512), 0, m->p_states,
                static_cast<const float *>(m->p_branch), m->layers[m->L - 1].mpost, kPostMlpOffset,
                static_cast<const uint16_t *>(nullptr), 0.0f, static_cast<float *>(nullptr), H,
                row_fuse(c, m, nullptr, T, 0, 0, down_parts)))
        return false;
    if (need_all_logits) {
        const RowFuse f = row_fuse(c, m, m->head, T, m->Vh, H, Deferred{});
        if (!launch(c, norm_rows_kernel<ROW_NORM>, dim3(T), dim3(512), 0, m->p_states,
                    static_cast<const float *>(nullptr), static_cast<const uint16_t *>(nullptr), 0.0f, m->norm,
                    1.0f, m->p_norm, H, f))
            return false;
        return projection(c, m, m->p_norm, H, m->head, m->p_logits, m->Vh, T, m->Vh, H, f.split != nullptr);
    }
    // Final norm and head for the last prompt token only (reference
    // src/prefill.s:136-158), with the greedy choice on the device.
    GemvParams h{};
    h.w = m->head;
    h.rows = m->Vh;
    h.cols = H;
    h.state_in = m->p_states + (T - 1) * H;
    h.norm2 = m->norm;
    h.off2 = 1.0f;
    h.state_out = m->final_state;
    h.norm_out = m->normalized;
    h.y = m->logits;
    h.arg_val = m->arg_val;
    h.arg_val2 = m->arg_val2;
    h.arg_idx = m->arg_idx;
    h.arg_nan = m->arg_nan;
    uint32_t grid = 0;
    if (!gemv<PRO_NORM, EPI_ARGMAX>(c, h, &grid)) return false;
    if (!greedy_choice(c, m, grid)) return false;
    if (!launch(c, advance_kernel, dim3(1), dim3(32), 0, m->d_appended, m->L, T)) return false;
    return !m->tp.active || launch(c, tp_epoch_kernel, dim3(1), dim3(32), 0, m->tp.epoch);
}

bool copy_outputs(plamo_cuda *c, DModel *m) {
    struct model *h = m->host;
    return note(c, "state", cudaMemcpyAsync(h->state, m->final_state, m->H * 4, cudaMemcpyDeviceToHost, c->stream)) &&
           note(c, "normalized", cudaMemcpyAsync(h->normalized, m->normalized, m->H * 4, cudaMemcpyDeviceToHost,
                                                 c->stream)) &&
           note(c, "logits", cudaMemcpyAsync(h->logits + m->tp.voff, m->logits, m->Vh * 4, cudaMemcpyDeviceToHost,
                                             c->stream));
}

bool sync_kv(plamo_cuda *c, DModel *m);

double elapsed(plamo_cuda *c) {
    float ms = 0;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    return ms * 1e-3;
}

}  // namespace

// ============================================================================
extern "C" {

struct plamo_cuda *plamo_cuda_open(const struct plamo_cuda_config *config, char *error, size_t cap) {
    plamo_cuda_config cfg{};
    if (config) cfg = *config;
    if (!cfg.max_context) cfg.max_context = 8192 + 16;
    if (!cfg.max_prefill) cfg.max_prefill = 4096;
    if (!cfg.reserve) cfg.reserve = 1ull << 30;
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count <= cfg.device || cfg.device < 0) {
        if (error && cap) snprintf(error, cap, "CUDA requires an available device (%s)",
                                   e == cudaSuccess ? "ordinal out of range" : cudaGetErrorString(e));
        return nullptr;
    }
    cudaDeviceProp prop{};
    if ((e = cudaSetDevice(cfg.device)) != cudaSuccess ||
        (e = cudaGetDeviceProperties(&prop, cfg.device)) != cudaSuccess) {
        if (error && cap) snprintf(error, cap, "cannot open CUDA device: %s", cudaGetErrorString(e));
        return nullptr;
    }
    if (prop.major < 10) {
        if (error && cap) snprintf(error, cap, "device %s is sm_%d%d; this build targets sm_100a", prop.name,
                                   prop.major, prop.minor);
        return nullptr;
    }
    auto *c = new plamo_cuda();
    c->device = cfg.device;
    c->config = cfg;
    memset(&c->info, 0, sizeof c->info);
    snprintf(c->info.device, sizeof c->info.device, "%.127s", prop.name);
    c->sm_count = prop.multiProcessorCount;
    c->info.sm_count = prop.multiProcessorCount;
    const char *pdl = getenv("PLAMO_CUDA_PDL");
    c->pdl = !pdl || strcmp(pdl, "0");
    const char *bulk = getenv("PLAMO_CUDA_BULK_GEMV");
    c->bulk_gemv = !bulk || strcmp(bulk, "0");
    const char *tc = getenv("PLAMO_CUDA_TC_GEMM");
    c->tc_gemm = !tc || strcmp(tc, "0");
    const char *pa = getenv("PLAMO_CUDA_PROMPT_ATTN");
    c->prompt_attn = !pa || strcmp(pa, "0");
    const char *pbuf = getenv("PLAMO_CUDA_PROMPT_BUFS");
    // One tile buffer lets three 32-row CTAs share an SM instead of two with
    // two buffers (8B 455-token prefill 17.36K -> 17.43K tok/s).
    c->prompt_bufs = pbuf && !strcmp(pbuf, "2") ? 2 : 1;
    const char *prow = getenv("PLAMO_CUDA_PROMPT_ROWS");
    c->prompt_rows = prow && (atoi(prow) == 32 || atoi(prow) == 64) ? atoi(prow) : 0;
    // The one-launch step is opt-in: on the 8B profile it measured 4.8 ms per
    // token against 3.38 ms for the graph (its per-phase grid barriers and
    // prologues cost more than the graph's programmatic launch boundaries).
    const char *pt = getenv("PLAMO_CUDA_PERSISTENT");
    c->persistent = pt && !strcmp(pt, "1");
    int coop = 0;
    cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, cfg.device);
    c->cooperative = coop != 0;
    const char *piece = getenv("PLAMO_CUDA_PT_PIECE_KB");
    c->pt_piece = 1024u * static_cast<uint32_t>(piece ? std::max(1, std::min(atoi(piece), 32)) : 8);
    const char *pst = getenv("PLAMO_CUDA_PT_STAGES");
    c->pt_stages = pst ? std::max(3, std::min(atoi(pst), kPtMaxStages)) : 0;
    // Draft confidence settings, parsed as reference runtime/worker.c:199-208
    // (invalid values fall back to the default rule).
    c->draft_margin = -1.0f;
    c->draft_min_tokens = 0;
    if (const char *dm = getenv("PLAMO_DRAFT_MIN_MARGIN")) {
        char *end = nullptr;
        const float v = strtof(dm, &end);
        if (*dm && end && !*end && std::isfinite(v) && v >= 0.0f) c->draft_margin = v;
    }
    if (const char *dt = getenv("PLAMO_DRAFT_MIN_TOKENS")) {
        char *end = nullptr;
        const unsigned long v = strtoul(dt, &end, 10);
        if (*dt && end && !*end && v >= 1 && v <= kVerifyMax) c->draft_min_tokens = static_cast<unsigned>(v);
    }
    const char *tc_st = getenv("PLAMO_CUDA_TC_STAGES");
    c->tc_stages = tc_st ? std::max(2, std::min(atoi(tc_st), kTcMaxStages)) : 0;
    const char *tokm = getenv("PLAMO_CUDA_TC_TOKM");
    c->tc_tokm = tokm && (!strcmp(tokm, "0") || !strcmp(tokm, "1")) ? atoi(tokm) : -1;
    const char *tokn = getenv("PLAMO_CUDA_TC_TOKN");
    c->tc_tokn = tokn && (!strcmp(tokn, "144") || !strcmp(tokn, "160") || !strcmp(tokn, "192")) ? atoi(tokn) : 0;
    const char *glu = getenv("PLAMO_CUDA_TC_GLU");
    c->tc_glu = !(glu && !strcmp(glu, "0"));
    const char *ring_kb = getenv("PLAMO_CUDA_GEMV_RING_KB");
    c->gemv_ring_kb = ring_kb ? std::max(16, atoi(ring_kb)) : 96;
    const char *ctas = getenv("PLAMO_CUDA_GEMV_CTAS");
    c->gemv_ctas = ctas ? std::max(1, atoi(ctas)) : 1;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess ||
        (e = cudaEventCreate(&c->ev0)) != cudaSuccess || (e = cudaEventCreate(&c->ev1)) != cudaSuccess ||
        (e = cudaMallocHost(&c->pinned_u32, 64 * 1024 * 4)) != cudaSuccess ||
        (e = cudaMalloc(&c->sink, 4)) != cudaSuccess) {
        if (error && cap) snprintf(error, cap, "cannot create CUDA stream: %s", cudaGetErrorString(e));
        if (c->pinned_u32) cudaFreeHost(c->pinned_u32);
        if (c->ev1) cudaEventDestroy(c->ev1);
        if (c->ev0) cudaEventDestroy(c->ev0);
        if (c->stream) cudaStreamDestroy(c->stream);
        delete c;
        return nullptr;
    }
    c->pinned_capacity = 64 * 1024;
    int optin = 0;
    cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, cfg.device);
    c->smem_optin = optin;
    int per_sm = 0;
    cudaDeviceGetAttribute(&per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, cfg.device);
    c->smem_per_sm = per_sm > 0 ? per_sm : optin;
    const char *carve = getenv("PLAMO_CUDA_CARVEOUT");
    // Max-shared carveout by default: the decode kernels' CTAs then land on SMs
    // still running the previous kernel (batched 8B decode step 4.77 -> 4.33 ms).
    const int carveout = carve ? std::max(-1, std::min(atoi(carve), 100)) : 100;
    set_gemv_smem_limits<PRO_X, EPI_STORE>(optin, carveout);
    set_gemv_smem_limits<PRO_NORM, EPI_STORE>(optin, carveout);
    set_gemv_smem_limits<PRO_RESID_NORM, EPI_STORE>(optin, carveout);
    set_gemv_smem_limits<PRO_EMBED_NORM, EPI_STORE>(optin, carveout);
    set_gemv_smem_limits<PRO_RESID_NORM, EPI_SWIGLU>(optin, carveout);
    set_gemv_smem_limits<PRO_RESID_NORM, EPI_ARGMAX>(optin, carveout);
    set_gemv_smem_limits<PRO_RESID_NORM_TP, EPI_STORE>(optin, carveout);
    set_gemv_smem_limits<PRO_RESID_NORM_TP, EPI_SWIGLU>(optin, carveout);
    set_gemv_smem_limits<PRO_RESID_NORM_TP, EPI_ARGMAX>(optin, carveout);
    set_gemv_smem_limits<PRO_NORM, EPI_ARGMAX>(optin, carveout);
    allow_smem(attention_kernel, optin, carveout);
    allow_smem(prompt_attention_kernel<64>, optin, carveout);
    allow_smem(prompt_attention_kernel<32>, optin, carveout);
    allow_smem(prompt_attention_kernel<32, 1>, optin, carveout);
    allow_smem(decode_attention128_kernel, optin, carveout);
    allow_smem(gemm_tc_kernel<16>, optin, carveout);
    allow_smem(gemm_tc_kernel<32>, optin, carveout);
    allow_smem(gemm_tc_kernel<64>, optin, carveout);
    allow_smem(gemm_tc_kernel<128>, optin, carveout);
    allow_smem(gemm_tc_kernel<144, true>, optin, carveout);
    allow_smem(gemm_tc_kernel<160, true>, optin, carveout);
    allow_smem(gemm_tc_kernel<192, true>, optin, carveout);
    allow_smem(decode_attention_kernel<128>, optin, carveout);
    allow_smem(decode_attention128_batch_kernel, optin, carveout);
    allow_smem(decode_attention_kernel<0>, optin, carveout);
    allow_smem(decode_token_kernel, optin, carveout);
    prefer_carveout(argmax_merge_kernel, carveout);
    prefer_carveout(advance_kernel, carveout);
    prefer_carveout(tp_epoch_kernel, carveout);
    cudaFuncSetAttribute(decode_attention128_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaFuncSetAttribute(decode_attention128_batch_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if ((e = cudaGetLastError()) != cudaSuccess) {
        if (error && cap) snprintf(error, cap, "cannot configure kernels: %s", cudaGetErrorString(e));
        plamo_cuda_close(c);
        return nullptr;
    }
    return c;
}

void plamo_cuda_close(struct plamo_cuda *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto &kv : c->models) free_model(c, kv.second.get());
    for (auto &kv : c->kv_pools) {
        for (float *chunk : kv.second.chunks) cudaFree(chunk);
        cudaFree(kv.second.spare);
    }
    for (auto &r : c->ropes) cudaFree(r->dev);
    for (Range &r : c->ranges) cudaFree(r.dev);
    cudaFreeHost(c->pinned_u32);
    cudaFree(c->sink);
    cudaFree(c->staging);
    cudaEventDestroy(c->ev0);
    cudaEventDestroy(c->ev1);
    cudaStreamDestroy(c->stream);
    delete c;
}

void plamo_cuda_maintain(struct plamo_cuda *c) {
    if (!c) return;
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    // KV page chunks go back to the device once no request maps any of their
    // pool's pages (the spare page stays: page tables point at it).
    for (auto &kv : c->kv_pools) {
        KvPool &pool = kv.second;
        if (pool.used || pool.chunks.empty()) continue;
        const uint64_t chunk_bytes = kKvChunkPages * kv_page_floats(kv.first) * 4;
        for (float *chunk : pool.chunks) cudaFree(chunk);
        c->info.kv_bytes -= pool.chunks.size() * chunk_bytes;
        c->info.allocated_bytes -= pool.chunks.size() * chunk_bytes;
        c->info.kv_pages_allocated -= pool.chunks.size() * kKvChunkPages;
        pool.chunks.clear();
        pool.free.clear();
    }
}

void plamo_cuda_get_info(const struct plamo_cuda *c, struct plamo_cuda_info *info) {
    if (!c || !info) return;
    *info = c->info;
}

int plamo_cuda_preload(struct plamo_cuda *c, const void *src, uint64_t bytes) {
    if (!c || !src || !bytes) return 0;
    if (find_range(c, src, bytes)) return 1;
    cudaSetDevice(c->device);
    char *dev = nullptr;
    if (!note(c, "preload alloc", cudaMalloc(&dev, bytes))) return 0;
    if (!note(c, "preload copy", cudaMemcpy(dev, src, bytes, cudaMemcpyHostToDevice))) {
        cudaFree(dev);
        return 0;
    }
    c->ranges.push_back({reinterpret_cast<uintptr_t>(src), bytes, dev});
    c->info.weight_bytes += bytes;
    c->info.allocated_bytes += bytes;
    return 1;
}

int plamo_cuda_preload_synthetic(struct plamo_cuda *c, const void *host_key, uint64_t count, uint64_t seed,
                                 float mean, float std) {
    if (!c || !host_key || !count) return 0;
    cudaSetDevice(c->device);
    char *dev = nullptr;
    if (!note(c, "synthetic alloc", cudaMalloc(&dev, count * 2))) return 0;
    if (!plamo_cuda_fill_synthetic_bf16(c, reinterpret_cast<uint16_t *>(dev), count, seed, mean, std)) {
        cudaFree(dev);
        return 0;
    }
    c->ranges.push_back({reinterpret_cast<uintptr_t>(host_key), count * 2, dev});
    c->info.weight_bytes += count * 2;
    c->info.allocated_bytes += count * 2;
    return 1;
}

int plamo_cuda_preload_synthetic_rows(struct plamo_cuda *c, const void *host_key, uint64_t cols, uint64_t full_cols,
                                      uint64_t col0, const uint64_t *row_start, const uint64_t *row_count,
                                      unsigned segments, uint64_t seed, float mean, float std) {
    if (!c || !host_key || !cols || col0 + cols > full_cols || !row_start || !row_count || !segments) return 0;
    uint64_t rows = 0;
    for (unsigned i = 0; i < segments; ++i) rows += row_count[i];
    if (!rows) return 0;
    cudaSetDevice(c->device);
    char *dev = nullptr;
    if (!note(c, "synthetic alloc", cudaMalloc(&dev, rows * cols * 2))) return 0;
    uint16_t *dst = reinterpret_cast<uint16_t *>(dev);
    for (unsigned i = 0; i < segments; ++i) {
        if (!row_count[i]) continue;
        fill_synthetic_rows_kernel<<<c->sm_count * 8, 256, 0, c->stream>>>(dst, row_count[i], cols, seed,
                                                                          row_start[i], col0, full_cols, mean, std);
        c->info.launches++;
        dst += row_count[i] * cols;
    }
    if (!note(c, "synthetic", cudaGetLastError()) || !note(c, "synthetic", cudaStreamSynchronize(c->stream))) {
        cudaFree(dev);
        return 0;
    }
    c->ranges.push_back({reinterpret_cast<uintptr_t>(host_key), rows * cols * 2, dev});
    c->info.weight_bytes += rows * cols * 2;
    c->info.allocated_bytes += rows * cols * 2;
    return 1;
}

int plamo_cuda_fill_synthetic_bf16(struct plamo_cuda *c, uint16_t *dst, uint64_t count, uint64_t seed, float mean,
                                   float std) {
    if (!c) return 0;
    fill_synthetic_bf16_kernel<<<c->sm_count * 8, 256, 0, c->stream>>>(dst, count, seed, mean, std);
    c->info.launches++;
    return note(c, "synthetic", cudaGetLastError()) && note(c, "synthetic", cudaStreamSynchronize(c->stream));
}

int plamo_cuda_fill_synthetic_f32(struct plamo_cuda *c, float *dst, uint64_t count, uint64_t seed, float mean,
                                  float std) {
    if (!c) return 0;
    fill_synthetic_f32_kernel<<<c->sm_count * 8, 256, 0, c->stream>>>(dst, count, seed, mean, std);
    c->info.launches++;
    return note(c, "synthetic", cudaGetLastError()) && note(c, "synthetic", cudaStreamSynchronize(c->stream));
}

int plamo_cuda_warm_cache(struct plamo_cuda *c) {
    if (!c) return 0;
    for (const Range &r : c->ranges) {
        touch_kernel<<<c->sm_count * 4, 256, 0, c->stream>>>(reinterpret_cast<const uint4 *>(r.dev), r.bytes / 16,
                                                              c->sink);
        c->info.launches++;
    }
    return note(c, "warm", cudaStreamSynchronize(c->stream));
}

// Device state of `model` whose head holds `head_rows` rows (the vocabulary,
// or a tensor-parallel rank's slice of it).
static int prepare_impl(struct plamo_cuda *c, struct model *model, uint64_t head_rows) {
    if (!c || !model || !model->count || !model->hidden || !model->vocab || !model->layers || !head_rows ||
        head_rows > model->vocab)
        return 0;
    cudaSetDevice(c->device);
    if (DModel *old = find_model(c, model)) {
        if (old->signature == model_signature(model) && old->Vh == head_rows && !old->tp.size) return 1;
        // Another descriptor now lives at this address: drop the stale state.
        cudaStreamSynchronize(c->stream);
        free_model(c, old);
        c->models.erase(model);
    }
    auto m = std::make_unique<DModel>();
    m->host = model;
    m->signature = model_signature(model);
    const struct qkv *q0 = model->layers[0]->mixer->qkv;
    m->H = model->hidden;
    m->QH = q0->qh;
    m->KH = q0->kh;
    m->D = q0->dim;
    m->I = model->layers[0]->mlp->intermediate;
    m->V = model->vocab;
    m->Vh = head_rows;
    m->L = model->count;
    m->QW = (m->QH + 2 * m->KH) * m->D;
    m->AW = m->QH * m->D;
    m->KVW = m->KH * m->D;
    if (!m->KH || m->QH % m->KH || !m->D || m->D % 2 || m->D > 512 || !m->I) {
        snprintf(c->info.note, sizeof c->info.note, "unsupported attention shape");
        return 0;
    }
    const uint64_t H = m->H;
    m->emb = resolve(c, model->embedding, m->V * H * 2, true);
    m->head = resolve(c, model->head, m->Vh * H * 2, true);
    m->norm = resolve(c, model->norm, H * 2, true);
    if (!m->emb || !m->head || !m->norm) return 0;
    m->d_appended = static_cast<uint64_t *>(dalloc(c, m.get(), m->L * 8));
    for (uint64_t l = 0; l < m->L; ++l) {
        struct layer *hl = model->layers[l];
        const struct qkv *q = hl->mixer->qkv;
        const struct mlp *p = hl->mlp;
        const struct cache *kc = hl->mixer->cache;
        if (q->qh != m->QH || q->kh != m->KH || q->dim != m->D || q->hidden != H || p->intermediate != m->I ||
            kc->width != m->KVW || !kc->capacity) {
            snprintf(c->info.note, sizeof c->info.note, "layers differ in shape");
            return 0;
        }
        DLayer L{};
        L.host = hl;
        L.qkv_w = resolve(c, q->weight, m->QW * H * 2, true);
        L.qn = resolve(c, q->qn, m->D * 2, true);
        L.kn = resolve(c, q->kn, m->D * 2, true);
        L.o_w = resolve(c, hl->mixer->weight, H * m->AW * 2, true);
        L.pre = resolve(c, hl->pre, H * 2, true);
        L.post = resolve(c, hl->post, H * 2, true);
        L.mpre = resolve(c, p->pre, H * 2, true);
        L.mpost = resolve(c, p->post, H * 2, true);
        L.gu = resolve(c, p->gu, 2 * m->I * H * 2, true);
        L.down = resolve(c, p->down, H * m->I * 2, true);
        if (!L.qkv_w || !L.qn || !L.kn || !L.o_w || !L.pre || !L.post || !L.mpre || !L.mpost || !L.gu || !L.down)
            return 0;
        L.capacity = kc->capacity;
        L.sliding = kc->sliding != 0;
        // A sliding ring keeps spare slots so that one speculative row can be
        // written without evicting a row still inside the window.
        L.ring = L.sliding ? kc->capacity + kVerifyMax + 1
                           : std::min<uint64_t>(kc->capacity, c->config.max_context);
        L.scale = model->scales[l];
        const uint64_t positions = L.sliding ? kc->capacity : std::min<uint64_t>(kc->capacity, c->config.max_context);
        L.rope = get_rope(c, hl->mixer->rotation->freq, m->D, L.scale, positions);
        if (!L.rope) return 0;
        // Page table: every entry on the spare page until a page is mapped;
        // a sliding ring maps all its pages now, a full layer as rows arrive.
        KvPool *pool = kv_pool(c, m->KVW);
        if (!pool) return 0;
        const uint64_t npages = (L.ring + kKvPageRows - 1) / kKvPageRows;
        L.pages.assign(npages, pool->spare);
        L.mapped = 0;
        L.d_pages = static_cast<float **>(dalloc(c, m.get(), npages * sizeof(float *)));
        if (!L.d_pages ||
            !note(c, "kv page table", cudaMemcpy(L.d_pages, L.pages.data(), npages * sizeof(float *),
                                                 cudaMemcpyHostToDevice)))
            return 0;
        L.appended = 0;
        m->layers.push_back(L);
        if (L.sliding && !kv_map(c, m.get(), m->layers.back(), L.ring)) return 0;
    }
    // Decode buffers.
    const uint64_t G = m->QH / m->KH;
    (void)G;
    m->splits = 16;
    const uint64_t before = c->info.allocated_bytes;
    m->state[0] = static_cast<float *>(dalloc(c, m.get(), H * 4));
    m->state[1] = static_cast<float *>(dalloc(c, m.get(), H * 4));
    m->final_state = m->state[0];
    m->normalized = static_cast<float *>(dalloc(c, m.get(), H * 4));
    m->logits = static_cast<float *>(dalloc(c, m.get(), m->Vh * 4));
    m->qkv = static_cast<float *>(dalloc(c, m.get(), m->QW * 4));
    m->q = static_cast<float *>(dalloc(c, m.get(), m->AW * 4));
    m->attn = static_cast<float *>(dalloc(c, m.get(), m->AW * 4));
    m->branch = static_cast<float *>(dalloc(c, m.get(), H * 4));
    m->mid = static_cast<float *>(dalloc(c, m.get(), m->I * 4));
    m->part = static_cast<float *>(dalloc(c, m.get(), m->QH * m->splits * (m->D + 2) * 4));
    m->tickets = static_cast<uint32_t *>(dalloc(c, m.get(), m->KH * 4));
    const uint64_t grid_max = static_cast<uint64_t>(c->sm_count) * 64;
    m->arg_val = static_cast<float *>(dalloc(c, m.get(), grid_max * 4));
    m->arg_val2 = static_cast<float *>(dalloc(c, m.get(), grid_max * 4));
    m->arg_idx = static_cast<uint32_t *>(dalloc(c, m.get(), grid_max * 4));
    m->arg_nan = static_cast<uint32_t *>(dalloc(c, m.get(), grid_max * 4));
    m->d_token = static_cast<uint32_t *>(dalloc(c, m.get(), 16));
    // [next token, error flag, top-2 margin bits]: one read returns all.
    m->d_next = static_cast<uint32_t *>(dalloc(c, m.get(), 16));
    m->d_error = m->d_next + 1;
    // Prompt buffers.
    m->tmax = std::max<uint64_t>(c->config.max_prefill, kVerifyMax);
    const uint64_t T = m->tmax;
    m->p_states = static_cast<float *>(dalloc(c, m.get(), T * H * 4));
    m->p_norm = static_cast<float *>(dalloc(c, m.get(), T * H * 4));
    m->p_qkv = static_cast<float *>(dalloc(c, m.get(), T * m->QW * 4));
    m->p_q = static_cast<float *>(dalloc(c, m.get(), T * m->AW * 4));
    m->p_attn = static_cast<float *>(dalloc(c, m.get(), T * m->AW * 4));
    m->p_branch = static_cast<float *>(dalloc(c, m.get(), T * H * 4));
    m->p_gu = static_cast<float *>(dalloc(c, m.get(), T * 2 * m->I * 4));
    m->p_logits = static_cast<float *>(dalloc(c, m.get(), kVerifyMax * m->Vh * 4));
    m->p_part = static_cast<float *>(dalloc(c, m.get(), kVerifyMax * m->QH * m->splits * (m->D + 2) * 4));
    m->p_tickets = static_cast<uint32_t *>(dalloc(c, m.get(), T * m->KH * 4));
    uint64_t rot_rows = 0;
    for (const DLayer &L : m->layers) rot_rows = std::max(rot_rows, L.capacity);
    m->p_rotk = static_cast<float *>(dalloc(c, m.get(), rot_rows * m->KVW * 4));
    m->p_ids = static_cast<uint32_t *>(dalloc(c, m.get(), T * 4));
    m->p_next = static_cast<uint32_t *>(dalloc(c, m.get(), kVerifyMax * 4));
    m->v_kv = static_cast<float *>(dalloc(c, m.get(), m->L * kVerifyMax * 2 * m->KVW * 4));
    const uint64_t kmax = std::max<uint64_t>(std::max<uint64_t>(H, m->AW), m->I);
    m->p_split = static_cast<uint16_t *>(dalloc(c, m.get(), 3 * T * kmax * 2));
    m->p_glu = T > 64 ? static_cast<uint16_t *>(dalloc(c, m.get(), 3 * T * m->I * 2)) : nullptr;
    m->p_splitk = static_cast<float *>(dalloc(c, m.get(), kSplitkFloats * 4));
    for (void *p : m->allocations)
        if (!p) return 0;
    c->info.workspace_bytes += c->info.allocated_bytes - before;
    // Start from the host's counts (zero for a fresh request).
    if (!reconcile(c, m.get())) {
        free_model(c, m.get());
        return 0;
    }
    if (!note(c, "prepare", cudaStreamSynchronize(c->stream))) return 0;
    c->models[model] = std::move(m);
    return 1;
}

int plamo_cuda_prepare_model(struct plamo_cuda *c, struct model *model) {
    return model ? prepare_impl(c, model, model->vocab) : 0;
}

int plamo_cuda_tp_prepare(struct plamo_cuda *c, struct model *model, unsigned rank, unsigned size,
                          uint64_t vocab_offset, uint64_t vocab_rows, struct plamo_cuda_tp_handle *handle) {
    if (!c || !model || !handle || size < 2 || size > kTpMax || rank >= size || !vocab_rows ||
        vocab_offset + vocab_rows > model->vocab || vocab_offset + vocab_rows > 0xffffffffull)
        return 0;
    cudaSetDevice(c->device);
    if (DModel *old = find_model(c, model)) {  // always a fresh shard
        cudaStreamSynchronize(c->stream);
        free_model(c, old);
        c->models.erase(model);
    }
    if (prepare_impl(c, model, vocab_rows) != 1) return 0;
    DModel *m = find_model(c, model);
    if (m->H % 4) {
        snprintf(c->info.note, sizeof c->info.note, "tensor parallelism needs hidden %% 4 == 0");
        return 0;
    }
    TpState &t = m->tp;
    t.rank = rank;
    t.size = size;
    t.voff = vocab_offset;
    auto align = [](uint64_t x) { return (x + 255) & ~uint64_t{255}; };
    uint64_t off = 0;
    t.off_dparts = off;
    off = align(off + 2 * m->L * size * m->H * 8);
    t.off_dflags = off;
    off = align(off + 2 * m->L * size * 4);
    t.off_pparts = off;
    off = align(off + 2 * size * m->tmax * m->H * 4);
    t.off_pflags = off;
    off = align(off + 2 * m->L * size * 4);
    t.off_args = off;
    off = align(off + kVerifyMax * size * 16);
    t.bytes = off;
    t.xbuf = static_cast<char *>(dalloc(c, m, t.bytes));
    t.tickets = static_cast<uint32_t *>(dalloc(c, m, 4 * m->L * 4));
    t.epoch = static_cast<uint32_t *>(dalloc(c, m, 4));
    t.lval = static_cast<float *>(dalloc(c, m, kVerifyMax * 4));
    t.lidx = static_cast<uint32_t *>(dalloc(c, m, kVerifyMax * 4));
    if (!t.xbuf || !t.tickets || !t.epoch || !t.lval || !t.lidx) return 0;
    c->info.workspace_bytes += t.bytes;
    cudaIpcMemHandle_t h{};
    if (!note(c, "tp handle", cudaIpcGetMemHandle(&h, t.xbuf))) return 0;
    static_assert(sizeof h <= sizeof handle->bytes, "IPC handle size");
    memset(handle->bytes, 0, sizeof handle->bytes);
    memcpy(handle->bytes, &h, sizeof h);
    return 1;
}

int plamo_cuda_tp_connect(struct plamo_cuda *c, struct model *model, const struct plamo_cuda_tp_handle *handles) {
    if (!c || !model || !handles) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || !m->tp.size || m->tp.active) return 0;
    TpState &t = m->tp;
    for (uint32_t r = 0; r < t.size; ++r) {
        if (r == t.rank) {
            t.peer[r] = t.xbuf;
            continue;
        }
        cudaIpcMemHandle_t h{};
        memcpy(&h, handles[r].bytes, sizeof h);
        void *p = nullptr;
        if (!note(c, "tp open", cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess))) return -1;
        t.peer[r] = static_cast<char *>(p);
    }
    t.active = true;
    if (m->graph_exec) {  // re-record with the exchanges
        cudaGraphExecDestroy(m->graph_exec);
        cudaGraphDestroy(m->graph);
        m->graph_exec = nullptr;
        m->graph = nullptr;
    }
    return 1;
}

int plamo_cuda_forward(struct plamo_cuda *c, struct model *model, uint64_t token) {
    uint32_t next;
    if (!c) return 0;
    DModel *m = find_model(c, model);
    if (!m || token >= model->vocab) {
        if (c) c->info.declines++;
        return 0;
    }
    const int r = plamo_cuda_forward_greedy(c, model, token, &next);
    if (r != 1) return r;
    if (!copy_outputs(c, m) || !note(c, "forward", cudaStreamSynchronize(c->stream))) return -1;
    if (c->config.copy_kv_to_host && !sync_kv(c, m)) return -1;
    return 1;
}

int plamo_cuda_forward_greedy_margin(struct plamo_cuda *c, struct model *model, uint64_t token, uint32_t *next,
                                     float *margin);

int plamo_cuda_forward_greedy(struct plamo_cuda *c, struct model *model, uint64_t token, uint32_t *next) {
    return plamo_cuda_forward_greedy_margin(c, model, token, next, nullptr);
}

int plamo_cuda_forward_greedy_margin(struct plamo_cuda *c, struct model *model, uint64_t token, uint32_t *next,
                                     float *margin) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || token >= model->vocab) {
        c->info.declines++;
        return 0;
    }
    if (!reconcile(c, m)) return -1;
    if (!fits(c, m, 1)) {
        c->info.declines++;
        return 0;
    }
    if (!ensure_graph(c, m)) return -1;
    m->verify_valid = false;
    c->pinned_u32[0] = static_cast<uint32_t>(token);
    if (!note(c, "token", cudaMemcpyAsync(m->d_token, c->pinned_u32, 4, cudaMemcpyHostToDevice, c->stream)))
        return -1;
    cudaEventRecord(c->ev0, c->stream);
    if (!launch_decode(c, m)) return -1;
    cudaEventRecord(c->ev1, c->stream);
    if (!note(c, "next", cudaMemcpyAsync(c->pinned_u32 + 1, m->d_next, 12, cudaMemcpyDeviceToHost, c->stream)) ||
        !note(c, "forward", cudaStreamSynchronize(c->stream)))
        return -1;
    if (c->pinned_u32[2] && !check_device_error(c, m)) return -1;
    c->info.gpu_seconds += elapsed(c);
    c->info.forwards++;
    publish_counts(m, 1);
    if (next) *next = c->pinned_u32[1];
    memcpy(&m->last_margin, c->pinned_u32 + 3, 4);
    if (margin) *margin = m->last_margin;
    return 1;
}

static int prompt(struct plamo_cuda *c, struct model *model, const uint32_t *ids, uint64_t tokens, float *states,
                  uint32_t *next) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || !tokens || !ids) {
        c->info.declines++;
        return 0;
    }
    for (uint64_t i = 0; i < tokens; ++i)
        if (ids[i] >= model->vocab) {
            snprintf(c->info.note, sizeof c->info.note, "prompt token %u outside the vocabulary", ids[i]);
            c->info.errors++;
            return -1;
        }
    if (tokens > m->tmax) {
        c->info.declines++;
        return 0;
    }
    if (!reconcile(c, m)) return -1;
    if (!fits(c, m, tokens)) {
        c->info.declines++;
        return 0;
    }
    m->verify_valid = false;
    if (!note(c, "ids", cudaMemcpyAsync(m->p_ids, ids, tokens * 4, cudaMemcpyHostToDevice, c->stream))) return -1;
    cudaEventRecord(c->ev0, c->stream);
    if (!record_prompt(c, m, tokens, 0, false)) return -1;
    cudaEventRecord(c->ev1, c->stream);
    if (states && !note(c, "states", cudaMemcpyAsync(states, m->p_states, tokens * m->H * 4, cudaMemcpyDeviceToHost,
                                                     c->stream)))
        return -1;
    if (!copy_outputs(c, m) ||
        !note(c, "next", cudaMemcpyAsync(c->pinned_u32 + 4, m->d_next, 8, cudaMemcpyDeviceToHost, c->stream)) ||
        !note(c, "prefill", cudaStreamSynchronize(c->stream)))
        return -1;
    if (c->pinned_u32[5] && !check_device_error(c, m)) return -1;
    c->info.gpu_seconds += elapsed(c);
    c->info.prefills++;
    publish_counts(m, tokens);
    if (c->config.copy_kv_to_host && !sync_kv(c, m)) return -1;
    if (next) *next = c->pinned_u32[4];
    return 1;
}

int plamo_cuda_prefill(struct plamo_cuda *c, struct model *model, const uint32_t *ids, uint64_t tokens,
                       float *states) {
    return prompt(c, model, ids, tokens, states, nullptr);
}

int plamo_cuda_prefill_greedy(struct plamo_cuda *c, struct model *model, const uint32_t *ids, uint64_t tokens,
                              uint32_t *next) {
    return prompt(c, model, ids, tokens, nullptr, next);
}

int plamo_cuda_verify(struct plamo_cuda *c, struct model *model, const uint32_t *ids, uint64_t tokens,
                      uint32_t *next) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || !tokens || tokens > kVerifyMax || !ids || !next) {
        c->info.declines++;
        return 0;
    }
    for (uint64_t i = 0; i < tokens; ++i)
        if (ids[i] >= model->vocab) {
            c->info.declines++;
            return 0;
        }
    if (!reconcile(c, m)) return -1;
    if (!fits(c, m, tokens)) {
        c->info.declines++;
        return 0;
    }
    if (!note(c, "ids", cudaMemcpyAsync(m->p_ids, ids, tokens * 4, cudaMemcpyHostToDevice, c->stream))) return -1;
    cudaEventRecord(c->ev0, c->stream);
    if (!record_prompt(c, m, tokens, 1, true)) return -1;
    const bool tp = m->tp.active;
    if (!rows_argmax(c, m, m->p_logits, m->Vh, static_cast<uint32_t>(tokens), tp ? m->tp.lidx : m->p_next,
                     tp ? m->tp.lval : nullptr))
        return -1;
    if (tp && (!launch(c, tp_argmax_kernel, dim3(1), dim3(128), 0, static_cast<const float *>(m->tp.lval),
                       static_cast<const uint32_t *>(m->tp.lidx), static_cast<uint32_t>(tokens),
                       static_cast<uint32_t>(m->tp.voff), tp_arg(m), m->p_next, static_cast<uint32_t *>(nullptr)) ||
               !launch(c, tp_epoch_kernel, dim3(1), dim3(32), 0, m->tp.epoch)))
        return -1;
    cudaEventRecord(c->ev1, c->stream);
    if (!note(c, "verify next", cudaMemcpyAsync(c->pinned_u32 + 16, m->p_next, tokens * 4, cudaMemcpyDeviceToHost,
                                                c->stream)) ||
        !note(c, "verify", cudaStreamSynchronize(c->stream)))
        return -1;
    if (!check_device_error(c, m)) return -1;
    memcpy(next, c->pinned_u32 + 16, tokens * 4);
    c->info.gpu_seconds += elapsed(c);
    c->info.verification_batches++;
    c->info.verified_tokens += tokens;
    m->verify_count = tokens;
    m->verify_committed = 0;
    m->verify_valid = true;
    return 1;
}

int plamo_cuda_commit(struct plamo_cuda *c, struct model *model, uint64_t index) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || !m->verify_valid || index != m->verify_committed || index >= m->verify_count) {
        if (c) c->info.declines++;
        return 0;
    }
    if (!fits(c, m, 1)) return 0;
    for (uint64_t l = 0; l < m->L; ++l) {
        AttnLayer al = attn_layer(m, l);
        const float *row = m->v_kv + (l * kVerifyMax + index) * 2 * m->KVW;
        kv_commit_kernel<<<1, 256, 0, c->stream>>>(al, m->KVW, row, row + m->KVW);
        c->info.launches++;
    }
    advance_kernel<<<1, 32, 0, c->stream>>>(m->d_appended, m->L, 1);
    c->info.launches++;
    struct model *h = model;
    // State of candidate `index`: final-layer state row; normalized and
    // logits of the same row.
    if (!note(c, "commit", cudaGetLastError()) ||
        !note(c, "commit state", cudaMemcpyAsync(h->state, m->p_states + index * m->H, m->H * 4,
                                                 cudaMemcpyDeviceToHost, c->stream)) ||
        !note(c, "commit norm", cudaMemcpyAsync(h->normalized, m->p_norm + index * m->H, m->H * 4,
                                                cudaMemcpyDeviceToHost, c->stream)) ||
        !note(c, "commit logits", cudaMemcpyAsync(h->logits + m->tp.voff, m->p_logits + index * m->Vh, m->Vh * 4,
                                                  cudaMemcpyDeviceToHost, c->stream)) ||
        !note(c, "commit", cudaStreamSynchronize(c->stream)))
        return -1;
    publish_counts(m, 1);
    m->verify_committed++;
    c->info.committed_tokens++;
    if (c->config.copy_kv_to_host && !sync_kv(c, m)) return -1;
    return 1;
}

int plamo_cuda_sync_host(struct plamo_cuda *c, struct model *model) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m) return 0;
    if (!sync_kv(c, m)) return -1;
    return 1;
}

int plamo_cuda_read_outputs(struct plamo_cuda *c, struct model *model) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m) return 0;
    return copy_outputs(c, m) && note(c, "outputs", cudaStreamSynchronize(c->stream)) ? 1 : -1;
}

int plamo_cuda_read_weights(struct plamo_cuda *c, const void *key, void *dst, uint64_t bytes) {
    if (!c || !key || !dst) return 0;
    const Range *r = find_range(c, key, bytes);
    if (!r) return 0;
    const char *src = r->dev + (reinterpret_cast<uintptr_t>(key) - r->host);
    return note(c, "read weights", cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost)) ? 1 : 0;
}

// One decoder layer's decode step for plamo_cuda_layer: state[0] -> state[1],
// the layer's K/V row appended (positions and page tables are read on the
// device, so the sequence is recorded once per layer and replayed).
bool record_layer(plamo_cuda *c, DModel *m, uint64_t index) {
    DLayer &L = m->layers[index];
    bool ok = true;
    GemvParams p{};
    p.w = L.qkv_w;
    p.rows = m->QW;
    p.cols = m->H;
    p.state_in = m->state[0];
    p.norm2 = L.pre;
    p.off2 = 1.0f;
    p.y = m->qkv;
    ok = gemv<PRO_NORM, EPI_STORE>(c, p);
    ok = ok && launch_decode_attention(c, m, index);
    GemvParams o{};
    o.w = L.o_w;
    o.rows = m->H;
    o.cols = m->AW;
    o.x = m->attn;
    o.y = m->branch;
    ok = ok && gemv<PRO_X, EPI_STORE>(c, o);
    GemvParams g{};
    g.w = L.gu;
    g.rows = 2 * m->I;
    g.cols = m->H;
    g.state_in = m->state[0];
    g.branch = m->branch;
    g.norm1 = L.post;
    g.off1 = kPostMixerOffset;
    g.norm2 = L.mpre;
    g.off2 = 1.0f;
    g.state_out = m->state[1];
    g.y = m->mid;
    ok = ok && gemv<PRO_RESID_NORM, EPI_SWIGLU>(c, g);
    GemvParams d{};
    d.w = L.down;
    d.rows = m->H;
    d.cols = m->I;
    d.x = m->mid;
    d.y = m->branch;
    ok = ok && gemv<PRO_X, EPI_STORE>(c, d);
    ok = ok && launch(c, norm_rows_kernel<ROW_RESID>, dim3(1), dim3(512), 0, m->state[1],
                      static_cast<const float *>(m->branch), L.mpost, kPostMlpOffset,
                      static_cast<const uint16_t *>(nullptr), 0.0f, static_cast<float *>(nullptr), m->H, RowFuse{});
    ok = ok && launch(c, advance_kernel, dim3(1), dim3(32), 0, m->d_appended + index, uint64_t{1}, uint64_t{1});
    return ok;
}

int plamo_cuda_layer(struct plamo_cuda *c, struct model *model, uint64_t index, float *state) {
    if (!c || !state) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || index >= m->L || m->tp.size) {
        c->info.declines++;
        return 0;
    }
    if (!reconcile(c, m)) return -1;
    DLayer &L = m->layers[index];
    if (!L.sliding && (L.appended + 1 > L.capacity || L.appended + 1 > L.ring || !kv_map(c, m, L, L.appended + 1))) {
        c->info.declines++;
        return 0;
    }
    m->verify_valid = false;
    if (m->layer_exec.size() != m->L) {
        m->layer_exec.assign(m->L, nullptr);
        m->layer_nodes.assign(m->L, 0);
    }
    if (!m->layer_exec[index]) {  // record this layer's launches once
        if (!note(c, "capture", cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal))) return -1;
        const uint64_t before = c->info.launches;
        const bool rec = record_layer(c, m, index);
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(c->stream, &graph);
        m->layer_nodes[index] = c->info.launches - before;
        c->info.launches = before;
        const bool inst = rec && note(c, "capture end", e) &&
                          note(c, "instantiate", cudaGraphInstantiate(&m->layer_exec[index], graph, 0));
        if (graph) cudaGraphDestroy(graph);
        if (!inst) {
            m->layer_exec[index] = nullptr;
            return -1;
        }
    }
    bool ok = note(c, "layer state", cudaMemcpyAsync(m->state[0], state, m->H * 4, cudaMemcpyHostToDevice,
                                                     c->stream));
    cudaEventRecord(c->ev0, c->stream);
    ok = ok && note(c, "layer graph", cudaGraphLaunch(m->layer_exec[index], c->stream));
    c->info.graph_launches++;
    c->info.launches += m->layer_nodes[index];
    cudaEventRecord(c->ev1, c->stream);
    ok = ok && note(c, "layer out", cudaMemcpyAsync(state, m->state[1], m->H * 4, cudaMemcpyDeviceToHost,
                                                    c->stream)) &&
         note(c, "layer", cudaStreamSynchronize(c->stream));
    if (!ok) return -1;
    c->info.gpu_seconds += elapsed(c);
    L.appended += 1;
    struct cache *hc = L.host->mixer->cache;
    hc->count = layer_count(L);
    L.host->mixer->rotation->processed_count = hc->count;
    L.host->mixer->rotation->scale_bits = float_to_bits(L.scale);
    if (c->config.copy_kv_to_host && !sync_kv(c, m)) return -1;
    return 1;
}

int plamo_cuda_release_model(struct plamo_cuda *c, struct model *model) {
    if (!c) return 0;
    DModel *m = find_model(c, model);
    if (!m) return 0;
    cudaStreamSynchronize(c->stream);
    free_model(c, m);
    c->models.erase(model);
    return 1;
}

int plamo_cuda_release_weights(struct plamo_cuda *c, const void *src, uint64_t bytes) {
    if (!c) return 0;
    const uintptr_t lo = reinterpret_cast<uintptr_t>(src), hi = lo + bytes;
    cudaStreamSynchronize(c->stream);
    int released = 0;
    for (size_t i = 0; i < c->ranges.size();) {
        const Range &r = c->ranges[i];
        if (r.host >= lo && r.host + r.bytes <= hi) {
            cudaFree(r.dev);
            c->info.weight_bytes -= r.bytes;
            c->ranges.erase(c->ranges.begin() + static_cast<long>(i));
            ++released;
        } else {
            ++i;
        }
    }
    if (released) {  // prepared models may point into the freed ranges
        for (auto &kv : c->models) free_model(c, kv.second.get());
        c->models.clear();
    }
    return released;
}

int plamo_cuda_invalidate(struct plamo_cuda *c, struct model *model) {
    if (!c) return 0;
    DModel *m = find_model(c, model);
    if (!m) return 0;
    for (DLayer &L : m->layers) L.stale = true;
    return 1;
}

void plamo_cuda_reset_request(struct plamo_cuda *c, struct model *model) {
    for (uint64_t i = 0; i < model->count; ++i) {
        struct layer *l = model->layers[i];
        l->state = model->state;
        l->mixer->cache->count = 0;
        l->mixer->rotation->processed_count = 0;
        l->mixer->rotation->scale_bits = 0;
        l->mixer->gqa->tokens = 0;
    }
    if (c) {
        DModel *m = find_model(c, model);
        if (m) reconcile(c, m);
    }
}

}  // extern "C"

namespace {

// Device staging of the host-buffer entry points (linear, mlp): one
// allocation per context, grown to the largest request seen and kept until
// close, carved into 256-byte aligned pieces. The last 256 bytes hold the
// projections' error flag.
struct Staging {
    char *base;
    uint64_t used;
    template <typename T>
    T *take(uint64_t count) {
        T *p = reinterpret_cast<T *>(base + used);
        used += (std::max<uint64_t>(count, 1) * sizeof(T) + 255) & ~255ull;
        return p;
    }
};
bool staging(plamo_cuda *c, uint64_t bytes, Staging *out) {
    bytes += 256;
    if (bytes > c->staging_bytes) {
        if (!note(c, "staging", cudaStreamSynchronize(c->stream))) return false;
        cudaFree(c->staging);
        c->staging = nullptr;
        c->staging_bytes = 0;
        if (!note(c, "staging alloc", cudaMalloc(&c->staging, bytes))) return false;
        c->staging_bytes = bytes;
        if (!note(c, "staging flag", cudaMemsetAsync(c->staging + bytes - 256, 0, 4, c->stream))) return false;
    }
    *out = Staging{c->staging, 0};
    return true;
}
uint32_t *staging_error(plamo_cuda *c) {
    return reinterpret_cast<uint32_t *>(c->staging + c->staging_bytes - 256);
}
uint64_t pad256(uint64_t bytes) { return (std::max<uint64_t>(bytes, 1) + 255) & ~255ull; }

// Read back and clear the projections' error flag after a synchronised call.
bool staging_ok(plamo_cuda *c) {
    uint32_t err = 0;
    if (!note(c, "staging flag", cudaMemcpy(&err, staging_error(c), 4, cudaMemcpyDeviceToHost))) return false;
    if (!err) return true;
    cudaMemset(staging_error(c), 0, 4);
    c->info.errors++;
    snprintf(c->info.note, sizeof c->info.note, "a tensor-core projection stalled for 2 s");
    return false;
}

}  // namespace

extern "C" {

int plamo_cuda_linear(struct plamo_cuda *c, const struct plamo_matmul *mm) {
    if (!c || !mm) return 0;
    if (!mm->rows || !mm->tokens) return 1;
    cudaSetDevice(c->device);
    const uint16_t *w = resolve(c, mm->weights, mm->rows * mm->columns * 2, false);
    if (!w) {
        c->info.declines++;
        return 0;
    }
    const uint64_t T = mm->tokens, K = mm->columns, R = mm->rows;
    Staging st{};
    if (!staging(c, pad256(T * K * 4) + pad256(T * R * 4) + pad256(3 * T * K * 2), &st)) return -1;
    float *x = st.take<float>(T * K), *y = st.take<float>(T * R);
    uint16_t *split = st.take<uint16_t>(3 * T * K);
    bool ok = !K || note(c, "linear in", cudaMemcpy2DAsync(x, K * 4, mm->input, mm->input_stride * 4, K * 4, T,
                                                          cudaMemcpyHostToDevice, c->stream));
    if (ok && !K) ok = note(c, "linear zero", cudaMemsetAsync(y, 0, T * R * 4, c->stream));
    else if (ok) ok = projection_with(c, x, K, w, y, R, T, R, K, split, staging_error(c));
    ok = ok && note(c, "linear out", cudaMemcpy2DAsync(mm->output, mm->output_stride * 4, y, R * 4, R * 4, T,
                                                       cudaMemcpyDeviceToHost, c->stream)) &&
         note(c, "linear", cudaStreamSynchronize(c->stream)) && staging_ok(c);
    return ok ? 1 : -1;
}

int plamo_cuda_linear_static(struct plamo_cuda *c, const struct plamo_matmul *mm) {
    if (!c || !mm) return 0;
    if (!mm->rows || !mm->tokens) return 1;
    cudaSetDevice(c->device);
    const uint64_t T = mm->tokens, K = mm->columns, R = mm->rows;
    // Each product is bounded before the sum is formed (T >= 1 here), so no
    // intermediate can wrap: K, R <= limit / T keeps T*K and T*R <= limit.
    if (K > kStaticLinearFloats / T || R > kStaticLinearFloats / T || T * K > kStaticLinearFloats - T * R) {
        c->info.declines++;
        snprintf(c->info.note, sizeof c->info.note,
                 "linear_static: %llu tokens x (%llu input + %llu output) floats exceed the static staging of %llu "
                 "floats",
                 static_cast<unsigned long long>(T), static_cast<unsigned long long>(K),
                 static_cast<unsigned long long>(R), static_cast<unsigned long long>(kStaticLinearFloats));
        return 0;
    }
    const uint16_t *w = resolve(c, mm->weights, R * K * 2, false);
    if (!w) {
        c->info.declines++;
        snprintf(c->info.note, sizeof c->info.note, "linear_static: weights are not preloaded");
        return 0;
    }
    // One-time set-up on this context's device (the first call, with the
    // device current): the device address of the static array.
    if (!c->static_scratch &&
        !note(c, "linear_static symbol",
              cudaGetSymbolAddress(reinterpret_cast<void **>(&c->static_scratch), g_linear_static_scratch)))
        return -1;
    float *x = c->static_scratch, *y = c->static_scratch + T * K;
    bool ok = !K || note(c, "linear_static in", cudaMemcpy2DAsync(x, K * 4, mm->input, mm->input_stride * 4, K * 4,
                                                                 T, cudaMemcpyHostToDevice, c->stream));
    if (ok && !K) ok = note(c, "linear_static zero", cudaMemsetAsync(y, 0, T * R * 4, c->stream));
    else if (ok) ok = gemm(c, x, K, w, y, R, T, R, K);
    ok = ok && note(c, "linear_static out", cudaMemcpy2DAsync(mm->output, mm->output_stride * 4, y, R * 4, R * 4, T,
                                                              cudaMemcpyDeviceToHost, c->stream)) &&
         note(c, "linear_static", cudaStreamSynchronize(c->stream));
    return ok ? 1 : -1;
}

int plamo_cuda_mlp(struct plamo_cuda *c, const struct mlp *p, float *states, uint64_t tokens) {
    if (!c || !p || !states) return 0;
    if (!tokens) return 1;
    cudaSetDevice(c->device);
    const uint64_t H = p->hidden, I = p->intermediate;
    const uint16_t *pre = resolve(c, p->pre, H * 2, false), *post = resolve(c, p->post, H * 2, false);
    const uint16_t *gu = resolve(c, p->gu, 2 * I * H * 2, false), *down = resolve(c, p->down, H * I * 2, false);
    if (!pre || !post || !gu || !down) {
        c->info.declines++;
        return 0;
    }
    const uint64_t T = tokens, KM = std::max<uint64_t>(H, I);
    Staging st{};
    if (!staging(c, 3 * pad256(T * H * 4) + pad256(T * 2 * I * 4) + pad256(3 * T * KM * 2), &st)) return -1;
    float *s = st.take<float>(T * H), *n = st.take<float>(T * H), *g = st.take<float>(T * 2 * I),
          *b = st.take<float>(T * H);
    uint16_t *split = st.take<uint16_t>(3 * T * KM);
    uint32_t *err = staging_error(c);
    bool ok = note(c, "mlp in", cudaMemcpyAsync(s, states, T * H * 4, cudaMemcpyHostToDevice, c->stream));
    ok = ok && launch(c, norm_rows_kernel<ROW_NORM>, dim3(T), dim3(512), 0, s, static_cast<const float *>(nullptr),
                      static_cast<const uint16_t *>(nullptr), 0.0f, pre, 1.0f, n, H, RowFuse{});
    ok = ok && projection_with(c, n, H, gu, g, 2 * I, T, 2 * I, H, split, err);
    ok = ok && swiglu_rows(c, g, I, T, RowFuse{});
    ok = ok && projection_with(c, g, 2 * I, down, b, H, T, H, I, split, err);
    ok = ok && launch(c, norm_rows_kernel<ROW_RESID>, dim3(T), dim3(512), 0, s, static_cast<const float *>(b), post,
                      kPostMlpOffset, static_cast<const uint16_t *>(nullptr), 0.0f, static_cast<float *>(nullptr), H,
                      RowFuse{});
    ok = ok && note(c, "mlp out", cudaMemcpyAsync(states, s, T * H * 4, cudaMemcpyDeviceToHost, c->stream)) &&
         note(c, "mlp", cudaStreamSynchronize(c->stream)) && staging_ok(c);
    return ok ? 1 : -1;
}

int64_t plamo_cuda_generate(struct plamo_cuda *c, struct model *model, const uint32_t *ids, uint64_t tokens,
                            uint64_t max_tokens, uint32_t *out, int (*on_token)(uint32_t, void *), void *context,
                            struct plamo_cuda_timing *timing) {
    plamo_cuda_timing local{};
    plamo_cuda_timing *t = timing ? timing : &local;
    memset(t, 0, sizeof *t);
    if (!c || !model || !out || !max_tokens || max_tokens > 4096 || !tokens || tokens > 4096) return -1;
    DModel *m = find_model(c, model);
    if (!m) return -1;
    t->prompt_tokens = tokens;
    auto now = [] {
        return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
    };
    const double start = now();
    uint32_t id = 0;
    plamo_cuda_reset_request(c, model);  // a request starts from empty caches (reference runtime/engine.c:451)
    if (plamo_cuda_prefill_greedy(c, model, ids, tokens, &id) != 1) return -1;
    t->prefill_seconds = now() - start;
    t->finish_reason = "length";
    const double decode_start = now();
    int64_t emitted = 0;
    for (;;) {
        // Emit the selected token (reference runtime/engine.c:395-420).
        if (id == 1 || id == 16) {
            t->finish_reason = "stop";
            break;
        }
        if (id >= model->vocab) {
            t->finish_reason = "error";
            return -1;
        }
        if (on_token && !on_token(id, context)) {
            t->finish_reason = "cancelled";
            break;
        }
        out[emitted++] = id;
        if (emitted == 1) t->first_token_seconds = now() - start;
        if (static_cast<uint64_t>(emitted) == max_tokens) break;
        uint32_t next = 0;
        if (plamo_cuda_forward_greedy(c, model, id, &next) != 1) return -1;
        t->decode_steps++;
        id = next;
    }
    t->decode_seconds = now() - decode_start;
    t->completion_tokens = static_cast<uint64_t>(emitted);
    return emitted;
}

int plamo_cuda_gemm_device(struct plamo_cuda *c, const float *x, uint64_t xs, const uint16_t *w, float *y,
                           uint64_t ys, uint64_t tokens, uint64_t rows, uint64_t cols) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    uint16_t *split = nullptr;
    float *part = nullptr;
    const uint64_t n = std::max<uint64_t>(tokens * cols, 1);
    if (!note(c, "gemm scratch", cudaMalloc(&split, 3 * n * 2)) ||
        !note(c, "gemm scratch", cudaMalloc(&part, kSplitkFloats * 4))) {
        cudaFree(split);
        return -1;
    }
    const bool ok = projection_with(c, x, xs, w, y, ys, tokens, rows, cols, split, nullptr, part, kSplitkFloats) &&
                    note(c, "gemm", cudaStreamSynchronize(c->stream));
    cudaFree(split);
    cudaFree(part);
    return ok ? 1 : -1;
}

double plamo_cuda_time_gemm(struct plamo_cuda *c, const float *x, const uint16_t *w, float *y, uint64_t tokens,
                            uint64_t rows, uint64_t cols, uint64_t repeats) {
    if (!c || !repeats) return -1;
    cudaSetDevice(c->device);
    uint16_t *split = nullptr;
    float *part = nullptr;
    const uint64_t n = std::max<uint64_t>(tokens * cols, 1);
    if (!note(c, "gemm scratch", cudaMalloc(&split, 3 * n * 2)) ||
        !note(c, "gemm scratch", cudaMalloc(&part, kSplitkFloats * 4))) {
        cudaFree(split);
        return -1;
    }
    cudaStreamSynchronize(c->stream);
    cudaEventRecord(c->ev0, c->stream);
    bool ok = true;
    for (uint64_t i = 0; i < repeats && ok; ++i)
        ok = projection_with(c, x, cols, w, y, rows, tokens, rows, cols, split, nullptr, part, kSplitkFloats);
    cudaEventRecord(c->ev1, c->stream);
    ok = ok && note(c, "time gemm", cudaStreamSynchronize(c->stream));
    float ms = 0;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    cudaFree(split);
    cudaFree(part);
    return ok ? ms : -1;
}

struct plamo_cuda_batch *plamo_cuda_batch_open(struct plamo_cuda *c, struct model *const *models, unsigned count) {
    if (!c || !models || !count || count > kVerifyMax) return nullptr;
    cudaSetDevice(c->device);
    std::vector<DModel *> ms;
    for (unsigned i = 0; i < count; ++i) {
        DModel *m = models[i] ? find_model(c, models[i]) : nullptr;
        if (!m || m->tp.size || m->D != 128 || m->QH / m->KH > 32 || m->tmax < count) return nullptr;
        for (DModel *o : ms)
            if (o == m) return nullptr;  // one cache per request
        ms.push_back(m);
    }
    const DModel *m0 = ms[0];
    for (const DModel *m : ms) {
        if (m->H != m0->H || m->QH != m0->QH || m->KH != m0->KH || m->I != m0->I || m->V != m0->V ||
            m->L != m0->L || m->emb != m0->emb || m->head != m0->head || m->norm != m0->norm)
            return nullptr;
        for (uint64_t l = 0; l < m->L; ++l) {
            const DLayer &a = m->layers[l], &z = m0->layers[l];
            if (a.qkv_w != z.qkv_w || a.o_w != z.o_w || a.gu != z.gu || a.down != z.down || a.pre != z.pre ||
                a.post != z.post || a.mpre != z.mpre || a.mpost != z.mpost || a.qn != z.qn || a.kn != z.kn ||
                a.scale != z.scale || a.sliding != z.sliding)
                return nullptr;
        }
    }
    auto b = std::make_unique<plamo_cuda_batch>();
    b->c = c;
    b->B = count;
    b->graph = nullptr;
    b->exec = nullptr;
    b->nodes = 0;
    for (unsigned i = 0; i < count; ++i) b->hosts.push_back(models[i]);
    std::vector<DecodeAttnParams> params;
    for (uint64_t l = 0; l < m0->L; ++l)
        for (unsigned i = 0; i < count; ++i)
            params.push_back(DecodeAttnParams{attn_layer(ms[i], l), static_cast<uint32_t>(m0->QH),
                                              static_cast<uint32_t>(m0->KH), static_cast<uint32_t>(m0->D),
                                              m0->p_qkv + i * m0->QW, m0->p_attn + i * m0->AW});
    std::vector<uint64_t *> counters;
    for (DModel *m : ms) counters.push_back(m->d_appended);
    b->d_attn = nullptr;
    b->d_counters = nullptr;
    b->d_tokens = nullptr;
    bool ok = note(c, "batch alloc", cudaMalloc(&b->d_attn, params.size() * sizeof(DecodeAttnParams))) &&
              note(c, "batch alloc", cudaMalloc(&b->d_counters, count * sizeof(uint64_t *))) &&
              note(c, "batch alloc", cudaMalloc(&b->d_tokens, 64 * 4)) &&
              note(c, "batch params", cudaMemcpy(b->d_attn, params.data(), params.size() * sizeof(DecodeAttnParams),
                                                 cudaMemcpyHostToDevice)) &&
              note(c, "batch params", cudaMemcpy(b->d_counters, counters.data(), count * sizeof(uint64_t *),
                                                 cudaMemcpyHostToDevice));
    if (ok) {
        ok = note(c, "capture", cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
        if (ok) {
            const uint64_t before = c->info.launches;
            const bool rec = record_batch(c, b.get(), ms[0]);
            const cudaError_t e = cudaStreamEndCapture(c->stream, &b->graph);
            b->nodes = c->info.launches - before;
            c->info.launches = before;
            ok = rec && note(c, "capture end", e) &&
                 note(c, "instantiate", cudaGraphInstantiate(&b->exec, b->graph, 0));
        }
    }
    if (!ok) {
        plamo_cuda_batch_close(b.release());
        return nullptr;
    }
    return b.release();
}

// Preflight of `steps` batch steps: every request prepared, reconciled with
// its host counts and able to take the rows.
static bool batch_ready(plamo_cuda_batch *b, uint64_t steps, std::vector<DModel *> &ms) {
    plamo_cuda *c = b->c;
    for (struct model *h : b->hosts) {
        DModel *m = find_model(c, h);
        if (!m || !reconcile(c, m) || !fits(c, m, steps)) return false;
        m->verify_valid = false;
        ms.push_back(m);
    }
    return true;
}

int plamo_cuda_batch_step(struct plamo_cuda_batch *b, const uint32_t *tokens, uint32_t *next) {
    if (!b || !tokens || !next) return 0;
    plamo_cuda *c = b->c;
    cudaSetDevice(c->device);
    std::vector<DModel *> ms;
    for (uint32_t i = 0; i < b->B; ++i)
        if (tokens[i] >= b->hosts[0]->vocab) {
            c->info.declines++;
            return 0;
        }
    if (!batch_ready(b, 1, ms)) {
        c->info.declines++;
        return 0;
    }
    memcpy(c->pinned_u32 + 32, tokens, b->B * 4);
    cudaEventRecord(c->ev0, c->stream);
    bool ok = note(c, "batch tokens", cudaMemcpyAsync(b->d_tokens, c->pinned_u32 + 32, b->B * 4,
                                                      cudaMemcpyHostToDevice, c->stream)) &&
              note(c, "batch graph", cudaGraphLaunch(b->exec, c->stream));
    cudaEventRecord(c->ev1, c->stream);
    ok = ok && note(c, "batch next", cudaMemcpyAsync(c->pinned_u32 + 32, b->d_tokens, b->B * 4,
                                                     cudaMemcpyDeviceToHost, c->stream)) &&
         note(c, "batch step", cudaStreamSynchronize(c->stream));
    if (!ok || !check_device_error(c, ms[0])) return -1;
    c->info.graph_launches++;
    c->info.launches += b->nodes;
    c->info.forwards += b->B;
    c->info.gpu_seconds += elapsed(c);
    memcpy(next, c->pinned_u32 + 32, b->B * 4);
    for (DModel *m : ms) {
        publish_counts(m, 1);
        if (c->config.copy_kv_to_host && !sync_kv(c, m)) return -1;
    }
    return 1;
}

double plamo_cuda_time_batch(struct plamo_cuda_batch *b, uint64_t steps) {
    if (!b || !steps) return -1;
    plamo_cuda *c = b->c;
    cudaSetDevice(c->device);
    std::vector<DModel *> ms;
    if (!batch_ready(b, steps, ms)) return -1;
    cudaStreamSynchronize(c->stream);
    cudaEventRecord(c->ev0, c->stream);
    bool ok = true;
    for (uint64_t i = 0; i < steps && ok; ++i) ok = note(c, "batch graph", cudaGraphLaunch(b->exec, c->stream));
    cudaEventRecord(c->ev1, c->stream);
    ok = ok && note(c, "time batch", cudaStreamSynchronize(c->stream));
    if (!ok || !check_device_error(c, ms[0])) return -1;
    c->info.graph_launches += steps;
    c->info.launches += b->nodes * steps;
    for (DModel *m : ms) publish_counts(m, steps);
    float ms_total = 0;
    cudaEventElapsedTime(&ms_total, c->ev0, c->ev1);
    return ms_total;
}

void plamo_cuda_batch_close(struct plamo_cuda_batch *b) {
    if (!b) return;
    cudaSetDevice(b->c->device);
    cudaStreamSynchronize(b->c->stream);
    if (b->exec) cudaGraphExecDestroy(b->exec);
    if (b->graph) cudaGraphDestroy(b->graph);
    cudaFree(b->d_attn);
    cudaFree(b->d_counters);
    cudaFree(b->d_tokens);
    delete b;
}

int plamo_cuda_rollback(struct plamo_cuda *c, struct model *model, uint64_t rows) {
    if (!c) return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || !reconcile(c, m)) return 0;
    for (const DLayer &L : m->layers) {
        // Rows evicted from a sliding window while they were appended must
        // still be in the ring's spare slots.
        if (rows > L.appended || rows > kVerifyMax + 1) {
            c->info.declines++;
            return 0;
        }
    }
    if (!rows) return 1;
    m->verify_valid = false;
    rollback_kernel<<<1, 32, 0, c->stream>>>(m->d_appended, m->L, rows);
    c->info.launches++;
    if (!note(c, "rollback", cudaGetLastError()) || !note(c, "rollback", cudaStreamSynchronize(c->stream)))
        return -1;
    for (uint64_t l = 0; l < m->L; ++l) {
        DLayer &L = m->layers[l];
        L.appended -= rows;
        struct cache *hc = L.host->mixer->cache;
        hc->count = layer_count(L);
        L.host->mixer->rotation->processed_count = hc->count;
    }
    if (c->config.copy_kv_to_host && !sync_kv(c, m)) return -1;
    return 1;
}

// Capture (reference runtime/prompt_cache.c:15-51). The acceptance test is the
// reference's, including its snapshot bound: a 16 MiB budget that starts with
// the reference record's own size and charges 12 bytes per cached element
// (K, V and rotated K), so the same models and prefixes are admitted.
struct plamo_cuda_prompt_cache *plamo_cuda_prompt_cache_capture(struct plamo_cuda *c, const struct model *model,
                                                                const uint32_t *ids, uint64_t tokens) {
    constexpr uint64_t kLimit = uint64_t{16} << 20;
    constexpr uint64_t kReferenceRecord = 8 + 3 * 8 + PLAMO_CUDA_PREFIX_LIMIT * 4 + 128 * 16;
    if (!c || !model || !ids || !tokens || tokens > PLAMO_CUDA_PREFIX_LIMIT || !model->count || model->count > 128)
        return nullptr;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, const_cast<struct model *>(model));
    if (!m || !reconcile(c, m)) return nullptr;
    uint64_t budget = kReferenceRecord;
    for (uint64_t l = 0; l < model->count; ++l) {
        const struct mixer *mx = model->layers[l]->mixer;
        const struct cache *hc = mx->cache;
        const DLayer &L = m->layers[l];
        if (!hc->width || hc->count != tokens || hc->capacity < tokens || mx->rotation->cache != hc ||
            mx->rotation->processed_count != tokens || !hc->k || !hc->v || !mx->rotation->out ||
            hc->width > (kLimit - budget) / (tokens * 12))
            return nullptr;
        budget += hc->width * tokens * 12;
        // The device rows must be logical rows 0..tokens-1 in slots 0..tokens-1.
        if (hc->width != m->KVW || L.appended != tokens || L.ring < tokens) return nullptr;
    }
    auto s = std::make_unique<plamo_cuda_prompt_cache>();
    s->model = model;
    s->owner = c;
    s->device = c->device;
    s->tokens = tokens;
    s->layers = model->count;
    s->kvw = m->KVW;
    s->bytes = model->count * 2 * tokens * m->KVW * 4;
    memcpy(s->ids, ids, tokens * 4);
    if (!note(c, "prompt cache alloc", cudaMalloc(&s->rows, s->bytes))) return nullptr;
    const uint64_t words = tokens * m->KVW;
    bool ok = true;
    for (uint64_t l = 0; l < model->count && ok; ++l) {
        const DLayer &L = m->layers[l];
        s->width.push_back(model->layers[l]->mixer->cache->width);
        s->scale_bits.push_back(model->layers[l]->mixer->rotation->scale_bits);
        ok = kv_copy_rows(c, m, L, tokens, s->rows + (2 * l) * words, s->rows + (2 * l + 1) * words, false,
                          cudaMemcpyDeviceToDevice);
    }
    ok = ok && note(c, "prompt cache capture", cudaStreamSynchronize(c->stream));
    if (!ok) {
        cudaFree(s->rows);
        return nullptr;
    }
    return s.release();
}

// Restore (reference runtime/prompt_cache.c:53-81): every destination is
// checked before any is written, so a miss changes nothing.
uint64_t plamo_cuda_prompt_cache_restore(struct plamo_cuda *c, const struct plamo_cuda_prompt_cache *s,
                                         struct model *model, const uint32_t *ids, uint64_t tokens) {
    if (!c || !s || s->model != model || !ids || tokens <= s->tokens || model->count != s->layers ||
        memcmp(ids, s->ids, s->tokens * 4))
        return 0;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (s->owner != c || !m || m->KVW != s->kvw) return 0;
    for (uint64_t l = 0; l < model->count; ++l) {
        const struct mixer *mx = model->layers[l]->mixer;
        const struct cache *hc = mx->cache;
        const DLayer &L = m->layers[l];
        if (hc->width != s->width[l] || hc->capacity < s->tokens || mx->rotation->cache != hc || !hc->k || !hc->v ||
            !mx->rotation->out || L.capacity < s->tokens || L.ring < s->tokens)
            return 0;
    }
    // Pages for the snapshot's rows, before anything is written.
    for (uint64_t l = 0; l < model->count; ++l)
        if (!kv_map(c, m, m->layers[l], s->tokens)) return 0;
    m->verify_valid = false;  // a pending verification's rows are gone
    const uint64_t words = s->tokens * s->kvw;
    bool ok = true;
    for (uint64_t l = 0; l < model->count && ok; ++l) {
        DLayer &L = m->layers[l];
        ok = kv_copy_rows(c, m, L, s->tokens, s->rows + (2 * l) * words, s->rows + (2 * l + 1) * words, true,
                          cudaMemcpyDeviceToDevice);
        L.appended = s->tokens;
        L.stale = false;
        struct mixer *mx = model->layers[l]->mixer;
        mx->cache->count = mx->rotation->processed_count = s->tokens;
        mx->rotation->scale_bits = s->scale_bits[l];
    }
    std::vector<uint64_t> counts(m->L, s->tokens);
    ok = ok && note(c, "counter upload", cudaMemcpyAsync(m->d_appended, counts.data(), m->L * 8,
                                                         cudaMemcpyHostToDevice, c->stream)) &&
         note(c, "prompt cache restore", cudaStreamSynchronize(c->stream));
    if (ok && c->config.copy_kv_to_host) ok = sync_kv(c, m);
    if (!ok) {
        // A failed copy leaves the rows unknown: drop the request state.
        plamo_cuda_reset_request(c, model);
        return 0;
    }
    return s->tokens;
}

uint64_t plamo_cuda_prompt_cache_tokens(const struct plamo_cuda_prompt_cache *s) { return s ? s->tokens : 0; }
uint64_t plamo_cuda_prompt_cache_bytes(const struct plamo_cuda_prompt_cache *s) { return s ? s->bytes : 0; }

void plamo_cuda_prompt_cache_free(struct plamo_cuda_prompt_cache *s) {
    if (!s) return;
    cudaSetDevice(s->device);
    cudaFree(s->rows);
    delete s;
}

// Speculative request loop (reference runtime/engine.c:523-586 with the draft
// proposer of runtime/worker.c:198-318 and its horizon rule, runtime/draft.c:
// 196-212): the draft model proposes greedily from the known token, the
// target verifies the block in one pass, the longest agreeing prefix is
// committed and the draft rolls back the rest. Emits exactly the target's
// greedy tokens.
int64_t plamo_cuda_generate_speculative(struct plamo_cuda *c, struct model *target, struct model *draft,
                                        const uint32_t *ids, uint64_t tokens, uint64_t max_tokens, unsigned block,
                                        uint32_t *out, int (*on_token)(uint32_t, void *), void *context,
                                        struct plamo_cuda_speculation *stats) {
    plamo_cuda_speculation local{};
    plamo_cuda_speculation *st = stats ? stats : &local;
    memset(st, 0, sizeof *st);
    if (!c || !target || !draft || !out || !max_tokens || max_tokens > 4096 || !tokens || tokens > 4096 || !block ||
        block > kVerifyMax || !find_model(c, target) || !find_model(c, draft))
        return -1;
    auto now = [] {
        return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
    };
    const double start = now();
    uint32_t id = 0, ignored = 0;
    // A request starts from empty caches (reference runtime/engine.c:451).
    plamo_cuda_reset_request(c, target);
    plamo_cuda_reset_request(c, draft);
    if (plamo_cuda_prefill_greedy(c, target, ids, tokens, &id) != 1) return -1;
    bool speculate = block > 1 && plamo_cuda_prefill_greedy(c, draft, ids, tokens, &ignored) == 1;
    st->prefill_seconds = now() - start;
    const double decode_start = now();
    unsigned horizon = 8;
    int64_t emitted = 0;
    st->finish_reason = "length";
    // reference runtime/engine.c:395-420: a stop id or a cancelling callback
    // ends the request before the token is committed (0); the token that
    // reaches max_tokens is counted and committed, then the request ends (2).
    auto emit = [&](uint32_t t) -> int {
        if (t == 1 || t == 16) {
            st->finish_reason = "stop";
            return 0;
        }
        if (t >= target->vocab) return -1;
        if (on_token && !on_token(t, context)) {
            st->finish_reason = "cancelled";
            return 0;
        }
        out[emitted++] = t;
        return static_cast<uint64_t>(emitted) == max_tokens ? 2 : 1;
    };
    int r = emit(id);
    while (r == 1) {
        if (speculate) {
            unsigned limit = static_cast<unsigned>(max_tokens - static_cast<uint64_t>(emitted));
            if (limit > block) limit = block;
            if (limit > horizon) limit = horizon;
            uint32_t proposed[kVerifyMax], next[kVerifyMax];
            proposed[0] = id;
            unsigned n = 1, processed = 0;
            bool failed = false;
            // Confidence rule of reference runtime/worker.c:243-286: blocks of
            // more than 8 stop once 8 are proposed and the smallest top-2
            // logit margin so far is below 1 (PLAMO_DRAFT_MIN_MARGIN /
            // PLAMO_DRAFT_MIN_TOKENS override, as there).
            const float need = c->draft_margin >= 0.0f ? c->draft_margin : (limit > 8 ? 1.0f : 0.0f);
            const unsigned minimum = c->draft_min_tokens ? c->draft_min_tokens : (limit > 8 ? 8u : 2u);
            float confidence = INFINITY;
            while (n < limit && proposed[n - 1] != 1 && proposed[n - 1] != 16) {
                if (need > 0.0f && n >= minimum && confidence < need) break;
                uint32_t t = 0;
                float margin = 0.0f;
                if (plamo_cuda_forward_greedy_margin(c, draft, proposed[n - 1], &t, &margin) != 1 ||
                    t >= draft->vocab) {
                    failed = true;
                    break;
                }
                ++processed;
                if (margin < confidence) confidence = margin;
                if (need > 0.0f && n >= minimum && confidence < need) break;
                proposed[n++] = t;
            }
            if (failed || plamo_cuda_verify(c, target, proposed, n, next) != 1) {
                speculate = false;  // the target state is untouched: continue exactly
            } else {
                ++st->verify_batches;
                st->proposed_tokens += n - 1;
                unsigned consumed = 0;
                for (unsigned j = 0; j < n; ++j) {
                    if (j) {
                        if (proposed[j] != next[j - 1]) break;
                        r = emit(proposed[j]);
                        if (r < 0) return -1;
                        if (r == 0) break;
                    }
                    if (plamo_cuda_commit(c, target, j) != 1) return -1;
                    ++consumed;
                    ++st->decode_steps;
                    if (r == 2) break;
                }
                st->accepted_tokens += consumed - 1;
                // Draft: keep exactly the consumed prefix.
                int ok = 1;
                if (consumed < processed) ok = plamo_cuda_rollback(c, draft, processed - consumed);
                else if (consumed == processed + 1) {
                    uint32_t t = 0;
                    ok = plamo_cuda_forward_greedy(c, draft, proposed[processed], &t);
                }
                if (ok != 1) speculate = false;
                if (consumed == 1 && n > 1) horizon = 2;
                else if (consumed < n || n < limit) horizon = 8;
                else if (horizon < 8) horizon *= 2;
                else horizon = kVerifyMax;
                if (r != 1) break;
                id = next[consumed - 1];
                r = emit(id);
                continue;
            }
        }
        uint32_t t = 0;
        if (plamo_cuda_forward_greedy(c, target, id, &t) != 1) return -1;
        ++st->decode_steps;
        id = t;
        r = emit(id);
    }
    if (r < 0) return -1;
    st->decode_seconds = now() - decode_start;
    st->completion_tokens = static_cast<uint64_t>(emitted);
    return emitted;
}

int plamo_cuda_gemv_device(struct plamo_cuda *c, const uint16_t *w, const float *x, float *y, uint64_t rows,
                           uint64_t cols) {
    if (!c) return 0;
    GemvParams p{};
    p.w = w;
    p.rows = rows;
    p.cols = cols;
    p.x = x;
    p.y = y;
    return gemv<PRO_X, EPI_STORE>(c, p) ? 1 : -1;
}

double plamo_cuda_time_gemv(struct plamo_cuda *c, const uint16_t *w, const float *x, float *y, uint64_t rows,
                            uint64_t cols, uint64_t repeats) {
    if (!c || !repeats) return -1;
    cudaStreamSynchronize(c->stream);
    cudaEventRecord(c->ev0, c->stream);
    for (uint64_t i = 0; i < repeats; ++i)
        if (plamo_cuda_gemv_device(c, w, x, y, rows, cols) != 1) return -1;
    cudaEventRecord(c->ev1, c->stream);
    if (!note(c, "time gemv", cudaStreamSynchronize(c->stream))) return -1;
    float ms = 0;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    return ms;
}

double plamo_cuda_time_gemv_copies(struct plamo_cuda *c, const uint16_t *w, uint64_t copies, const float *x, float *y,
                                   uint64_t rows, uint64_t cols, uint64_t repeats) {
    if (!c || !repeats || !copies) return -1;
    cudaStreamSynchronize(c->stream);
    cudaEventRecord(c->ev0, c->stream);
    for (uint64_t i = 0; i < repeats; ++i)
        if (plamo_cuda_gemv_device(c, w + (i % copies) * rows * cols, x, y, rows, cols) != 1) return -1;
    cudaEventRecord(c->ev1, c->stream);
    if (!note(c, "time gemv", cudaStreamSynchronize(c->stream))) return -1;
    float ms = 0;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    return ms;
}

double plamo_cuda_time_decode(struct plamo_cuda *c, struct model *model, uint64_t repeats) {
    if (!c || !repeats) return -1;
    DModel *m = find_model(c, model);
    if (!m || !reconcile(c, m) || !fits(c, m, repeats) || !ensure_graph(c, m)) return -1;
    m->verify_valid = false;
    cudaStreamSynchronize(c->stream);
    cudaEventRecord(c->ev0, c->stream);
    for (uint64_t i = 0; i < repeats; ++i)
        if (!launch_decode(c, m)) return -1;
    cudaEventRecord(c->ev1, c->stream);
    if (!note(c, "time decode", cudaStreamSynchronize(c->stream))) return -1;
    if (!check_device_error(c, m)) return -1;
    publish_counts(m, repeats);
    float ms = 0;
    cudaEventElapsedTime(&ms, c->ev0, c->ev1);
    return ms;
}

uint64_t plamo_cuda_kernel_launches(const struct plamo_cuda *c) {
    return c ? c->info.launches : 0;
}

// One decode step of the graph path with every projection and attention
// launch stamping its timeline record: a graph of the traced step is
// captured, launched once and released.
double graph_trace(plamo_cuda *c, DModel *m, uint64_t token, uint64_t *stamps, uint64_t capacity) {
    const uint64_t n = kTraceWords * (5 * m->L + 1);
    if (capacity < n) return -1;
    auto *trace = static_cast<unsigned long long *>(plamo_cuda_device_alloc(c, n * 8));
    if (!trace) return -1;
    m->trace = trace;
    m->trace_slot = 0;
    const uint64_t before = c->info.launches;
    cudaGraph_t graph = nullptr;
    cudaGraphExec_t exec = nullptr;
    bool ok = note(c, "capture", cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    if (ok) {
        const bool recorded = record_decode(c, m);
        ok = note(c, "capture end", cudaStreamEndCapture(c->stream, &graph)) && recorded;
    }
    m->trace = nullptr;
    c->info.launches = before;
    ok = ok && note(c, "instantiate", cudaGraphInstantiate(&exec, graph, 0));
    m->verify_valid = false;
    c->pinned_u32[0] = static_cast<uint32_t>(token);
    ok = ok && note(c, "trace", cudaMemsetAsync(trace, 0, n * 8, c->stream)) &&
         note(c, "token", cudaMemcpyAsync(m->d_token, c->pinned_u32, 4, cudaMemcpyHostToDevice, c->stream)) &&
         note(c, "graph launch", cudaGraphLaunch(exec, c->stream)) &&
         note(c, "trace", cudaMemcpyAsync(stamps, trace, n * 8, cudaMemcpyDeviceToHost, c->stream)) &&
         note(c, "trace", cudaStreamSynchronize(c->stream));
    if (exec) cudaGraphExecDestroy(exec);
    if (graph) cudaGraphDestroy(graph);
    cudaFree(trace);
    if (!ok || !check_device_error(c, m)) return -1;
    for (uint64_t i = 0; i < n; i += kTraceWords) {  // minima were kept complemented
        stamps[i] = ~0ull - stamps[i];
        stamps[i + 2] = ~0ull - stamps[i + 2];
    }
    publish_counts(m, 1);
    return static_cast<double>(n);
}

double plamo_cuda_decode_trace(struct plamo_cuda *c, struct model *model, uint64_t token, uint64_t *stamps,
                               uint64_t capacity) {
    if (!c || !stamps) return -1;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || token >= model->vocab || !reconcile(c, m) || !fits(c, m, 1) || !ensure_graph(c, m)) return -1;
    if (!m->pt_ready) return graph_trace(c, m, token, stamps, capacity);
    const uint64_t n = 1 + (5 * m->L + 1) + (4 * m->L + 1);
    if (capacity < n) return -1;
    auto *trace = static_cast<unsigned long long *>(plamo_cuda_device_alloc(c, n * 8));
    if (!trace) return -1;
    m->verify_valid = false;
    c->pinned_u32[0] = static_cast<uint32_t>(token);
    m->pt.trace = trace;
    bool ok = note(c, "trace", cudaMemsetAsync(trace, 0, n * 8, c->stream)) &&
              note(c, "token", cudaMemcpyAsync(m->d_token, c->pinned_u32, 4, cudaMemcpyHostToDevice, c->stream)) &&
              launch_decode(c, m) &&
              note(c, "trace", cudaMemcpyAsync(stamps, trace, n * 8, cudaMemcpyDeviceToHost, c->stream)) &&
              note(c, "trace", cudaStreamSynchronize(c->stream));
    m->pt.trace = nullptr;
    cudaFree(trace);
    if (!ok || !check_device_error(c, m)) return -1;
    publish_counts(m, 1);
    return static_cast<double>(n);
}

const char *plamo_cuda_decode_path(struct plamo_cuda *c, struct model *model) {
    static thread_local char text[128];
    if (!c) return nullptr;
    cudaSetDevice(c->device);
    DModel *m = find_model(c, model);
    if (!m || !ensure_graph(c, m)) return nullptr;
    if (m->pt_ready) return "persistent";
    snprintf(text, sizeof text, "graph: %s", m->pt_reason);
    return text;
}

void *plamo_cuda_device_alloc(struct plamo_cuda *c, uint64_t bytes) {
    if (!c) return nullptr;
    void *p = nullptr;
    cudaSetDevice(c->device);
    if (!note(c, "alloc", cudaMalloc(&p, bytes ? bytes : 16))) return nullptr;
    return p;
}

void plamo_cuda_device_free(struct plamo_cuda *c, void *p) {
    if (c && p) cudaFree(p);
}

int plamo_cuda_copy_to_device(struct plamo_cuda *c, void *dst, const void *src, uint64_t bytes) {
    return c && note(c, "copy", cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice)) ? 1 : 0;
}

int plamo_cuda_copy_to_host(struct plamo_cuda *c, void *dst, const void *src, uint64_t bytes) {
    return c && note(c, "copy", cudaStreamSynchronize(c->stream)) &&
                   note(c, "copy", cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost))
               ? 1
               : 0;
}

int plamo_cuda_synchronize(struct plamo_cuda *c) {
    return c && note(c, "synchronize", cudaStreamSynchronize(c->stream)) ? 1 : 0;
}

}  // extern "C"

namespace {
bool sync_kv(plamo_cuda *c, DModel *m) {
    for (uint64_t l = 0; l < m->L; ++l) {
        DLayer &L = m->layers[l];
        const uint64_t count = layer_count(L);
        struct cache *hc = L.host->mixer->cache;
        struct rotation *r = L.host->mixer->rotation;
        if (count) {
            float *k = nullptr, *v = nullptr, *rot = nullptr;
            const uint64_t bytes = count * m->KVW * 4;
            if (!note(c, "sync alloc", cudaMalloc(&k, bytes)) || !note(c, "sync alloc", cudaMalloc(&v, bytes)) ||
                !note(c, "sync alloc", cudaMalloc(&rot, bytes))) {
                cudaFree(k);
                cudaFree(v);
                return false;
            }
            AttnLayer al = attn_layer(m, l);
            kv_gather_kernel<<<count, 256, 0, c->stream>>>(al, m->KVW, m->KH, m->D, count, k, v, rot);
            c->info.launches++;
            bool ok = note(c, "gather", cudaGetLastError()) &&
                      note(c, "sync k", cudaMemcpyAsync(hc->k, k, bytes, cudaMemcpyDeviceToHost, c->stream)) &&
                      note(c, "sync v", cudaMemcpyAsync(hc->v, v, bytes, cudaMemcpyDeviceToHost, c->stream)) &&
                      note(c, "sync rot", cudaMemcpyAsync(r->out, rot, bytes, cudaMemcpyDeviceToHost, c->stream)) &&
                      note(c, "sync", cudaStreamSynchronize(c->stream));
            cudaFree(k);
            cudaFree(v);
            cudaFree(rot);
            if (!ok) return false;
            // cos/sin scratch at the newest local position, as the CPU leaves it.
            const uint64_t half = m->D / 2;
            std::vector<float> row(m->D);
            build_rope_rows(L.rope->freq.data(), m->D, L.scale, count - 1, count, row.data());
            memcpy(r->cos, row.data(), half * 4);
            memcpy(r->sin, row.data() + half, half * 4);
        }
        hc->count = count;
        r->processed_count = count;
        r->scale_bits = float_to_bits(L.scale);
        L.host_hash = newest_row_hash(m, L);
    }
    return true;
}
}  // namespace
