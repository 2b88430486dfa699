// Run-time model descriptor builder (interface: include/plamo_layout.h).
//
// Makes the records the reference generates at build time (reference
// tools/model_layout.py:71-199 for the records and their wiring,
// tools/weight_schema.py:15-42 for the slot order, tools/rope_constants.py:
// 21-76 for the frequency tables and the concentration). Host memory only.
#include "../../include/plamo_layout.h"

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <new>
#include <string>
#include <vector>

namespace {

float fp(double v) { return static_cast<float>(v); }

// Frequency table of reference tools/rope_constants.py:21-52: every
// intermediate rounded to FP32 as the upstream tensor operations do.
void frequencies(double base, uint64_t half, bool yarn, double factor, double original, double beta_fast,
                 double beta_slow, float *out) {
    const double two_pi = 2.0 * 3.141592653589793;
    double low = 0.0, high = 0.0;
    if (yarn) {
        low = static_cast<double>(half) * std::log(original / (beta_fast * two_pi)) / std::log(base);
        high = static_cast<double>(half) * std::log(original / (beta_slow * two_pi)) / std::log(base);
    }
    for (uint64_t i = 0; i < half; ++i) {
        const float frequency = fp(std::pow(base, static_cast<double>(i) / static_cast<double>(half)));
        float value = fp(1.0 / static_cast<double>(frequency));
        if (yarn) {
            const float ramp = fp(static_cast<double>(fp(static_cast<double>(i) - static_cast<double>(fp(low)))) /
                                  static_cast<double>(fp(high - low)));
            const double clamped = std::fmax(0.0, std::fmin(1.0, static_cast<double>(ramp)));
            const float mask = fp(1.0 - clamped);
            const float interpolated = fp(1.0 / static_cast<double>(fp(factor * static_cast<double>(frequency))));
            const float keep = fp(1.0 - static_cast<double>(mask));
            value = fp(static_cast<double>(fp(static_cast<double>(interpolated) * static_cast<double>(keep))) +
                       static_cast<double>(fp(static_cast<double>(value) * static_cast<double>(mask))));
        }
        out[i] = value;
    }
}

// Per-layer tensors in the reference's slot order (tools/weight_schema.py:30-41).
const char *const kLayerTensors[10] = {
    "mixer.qkv_proj.weight",  "mixer.o_proj.weight",    "mixer.q_norm.weight",  "mixer.k_norm.weight",
    "mlp.gate_up_proj.weight", "mlp.down_proj.weight",  "pre_mixer_norm.weight", "post_mixer_norm.weight",
    "pre_mlp_norm.weight",     "post_mlp_norm.weight",
};

bool mul_ok(uint64_t a, uint64_t b, uint64_t *out) {
    if (a && b > UINT64_MAX / a) return false;
    *out = a * b;
    return true;
}

}  // namespace

struct plamo_model_layout {
    plamo_model_config cfg;
    uint64_t full_capacity;
    std::vector<qkv> qkvs;
    std::vector<cache> caches;
    std::vector<rotation> rotations;
    std::vector<gqa> gqas;
    std::vector<mixer> mixers;
    std::vector<mlp> mlps;
    std::vector<layer> layers;
    std::vector<layer *> layer_ptrs;
    model m;
    float *arena;
    uint64_t arena_bytes;
    std::vector<std::string> names;
    std::vector<std::vector<uint64_t>> shapes;
    std::vector<plamo_weight_spec> schema;
};

extern "C" {

int plamo_model_config_profile(const char *name, struct plamo_model_config *cfg) {
    if (!name || !cfg) return 0;
    struct Row {
        const char *name;
        uint64_t hidden, layers, qh, kh, inter, tied;
    };
    // reference tools/profiles/<name>/config.json
    static const Row rows[] = {
        {"0.8b", 1536, 16, 16, 1, 6144, 0},
        {"2b", 2560, 24, 24, 4, 10240, 0},
        {"8b", 4096, 32, 32, 4, 16384, 0},
        {"31b", 5120, 64, 64, 8, 25600, 1},
    };
    for (const Row &r : rows) {
        if (strcmp(r.name, name)) continue;
        memset(cfg, 0, sizeof *cfg);
        cfg->hidden = r.hidden;
        cfg->layers = r.layers;
        cfg->query_heads = r.qh;
        cfg->kv_heads = r.kh;
        cfg->head_dim = 128;
        cfg->intermediate = r.inter;
        cfg->vocab = 107520;
        cfg->window = 2048;
        cfg->pattern = 8;
        cfg->max_position = 262144;
        cfg->tied = r.tied;
        cfg->local_theta = 10000.0;
        cfg->global_theta = 1000000.0;
        cfg->yarn_factor = 256.0;
        cfg->yarn_original = 4096.0;
        cfg->beta_fast = 32.0;
        cfg->beta_slow = 1.0;
        return 1;
    }
    return 0;
}

void plamo_rope_frequencies(const struct plamo_model_config *cfg, int yarn, float *out) {
    if (!cfg || !out) return;
    const uint64_t half = cfg->head_dim / 2;
    if (yarn)
        frequencies(cfg->global_theta, half, true, cfg->yarn_factor, cfg->yarn_original, cfg->beta_fast,
                    cfg->beta_slow, out);
    else
        frequencies(cfg->local_theta, half, false, 0.0, 0.0, 0.0, 0.0, out);
}

struct plamo_model_layout *plamo_model_layout_create(const struct plamo_model_config *cfg, uint64_t full_capacity,
                                                     char *error, size_t cap) {
    auto fail = [&](const char *why) -> plamo_model_layout * {
        if (error && cap) snprintf(error, cap, "%s", why);
        return nullptr;
    };
    if (!cfg) return fail("no configuration");
    const plamo_model_config &c = *cfg;
    if (!c.hidden || !c.layers || !c.query_heads || !c.kv_heads || !c.head_dim || !c.intermediate || !c.vocab ||
        !c.pattern || !c.max_position || c.head_dim % 2 || c.query_heads % c.kv_heads)
        return fail("invalid model dimensions");
    if (!(c.local_theta > 1.0) || !(c.global_theta > 1.0) || !(c.yarn_factor > 0.0) || !(c.yarn_original > 0.0) ||
        !(c.beta_fast > 0.0) || !(c.beta_slow > 0.0) || c.beta_fast == c.beta_slow)
        return fail("invalid RoPE parameters");
    const uint64_t full_rows = full_capacity ? std::min(full_capacity, c.max_position) : c.max_position;
    const uint64_t sliding_rows = c.window + 1;
    const uint64_t h = c.hidden, dim = c.head_dim, half = dim / 2, L = c.layers;
    const uint64_t qw = (c.query_heads + 2 * c.kv_heads) * dim, aw = c.query_heads * dim, kvw = c.kv_heads * dim;
    const uint64_t max_rows = std::max(full_rows, sliding_rows);

    // Work buffers (reference tools/model_layout.py:142-155), then per layer
    // keys, values and rotated keys; 16-float alignment for every buffer.
    auto rounded = [](uint64_t n) { return (n + 15) & ~15ull; };
    const uint64_t work[] = {h, h, h, qw, aw, 2 * c.intermediate, max_rows, half, half, c.vocab, L, half, half};
    uint64_t floats = 0;
    for (uint64_t n : work) floats += rounded(n);
    uint64_t per_layer_rows = 0;
    for (uint64_t i = 0; i < L; ++i) {
        const bool full = (i + 1) % c.pattern == 0;
        uint64_t rows_floats;
        if (!mul_ok(full ? full_rows : sliding_rows, kvw, &rows_floats)) return fail("cache too large");
        per_layer_rows += 3 * rounded(rows_floats);
        if (per_layer_rows > UINT64_MAX / 8) return fail("cache too large");
    }
    floats += per_layer_rows;
    uint64_t bytes;
    if (!mul_ok(floats, sizeof(float), &bytes)) return fail("cache too large");

    auto *lay = new (std::nothrow) plamo_model_layout();
    if (!lay) return fail("out of memory");
    lay->cfg = c;
    lay->full_capacity = full_rows;
    // calloc: zeroed, and pages of unused KV rows are never touched.
    lay->arena = static_cast<float *>(calloc(floats, sizeof(float)));
    if (!lay->arena) {
        delete lay;
        return fail("out of memory");
    }
    lay->arena_bytes = bytes;
    float *next = lay->arena;
    auto take = [&](uint64_t n) {
        float *p = next;
        next += rounded(n);
        return p;
    };
    float *state = take(h), *normalized = take(h), *branch = take(h), *qkvout = take(qw), *attention = take(aw);
    float *mlp_scratch = take(2 * c.intermediate), *scores = take(max_rows), *cosv = take(half), *sinv = take(half);
    float *logits = take(c.vocab), *scales = take(L), *local = take(half), *global = take(half);
    plamo_rope_frequencies(&c, 0, local);
    plamo_rope_frequencies(&c, 1, global);
    const float concentration = fp(1.0 + 0.1 * std::log(c.yarn_factor));

    lay->qkvs.resize(L);
    lay->caches.resize(L);
    lay->rotations.resize(L);
    lay->gqas.resize(L);
    lay->mixers.resize(L);
    lay->mlps.resize(L);
    lay->layers.resize(L);
    lay->layer_ptrs.resize(L);
    for (uint64_t i = 0; i < L; ++i) {
        const bool full = (i + 1) % c.pattern == 0;
        const uint64_t rows = full ? full_rows : sliding_rows;
        float *k = take(rows * kvw), *v = take(rows * kvw), *rot = take(rows * kvw);
        scales[i] = full ? concentration : 1.0f;
        lay->qkvs[i] = qkv{normalized, nullptr, nullptr, nullptr, qkvout, h, c.query_heads, c.kv_heads, dim};
        lay->caches[i] = cache{k, v, rows, 0, kvw, full ? 0ull : 1ull};
        lay->rotations[i] =
            rotation{&lay->caches[i], rot, full ? global : local, cosv, sinv, c.kv_heads, dim, 0, 0};
        lay->gqas[i] = gqa{qkvout, rot, v, attention, scores, 0, dim, c.query_heads, c.kv_heads};
        lay->mixers[i] = mixer{&lay->qkvs[i], &lay->caches[i], &lay->rotations[i], &lay->gqas[i], nullptr, branch, h};
        lay->mlps[i] = mlp{state, nullptr, nullptr, nullptr, nullptr, normalized, branch, mlp_scratch,
                           h, c.intermediate};
        lay->layers[i] = layer{state, nullptr, nullptr, normalized, branch, &lay->mixers[i], &lay->mlps[i], h};
        lay->layer_ptrs[i] = &lay->layers[i];
    }
    lay->m = model{nullptr, c.vocab, h, state, lay->layer_ptrs.data(), L, scales, nullptr, normalized, nullptr,
                   logits};

    // Schema (reference tools/weight_schema.py:15-42): names, shapes, slots.
    const uint64_t rows_count = 2 + (c.tied ? 0 : 1) + 10 * L;
    lay->names.reserve(rows_count);
    lay->shapes.reserve(rows_count);
    std::vector<void **> slots;
    auto add = [&](std::string name, std::vector<uint64_t> shape, void *slot) {
        lay->names.push_back(std::move(name));
        lay->shapes.push_back(std::move(shape));
        slots.push_back(static_cast<void **>(slot));
    };
    model &m = lay->m;
    add("model.embed_tokens.weight", {c.vocab, h}, &m.embedding);
    add("model.norm.weight", {h}, &m.norm);
    if (!c.tied) add("lm_head.weight", {c.vocab, h}, &m.head);
    for (uint64_t i = 0; i < L; ++i) {
        const std::string prefix = "model.layers.layers." + std::to_string(i) + ".";
        void *fields[10] = {&lay->qkvs[i].weight, &lay->mixers[i].weight, &lay->qkvs[i].qn, &lay->qkvs[i].kn,
                            &lay->mlps[i].gu,     &lay->mlps[i].down,     &lay->layers[i].pre, &lay->layers[i].post,
                            &lay->mlps[i].pre,    &lay->mlps[i].post};
        const std::vector<uint64_t> shapes[10] = {{qw, h}, {h, aw},      {dim}, {dim}, {2 * c.intermediate, h},
                                                  {h, c.intermediate}, {h}, {h}, {h}, {h}};
        for (int t = 0; t < 10; ++t) add(prefix + kLayerTensors[t], shapes[t], fields[t]);
    }
    lay->schema.resize(rows_count + 1);
    for (uint64_t r = 0; r < rows_count; ++r)
        lay->schema[r] = plamo_weight_spec{lay->names[r].c_str(), lay->shapes[r].size(), lay->shapes[r].data(),
                                           slots[r]};
    lay->schema[rows_count] = plamo_weight_spec{nullptr, 0, nullptr, nullptr};
    return lay;
}

const struct plamo_weight_spec *plamo_model_layout_schema(const struct plamo_model_layout *layout) {
    return layout ? layout->schema.data() : nullptr;
}

int plamo_model_layout_finish(struct plamo_model_layout *layout) {
    if (!layout) return 0;
    if (layout->cfg.tied) layout->m.head = layout->m.embedding;
    for (const plamo_weight_spec &s : layout->schema)
        if (s.name && !*s.slot) return 0;
    return layout->m.embedding && layout->m.head && layout->m.norm ? 1 : 0;
}

struct model *plamo_model_layout_model(struct plamo_model_layout *layout) { return layout ? &layout->m : nullptr; }

uint64_t plamo_model_layout_buffer_bytes(const struct plamo_model_layout *layout) {
    return layout ? layout->arena_bytes : 0;
}

void plamo_model_layout_destroy(struct plamo_model_layout *layout) {
    if (!layout) return;
    free(layout->arena);
    delete layout;
}

}  // extern "C"
