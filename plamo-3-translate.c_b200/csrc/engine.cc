// Linux translation engine over the CUDA backend (include/plamo_engine.h).
//
// The request path of reference runtime/engine.c (open :101-227, prepare
// :343-388, translate :428-617) composed from this library's parts: the
// tokenizer wraps and encodes the text, the mapped checkpoint is bound into
// run-time descriptors, the CUDA backend keeps the weights in HBM and runs
// prefill and greedy decode on the device, and the template prefix of each
// translation direction is a device snapshot restored into every request that
// starts with it. Only token ids cross to the host during decode; bytes are
// decoded here and streamed through the caller's callbacks.
#include "../../include/plamo_engine.h"
#include "../../include/plamo_safetensors.h"
#include "../../include/plamo_tokenizer.h"

#include <dirent.h>
#include <sys/resource.h>

#include <algorithm>
#include <chrono>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>
#include <string>
#include <vector>

namespace {

constexpr uint64_t kMaxPrompt = 4096;
constexpr unsigned kMaxTokens = 4096;

double wall_seconds() {
    return std::chrono::duration<double>(std::chrono::steady_clock::now().time_since_epoch()).count();
}

void say(char *error, size_t cap, const char *fmt, ...) {
    if (!error || !cap) return;
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(error, cap, fmt, ap);
    va_end(ap);
}

// 64-bit FNV-1a: the reference's result hashes of logits and state
// (runtime/engine.c:31-39), kept alike so hashes compare across backends.
uint64_t fnv1a(const void *data, size_t bytes) {
    const unsigned char *p = static_cast<const unsigned char *>(data);
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < bytes; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

bool ends_with(const std::string &s, const char *suffix) {
    const size_t n = strlen(suffix);
    return s.size() >= n && s.compare(s.size() - n, n, suffix) == 0;
}

}  // namespace

struct plamo_engine {
    plamo_engine_info info{};
    plamo_tokenizer *tokenizer = nullptr;
    std::vector<plamo_mapping> shards;
    plamo_model_layout *layout = nullptr;
    model *net = nullptr;
    plamo_cuda *cuda = nullptr;
    plamo_cuda_prompt_cache *prefix[2] = {nullptr, nullptr};
    bool tokenizer_only = false, uploaded = false, prepared = false, prefixes_done = false;

    ~plamo_engine() {
        for (plamo_cuda_prompt_cache *p : prefix) plamo_cuda_prompt_cache_free(p);
        if (cuda) {
            if (net) plamo_cuda_release_model(cuda, net);
            plamo_cuda_close(cuda);
        }
        plamo_model_layout_destroy(layout);
        for (plamo_mapping &m : shards) plamo_unmap_file(&m);
        plamo_tokenizer_close(tokenizer);
    }

    void refresh_info() {
        if (cuda) plamo_cuda_get_info(cuda, &info.gpu);
    }

    // Every shard into HBM (once); the bound tensors are found inside them
    // by host address.
    bool upload(char *error, size_t cap) {
        if (uploaded) return true;
        const double t0 = wall_seconds();
        for (const plamo_mapping &m : shards)
            if (!plamo_cuda_preload(cuda, m.base, m.bytes)) {
                refresh_info();
                say(error, cap, "engine: cannot copy the checkpoint into device memory (%s)", info.gpu.note);
                return false;
            }
        info.preloaded_weight_bytes = info.weight_bytes;
        info.preload_seconds += wall_seconds() - t0;
        uploaded = true;
        return true;
    }

    bool prepare_model(char *error, size_t cap) {
        if (prepared) return true;
        if (!upload(error, cap)) return false;
        if (plamo_cuda_prepare_model(cuda, net) != 1) {
            refresh_info();
            say(error, cap, "engine: the backend cannot prepare this model (%s)", info.gpu.note);
            return false;
        }
        prepared = true;
        return true;
    }

    void reset() { plamo_cuda_reset_request(cuda, net); }

    // Emit one generated id: 1 emitted, 0 stop or cancel (finish reason set),
    // -1 error.
    int emit(uint32_t id, const plamo_callbacks *cb, plamo_result *r, double start, char *error, size_t cap) {
        if (id == 1 || id == 16) {  // end of text (reference runtime/engine.c:395-420)
            r->finish_reason = "stop";
            return 0;
        }
        if (id >= net->vocab) {
            say(error, cap, "engine: the device produced token %u outside the vocabulary", id);
            return -1;
        }
        const char *bytes = nullptr;
        const uint64_t n = plamo_tokenizer_decode(tokenizer, id, &bytes);
        if (n == UINT64_MAX) {
            say(error, cap, "engine: token %u has no byte form", id);
            return -1;
        }
        const double ready = wall_seconds() - start;
        if (cb && cb->token && !cb->token(id, bytes, static_cast<size_t>(n), cb->context)) {
            r->finish_reason = "cancelled";
            return 0;
        }
        if (r->completion_tokens == 0) r->first_token_seconds = ready;
        ++r->completion_tokens;
        return 1;
    }
};

extern "C" {

struct plamo_engine *plamo_engine_open_files(const struct plamo_engine_files *files, enum plamo_memory_mode mode,
                                             int tokenizer_only, unsigned threads, enum plamo_backend backend,
                                             struct plamo_engine_info *info, char *error, size_t cap) {
    (void)threads;  // the token loop runs on the GPU; no host worker threads
    const double t0 = wall_seconds();
    if (!files || !files->tokenizer) {
        say(error, cap, "engine: no tokenizer file given");
        return nullptr;
    }
    std::unique_ptr<plamo_engine> e(new (std::nothrow) plamo_engine());
    if (!e) {
        say(error, cap, "engine: out of memory");
        return nullptr;
    }
    e->info.threads = 1;
    e->info.backend = "none";
    e->info.memory_mode = tokenizer_only ? "tokenizer" : (mode == PLAMO_MEMORY_RESIDENT ? "resident" : "adaptive");
    e->tokenizer_only = tokenizer_only != 0;
    e->tokenizer = plamo_tokenizer_open(files->tokenizer, error, cap);
    if (!e->tokenizer) return nullptr;
    if (!tokenizer_only) {
        if (backend == PLAMO_BACKEND_CPU) {
            say(error, cap, "engine: this library runs the token loop on CUDA only");
            return nullptr;
        }
        plamo_model_config cfg{};
        if (files->profile ? !plamo_model_config_profile(files->profile, &cfg) : !files->config) {
            say(error, cap, "engine: unknown model profile %s", files->profile ? files->profile : "(none)");
            return nullptr;
        }
        if (!files->profile) cfg = *files->config;
        const uint64_t max_context = files->max_context ? files->max_context : 8192 + 16;
        e->layout = plamo_model_layout_create(&cfg, max_context, error, cap);
        if (!e->layout) return nullptr;
        if (!files->weights || !files->weight_count) {
            say(error, cap, "engine: no checkpoint shards given");
            return nullptr;
        }
        for (unsigned i = 0; i < files->weight_count; ++i) {
            plamo_mapping m{};
            if (!plamo_map_file(files->weights[i], &m)) {
                say(error, cap, "engine: cannot map checkpoint shard %s", files->weights[i]);
                return nullptr;
            }
            e->shards.push_back(m);
            e->info.weight_bytes += m.bytes;
        }
        if (!plamo_bind_weights(e->shards.data(), e->shards.size(), plamo_model_layout_schema(e->layout)) ||
            !plamo_model_layout_finish(e->layout)) {
            say(error, cap, "engine: the checkpoint does not hold every tensor of this profile with its shape");
            return nullptr;
        }
        e->net = plamo_model_layout_model(e->layout);
        plamo_cuda_config cc{};
        cc.device = files->device;
        cc.max_context = max_context;
        e->cuda = plamo_cuda_open(&cc, error, cap);
        if (!e->cuda) return nullptr;
        e->info.backend = "cuda";
        if (mode == PLAMO_MEMORY_RESIDENT && !e->upload(error, cap)) return nullptr;
        e->refresh_info();
    }
    e->info.load_seconds = wall_seconds() - t0;
    if (info) *info = e->info;
    return e.release();
}

struct plamo_engine *plamo_engine_open(enum plamo_memory_mode mode, int tokenizer_only, unsigned threads,
                                       enum plamo_backend backend, struct plamo_engine_info *info, char *error,
                                       size_t cap) {
    const char *dir = getenv("PLAMO_MODEL_DIR");
    if (!dir || !*dir) {
        say(error, cap, "engine: set PLAMO_MODEL_DIR to the directory holding tokenizer.jsonl and the shards");
        return nullptr;
    }
    const std::string root(dir);
    const std::string vocab = root + "/tokenizer.jsonl";
    std::vector<std::string> names;
    if (DIR *d = opendir(dir)) {
        while (const dirent *ent = readdir(d)) {
            const std::string name = ent->d_name;
            if (ends_with(name, ".safetensors")) names.push_back(root + "/" + name);
        }
        closedir(d);
    }
    std::sort(names.begin(), names.end());
    std::vector<const char *> paths;
    for (const std::string &n : names) paths.push_back(n.c_str());
    const char *profile = getenv("PLAMO_MODEL_PROFILE");
    plamo_engine_files files{};
    files.tokenizer = vocab.c_str();
    files.weights = paths.data();
    files.weight_count = static_cast<unsigned>(paths.size());
    files.profile = profile && *profile ? profile : "8b";
    return plamo_engine_open_files(&files, mode, tokenizer_only, threads, backend, info, error, cap);
}

void plamo_engine_close(struct plamo_engine *e) { delete e; }

void plamo_engine_get_info(struct plamo_engine *e, struct plamo_engine_info *out) {
    if (!e || !out) return;
    e->refresh_info();
    *out = e->info;
}

void plamo_engine_maintain_memory(struct plamo_engine *e) {
    if (e && e->cuda) plamo_cuda_maintain(e->cuda);
}

int plamo_engine_prepare(struct plamo_engine *e, char *error, size_t cap) {
    if (!e) return 0;
    const char *setting = getenv("PLAMO_PREFIX_CACHE");
    if (setting && strcmp(setting, "0") && strcmp(setting, "1")) {
        say(error, cap, "engine: PLAMO_PREFIX_CACHE takes 0 or 1");
        return 0;
    }
    if (e->tokenizer_only) return 1;
    const double t0 = wall_seconds();
    if (!e->prepare_model(error, cap)) return 0;
    e->info.load_seconds += wall_seconds() - t0;
    if (e->prefixes_done || (setting && !strcmp(setting, "0"))) return 1;
    // The fixed head of the translation template, per source language: one
    // prefill each, snapshotted on the device (reference runtime/engine.c:
    // 343-388; a prefix too long for a snapshot is simply not cached).
    const double p0 = wall_seconds();
    for (unsigned d = 0; d < 2; ++d) {
        const uint32_t *ids = nullptr;
        const uint64_t n = plamo_tokenizer_prefix(e->tokenizer, d, &ids, error, cap);
        if (n == UINT64_MAX || n == 0 || n > PLAMO_CUDA_PREFIX_LIMIT) continue;
        std::vector<uint32_t> copy(ids, ids + n);  // the tokenizer's buffer is reused
        e->reset();
        const int r = plamo_cuda_prefill(e->cuda, e->net, copy.data(), n, nullptr);
        if (r < 0) {
            e->reset();
            e->refresh_info();
            say(error, cap, "engine: prefilling the template prefix failed (%s)", e->info.gpu.note);
            return 0;
        }
        if (r == 0) continue;
        e->prefix[d] = plamo_cuda_prompt_cache_capture(e->cuda, e->net, copy.data(), n);
        e->info.prefix_tokens[d] = plamo_cuda_prompt_cache_tokens(e->prefix[d]);
        e->info.prefix_bytes += plamo_cuda_prompt_cache_bytes(e->prefix[d]);
    }
    e->reset();
    e->info.prefix_seconds = wall_seconds() - p0;
    e->info.preload_seconds += e->info.prefix_seconds;
    e->info.load_seconds += e->info.prefix_seconds;
    e->prefixes_done = true;
    return 1;
}

uint64_t plamo_engine_tokenize(struct plamo_engine *e, const char *text, unsigned direction, const uint32_t **ids,
                               char *error, size_t cap) {
    if (!e) return UINT64_MAX;
    return plamo_tokenizer_encode(e->tokenizer, text, direction, ids, error, cap);
}

int plamo_engine_translate(struct plamo_engine *e, const char *text, unsigned direction, unsigned max_tokens,
                           const struct plamo_callbacks *cb, struct plamo_result *result, char *error, size_t cap) {
    if (!e || !result) return 0;
    memset(result, 0, sizeof *result);
    if (e->tokenizer_only || max_tokens == 0 || max_tokens > kMaxTokens) {
        say(error, cap, "engine: translation needs a loaded model and 1..%u tokens", kMaxTokens);
        return 0;
    }
    const double start = wall_seconds();
    const uint32_t *borrowed = nullptr;
    const uint64_t count = plamo_engine_tokenize(e, text, direction, &borrowed, error, cap);
    if (count == UINT64_MAX) return 0;
    if (count == 0) {
        say(error, cap, "engine: the prompt is empty");
        return 0;
    }
    if (count > kMaxPrompt) {
        say(error, cap, "engine: the prompt has %llu tokens, more than %llu", static_cast<unsigned long long>(count),
            static_cast<unsigned long long>(kMaxPrompt));
        return 0;
    }
    const std::vector<uint32_t> ids(borrowed, borrowed + count);
    result->prompt_tokens = count;
    result->tokenize_seconds = wall_seconds() - start;
    if (!e->prepare_model(error, cap)) return 0;
    e->reset();
    if (cb && cb->prefill) cb->prefill(count, cb->context);

    plamo_cuda_info before{}, mid{}, after{};
    plamo_cuda_get_info(e->cuda, &before);
    const double prefill_start = wall_seconds();
    if (direction && e->prefix[direction - 1])
        result->cached_prompt_tokens =
            plamo_cuda_prompt_cache_restore(e->cuda, e->prefix[direction - 1], e->net, ids.data(), count);
    uint32_t id = 0;
    const int ok = plamo_cuda_prefill_greedy(e->cuda, e->net, ids.data() + result->cached_prompt_tokens,
                                             count - result->cached_prompt_tokens, &id);
    result->prefill_seconds = wall_seconds() - prefill_start;
    plamo_cuda_get_info(e->cuda, &mid);
    result->prefill_gpu_seconds = mid.gpu_seconds - before.gpu_seconds;
    result->prefill_command_buffers = mid.graph_launches - before.graph_launches;
    result->prefill_gpu_dispatches = mid.launches - before.launches;
    if (ok != 1) {
        e->refresh_info();
        say(error, cap, "engine: prefill %s (%s)", ok == 0 ? "declined" : "failed", e->info.gpu.note);
        return 0;
    }
    result->prefill_logits_hash = fnv1a(e->net->logits, e->net->vocab * 4);
    result->prefill_state_hash = fnv1a(e->net->state, e->net->hidden * 4);
    result->finish_reason = "length";

    const double decode_start = wall_seconds();
    for (;;) {
        const int emitted = e->emit(id, cb, result, start, error, cap);
        if (emitted < 0) return 0;
        if (emitted == 0 || result->completion_tokens == max_tokens) break;
        uint32_t next = 0;
        if (plamo_cuda_forward_greedy(e->cuda, e->net, id, &next) != 1) {
            e->refresh_info();
            say(error, cap, "engine: decode step failed (%s)", e->info.gpu.note);
            return 0;
        }
        ++result->decode_steps;
        id = next;
    }
    result->decode_seconds = wall_seconds() - decode_start;
    plamo_cuda_get_info(e->cuda, &after);
    result->decode_gpu_seconds = after.gpu_seconds - mid.gpu_seconds;
    result->decode_command_buffers = after.graph_launches - mid.graph_launches;
    result->decode_gpu_dispatches = after.launches - mid.launches;
    // Final state and logits on the host for the result hashes.
    if (result->decode_steps && plamo_cuda_read_outputs(e->cuda, e->net) != 1) {
        say(error, cap, "engine: cannot read the final state back");
        return 0;
    }
    result->logits_hash = fnv1a(e->net->logits, e->net->vocab * 4);
    result->state_hash = fnv1a(e->net->state, e->net->hidden * 4);
    result->total_seconds = wall_seconds() - start;
    return 1;
}

// JSON string literal of `text` (quotes, backslashes and control bytes escaped).
static std::string json_text(const char *text) {
    std::string out = "\"";
    for (const unsigned char *p = reinterpret_cast<const unsigned char *>(text ? text : ""); *p; ++p) {
        if (*p == '"' || *p == '\\') {
            out += '\\';
            out += static_cast<char>(*p);
        } else if (*p < 0x20) {
            char esc[8];
            snprintf(esc, sizeof esc, "\\u%04x", *p);
            out += esc;
        } else {
            out += static_cast<char>(*p);
        }
    }
    return out + "\"";
}

static std::string compute_json(plamo_engine *e) {
    e->refresh_info();
    const plamo_cuda_info &g = e->info.gpu;
    const char *path = e->cuda && e->net ? plamo_cuda_decode_path(e->cuda, e->net) : nullptr;
    char buf[1024];
    snprintf(buf, sizeof buf,
             "\"precision\":\"fp32\",\"weight_storage\":\"bf16\",\"packed_weight_bytes\":0,"
             "\"weight_heap_bytes\":0,\"private_weight_bytes\":%llu,\"disk_cache_hits\":0,"
             "\"disk_cache_weight_bytes\":0,\"disk_cache_storage_bytes\":0,\"disk_cache_mapped_bytes\":0,"
             "\"disk_cache_mapping_bytes\":0,\"residency_sets\":false,\"verification_batches\":%llu,"
             "\"verified_tokens\":%llu,\"committed_tokens\":%llu,\"gpu_dispatches\":%llu,"
             "\"command_buffers\":%llu,\"fused_mlps\":0,\"fused_decodes\":%llu,\"fused_prefills\":%llu,"
             "\"cpu_fallbacks\":0,\"errors\":%llu,\"gpu_seconds\":%.9f,\"allocated_bytes\":%llu,"
             "\"recommended_working_set_bytes\":0,\"kv_bytes\":%llu,\"workspace_bytes\":%llu,"
             "\"sm_count\":%llu,\"declines\":%llu,\"kv_pages_used\":%llu,\"kv_pages_allocated\":%llu,",
             static_cast<unsigned long long>(g.weight_bytes), static_cast<unsigned long long>(g.verification_batches),
             static_cast<unsigned long long>(g.verified_tokens), static_cast<unsigned long long>(g.committed_tokens),
             static_cast<unsigned long long>(g.launches), static_cast<unsigned long long>(g.graph_launches),
             static_cast<unsigned long long>(g.forwards), static_cast<unsigned long long>(g.prefills),
             static_cast<unsigned long long>(g.errors), g.gpu_seconds,
             static_cast<unsigned long long>(g.allocated_bytes), static_cast<unsigned long long>(g.kv_bytes),
             static_cast<unsigned long long>(g.workspace_bytes), static_cast<unsigned long long>(g.sm_count),
             static_cast<unsigned long long>(g.declines), static_cast<unsigned long long>(g.kv_pages_used),
             static_cast<unsigned long long>(g.kv_pages_allocated));
    return "{\"backend\":" + json_text(e->info.backend) + ",\"device\":" + json_text(g.device) + "," + buf +
           "\"decode_path\":" + json_text(path ? path : "") + ",\"note\":" + json_text(g.note) + "}";
}

size_t plamo_engine_report_json(struct plamo_engine *e, const struct plamo_result *r, char *out, size_t cap) {
    if (!e) return 0;
    std::string json;
    if (!r) {
        json = compute_json(e);
    } else {
        struct rusage usage {};
        getrusage(RUSAGE_SELF, &usage);
        char head[2048];
        snprintf(head, sizeof head,
                 "{\"event\":\"done\",\"finish_reason\":%s,\"usage\":{\"prompt_tokens\":%llu,"
                 "\"completion_tokens\":%llu,\"total_tokens\":%llu,\"cached_prompt_tokens\":%llu},"
                 "\"timings\":{\"tokenize_seconds\":%.9f,\"prefill_seconds\":%.9f,\"decode_seconds\":%.9f,"
                 "\"first_token_seconds\":%.9f,\"total_seconds\":%.9f,\"decode_steps\":%llu,"
                 "\"prefill_gpu_seconds\":%.9f,\"prefill_command_buffers\":%llu,\"prefill_gpu_dispatches\":%llu,"
                 "\"decode_gpu_seconds\":%.9f,\"decode_command_buffers\":%llu,\"decode_gpu_dispatches\":%llu},"
                 "\"weight_io\":{\"staged_bytes\":0,\"read_calls\":0,\"cache_hits\":0,\"cache_hit_bytes\":0,"
                 "\"cache_misses\":0,\"decode_staged_bytes\":0,\"decode_read_calls\":0,\"decode_mapped_bytes\":0},"
                 "\"process_peak_rss_bytes\":%ld,\"verification\":{\"prefill_logits_hash\":\"%016llx\","
                 "\"prefill_state_hash\":\"%016llx\",\"logits_hash\":\"%016llx\",\"state_hash\":\"%016llx\"},"
                 "\"speculative\":{\"enabled\":%s,\"block_tokens\":%u,\"batches\":%llu,\"consumed_tokens\":%llu,"
                 "\"proposed_tokens\":%llu,\"accepted_tokens\":%llu,\"draft_seconds\":%.9f},\"compute\":",
                 json_text(r->finish_reason ? r->finish_reason : "").c_str(),
                 static_cast<unsigned long long>(r->prompt_tokens),
                 static_cast<unsigned long long>(r->completion_tokens),
                 static_cast<unsigned long long>(r->prompt_tokens + r->completion_tokens),
                 static_cast<unsigned long long>(r->cached_prompt_tokens), r->tokenize_seconds, r->prefill_seconds,
                 r->decode_seconds, r->first_token_seconds, r->total_seconds,
                 static_cast<unsigned long long>(r->decode_steps), r->prefill_gpu_seconds,
                 static_cast<unsigned long long>(r->prefill_command_buffers),
                 static_cast<unsigned long long>(r->prefill_gpu_dispatches), r->decode_gpu_seconds,
                 static_cast<unsigned long long>(r->decode_command_buffers),
                 static_cast<unsigned long long>(r->decode_gpu_dispatches), usage.ru_maxrss,
                 static_cast<unsigned long long>(r->prefill_logits_hash),
                 static_cast<unsigned long long>(r->prefill_state_hash),
                 static_cast<unsigned long long>(r->logits_hash), static_cast<unsigned long long>(r->state_hash),
                 e->info.speculative_tokens ? "true" : "false", e->info.speculative_tokens,
                 static_cast<unsigned long long>(r->speculative_batches),
                 static_cast<unsigned long long>(r->speculative_tokens),
                 static_cast<unsigned long long>(r->proposed_tokens),
                 static_cast<unsigned long long>(r->accepted_tokens), r->draft_seconds);
        json = std::string(head) + compute_json(e) + "}";
    }
    if (out && cap) snprintf(out, cap, "%s", json.c_str());
    return json.size();
}

}  // extern "C"
