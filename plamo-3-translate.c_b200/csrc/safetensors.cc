// Host-side BF16 safetensors loader: mapping, header validation, tensor
// lookup and schema binding (interface: include/plamo_safetensors.h).
//
// Follows the reference's loader contract (src/load.s envelope, src/json.s
// restricted lexer, src/tensor.s descriptor rules, src/find.s lookup,
// src/resolve.s shape check, src/bind.s all-or-nothing binding): a strict
// subset of JSON with raw ASCII names, unsigned integers without leading
// zeros, BF16 tensors of rank <= 4 whose byte range lies inside the file and
// matches the shape. Weights stay where the mapping put them; the CUDA
// backend uploads them by host address (plamo_cuda_preload).
#include "../../include/plamo_safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace {

constexpr uint64_t kMaxHeader = 100000000;  // the format's own header limit

enum Token { T_END = 0, T_INVALID = -1, T_STRING = 256, T_UINT = 257 };

struct Lexer {
    const char *p, *end;
    const char *str;  // T_STRING: raw bytes between the quotes
    uint64_t len;
    uint64_t value;   // T_UINT

    int next() {
        while (p < end && (*p == ' ' || *p == '\t' || *p == '\n' || *p == '\r')) ++p;
        if (p == end) return T_END;
        const char c = *p;
        if (c == '{' || c == '}' || c == '[' || c == ']' || c == ':' || c == ',') {
            ++p;
            return c;
        }
        if (c == '"') {
            const char *s = ++p;
            while (p < end && *p != '"') {
                if (*p == '\\') {
                    if (++p == end) return T_INVALID;
                }
                ++p;
            }
            if (p == end) return T_INVALID;
            str = s;
            len = static_cast<uint64_t>(p - s);
            ++p;
            return T_STRING;
        }
        plamo_u64 n;
        if (plamo_parse_u64(p, end, &n)) {
            p = n.next;
            value = n.value;
            return T_UINT;
        }
        return T_INVALID;
    }
    bool is(const char *word) const { return len == strlen(word) && memcmp(str, word, len) == 0; }
};

// One tensor descriptor object (fields in any order, each exactly once).
bool descriptor(Lexer &lx, uint64_t data_size, plamo_tensor *t, uint64_t *offset) {
    memset(t, 0, sizeof *t);
    unsigned seen = 0;
    uint64_t count = 1;
    if (lx.next() != '{') return false;
    for (;;) {
        if (lx.next() != T_STRING) return false;
        if (lx.is("dtype")) {
            if (seen & 1) return false;
            seen |= 1;
            if (lx.next() != ':' || lx.next() != T_STRING || !lx.is("BF16")) return false;
        } else if (lx.is("shape")) {
            if (seen & 2) return false;
            seen |= 2;
            if (lx.next() != ':' || lx.next() != '[') return false;
            int tok = lx.next();
            while (tok != ']') {
                if (tok != T_UINT || t->rank >= 4) return false;
                if (lx.value && count > UINT64_MAX / lx.value) return false;
                count *= lx.value;
                t->dims[t->rank++] = lx.value;
                tok = lx.next();
                if (tok == ',') tok = lx.next();
                else if (tok != ']') return false;
            }
        } else if (lx.is("data_offsets")) {
            if (seen & 4) return false;
            seen |= 4;
            if (lx.next() != ':' || lx.next() != '[' || lx.next() != T_UINT) return false;
            const uint64_t begin = lx.value;
            if (lx.next() != ',' || lx.next() != T_UINT) return false;
            const uint64_t stop = lx.value;
            if (stop < begin || stop > data_size || lx.next() != ']') return false;
            *offset = begin;
            t->bytes = stop - begin;
        } else {
            return false;
        }
        const int sep = lx.next();
        if (sep == ',') continue;
        if (sep != '}' || seen != 7) return false;
        break;
    }
    if (count >> 63 || count * 2 != t->bytes) return false;
    return true;
}

}  // namespace

extern "C" {

int plamo_safetensors_view(const void *file, uint64_t size, struct plamo_safetensors_view *v) {
    memset(v, 0, sizeof *v);
    if (!file || size < 10) return 0;
    uint64_t n;
    memcpy(&n, file, 8);
    if (n > size - 8 || n < 2 || n > kMaxHeader) return 0;
    const char *h = static_cast<const char *>(file) + 8;
    if (h[0] != '{') return 0;
    uint64_t last = n - 1;
    while (last > 0 && h[last] == ' ') --last;  // the format pads headers with spaces
    if (h[last] != '}') return 0;
    v->header = h;
    v->header_size = n;
    v->data = h + n;
    v->data_size = size - 8 - n;
    return 1;
}

int plamo_parse_u64(const char *begin, const char *end, plamo_u64 *out) {
    out->next = nullptr;
    out->value = 0;
    if (!begin || begin >= end || *begin < '0' || *begin > '9') return 0;
    const char *p = begin;
    uint64_t v = 0;
    while (p < end && *p >= '0' && *p <= '9') {
        const uint64_t d = static_cast<uint64_t>(*p - '0');
        if (v > (UINT64_MAX - d) / 10) return 0;
        v = v * 10 + d;
        ++p;
    }
    if (*begin == '0' && p - begin > 1) return 0;  // no leading zeros
    out->next = p;
    out->value = v;
    return 1;
}

int plamo_find_tensor(const void *file, uint64_t size, const char *name, plamo_tensor *out) {
    memset(out, 0, sizeof *out);
    struct plamo_safetensors_view v;
    if (!name || !plamo_safetensors_view(file, size, &v)) return 0;
    Lexer lx{v.header, v.header + v.header_size, nullptr, 0, 0};
    if (lx.next() != '{' || lx.next() != T_STRING) return 0;
    for (;;) {
        const bool wanted = lx.is(name);
        if (lx.is("__metadata__")) {
            if (lx.next() != ':' || lx.next() != '{') return 0;
            int tok = lx.next();
            while (tok != '}') {
                if (tok != T_STRING || lx.next() != ':' || lx.next() != T_STRING) return 0;
                tok = lx.next();
                if (tok == ',') tok = lx.next();
                else if (tok != '}') return 0;
            }
        } else {
            if (lx.next() != ':') return 0;
            plamo_tensor t;
            uint64_t offset = 0;
            if (!descriptor(lx, v.data_size, &t, &offset)) return 0;
            if (wanted) {
                *out = t;
                out->data = reinterpret_cast<const uint16_t *>(static_cast<const char *>(v.data) + offset);
                return 1;
            }
        }
        if (lx.next() != ',' || lx.next() != T_STRING) return 0;
    }
}

const uint16_t *plamo_resolve_weight(const plamo_mapping *shards, uint64_t count, const char *name, uint64_t rank,
                                     const uint64_t *dims) {
    if (!shards || rank > 4) return nullptr;
    for (uint64_t i = 0; i < count; ++i) {
        plamo_tensor t;
        if (!plamo_find_tensor(shards[i].base, shards[i].bytes, name, &t)) continue;
        if (t.rank != rank) return nullptr;
        for (uint64_t d = 0; d < rank; ++d)
            if (t.dims[d] != dims[d]) return nullptr;
        return t.data;
    }
    return nullptr;
}

int plamo_bind_weights(const plamo_mapping *shards, uint64_t count, const plamo_weight_spec *schema) {
    if (!schema) return 0;
    for (const plamo_weight_spec *s = schema; s->name; ++s) {
        const uint16_t *p = plamo_resolve_weight(shards, count, s->name, s->rank, s->shape);
        if (!p) {
            for (const plamo_weight_spec *z = schema; z->name; ++z) *z->slot = nullptr;
            return 0;
        }
        *s->slot = const_cast<uint16_t *>(p);
    }
    return 1;
}

int plamo_map_file(const char *path, plamo_mapping *out) {
    out->base = nullptr;
    out->bytes = 0;
    if (!path) return 0;
    const int fd = open(path, O_RDONLY | O_CLOEXEC);
    if (fd < 0) return 0;
    struct stat st;
    if (fstat(fd, &st) != 0 || !S_ISREG(st.st_mode) || st.st_size <= 0) {
        close(fd);
        return 0;
    }
    void *p = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
    close(fd);
    if (p == MAP_FAILED) return 0;
    out->base = p;
    out->bytes = static_cast<uint64_t>(st.st_size);
    return 1;
}

void plamo_unmap_file(plamo_mapping *m) {
    if (m && m->base) munmap(m->base, static_cast<size_t>(m->bytes));
    if (m) {
        m->base = nullptr;
        m->bytes = 0;
    }
}

}  // extern "C"
