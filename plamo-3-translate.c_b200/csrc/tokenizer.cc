// PLaMo-3 tokenizer for Linux hosts (interface: include/plamo_tokenizer.h).
//
// Restates the reference's tokenizer assembly (reference src/utf8.s,
// string.s, json.s, score.s, vocab.s, vocab_load.s, trie.s, unigram.s,
// encode.s, marked.s, boundary.s, preprocess.s, decode.s, prompt.s) with the
// same entry points, records, validation rules and tie-breaking, and provides
// the engine-facing API of reference runtime/tokenizer.h over them.
#include "../../include/plamo_tokenizer.h"
#include "../../include/plamo_safetensors.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdio>
#include <cstring>
#include <memory>
#include <new>
#include <vector>

namespace {

constexpr uint64_t kFail = UINT64_MAX;
constexpr uint32_t kScalarLimit = 0x110000;
constexpr int32_t kFallbackScore = -10000000;  // byte fallback piece, score x 10000
constexpr int32_t kDeadScore = -20000000;       // candidates at or below never win

bool is_surrogate(uint64_t cp) { return cp >= 0xd800 && cp < 0xe000; }

// Hex digit value of an ASCII scalar (either case).
bool hex_value(uint32_t c, uint32_t *v) {
    if (c - '0' <= 9) {
        *v = c - '0';
        return true;
    }
    const uint32_t l = c | 32;
    if (l - 'a' <= 5) {
        *v = l - 'a' + 10;
        return true;
    }
    return false;
}

// UTF-8 bytes of a valid scalar; returns the byte count.
unsigned utf8_bytes(uint64_t cp, uint8_t *b) {
    if (cp < 0x80) {
        b[0] = static_cast<uint8_t>(cp);
        return 1;
    }
    unsigned n = cp < 0x800 ? 2 : cp < 0x10000 ? 3 : 4;
    static const uint8_t lead[5] = {0, 0, 0xc0, 0xe0, 0xf0};
    b[0] = static_cast<uint8_t>(lead[n] | (cp >> (6 * (n - 1))));
    for (unsigned i = 1; i < n; ++i) b[i] = static_cast<uint8_t>(0x80 | ((cp >> (6 * (n - 1 - i))) & 63));
    return n;
}

bool json_space(char c) { return c == ' ' || c == '\t' || c == '\n' || c == '\r'; }

// Python str.isspace() over the scalars that can appear in a special token body.
bool python_space(uint32_t c) {
    return (c >= 9 && c <= 13) || (c >= 28 && c <= 32) || c == 0x85 || c == 0xa0 || c == 0x1680 ||
           (c >= 0x2000 && c <= 0x200a) || c == 0x2028 || c == 0x2029 || c == 0x202f || c == 0x205f ||
           c == 0x3000;
}

// The template strings of the official PFML3 chat template for one
// translation request (reference src/prompt.s).
const char kPromptHead[] =
    "<|plamo:bos|><|plamo:tag|>dataset<|plamo:msg|>translation<|plamo:tag|>input<|plamo:key|>lang<|plamo:val|>";
const char kPromptMessage[] = "<|plamo:msg|>";
const char kPromptOutput[] = "<|plamo:tag|>output<|plamo:key|>lang<|plamo:val|>";

}  // namespace

extern "C" {

// ---- UTF-8 (reference src/utf8.s) -------------------------------------------
int plamo_utf8_next(const char *cursor, const char *end, struct plamo_scalar *out) {
    out->next = nullptr;
    out->cp = 0;
    if (cursor >= end) return 0;
    const uint8_t *p = reinterpret_cast<const uint8_t *>(cursor);
    const uint8_t *e = reinterpret_cast<const uint8_t *>(end);
    const uint8_t b = *p++;
    if (b < 0x80) {
        out->next = reinterpret_cast<const char *>(p);
        out->cp = b;
        return 1;
    }
    unsigned more;
    uint32_t cp, smallest;
    if (b < 0xc2) return 0;  // continuation byte or overlong two-byte lead
    if (b < 0xe0) {
        more = 1, cp = b & 31, smallest = 0x80;
    } else if (b < 0xf0) {
        more = 2, cp = b & 15, smallest = 0x800;
    } else if (b < 0xf5) {
        more = 3, cp = b & 7, smallest = 0x10000;
    } else {
        return 0;
    }
    for (; more; --more) {
        if (p >= e || (*p & 0xc0) != 0x80) return 0;
        cp = (cp << 6) | (*p++ & 63);
    }
    if (cp < smallest || is_surrogate(cp) || cp >= kScalarLimit) return 0;
    out->next = reinterpret_cast<const char *>(p);
    out->cp = cp;
    return 1;
}

uint64_t plamo_byte_fallback(uint64_t cp, const uint32_t *byte_ids, uint32_t *out) {
    if (cp >= kScalarLimit || is_surrogate(cp)) return 0;
    uint8_t b[4];
    const unsigned n = utf8_bytes(cp, b);
    for (unsigned i = 0; i < n; ++i) out[i] = byte_ids[b[i]];
    return n;
}

// ---- restricted JSON (reference src/json.s, src/string.s) -------------------
int plamo_json_next(const char *cursor, const char *end, struct plamo_json_token *out) {
    memset(out, 0, sizeof *out);
    while (cursor < end && json_space(*cursor)) ++cursor;
    if (cursor >= end) {
        out->next = cursor;
        return 0;
    }
    const char c = *cursor;
    if (c == '{' || c == '}' || c == '[' || c == ']' || c == ':' || c == ',') {
        out->next = cursor + 1;
        out->start = cursor;
        out->length = 1;
        return c;
    }
    if (c == '"') {
        const char *p = cursor + 1;
        while (p < end) {
            const uint8_t ch = static_cast<uint8_t>(*p++);
            if (ch == '"') {
                out->next = p;
                out->start = cursor + 1;
                out->length = static_cast<uint64_t>(p - cursor - 2);
                return 256;
            }
            if (ch < 32) return -1;
            if (ch != '\\') continue;
            if (p >= end) return -1;
            const char esc = *p++;
            if (strchr("\"\\/bfnrt", esc) && esc) continue;
            if (esc != 'u') return -1;
            for (int i = 0; i < 4; ++i) {
                uint32_t v;
                if (p >= end || !hex_value(static_cast<uint8_t>(*p++), &v)) return -1;
            }
        }
        return -1;
    }
    plamo_u64 n;
    if (!plamo_parse_u64(cursor, end, &n)) return -1;
    if (n.next < end) {
        const char d = *n.next;
        if (!json_space(d) && d != ',' && d != ']' && d != '}') return -1;
    }
    out->next = n.next;
    out->start = cursor;
    out->length = static_cast<uint64_t>(n.next - cursor);
    out->value = n.value;
    return 257;
}

uint64_t plamo_json_string(const char *start, const char *end, uint32_t *out, uint64_t capacity) {
    uint64_t count = 0;
    const char *p = start;
    auto hex4 = [&](uint32_t *v) {
        if (end - p < 4) return false;
        *v = 0;
        for (int i = 0; i < 4; ++i) {
            uint32_t d;
            if (!hex_value(static_cast<uint8_t>(*p++), &d)) return false;
            *v = (*v << 4) | d;
        }
        return true;
    };
    while (p < end) {
        if (count >= capacity) return kFail;
        const uint8_t c = static_cast<uint8_t>(*p);
        if (c < 32 || c == '"') return kFail;
        uint32_t value;
        if (c != '\\') {
            plamo_scalar s;
            if (!plamo_utf8_next(p, end, &s)) return kFail;
            p = s.next;
            value = static_cast<uint32_t>(s.cp);
        } else {
            if (++p >= end) return kFail;
            switch (*p++) {
            case '"': value = '"'; break;
            case '\\': value = '\\'; break;
            case '/': value = '/'; break;
            case 'b': value = 8; break;
            case 'f': value = 12; break;
            case 'n': value = 10; break;
            case 'r': value = 13; break;
            case 't': value = 9; break;
            case 'u': {
                if (!hex4(&value)) return kFail;
                if (!is_surrogate(value)) break;
                if (value >= 0xdc00) return kFail;  // a low surrogate first
                const uint32_t high = value - 0xd800;
                if (end - p < 6 || p[0] != '\\' || p[1] != 'u') return kFail;
                p += 2;
                uint32_t low;
                if (!hex4(&low) || low < 0xdc00 || low >= 0xe000) return kFail;
                value = 0x10000 + (high << 10) + (low - 0xdc00);
                break;
            }
            default: return kFail;
            }
        }
        out[count++] = value;
    }
    return count;
}

// ---- vocabulary (reference src/score.s, vocab.s, vocab_load.s) --------------
int plamo_parse_score(const char *cursor, const char *end, struct plamo_score *out) {
    out->next = nullptr;
    out->value = 0;
    if (cursor >= end) return 0;
    const bool negative = *cursor == '-';
    if (negative) ++cursor;
    int64_t value = 0;
    unsigned digits = 0;
    while (cursor < end && static_cast<uint8_t>(*cursor - '0') <= 9) {
        if (digits && !value) return 0;  // leading zero
        value = value * 10 + (*cursor - '0');
        if (value > 1000) return 0;
        ++digits;
        ++cursor;
    }
    if (!digits) return 0;
    value *= 10000;
    if (cursor < end && *cursor == '.') {
        ++cursor;
        int64_t place = 1000;
        unsigned fraction = 0;
        while (cursor < end && static_cast<uint8_t>(*cursor - '0') <= 9) {
            if (!place) return 0;  // more than four decimals
            value += (*cursor - '0') * place;
            place /= 10;
            ++fraction;
            ++cursor;
        }
        if (!fraction) return 0;
    }
    if (cursor < end) {
        const char d = *cursor;
        if (d != ',' && d != ']' && d != ' ' && d != '\t' && d != '\n' && d != '\r') return 0;
    }
    out->next = cursor;
    out->value = negative ? -value : value;
    return 1;
}

int plamo_vocab_row(const char *start, const char *end, uint32_t *cp, uint64_t capacity,
                    struct plamo_vocab_entry *out) {
    memset(out, 0, sizeof *out);
    plamo_json_token t;
    const char *p = start;
    auto expect = [&](int kind) {
        const int k = plamo_json_next(p, end, &t);
        p = t.next;
        return k == kind;
    };
    if (!expect('[') || !expect(256)) return 0;
    const uint64_t length = plamo_json_string(t.start, t.start + t.length, cp, capacity);
    if (length == kFail || !expect(',')) return 0;
    while (p < end && (*p == ' ' || *p == '\t')) ++p;
    plamo_score s;
    if (p >= end || !plamo_parse_score(p, end, &s)) return 0;
    p = s.next;
    if (!expect(',') || !expect(256)) return 0;
    static const char *const types[4] = {"NORMAL", "BYTE", "CONTROL", "UNKNOWN"};
    uint64_t type = 4;
    for (uint64_t i = 0; i < 4; ++i)
        if (strlen(types[i]) == t.length && !memcmp(types[i], t.start, t.length)) type = i;
    if (type == 4 || !expect(']') || !expect(0)) return 0;
    out->length = length;
    out->score = s.value;
    out->type = type;
    return 1;
}

// Byte value of a "<0xHH>" piece (scalars), or -1.
static int byte_piece(const uint32_t *cp, uint64_t length, bool check_frame) {
    if (length != 6) return -1;
    if (check_frame && (cp[0] != '<' || cp[1] != '0' || cp[2] != 'x' || cp[5] != '>')) return -1;
    uint32_t hi, lo;
    if (!hex_value(cp[3], &hi) || !hex_value(cp[4], &lo)) return -1;
    return static_cast<int>(hi * 16 + lo);
}

uint64_t plamo_vocab_load(const char *start, const char *end, struct plamo_trie *trie, uint32_t *scratch,
                          uint64_t scratch_capacity, uint32_t *byte_ids) {
    uint64_t row = 0;
    for (const char *line = start; line < end; ++row) {
        const char *next = static_cast<const char *>(memchr(line, '\n', static_cast<size_t>(end - line)));
        next = next ? next + 1 : end;
        plamo_vocab_entry e;
        if (!plamo_vocab_row(line, next, scratch, scratch_capacity, &e)) return kFail;
        if (e.type == 1) {
            const int b = byte_piece(scratch, e.length, true);
            if (b < 0 || !row || byte_ids[b]) return kFail;  // ids are nonzero and unique
            byte_ids[b] = static_cast<uint32_t>(row);
        } else if (!plamo_trie_insert(trie, scratch, e.length, static_cast<int32_t>(row),
                                      static_cast<int32_t>(e.score))) {
            return kFail;
        }
        line = next;
    }
    for (int b = 0; b < 256; ++b)
        if (!byte_ids[b]) return kFail;
    return row;
}

// ---- trie (reference src/trie.s) --------------------------------------------
int plamo_trie_insert(struct plamo_trie *trie, const uint32_t *cp, uint64_t length, int32_t id, int32_t score) {
    if (!length || trie->used > trie->capacity || length > trie->capacity - trie->used) return 0;
    plamo_trie_node *nodes = trie->nodes;
    uint64_t used = trie->used;
    uint32_t at = 0;  // root
    for (uint64_t k = 0; k < length; ++k) {
        const uint32_t c = cp[k];
        uint32_t *index = (at == 0 && trie->roots && c < kScalarLimit) ? &trie->roots[c] : nullptr;
        uint32_t found = 0;
        if (index) {
            found = *index;
        } else {
            for (uint32_t n = nodes[at].child; n; n = nodes[n].sibling)
                if (nodes[n].cp == c) {
                    found = n;
                    break;
                }
        }
        if (!found) {
            found = static_cast<uint32_t>(used++);
            nodes[found] = plamo_trie_node{c, 0, nodes[at].child, 0, 0, 0};
            nodes[at].child = found;
            if (index) *index = found;
        }
        at = found;
    }
    nodes[at].id = id;
    nodes[at].score = score;
    nodes[at].terminal = 1;
    trie->used = used;
    return 1;
}

uint64_t plamo_trie_match(const struct plamo_trie *trie, const uint32_t *cp, uint64_t available,
                          struct plamo_candidate *out, uint64_t capacity) {
    const plamo_trie_node *nodes = trie->nodes;
    uint64_t count = 0;
    uint32_t at = 0;
    for (uint64_t k = 0; k < available; ++k) {
        const uint32_t c = cp[k];
        uint32_t found = 0;
        if (k == 0 && trie->roots && c < kScalarLimit) {
            found = trie->roots[c];
        } else {
            for (uint32_t n = nodes[at].child; n; n = nodes[n].sibling)
                if (nodes[n].cp == c) {
                    found = n;
                    break;
                }
        }
        if (!found) break;
        at = found;
        if (!nodes[at].terminal) continue;
        if (count >= capacity) return kFail;
        out[count++] = plamo_candidate{static_cast<uint32_t>(k + 1), nodes[at].id, nodes[at].score, 0};
    }
    return count;
}

// ---- Unigram segmentation (reference src/unigram.s, encode.s, marked.s) -----
int plamo_unigram_step(const int64_t *costs, const struct plamo_candidate *candidates, uint64_t count,
                       uint64_t available, struct plamo_unigram_path *out) {
    int64_t best = int64_t{1} << 60;
    uint64_t best_length = 0;
    int64_t best_id = -1;
    for (uint64_t i = 0; i < count; ++i) {
        const plamo_candidate &c = candidates[i];
        if (!c.length || c.length > available || c.score <= kDeadScore) continue;
        int64_t cost;
        if (__builtin_sub_overflow(costs[c.length], static_cast<int64_t>(c.score), &cost)) continue;
        if (cost > best || (cost == best && c.length <= best_length)) continue;
        best = cost;
        best_length = c.length;
        best_id = c.id;
    }
    out->cost = best;
    out->length = static_cast<int64_t>(best_length);
    out->id = best_id;
    return best_length != 0;
}

uint64_t plamo_encode_segment(const struct plamo_encoder *e) {
    const uint64_t n = e->count;
    e->costs[n] = 0;
    if (!e->capacity) return kFail;
    auto *paths = static_cast<plamo_unigram_path *>(e->paths);
    auto *cands = static_cast<plamo_candidate *>(e->candidates);
    // Backward: the cheapest way to finish from every position.
    for (uint64_t pos = n; pos-- > 0;) {
        const uint64_t found = plamo_trie_match(e->trie, e->cp + pos, n - pos, cands, e->capacity - 1);
        if (found == kFail) return kFail;
        cands[found] = plamo_candidate{1, -1, kFallbackScore, 0};
        if (!plamo_unigram_step(e->costs + pos, cands, found + 1, n - pos, &paths[pos])) return kFail;
        e->costs[pos] = paths[pos].cost;
    }
    // Forward: emit the chosen pieces, byte fallback for id -1.
    uint64_t written = 0;
    for (uint64_t pos = 0; pos < n;) {
        const plamo_unigram_path &p = paths[pos];
        if (p.id < 0) {
            uint32_t ids[4];
            const uint64_t k = plamo_byte_fallback(e->cp[pos], e->bytes, ids);
            if (!k || k > e->out_capacity - written) return kFail;
            memcpy(e->out + written, ids, k * sizeof(uint32_t));
            written += k;
            pos += 1;
        } else {
            if (written >= e->out_capacity) return kFail;
            e->out[written++] = static_cast<uint32_t>(p.id);
            pos += static_cast<uint64_t>(p.length);
        }
    }
    return written;
}

uint64_t plamo_encode_marked(const struct plamo_encoder *e) {
    plamo_encoder segment = *e;
    uint64_t written = 0;
    for (uint64_t i = 0; i < e->count;) {
        if (e->cp[i] == PLAMO_SEGMENT_MARKER) {
            ++i;
            continue;
        }
        uint64_t j = i + 1;
        while (j < e->count && e->cp[j] != PLAMO_SEGMENT_MARKER) ++j;
        segment.cp = e->cp + i;
        segment.count = j - i;
        segment.out = e->out + written;
        segment.out_capacity = e->out_capacity - written;
        const uint64_t k = plamo_encode_segment(&segment);
        if (k == kFail) return kFail;
        written += k;
        i = j;
    }
    return written;
}

// ---- preprocessing (reference src/boundary.s, preprocess.s) -----------------
void plamo_repeat_boundaries(const uint32_t *cp, uint64_t count, uint8_t *flags) {
    for (uint64_t i = 0; i < count;) {
        uint64_t j = i + 1;
        while (j < count && cp[j] == cp[i]) ++j;
        const uint64_t run = j - i;
        const bool mark = (cp[i] == ' ' && run >= 2) || (cp[i] != '\n' && run >= 4);
        if (mark) flags[i] = flags[j] = 1;
        i = j;
    }
}

void plamo_special_boundaries(const uint32_t *cp, uint64_t count, uint8_t *flags) {
    static const char prefix[] = "<|plamo:";
    uint64_t i = 0;
    while (count - i >= 10 && i < count) {
        bool open = true;
        for (int k = 0; k < 8 && open; ++k) open = cp[i + k] == static_cast<uint32_t>(prefix[k]);
        uint64_t close = 0;
        if (open) {
            for (uint64_t j = i + 8, body = 0; j < count; ++j, ++body) {
                if (cp[j] == '|') {
                    if (j + 1 < count && cp[j + 1] == '>') close = j + 2;
                    break;
                }
                if (body >= 64 || python_space(cp[j])) break;
            }
        }
        if (close) {
            flags[i] = flags[close] = 1;
            i = close;
        } else {
            ++i;
        }
    }
}

// Scalars of `in` with a marker before every flagged position (flags[count]
// included); the output count or kFail.
static uint64_t expand_markers(const uint32_t *in, uint64_t count, const uint8_t *flags, uint32_t *out,
                               uint64_t capacity) {
    uint64_t w = 0;
    for (uint64_t i = 0;; ++i) {
        if (flags[i]) {
            if (w >= capacity) return kFail;
            out[w++] = PLAMO_SEGMENT_MARKER;
        }
        if (i >= count) return w;
        if (w >= capacity) return kFail;
        out[w++] = in[i];
    }
}

uint64_t plamo_preprocess(const struct plamo_preprocess_args *a) {
    memset(a->flags, 0, a->count + 1);
    plamo_special_boundaries(a->in, a->count, a->flags);
    const uint64_t n = expand_markers(a->in, a->count, a->flags, a->temp, a->temp_capacity);
    if (n == kFail) return kFail;
    memset(a->flags, 0, n + 1);
    plamo_repeat_boundaries(a->temp, n, a->flags);
    return expand_markers(a->temp, n, a->flags, a->out, a->capacity);
}

// ---- decoding and prompts (reference src/decode.s, prompt.s) ----------------
uint64_t plamo_decode_token(const char *vocab, const char *end, uint64_t id, char *out, uint64_t capacity,
                            uint32_t *scratch, uint64_t scratch_capacity) {
    const char *line = vocab;
    for (uint64_t skip = id; skip; --skip) {
        const char *nl = static_cast<const char *>(memchr(line, '\n', static_cast<size_t>(end - line)));
        if (!nl) return kFail;
        line = nl + 1;
    }
    const char *nl = static_cast<const char *>(memchr(line, '\n', static_cast<size_t>(end - line)));
    plamo_vocab_entry e;
    if (!plamo_vocab_row(line, nl ? nl + 1 : end, scratch, scratch_capacity, &e)) return kFail;
    if (e.type == 1) {  // a raw byte
        const int b = byte_piece(scratch, e.length, false);
        if (!capacity || b < 0) return kFail;
        out[0] = static_cast<char>(b);
        return 1;
    }
    uint64_t written = 0;
    for (uint64_t i = 0; i < e.length; ++i) {
        if (scratch[i] >= kScalarLimit || is_surrogate(scratch[i])) return kFail;
        uint8_t b[4];
        const unsigned n = utf8_bytes(scratch[i], b);
        if (n > capacity - written) return kFail;
        memcpy(out + written, b, n);
        written += n;
    }
    return written;
}

uint64_t plamo_translation_prompt(const char *text, const char *source, const char *target, char *out,
                                  uint64_t capacity) {
    const char *const parts[7] = {kPromptHead, source, kPromptMessage, text, kPromptOutput, target, kPromptMessage};
    uint64_t w = 0;
    for (const char *part : parts) {
        if (!part) break;  // the prefix stops before the text
        for (const char *c = part; *c; ++c) {
            if (w + 1 >= capacity) return kFail;
            out[w++] = *c;
        }
    }
    if (w >= capacity) return kFail;
    out[w] = 0;
    return w;
}

uint64_t plamo_translation_prefix(const char *source, char *out, uint64_t capacity) {
    return plamo_translation_prompt(nullptr, source, nullptr, out, capacity);
}

}  // extern "C"

// ---- the engine's tokenizer (reference runtime/tokenizer.h) -------------------
//
// One object per opened vocabulary. It keeps the file's bytes mapped read-only
// (a decoded token is a slice of its row), the trie and the byte-piece ids
// built from them, an index of row starts, and every buffer a request needs,
// sized once at open so that encoding and decoding allocate nothing.
namespace {

// Capacities of one request (the reference engine's limits).
constexpr uint64_t kTrieNodes = 1000000;
constexpr uint64_t kMaxScalars = 4096;       // Unicode scalars of the text
constexpr uint64_t kTempCapacity = 16384;    // after special-token marking
constexpr uint64_t kMarkedCapacity = 49152;  // after repeated-run marking
constexpr uint64_t kMaxIds = 16384;
constexpr uint64_t kCandidates = 4097;       // trie matches at one position, plus the fallback
constexpr size_t kTextBytes = 16384;         // a wrapped prompt, a decoded piece

enum class TokStatus { Ok, NoMemory, Unreadable, BadRows, BadLineBreaks, BadArguments, BadDirection,
                       PromptTooLong, BadText, MarkingOverflow, SegmentOverflow };

const char *status_text(TokStatus s) {
    switch (s) {
    case TokStatus::NoMemory: return "tokenizer: out of memory";
    case TokStatus::Unreadable: return "tokenizer: vocabulary file missing or unreadable";
    case TokStatus::BadRows: return "tokenizer: vocabulary file is not 107520 well-formed rows";
    case TokStatus::BadLineBreaks: return "tokenizer: vocabulary line breaks do not match its rows";
    case TokStatus::BadArguments: return "tokenizer: null tokenizer, text or output";
    case TokStatus::BadDirection: return "tokenizer: translation direction must be 0, 1 or 2";
    case TokStatus::PromptTooLong: return "tokenizer: text too long for the translation template";
    case TokStatus::BadText: return "tokenizer: text is not UTF-8 or longer than 4096 characters";
    case TokStatus::MarkingOverflow: return "tokenizer: text too long after marking special runs";
    case TokStatus::SegmentOverflow: return "tokenizer: segmentation ran out of room";
    default: return "";
    }
}

void put_status(TokStatus s, char *error, size_t cap) {
    if (s != TokStatus::Ok && error && cap) snprintf(error, cap, "%s", status_text(s));
}

// A whole file mapped read-only; unmapped with the object.
class MappedFile {
  public:
    MappedFile() = default;
    MappedFile(const MappedFile &) = delete;
    MappedFile &operator=(const MappedFile &) = delete;
    ~MappedFile() {
        if (data_) munmap(const_cast<char *>(data_), size_);
    }
    bool map(const char *path) {
        if (!path) return false;
        const int fd = open(path, O_RDONLY | O_CLOEXEC);
        if (fd < 0) return false;
        struct stat st;
        void *m = MAP_FAILED;
        if (fstat(fd, &st) == 0 && st.st_size > 0)
            m = mmap(nullptr, static_cast<size_t>(st.st_size), PROT_READ, MAP_PRIVATE, fd, 0);
        close(fd);
        if (m == MAP_FAILED) return false;
        data_ = static_cast<const char *>(m);
        size_ = static_cast<size_t>(st.st_size);
        return true;
    }
    const char *begin() const { return data_; }
    const char *end() const { return data_ + size_; }

  private:
    const char *data_ = nullptr;
    size_t size_ = 0;
};

}  // namespace

struct plamo_tokenizer {
    MappedFile file;
    std::vector<plamo_trie_node> nodes;
    std::vector<uint32_t> first_scalar;  // direct index of the trie's first level
    plamo_trie trie{};
    uint32_t byte_ids[256] = {};
    std::vector<const char *> row_start;  // PLAMO_VOCAB_ROWS starts, then the end of the last row
    // Request buffers.
    std::vector<uint32_t> scalars, text, special, marked, ids;
    std::vector<uint8_t> flags;
    std::vector<int64_t> costs;
    std::vector<plamo_unigram_path> paths;
    std::vector<plamo_candidate> candidates;
    std::vector<char> wrapped, piece;

    TokStatus load(const char *path);
    TokStatus index_rows();
    TokStatus scalars_of(const char *utf8, uint64_t *count);
    TokStatus encode(const char *utf8, unsigned direction, uint64_t *count);
};

TokStatus plamo_tokenizer::load(const char *path) {
    if (!file.map(path)) return TokStatus::Unreadable;
    try {
        nodes.assign(kTrieNodes, plamo_trie_node{});
        first_scalar.assign(kScalarLimit, 0);
        scalars.resize(kMaxScalars);
        text.resize(kMaxScalars);
        special.resize(kTempCapacity);
        marked.resize(kMarkedCapacity);
        ids.resize(kMaxIds);
        flags.resize(kTempCapacity + 1);
        costs.resize(kMarkedCapacity + 1);
        paths.resize(kMarkedCapacity);
        candidates.resize(kCandidates);
        wrapped.resize(kTextBytes);
        piece.resize(kTextBytes);
        row_start.reserve(PLAMO_VOCAB_ROWS + 2);
    } catch (const std::bad_alloc &) {
        return TokStatus::NoMemory;
    }
    trie = plamo_trie{nodes.data(), kTrieNodes, 1, first_scalar.data()};
    if (plamo_vocab_load(file.begin(), file.end(), &trie, scalars.data(), kMaxScalars, byte_ids) != PLAMO_VOCAB_ROWS)
        return TokStatus::BadRows;
    return index_rows();
}

// Row i spans [row_start[i], row_start[i + 1]); a final row may lack its
// line break.
TokStatus plamo_tokenizer::index_rows() {
    const char *p = file.begin(), *end = file.end();
    row_start.push_back(p);
    while (p < end && row_start.size() <= PLAMO_VOCAB_ROWS) {
        const void *nl = memchr(p, '\n', static_cast<size_t>(end - p));
        if (!nl) break;
        p = static_cast<const char *>(nl) + 1;
        row_start.push_back(p);
    }
    if (row_start.back() != end) row_start.push_back(end);
    return row_start.size() == PLAMO_VOCAB_ROWS + 1 ? TokStatus::Ok : TokStatus::BadLineBreaks;
}

TokStatus plamo_tokenizer::scalars_of(const char *utf8, uint64_t *count) {
    const char *end = utf8 + strlen(utf8);
    uint64_t n = 0;
    for (const char *p = utf8; p < end; ++n) {
        plamo_scalar sc;
        if (n == kMaxScalars || !plamo_utf8_next(p, end, &sc)) return TokStatus::BadText;
        text[n] = static_cast<uint32_t>(sc.cp);
        p = sc.next;
    }
    *count = n;
    return TokStatus::Ok;
}

// Direction 1 wraps the text for English -> Japanese, 2 for Japanese ->
// English, 0 encodes it as given; then scalars, special/repeat marking and
// the Unigram segmentation.
TokStatus plamo_tokenizer::encode(const char *utf8, unsigned direction, uint64_t *count) {
    if (direction > 2) return TokStatus::BadDirection;
    const char *source = utf8;
    if (direction != 0) {
        const char *from = direction == 1 ? "en" : "ja", *to = direction == 1 ? "ja" : "en";
        if (plamo_translation_prompt(utf8, from, to, wrapped.data(), wrapped.size()) == kFail)
            return TokStatus::PromptTooLong;
        source = wrapped.data();
    }
    uint64_t n = 0;
    if (const TokStatus st = scalars_of(source, &n); st != TokStatus::Ok) return st;
    const plamo_preprocess_args marking{text.data(),    n,        special.data(), kTempCapacity,
                                        marked.data(), kMarkedCapacity, flags.data()};
    const uint64_t width = plamo_preprocess(&marking);
    if (width == kFail) return TokStatus::MarkingOverflow;
    const plamo_encoder seg{&trie,        marked.data(),     width,       byte_ids, costs.data(),
                            paths.data(), candidates.data(), kCandidates, ids.data(), kMaxIds};
    const uint64_t produced = plamo_encode_marked(&seg);
    if (produced == kFail) return TokStatus::SegmentOverflow;
    *count = produced;
    return TokStatus::Ok;
}

extern "C" {

struct plamo_tokenizer *plamo_tokenizer_open(const char *path, char *error, size_t cap) {
    std::unique_ptr<plamo_tokenizer> t(new (std::nothrow) plamo_tokenizer());
    const TokStatus st = t ? t->load(path) : TokStatus::NoMemory;
    if (st != TokStatus::Ok) {
        put_status(st, error, cap);
        return nullptr;
    }
    return t.release();
}

void plamo_tokenizer_close(struct plamo_tokenizer *t) { delete t; }

uint64_t plamo_tokenizer_encode(struct plamo_tokenizer *t, const char *text, unsigned direction,
                                const uint32_t **ids, char *error, size_t cap) {
    uint64_t n = 0;
    const TokStatus st = (!t || !text || !ids) ? TokStatus::BadArguments : t->encode(text, direction, &n);
    if (st != TokStatus::Ok) {
        put_status(st, error, cap);
        return kFail;
    }
    *ids = t->ids.data();
    return n;
}

uint64_t plamo_tokenizer_prefix(struct plamo_tokenizer *t, unsigned direction, const uint32_t **ids, char *error,
                                size_t cap) {
    // The template's fixed head up to the source language (0: English source,
    // 1: Japanese source), encoded as plain text.
    if (!t || !ids || direction > 1) return kFail;
    if (plamo_translation_prefix(direction == 0 ? "en" : "ja", t->wrapped.data(), t->wrapped.size()) == kFail)
        return kFail;
    uint64_t n = 0;
    const TokStatus st = t->encode(t->wrapped.data(), 0, &n);
    if (st != TokStatus::Ok) {
        put_status(st, error, cap);
        return kFail;
    }
    *ids = t->ids.data();
    return n;
}

uint64_t plamo_tokenizer_decode(struct plamo_tokenizer *t, uint32_t id, const char **bytes) {
    if (!t || id >= PLAMO_VOCAB_ROWS) return kFail;
    const uint64_t n = plamo_decode_token(t->row_start[id], t->row_start[id + 1], 0, t->piece.data(), t->piece.size(),
                                          t->scalars.data(), t->scalars.size());
    if (n != kFail && bytes) *bytes = t->piece.data();
    return n;
}

}  // extern "C"
