/* PLaMo-3 tokenizer on Linux: UTF-8 text -> token ids, ids -> bytes.
 *
 * The reference's tokenizer is AArch64 assembly for Darwin (reference
 * src/{utf8,string,json,score,vocab,vocab_load,trie,unigram,encode,marked,
 * boundary,preprocess,decode,prompt}.s) behind a small C API (reference
 * runtime/tokenizer.h). This library exports the same entry points with the
 * same records, so the engine links it unchanged and the reference's own
 * tokenizer tests build against it:
 *
 *   vocabulary  tokenizer.jsonl rows ["piece", score, "TYPE"], 107520 of them;
 *               scores are fixed-point (x 10000, at most 4 decimals, |s| <= 1000);
 *               BYTE rows "<0xHH>" give the byte-fallback ids, every other row
 *               goes into a Unicode trie;
 *   encoding    text -> Unicode scalars (strict UTF-8) -> U+EE00 segment
 *               markers around <|plamo:...|> specials and around runs of >= 2
 *               spaces or >= 4 equal characters (line feeds excepted) ->
 *               per segment, a backward dynamic program choosing pieces by
 *               score (ties: the longer piece, then the earlier candidate),
 *               with UTF-8 byte fallback (score -1000 x 10000) for characters
 *               no piece covers;
 *   prompts     direction 1 (en -> ja) / 2 (ja -> en) wraps the text in the
 *               PFML3 translation template before encoding.
 */
#ifndef PLAMO_TOKENIZER_H
#define PLAMO_TOKENIZER_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PLAMO_VOCAB_ROWS 107520u
#define PLAMO_SEGMENT_MARKER 0xee00u

/* ---- records (byte layouts of the reference's assembly interfaces) ---- */
struct plamo_scalar { /* one decoded UTF-8 scalar */
    const char *next;
    uint64_t cp;
};
struct plamo_json_token { /* restricted JSON lexer output */
    const char *next, *start;
    uint64_t length, value;
};
struct plamo_score { /* fixed-point score x 10000 */
    const char *next;
    int64_t value;
};
struct plamo_vocab_entry { /* one parsed vocabulary row */
    uint64_t length; /* Unicode scalars of the piece */
    int64_t score;
    uint64_t type; /* NORMAL 0, BYTE 1, CONTROL 2, UNKNOWN 3 */
};
struct plamo_trie_node {
    uint32_t cp, child, sibling;
    int32_t id, score;
    uint32_t terminal;
};
struct plamo_trie { /* node 0 is the root; used starts at 1; roots optional */
    struct plamo_trie_node *nodes;
    uint64_t capacity, used;
    uint32_t *roots; /* NULL or zeroed uint32[0x110000]: direct first-scalar index */
};
struct plamo_candidate {
    uint32_t length;
    int32_t id, score;
    uint32_t reserved;
};
struct plamo_unigram_path {
    int64_t cost, length, id;
};
struct plamo_encoder { /* plamo_encode_segment / plamo_encode_marked */
    struct plamo_trie *trie;
    const uint32_t *cp;
    uint64_t count;
    uint32_t *bytes;      /* byte-fallback ids [256] */
    int64_t *costs;       /* [count + 1] */
    void *paths;          /* struct plamo_unigram_path [count] */
    void *candidates;     /* struct plamo_candidate [capacity], one kept for the fallback */
    uint64_t capacity;
    uint32_t *out;
    uint64_t out_capacity;
};
struct plamo_preprocess_args {
    const uint32_t *in;
    uint64_t count;
    uint32_t *temp;
    uint64_t temp_capacity;
    uint32_t *out;
    uint64_t capacity;
    uint8_t *flags; /* >= max(count, temp_capacity) + 1 */
};

/* ---- pieces (the reference assembly entry points; UINT64_MAX = failure) ---- */
int plamo_utf8_next(const char *cursor, const char *end, struct plamo_scalar *out);
uint64_t plamo_byte_fallback(uint64_t cp, const uint32_t *byte_ids, uint32_t *out);
int plamo_json_next(const char *cursor, const char *end, struct plamo_json_token *out);
uint64_t plamo_json_string(const char *start, const char *end, uint32_t *out, uint64_t capacity);
int plamo_parse_score(const char *cursor, const char *end, struct plamo_score *out);
int plamo_vocab_row(const char *start, const char *end, uint32_t *cp, uint64_t capacity,
                    struct plamo_vocab_entry *out);
uint64_t plamo_vocab_load(const char *start, const char *end, struct plamo_trie *trie, uint32_t *scratch,
                          uint64_t scratch_capacity, uint32_t *byte_ids);
int plamo_trie_insert(struct plamo_trie *trie, const uint32_t *cp, uint64_t length, int32_t id, int32_t score);
uint64_t plamo_trie_match(const struct plamo_trie *trie, const uint32_t *cp, uint64_t available,
                          struct plamo_candidate *out, uint64_t capacity);
int plamo_unigram_step(const int64_t *costs, const struct plamo_candidate *candidates, uint64_t count,
                       uint64_t available, struct plamo_unigram_path *out);
uint64_t plamo_encode_segment(const struct plamo_encoder *encoder);
uint64_t plamo_encode_marked(const struct plamo_encoder *encoder);
void plamo_repeat_boundaries(const uint32_t *cp, uint64_t count, uint8_t *flags);
void plamo_special_boundaries(const uint32_t *cp, uint64_t count, uint8_t *flags);
uint64_t plamo_preprocess(const struct plamo_preprocess_args *args);
uint64_t plamo_decode_token(const char *vocab, const char *end, uint64_t id, char *out, uint64_t capacity,
                            uint32_t *scratch, uint64_t scratch_capacity);
uint64_t plamo_translation_prompt(const char *text, const char *source, const char *target, char *out,
                                  uint64_t capacity);
uint64_t plamo_translation_prefix(const char *source, char *out, uint64_t capacity);

/* ---- the engine's API (reference runtime/tokenizer.h) ---- */
struct plamo_tokenizer;
struct plamo_tokenizer *plamo_tokenizer_open(const char *path, char *error, size_t cap);
void plamo_tokenizer_close(struct plamo_tokenizer *);
/* direction: 0 raw, 1 English to Japanese, 2 Japanese to English. Ids are
   borrowed until the next call on this tokenizer. */
uint64_t plamo_tokenizer_encode(struct plamo_tokenizer *, const char *text, unsigned direction,
                                const uint32_t **ids, char *error, size_t cap);
/* Fixed input prefix: direction 0 selects English, 1 selects Japanese. */
uint64_t plamo_tokenizer_prefix(struct plamo_tokenizer *, unsigned direction, const uint32_t **ids, char *error,
                                size_t cap);
uint64_t plamo_tokenizer_decode(struct plamo_tokenizer *, uint32_t id, const char **bytes);

#ifdef __cplusplus
#define PLAMO_TOKENIZER_ASSERT static_assert
#else
#define PLAMO_TOKENIZER_ASSERT _Static_assert
#endif
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_scalar) == 16, "UTF-8 result ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_json_token) == 32, "JSON token ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_score) == 16, "score ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_vocab_entry) == 24, "vocabulary row ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_trie_node) == 24, "trie node ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_trie) == 32, "trie ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_candidate) == 16, "candidate ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_unigram_path) == 24, "unigram path ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_encoder) == 80, "encoder ABI");
PLAMO_TOKENIZER_ASSERT(sizeof(struct plamo_preprocess_args) == 56, "preprocess ABI");

#ifdef __cplusplus
}
#endif
#endif
