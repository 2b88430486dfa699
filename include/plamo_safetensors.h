/* BF16 safetensors checkpoints on the host: map the shards, find and validate
   tensors, bind a weight schema to the mapped bytes. The entry points and
   records are the reference's (src/load.s, src/find.s, src/tensor.s,
   src/resolve.s, src/bind.s, src/io.s), so its loader tests link against them;
   the bound host addresses are what plamo_cuda_preload uploads to HBM.

   File layout: 8-byte little-endian header length n, n bytes of JSON
   {"__metadata__": {string: string}, name: {"dtype": "BF16", "shape": [..],
   "data_offsets": [begin, end]}, ...}, then the data. Only BF16 tensors of
   rank <= 4 are accepted; names are raw (unescaped) ASCII. */
#ifndef PLAMO_SAFETENSORS_H
#define PLAMO_SAFETENSORS_H
#include <stddef.h>
#include <stdint.h>

#include "plamo_model.h"

#ifdef __cplusplus
extern "C" {
#endif

/* reference tests/load.c:4-13 */
struct plamo_safetensors_view {
    const char *header;
    uint64_t header_size;
    const void *data;
    uint64_t data_size;
};
struct plamo_u64 {
    const char *next;
    uint64_t value;
};
/* reference tests/find.c:4-7 */
struct plamo_tensor {
    const uint16_t *data;
    uint64_t bytes, rank, dims[4], reserved;
};

/* Split a mapped file into header and data. 1, or 0 with the view cleared. */
int plamo_safetensors_view(const void *file, uint64_t size, struct plamo_safetensors_view *view);
/* Decimal unsigned integer at [begin, end): no sign, no leading zero, no
   overflow. 1 with next = the first byte after it, or 0 with {NULL, 0}. */
int plamo_parse_u64(const char *begin, const char *end, struct plamo_u64 *out);
/* Tensor `name` of a mapped file: 1 with its data pointer (inside the file),
   byte length and shape, or 0 with the result cleared (absent, not BF16,
   malformed header, or data outside the file). */
int plamo_find_tensor(const void *file, uint64_t size, const char *name, struct plamo_tensor *out);
/* First shard holding `name` with exactly this rank and shape: its data, or NULL. */
const uint16_t *plamo_resolve_weight(const struct plamo_mapping *shards, uint64_t count, const char *name,
                                     uint64_t rank, const uint64_t *dims);
/* Resolve every entry of a schema terminated by a NULL name into its slot.
   1, or 0 with every slot cleared. */
int plamo_bind_weights(const struct plamo_mapping *shards, uint64_t count, const struct plamo_weight_spec *schema);
/* Read-only mapping of a whole file (0 on failure: missing, empty, unreadable). */
int plamo_map_file(const char *path, struct plamo_mapping *out);
void plamo_unmap_file(struct plamo_mapping *mapping);

#ifdef __cplusplus
}
#endif
#endif
