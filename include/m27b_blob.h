/*
 * m27b_blob.h — the mono27b `.m27b` weight blob: packer and reader.
 *
 * The on-disk layout is the reference's (include/mono27b_format.h:7-84,
 * writer src/mono27b_blob.cpp:378-438, reader :181-258), restated here so a
 * blob written by either side reads on the other:
 *
 *   header (136 B) | section table (24 B each: tokenizer, weights) |
 *   tokenizer section (32 B + payload) | weights section (16 B) |
 *   entry table (104 B each) | raw GGUF block payload
 *
 * Entry data offsets are relative to the weights section's offset
 * (src/mono27b_blob.cpp:241).  Payload offsets are not aligned: readers copy
 * each tensor to aligned device memory (the engine loader does, and repacks
 * q6_K / q8_0 there).  The reference packer (mono27b_pack) is not in its
 * source tree; m27b_blob_pack writes the same layout from caller tensors.
 * The tokenizer section carries only its fixed fields here (the tokenizer is
 * outside this library's scope); the reference validator needs vocab_size > 0.
 *
 * Conventions as in m27b_qmv.h: bool + error buffer.
 */
#ifndef M27B_BLOB_H
#define M27B_BLOB_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#include "m27b_qmv.h"

#ifdef __cplusplus
extern "C" {
#endif

#define M27B_BLOB_MAGIC 0x4237324du      /* "M27B" */
#define M27B_BLOB_SCHEMA 4u
#define M27B_TOKENIZER_MAGIC 0x544b324du /* "M2KT" */
#define M27B_WEIGHTS_MAGIC 0x5754324du   /* "M2TW" */
#define M27B_SECTION_TOKENIZER 1u
#define M27B_SECTION_WEIGHTS 2u
#define M27B_SOURCE_TARGET 1u
#define M27B_SOURCE_DRAFT 2u
#define M27B_ROLE_TARGET_MATVEC 1u
#define M27B_ROLE_DRAFT_MATVEC 2u
#define M27B_ROLE_OUTPUT_HEAD 3u

typedef struct M27BBlobHeader {
    uint32_t magic, schema_version, section_count, reserved0;
    uint64_t file_bytes, tensor_table_offset, section_table_offset, tokenizer_offset, tokenizer_bytes;
    uint32_t max_ctx_hint, target_layers, draft_layers;
    char target_arch[16], draft_arch[16], target_quant[16], draft_quant[16];
} M27BBlobHeader;

typedef struct M27BBlobSection {
    uint32_t kind, reserved;
    uint64_t offset, bytes;
} M27BBlobSection;

typedef struct M27BTokenizerSection {
    uint32_t magic, version, vocab_size, merges_count, bos_id, eos_id, im_start_id, im_end_id;
} M27BTokenizerSection;

typedef struct M27BWeightsSection {
    uint32_t magic, version, entry_count, reserved;
} M27BWeightsSection;

typedef struct M27BWeightEntry {
    char name[64];
    uint32_t ggml_type, source_model, role, row_elems, row_count, reserved;
    uint64_t data_offset; /* from the weights section's offset */
    uint64_t data_bytes;
} M27BWeightEntry;

/* One tensor for the packer. */
typedef struct M27BPackTensor {
    const char *name;    /* GGUF name, < 64 bytes */
    uint32_t ggml_type;  /* 0 f32, 8 q8_0, 12 q4_K, 14 q6_K, ... */
    uint32_t source;     /* M27B_SOURCE_* */
    uint32_t role;       /* M27B_ROLE_* (0: not a matrix, e.g. a norm) */
    uint32_t row_elems, row_count;
    const void *data;    /* host bytes in GGUF layout */
    uint64_t bytes;
} M27BPackTensor;

/* Header fields the packer takes from the caller. */
typedef struct M27BPackInfo {
    uint32_t max_ctx_hint, target_layers, draft_layers;
    const char *target_arch, *draft_arch, *target_quant, *draft_quant; /* < 16 bytes each */
    uint32_t vocab_size, bos_id, eos_id, im_start_id, im_end_id;       /* tokenizer section fields */
} M27BPackInfo;

/* Write a blob of n tensors to `path` (tensor payloads in the given order). */
M27B_API bool m27b_blob_pack(const char *path, const M27BPackInfo *info, const M27BPackTensor *tensors, size_t n,
                             char *err, size_t err_cap);

typedef struct M27BBlob M27BBlob;

/* Map and validate a blob: magic, schema, file size, section and entry
 * bounds, matrix metadata, and at least one target-matvec and one
 * output-head entry (the reference's validation, src/mono27b_blob.cpp:26-132,
 * without its fixed layer-count and tag checks, which the caller can read
 * from the header). */
M27B_API bool m27b_blob_open(const char *path, M27BBlob **out, char *err, size_t err_cap);
M27B_API const M27BBlobHeader *m27b_blob_header(const M27BBlob *b);
M27B_API size_t m27b_blob_count(const M27BBlob *b);
/* Entry i and a pointer to its payload (inside the read-only mapping). */
M27B_API bool m27b_blob_entry(const M27BBlob *b, size_t i, M27BWeightEntry *entry, const void **data, char *err,
                              size_t err_cap);
M27B_API void m27b_blob_close(M27BBlob *b);

#ifdef __cplusplus
}
#endif

#endif /* M27B_BLOB_H */
