// blob.cpp — `.m27b` blob packer and reader (include/m27b_blob.h).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <vector>

#include "m27b_blob.h"

static_assert(sizeof(M27BBlobHeader) == 136, "blob header layout");
static_assert(sizeof(M27BBlobSection) == 24, "section descriptor layout");
static_assert(sizeof(M27BTokenizerSection) == 32, "tokenizer section layout");
static_assert(sizeof(M27BWeightsSection) == 16, "weights section layout");
static_assert(sizeof(M27BWeightEntry) == 104, "weight entry layout");

struct M27BBlob {
    int fd = -1;
    const uint8_t *map = nullptr;
    size_t size = 0;
    M27BBlobHeader header{};
    uint64_t weights_offset = 0, weights_bytes = 0;
    std::vector<M27BWeightEntry> entries;
};

namespace {

bool bfail(char *err, size_t cap, const char *fmt, ...) {
    if (err && cap) {
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(err, cap, fmt, ap);
        va_end(ap);
    }
    return false;
}

bool ok_msg(char *err, size_t cap) {
    if (err && cap) err[0] = '\0';
    return true;
}

void put_tag(char (&dst)[16], const char *src) {
    std::memset(dst, 0, sizeof(dst));
    if (src) std::strncpy(dst, src, sizeof(dst) - 1);
}

bool is_matrix_role(uint32_t role) {
    return role == M27B_ROLE_TARGET_MATVEC || role == M27B_ROLE_DRAFT_MATVEC || role == M27B_ROLE_OUTPUT_HEAD;
}

}  // namespace

extern "C" {

bool m27b_blob_pack(const char *path, const M27BPackInfo *info, const M27BPackTensor *tensors, size_t n, char *err,
                    size_t err_cap) {
    if (!path || !info || (!tensors && n)) return bfail(err, err_cap, "m27b_blob_pack: null argument");
    if (n == 0 || n > 0xffffffffu) return bfail(err, err_cap, "m27b_blob_pack: no tensors");
    // layout: header | 2 section descriptors | tokenizer | weights section | entries | payload
    const uint64_t sec_off = sizeof(M27BBlobHeader);
    const uint64_t tok_off = sec_off + 2 * sizeof(M27BBlobSection);
    const uint64_t tok_bytes = sizeof(M27BTokenizerSection);
    const uint64_t w_off = tok_off + tok_bytes;
    const uint64_t table_bytes = sizeof(M27BWeightsSection) + (uint64_t)n * sizeof(M27BWeightEntry);
    std::vector<M27BWeightEntry> entries(n);
    uint64_t rel = table_bytes;  // payload offsets relative to the weights section
    for (size_t i = 0; i < n; ++i) {
        const M27BPackTensor &t = tensors[i];
        if (!t.name || std::strlen(t.name) >= sizeof(entries[i].name))
            return bfail(err, err_cap, "m27b_blob_pack: tensor %zu: name missing or longer than 63 bytes", i);
        if (!t.data || t.bytes == 0) return bfail(err, err_cap, "m27b_blob_pack: tensor %s: no data", t.name);
        if (is_matrix_role(t.role) && (t.row_elems == 0 || t.row_count == 0))
            return bfail(err, err_cap, "m27b_blob_pack: matrix %s needs row_elems and row_count", t.name);
        M27BWeightEntry &e = entries[i];
        std::memset(&e, 0, sizeof(e));
        std::strncpy(e.name, t.name, sizeof(e.name) - 1);
        e.ggml_type = t.ggml_type;
        e.source_model = t.source;
        e.role = t.role;
        e.row_elems = t.row_elems;
        e.row_count = t.row_count;
        e.data_offset = rel;
        e.data_bytes = t.bytes;
        rel += t.bytes;
    }
    M27BBlobHeader h;
    std::memset(&h, 0, sizeof(h));
    h.magic = M27B_BLOB_MAGIC;
    h.schema_version = M27B_BLOB_SCHEMA;
    h.section_count = 2;
    h.section_table_offset = sec_off;
    h.tokenizer_offset = tok_off;
    h.tokenizer_bytes = tok_bytes;
    h.file_bytes = w_off + rel;
    h.max_ctx_hint = info->max_ctx_hint;
    h.target_layers = info->target_layers;
    h.draft_layers = info->draft_layers;
    put_tag(h.target_arch, info->target_arch);
    put_tag(h.draft_arch, info->draft_arch);
    put_tag(h.target_quant, info->target_quant);
    put_tag(h.draft_quant, info->draft_quant);
    const M27BBlobSection secs[2] = {{M27B_SECTION_TOKENIZER, 0, tok_off, tok_bytes},
                                     {M27B_SECTION_WEIGHTS, 0, w_off, rel}};
    M27BTokenizerSection tok;
    std::memset(&tok, 0, sizeof(tok));
    tok.magic = M27B_TOKENIZER_MAGIC;
    tok.version = 1;
    tok.vocab_size = info->vocab_size;
    tok.bos_id = info->bos_id;
    tok.eos_id = info->eos_id;
    tok.im_start_id = info->im_start_id;
    tok.im_end_id = info->im_end_id;
    M27BWeightsSection ws;
    std::memset(&ws, 0, sizeof(ws));
    ws.magic = M27B_WEIGHTS_MAGIC;
    ws.version = 1;
    ws.entry_count = (uint32_t)n;

    FILE *fp = std::fopen(path, "wb");
    if (!fp) return bfail(err, err_cap, "m27b_blob_pack: cannot create %s", path);
    bool ok = std::fwrite(&h, sizeof(h), 1, fp) == 1 && std::fwrite(secs, sizeof(secs), 1, fp) == 1 &&
              std::fwrite(&tok, sizeof(tok), 1, fp) == 1 && std::fwrite(&ws, sizeof(ws), 1, fp) == 1 &&
              std::fwrite(entries.data(), sizeof(M27BWeightEntry), n, fp) == n;
    for (size_t i = 0; ok && i < n; ++i)
        ok = std::fwrite(tensors[i].data, 1, (size_t)tensors[i].bytes, fp) == tensors[i].bytes;
    ok = (std::fclose(fp) == 0) && ok;
    if (!ok) return bfail(err, err_cap, "m27b_blob_pack: write to %s failed", path);
    return ok_msg(err, err_cap);
}

bool m27b_blob_open(const char *path, M27BBlob **out, char *err, size_t err_cap) {
    if (!path || !out) return bfail(err, err_cap, "m27b_blob_open: null argument");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY);
    if (fd < 0) return bfail(err, err_cap, "m27b_blob_open: missing blob %s", path);
    struct stat st;
    if (::fstat(fd, &st) != 0 || st.st_size < (off_t)sizeof(M27BBlobHeader)) {
        ::close(fd);
        return bfail(err, err_cap, "m27b_blob_open: %s is smaller than a blob header", path);
    }
    const size_t size = (size_t)st.st_size;
    void *m = ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        ::close(fd);
        return bfail(err, err_cap, "m27b_blob_open: cannot map %s", path);
    }
    M27BBlob *b = new M27BBlob();
    b->fd = fd;
    b->map = (const uint8_t *)m;
    b->size = size;
    auto bad = [&](const char *fmt, const char *what) {
        char e2[384];
        std::snprintf(e2, sizeof(e2), fmt, what);
        m27b_blob_close(b);
        return bfail(err, err_cap, "m27b_blob_open: %s (%s)", e2, path);
    };
    std::memcpy(&b->header, b->map, sizeof(M27BBlobHeader));
    const M27BBlobHeader &h = b->header;
    if (h.magic != M27B_BLOB_MAGIC) return bad("%s", "bad magic");
    if (h.schema_version != M27B_BLOB_SCHEMA) return bad("%s", "schema mismatch");
    if (h.file_bytes != size) return bad("%s", "file size differs from the header");
    if (h.section_count < 2 || h.section_count > 16) return bad("%s", "bad section count");
    if (h.section_table_offset > size || h.section_count * sizeof(M27BBlobSection) > size - h.section_table_offset)
        return bad("%s", "section table out of bounds");
    if (h.tokenizer_offset == 0 || h.tokenizer_bytes < sizeof(M27BTokenizerSection) || h.tokenizer_offset > size ||
        h.tokenizer_bytes > size - h.tokenizer_offset)
        return bad("%s", "tokenizer section missing or out of bounds");
    bool have_tok = false, have_w = false;
    for (uint32_t i = 0; i < h.section_count; ++i) {
        M27BBlobSection s;
        std::memcpy(&s, b->map + h.section_table_offset + i * sizeof(M27BBlobSection), sizeof(s));
        if (s.offset > size || s.bytes > size - s.offset) return bad("%s", "section out of bounds");
        if (s.kind == M27B_SECTION_TOKENIZER) {
            if (s.offset != h.tokenizer_offset || s.bytes != h.tokenizer_bytes) return bad("%s", "tokenizer section mismatch");
            have_tok = true;
        } else if (s.kind == M27B_SECTION_WEIGHTS && !have_w) {
            b->weights_offset = s.offset;
            b->weights_bytes = s.bytes;
            have_w = true;
        }
    }
    if (!have_tok || !have_w) return bad("%s", "missing tokenizer or weights section");
    M27BTokenizerSection tok;
    std::memcpy(&tok, b->map + h.tokenizer_offset, sizeof(tok));
    if (tok.magic != M27B_TOKENIZER_MAGIC || tok.version != 1 || tok.vocab_size == 0)
        return bad("%s", "bad tokenizer section");
    if (b->weights_bytes < sizeof(M27BWeightsSection)) return bad("%s", "weights section too small");
    M27BWeightsSection ws;
    std::memcpy(&ws, b->map + b->weights_offset, sizeof(ws));
    if (ws.magic != M27B_WEIGHTS_MAGIC || ws.version != 1 || ws.entry_count == 0)
        return bad("%s", "bad weights section header");
    if ((uint64_t)ws.entry_count * sizeof(M27BWeightEntry) > b->weights_bytes - sizeof(M27BWeightsSection))
        return bad("%s", "entry table out of bounds");
    b->entries.resize(ws.entry_count);
    std::memcpy(b->entries.data(), b->map + b->weights_offset + sizeof(M27BWeightsSection),
                ws.entry_count * sizeof(M27BWeightEntry));
    bool target_mv = false, head = false;
    for (const M27BWeightEntry &e : b->entries) {
        if (std::memchr(e.name, 0, sizeof(e.name)) == nullptr) return bad("%s", "entry name not terminated");
        if (e.data_bytes == 0 || e.data_offset > b->weights_bytes || e.data_bytes > b->weights_bytes - e.data_offset)
            return bad("entry %s out of the weights section", e.name);
        if (is_matrix_role(e.role) && (e.row_elems == 0 || e.row_count == 0))
            return bad("matrix entry %s without shape", e.name);
        target_mv = target_mv || e.role == M27B_ROLE_TARGET_MATVEC;
        head = head || e.role == M27B_ROLE_OUTPUT_HEAD;
    }
    if (!target_mv) return bad("%s", "no target matvec entry");
    if (!head) return bad("%s", "no output head entry");
    *out = b;
    return ok_msg(err, err_cap);
}

const M27BBlobHeader *m27b_blob_header(const M27BBlob *b) { return b ? &b->header : nullptr; }

size_t m27b_blob_count(const M27BBlob *b) { return b ? b->entries.size() : 0; }

bool m27b_blob_entry(const M27BBlob *b, size_t i, M27BWeightEntry *entry, const void **data, char *err,
                     size_t err_cap) {
    if (!b || !entry) return bfail(err, err_cap, "m27b_blob_entry: null argument");
    if (i >= b->entries.size()) return bfail(err, err_cap, "m27b_blob_entry: index %zu of %zu", i, b->entries.size());
    *entry = b->entries[i];
    if (data) *data = b->map + b->weights_offset + b->entries[i].data_offset;
    return ok_msg(err, err_cap);
}

void m27b_blob_close(M27BBlob *b) {
    if (!b) return;
    if (b->map) ::munmap((void *)b->map, b->size);
    if (b->fd >= 0) ::close(b->fd);
    delete b;
}

}  // extern "C"
