// ref_blob_tool.cpp — drives the reference's own .m27b reader and writer
// (src/mono27b_blob.cpp, compiled in place from the reference checkout by
// oracle/build.py into oracle/_ref/ref_blob_tool).  Test infrastructure: the
// CPU tests use it to check that blobs written by m27b_blob_pack pass the
// reference's validation and read back entry for entry, and that a blob the
// reference writes opens with m27b_blob_open.
//
//   ref_blob_tool validate PATH   mono27b_validate_blob_file, then
//                                 mono27b_read_weights_section: prints "valid"
//                                 and one line per entry (name type source
//                                 role row_elems row_count data_offset
//                                 data_bytes), or "invalid: <message>"
//   ref_blob_tool write PATH      mono27b_write_stub_blob of a fixed small
//                                 set of entries (payload byte i = i * 7 + 3
//                                 mod 256), printing the same entry lines
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

#include "mono27b_format.h"

static void print_entry(const Mono27BWeightEntry &e) {
    std::printf("%s %u %u %u %u %u %llu %llu\n", e.name, e.ggml_type, e.source_model, e.role, e.row_elems, e.row_count,
                (unsigned long long)e.data_offset, (unsigned long long)e.data_bytes);
}

int main(int argc, char **argv) {
    if (argc != 3) {
        std::fprintf(stderr, "usage: ref_blob_tool validate|write PATH\n");
        return 2;
    }
    const std::string cmd = argv[1], path = argv[2];
    std::string err;
    if (cmd == "validate") {
        if (!mono27b_validate_blob_file(path, err)) {
            std::printf("invalid: %s\n", err.c_str());
            return 0;
        }
        Mono27BWeightsSection ws{};
        std::vector<Mono27BWeightEntry> es(4096);
        if (!mono27b_read_weights_section(path, ws, es.data(), es.size(), err)) {
            std::printf("invalid: %s\n", err.c_str());
            return 0;
        }
        std::printf("valid %u\n", ws.entry_count);
        for (uint32_t i = 0; i < ws.entry_count && i < es.size(); ++i) print_entry(es[i]);
        return 0;
    }
    if (cmd == "write") {
        struct T { const char *name; uint32_t type, source, role, elems, rows; uint64_t bytes; };
        const T ts[] = {
            {"token_embd.weight", 12, MONO27B_SOURCE_TARGET, 0, 512, 3, 3 * 2 * 144},
            {"blk.0.ffn_down.weight", 14, MONO27B_SOURCE_TARGET, MONO27B_ROLE_TARGET_MATVEC, 512, 2, 2 * 2 * 210},
            {"output_norm.weight", 0, MONO27B_SOURCE_TARGET, 0, 512, 1, 512 * 4},
            {"output.weight", 14, MONO27B_SOURCE_TARGET, MONO27B_ROLE_TARGET_OUTPUT_HEAD, 256, 5, 5 * 210},
            {"blk.0.attn_q.weight", 8, MONO27B_SOURCE_DRAFT, MONO27B_ROLE_DRAFT_MATVEC, 64, 4, 4 * 2 * 34},
        };
        const uint32_t n = sizeof(ts) / sizeof(ts[0]);
        std::vector<Mono27BWeightEntry> es(n);
        uint64_t off = 0;
        for (uint32_t i = 0; i < n; ++i) {
            std::snprintf(es[i].name, sizeof(es[i].name), "%s", ts[i].name);
            es[i].ggml_type = ts[i].type;
            es[i].source_model = ts[i].source;
            es[i].role = ts[i].role;
            es[i].row_elems = ts[i].elems;
            es[i].row_count = ts[i].rows;
            es[i].data_bytes = ts[i].bytes;
            off += ts[i].bytes;
        }
        // data offsets are relative to the weights section (reference blob.cpp:241)
        const uint64_t payload0 = sizeof(Mono27BWeightsSection) + (uint64_t)n * sizeof(Mono27BWeightEntry);
        uint64_t at = payload0;
        for (auto &e : es) {
            e.data_offset = at;
            at += e.data_bytes;
        }
        std::vector<unsigned char> payload(off);
        for (size_t i = 0; i < payload.size(); ++i) payload[i] = (unsigned char)((i * 7 + 3) & 0xff);
        Mono27BTokenizerSection tk{};
        tk.vocab_size = 1000;
        const unsigned char tok_bytes[8] = {1, 2, 3, 4, 5, 6, 7, 8};
        Mono27BWeightsSection ws{};
        ws.entry_count = n;
        if (!mono27b_write_stub_blob(path, 4096, tk, tok_bytes, sizeof(tok_bytes), ws, es.data(), payload.data(),
                                     payload.size(), err)) {
            std::printf("error: %s\n", err.c_str());
            return 1;
        }
        std::printf("written %u\n", n);
        for (const auto &e : es) print_entry(e);
        return 0;
    }
    return 2;
}
