// gguf.h — minimal GGUF v2/v3 reader for the model loader.
//
// Replaces the reference's use of ggml's gguf_init_from_file + per-tensor
// fread (src/ppdoclayout.cpp:217-246).  Only what the loader needs: the
// tensor directory (name, ggml ne[], type, offset) and the data offset; the
// key/value section is parsed for the alignment and otherwise skipped.
#pragma once

#include <stdint.h>

#include <string>
#include <vector>

namespace ppdl {

struct GgufTensor {
    std::string name;
    int n_dims = 0;
    int64_t ne[4] = {1, 1, 1, 1};
    uint32_t type = 0;     // 0 = F32 (the only type this model uses)
    uint64_t offset = 0;   // relative to the data section
    uint64_t nbytes = 0;
};

struct GgufFile {
    uint32_t version = 0;
    uint64_t alignment = 32;
    uint64_t data_offset = 0;
    uint64_t file_size = 0;
    std::vector<GgufTensor> tensors;
};

// Parses the header of `path`.  Returns false and fills `err` on any
// malformed, truncated or unsupported content.
bool gguf_read_header(const char *path, GgufFile *out, std::string *err);

}  // namespace ppdl
