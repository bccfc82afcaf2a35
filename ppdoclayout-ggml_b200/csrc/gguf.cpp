// gguf.cpp — minimal GGUF reader (see gguf.h).
#include "gguf.h"

#include <cstdio>
#include <cstring>

namespace ppdl {

namespace {

struct Reader {
    FILE *f = nullptr;
    uint64_t size = 0;
    bool ok = true;

    bool raw(void *dst, size_t n) {
        if (!ok) return false;
        if (fread(dst, 1, n, f) != n) ok = false;
        return ok;
    }
    template <typename T> T get() {
        T v{};
        raw(&v, sizeof v);
        return v;
    }
    bool str(std::string *s) {
        const uint64_t n = get<uint64_t>();
        if (!ok || n > (1u << 20)) return ok = false;
        s->resize(n);
        return n == 0 || raw(&(*s)[0], n);
    }
    bool skip(uint64_t n) {
        if (!ok) return false;
        if (fseeko(f, (off_t)n, SEEK_CUR) != 0) ok = false;
        return ok;
    }
};

// GGUF value types
enum { T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 };

int scalar_size(uint32_t t) {
    switch (t) {
        case T_U8: case T_I8: case T_BOOL: return 1;
        case T_U16: case T_I16: return 2;
        case T_U32: case T_I32: case T_F32: return 4;
        case T_U64: case T_I64: case T_F64: return 8;
        default: return -1;
    }
}

bool skip_value(Reader &r, uint32_t t, int depth = 0) {
    if (t == T_STR) {
        std::string s;
        return r.str(&s);
    }
    if (t == T_ARR) {
        if (depth > 2) return false;
        const uint32_t et = r.get<uint32_t>();
        const uint64_t n = r.get<uint64_t>();
        if (!r.ok) return false;
        const int es = scalar_size(et);
        if (es > 0) return r.skip(n * (uint64_t)es);
        for (uint64_t i = 0; i < n; i++)
            if (!skip_value(r, et, depth + 1)) return false;
        return true;
    }
    const int s = scalar_size(t);
    return s > 0 && r.skip((uint64_t)s);
}

}  // namespace

bool gguf_read_header(const char *path, GgufFile *out, std::string *err) {
    Reader r;
    r.f = fopen(path, "rb");
    if (!r.f) {
        *err = std::string("cannot open ") + path;
        return false;
    }
    fseeko(r.f, 0, SEEK_END);
    r.size = (uint64_t)ftello(r.f);
    fseeko(r.f, 0, SEEK_SET);
    out->file_size = r.size;
    char magic[4];
    bool good = r.raw(magic, 4) && memcmp(magic, "GGUF", 4) == 0;
    if (!good) {
        *err = "not a GGUF file (bad magic)";
        fclose(r.f);
        return false;
    }
    out->version = r.get<uint32_t>();
    const uint64_t n_tensors = r.get<uint64_t>();
    const uint64_t n_kv = r.get<uint64_t>();
    if (!r.ok || out->version < 2 || out->version > 3 || n_tensors > 100000 || n_kv > 100000) {
        *err = "unsupported GGUF version or corrupt header";
        fclose(r.f);
        return false;
    }
    for (uint64_t i = 0; i < n_kv && r.ok; i++) {
        std::string key;
        if (!r.str(&key)) break;
        const uint32_t t = r.get<uint32_t>();
        if (key == "general.alignment" && t == T_U32) {
            out->alignment = r.get<uint32_t>();
        } else if (!skip_value(r, t)) {
            r.ok = false;
        }
    }
    if (!r.ok || out->alignment == 0 || (out->alignment & (out->alignment - 1))) {
        *err = "corrupt GGUF key/value section";
        fclose(r.f);
        return false;
    }
    out->tensors.resize(n_tensors);
    for (uint64_t i = 0; i < n_tensors && r.ok; i++) {
        GgufTensor &t = out->tensors[i];
        r.str(&t.name);
        t.n_dims = (int)r.get<uint32_t>();
        if (!r.ok || t.n_dims < 1 || t.n_dims > 4) {
            r.ok = false;
            break;
        }
        uint64_t nel = 1;
        for (int d = 0; d < t.n_dims; d++) {
            t.ne[d] = (int64_t)r.get<uint64_t>();
            if (t.ne[d] <= 0 || t.ne[d] > (1ll << 32)) r.ok = false;
            nel *= (uint64_t)(t.ne[d] > 0 ? t.ne[d] : 1);
        }
        t.type = r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        t.nbytes = nel * 4;
    }
    if (!r.ok) {
        *err = "corrupt or truncated GGUF tensor directory";
        fclose(r.f);
        return false;
    }
    const uint64_t pos = (uint64_t)ftello(r.f);
    out->data_offset = (pos + out->alignment - 1) / out->alignment * out->alignment;
    fclose(r.f);
    for (const GgufTensor &t : out->tensors) {
        if (t.type != 0) {
            *err = "tensor " + t.name + " is not F32 (this build reads F32 GGUF only)";
            return false;
        }
        if (out->data_offset + t.offset + t.nbytes > out->file_size) {
            *err = "tensor " + t.name + " runs past the end of the file (truncated GGUF)";
            return false;
        }
    }
    return true;
}

}  // namespace ppdl
