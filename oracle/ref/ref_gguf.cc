// ref_gguf.cc -- a C entry layer over the REFERENCE's own GGUF reader.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile (target `gguf`) compiles this
// file with the reference's unmodified src/gguf.cc (read in place) into
// oracle/_ref/libref_gguf.so.  tests/test_gguf.py uses it to check that the
// library's GGUF parser (mlq_gguf_open) accepts and rejects the same files
// and reads the same tensor table and bytes as the reference.
//
// Functions wrapped (reference include/mini_llama/gguf.h):
//   GgufReader::load       gguf.h:80  (src/gguf.cc:396-575)
//   readGgufTensorRaw      gguf.h:94  (src/gguf.cc:614-662)
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "mini_llama/gguf.h"

using namespace mini_llama;

namespace {
struct Held {
    GgufReader r;
    std::string path;
    bool ok = false;
};
}  // namespace

extern "C" {

void* ref_gguf_open(const char* path) {
    Held* h = new Held();
    h->path = path;
    h->ok = h->r.load(path);
    return h;
}

int ref_gguf_ok(void* p) { return static_cast<Held*>(p)->ok ? 1 : 0; }

const char* ref_gguf_error(void* p) { return static_cast<Held*>(p)->r.load_error.c_str(); }

uint64_t ref_gguf_data_offset(void* p) { return static_cast<Held*>(p)->r.data_offset; }

int64_t ref_gguf_count(void* p) { return static_cast<int64_t>(static_cast<Held*>(p)->r.tensors.size()); }

// name (NUL-terminated, truncated to cap), dims (up to 8), type, offset.
int ref_gguf_tensor(void* p, int64_t i, char* name, int cap, uint64_t* dims, uint32_t* type, uint64_t* offset) {
    const auto& t = static_cast<Held*>(p)->r.tensors[static_cast<size_t>(i)];
    std::strncpy(name, t.name.c_str(), static_cast<size_t>(cap - 1));
    name[cap - 1] = 0;
    for (size_t d = 0; d < t.shape.size() && d < 8; ++d) dims[d] = t.shape[d];
    *type = t.type;
    *offset = t.offset;
    return static_cast<int>(t.shape.size());
}

// The tensor's bytes as the reference reads them; returns the byte count
// (0 on error or for a type the reference gives no size).
uint64_t ref_gguf_read(void* p, int64_t i, uint8_t* out, uint64_t cap) {
    Held* h = static_cast<Held*>(p);
    std::vector<uint8_t> raw = readGgufTensorRaw(h->path, h->r.tensors[static_cast<size_t>(i)], h->r.data_offset);
    if (raw.size() > cap) return 0;
    if (!raw.empty()) std::memcpy(out, raw.data(), raw.size());
    return raw.size();
}

void ref_gguf_free(void* p) { delete static_cast<Held*>(p); }

}  // extern "C"
