// mlq_gguf.cu -- GGUF (v3) block ingestion straight to device memory.
//
// Replaces the weight path of the reference's GGUF loader: GgufReader::load
// (src/gguf.cc:396-575: header, metadata, tensor table, data offset and
// bounds checks), readGgufTensorRaw (src/gguf.cc:614-662) and
// loadQuantizedTensor (src/gguf_loader.cc:118-196), which read each tensor
// into host vectors before cuda_weight_upload.cc copies them to the GPU.
// Here a tensor's blocks go from the file to device memory in one pass
// through two pinned staging buffers (the read of one chunk overlaps the
// host-to-device copy of the previous one), and only the rows a rank owns
// are read: a row range of a quantized matrix is a contiguous byte range of
// the file, so a sharded rank loads its shard at load time and never holds
// the rest.  Host code only; no kernels.
//
// The format, as the reference reads it: "GGUF", u32 version (3), u64
// tensor count, u64 metadata count; metadata = (string key, u32 type,
// value), strings = u64 length + bytes, arrays = u32 element type + u64
// count + elements; tensor info = (string name, u32 n_dims, u64 dims[n_dims]
// fastest first, u32 ggml type, u64 offset); the data section starts at the
// next multiple of general.alignment (default 32).  Limits and checks are
// the reference's (same error cases; messages in this library's words).
#include <cuda_runtime.h>
#include <fcntl.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstdint>
#include <cstring>
#include <limits>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "mlq.h"
#include "mlq_kernels.h"

namespace {

constexpr uint64_t kDefaultAlignment = 32;
constexpr uint64_t kMaxAlignment = 1u << 20;
constexpr uint64_t kMaxStringBytes = 16u << 20;
constexpr uint64_t kMaxMetadata = 1000000;
constexpr uint64_t kMaxTensors = 1000000;
constexpr uint64_t kMaxArray = 10000000;
constexpr uint32_t kMaxDims = 8;

// GGUF value types
enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7,
    kString = 8, kArray = 9, kU64 = 10, kI64 = 11, kF64 = 12,
};

mlq_status gguf_fail(mlq_status st, const std::string& msg) {
    mlq::set_last_error(msg);  // read back through mlq_last_error()
    return st;
}

bool mul_ok(uint64_t a, uint64_t b, uint64_t* out) {
    if (a != 0 && b > std::numeric_limits<uint64_t>::max() / a) return false;
    *out = a * b;
    return true;
}

bool add_ok(uint64_t a, uint64_t b, uint64_t* out) {
    if (b > std::numeric_limits<uint64_t>::max() - a) return false;
    *out = a + b;
    return true;
}

// Buffered little-endian reader over a file descriptor.
class Reader {
   public:
    explicit Reader(int fd) : fd_(fd) {}
    bool bytes(void* dst, size_t n) {
        uint8_t* d = static_cast<uint8_t*>(dst);
        while (n > 0) {
            if (pos_ == len_) {
                const ssize_t r = ::pread(fd_, buf_, sizeof(buf_), (off_t)file_pos_);
                if (r <= 0) return false;
                len_ = (size_t)r;
                pos_ = 0;
                file_pos_ += (uint64_t)r;
            }
            const size_t k = n < len_ - pos_ ? n : len_ - pos_;
            std::memcpy(d, buf_ + pos_, k);
            pos_ += k;
            d += k;
            n -= k;
        }
        return true;
    }
    template <typename T>
    bool le(T* v) {
        return bytes(v, sizeof(T));
    }
    bool string(std::string* s) {
        uint64_t n = 0;
        if (!le(&n) || n > kMaxStringBytes) return false;
        s->resize(n);
        return n == 0 || bytes(&(*s)[0], n);
    }
    bool skip(uint64_t n) {
        uint8_t tmp[256];
        while (n > 0) {
            const size_t k = n < sizeof(tmp) ? (size_t)n : sizeof(tmp);
            if (!bytes(tmp, k)) return false;
            n -= k;
        }
        return true;
    }
    uint64_t tell() const { return file_pos_ - (len_ - pos_); }

   private:
    int fd_;
    uint8_t buf_[1 << 16];
    size_t pos_ = 0, len_ = 0;
    uint64_t file_pos_ = 0;
};

size_t scalar_bytes(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

struct Meta {
    std::string key;
    uint32_t type = 0;
    bool has_int = false, has_float = false;
    int64_t i = 0;
    double f = 0.0;
};

// Reads one value of type t; scalars are kept (as integer / float), strings
// and arrays skipped.
bool read_value(Reader& r, uint32_t t, Meta* m, int depth) {
    if (t == kString) {
        std::string s;
        return r.string(&s);
    }
    if (t == kArray) {
        uint32_t et = 0;
        uint64_t n = 0;
        if (depth > 16 || !r.le(&et) || !r.le(&n) || n > kMaxArray) return false;
        if (et != kString && et != kArray) {
            const size_t b = scalar_bytes(et);
            uint64_t total = 0;
            return b != 0 && mul_ok(n, b, &total) && r.skip(total);
        }
        for (uint64_t k = 0; k < n; ++k)
            if (!read_value(r, et, nullptr, depth + 1)) return false;
        return true;
    }
    uint8_t v[8] = {};
    const size_t b = scalar_bytes(t);
    if (b == 0 || !r.bytes(v, b)) return false;
    if (!m) return true;
    switch (t) {
        case kU8: m->i = v[0]; break;
        case kI8: m->i = (int8_t)v[0]; break;
        case kBool: m->i = v[0] != 0; break;
        case kU16: { uint16_t x; std::memcpy(&x, v, 2); m->i = x; break; }
        case kI16: { int16_t x; std::memcpy(&x, v, 2); m->i = x; break; }
        case kU32: { uint32_t x; std::memcpy(&x, v, 4); m->i = x; break; }
        case kI32: { int32_t x; std::memcpy(&x, v, 4); m->i = x; break; }
        case kU64: { uint64_t x; std::memcpy(&x, v, 8); m->i = (int64_t)x; break; }
        case kI64: { int64_t x; std::memcpy(&x, v, 8); m->i = x; break; }
        case kF32: { float x; std::memcpy(&x, v, 4); m->f = x; m->has_float = true; return true; }
        case kF64: { double x; std::memcpy(&x, v, 8); m->f = x; m->has_float = true; return true; }
    }
    m->has_int = true;
    m->f = (double)m->i;
    return true;
}

// Data bytes of a tensor (the reference's tensorDataSize: f32, f16 and the
// three block formats, whose element count must be whole blocks); other
// types have no size here (0), as in the reference.
bool data_bytes(uint32_t type, const std::vector<uint64_t>& dims, uint64_t* out) {
    uint64_t n = 1;
    for (uint64_t d : dims)
        if (d == 0 || !mul_ok(n, d, &n)) return false;
    switch (type) {
        case 0: return mul_ok(n, 4, out);
        case 1: return mul_ok(n, 2, out);
        case MLQ_Q4_0: case MLQ_Q4_1: case MLQ_Q8_0:
            if (n % 32) return false;
            return mul_ok(n / 32, mlq_block_bytes((mlq_format)type), out);
        default: *out = 0; return true;
    }
}

}  // namespace

struct mlq_gguf {
    int fd = -1;
    uint32_t version = 0;
    uint64_t data_offset = 0, file_size = 0, alignment = kDefaultAlignment;
    std::vector<Meta> meta;
    struct Tensor {
        std::string name;
        std::vector<uint64_t> dims;
        uint32_t type = 0;
        uint64_t offset = 0, nbytes = 0;
    };
    std::vector<Tensor> tensors;
    std::unordered_map<std::string, int64_t> by_name;
};

namespace {

mlq_status parse(mlq_gguf* g) {
    Reader r(g->fd);
    char magic[4];
    if (!r.bytes(magic, 4) || std::memcmp(magic, "GGUF", 4) != 0) return gguf_fail(MLQ_ERR_FORMAT, "not a GGUF file (magic)");
    if (!r.le(&g->version)) return gguf_fail(MLQ_ERR_FORMAT, "truncated header (version)");
    if (g->version != 3) return gguf_fail(MLQ_ERR_FORMAT, "GGUF version " + std::to_string(g->version) + " (only 3)");
    uint64_t nt = 0, nm = 0;
    if (!r.le(&nt) || !r.le(&nm)) return gguf_fail(MLQ_ERR_FORMAT, "truncated header (counts)");
    if (nt > kMaxTensors) return gguf_fail(MLQ_ERR_RANGE, "too many tensors: " + std::to_string(nt));
    if (nm > kMaxMetadata) return gguf_fail(MLQ_ERR_RANGE, "too many metadata entries: " + std::to_string(nm));
    std::unordered_set<std::string> keys;
    g->meta.reserve(nm);
    for (uint64_t k = 0; k < nm; ++k) {
        Meta m;
        if (!r.string(&m.key)) return gguf_fail(MLQ_ERR_FORMAT, "metadata key " + std::to_string(k) + " unreadable");
        if (!keys.insert(m.key).second) return gguf_fail(MLQ_ERR_FORMAT, "metadata key repeated: " + m.key);
        if (!r.le(&m.type) || !read_value(r, m.type, &m, 0))
            return gguf_fail(MLQ_ERR_FORMAT, "metadata value unreadable: " + m.key);
        if (m.key == "general.alignment") {
            // the reference parses the value as a decimal integer: integer types only
            if (!m.has_int && m.has_float && m.f >= 1.0 && m.f <= (double)kMaxAlignment && m.f == (double)(int64_t)m.f) {
                m.has_int = true;  // an integral float, as the reference's decimal parse accepts
                m.i = (int64_t)m.f;
            }
            if (!m.has_int || m.i <= 0 || (uint64_t)m.i > kMaxAlignment || (m.i & (m.i - 1)) != 0)
                return gguf_fail(MLQ_ERR_FORMAT, "general.alignment is not a power of two <= 1 MiB");
            g->alignment = (uint64_t)m.i;
        }
        g->meta.push_back(std::move(m));
    }
    g->tensors.reserve(nt);
    for (uint64_t k = 0; k < nt; ++k) {
        mlq_gguf::Tensor t;
        uint32_t nd = 0;
        if (!r.string(&t.name)) return gguf_fail(MLQ_ERR_FORMAT, "tensor name " + std::to_string(k) + " unreadable");
        if (!r.le(&nd)) return gguf_fail(MLQ_ERR_FORMAT, "tensor dims unreadable: " + t.name);
        if (nd == 0 || nd > kMaxDims) return gguf_fail(MLQ_ERR_FORMAT, "tensor has " + std::to_string(nd) + " dims: " + t.name);
        t.dims.resize(nd);
        for (uint32_t d = 0; d < nd; ++d) {
            if (!r.le(&t.dims[d])) return gguf_fail(MLQ_ERR_FORMAT, "tensor shape unreadable: " + t.name);
            if (t.dims[d] == 0) return gguf_fail(MLQ_ERR_FORMAT, "tensor has a zero dimension: " + t.name);
        }
        if (!r.le(&t.type) || !r.le(&t.offset)) return gguf_fail(MLQ_ERR_FORMAT, "tensor type/offset unreadable: " + t.name);
        if (!g->by_name.emplace(t.name, (int64_t)g->tensors.size()).second)
            return gguf_fail(MLQ_ERR_FORMAT, "tensor name repeated: " + t.name);
        g->tensors.push_back(std::move(t));
    }
    g->data_offset = r.tell();
    g->data_offset += (g->alignment - g->data_offset % g->alignment) % g->alignment;
    struct stat sb;
    if (fstat(g->fd, &sb) != 0) return gguf_fail(MLQ_ERR_FORMAT, "cannot stat the file");
    g->file_size = (uint64_t)sb.st_size;
    if (g->file_size < g->data_offset) return gguf_fail(MLQ_ERR_FORMAT, "file ends before its data section");
    for (auto& t : g->tensors) {
        if (!data_bytes(t.type, t.dims, &t.nbytes)) return gguf_fail(MLQ_ERR_FORMAT, "tensor size invalid: " + t.name);
        if (t.nbytes == 0) continue;
        uint64_t beg = 0, end = 0;
        if (!add_ok(g->data_offset, t.offset, &beg) || !add_ok(beg, t.nbytes, &end))
            return gguf_fail(MLQ_ERR_FORMAT, "tensor range overflows: " + t.name);
        if (end > g->file_size) return gguf_fail(MLQ_ERR_FORMAT, "tensor data past the end of the file: " + t.name);
    }
    return MLQ_OK;
}

// Pinned staging of the uploads: two buffers per host thread, kept.
struct Staging {
    void* buf[2] = {nullptr, nullptr};
    cudaEvent_t done[2] = {nullptr, nullptr};
    int device = -1;
    ~Staging() {
        for (int k = 0; k < 2; ++k) {
            if (buf[k]) cudaFreeHost(buf[k]);
            if (done[k]) cudaEventDestroy(done[k]);
        }
    }
};

constexpr size_t kStageBytes = 8u << 20;

}  // namespace

extern "C" {

MLQ_API mlq_status mlq_gguf_open(const char* path, mlq_gguf** file) {
    try {
        if (!path || !file) return gguf_fail(MLQ_ERR_NULL, "mlq_gguf_open: null argument");
        *file = nullptr;
        mlq_gguf* g = new mlq_gguf();
        g->fd = ::open(path, O_RDONLY | O_CLOEXEC);
        if (g->fd < 0) {
            delete g;
            return gguf_fail(MLQ_ERR_FORMAT, std::string("cannot open ") + path);
        }
        const mlq_status st = parse(g);
        if (st != MLQ_OK) {
            ::close(g->fd);
            delete g;
            return st;
        }
        *file = g;
        return MLQ_OK;
    } catch (...) {
        return gguf_fail(MLQ_ERR_RANGE, "mlq_gguf_open: out of host memory");
    }
}

MLQ_API void mlq_gguf_close(mlq_gguf* file) {
    if (!file) return;
    if (file->fd >= 0) ::close(file->fd);
    delete file;
}

MLQ_API int64_t mlq_gguf_tensor_count(const mlq_gguf* file) { return file ? (int64_t)file->tensors.size() : -1; }

MLQ_API uint64_t mlq_gguf_data_offset(const mlq_gguf* file) { return file ? file->data_offset : 0; }

MLQ_API int64_t mlq_gguf_find(const mlq_gguf* file, const char* name) {
    if (!file || !name) return -1;
    auto it = file->by_name.find(name);
    return it == file->by_name.end() ? -1 : it->second;
}

MLQ_API mlq_status mlq_gguf_tensor_info(const mlq_gguf* file, int64_t index, mlq_gguf_tensor* info) {
    if (!file || !info) return gguf_fail(MLQ_ERR_NULL, "mlq_gguf_tensor_info: null argument");
    if (index < 0 || index >= (int64_t)file->tensors.size())
        return gguf_fail(MLQ_ERR_RANGE, "mlq_gguf_tensor_info: no tensor " + std::to_string(index));
    const auto& t = file->tensors[(size_t)index];
    std::memset(info, 0, sizeof(*info));
    info->name = t.name.c_str();
    info->n_dims = (int)t.dims.size();
    for (size_t d = 0; d < t.dims.size(); ++d) info->dims[d] = t.dims[d];
    info->type = t.type;
    info->offset = t.offset;
    info->nbytes = t.nbytes;
    info->rows = 1;
    for (size_t d = 1; d < t.dims.size(); ++d) info->rows *= t.dims[d];
    info->row_bytes = t.nbytes / info->rows;
    return MLQ_OK;
}

MLQ_API mlq_status mlq_gguf_metadata_int(const mlq_gguf* file, const char* key, int64_t* value) {
    if (!file || !key || !value) return gguf_fail(MLQ_ERR_NULL, "mlq_gguf_metadata_int: null argument");
    for (const auto& m : file->meta)
        if (m.key == key) {
            if (!m.has_int) return gguf_fail(MLQ_ERR_FORMAT, std::string("metadata ") + key + " is not an integer");
            *value = m.i;
            return MLQ_OK;
        }
    return gguf_fail(MLQ_ERR_RANGE, std::string("no metadata key ") + key);
}

MLQ_API mlq_status mlq_gguf_metadata_float(const mlq_gguf* file, const char* key, double* value) {
    if (!file || !key || !value) return gguf_fail(MLQ_ERR_NULL, "mlq_gguf_metadata_float: null argument");
    for (const auto& m : file->meta)
        if (m.key == key) {
            if (!m.has_int && !m.has_float) return gguf_fail(MLQ_ERR_FORMAT, std::string("metadata ") + key + " is not a number");
            *value = m.f;
            return MLQ_OK;
        }
    return gguf_fail(MLQ_ERR_RANGE, std::string("no metadata key ") + key);
}

MLQ_API mlq_status mlq_gguf_upload_rows(const mlq_gguf* file, int64_t index, int64_t row_begin, int64_t row_end,
                                        void* dst, size_t dst_bytes, int device, mlq_stream stream) {
    try {
        mlq_gguf_tensor ti;
        mlq_status st = mlq_gguf_tensor_info(file, index, &ti);
        if (st != MLQ_OK) return st;
        if (!dst) return gguf_fail(MLQ_ERR_NULL, "mlq_gguf_upload_rows: null destination");
        if (ti.nbytes == 0) return gguf_fail(MLQ_ERR_FORMAT, std::string("tensor of an unsupported type: ") + ti.name);
        if (row_begin < 0 || row_end < row_begin || (uint64_t)row_end > ti.rows)
            return gguf_fail(MLQ_ERR_RANGE, "mlq_gguf_upload_rows: rows outside the tensor");
        const uint64_t n = (uint64_t)(row_end - row_begin) * ti.row_bytes;
        if (dst_bytes < n)
            return gguf_fail(MLQ_ERR_RANGE, "mlq_gguf_upload_rows: destination holds " + std::to_string(dst_bytes) +
                                                " bytes, the rows need " + std::to_string(n));
        if (n == 0) return MLQ_OK;
        int count = 0;
        if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
            cudaGetLastError();
            return gguf_fail(MLQ_ERR_DEVICE, "mlq_gguf_upload_rows: no device " + std::to_string(device));
        }
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(device);
        thread_local Staging stg;
        cudaError_t e = cudaSuccess;
        if (stg.device != device) {
            stg.~Staging();
            new (&stg) Staging();
            for (int k = 0; k < 2 && e == cudaSuccess; ++k) {
                e = cudaHostAlloc(&stg.buf[k], kStageBytes, cudaHostAllocDefault);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&stg.done[k], cudaEventDisableTiming);
            }
            if (e != cudaSuccess) {
                cudaGetLastError();
                cudaSetDevice(prev);
                return gguf_fail(MLQ_ERR_CUDA, std::string("pinned staging: ") + cudaGetErrorString(e));
            }
            stg.device = device;
        }
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        uint64_t src = file->data_offset + ti.offset + (uint64_t)row_begin * ti.row_bytes;
        uint8_t* d = static_cast<uint8_t*>(dst);
        int k = 0;
        bool used[2] = {false, false};
        for (uint64_t done = 0; done < n && e == cudaSuccess; k ^= 1) {
            const size_t len = (size_t)(n - done < kStageBytes ? n - done : kStageBytes);
            // the buffer's previous copy must have left it before the next read
            if (used[k]) e = cudaEventSynchronize(stg.done[k]);
            if (e != cudaSuccess) break;
            size_t got = 0;
            while (got < len) {
                const ssize_t r = ::pread(file->fd, static_cast<uint8_t*>(stg.buf[k]) + got, len - got,
                                          (off_t)(src + done + got));
                if (r <= 0) {
                    cudaSetDevice(prev);
                    return gguf_fail(MLQ_ERR_FORMAT, std::string("read failed in tensor ") + ti.name);
                }
                got += (size_t)r;
            }
            e = cudaMemcpyAsync(d + done, stg.buf[k], len, cudaMemcpyHostToDevice, s);
            if (e == cudaSuccess) e = cudaEventRecord(stg.done[k], s);
            used[k] = true;
            done += len;
        }
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        cudaSetDevice(prev);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return gguf_fail(MLQ_ERR_CUDA, std::string("upload: ") + cudaGetErrorString(e));
        }
        return MLQ_OK;
    } catch (...) {
        return gguf_fail(MLQ_ERR_CUDA, "mlq_gguf_upload_rows: host exception");
    }
}

}  // extern "C"
