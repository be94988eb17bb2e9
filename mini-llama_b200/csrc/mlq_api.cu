// mlq_api.cu -- the C ABI of libmlq.so (declared in include/mlq.h).
//
// Host-side validation follows the reference's checks
// (src/cuda_quant.cu:188-227, 305-307, 342-345) and runs before any CUDA
// call, so a rejected call never touches the GPU.  Nothing here throws
// across the ABI: failures return an mlq_status and leave a message for
// mlq_last_error().
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "mlq.h"
#include "mlq_device.cuh"
#include "mlq_kernels.h"
#include "mlq_tmap.h"

// Device-side error flag, one per device context (see mlq_device_error).
__device__ int g_mlq_device_error = 0;

// Scratch of mlq_linear_noalloc: the split of x (and the partial sums) that
// its tensor-core GEMM calls read.  It lives in the module's own device memory
// (one copy per device context, created when the module loads), so that
// entry point never calls cudaMalloc/cudaFree.  Every call on a device uses
// this one array: a GEMM call rewrites the part it reads before reading it,
// so nothing in it has to start at zero, but two such calls whose kernels
// overlap in time (different streams, or host threads without stream order
// between them) race on it.
static_assert(MLQ_NOALLOC_SCRATCH_BYTES % 256 == 0, "scratch size");
static __device__ __align__(256) unsigned char g_mlq_noalloc_scratch[MLQ_NOALLOC_SCRATCH_BYTES];

namespace {

thread_local std::string t_last_error;

mlq_status fail(mlq_status st, const std::string& msg) {
    t_last_error = msg;
    return st;
}

mlq_status fail_cuda(const char* what, cudaError_t e) {
    cudaGetLastError();  // clear a sticky launch error so the next call starts clean
    return fail(MLQ_ERR_CUDA, std::string("CUDA error in ") + what + ": " + cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;
constexpr int kFlagBytes = 256;  // per-rank flag buffer of the sharded calls
constexpr int kDoneWord = 32;    // its CTA completion counter (own 128-B line)

// Device workspace of one stream (the bf16 hi/lo split of x for the GEMM).
struct Workspace {
    void* ptr = nullptr;
    size_t cap = 0;
};

struct DeviceState {
    std::once_flag once;
    cudaError_t init_err = cudaSuccess;
    int sm_count = 0;
    int smem_per_sm = 0;
    int* err_flag = nullptr;  // device address of g_mlq_device_error
    std::mutex ws_mu;
    std::map<cudaStream_t, Workspace> ws;  // one per stream: calls on a stream are ordered
    std::mutex host_mu;       // serialises the *_host entry points' staging
    float* x_stage = nullptr;
    float* y_stage = nullptr;
    size_t x_cap = 0, y_cap = 0;
    // mlq_linear_batch_host's download stream and its two events (created
    // on first use, kept): the y of a step's first part is copied back here
    // while the last rows of its largest product compute
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t part_done = nullptr, copies_done = nullptr;
};

DeviceState g_dev[kMaxDevices];

// Must be called with `dev` current.
DeviceState* device_state(int dev, mlq_status* st) {
    if (dev < 0 || dev >= kMaxDevices) {
        *st = fail(MLQ_ERR_DEVICE, "device id out of range");
        return nullptr;
    }
    DeviceState& s = g_dev[dev];
    std::call_once(s.once, [&] {
        cudaError_t e = cudaDeviceGetAttribute(&s.sm_count, cudaDevAttrMultiProcessorCount, dev);
        if (e == cudaSuccess)
            e = cudaDeviceGetAttribute(&s.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&s.err_flag), g_mlq_device_error);
        s.init_err = e;
    });
    if (s.init_err != cudaSuccess) {
        *st = fail_cuda("device setup", s.init_err);
        return nullptr;
    }
    return &s;
}

// Workspace of at least `bytes` for `stream`.  Growing it waits for the
// stream (the old buffer may still be read by queued kernels), so the first
// call with the largest shape on a stream should come before any stream
// capture.
mlq_status stream_workspace(DeviceState* ds, cudaStream_t stream, size_t bytes, void** out) {
    std::lock_guard<std::mutex> lock(ds->ws_mu);
    Workspace& w = ds->ws[stream];
    if (w.cap < bytes) {
        if (w.ptr) {
            cudaError_t e = cudaStreamSynchronize(stream);
            if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize (workspace)", e);
            cudaFree(w.ptr);
            w.ptr = nullptr;
            w.cap = 0;
        }
        size_t cap = bytes < (1u << 20) ? (1u << 20) : bytes;
        cudaError_t e = cudaMalloc(&w.ptr, cap);
        if (e != cudaSuccess) return fail_cuda("cudaMalloc (workspace)", e);
        w.cap = cap;
    }
    *out = w.ptr;
    return MLQ_OK;
}

bool known_format(int fmt) { return fmt == MLQ_Q8_0 || fmt == MLQ_Q4_0 || fmt == MLQ_Q4_1; }

const char* fmt_name(int fmt) {
    return fmt == MLQ_Q8_0 ? "Q80" : (fmt == MLQ_Q4_0 ? "Q40" : (fmt == MLQ_Q4_1 ? "Q41" : "?"));
}

// The reference's validateQuantLinearShape (src/cuda_quant.cu:198-227) plus
// its null-weight check (:305-307), in the same order.
mlq_status validate_linear(int fmt, const void* w, size_t block_count, int out, int in,
                           const void* x, int rows, const void* y, const char* caller) {
    if (!known_format(fmt)) return fail(MLQ_ERR_FORMAT, std::string(caller) + ": unknown block format");
    const std::string who = std::string(caller) + "(" + fmt_name(fmt) + ")";
    if (w == nullptr) return fail(MLQ_ERR_NULL, who + ": null weight pointer");
    if (in <= 0 || out <= 0 || rows <= 0)
        return fail(MLQ_ERR_EMPTY, who + ": empty tensors are not supported");
    if (x == nullptr || y == nullptr) return fail(MLQ_ERR_NULL, who + ": null input/output pointer");
    const size_t expected = mlq_block_count(out, in);
    if (block_count != expected)
        return fail(MLQ_ERR_BLOCK_COUNT, who + ": block count mismatch: expected " +
                                             std::to_string(expected) + ", got " +
                                             std::to_string(block_count));
    return MLQ_OK;
}

// Shard/gather description of one streaming call (a plain call is world 1).
struct Gather {
    int world = 1, rank = 0;
    int row_offset = 0;          // global row of the streamed rows' first row
    int y_stride = 0;            // total output features
    float* const* ys = nullptr;  // world output bases (plain call: &y)
    uint32_t* const* flags = nullptr;
    uint32_t epoch = 0;
    bool wait = true;  // false: publish the epoch only (a deferred wait follows)
};

bool streamable(int fmt, const void* w, const float* x, int in) {
    const int bpr = (in + mlq::kQK - 1) / mlq::kQK;
    const int gblocks = fmt == MLQ_Q4_1 ? 1 : 2;
    return reinterpret_cast<uintptr_t>(w) % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 &&
           bpr % gblocks == 0 && in % 4 == 0;
}

// What follows the product in one call: nothing, a bias add, or the SwiGLU
// of a gate/up pair (w being the gate).
struct Epilogue {
    const void* w2 = nullptr;     // up projection of a SwiGLU pair, or null
    const float* bias = nullptr;  // [out] added to every row, or null
};

// Streams `out` rows starting at w through the streaming GEMV, one launch
// per <= 8 rows of x.
mlq_status run_stream(int fmt, const void* w, int out, int in, const float* x, int rows,
                      const Gather& g, cudaStream_t stream, const Epilogue& ep = Epilogue(),
                      int pdl_mode = mlq::kPdlNormal) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
    mlq_status st = MLQ_OK;
    DeviceState* ds = device_state(dev, &st);
    if (!ds) return st;
    const int bpr = (in + mlq::kQK - 1) / mlq::kQK;
    const int gblocks = fmt == MLQ_Q4_1 ? 1 : 2;
    mlq::GemvArgs a{};
    a.w = static_cast<const uint8_t*>(w);
    a.w2 = static_cast<const uint8_t*>(ep.w2);
    a.bias = ep.bias;
    a.out = out;
    a.in = in;
    a.bpr = bpr;
    a.gpr = bpr / gblocks;
    a.ktiles = (a.gpr + 31) / 32;
    a.y_stride = g.y_stride;
    a.row_offset = g.row_offset;
    a.ny = g.world;
    a.row_bytes = (long long)bpr * mlq::block_bytes(fmt);
    a.total_bytes = a.row_bytes * out;
    a.err = ds->err_flag;
    a.rank = g.rank;
    a.epoch = g.epoch;
    a.pdl_mode = pdl_mode;
    if (g.world > 1) {
        for (int r = 0; r < g.world; ++r) a.peer_flags[r] = g.flags[r];
        a.local_flags = g.flags[g.rank];
        a.done_counter = reinterpret_cast<unsigned int*>(g.flags[g.rank] + kDoneWord);
        a.wait = g.wait ? 1 : 0;
    }
    for (int m0 = 0; m0 < rows;) {
        const int mt = mlq::gemv_tokens_per_pass(rows - m0);
        a.x = x + (long long)m0 * in;
        a.M = rows - m0 < mt ? rows - m0 : mt;
        for (int r = 0; r < g.world; ++r) a.ys[r] = g.ys[r] + (long long)m0 * g.y_stride;
        // only the last pass runs the cross-rank handshake: it is stream-ordered
        // after the earlier passes' stores
        a.world = (m0 + a.M >= rows) ? g.world : 1;
        e = mlq::launch_gemv_stream(fmt, a, mt, ds->sm_count, ds->smem_per_sm, stream);
        if (e != cudaSuccess) return fail_cuda("gemv_stream launch", e);
        m0 += a.M;
    }
    return MLQ_OK;
}

// Which kernel takes a call: the batched-decode GEMM for 3..32 rows of x,
// the tcgen05 GEMM (bf16 hi/lo) for larger calls by MLQ_GEMM_ROWS_RULE, the
// streaming GEMV otherwise (and the any-alignment GEMV for layouts the
// streaming kernel does not take).
enum class Route { kStream, kGeneric, kBgemm, kGemm };

bool bgemm_supported(int fmt, const void* w, int out, int in, int rows) {
    return mlq::bgemm_shape_ok(fmt, w, out, in, rows) && mlq::encode_fn() != nullptr;
}

Route route_of(int fmt, const void* w, const void* w2, int out, int in, const float* x, int rows) {
    if (bgemm_supported(fmt, w, out, in, rows) && (w2 == nullptr || bgemm_supported(fmt, w2, out, in, rows)))
        return Route::kBgemm;
    if (mlq::gemm_supported(fmt, w, out, in, rows) && (w2 == nullptr || mlq::gemm_supported(fmt, w2, out, in, rows)))
        return Route::kGemm;
    if (streamable(fmt, w, x, in) && (w2 == nullptr || streamable(fmt, w2, x, in))) return Route::kStream;
    return Route::kGeneric;
}

// The tensor-core and any-alignment routes of a call (`ws`: its workspace,
// laid out as the route needs, then -- pair -- the up projection's output).
mlq_status run_nonstream(Route rt, int fmt, const void* w, int out, int in, const float* x, int rows, float* y,
                         cudaStream_t stream, const Epilogue& ep, DeviceState* ds, void* ws, size_t wbytes,
                         int split) {
    float* u = ep.w2 ? reinterpret_cast<float*>(static_cast<char*>(ws) + wbytes) : nullptr;
    cudaError_t e = cudaSuccess;
    if (rt == Route::kBgemm) {
        if (ep.w2) {
            // the pair as one grouped launch: gate rows to y, up rows to u
            const uint8_t* wm[2] = {static_cast<const uint8_t*>(w), static_cast<const uint8_t*>(ep.w2)};
            float* ym[2] = {y, u};
            const int om[2] = {out, out};
            e = mlq::launch_bgemm_group(fmt, 2, wm, ym, om, nullptr, x, in, rows, ws, ds->sm_count, ds->err_flag,
                                        stream);
        } else {
            e = mlq::launch_bgemm(fmt, static_cast<const uint8_t*>(w), x, y, out, in, rows, ep.bias, ws,
                                  ds->sm_count, ds->err_flag, stream);
        }
        if (e != cudaSuccess) return fail_cuda("bgemm launch", e);
    } else if (rt == Route::kGemm) {
        // many rows of x: the tensor-core GEMM (bias in its store; a pair
        // runs it per matrix, then one SwiGLU pass)
        e = mlq::launch_gemm(fmt, static_cast<const uint8_t*>(w), x, y, out, in, rows, ep.bias, ws, split,
                             ds->sm_count, ds->err_flag, stream);
        if (e == cudaSuccess && ep.w2)
            e = mlq::launch_gemm(fmt, static_cast<const uint8_t*>(ep.w2), x, u, out, in, rows, nullptr, ws, split,
                                 ds->sm_count, ds->err_flag, stream);
        if (e != cudaSuccess) return fail_cuda("gemm launch", e);
    } else {
        // layouts the streaming kernel does not take: the any-alignment GEMV
        const int bpr = (in + mlq::kQK - 1) / mlq::kQK;
        e = mlq::launch_gemv_generic(fmt, static_cast<const uint8_t*>(w), x, y, out, in, rows, bpr, stream);
        if (e == cudaSuccess && ep.w2)
            e = mlq::launch_gemv_generic(fmt, static_cast<const uint8_t*>(ep.w2), x, u, out, in, rows, bpr, stream);
        if (e == cudaSuccess && ep.bias && !ep.w2) e = mlq::launch_add_bias(y, ep.bias, rows, out, stream);
        if (e != cudaSuccess) return fail_cuda("gemv_generic launch", e);
    }
    if (ep.w2) {
        e = mlq::launch_swiglu(y, u, (long long)rows * out, stream);
        if (e != cudaSuccess) return fail_cuda("swiglu launch", e);
    }
    return MLQ_OK;
}

mlq_status run_linear(int fmt, const void* w, int out, int in, const float* x, int rows, float* y,
                      cudaStream_t stream, const Epilogue& ep = Epilogue(), int pdl_mode = mlq::kPdlNormal) {
    const Route rt = route_of(fmt, w, ep.w2, out, in, x, rows);
    if (rt != Route::kStream) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
        mlq_status st = MLQ_OK;
        DeviceState* ds = device_state(dev, &st);
        if (!ds) return st;
        // workspace: the route's own (x split, scales, partial sums), 256-B
        // aligned, then (pair) the up projection's output
        int split = 1;
        size_t wb = 0;
        if (rt == Route::kBgemm) {
            const int om[2] = {out, out};
            wb = mlq::bgemm_group_workspace_bytes(fmt, in, rows, om, ep.w2 ? 2 : 1, ds->sm_count);
        } else if (rt == Route::kGemm) {
            split = mlq::gemm_split(out, in, rows, ds->sm_count);
            wb = mlq::gemm_workspace_bytes(in, rows, out, split);
        }
        wb = (wb + 255) & ~(size_t)255;
        const size_t ubytes = ep.w2 ? (size_t)rows * out * sizeof(float) : 0;
        void* ws = nullptr;
        if (wb + ubytes > 0) {
            st = stream_workspace(ds, stream, wb + ubytes, &ws);
            if (st != MLQ_OK) return st;
        }
        return run_nonstream(rt, fmt, w, out, in, x, rows, y, stream, ep, ds, ws, wb, split);
    }
    Gather g;
    g.y_stride = out;
    g.ys = &y;
    return run_stream(fmt, w, out, in, x, rows, g, stream, ep, pdl_mode);
}

// Device address of g_mlq_noalloc_scratch, looked up once per device (with
// that device current) and kept.
struct ScratchSlot {
    std::once_flag once;
    cudaError_t err = cudaSuccess;
    void* ptr = nullptr;
};

ScratchSlot g_scratch[kMaxDevices];

// mlq_linear without any device allocation.  The streaming and
// any-alignment GEMVs need no scratch, so the calls they take run as in
// mlq_linear; the tensor-core kernels read their x split (and partial sums)
// from the static array instead of the per-stream workspace.  A call that
// mlq_linear would give the batched-decode GEMM whose scratch does not fit
// the array runs the streaming GEMV (the bf16 GEMM's limit is checked by
// the caller before any CUDA call).
mlq_status run_linear_noalloc(int fmt, const void* w, int out, int in, const float* x, int rows,
                              float* y, cudaStream_t stream) {
    Route rt = route_of(fmt, w, nullptr, out, in, x, rows);
    if (rt == Route::kStream || rt == Route::kGeneric) return run_linear(fmt, w, out, in, x, rows, y, stream);
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
    mlq_status st = MLQ_OK;
    DeviceState* ds = device_state(dev, &st);
    if (!ds) return st;
    if (rt == Route::kBgemm &&
        mlq::bgemm_workspace_bytes(fmt, in, rows, out, ds->sm_count) > (size_t)MLQ_NOALLOC_SCRATCH_BYTES) {
        Gather g;
        g.y_stride = out;
        g.ys = &y;
        if (streamable(fmt, w, x, in)) return run_stream(fmt, w, out, in, x, rows, g, stream);
        return run_nonstream(Route::kGeneric, fmt, w, out, in, x, rows, y, stream, Epilogue(), ds, nullptr, 0, 1);
    }
    ScratchSlot& sl = g_scratch[dev];
    std::call_once(sl.once, [&] { sl.err = cudaGetSymbolAddress(&sl.ptr, g_mlq_noalloc_scratch); });
    if (sl.err != cudaSuccess || sl.ptr == nullptr)
        return fail_cuda("cudaGetSymbolAddress (static scratch)", sl.err != cudaSuccess ? sl.err : cudaErrorInvalidSymbol);
    int split = 1;
    if (rt == Route::kGemm) {
        // split-K as mlq_linear chooses it, lowered to the largest count whose
        // partial sums fit the scratch next to the x split (1 always fits: the
        // caller checked the x split against the scratch size)
        split = mlq::gemm_split(out, in, rows, ds->sm_count);
        while (split > 1 && mlq::gemm_workspace_bytes(in, rows, out, split) > (size_t)MLQ_NOALLOC_SCRATCH_BYTES)
            --split;
    }
    return run_nonstream(rt, fmt, w, out, in, x, rows, y, stream, Epilogue(), ds, sl.ptr, 0, split);
}

// Grows a per-device staging buffer (called under host_mu, device current).
mlq_status ensure(float** buf, size_t* cap, size_t bytes) {
    if (*cap >= bytes) return MLQ_OK;
    if (*buf) cudaFree(*buf);
    *buf = nullptr;
    *cap = 0;
    cudaError_t e = cudaMalloc(reinterpret_cast<void**>(buf), bytes);
    if (e != cudaSuccess) return fail_cuda("cudaMalloc (staging)", e);
    *cap = bytes;
    return MLQ_OK;
}

mlq_status set_device(int device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) return fail_cuda("cudaGetDeviceCount", e);
    if (device < 0 || device >= count)
        return fail(MLQ_ERR_DEVICE, "device id " + std::to_string(device) + " not present (" +
                                        std::to_string(count) + " devices)");
    e = cudaSetDevice(device);
    return e == cudaSuccess ? MLQ_OK : fail_cuda("cudaSetDevice", e);
}

// mlq_linear_allgather's checks (shard, peers, epoch), before any CUDA call.
mlq_status validate_gather(int fmt, const void* w_shard, size_t shard_block_count, int out_features,
                           int in_features, const float* x, int rows, const mlq_gather& g, const char* who) {
    if (!known_format(fmt)) return fail(MLQ_ERR_FORMAT, std::string(who) + ": unknown block format");
    if (in_features <= 0 || out_features <= 0 || rows <= 0)
        return fail(MLQ_ERR_EMPTY, std::string(who) + ": empty tensors are not supported");
    if (rows > 64) return fail(MLQ_ERR_RANGE, std::string(who) + ": at most 64 rows of x");
    if (g.world_size < 1 || g.world_size > mlq::kMaxWorld || g.rank < 0 || g.rank >= g.world_size)
        return fail(MLQ_ERR_COMM, std::string(who) + ": world_size must be 1..8 and 0 <= rank < world_size");
    if (g.row_begin < 0 || g.row_end < g.row_begin || g.row_end > out_features)
        return fail(MLQ_ERR_COMM, std::string(who) + ": row range outside [0, out_features]");
    if (g.epoch == 0) return fail(MLQ_ERR_COMM, std::string(who) + ": epoch starts at 1");
    if (g.defer_wait != 0 && g.defer_wait != 1) return fail(MLQ_ERR_COMM, std::string(who) + ": defer_wait must be 0 or 1");
    if (!x || !g.peer_y || !g.peer_flags) return fail(MLQ_ERR_NULL, std::string(who) + ": null pointer");
    for (int r = 0; r < g.world_size; ++r)
        if (!g.peer_y[r] || !g.peer_flags[r])
            return fail(MLQ_ERR_NULL, std::string(who) + ": null peer pointer for rank " + std::to_string(r));
    const int shard_rows = g.row_end - g.row_begin;
    const size_t expected = (size_t)shard_rows * (size_t)((in_features + mlq::kQK - 1) / mlq::kQK);
    if (shard_block_count != expected)
        return fail(MLQ_ERR_BLOCK_COUNT, std::string(who) + ": block count mismatch: expected " +
                                             std::to_string(expected) + ", got " +
                                             std::to_string(shard_block_count));
    if (shard_rows > 0 && !w_shard) return fail(MLQ_ERR_NULL, std::string(who) + ": null weight pointer");
    static const uint8_t kAligned[16] = {};
    const void* wcheck = shard_rows > 0 ? w_shard : kAligned;
    if (!streamable(fmt, wcheck, x, in_features) || reinterpret_cast<uintptr_t>(w_shard) % 16 != 0)
        return fail(MLQ_ERR_SHAPE, std::string(who) +
                                       ": needs 16-B aligned weights and x, an even block count per "
                                       "row (q8_0/q4_0) and in_features % 4 == 0");
    return MLQ_OK;
}

// The shard's product with the gather fused in (validated arguments): the
// batched-decode GEMM for the rows it takes, else the streaming GEMV; both
// store every value to each rank's y and end with the same epoch handshake.
mlq_status run_gather(int fmt, const void* w_shard, int out_features, int in_features, const float* x,
                      int rows, const float* bias, const mlq_gather& mg, cudaStream_t stream) {
    const int shard = mg.row_end - mg.row_begin;
    if (shard > 0 && bgemm_supported(fmt, w_shard, shard, in_features, rows)) {
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
        mlq_status st = MLQ_OK;
        DeviceState* ds = device_state(dev, &st);
        if (!ds) return st;
        void* ws = nullptr;
        st = stream_workspace(ds, stream, mlq::bgemm_workspace_bytes(fmt, in_features, rows, shard, ds->sm_count),
                              &ws);
        if (st != MLQ_OK) return st;
        mlq::BgemmGather bg;
        bg.world = mg.world_size;
        bg.rank = mg.rank;
        bg.row_offset = mg.row_begin;
        bg.y_stride = out_features;
        bg.epoch = mg.epoch;
        for (int r = 0; r < mg.world_size; ++r) {
            bg.ys[r] = mg.peer_y[r];
            bg.peer_flags[r] = mg.peer_flags[r];
        }
        bg.local_flags = mg.peer_flags[mg.rank];
        bg.done_counter = reinterpret_cast<unsigned int*>(mg.peer_flags[mg.rank] + kDoneWord);
        bg.wait = mg.defer_wait ? 0 : 1;
        e = mlq::launch_bgemm(fmt, static_cast<const uint8_t*>(w_shard), x, nullptr, shard, in_features, rows,
                              bias ? bias + mg.row_begin : nullptr, ws, ds->sm_count, ds->err_flag, stream, &bg);
        return e == cudaSuccess ? MLQ_OK : fail_cuda("bgemm launch", e);
    }
    Gather g;
    g.world = mg.world_size;
    g.rank = mg.rank;
    g.row_offset = mg.row_begin;
    g.y_stride = out_features;
    g.ys = mg.peer_y;
    g.flags = mg.peer_flags;
    g.epoch = mg.epoch;
    g.wait = !mg.defer_wait;
    Epilogue ep;
    ep.bias = bias;
    return run_stream(fmt, w_shard, mg.row_end - mg.row_begin, in_features, x, rows, g, stream, ep);
}

// One op of a batch: validation (no CUDA call) ...
mlq_status validate_op(const mlq_linear_op& op, int i, bool host) {
    const std::string who = std::string(host ? "mlq_linear_batch_host" : "mlq_linear_batch") + " op " +
                            std::to_string(i);
    if (op.gather) {
        if (op.w_up) return fail(MLQ_ERR_RANGE, who + ": a gathered op takes no up projection");
        if (host && !op.y) return fail(MLQ_ERR_NULL, who + ": null host y");
        return validate_gather(op.fmt, op.w, op.block_count, op.out_features, op.in_features, op.x, op.rows,
                               *op.gather, who.c_str());
    }
    mlq_status st = validate_linear(op.fmt, op.w, op.block_count, op.out_features, op.in_features, op.x,
                                    op.rows, op.y, who.c_str());
    if (st != MLQ_OK) return st;
    if (op.w_up && op.bias) return fail(MLQ_ERR_RANGE, who + ": a SwiGLU pair takes no bias");
    return MLQ_OK;
}

// ... and its launch (x, y: device pointers).
mlq_status run_op(const mlq_linear_op& op, const float* x, float* y, cudaStream_t stream) {
    if (op.gather)
        return run_gather(op.fmt, op.w, op.out_features, op.in_features, x, op.rows, op.bias, *op.gather, stream);
    Epilogue ep;
    ep.w2 = op.w_up;
    ep.bias = op.bias;
    return run_linear(op.fmt, op.w, op.out_features, op.in_features, x, op.rows, y, stream, ep);
}

// A batch op as a member of a run of one-row products (x, y: its device x
// and y).  A gathered op streams its shard's rows into every rank's y.
mlq::GemvRunOp run_op_of(const mlq_linear_op& op, const float* x, float* y) {
    mlq::GemvRunOp r;
    std::memset(&r, 0, sizeof(r));
    r.w = static_cast<const uint8_t*>(op.w);
    r.x = x;
    r.in = op.in_features;
    r.world = 1;
    if (!op.gather) {
        r.bias = op.bias;
        r.out = op.out_features;
        r.y[0] = y;
        r.ny = 1;
        return r;
    }
    const mlq_gather& g = *op.gather;
    r.out = g.row_end - g.row_begin;
    r.bias = op.bias ? op.bias + g.row_begin : nullptr;
    r.row_offset = g.row_begin;
    r.ny = g.world_size;
    for (int d = 0; d < g.world_size && d < mlq::kMaxWorld; ++d) r.y[d] = g.peer_y[d];
    if (g.world_size > 1) {
        r.world = g.world_size;
        r.rank = g.rank;
        for (int d = 0; d < g.world_size && d < mlq::kMaxWorld; ++d) r.flags[d] = g.peer_flags[d];
        r.done_counter = reinterpret_cast<unsigned int*>(g.peer_flags[g.rank] + kDoneWord);
        r.epoch = g.epoch;
        r.wait = g.defer_wait ? 0 : 1;
    }
    return r;
}

// A batch's ops in order.
//  * Consecutive plain ops that share x (the same device x, format,
//    in_features and rows) and all take the batched-decode GEMM run as one
//    grouped launch (up to kBgemmMaxGroup): Q, K and V of a layer read one x
//    (src/forward.cc:425-435).
//  * Consecutive ops that do not touch one another's outputs (no op's x,
//    bias or y overlaps an earlier op's y, no op's y overlaps an earlier
//    op's x) form a run.  A run of one-row ops of one format in the run
//    kernel's layout -- plain, bias or gathered (the gathered ones sharing
//    their flag words) -- takes one persistent launch per kGemvRunMaxOps ops
//    (launch_gemv_run; the launch publishes once for all its gathered ops).
//    Otherwise a run of ops that each take one streaming-GEMV launch goes
//    back to back: the first waits for the kernel before the batch, the
//    others read x at once, and a join launch closes the run, so what
//    follows sees every y.
// xs[i] / ys[i]: op i's device x and y.
mlq_status run_ops(const mlq_linear_op* ops, int n, const float* const* xs, float* const* ys, cudaStream_t stream) {
    auto groupable = [&](int i) {
        const mlq_linear_op& o = ops[i];
        return !o.gather && !o.w_up && route_of(o.fmt, o.w, nullptr, o.out_features, o.in_features, xs[i], o.rows) ==
                                           Route::kBgemm;
    };
    auto one_gemv = [&](int i) {
        const mlq_linear_op& o = ops[i];
        return !o.gather && o.rows <= mlq::gemv_tokens_per_pass(o.rows) &&
               route_of(o.fmt, o.w, o.w_up, o.out_features, o.in_features, xs[i], o.rows) == Route::kStream;
    };
    auto overlap = [](const void* a, size_t na, const void* b, size_t nb) {
        const uintptr_t pa = reinterpret_cast<uintptr_t>(a), pb = reinterpret_cast<uintptr_t>(b);
        return a && b && pa < pb + nb && pb < pa + na;
    };
    auto ybytes = [&](int i) { return (size_t)ops[i].rows * ops[i].out_features * sizeof(float); };
    auto xbytes = [&](int i) { return (size_t)ops[i].rows * ops[i].in_features * sizeof(float); };
    // op j may run without waiting for ops [i, j)
    auto independent = [&](int i, int j) {
        for (int k = i; k < j; ++k) {
            if (overlap(xs[j], xbytes(j), ys[k], ybytes(k)) || overlap(ys[j], ybytes(j), ys[k], ybytes(k)) ||
                overlap(ys[j], ybytes(j), xs[k], xbytes(k)) ||
                overlap(ops[j].bias, ops[j].out_features * sizeof(float), ys[k], ybytes(k)) ||
                overlap(ys[j], ybytes(j), ops[k].bias, ops[k].out_features * sizeof(float)))
                return false;
        }
        return true;
    };
    // op i can join a run launch
    auto run_member = [&](int i) {
        const mlq_linear_op& o = ops[i];
        if (o.rows != 1 || o.w_up) return false;
        if (!o.gather && route_of(o.fmt, o.w, nullptr, o.out_features, o.in_features, xs[i], 1) != Route::kStream)
            return false;
        return mlq::gemv_run_ok(o.fmt, run_op_of(o, xs[i], ys[i]));
    };
    // op j's gather (if any) matches the gathers of ops [i, j)
    auto run_compatible = [&](int i, int j) {
        const mlq::GemvRunOp b = run_op_of(ops[j], xs[j], ys[j]);
        for (int k = i; k < j; ++k)
            if (!mlq::gemv_run_compatible(run_op_of(ops[k], xs[k], ys[k]), b)) return false;
        return true;
    };
    for (int i = 0; i < n;) {
        // a run of independent one-row ops: one persistent launch per
        // kGemvRunMaxOps ops
        int r = i;
        if (run_member(i))
            for (r = i + 1; r < n && run_member(r) && ops[r].fmt == ops[i].fmt && independent(i, r) &&
                            run_compatible(i, r);
                 ++r) {
            }
        if (r - i >= 2) {
            int dev = 0;
            cudaError_t e = cudaGetDevice(&dev);
            if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
            mlq_status st = MLQ_OK;
            DeviceState* ds = device_state(dev, &st);
            if (!ds) return st;
            for (int k = i; k < r; k += mlq::kGemvRunMaxOps) {
                const int nk = r - k < mlq::kGemvRunMaxOps ? r - k : mlq::kGemvRunMaxOps;
                mlq::GemvRunOp run[mlq::kGemvRunMaxOps];
                for (int q = 0; q < nk; ++q) run[q] = run_op_of(ops[k + q], xs[k + q], ys[k + q]);
                void* ws = nullptr;
                st = stream_workspace(ds, stream, mlq::gemv_run_workspace_bytes(ops[i].fmt, run, nk), &ws);
                if (st != MLQ_OK) return st;
                e = mlq::launch_gemv_run(ops[i].fmt, run, nk, ws, ds->sm_count, ds->smem_per_sm, ds->err_flag,
                                         stream);
                if (e != cudaSuccess) return fail_cuda("gemv run launch", e);
            }
            i = r;
            continue;
        }
        // a run of independent one-launch GEMVs
        r = i;
        if (one_gemv(i))
            for (r = i + 1; r < n && one_gemv(r) && independent(i, r); ++r) {
            }
        if (r - i >= 2) {
            for (int k = i; k < r; ++k) {
                Epilogue ep;
                ep.w2 = ops[k].w_up;
                ep.bias = ops[k].bias;
                mlq_status st = run_linear(ops[k].fmt, ops[k].w, ops[k].out_features, ops[k].in_features, xs[k],
                                           ops[k].rows, ys[k], stream, ep, k == i ? mlq::kPdlFirst : mlq::kPdlNoWait);
                if (st != MLQ_OK) return st;
            }
            cudaError_t e = mlq::launch_join(stream);
            if (e != cudaSuccess) return fail_cuda("join launch", e);
            i = r;
            continue;
        }
        int j = i + 1;
        if (groupable(i))
            while (j < n && j - i < mlq::kBgemmMaxGroup && groupable(j) && xs[j] == xs[i] &&
                   ops[j].fmt == ops[i].fmt && ops[j].in_features == ops[i].in_features &&
                   ops[j].rows == ops[i].rows)
                ++j;
        if (j - i == 1) {
            mlq_status st = run_op(ops[i], xs[i], ys[i], stream);
            if (st != MLQ_OK) return st;
            i = j;
            continue;
        }
        int dev = 0;
        cudaError_t e = cudaGetDevice(&dev);
        if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
        mlq_status st = MLQ_OK;
        DeviceState* ds = device_state(dev, &st);
        if (!ds) return st;
        const uint8_t* wm[mlq::kBgemmMaxGroup];
        float* ym[mlq::kBgemmMaxGroup];
        int om[mlq::kBgemmMaxGroup];
        const float* bm[mlq::kBgemmMaxGroup];
        for (int k = i; k < j; ++k) {
            wm[k - i] = static_cast<const uint8_t*>(ops[k].w);
            ym[k - i] = ys[k];
            om[k - i] = ops[k].out_features;
            bm[k - i] = ops[k].bias;
        }
        void* ws = nullptr;
        st = stream_workspace(
            ds, stream,
            mlq::bgemm_group_workspace_bytes(ops[i].fmt, ops[i].in_features, ops[i].rows, om, j - i, ds->sm_count),
            &ws);
        if (st != MLQ_OK) return st;
        e = mlq::launch_bgemm_group(ops[i].fmt, j - i, wm, ym, om, bm, xs[i], ops[i].in_features, ops[i].rows, ws,
                                    ds->sm_count, ds->err_flag, stream);
        if (e != cudaSuccess) return fail_cuda("bgemm launch", e);
        i = j;
    }
    return MLQ_OK;
}


}  // namespace

void mlq::set_last_error(const char* msg) { t_last_error = msg ? msg : ""; }

extern "C" {

MLQ_API int mlq_built(void) { return 1; }

MLQ_API size_t mlq_block_bytes(mlq_format fmt) { return (size_t)mlq::block_bytes((int)fmt); }

MLQ_API size_t mlq_block_count(int out_features, int in_features) {
    if (out_features <= 0 || in_features <= 0) return 0;
    return (size_t)out_features * (size_t)((in_features + mlq::kQK - 1) / mlq::kQK);
}

MLQ_API const char* mlq_status_string(mlq_status s) {
    switch (s) {
        case MLQ_OK: return "ok";
        case MLQ_ERR_FORMAT: return "unknown block format";
        case MLQ_ERR_NULL: return "null pointer";
        case MLQ_ERR_EMPTY: return "empty tensors are not supported";
        case MLQ_ERR_SHAPE: return "dimension mismatch";
        case MLQ_ERR_BLOCK_COUNT: return "block count mismatch";
        case MLQ_ERR_DEVICE: return "invalid device";
        case MLQ_ERR_CUDA: return "CUDA error";
        case MLQ_ERR_TIMEOUT: return "kernel wait timed out";
        case MLQ_ERR_RANGE: return "size out of range";
        case MLQ_ERR_COMM: return "inconsistent sharding arguments";
    }
    return "unknown status";
}

MLQ_API const char* mlq_last_error(void) { return t_last_error.c_str(); }

MLQ_API mlq_status mlq_device_error(int device, int* code) {
    try {
        if (!code) return fail(MLQ_ERR_NULL, "mlq_device_error: null code pointer");
        int prev = 0;
        cudaGetDevice(&prev);
        mlq_status st = set_device(device);
        if (st != MLQ_OK) return st;
        DeviceState* ds = device_state(device, &st);
        if (ds) {
            cudaError_t e = cudaDeviceSynchronize();
            int v = 0;
            if (e == cudaSuccess) e = cudaMemcpy(&v, ds->err_flag, sizeof(int), cudaMemcpyDeviceToHost);
            if (e == cudaSuccess) e = cudaMemset(ds->err_flag, 0, sizeof(int));
            // a launch that gave up may have left its tile-queue pair counted
            // but not reset: start every queue from zero again
            if (e == cudaSuccess && v != 0) e = mlq::reset_tile_queues();
            if (e == cudaSuccess) e = cudaDeviceSynchronize();
            if (e != cudaSuccess) st = fail_cuda("mlq_device_error", e);
            *code = v;
        }
        cudaSetDevice(prev);
        return st;
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_device_error: host exception");
    }
}

MLQ_API mlq_status mlq_linear(mlq_format fmt, const void* w, size_t block_count, int out_features,
                              int in_features, const float* x, int rows, float* y,
                              mlq_stream stream) {
    try {
        mlq_status st =
            validate_linear(fmt, w, block_count, out_features, in_features, x, rows, y, "mlq_linear");
        if (st != MLQ_OK) return st;
        return run_linear(fmt, w, out_features, in_features, x, rows, y,
                          reinterpret_cast<cudaStream_t>(stream));
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear: host exception");
    }
}

MLQ_API mlq_status mlq_linear_noalloc(mlq_format fmt, const void* w, size_t block_count,
                                      int out_features, int in_features, const float* x, int rows,
                                      float* y, mlq_stream stream) {
    try {
        mlq_status st = validate_linear(fmt, w, block_count, out_features, in_features, x, rows, y,
                                        "mlq_linear_noalloc");
        if (st != MLQ_OK) return st;
        // only a call that takes the tensor-core GEMM uses the scratch (the
        // same routing test as mlq_linear: rows rule, alignment, in % 8)
        const size_t need = mlq::gemm_workspace_bytes(in_features, rows, out_features, 1);
        if (!mlq::bgemm_shape_ok(fmt, w, out_features, in_features, rows) &&
            mlq::gemm_shape_ok(fmt, w, out_features, in_features, rows) && need > (size_t)MLQ_NOALLOC_SCRATCH_BYTES)
            return fail(MLQ_ERR_RANGE,
                        "mlq_linear_noalloc: rows * in_features * 4 = " + std::to_string(need) +
                            " bytes of x split exceed the " +
                            std::to_string((size_t)MLQ_NOALLOC_SCRATCH_BYTES) +
                            "-byte static scratch (use mlq_linear, or fewer rows per call)");
        return run_linear_noalloc(fmt, w, out_features, in_features, x, rows, y,
                                  reinterpret_cast<cudaStream_t>(stream));
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_noalloc: host exception");
    }
}

MLQ_API mlq_status mlq_linear_bias(mlq_format fmt, const void* w, size_t block_count,
                                   int out_features, int in_features, const float* x, int rows,
                                   const float* bias, float* y, mlq_stream stream) {
    try {
        mlq_status st = validate_linear(fmt, w, block_count, out_features, in_features, x, rows, y,
                                        "mlq_linear_bias");
        if (st != MLQ_OK) return st;
        Epilogue ep;
        ep.bias = bias;
        return run_linear(fmt, w, out_features, in_features, x, rows, y,
                          reinterpret_cast<cudaStream_t>(stream), ep);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_bias: host exception");
    }
}

MLQ_API mlq_status mlq_linear_swiglu(mlq_format fmt, const void* w_gate, const void* w_up,
                                     size_t block_count, int out_features, int in_features,
                                     const float* x, int rows, float* h, mlq_stream stream) {
    try {
        mlq_status st = validate_linear(fmt, w_gate, block_count, out_features, in_features, x, rows, h,
                                        "mlq_linear_swiglu");
        if (st != MLQ_OK) return st;
        if (w_up == nullptr)
            return fail(MLQ_ERR_NULL, std::string("mlq_linear_swiglu(") + fmt_name(fmt) +
                                          "): null up-projection weight pointer");
        Epilogue ep;
        ep.w2 = w_up;
        return run_linear(fmt, w_gate, out_features, in_features, x, rows, h,
                          reinterpret_cast<cudaStream_t>(stream), ep);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_swiglu: host exception");
    }
}

MLQ_API mlq_status mlq_linear_host(mlq_format fmt, const void* w, size_t block_count,
                                   int out_features, int in_features, const float* x_host,
                                   int rows, const float* bias_host, float* y_host, int device,
                                   mlq_stream stream) {
    try {
        mlq_status st = validate_linear(fmt, w, block_count, out_features, in_features, x_host, rows,
                                        y_host, "mlq_linear_host");
        if (st != MLQ_OK) return st;
        st = set_device(device);
        if (st != MLQ_OK) return st;
        DeviceState* ds = device_state(device, &st);
        if (!ds) return st;
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        std::lock_guard<std::mutex> lock(ds->host_mu);
        const size_t xb = (size_t)rows * in_features * sizeof(float);
        const size_t yb = (size_t)rows * out_features * sizeof(float);
        if ((st = ensure(&ds->x_stage, &ds->x_cap, xb)) != MLQ_OK) return st;
        if ((st = ensure(&ds->y_stage, &ds->y_cap, yb)) != MLQ_OK) return st;
        cudaError_t e = cudaMemcpyAsync(ds->x_stage, x_host, xb, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return fail_cuda("cudaMemcpyAsync (x upload)", e);
        st = run_linear(fmt, w, out_features, in_features, ds->x_stage, rows, ds->y_stage, s);
        if (st != MLQ_OK) return st;
        e = cudaMemcpyAsync(y_host, ds->y_stage, yb, cudaMemcpyDeviceToHost, s);
        if (e != cudaSuccess) return fail_cuda("cudaMemcpyAsync (y download)", e);
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize", e);
        if (bias_host) {
            // Bias on the host after the download, as src/cuda_quant.cu:326-329 does.
            for (int r = 0; r < rows; ++r) {
                float* yr = y_host + (size_t)r * out_features;
                for (int c = 0; c < out_features; ++c) yr[c] += bias_host[c];
            }
        }
        return MLQ_OK;
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_host: host exception");
    }
}

MLQ_API mlq_status mlq_linear_host_weight(mlq_format fmt, const void* w_host, size_t block_count,
                                          int out_features, int in_features,
                                          const float* x_host, int rows, const float* bias_host,
                                          float* y_host, int device) {
    try {
        mlq_status st = validate_linear(fmt, w_host, block_count, out_features, in_features, x_host,
                                        rows, y_host, "mlq_linear_host_weight");
        if (st != MLQ_OK) return st;
        st = set_device(device);
        if (st != MLQ_OK) return st;
        const size_t wb = block_count * mlq_block_bytes(fmt);
        void* wd = nullptr;
        cudaError_t e = cudaMalloc(&wd, wb);
        if (e != cudaSuccess) return fail_cuda("cudaMalloc (weights)", e);
        e = cudaMemcpy(wd, w_host, wb, cudaMemcpyHostToDevice);
        if (e == cudaSuccess) {
            st = mlq_linear_host(fmt, wd, block_count, out_features, in_features, x_host, rows,
                                 bias_host, y_host, device, nullptr);
        } else {
            st = fail_cuda("cudaMemcpy (weights)", e);
        }
        cudaFree(wd);
        return st;
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_host_weight: host exception");
    }
}

MLQ_API mlq_status mlq_dequantize(mlq_format fmt, const void* w, size_t block_count,
                                  int out_features, int in_features, float* dst,
                                  mlq_stream stream) {
    try {
        mlq_status st = validate_linear(fmt, w, block_count, out_features, in_features, dst, 1, dst,
                                        "mlq_dequantize");
        if (st != MLQ_OK) return st;
        cudaError_t e = mlq::launch_dequantize(fmt, static_cast<const uint8_t*>(w), out_features,
                                               in_features, dst, reinterpret_cast<cudaStream_t>(stream));
        return e == cudaSuccess ? MLQ_OK : fail_cuda("dequantize launch", e);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_dequantize: host exception");
    }
}

MLQ_API mlq_status mlq_quantize(mlq_format fmt, const float* src, int rows, int cols, void* blocks,
                                mlq_stream stream) {
    try {
        if (!known_format(fmt)) return fail(MLQ_ERR_FORMAT, "mlq_quantize: unknown block format");
        if (rows <= 0 || cols <= 0) return fail(MLQ_ERR_EMPTY, "mlq_quantize: empty tensors are not supported");
        if (!src || !blocks) return fail(MLQ_ERR_NULL, "mlq_quantize: null pointer");
        cudaError_t e = mlq::launch_quantize(fmt, src, rows, cols, static_cast<uint8_t*>(blocks),
                                             reinterpret_cast<cudaStream_t>(stream));
        return e == cudaSuccess ? MLQ_OK : fail_cuda("quantize launch", e);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_quantize: host exception");
    }
}

MLQ_API mlq_status mlq_transcode(int src_type, const void* src, mlq_format dst_fmt, void* dst, int rows, int cols,
                                 mlq_stream stream) {
    try {
        const char* who = "mlq_transcode";
        if (src_type != 0 && !known_format(src_type))
            return fail(MLQ_ERR_FORMAT, std::string(who) + ": source type must be 0 (fp32) or a block format");
        if (!known_format(dst_fmt)) return fail(MLQ_ERR_FORMAT, std::string(who) + ": unknown block format");
        if (rows <= 0 || cols <= 0) return fail(MLQ_ERR_EMPTY, std::string(who) + ": empty tensors are not supported");
        if (!src || !dst) return fail(MLQ_ERR_NULL, std::string(who) + ": null pointer");
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        cudaError_t e;
        if (src_type == 0) {
            e = mlq::launch_quantize(dst_fmt, static_cast<const float*>(src), rows, cols, static_cast<uint8_t*>(dst), s);
        } else if (src_type == (int)dst_fmt) {
            // the reference leaves a tensor already in the target format untouched
            e = cudaMemcpyAsync(dst, src, mlq_block_count(rows, cols) * mlq::block_bytes(dst_fmt),
                                cudaMemcpyDeviceToDevice, s);
        } else {
            e = mlq::launch_transcode(src_type, static_cast<const uint8_t*>(src), dst_fmt, static_cast<uint8_t*>(dst),
                                      rows, cols, s);
        }
        return e == cudaSuccess ? MLQ_OK : fail_cuda("transcode", e);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_transcode: host exception");
    }
}

MLQ_API mlq_status mlq_quantize_model(const mlq_quantize_op* ops, int n, mlq_stream stream) {
    try {
        if (n < 0) return fail(MLQ_ERR_EMPTY, "mlq_quantize_model: negative op count");
        if (n > 0 && !ops) return fail(MLQ_ERR_NULL, "mlq_quantize_model: null op list");
        for (int i = 0; i < n; ++i) {
            const mlq_quantize_op& o = ops[i];
            const std::string who = "mlq_quantize_model op " + std::to_string(i);
            if (o.src_type != 0 && !known_format(o.src_type))
                return fail(MLQ_ERR_FORMAT, who + ": source type must be 0 (fp32) or a block format");
            if (!known_format(o.dst_fmt)) return fail(MLQ_ERR_FORMAT, who + ": unknown block format");
            if (o.rows <= 0 || o.cols <= 0) return fail(MLQ_ERR_EMPTY, who + ": empty tensors are not supported");
            if (!o.src || !o.dst) return fail(MLQ_ERR_NULL, who + ": null pointer");
        }
        for (int i = 0; i < n; ++i) {
            mlq_status st = mlq_transcode(ops[i].src_type, ops[i].src, (mlq_format)ops[i].dst_fmt, ops[i].dst,
                                          ops[i].rows, ops[i].cols, stream);
            if (st != MLQ_OK) return st;
        }
        return MLQ_OK;
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_quantize_model: host exception");
    }
}

MLQ_API size_t mlq_flag_bytes(void) { return kFlagBytes; }

// The deferred wait of a sharded op (validated gather), in stream order.
mlq_status run_gather_wait(const mlq_gather& g, cudaStream_t stream) {
    if (g.world_size == 1) return MLQ_OK;  // one rank: stream order is all there is to wait for
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail_cuda("cudaGetDevice", e);
    mlq_status st = MLQ_OK;
    DeviceState* ds = device_state(dev, &st);
    if (!ds) return st;
    e = mlq::launch_gather_wait(g.peer_flags[g.rank], g.world_size, g.epoch, ds->err_flag, stream);
    return e == cudaSuccess ? MLQ_OK : fail_cuda("gather wait launch", e);
}

MLQ_API mlq_status mlq_gather_wait(const mlq_gather* g, mlq_stream stream) {
    try {
        if (!g) return fail(MLQ_ERR_NULL, "mlq_gather_wait: null gather");
        if (g->world_size < 1 || g->world_size > mlq::kMaxWorld || g->rank < 0 || g->rank >= g->world_size)
            return fail(MLQ_ERR_COMM, "mlq_gather_wait: world_size must be 1..8 and 0 <= rank < world_size");
        if (g->epoch == 0) return fail(MLQ_ERR_COMM, "mlq_gather_wait: epoch starts at 1");
        if (!g->peer_flags || !g->peer_flags[g->rank])
            return fail(MLQ_ERR_NULL, "mlq_gather_wait: null flag pointer for this rank");
        return run_gather_wait(*g, reinterpret_cast<cudaStream_t>(stream));
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_gather_wait: host exception");
    }
}

MLQ_API mlq_status mlq_linear_allgather(mlq_format fmt, const void* w_shard,
                                        size_t shard_block_count, int out_features,
                                        int in_features, int row_begin, int row_end,
                                        const float* x, int rows, float* const* peer_y,
                                        uint32_t* const* peer_flags, int world_size, int rank,
                                        uint32_t epoch, mlq_stream stream) {
    try {
        mlq_gather g{world_size, rank, row_begin, row_end, peer_y, peer_flags, epoch};
        mlq_status st = validate_gather(fmt, w_shard, shard_block_count, out_features, in_features, x, rows, g,
                                        "mlq_linear_allgather");
        if (st != MLQ_OK) return st;
        return run_gather(fmt, w_shard, out_features, in_features, x, rows, nullptr, g,
                          reinterpret_cast<cudaStream_t>(stream));
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_allgather: host exception");
    }
}

MLQ_API mlq_status mlq_linear_batch(const mlq_linear_op* ops, int n, mlq_stream stream) {
    try {
        if (n < 0) return fail(MLQ_ERR_EMPTY, "mlq_linear_batch: negative op count");
        if (n > 0 && !ops) return fail(MLQ_ERR_NULL, "mlq_linear_batch: null op list");
        for (int i = 0; i < n; ++i) {
            mlq_status st = validate_op(ops[i], i, false);
            if (st != MLQ_OK) return st;
        }
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        std::vector<const float*> xs(n);
        std::vector<float*> ys(n);
        for (int i = 0; i < n; ++i) {
            xs[i] = ops[i].x;
            ys[i] = ops[i].y;
        }
        return run_ops(ops, n, xs.data(), ys.data(), s);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_batch: host exception");
    }
}

// mlq_linear_batch_host splits a step when its y download is at least
// kSplitMinDownload bytes and a plain one-row op has at least kSplitMinRows
// rows; kHbmOverPcie is the ratio of weight-streaming to download speed it
// assumes when sizing the second part (B200 HBM against a PCIe Gen5 link).
constexpr size_t kSplitMinDownload = 256 * 1024;
constexpr int kSplitMinRows = 4096;
constexpr double kHbmOverPcie = 128.0;

MLQ_API mlq_status mlq_linear_batch_host(const mlq_linear_op* ops, int n, int device, mlq_stream stream) {
    try {
        if (n < 0) return fail(MLQ_ERR_EMPTY, "mlq_linear_batch_host: negative op count");
        if (n > 0 && !ops) return fail(MLQ_ERR_NULL, "mlq_linear_batch_host: null op list");
        for (int i = 0; i < n; ++i) {
            mlq_status st = validate_op(ops[i], i, true);
            if (st != MLQ_OK) return st;
        }
        if (n == 0) return MLQ_OK;
        mlq_status st = set_device(device);
        if (st != MLQ_OK) return st;
        DeviceState* ds = device_state(device, &st);
        if (!ds) return st;
        cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
        std::lock_guard<std::mutex> lock(ds->host_mu);
        // every op's x and y in one staging buffer each, 256-B aligned
        // slices; ops with the same host x (pointer and size) share one upload
        std::vector<size_t> xo(n), yo(n);
        std::vector<bool> upload(n, true);
        size_t xt = 0, yt = 0;
        for (int i = 0; i < n; ++i) {
            yo[i] = yt;
            if (!ops[i].gather) yt += ((size_t)ops[i].rows * ops[i].out_features * sizeof(float) + 255) & ~(size_t)255;
            int same = -1;
            for (int k = 0; k < i && same < 0; ++k)
                if (upload[k] && ops[k].x == ops[i].x && ops[k].rows == ops[i].rows &&
                    ops[k].in_features == ops[i].in_features)
                    same = k;
            if (same >= 0) {
                xo[i] = xo[same];
                upload[i] = false;
                continue;
            }
            xo[i] = xt;
            xt += ((size_t)ops[i].rows * ops[i].in_features * sizeof(float) + 255) & ~(size_t)255;
        }
        if ((st = ensure(&ds->x_stage, &ds->x_cap, xt)) != MLQ_OK) return st;
        if (yt > 0 && (st = ensure(&ds->y_stage, &ds->y_cap, yt)) != MLQ_OK) return st;
        char* xs = reinterpret_cast<char*>(ds->x_stage);
        char* ys = reinterpret_cast<char*>(ds->y_stage);
        // Copies in op order; one copy per run of ops whose host buffers and
        // staging slices both follow on directly (a caller that lays its x,
        // or its y, out back to back in one pinned buffer gets one copy per
        // direction: each copy costs a DMA setup).
        struct Copy {
            char* dst;
            const char* src;
            size_t bytes;
        };
        auto add = [](std::vector<Copy>& v, void* dst, const void* src, size_t bytes) {
            char* d = static_cast<char*>(dst);
            const char* sp = static_cast<const char*>(src);
            if (!v.empty() && v.back().dst + v.back().bytes == d && v.back().src + v.back().bytes == sp)
                v.back().bytes += bytes;
            else
                v.push_back(Copy{d, sp, bytes});
        };
        std::vector<Copy> ups;
        for (int i = 0; i < n; ++i)
            if (upload[i]) add(ups, xs + xo[i], ops[i].x, (size_t)ops[i].rows * ops[i].in_features * sizeof(float));
        cudaError_t e = cudaSuccess;
        for (size_t k = 0; k < ups.size() && e == cudaSuccess; ++k)
            e = cudaMemcpyAsync(ups[k].dst, ups[k].src, ups[k].bytes, cudaMemcpyHostToDevice, s);
        if (e != cudaSuccess) return fail_cuda("cudaMemcpyAsync (x upload)", e);
        std::vector<const float*> xd(n);
        std::vector<float*> yd(n);
        for (int i = 0; i < n; ++i) {
            xd[i] = reinterpret_cast<const float*>(xs + xo[i]);
            yd[i] = reinterpret_cast<float*>(ys + yo[i]);
        }
        // A large download overlaps the step's last compute: the rows
        // [split_row, out) of the largest plain one-row op run as a second
        // launch, and every other y range is copied back on the download
        // stream while they compute.  Each row's arithmetic is the same.
        int split_op = -1, split_row = 0;
        {
            size_t ybytes = 0;
            for (int i = 0; i < n; ++i) ybytes += (size_t)ops[i].rows * ops[i].out_features * sizeof(float);
            for (int i = 0; i < n; ++i)
                if (!ops[i].gather && !ops[i].w_up && ops[i].rows == 1 && ops[i].out_features >= kSplitMinRows &&
                    (split_op < 0 || ops[i].out_features > ops[split_op].out_features))
                    split_op = i;
            if (ybytes < kSplitMinDownload) split_op = -1;
            if (split_op >= 0) {
                // the second part's weights take about as long to stream as
                // the first part's y to copy back (HBM ~kHbmOverPcie x PCIe)
                const mlq_linear_op& o = ops[split_op];
                const double wrow = (double)mlq_block_count(1, o.in_features) * mlq::block_bytes(o.fmt);
                const double rows_b = kHbmOverPcie * (double)ybytes / (wrow + kHbmOverPcie * sizeof(float));
                // (an op too small to hide the download is not split)
                const int rb = (int)rows_b / 256 * 256;
                if (rb < 256 || rb > o.out_features - 256) split_op = -1;
                else split_row = o.out_features - rb;
            }
            if (split_op >= 0 && !ds->copy_stream) {
                e = cudaStreamCreateWithFlags(&ds->copy_stream, cudaStreamNonBlocking);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ds->part_done, cudaEventDisableTiming);
                if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ds->copies_done, cudaEventDisableTiming);
                if (e != cudaSuccess) return fail_cuda("download stream setup", e);
            }
        }
        std::vector<mlq_linear_op> ops_a(ops, ops + n);
        if (split_op >= 0) {
            ops_a[split_op].out_features = split_row;
            ops_a[split_op].block_count = mlq_block_count(split_row, ops[split_op].in_features);
        }
        st = run_ops(ops_a.data(), n, xd.data(), yd.data(), s);
        if (st != MLQ_OK) return st;
        // deferred sharded ops: every rank's rows in y before it is copied
        // back.  One wait per flag array (this rank's flag words), for the
        // highest epoch among its ops: epochs rise from op to op on one
        // array, so that wait covers the others.
        std::vector<mlq_gather> waits;
        for (int i = 0; i < n; ++i) {
            if (!ops[i].gather || !ops[i].gather->defer_wait) continue;
            const mlq_gather& g = *ops[i].gather;
            bool merged = false;
            for (mlq_gather& w : waits)
                if (w.world_size == g.world_size && w.peer_flags[w.rank] == g.peer_flags[g.rank]) {
                    if ((int)(g.epoch - w.epoch) > 0) w.epoch = g.epoch;
                    merged = true;
                    break;
                }
            if (!merged) waits.push_back(g);
        }
        for (const mlq_gather& w : waits)
            if ((st = run_gather_wait(w, s)) != MLQ_OK) return st;
        std::vector<Copy> downs;
        for (int i = 0; i < n; ++i) {
            // a gathered op's full y is this rank's peer_y entry
            const void* src = ops[i].gather ? static_cast<const void*>(ops[i].gather->peer_y[ops[i].gather->rank])
                                            : static_cast<const void*>(ys + yo[i]);
            add(downs, ops[i].y, src, (size_t)ops[i].rows * ops_a[i].out_features * sizeof(float));
        }
        cudaStream_t ds_s = s;  // where the first part's y goes back
        if (split_op >= 0) {
            // the first part done: its y back on the download stream while
            // the second part computes on `s`
            e = cudaEventRecord(ds->part_done, s);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(ds->copy_stream, ds->part_done, 0);
            if (e != cudaSuccess) return fail_cuda("download stream order", e);
            ds_s = ds->copy_stream;
        }
        for (size_t k = 0; k < downs.size() && e == cudaSuccess; ++k)
            e = cudaMemcpyAsync(downs[k].dst, downs[k].src, downs[k].bytes, cudaMemcpyDeviceToHost, ds_s);
        if (e != cudaSuccess) return fail_cuda("cudaMemcpyAsync (y download)", e);
        if (split_op >= 0) {
            const mlq_linear_op& o = ops[split_op];
            const size_t row_bytes = mlq_block_count(1, o.in_features) * mlq::block_bytes(o.fmt);
            mlq_linear_op b = o;
            b.w = static_cast<const uint8_t*>(o.w) + (size_t)split_row * row_bytes;
            b.out_features = o.out_features - split_row;
            b.block_count = mlq_block_count(b.out_features, o.in_features);
            b.bias = o.bias ? o.bias + split_row : nullptr;
            const float* xb = xd[split_op];
            float* yb = yd[split_op] + split_row;
            st = run_ops(&b, 1, &xb, &yb, s);
            if (st != MLQ_OK) return st;
            e = cudaMemcpyAsync(o.y + split_row, yb, (size_t)b.out_features * sizeof(float), cudaMemcpyDeviceToHost, s);
            if (e == cudaSuccess) e = cudaEventRecord(ds->copies_done, ds->copy_stream);
            if (e == cudaSuccess) e = cudaStreamWaitEvent(s, ds->copies_done, 0);
            if (e != cudaSuccess) return fail_cuda("cudaMemcpyAsync (y download, last part)", e);
        }
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail_cuda("cudaStreamSynchronize", e);
        return MLQ_OK;
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_linear_batch_host: host exception");
    }
}

MLQ_API mlq_status mlq_peer_alloc(size_t bytes, void** ptr, mlq_ipc_handle* handle) {
    try {
        if (!ptr || !handle) return fail(MLQ_ERR_NULL, "mlq_peer_alloc: null pointer");
        if (bytes == 0) return fail(MLQ_ERR_EMPTY, "mlq_peer_alloc: zero bytes");
        *ptr = nullptr;
        cudaError_t e = cudaMalloc(ptr, bytes);
        if (e != cudaSuccess) return fail_cuda("cudaMalloc (peer buffer)", e);
        e = cudaMemset(*ptr, 0, bytes);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        cudaIpcMemHandle_t h;
        if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, *ptr);
        if (e != cudaSuccess) {
            cudaFree(*ptr);
            *ptr = nullptr;
            return fail_cuda("cudaIpcGetMemHandle", e);
        }
        static_assert(sizeof(h) == sizeof(handle->bytes), "IPC handle size");
        std::memcpy(handle->bytes, &h, sizeof(h));
        return MLQ_OK;
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_peer_alloc: host exception");
    }
}

MLQ_API mlq_status mlq_peer_open(const mlq_ipc_handle* handle, void** ptr) {
    try {
        if (!ptr || !handle) return fail(MLQ_ERR_NULL, "mlq_peer_open: null pointer");
        cudaIpcMemHandle_t h;
        std::memcpy(&h, handle->bytes, sizeof(h));
        cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
        return e == cudaSuccess ? MLQ_OK : fail_cuda("cudaIpcOpenMemHandle", e);
    } catch (...) {
        return fail(MLQ_ERR_CUDA, "mlq_peer_open: host exception");
    }
}

MLQ_API mlq_status mlq_peer_close(void* ptr) {
    cudaError_t e = cudaIpcCloseMemHandle(ptr);
    return e == cudaSuccess ? MLQ_OK : fail_cuda("cudaIpcCloseMemHandle", e);
}

MLQ_API mlq_status mlq_peer_free(void* ptr) {
    cudaError_t e = cudaFree(ptr);
    return e == cudaSuccess ? MLQ_OK : fail_cuda("cudaFree (peer buffer)", e);
}

}  // extern "C"
