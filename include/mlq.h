/*
 * mlq.h -- C ABI of the B200 quantized-matmul library (libmlq.so).
 *
 * Replaces the GPU half of the reference's quantized linear path
 * (Haobin-Lee/mini-llama): include/mini_llama/cuda_quant.h and the kernels
 * in src/cuda_quant.cu.  Plain C: pointers, sizes, status codes, a CUDA
 * stream handle.  No C++ types, no exceptions, no torch types cross it.
 *
 * Conventions shared by every entry point
 *   - Weights are the reference's packed block arrays, byte-identical to
 *     std::vector<BlockQ80/BlockQ40/BlockQ41>::data()
 *     (include/mini_llama/quantized_tensor.h:36-72): row-major [out][bpr]
 *     with bpr = ceil(in/32) blocks per row.
 *   - x is fp32 row-major [rows][in]; y is fp32 row-major [rows][out];
 *     y = x * W^T, overwritten (not accumulated into).
 *   - Arguments are validated on the host BEFORE any CUDA call, with the
 *     reference's checks (src/cuda_quant.cu:188-227, 305-307, 342-345);
 *     a failing check returns a status and leaves the GPU untouched.
 *     mlq_last_error() then returns a message (per host thread).
 *   - `stream` is a cudaStream_t (NULL = the legacy default stream, which
 *     is what the reference launches on).  Device-side entry points are
 *     asynchronous on that stream; *_host entry points are synchronous.
 *   - The current CUDA device must own every device pointer passed.
 *   - Ordering with the previous kernel on the stream: the streaming GEMV,
 *     the batched-decode GEMM (its x split and the GEMM) and a batch's run
 *     launch (its x slicing and the run kernel, see mlq_linear_batch) are
 *     launched with programmatic dependent launch, so they may start while the kernel
 *     before them on the stream is still running.  They read x and the bias,
 *     and write y and their workspace, only after that kernel has completed;
 *     they stream the WEIGHTS before.  So the weights must be complete before
 *     the stream's previous kernel started, whenever that kernel lets its
 *     dependents start early (this library's GEMV, batched-decode GEMM, run
 *     launches and mlq_gather_wait's kernel do; its quantizer and the other
 *     kernels here do not, so a quantize followed by a linear on one stream
 *     is ordered).
 */
#ifndef MLQ_H_
#define MLQ_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MLQ_API __attribute__((visibility("default")))
#else
#define MLQ_API
#endif

/* A cudaStream_t, spelled without including the CUDA headers. */
typedef struct CUstream_st* mlq_stream;

/* Block formats; the values are the GGUF tensor type ids the reference's
 * loader maps to QuantType (include/mini_llama/gguf.h:16-22). */
typedef enum mlq_format {
    MLQ_Q4_0 = 2, /* BlockQ40: fp16 d + 16 nibble bytes, 18 B / 32 values */
    MLQ_Q4_1 = 3, /* BlockQ41: fp16 d, fp16 m + 16 bytes, 20 B / 32 values */
    MLQ_Q8_0 = 8  /* BlockQ80: fp16 d + 32 int8,          34 B / 32 values */
} mlq_format;

typedef enum mlq_status {
    MLQ_OK = 0,
    MLQ_ERR_FORMAT = 1,      /* unknown mlq_format */
    MLQ_ERR_NULL = 2,        /* null pointer ("null weight pointer", cuda_quant.cu:305-307) */
    MLQ_ERR_EMPTY = 3,       /* a dimension <= 0 ("empty tensors are not supported", :209-212) */
    MLQ_ERR_SHAPE = 4,       /* x/W in_features mismatch (:213-218) */
    MLQ_ERR_BLOCK_COUNT = 5, /* block_count != out*ceil(in/32) (:219-226) */
    MLQ_ERR_DEVICE = 6,      /* bad device id / pointer on another device (:342-345) */
    MLQ_ERR_CUDA = 7,        /* a CUDA runtime call failed (:20-29) */
    MLQ_ERR_TIMEOUT = 8,     /* a kernel's bounded wait expired (device error flag set) */
    MLQ_ERR_RANGE = 9,       /* a size too large for this entry point */
    MLQ_ERR_COMM = 10        /* a sharded call's peer/rank arguments are inconsistent */
} mlq_status;

/* ---------------------------------------------------------------------------
 * Library facts
 * ------------------------------------------------------------------------- */

/* 1 when the CUDA kernels are compiled in.  Replaces cudaQuantBuilt()
 * (include/mini_llama/cuda_quant.h:13). */
MLQ_API int mlq_built(void);

/* Bytes of one block (34/18/20) or 0 for an unknown format
 * (sizeof(BlockQ80/Q40/Q41), quantized_tensor.h:41,55,71). */
MLQ_API size_t mlq_block_bytes(mlq_format fmt);

/* out * ceil(in/32): the block count the validation expects
 * (src/cuda_quant.cu:219-220); 0 when a dimension is not positive. */
MLQ_API size_t mlq_block_count(int out_features, int in_features);

MLQ_API const char* mlq_status_string(mlq_status status);

/* Message for the last failing call on this host thread ("" if none). */
MLQ_API const char* mlq_last_error(void);

/* Reads and clears the device-side error flag of `device` (non-zero after
 * a kernel gave up on a bounded wait).  Synchronizes that device.  When the
 * flag was set it also resets the streaming GEMV's row-tile queues on that
 * device, so launches after a failed one start clean. */
MLQ_API mlq_status mlq_device_error(int device, int* code);

/* ---------------------------------------------------------------------------
 * Quantized linear
 * ------------------------------------------------------------------------- */

/* Device weight, device x, device y:  y[rows,out] = x[rows,in] * W^T.
 * Replaces cudaQ80LinearDeviceInput / cudaQ40LinearDeviceInput /
 * cudaQ41LinearDeviceInput (include/mini_llama/cuda_quant.h:29-33, 50-54,
 * 69-73; src/cuda_quant.cu:333-361, 411-439, 489-517), except that the
 * caller passes y instead of receiving a freshly cudaMalloc'd CudaTensor.
 * rows >= 1 (the reference's rank-1 x is rows == 1).  Asynchronous. */
MLQ_API mlq_status mlq_linear(mlq_format fmt, const void* w, size_t block_count,
                              int out_features, int in_features, const float* x, int rows,
                              float* y, mlq_stream stream);

/* Which kernel a call takes.
 *
 * From MLQ_BGEMM_MIN_ROWS to MLQ_BGEMM_MAX_ROWS rows of x (batched decode),
 * when in_features % 32 == 0 and the weights are 16-B aligned with a 16-B
 * multiple row pitch: the batched-decode tensor-core GEMM (exact fp16
 * weight codes, each row of x split into fp16 hi/lo against a power-of-two
 * scale of its own, one TMEM accumulator per 32-value block folded in fp32
 * on the CUDA cores; the work split evenly over the SMs, a split row tile
 * summed in a fixed order by the last of its CTAs to finish).  Two rows
 * take the streaming GEMV's two-row pass, which is faster there.
 * Otherwise the rule below. */
#define MLQ_BGEMM_MIN_ROWS 3
#define MLQ_BGEMM_MAX_ROWS 32

/* The tensor-core (tcgen05) GEMM's time hardly
 * depends on the rows of x (one decode of every weight per 128-row tile,
 * split along K when the tiles cannot fill the SMs), the streaming GEMV's
 * grows with every pass of <= 8 rows.  A call takes the GEMM when it has
 * at least MLQ_GEMM_MIN_ROWS rows of x, or at least MLQ_GEMM_LARGE_MIN_ROWS
 * rows on a matrix of at least MLQ_GEMM_LARGE_MIN_WEIGHTS weights
 * (out_features * in_features); MLQ_GEMM_ROWS_RULE(rows, out, in) is that
 * test (for calls the batched-decode GEMM does not take).  The GEMM also
 * needs 16-B aligned weights with a 16-B multiple row pitch and
 * in_features % 8 == 0; other calls take the streaming GEMV.
 * (Measured on B200 at 8 rows: q4_0 8192x28672, GEMM 158 us vs GEMV
 * 213 us; q4_0 4608x3584, GEMM 24.8 us vs GEMV 18.6 us.) */
#define MLQ_GEMM_MIN_ROWS 9
#define MLQ_GEMM_LARGE_MIN_ROWS 5
#define MLQ_GEMM_LARGE_MIN_WEIGHTS (1LL << 25)
#define MLQ_GEMM_ROWS_RULE(rows, out, in)                                         \
    ((rows) >= MLQ_GEMM_MIN_ROWS ||                                               \
     ((rows) >= MLQ_GEMM_LARGE_MIN_ROWS &&                                        \
      (long long)(out) * (long long)(in) >= MLQ_GEMM_LARGE_MIN_WEIGHTS))

/* mlq_linear that never allocates device memory.  No counterpart in the
 * reference (its GPU linear cudaMallocs its output on every call,
 * src/cuda_quant.cu:333-361).
 *
 * Meant for callers that must not allocate: a serving loop that reserved
 * the whole device up front (weights + KV cache) and treats any later
 * cudaMalloc as an out-of-memory risk, or a latency-critical loop that
 * cannot afford cudaFree's device-wide synchronisation (mlq_linear grows
 * its per-stream workspace by free + malloc when a larger shape arrives).
 *
 * Same arguments, results and validation as mlq_linear.  The tensor-core
 * paths keep the split of x (and their partial sums) in a static
 * MLQ_NOALLOC_SCRATCH_BYTES array of the library's device module instead
 * of a workspace.  A call that mlq_linear gives the batched-decode GEMM
 * runs it in the array when its scratch fits there, else the streaming
 * GEMV (no scratch).  A call that takes the bf16 GEMM (MLQ_GEMM_ROWS_RULE(rows,
 * out_features, in_features) true, 16-B aligned weights with a 16-B multiple
 * row pitch, in_features % 8 == 0) and has rows * in_features * 4 bytes above
 * that size returns MLQ_ERR_RANGE before any CUDA call; every other call
 * takes the streaming GEMV, which needs no scratch, and is accepted at any
 * size.  The GEMM's split-K partial sums share the array: the call uses the
 * largest K split (at most mlq_linear's) whose partials fit next to the x
 * split, so it can sum in another order than mlq_linear and differ from it
 * by fp32 rounding.  The array is one per
 * device, shared by every call: calls ordered on one stream are fine,
 * calls whose kernels may overlap (several streams, several host threads)
 * race on it.  Nothing in it needs to start zeroed.  The first call on a
 * device does one-time setup (attribute queries, the scratch's address via
 * cudaGetSymbolAddress, kernel shared-memory attributes); make that first
 * call before any stream capture. */
#define MLQ_NOALLOC_SCRATCH_BYTES (16u << 20)

MLQ_API mlq_status mlq_linear_noalloc(mlq_format fmt, const void* w, size_t block_count,
                                      int out_features, int in_features, const float* x, int rows,
                                      float* y, mlq_stream stream);

/* mlq_linear plus a device bias: y[r][o] = (x W^T)[r][o] + bias[o], one fp32
 * add per output in the kernel's own store (no extra pass over y).
 * Replaces a DeviceInput linear followed by addOptionalBiasDevice
 * (src/forward.cc:384-400, used for the q/k/v biases at :432-434), whose
 * cudaElementwiseAddDeviceWeight makes the same fp32 add in a second
 * kernel.  bias: out_features floats of device memory; null = no bias. */
MLQ_API mlq_status mlq_linear_bias(mlq_format fmt, const void* w, size_t block_count,
                                   int out_features, int in_features, const float* x, int rows,
                                   const float* bias, float* y, mlq_stream stream);

/* The SwiGLU input of a feed-forward block in one call:
 *     h = silu(x W_gate^T) * (x W_up^T),   silu(v) = v / (1 + exp(-v)),
 * with the reference's fp32 steps.  Both matrices have one format and the
 * shape [out_features, in_features] (block_count blocks each); h is
 * rows x out_features.  Replaces the gate and up forwardLinearDevice calls
 * and forwardSwiGluDevice of ffnForwardDevice (src/forward.cc:573-581,
 * 361-369).  A call that takes the GEMV (see MLQ_GEMM_ROWS_RULE) is one
 * streaming launch whose row tiles carry matching rows of both matrices, so
 * gate and up are never stored; a GEMM call runs one tensor-core GEMM per
 * matrix (up into the per-stream workspace) and one elementwise pass. */
MLQ_API mlq_status mlq_linear_swiglu(mlq_format fmt, const void* w_gate, const void* w_up,
                                     size_t block_count, int out_features, int in_features,
                                     const float* x, int rows, float* h, mlq_stream stream);

/* Device weight, HOST x, HOST y, optional HOST bias[out] added to every row
 * after the product.  Replaces cudaQ80LinearDeviceWeight /
 * cudaQ40LinearDeviceWeight / cudaQ41LinearDeviceWeight
 * (cuda_quant.h:22-27, 43-48, 62-67; src/cuda_quant.cu:300-331).  Runs on
 * `device` and returns after y is on the host.  x/y may be pageable; with
 * pinned memory the copies are asynchronous DMA on `stream`. */
MLQ_API mlq_status mlq_linear_host(mlq_format fmt, const void* w, size_t block_count,
                                   int out_features, int in_features, const float* x_host,
                                   int rows, const float* bias_host, float* y_host, int device,
                                   mlq_stream stream);

/* HOST weight blocks, HOST x, HOST y, optional HOST bias.  Uploads the
 * weights for this one call.  Replaces cudaQ80Linear / cudaQ40Linear /
 * cudaQ41Linear (cuda_quant.h:17-20, 39-41, 58-60; cuda_quant.cu:289-298). */
MLQ_API mlq_status mlq_linear_host_weight(mlq_format fmt, const void* w_host, size_t block_count,
                                          int out_features, int in_features,
                                          const float* x_host, int rows, const float* bias_host,
                                          float* y_host, int device);

/* ---------------------------------------------------------------------------
 * Format conversion on the device
 * ------------------------------------------------------------------------- */

/* Blocks -> fp32 [out][in], bit-identical to the reference's
 * dequantizeFromQ80/Q40/Q41 (src/quant.cc:192-223, 304-345, 350-392). */
MLQ_API mlq_status mlq_dequantize(mlq_format fmt, const void* w, size_t block_count,
                                  int out_features, int in_features, float* dst,
                                  mlq_stream stream);

/* fp32 [rows][cols] -> blocks.  q8_0 and q4_0 are bit-identical to the
 * reference's quantizeToQ80 / quantizeToQ40 (src/quant.cc:130-190,
 * 228-302).  q4_1 has no reference quantizer; this library's rule is
 * d = (max-min)/15, m = min (fp16, the reference's encoder), codes
 * round((x - m)/d) against the stored d, m. */
MLQ_API mlq_status mlq_quantize(mlq_format fmt, const float* src, int rows, int cols,
                                void* blocks, mlq_stream stream);

/* Tensor of `src_type` (0 = fp32 values [rows][cols], or a block format)
 * -> blocks of `dst_fmt`, on the device.  Replaces the reference's
 * quantizeQtToQ80 / quantizeQtToQ40 (src/model.cc:94-149): fp32 input is
 * quantized as mlq_quantize does; block input is dequantized and
 * re-quantized per block in registers, bit-identical to the reference's
 * quantizedTensorToF32 followed by quantizeTo*; a tensor already in the
 * target format is copied unchanged (the reference leaves it as is).
 * q4_1 targets use this library's q4_1 rule (see mlq_quantize). */
MLQ_API mlq_status mlq_transcode(int src_type, const void* src, mlq_format dst_fmt, void* dst,
                                 int rows, int cols, mlq_stream stream);

/* One tensor of a model-level pass. */
typedef struct mlq_quantize_op {
    int src_type;      /* 0 = fp32, or a block format */
    const void* src;   /* device */
    int dst_fmt;       /* mlq_format */
    void* dst;         /* device: rows * ceil(cols/32) blocks */
    int rows, cols;
} mlq_quantize_op;

/* A whole model's linear weights in one call, in list order on `stream`
 * (every op validated first): the device form of quantizeModelToQ80 /
 * quantizeModelToQ40 (src/model.cc:110-149), which loop over lm_head and
 * every layer's wq, wk, wv, wo, w_gate, w_up, w_down on the host. */
MLQ_API mlq_status mlq_quantize_model(const mlq_quantize_op* ops, int n, mlq_stream stream);

/* ---------------------------------------------------------------------------
 * Row-sharded linear with the all-gather fused into the kernel
 * (one process per GPU, peers reachable over NVLink)
 *
 * The reference runs every linear on one device (cuda_weight_upload.h:46,
 * backend.h:15-19) and has no multi-GPU code.  This is the sharded form of
 * forwardLinearDevice (src/forward.cc:190-225): rank r keeps rows
 * [row_begin, row_end) of W resident (w_shard = those rows' blocks, e.g.
 * w + row_begin * ceil(in/32) blocks), computes those outputs and stores
 * them straight into EVERY rank's y over NVLink (peer_y[q] is rank q's y
 * mapped into this process, peer_y[rank] the local one; each y is
 * [rows][out_features]).  The kernel then signals the peers and waits,
 * bounded (2 s, then MLQ_ERR_TIMEOUT via mlq_device_error), until every
 * rank's rows have landed in its own y -- when it completes, y is complete
 * on this GPU.  The row ranges of all ranks must tile [0, out_features);
 * a rank may own zero rows (it then only takes part in the handshake).
 *
 * peer_flags[q] is rank q's flag buffer (mlq_flag_bytes() bytes, zeroed
 * once before the first call).  `epoch` is 1 on the first call and grows
 * by one per call on every rank, in the same call order on every rank.
 * Consecutive calls should alternate between two y buffers, so a fast rank
 * never overwrites a y a slow peer is still reading.  Requirements: weights
 * and x 16-B aligned, an even block count per row for q8_0/q4_0,
 * in_features % 4 == 0, rows <= 64, world_size <= 8.
 * ------------------------------------------------------------------------- */
MLQ_API mlq_status mlq_linear_allgather(mlq_format fmt, const void* w_shard,
                                        size_t shard_block_count, int out_features,
                                        int in_features, int row_begin, int row_end,
                                        const float* x, int rows, float* const* peer_y,
                                        uint32_t* const* peer_flags, int world_size, int rank,
                                        uint32_t epoch, mlq_stream stream);

/* Bytes of one rank's flag buffer for mlq_linear_allgather (256). */
MLQ_API size_t mlq_flag_bytes(void);

/* ---------------------------------------------------------------------------
 * Batches: every quantized matmul of one decode step in one call
 *
 * The reference's forward pass (src/forward.cc:190-225, 425-435, 574-582,
 * 741-742) makes one cudaQ*LinearDeviceInput call per matrix, each with its
 * own host round trip.  A batch launches a list of products in list order
 * on one stream with one call; the *_host form also moves every x to the
 * device and every y back with a single synchronisation for the whole list.
 * ------------------------------------------------------------------------- */

/* Row-sharded form of one product in a batch: the arguments of
 * mlq_linear_allgather that describe the shard and the gather.  The op's
 * w / block_count are this rank's shard (rows [row_begin, row_end)); its y
 * is ignored: the output lands in peer_y[rank] (and every peer's y).
 *
 * defer_wait = 0: as mlq_linear_allgather, the op's last kernel ends once
 * every rank's rows have landed in this GPU's y.  defer_wait = 1: it ends
 * after publishing this rank's epoch; whoever reads y first calls
 * mlq_gather_wait (in stream order), so a step of several sharded products
 * pays one cross-rank wait instead of one per product.  Each rank's epochs
 * must rise from op to op on one flag array: a wait for epoch E then also
 * covers every earlier epoch of that array.  mlq_linear_batch_host waits
 * before it copies the y of a deferred op back: once per flag array, for
 * the highest epoch among its deferred ops. */
typedef struct mlq_gather {
    int world_size, rank;
    int row_begin, row_end;
    float* const* peer_y;         /* world_size pointers */
    uint32_t* const* peer_flags;  /* world_size pointers */
    uint32_t epoch;
    int defer_wait;               /* 0: wait in the op; 1: mlq_gather_wait later */
} mlq_gather;

/* Waits, in stream order on `stream`, until every rank of g has published
 * an epoch >= g->epoch to this rank's flags (g->peer_flags[g->rank]): the
 * y of every deferred op with that epoch or an earlier one is then complete
 * here.  One tiny kernel, bounded (2 s, then device error code 4, see
 * mlq_device_error); nothing to launch in a world of one. */
MLQ_API mlq_status mlq_gather_wait(const mlq_gather* g, mlq_stream stream);

/* One product y[rows,out] = x[rows,in] W^T (+ bias), or -- w_up set -- the
 * SwiGLU pair h = silu(x W^T) * (x W_up^T) of mlq_linear_swiglu. */
typedef struct mlq_linear_op {
    int fmt;                   /* mlq_format */
    int out_features, in_features, rows;
    const void* w;             /* device blocks (the shard when gather != NULL) */
    const void* w_up;          /* device blocks of the up projection, or NULL */
    size_t block_count;        /* blocks of w (and of w_up) */
    const float* x;            /* device (mlq_linear_batch) or host (mlq_linear_batch_host) */
    const float* bias;         /* DEVICE [out_features] bias, or NULL (not with w_up) */
    float* y;                  /* device (mlq_linear_batch) or host (mlq_linear_batch_host) */
    const mlq_gather* gather;  /* NULL: this GPU computes every row */
} mlq_linear_op;

/* Launches ops[0..n) in order on `stream`; asynchronous.  Every op is
 * validated (as mlq_linear / mlq_linear_bias / mlq_linear_swiglu /
 * mlq_linear_allgather) before the first launch, so a batch with a bad op
 * launches nothing.  A gathered op takes no w_up.
 *
 * Consecutive ops that do not touch one another's outputs (no op's x, bias
 * or y overlaps an earlier one's y, no y overlaps an earlier x) and take
 * one row of x each -- one format, weights and x 16-byte aligned, a row
 * pitch that is a multiple of 16 bytes, in_features % 4 == 0, plain, bias
 * or gathered -- form a run: one persistent launch per
 * MLQ_BATCH_RUN_MAX_OPS ops (after one small launch that slices every op's
 * x), so the ops share the SMs instead of each paying a launch's start-up.
 * Each y equals the op run alone, bit for bit.  The gathered ops of a run
 * must share their flag arrays (world, rank, peer_flags); the launch
 * publishes once, when all its ops are done, the highest epoch among them.
 * A run uses the stream's workspace (grown on first use: make the first
 * call of the largest batch before capturing the stream in a graph). */
#define MLQ_BATCH_RUN_MAX_OPS 8
MLQ_API mlq_status mlq_linear_batch(const mlq_linear_op* ops, int n, mlq_stream stream);

/* mlq_linear_batch with HOST x and y (weights and bias on the device):
 * copies every x to device staging, launches the products, copies every y
 * back, then synchronises `stream` once.  Runs on `device`.  With pinned
 * host buffers the copies are asynchronous DMA.  Ops with the same host x
 * share one upload; consecutive ops whose host x (or y) buffers follow on
 * directly (one pinned buffer, laid out in op order, each x and y a
 * multiple of 256 bytes) share one copy.  When the y to download is large
 * (>= 256 KB), the last rows of the largest plain one-row op run as a
 * second launch while every other y is copied back on an internal stream
 * (each y is the same, bit for bit).  Calls on one device are serialised
 * (the staging is per device). */
MLQ_API mlq_status mlq_linear_batch_host(const mlq_linear_op* ops, int n, int device,
                                         mlq_stream stream);

/* Device memory shared with the other ranks' processes (CUDA IPC; plain
 * peer mappings, no multicast objects).  mlq_peer_alloc allocates `bytes`
 * on the current device, zeroes it and returns an opaque handle to send to
 * the peers; mlq_peer_open maps a peer's handle into this process (peer
 * access enabled lazily); mlq_peer_close unmaps it, mlq_peer_free frees the
 * local allocation. */
typedef struct mlq_ipc_handle {
    unsigned char bytes[64];
} mlq_ipc_handle;

MLQ_API mlq_status mlq_peer_alloc(size_t bytes, void** ptr, mlq_ipc_handle* handle);
MLQ_API mlq_status mlq_peer_open(const mlq_ipc_handle* handle, void** ptr);
MLQ_API mlq_status mlq_peer_close(void* ptr);
MLQ_API mlq_status mlq_peer_free(void* ptr);

/* ---------------------------------------------------------------------------
 * GGUF ingestion: quantized blocks from a GGUF (v3) file straight to device
 * memory.  Replaces GgufReader::load (src/gguf.cc:396-575),
 * readGgufTensorRaw (src/gguf.cc:614-662) and loadQuantizedTensor
 * (src/gguf_loader.cc:118-196), which read every tensor into host vectors
 * before the upload.  The parser makes the reference's checks (magic,
 * version 3, entry limits, repeated keys or names, 1..8 non-zero dims,
 * general.alignment a power of two <= 1 MiB, whole blocks, tensor data
 * inside the file) and fails with MLQ_ERR_FORMAT / MLQ_ERR_RANGE and a
 * message (mlq_last_error).  A 2-D tensor of dims {in, out} (fastest first,
 * as stored) is the reference's [out, in] matrix: `rows` = out, `row_bytes`
 * = ceil(in / 32) blocks; a row range is a contiguous byte range of the
 * file, so a rank of a row-sharded model reads only its own rows.
 * ------------------------------------------------------------------------- */
typedef struct mlq_gguf mlq_gguf; /* an open file: header, metadata, tensor table */

typedef struct mlq_gguf_tensor {
    const char* name;   /* valid until mlq_gguf_close */
    int n_dims;
    uint64_t dims[8];   /* fastest first */
    uint32_t type;      /* ggml type: 0 f32, 1 f16, 2 q4_0, 3 q4_1, 8 q8_0 (others: nbytes 0) */
    uint64_t offset;    /* from the start of the data section */
    uint64_t nbytes;    /* bytes of data */
    uint64_t rows;      /* product of dims[1..] */
    uint64_t row_bytes; /* nbytes / rows */
} mlq_gguf_tensor;

MLQ_API mlq_status mlq_gguf_open(const char* path, mlq_gguf** file);
MLQ_API void mlq_gguf_close(mlq_gguf* file);
MLQ_API int64_t mlq_gguf_tensor_count(const mlq_gguf* file);
/* Absolute file offset of the data section (aligned to general.alignment). */
MLQ_API uint64_t mlq_gguf_data_offset(const mlq_gguf* file);
/* Index of the tensor named `name`, or -1. */
MLQ_API int64_t mlq_gguf_find(const mlq_gguf* file, const char* name);
MLQ_API mlq_status mlq_gguf_tensor_info(const mlq_gguf* file, int64_t index, mlq_gguf_tensor* info);
/* A scalar metadata value (integer types, bool; float types for _float). */
MLQ_API mlq_status mlq_gguf_metadata_int(const mlq_gguf* file, const char* key, int64_t* value);
MLQ_API mlq_status mlq_gguf_metadata_float(const mlq_gguf* file, const char* key, double* value);

/* Rows [row_begin, row_end) of tensor `index` -- (row_end - row_begin) *
 * row_bytes bytes, byte-identical to the file -- into device memory `dst`
 * (dst_bytes at least that) on `device`, through two pinned 8 MiB staging
 * buffers per host thread (a read overlaps the previous chunk's copy);
 * returns after the copy has landed.  For a quantized matrix the result is
 * what mlq_linear takes as w (the shard of mlq_linear_allgather for a row
 * range). */
MLQ_API mlq_status mlq_gguf_upload_rows(const mlq_gguf* file, int64_t index, int64_t row_begin,
                                        int64_t row_end, void* dst, size_t dst_bytes, int device,
                                        mlq_stream stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* MLQ_H_ */
