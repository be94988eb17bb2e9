// mlq_kernels.h -- host-side launch interface of the mlq kernels (internal).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <string>

#include "mlq.h"

namespace mlq {

// Arguments of the streaming GEMV (mlq_gemv.cu).
struct GemvArgs {
    const uint8_t* w;        // packed blocks, row-major [out][bpr]
    // SwiGLU pair: a second matrix of w's shape and format (the up
    // projection, w being the gate); y = silu(x W^T) * (x W2^T).  Null: plain.
    const uint8_t* w2;
    const float* bias;       // [global rows] added to every output row, or null (not with w2)
    const float* x;          // [M][in]
    float* ys[8];            // output copies: [0] = this GPU's y, then peers' y
    int ny;                  // number of valid ys
    int row_offset;          // global index of this launch's row 0 (row shard start)
    int out, in, M;          // out = rows streamed here; M <= tokens per pass
    int bpr;                 // blocks per row
    int gpr;                 // lane-groups per row (bpr / blocks per group)
    int ktiles;              // ceil(gpr / 32)
    int nstages;             // pipeline depth (set by the dispatcher)
    int y_stride;            // row stride of y in floats
    long long row_bytes;     // bpr * block bytes
    long long total_bytes;   // out * row_bytes
    int* err;                // device error flag
    int tma2d;               // weights streamed by 2-D tensor map (set by the launcher)
    int x_resident;          // ktiles <= nstages: x tiles built once, kept for every row tile
    int x_staged;            // resident one-token mode: bytes of x copied to shared memory by one
                             // bulk copy before the x tiles are built from it (0: built from global)
    unsigned int* tiles;     // dynamic row-tile queue {next, done} of this launch, or null
    // sharded calls only (world > 1): completion handshake
    int world, rank;
    uint32_t epoch;
    uint32_t* peer_flags[8];     // rank r's flag words, mapped here
    uint32_t* local_flags;       // this rank's flag words (world entries)
    unsigned int* done_counter;  // this rank's CTA completion counter
    int wait;                    // 1: wait for every rank after publishing; 0: publish only
    // ordering with the previous kernel (programmatic dependent launch):
    // kPdlNormal waits for it before reading x, and lets the next kernel
    // start at once; kPdlFirst waits too, but lets the next kernel start only
    // after that wait; kPdlNoWait reads x at once (the previous kernel was a
    // kPdlFirst / kPdlNoWait launch whose outputs this one does not touch)
    int pdl_mode;
};

constexpr int kMaxWorld = 8;

// Tokens per pass for `rows_left` remaining rows of x: 1, 2, 4 or 8.
int gemv_tokens_per_pass(int rows_left);

// Streaming GEMV, tokens-per-pass `mt` in {1,2,4,8}; persistent grid of one
// or two CTAs per SM (`sm_count` SMs with `smem_per_sm` bytes of shared
// memory each).  Needs no workspace.
cudaError_t launch_gemv_stream(int fmt, const GemvArgs& args, int mt, int sm_count,
                               int smem_per_sm, cudaStream_t stream);

// A run of independent one-row products in one persistent launch (plus a
// small launch that slices every op's x once into the workspace): one
// tile queue over all ops' row tiles, so the ops do not each pay a launch's
// start-up.  All ops of a run share the format.
constexpr int kGemvRunMaxOps = MLQ_BATCH_RUN_MAX_OPS;
struct GemvRunOp {
    const uint8_t* w;    // the op's `out` rows (null allowed when out == 0)
    const float* x;      // [in], one row
    const float* bias;   // [out] (the op's rows) or null
    int out, in;
    // Where the rows go: y[d][row_offset + i] for d < ny.  A plain op: ny 1,
    // row_offset 0.  A row-sharded op (world > 1): every rank's y (ny =
    // world, this rank's at index rank), after which the launch publishes
    // epoch to every rank's flags (the streaming GEMV's sharded protocol).
    float* y[kMaxWorld];
    int ny, row_offset;
    int world, rank;
    uint32_t* flags[kMaxWorld];  // every rank's flag words (world > 1)
    unsigned int* done_counter;  // this rank's CTA completion counter (world > 1)
    uint32_t epoch;
    int wait;                    // 1: wait for every rank after publishing
};

// True when an op can join a run: one row of x, weights and x 16-B aligned
// with a 16-B multiple row pitch (2-D tensor map), whole lane-groups per
// row, in % 4 == 0, and the driver's tensor-map encoder reachable.  The
// sharded ops of one run must share world, rank and flag words
// (gemv_run_compatible).
bool gemv_run_ok(int fmt, const GemvRunOp& op);
bool gemv_run_compatible(const GemvRunOp& a, const GemvRunOp& b);

// Workspace of a run: the sliced x tiles of every op.
size_t gemv_run_workspace_bytes(int fmt, const GemvRunOp* ops, int nop);

// y[k] = x[k] W[k]^T (+ bias[k]) for nop <= kGemvRunMaxOps ops that pass
// gemv_run_ok and do not touch one another's outputs; waits for the
// previous kernel on the stream before reading any x, bias or writing y.
cudaError_t launch_gemv_run(int fmt, const GemvRunOp* ops, int nop, void* ws, int sm_count, int smem_per_sm,
                            int* err, cudaStream_t stream);

// Sets the message mlq_last_error() returns on this host thread.
void set_last_error(const char* msg);
inline void set_last_error(const std::string& msg) { set_last_error(msg.c_str()); }

// Zeroes the streaming GEMV's dynamic tile-queue ring of the current device
// (called after a kernel reported an error, the device synchronised).
cudaError_t reset_tile_queues();

// Any-alignment fallback GEMV (one warp per output row).
cudaError_t launch_gemv_generic(int fmt, const uint8_t* w, const float* x, float* y, int out,
                                int in, int M, int bpr, cudaStream_t stream);

// Arguments of the tensor-core GEMM (mlq_gemm.cu).
struct GemmArgs {
    float* y;      // [T][out]
    const float* bias;  // [out] added to every row of y, or null
    int out, in;   // W is [out][in] in blocks
    int T;         // rows of x (tokens)
    int* err;      // device error flag
    // split-K: the K extent in `split` ranges (whole 256-value W chunks),
    // each tile's partial sums to part[range][T][out], summed in range
    // order by a second kernel.  split == 1: y directly.
    int split;
    int kchunks_per_split;  // W chunks (KSUB K-steps each) per range
    float* part;
};

// True when the tcgen05 GEMM takes this call: MLQ_GEMM_ROWS_RULE(rows, out, in), weights 16-B
// aligned with a 16-B multiple row pitch, in % 8 == 0 (gemm_shape_ok, host values only), and
// the driver's tensor-map encoder is reachable.
bool gemm_shape_ok(int fmt, const void* w, int out, int in, int rows);
bool gemm_supported(int fmt, const void* w, int out, int in, int rows);

// Split-K ranges for a GEMM call on `sm_count` SMs: 1 when its output
// tiles already occupy the SMs, else enough ranges to (about) fill them.
int gemm_split(int out, int in, int rows, int sm_count);

// Workspace bytes of the GEMM: x split into bf16 hi/lo, plus the partial
// sums of `split` K ranges when split > 1.
size_t gemm_workspace_bytes(int in, int rows, int out, int split);

// y[T][out] = x[T][in] * W^T (+ bias[out], when not null) on the tensor
// cores, over `split` K ranges (gemm_split); ws holds
// gemm_workspace_bytes(in, rows, out, split) bytes.
cudaError_t launch_gemm(int fmt, const uint8_t* w, const float* x, float* y, int out, int in, int rows,
                        const float* bias, void* ws, int split, int sm_count, int* err, cudaStream_t stream);

// Batched-decode GEMM (mlq_bgemm.cu): 2..kBgemmMaxRows rows of x on the
// tensor cores with exact fp16 weight codes, x split per token into fp16
// hi / lo, and per-block fp32 folds.  Two launches: the x split, the GEMM.
constexpr int kBgemmMaxRows = MLQ_BGEMM_MAX_ROWS;

// Host-value conditions of the batched-decode GEMM: 2 <= rows <= 32,
// in % 32 == 0, 16-B aligned weights with a 16-B multiple row pitch, at
// most 2^23 (row tile, block) units.
bool bgemm_shape_ok(int fmt, const void* w, int out, int in, int rows);

// Workspace of one launch: x split (fp16 hi/lo), token exponents (and q4_1
// block sums), split-tile counters and the split row tiles' partial sums.
size_t bgemm_workspace_bytes(int fmt, int in, int rows, int out, int sm_count);

// A row-sharded call (world > 1): this rank's `out` rows are rows
// [row_offset, row_offset + out) of a y with y_stride features; every value
// is stored to each rank's y (ys[r], peer memory), then the launch's last
// CTA publishes `epoch` to every rank's flags and waits (bounded) for every
// rank's (the streaming GEMV's sharded-call protocol).
struct BgemmGather {
    int world = 1, rank = 0;
    int row_offset = 0, y_stride = 0;
    float* ys[kMaxWorld] = {};
    uint32_t epoch = 0;
    uint32_t* peer_flags[kMaxWorld] = {};
    uint32_t* local_flags = nullptr;
    unsigned int* done_counter = nullptr;
    int wait = 1;  // 1: wait for every rank after publishing; 0: publish only
};

constexpr int kPdlNormal = 0, kPdlFirst = 1, kPdlNoWait = 2;

// An empty kernel launched without programmatic dependent launch: it and
// everything after it on the stream start once every earlier kernel has
// completed (closes a run of kPdlNoWait launches).
cudaError_t launch_join(cudaStream_t stream);

// Waits (bounded, one thread) until local_flags[r] >= epoch for every
// rank r < world: the deferred half of a sharded call's handshake.
cudaError_t launch_gather_wait(const uint32_t* local_flags, int world, uint32_t epoch, int* err,
                               cudaStream_t stream);

// Matrices one batched-decode launch may compute (sharing x).
constexpr int kBgemmMaxGroup = 4;

// Workspace of a grouped launch over nmat matrices of out[m] rows.
size_t bgemm_group_workspace_bytes(int fmt, int in, int rows, const int* out, int nmat, int sm_count);

// y[m][rows][out[m]] = x W[m]^T (+ bias[m]) for nmat <= kBgemmMaxGroup
// matrices sharing x, format and in_features (each bgemm_shape_ok): one x
// split, one GEMM launch over all their row tiles.  bias may be null, or an
// array of nmat (possibly null) pointers.
cudaError_t launch_bgemm_group(int fmt, int nmat, const uint8_t* const* w, float* const* y, const int* out,
                               const float* const* bias, const float* x, int in, int rows, void* ws, int sm_count,
                               int* err, cudaStream_t stream);

// y[rows][out] = x W^T (+ bias); ws holds bgemm_workspace_bytes(...) bytes.
// With g (a sharded call), y is unused: the output goes to g->ys.
cudaError_t launch_bgemm(int fmt, const uint8_t* w, const float* x, float* y, int out, int in, int rows,
                         const float* bias, void* ws, int sm_count, int* err, cudaStream_t stream,
                         const BgemmGather* g = nullptr);

// Quantize fp32 [rows][cols] -> blocks, reference rules (mlq_convert.cu).
cudaError_t launch_quantize(int fmt, const float* src, long long rows, int cols, uint8_t* blocks,
                            cudaStream_t stream);

// Blocks -> fp32 [rows][cols], reference rules (mlq_convert.cu).
cudaError_t launch_dequantize(int fmt, const uint8_t* blocks, long long rows, int cols, float* dst,
                              cudaStream_t stream);

// Blocks of one format -> blocks of another (formats differ): the
// reference's dequantize then quantize per block, bit for bit.
cudaError_t launch_transcode(int src_fmt, const uint8_t* src, int dst_fmt, uint8_t* dst, long long rows, int cols,
                             cudaStream_t stream);

// y[r][c] += bias[c] for r < rows, c < cols.
cudaError_t launch_add_bias(float* y, const float* bias, int rows, int cols, cudaStream_t stream);

// h[i] = silu(h[i]) * u[i] for i < n (silu(v) = v / (1 + exp(-v))).
cudaError_t launch_swiglu(float* h, const float* u, long long n, cudaStream_t stream);

}  // namespace mlq
