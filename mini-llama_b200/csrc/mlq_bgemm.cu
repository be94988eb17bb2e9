// mlq_bgemm.cu -- batched-decode GEMM on the tensor cores: 3..32 rows of x
// against a quantized matrix, the regime of batched decoding (a handful of
// sequences, one new token each) where the work is still bound by reading
// the weights once, but too many rows for the CUDA-core GEMV.
//
// The reference decodes a batch one token at a time through its GEMV
// (forwardBatch -> forwardToken, src/batch.cc:32-55; q80/q40/q41LinearKernel,
// src/cuda_quant.cu:78-182).  Same arithmetic contract here: exact weights,
// fp32-level activations, fp32 accumulation; only the summation order
// differs.
//
// Arithmetic, per 32-value block b of a weight row and token t:
//   * The block's integer codes go to the tensor cores as fp16 values,
//     exactly: q8_0 q in [-128, 127], q4_0 q - 8 in [-8, 7], q4_1 q in
//     [0, 15].  (One byte permute drops a code into the mantissa of 1024.0,
//     one packed subtract removes the 1024 + offset: ~1.3 operations per
//     weight, one fp16 A tile.)
//   * x is scaled per token by a power of two s_t > max|x_t| over the whole
//     row and split x/s_t = xh + xl into two fp16 values (xsplit kernel
//     below): exact to 2^-25 of s_t, the level of one fp32 rounding of the
//     token's largest value.
//   * Per block, the tensor cores form Dh[row][t] = sum q xh and Dl[row][t] =
//     sum q xl in one TMEM accumulator of the block: two kind::f16 MMAs of
//     128 x N x 16, N = 2 x padded tokens (the hi and lo rows of x, per
//     half of the tokens, are the B operand).  An MMA costs about the same
//     for any N up to 64, so hi and lo share one instruction.
//   * CUDA-core "fold" warps read the block's accumulator and add
//     d * (Dh + Dl) (+ m * sum(x / s_t) for q4_1) to the fp32 total of
//     (row, t); the total is multiplied by s_t once, when it is stored.  The
//     block scales never enter the tensor-core sums.
//
// CTA = 18 warps, one CTA per SM:
//   warp 0      TMA producer: W chunks (8 blocks x 128 rows, 2-D tensor map
//               over the AoS bytes) and the chunk's x tiles (fp16 [hi; lo],
//               128-B swizzle).
//   warp 1      TMEM allocation; lane 0 issues the MMAs and commits.
//   warps 2-9   decode: two threads per W row, each turning its half of an
//               A stage's blocks into fp16 codes in TMEM (the MMA's A
//               operand).
//   warps 10-17 fold: thread = W row = TMEM lane; two warps per lane
//               quarter, one per half of the tokens; a block's scale d (and
//               q4_1 minimum m) is read from the W chunk in shared memory.
// A stage's blocks (four; two with 32 padded tokens) are committed as one
// TMEM group: one barrier per stage between the MMA thread and the decode /
// fold warps.
// Work split ("stream-K"): the matrix is a list of (row tile, block) units;
// CTA c takes the contiguous range [c W / G, (c + 1) W / G).  A row tile a
// CTA covers whole is stored straight to y; the at most two partly covered
// tiles at the ends of its range go to a workspace, and the last CTA to
// finish a split tile (a counter per tile) adds its parts in CTA order
// (deterministic) plus the bias.
// Two launches per call: the x split, then the GEMM, each with programmatic
// dependent launch (the GEMM streams its first weight chunks while the split
// runs).  Every mbarrier wait is bounded (2 s); no TMA multicast anywhere.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <type_traits>

#include "mlq.h"
#include "mlq_device.cuh"
#include "mlq_kernels.h"
#include "mlq_tc.cuh"
#include "mlq_tmap.h"

namespace mlq {
namespace {

constexpr int BM = 128;             // W rows per tile = MMA M = TMEM lanes
constexpr int KC = 256;             // values per W chunk
constexpr int BPC = KC / kQK;       // blocks per chunk (8)
constexpr int kDecodeWarps = 8;     // warps 2..9: two per row
// fold warps from warp 10 on: two per TMEM lane quarter, one per half of
// the tokens (measured faster than one per quarter at 8, 16 and 32 padded
// tokens, though 18 warps leave 96 registers per thread, 14 leave 128)
constexpr int kFoldWarp0 = 2 + kDecodeWarps;
constexpr int fold_warps(int) { return 8; }
constexpr int threads_of(int tp) { return 32 * (2 + kDecodeWarps + fold_warps(tp)); }
constexpr int kSmemMax = 232448 - 1024;  // dynamic shared memory per CTA: 227 KB less the static part
constexpr int kMinBlocksPerCta = 16;

constexpr int cmin(int a, int b) { return a < b ? a : b; }
constexpr int kBadExp = 0x7fffffff;  // token exponent of an x row holding NaN / Inf
constexpr unsigned int kBgemmDonePoison = 1u << 16;  // added to the completion count by a CTA that gave up

// the weights' tensor maps of a launch's matrices
struct WMaps {
    CUtensorMap m[kBgemmMaxGroup];
};

// TP: padded tokens (8, 16 or 32); the MMA's N is 2 TP: per half of the
// tokens, their hi rows of x then their lo rows (so a fold warp's columns,
// one half's hi and lo, are adjacent in TMEM: one load per block).
template <int F, int TP>
struct BCfg {
    static constexpr int BS = Fmt<F>::kBlockBytes;
    static constexpr int N = 2 * TP;
    // blocks per A stage = per TMEM accumulator group: 4 (K = 128), or 2 at
    // 32 tokens so that three groups still fit
    static constexpr int SB = TP == 32 ? 2 : 4;
    static constexpr int SPC = BPC / SB;               // A stages per chunk
    static constexpr int W_ROW = BPC * BS;             // 272 / 144 / 160 bytes of a row's chunk
    static constexpr int W_ESZ = F == kQ8_0 ? 2 : 1;   // tensor-map element (inner box <= 256 elements)
    static constexpr int W_TILE = BM * W_ROW;
    static constexpr int B_SUB = 2 * TP * 128;         // [hi; lo] x tile of 64 values (fp16, 128-B rows)
    static constexpr int B_TILE = (KC / 64) * B_SUB;
    // q4_1: the chunk's x block sums, [8 blocks][TP] floats
    static constexpr int SC_BYTES = F == kQ4_1 ? BPC * TP * 4 : 0;
    static constexpr int C_STAGE = (W_TILE + B_TILE + SC_BYTES + 1023) / 1024 * 1024;  // W, x tiles, x sums
    // A (fp16 codes) lives in TMEM: a block is 32 values x 2 B / 4 B per
    // column = 16 columns; 128 columns of A stages, the accumulator groups
    // (SB blocks x N columns each) take the rest of the 512 columns
    static constexpr int A_COLS = SB * kQK / 2;
    static constexpr int AS = 128 / A_COLS;
    static constexpr int ACC_COL0 = 128;
    static constexpr int NG = cmin(8, (512 - ACC_COL0) / (SB * N));
    static constexpr uint32_t TMEM_COLS = 512;
    static constexpr int fixed = 1024;                 // 1024-B alignment slack
    static constexpr int CS = cmin(4, (kSmemMax - fixed) / C_STAGE);
    // at least half an SM's shared memory, so no two CTAs share an SM (each
    // allocates all 512 TMEM columns)
    static constexpr int SMEM = CS * C_STAGE + fixed < 120 * 1024 ? 120 * 1024 : CS * C_STAGE + fixed;
    static_assert(NG >= 1 && CS >= 2, "bgemm stages must fit");
    static_assert(SMEM <= kSmemMax, "bgemm stages must fit shared memory");
    static_assert(W_TILE % 1024 == 0 && B_SUB % 1024 == 0,
                  "SW128 tiles need 1024-B alignment");
    static_assert(W_ROW % 16 == 0, "W chunk row must be 16-byte granular");
};

// A launch computes 1..kBgemmMaxGroup matrices that share x (and the
// format and in_features): their row tiles one after another, tiles
// [tile0[m], tile0[m + 1]) being matrix m's.
struct BgemmArgs {
    int nmat;
    int tile0[kBgemmMaxGroup + 1];
    int out_m[kBgemmMaxGroup];             // rows of matrix m
    float* ym[kBgemmMaxGroup];             // y of matrix m, [T][out_m] (nmat > 1)
    const float* bias_m[kBgemmMaxGroup];   // bias of matrix m ([out_m]) or null
    // nmat == 1: output copies (this GPU's y, then -- sharded -- the peers'), [T][y_stride]
    float* ys[kMaxWorld];
    int ny;                // copies
    int y_stride;          // features of a y row
    int row_offset;        // y column of this launch's row 0
    const int* tok_exp;   // [TP]: x row t was scaled by 2^-tok_exp[t] (kBadExp: it holds NaN / Inf)
    const float* xsum;    // [kb rounded up to 8][TP]: block sums of the scaled x (q4_1), else null
    float* part;          // [grid][2][TP][BM]: partial sums of partly covered row tiles
    int* tile_cnt;        // [row tiles]: CTAs done with a split tile (zeroed by the x-split kernel)
    // sharded calls (world > 1): the completion handshake
    int world, rank;
    uint32_t epoch;
    uint32_t* peer_flags[kMaxWorld];
    uint32_t* local_flags;
    unsigned int* done_counter;
    int wait;  // 1: wait for every rank after publishing; 0: publish only
    int in, T, kb;        // kb = blocks per row
    int total;            // units = row tiles x kb (<= kMaxUnits)
    int* err;
};

// The units [f0, f1) of CTA c among G.  total x G < 2^31 (kMaxUnits and at
// most 256 CTAs), so 32-bit arithmetic (a 64-bit division costs hundreds of
// instructions on the device).
constexpr int kMaxUnits = 1 << 23;
__host__ __device__ __forceinline__ int unit_begin(int total, int c, int G) {
    return (int)((unsigned)c * (unsigned)total / (unsigned)G);
}

// fp16 codes of one block (32 values) as 16 half2 words, element order.
// Bytes b of a word u become half(1024 + b) by a byte permute under 0x64;
// the packed subtract of `off` (1024 + the format's code offset) is exact.
__device__ __forceinline__ uint32_t h2_sub(uint32_t h, uint32_t off2) {
    __half2 r = __hsub2(*reinterpret_cast<const __half2*>(&h), *reinterpret_cast<const __half2*>(&off2));
    return *reinterpret_cast<const uint32_t*>(&r);
}

template <int F>
__device__ __forceinline__ void codes_f16(const uint32_t* qw, uint32_t (&c)[16]) {
    if constexpr (F == kQ8_0) {
        const uint32_t off2 = 0x64806480u;  // half2(1152, 1152): 1024 + 128
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t u = qw[i] ^ 0x80808080u;  // q + 128, one byte each
            c[2 * i] = h2_sub(__byte_perm(u, 0x64646464u, 0x4140), off2);
            c[2 * i + 1] = h2_sub(__byte_perm(u, 0x64646464u, 0x4342), off2);
        }
    } else {
        const uint32_t off2 = F == kQ4_0 ? 0x64086408u : 0x64006400u;  // 1024 + 8 / 1024
#pragma unroll
        for (int i = 0; i < 4; ++i) {  // qs word i: elements 4i.. (low nibbles), 16 + 4i.. (high)
            const uint32_t lo = qw[i] & 0x0F0F0F0Fu, hi = (qw[i] >> 4) & 0x0F0F0F0Fu;
            c[2 * i] = h2_sub(__byte_perm(lo, 0x64646464u, 0x4140), off2);
            c[2 * i + 1] = h2_sub(__byte_perm(lo, 0x64646464u, 0x4342), off2);
            c[8 + 2 * i] = h2_sub(__byte_perm(hi, 0x64646464u, 0x4140), off2);
            c[9 + 2 * i] = h2_sub(__byte_perm(hi, 0x64646464u, 0x4342), off2);
        }
    }
}

// Walks the CTA's range chunk by chunk: fn(tile, chunk, b_lo, b_hi) with
// [b_lo, b_hi) the blocks of the tile's row that the CTA covers.
template <typename Fn>
__device__ __forceinline__ void for_each_chunk(int f0, int f1, int kb, Fn&& fn) {
    if (f1 <= f0) return;
    const int t0 = f0 / kb, t1 = (f1 - 1) / kb;
    for (int t = t0; t <= t1; ++t) {
        const int b_lo = f0 > t * kb ? f0 - t * kb : 0;
        const int b_hi = f1 < (t + 1) * kb ? f1 - t * kb : kb;
        for (int c = b_lo / BPC; c <= (b_hi - 1) / BPC; ++c)
            if (!fn(t, c, b_lo, b_hi)) return;
    }
}

template <int F, int TP>
__global__ void __launch_bounds__(threads_of(TP), 1)
    bgemm_kernel(const __grid_constant__ WMaps tm_w, const __grid_constant__ CUtensorMap tm_x, BgemmArgs a) {
    using C = BCfg<F, TP>;
    constexpr int CS = C::CS, AS = C::AS, NG = C::NG, N = C::N, SB = C::SB, SPC = C::SPC;
    constexpr int kFoldWarps = fold_warps(TP), kThreads = threads_of(TP);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t c_full[CS], c_empty[CS], a_full[AS], a_empty[AS];
    __shared__ __align__(8) uint64_t g_full[NG], g_empty[NG];
    __shared__ __align__(8) uint64_t drain_bar, end_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_flag;
    __shared__ int fix_tile[2];  // split tiles (first / last of the range) this CTA finished last, else -1
    __shared__ int tok_exp_s[TP];  // the token exponents (fold warps, after the x split)

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    auto w_st = [&](int s) { return base + (uint32_t)(s * C::C_STAGE); };
    auto x_st = [&](int s) { return w_st(s) + (uint32_t)C::W_TILE; };
    auto sc_st = [&](int s) { return x_st(s) + (uint32_t)C::B_TILE; };  // q4_1: [8][TP] x block sums

    if (threadIdx.x == 0) {
        for (int s = 0; s < CS; ++s) {
            mbar_init(smem_u32(&c_full[s]), 1);
            // decode warps (W codes), fold warps (W scales) and the chunk's last MMA commit (x tiles)
            mbar_init(smem_u32(&c_empty[s]), kDecodeWarps + kFoldWarps + 1);
        }
        for (int s = 0; s < AS; ++s) {
            mbar_init(smem_u32(&a_full[s]), kDecodeWarps);
            mbar_init(smem_u32(&a_empty[s]), 1);
        }
        for (int g = 0; g < NG; ++g) {
            mbar_init(smem_u32(&g_full[g]), 1);
            mbar_init(smem_u32(&g_empty[g]), kFoldWarps);
        }
        mbar_init(smem_u32(&drain_bar), 1);
        mbar_init(smem_u32(&end_bar), kThreads / 32);
        abort_flag = 0;
        fix_tile[0] = fix_tile[1] = -1;
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_base_s), C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    // the next kernel on the stream may be scheduled; whatever it reads from
    // this one, it waits for this grid to complete
    launch_dependents();

    const int G = gridDim.x;
    const int f0 = unit_begin(a.total, blockIdx.x, G), f1 = unit_begin(a.total, blockIdx.x + 1, G);
    auto aborted = [&]() { return *(volatile int*)&abort_flag != 0; };
    auto fail = [&](int code) {
        report_error(a.err, code);
        abort_flag = 1;
    };
    // the fold warps' own barrier (named barrier 1)
    auto fold_bar_sync = [&]() { asm volatile("bar.sync 1, %0;" ::"n"(kFoldWarps * 32) : "memory"); };
    // Per-matrix arguments by constant indices only: a kernel-parameter
    // array indexed at run time is read far more slowly.
    auto pick = [](const auto& arr, int m) {
        auto v = arr[0];
#pragma unroll
        for (int k = 1; k < kBgemmMaxGroup; ++k)
            if (m == k) v = arr[k];
        return v;
    };
    // the matrix of row tile t
    auto mat_of = [&](int t) {
        int m = 0;
#pragma unroll
        for (int k = 1; k < kBgemmMaxGroup; ++k)
            if (k < a.nmat && t >= a.tile0[k]) m = k;
        return m;
    };
    // y of token tt from an unscaled total: times 2^e_t (a multiply by an
    // exact power of two while 2^e_t is a normal float: the same correctly
    // rounded result as ldexpf), plus the bias bo if has_bias
    auto scaled = [&](int tt, float v, bool has_bias, float bo) {
        const int e = tok_exp_s[tt];
        if (e >= -126 && e <= 127) v = __fmul_rn(v, __int_as_float((e + 127) << 23));
        else v = e == kBadExp ? __int_as_float(0x7fc00000) : ldexpf(v, e);
        return has_bias ? __fadd_rn(v, bo) : v;
    };
    // where matrix m's row o of token 0 goes, and the stride between tokens
    auto y_row = [&](int m, int o, long long& stride) {
        if (a.nmat == 1) {
            stride = a.y_stride;
            return a.ys[0] + a.row_offset + o;
        }
        stride = pick(a.out_m, m);
        return pick(a.ym, m) + o;
    };
    // the stores of one value: y, and -- sharded -- every peer's y
    auto store_y = [&](float* yp, long long off, float v) {
        yp[off] = v;
        if (a.ny > 1) {
            const long long base = yp + off - a.ys[0];
#pragma unroll
            for (int d = 1; d < kMaxWorld; ++d)
                if (d < a.ny) a.ys[d][base] = v;
        }
    };
    // the CTAs [c0, c1] whose ranges cover row tile t
    auto tile_ctas = [&](int t, int& c0, int& c1) {
        const int u0 = t * a.kb, u1 = u0 + a.kb - 1;
        c0 = (int)((unsigned)u0 * (unsigned)G / (unsigned)a.total);
        c1 = (int)((unsigned)u1 * (unsigned)G / (unsigned)a.total);
        while (c0 + 1 < G && unit_begin(a.total, c0 + 1, G) <= u0) ++c0;
        while (c0 > 0 && unit_begin(a.total, c0, G) > u0) --c0;
        while (c1 + 1 < G && unit_begin(a.total, c1 + 1, G) <= u1) ++c1;
        while (c1 > 0 && unit_begin(a.total, c1, G) > u1) --c1;
    };
    // valid-block mask of A stage j of chunk c (bit b: block c * 8 + SB j + b)
    auto stage_mask = [&](int c, int j, int b_lo, int b_hi) {
        unsigned m = 0;
#pragma unroll
        for (int b = 0; b < SB; ++b) {
            const int k = c * BPC + SB * j + b;
            if (k >= b_lo && k < b_hi) m |= 1u << b;
        }
        return m;
    };

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            // The weights are read-only here: the first CS chunks of W are
            // requested before the wait for the x-split kernel (programmatic
            // dependent launch), their x tiles (and x sums) after it.
            auto issue_x = [&](int s, int c) {
                const uint32_t fb = smem_u32(&c_full[s]);
#pragma unroll
                for (int q = 0; q < KC / 64; ++q) tma_load_2d(x_st(s) + (uint32_t)(q * C::B_SUB), &tm_x, c * KC + q * 64, 0, fb);
                // q4_1: x block sums of the chunk's 8 blocks (the array is
                // padded to whole chunks, so this never reads past it)
                if constexpr (F == kQ4_1)
                    bulk_g2s(sc_st(s), a.xsum + (long long)c * BPC * TP, (uint32_t)(BPC * TP * 4), fb);
            };
            int pend_s[CS], pend_c[CS], npend = 0;
            bool dep = false;
            auto flush_pending = [&]() {
                grid_dependency_wait();
                dep = true;
                for (int k = 0; k < npend; ++k) issue_x(pend_s[k], pend_c[k]);
                npend = 0;
            };
            uint32_t cseq = 0;
            for_each_chunk(f0, f1, a.kb, [&](int t, int c, int, int) {
                const int s = (int)(cseq % CS);
                if (!mbar_wait(smem_u32(&c_empty[s]), ((cseq / CS) & 1u) ^ 1u)) {
                    fail(20);
                    return false;
                }
                if (aborted()) return false;
                const uint32_t fb = smem_u32(&c_full[s]);
                mbar_arrive_expect_tx(fb, (uint32_t)(C::W_TILE + C::B_TILE + C::SC_BYTES));
                const int m = mat_of(t);
                tma_load_2d(w_st(s), &tm_w.m[m], c * (C::W_ROW / C::W_ESZ), (t - pick(a.tile0, m)) * BM, fb);
                if (dep) {
                    issue_x(s, c);
                } else {
                    pend_s[npend] = s;
                    pend_c[npend] = c;
                    if (++npend == CS) flush_pending();
                }
                ++cseq;
                return true;
            });
            if (!dep) flush_pending();
            // the CTA's shared memory must outlive every copy still landing
            for (uint32_t k = cseq >= (uint32_t)CS ? cseq - CS : 0; k < cseq; ++k)
                if (!mbar_wait(smem_u32(&c_full[k % CS]), (k / CS) & 1u)) {
                    report_error(a.err, 21);
                    break;
                }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        // per A stage: its valid blocks, each into its own accumulator of the
        // stage's TMEM group, one commit for the group and one for the A stage
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_f16kind(false, BM, N);
            uint32_t cseq = 0, aseq = 0;
            for_each_chunk(f0, f1, a.kb, [&](int, int c, int b_lo, int b_hi) {
                const int cs = (int)(cseq % CS);
                // operand addresses: per-stage bases plus compile-time offsets
                const uint64_t bd0 = sw128_desc(x_st(cs));
#pragma unroll
                for (int j = 0; j < SPC; ++j) {
                    const unsigned m = stage_mask(c, j, b_lo, b_hi);
                    if (!m) continue;
                    const int as = (int)(aseq % AS), g = (int)(aseq % NG);
                    // The one wait per stage: the decode warps arrive on a_full
                    // after their own waits for the chunk's tiles (c_full) and
                    // for the fold to release the stage's accumulator group
                    // (g_empty).  Each wait here sits between MMAs and idles
                    // the tensor pipe for its latency.
                    if (!mbar_wait(smem_u32(&a_full[as]), (aseq / AS) & 1u)) {
                        fail(22);
                        return false;
                    }
                    tc_fence_after();
                    const uint32_t ta0 = tmem + (uint32_t)(as * C::A_COLS);
                    const uint32_t td0 = tmem + (uint32_t)(C::ACC_COL0 + g * SB * N);
#pragma unroll
                    for (int b = 0; b < SB; ++b) {
                        if (!(m >> b & 1u)) continue;
                        const int k = SB * j + b;  // block of the chunk: x sub-tile k / 2, K bytes (k & 1) * 64
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {
                            // A: the block's 16 columns in TMEM (8 per K = 16);
                            // B: all 2 TP rows (hi, lo) of the sub-tile
                            const uint64_t boff = (uint64_t)(((k >> 1) * C::B_SUB + (k & 1) * 64 + kk * 32) >> 4);
                            mma_f16kind_ta(td0 + (uint32_t)(b * N), ta0 + (uint32_t)(b * 16 + kk * 8), bd0 + boff,
                                           idesc, kk);
                        }
                    }
                    mma_commit(smem_u32(&g_full[g]));
                    mma_commit(smem_u32(&a_empty[as]));
                    ++aseq;
                }
                mma_commit(smem_u32(&c_empty[cs]));  // the chunk's x tiles are read
                ++cseq;
                return true;
            });
            // every MMA issued has completed before TMEM goes away
            mma_commit(smem_u32(&drain_bar));
            if (!mbar_wait(smem_u32(&drain_bar), 0u)) report_error(a.err, 23);
        }
    } else if (warp < kFoldWarp0) {
        // --------------------- decode: codes -> fp16 A tiles ---------------------
        // two threads per W row, `half` h: with four blocks per stage, blocks
        // 2h and 2h + 1 of the stage; with two, block h
        // a warp writes only its TMEM lane quarter (warp % 4): its rows
        const int row = (warp & 3) * 32 + lane;
        const int half = (warp - 2) >> 2;
        const uint32_t tlane = tmem + ((uint32_t)((warp & 3) * 32) << 16);
        uint32_t cseq = 0, aseq = 0;
        for_each_chunk(f0, f1, a.kb, [&](int, int c, int b_lo, int b_hi) {
            const int cs = (int)(cseq % CS);
            if (!mbar_wait(smem_u32(&c_full[cs]), (cseq / CS) & 1u)) {
                fail(24);
                return false;
            }
            const uint32_t wrow = w_st(cs) + (uint32_t)(row * C::W_ROW);
#pragma unroll
            for (int j = 0; j < SPC; ++j) {
                const unsigned m = stage_mask(c, j, b_lo, b_hi);
                if (!m) continue;
                const int as = (int)(aseq % AS);
                if (!mbar_wait(smem_u32(&a_empty[as]), ((aseq / AS) & 1u) ^ 1u)) {
                    fail(24);
                    return false;
                }
                if (aborted()) return false;
                tc_fence_after();  // the MMAs that read this A stage are complete
                // the pair of blocks this thread reads (pb, pb + 1 of the chunk:
                // 4 j + 2 half, or 2 j) and the ones of them it decodes (bit h:
                // block pb + h)
                const unsigned mine = SB == 4 ? (m >> (2 * half)) & 3u : m & (1u << half);
                // the two halves as compile-time cases, so every register index
                // below is a constant
                auto decode_half = [&](auto HALF) {
                    constexpr int half = decltype(HALF)::value;
                    // the pair: 2 BS bytes from byte pb BS of the row's chunk (pb
                    // even: a word boundary), read as the 16-B units that cover
                    // them (rows are 17 / 9 / 10 units apart: the 8 lanes of a
                    // load phase hit distinct bank groups)
                    constexpr int NW = 2 * C::BS / 4;
                    const int pbc = SB == 4 ? SB * j + 2 * half : SB * j;  // pb, from the compile-time half
                    const int sb = pbc * C::BS;
                    const int sh = (sb % 16) / 4;
                    const int nu = (sh * 4 + 2 * C::BS + 15) / 16;
                    uint32_t wb[24];
#pragma unroll
                    for (int u = 0; u < 6; ++u) {
                        if (u < nu) {
                            const uint4 t4 = lds_u4(wrow + (uint32_t)(16 * (sb / 16 + u)));
                            wb[4 * u] = t4.x;
                            wb[4 * u + 1] = t4.y;
                            wb[4 * u + 2] = t4.z;
                            wb[4 * u + 3] = t4.w;
                        }
                    }
                    uint32_t w[NW + 1];
#pragma unroll
                    for (int i = 0; i < NW; ++i) w[i] = wb[i + sh];
                    w[NW] = 0;
                    const uint32_t arow = tlane + (uint32_t)(as * C::A_COLS + (pbc - SB * j) * 16);
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        if (!(mine >> h & 1u)) continue;  // no MMA reads this block
                        uint32_t qw[8];
                        if constexpr (F == kQ8_0) {
                            // block 0: codes at bytes 2..33; block 1: 36..67
#pragma unroll
                            for (int i = 0; i < 8; ++i) qw[i] = h ? w[9 + i] : __funnelshift_r(w[i], w[i + 1], 16);
                        } else if constexpr (F == kQ4_0) {
                            // block 0: qs at bytes 2..17; block 1: 20..35
#pragma unroll
                            for (int i = 0; i < 4; ++i) qw[i] = h ? w[5 + i] : __funnelshift_r(w[i], w[i + 1], 16);
                        } else {
                            // (d, m) then qs: words 0 / 1..4 and 5 / 6..9
#pragma unroll
                            for (int i = 0; i < 4; ++i) qw[i] = w[5 * h + 1 + i];
                        }
                        uint32_t cw[16];
                        codes_f16<F>(qw, cw);
                        tmem_st16(arow + (uint32_t)(h * 16), cw);  // the block's 16 columns of this row
                    }
                };
                if (mine) {
                    if (half) decode_half(std::integral_constant<int, 1>{});
                    else decode_half(std::integral_constant<int, 0>{});
                }
                tmem_wait_st();
                tc_fence_before();
                // the first decode warp also waits for the fold to release the
                // stage's accumulator group, so the MMA thread needs no wait of
                // its own for it
                bool ok = true;
                if (warp == 2 && lane == 0)
                    ok = mbar_wait(smem_u32(&g_empty[aseq % NG]), ((aseq / NG) & 1u) ^ 1u);
                if (!__all_sync(0xffffffffu, ok)) {
                    fail(24);
                    return false;
                }
                if (lane == 0) mbar_arrive(smem_u32(&a_full[as]));
                ++aseq;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&c_empty[cs]));  // W codes of this chunk are read
            ++cseq;
            return true;
        });
    } else {
        // ------------------ fold: TMEM block sums -> fp32 totals ------------------
        // Two warps per TMEM lane quarter, each owning half of the tokens:
        // thread = W row = TMEM lane, tokens [tb, tb + TH).
        constexpr int TH = TP * 4 / kFoldWarps;  // tokens per fold warp
        const int quarter = warp & 3;          // TMEM lanes 32 quarter .. + 31
        const int row = quarter * 32 + lane;   // tile row
        const int tb = ((warp - kFoldWarp0) >> 2) * TH;
        // tokens folded here: T rounded up to 4, less tb (the padding columns are zero)
        const int nt = min(TH, max(0, ((a.T + 3) & ~3) - tb));
        grid_dependency_wait();  // the token exponents come from the x-split kernel
        if (threadIdx.x - 32 * kFoldWarp0 < TP) tok_exp_s[threadIdx.x - 32 * kFoldWarp0] = a.tok_exp[threadIdx.x - 32 * kFoldWarp0];
        fold_bar_sync();
        float acc[TH];
#pragma unroll
        for (int t = 0; t < TH; ++t) acc[t] = 0.f;
        uint32_t cseq = 0, aseq = 0;
        int seg_tile = -1;
        auto flush = [&](int t, int b_lo, int b_hi) {
            // the CTA's segment of row tile t ends
            const int m = mat_of(t);
            const int o = (t - pick(a.tile0, m)) * BM + row;
            const int om = pick(a.out_m, m);
            const float* bm = pick(a.bias_m, m);
            const float bo = (bm && o < om) ? bm[o] : 0.f;
            if (b_lo == 0 && b_hi == a.kb) {
                if (o < om) {
                    long long ys;
                    float* yp = y_row(m, o, ys);
#pragma unroll
                    for (int u = 0; u < TH; ++u) {
                        if (tb + u >= a.T) break;
                        store_y(yp, (tb + u) * ys, scaled(tb + u, acc[u], bm != nullptr, bo));
                    }
                }
            } else {
                // A split tile: the part goes to the workspace (unscaled); the
                // last of the tile's CTAs to finish adds the parts in CTA order
                // (the same order whichever CTA is last) and stores y.
                const int slot01 = f0 >= t * a.kb ? 0 : 1;
                float* p = a.part + ((long long)blockIdx.x * 2 + slot01) * TP * BM;
#pragma unroll
                for (int u = 0; u < TH; ++u) p[(tb + u) * BM + row] = acc[u];
                fold_bar_sync();  // every fold thread's part is stored
                if (warp == kFoldWarp0 && lane == 0) {
                    int c0, c1;
                    tile_ctas(t, c0, c1);
                    __threadfence();  // this CTA's part, before its count
                    if (atomicAdd(&a.tile_cnt[t], 1) == c1 - c0) {
                        __threadfence();  // the other CTAs' parts (their counts came first)
                        fix_tile[slot01] = t;  // summed after the loop, past a fold barrier
                    }
                }
            }
#pragma unroll
            for (int u = 0; u < TH; ++u) acc[u] = 0.f;
        };
        int last_t = -1, last_lo = 0, last_hi = 0;
        const uint32_t tq = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)C::ACC_COL0;
        for_each_chunk(f0, f1, a.kb, [&](int t, int c, int b_lo, int b_hi) {
            if (t != seg_tile) {
                if (seg_tile >= 0) flush(last_t, last_lo, last_hi);
                seg_tile = t;
            }
            last_t = t;
            last_lo = b_lo;
            last_hi = b_hi;
            const int cs = (int)(cseq % CS);
            // the chunk's W bytes hold each block's scale d (and minimum m)
            if (!mbar_wait(smem_u32(&c_full[cs]), (cseq / CS) & 1u)) {
                fail(25);
                return false;
            }
            const uint32_t wrow = w_st(cs) + (uint32_t)(row * C::W_ROW);
            for (int j = 0; j < SPC; ++j) {
                const unsigned m = stage_mask(c, j, b_lo, b_hi);
                if (!m) continue;
                const int g = (int)(aseq % NG);
                if (!mbar_wait(smem_u32(&g_full[g]), (aseq / NG) & 1u)) {
                    fail(25);
                    return false;
                }
                tc_fence_after();
                if (nt > 0) {
                    // PB blocks of the stage per TMEM wait, this warp's 2 TH
                    // columns of each (its tokens' hi, then their lo)
                    constexpr int PB = TH <= 4 ? SB : (TH == 8 ? 2 : 1);
#pragma unroll
                    for (int b2 = 0; b2 < SB; b2 += PB) {
                        uint32_t v[PB][2 * TH];
#pragma unroll
                        for (int h = 0; h < PB; ++h) {
                            if (!(m >> (b2 + h) & 1u)) continue;
                            const uint32_t ta = tq + (uint32_t)((g * SB + b2 + h) * N + 2 * tb);
                            tmem_ld_issue<2 * TH>(ta, v[h]);
                        }
                        tmem_wait_ld(*reinterpret_cast<uint32_t(*)[PB * 2 * TH]>(&v[0][0]));
#pragma unroll
                        for (int h = 0; h < PB; ++h) {
                            const int b = b2 + h;
                            if (!(m >> b & 1u)) continue;
                            // acc[u] += d * (hi[u] + lo[u]) (+ m * xsum[tb + u])
                            const uint32_t boff = wrow + (uint32_t)((SB * j + b) * C::BS);
                            const float d = half_bits_to_float(lds_u16(boff));
#pragma unroll
                            for (int u = 0; u < TH; ++u) {
                                if (u >= nt) break;
                                acc[u] = fmaf(__uint_as_float(v[h][u]) + __uint_as_float(v[h][TH + u]), d, acc[u]);
                            }
                            if constexpr (F == kQ4_1) {
                                const float mn = half_bits_to_float(lds_u16(boff + 2u));
                                const uint32_t sb = sc_st(cs) + (uint32_t)(((SB * j + b) * TP + tb) * 4);
#pragma unroll
                                for (int q = 0; q < TH / 4; ++q) {
                                    if (4 * q >= nt) break;
                                    const float4 m4 = lds_f4(sb + 16u * q);  // the same address in every lane
                                    acc[4 * q] = fmaf(mn, m4.x, acc[4 * q]);
                                    acc[4 * q + 1] = fmaf(mn, m4.y, acc[4 * q + 1]);
                                    acc[4 * q + 2] = fmaf(mn, m4.z, acc[4 * q + 2]);
                                    acc[4 * q + 3] = fmaf(mn, m4.w, acc[4 * q + 3]);
                                }
                            }
                        }
                    }
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&g_empty[g]));
                ++aseq;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&c_empty[cs]));  // W scales of this chunk are read
            ++cseq;
            return !aborted();
        });
        if (last_t >= 0 && !aborted()) flush(last_t, last_lo, last_hi);
        // Split tiles this CTA finished last: y = the tile's parts added in
        // CTA order, scaled, plus the bias.  A fold thread owns a row and its
        // tokens; the loads of its parts (2-4 CTAs at a time) go out together.
        fold_bar_sync();
        for (int k = 0; k < 2; ++k) {
            const int t = fix_tile[k];
            if (t < 0 || aborted() || tb >= a.T) continue;
            const int m = mat_of(t);
            const int o = (t - pick(a.tile0, m)) * BM + row;
            if (o >= pick(a.out_m, m)) continue;
            int c0, c1;
            tile_ctas(t, c0, c1);
            const int u0 = t * a.kb;
            const float* bm = pick(a.bias_m, m);
            const float bo = bm ? bm[o] : 0.f;
            long long ys;
            float* yp = y_row(m, o, ys);
            float v[TH];
#pragma unroll
            for (int u = 0; u < TH; ++u) v[u] = 0.f;
            constexpr int QF = TH >= 16 ? 2 : 4;  // CTAs' parts per round of loads
            for (int c = c0; c <= c1; c += QF) {
                float pv[QF][TH];
#pragma unroll
                for (int q = 0; q < QF; ++q) {
                    const int cc = c + q <= c1 ? c + q : c1;
                    const int sl = unit_begin(a.total, cc, G) >= u0 ? 0 : 1;
                    const float* pp = a.part + (((long long)cc * 2 + sl) * TP + tb) * BM + row;
#pragma unroll
                    for (int u = 0; u < TH; ++u) pv[q][u] = __ldcg(pp + u * BM);
                }
#pragma unroll
                for (int q = 0; q < QF; ++q)
                    if (c + q <= c1)
#pragma unroll
                        for (int u = 0; u < TH; ++u) v[u] = c + q == c0 ? pv[q][u] : __fadd_rn(v[u], pv[q][u]);
            }
#pragma unroll
            for (int u = 0; u < TH; ++u)
                if (tb + u < a.T) store_y(yp, (tb + u) * ys, scaled(tb + u, v[u], bm != nullptr, bo));
        }
    }

    // every warp is done with TMEM and shared memory; warp 1 frees TMEM
    __syncwarp();
    if (lane == 0) mbar_arrive(smem_u32(&end_bar));
    if (warp == 1) {
        if (!mbar_wait(smem_u32(&end_bar), 0u)) report_error(a.err, 26);
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, C::TMEM_COLS);
    }

    if (a.world > 1) {
        // Sharded call: this CTA's rows are in every rank's y.  Every CTA
        // counts itself once (with kBgemmDonePoison after giving up), so the
        // counter is back at zero for the next call; the last CTA publishes
        // the epoch to every rank, unless one gave up (then the peers' waits
        // run out and report code 4), and waits until every rank's slice
        // has landed here.  Ordering: this CTA's y stores happen before the
        // GPU-scope acquire-release count (__syncthreads, CTA scope); the
        // last CTA's one system-scope fence then publishes every CTA's stores
        // ahead of the flags (the fence is cumulative).
        __syncthreads();
        if (threadIdx.x == 0) {
            const bool ok = !aborted();
            const unsigned int prev = atom_add_acq_rel_gpu(a.done_counter, ok ? 1u : 1u + kBgemmDonePoison);
            if ((prev & (kBgemmDonePoison - 1u)) == gridDim.x - 1) {
                *a.done_counter = 0u;  // every CTA of this launch has counted
                if (ok && prev < kBgemmDonePoison) {
                    fence_acq_rel_sys();
                    for (int r = 0; r < a.world; ++r) st_relaxed_sys(a.peer_flags[r] + a.rank, a.epoch);
                    const uint64_t t0 = global_ns();
                    for (int r = 0; r < (a.wait ? a.world : 0); ++r) {
                        while ((int)(ld_acquire_sys(a.local_flags + r) - a.epoch) < 0) {
                            if (global_ns() - t0 > kWaitLimitNs) {
                                report_error(a.err, 4);
                                return;
                            }
                            __nanosleep(64);
                        }
                    }
                }
            }
        }
    }
}

// x fp32 [T][in] -> the B operand fp16 [2 TP][in] (token t of half
// h = t / (TP/2), i = t % (TP/2): hi in row h TP + i, lo in row h TP +
// TP/2 + i; tokens >= T zero), the exponent e_t of each token's power-of-two scale
// (2^e_t > max|x_t|) and, for q4_1, the block sums of x / 2^e_t.  One CTA
// per padded token: a max pass over the row, then the split pass (x stays
// in registers between them up to 16384 values).  Block 0 also zeroes the
// GEMM's split-tile counters.
constexpr int kSplitThreads = 512;
constexpr int kSplitRegs = 8;  // float4 per thread kept between the passes

template <int TP>
__global__ void __launch_bounds__(kSplitThreads)
    bgemm_xsplit_kernel(const float* __restrict__ x, int T, int in, __half* __restrict__ xb,
                        int* __restrict__ tok_exp, float* __restrict__ xsum, int* __restrict__ tile_cnt,
                        int tiles) {
    launch_dependents();     // the GEMM may start streaming its weights
    grid_dependency_wait();  // x, and the workspace the previous call on the stream used
    __shared__ float red[kSplitThreads / 32];
    __shared__ int ex_s;
    const int t = blockIdx.x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (t == 0)
        for (int i = threadIdx.x; i < tiles; i += kSplitThreads) tile_cnt[i] = 0;
    const int in4 = in / 4;
    const float* xrow = x + (long long)t * in;
    const bool vec = (reinterpret_cast<uintptr_t>(xrow) & 15u) == 0;  // the caller's x may be offset
    auto load4 = [&](int i) {
        if (vec) return reinterpret_cast<const float4*>(xrow)[i];
        return make_float4(xrow[4 * i], xrow[4 * i + 1], xrow[4 * i + 2], xrow[4 * i + 3]);
    };
    const bool keep = in4 <= kSplitRegs * kSplitThreads;
    float4 kv[kSplitRegs];
    float mx = 0.f;
    int bad = 0;
    auto scan = [&](const float4& v) {
        const float m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
        mx = fmaxf(mx, m);
        // NaN / Inf anywhere (fmaxf drops NaN, so test every value)
        bad |= !(fabsf(v.x) <= 3.402823466e38f) | !(fabsf(v.y) <= 3.402823466e38f) |
               !(fabsf(v.z) <= 3.402823466e38f) | !(fabsf(v.w) <= 3.402823466e38f);
    };
    if (keep) {
#pragma unroll
        for (int r = 0; r < kSplitRegs; ++r) {
            const int i = threadIdx.x + r * kSplitThreads;
            kv[r] = (t < T && i < in4) ? load4(i) : make_float4(0.f, 0.f, 0.f, 0.f);
            scan(kv[r]);
        }
    } else if (t < T) {
        for (int i = threadIdx.x; i < in4; i += kSplitThreads) scan(load4(i));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) red[warp] = mx;
    bad = __syncthreads_or(bad);
    if (threadIdx.x == 0) {
        float m = 0.f;
        for (int w = 0; w < kSplitThreads / 32; ++w) m = fmaxf(m, red[w]);
        int ex = 0;
        if (m > 0.f && !bad) frexpf(m, &ex);  // m = f 2^ex, f in [0.5, 1): |x / 2^ex| < 1
        ex_s = ex;
        tok_exp[t] = bad ? kBadExp : ex;
    }
    __syncthreads();
    const int ex = bad ? 0 : ex_s;
    constexpr int TH = TP / 2;  // tokens per fold warp
    __half* hi = xb + (long long)((t / TH) * TP + t % TH) * in;
    __half* lo = hi + (long long)TH * in;
    auto split = [&](int i, float4 v) {
        // exact power-of-two scaling, then the fp16 hi / lo split
        const float s[4] = {ldexpf(v.x, -ex), ldexpf(v.y, -ex), ldexpf(v.z, -ex), ldexpf(v.w, -ex)};
        __half h[4], l[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            h[k] = __float2half_rn(s[k]);
            l[k] = __float2half_rn(s[k] - __half2float(h[k]));
        }
        if (i < in4) {
            *reinterpret_cast<__half2*>(hi + 4 * i) = __halves2half2(h[0], h[1]);
            *reinterpret_cast<__half2*>(hi + 4 * i + 2) = __halves2half2(h[2], h[3]);
            *reinterpret_cast<__half2*>(lo + 4 * i) = __halves2half2(l[0], l[1]);
            *reinterpret_cast<__half2*>(lo + 4 * i + 2) = __halves2half2(l[2], l[3]);
        }
        if (xsum) {
            // 8 lanes hold a block's 32 values (in4 is a multiple of 8)
            float sum = (s[0] + s[1]) + (s[2] + s[3]);
            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
            if ((lane & 7) == 0 && i < in4) xsum[(long long)(i / 8) * TP + t] = sum;
        }
    };
    // warp-uniform trip counts: the sums shuffle across all 32 lanes
    if (keep) {
#pragma unroll
        for (int r = 0; r < kSplitRegs; ++r) {
            const int i = threadIdx.x + r * kSplitThreads;
            if (r * kSplitThreads + warp * 32 >= in4) break;
            split(i, bad ? make_float4(0.f, 0.f, 0.f, 0.f) : kv[r]);
        }
    } else {
        for (int base = warp * 32; base < in4; base += kSplitThreads) {
            const int i = base + lane;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (i < in4 && t < T && !bad) v = load4(i);
            split(i, v);
        }
    }
}

int tp_for(int T) { return T <= 8 ? 8 : (T <= 16 ? 16 : 32); }

int grid_for(int total, int sm_count) {
    long long g = (total + kMinBlocksPerCta - 1) / kMinBlocksPerCta;
    if (g > sm_count) g = sm_count;
    if (g > 256) g = 256;  // total x G < 2^31
    return g < 1 ? 1 : (int)g;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

// One matrix of a launch.
struct GroupMat {
    const uint8_t* w;
    float* y;
    int out;
    const float* bias;
};

template <int F, int TP>
cudaError_t launch_t(const GroupMat* mats, int nmat, const float* x, int in, int T, void* ws, int sm_count, int* err,
                     cudaStream_t stream, const BgemmGather* g) {
    using C = BCfg<F, TP>;
    const int kb = in / kQK;
    int tiles = 0;
    for (int m = 0; m < nmat; ++m) tiles += (mats[m].out + BM - 1) / BM;
    char* p = static_cast<char*>(ws);
    __half* xb = reinterpret_cast<__half*>(p);
    p += align256((size_t)2 * TP * in * sizeof(__half));
    int* tok_exp = reinterpret_cast<int*>(p);
    p += align256((size_t)TP * sizeof(int));
    float* xsum = nullptr;
    if (F == kQ4_1) {
        // padded to whole 8-block chunks (the kernel copies a chunk's worth at a time)
        const size_t kbp = (size_t)(kb + BPC - 1) / BPC * BPC;
        xsum = reinterpret_cast<float*>(p);
        p += align256(kbp * TP * sizeof(float));
    }
    int* tile_cnt = reinterpret_cast<int*>(p);
    p += align256((size_t)tiles * sizeof(int));
    float* part = reinterpret_cast<float*>(p);

    const long long row_bytes = (long long)kb * C::BS;
    WMaps mw{};
    for (int m = 0; m < nmat; ++m)
        if (!make_map_2d(&mw.m[m], F == kQ8_0 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                         const_cast<uint8_t*>(mats[m].w), (uint64_t)(row_bytes / C::W_ESZ), (uint64_t)mats[m].out,
                         (uint64_t)row_bytes, (uint32_t)(C::W_ROW / C::W_ESZ), BM, CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
    CUtensorMap mx;
    if (!make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xb, (uint64_t)in, (uint64_t)(2 * TP), (uint64_t)in * 2, 64,
                     (uint32_t)(2 * TP), CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;

    static std::atomic<bool> attr_set[64];  // one value per instantiation: racing first calls agree
    int dev = 0;
    cudaGetDevice(&dev);
    cudaError_t e = cudaSuccess;
    if (dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(bgemm_kernel<F, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }

    // both launches may start while the kernel before them drains
    // (programmatic dependent launch); each waits on the device for the data
    // it reads
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(TP);
    cfg.blockDim = dim3(kSplitThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, bgemm_xsplit_kernel<TP>, x, T, in, xb, tok_exp, xsum, tile_cnt, tiles);
    if (e != cudaSuccess) return e;

    BgemmArgs a{};
    a.nmat = nmat;
    a.tile0[0] = 0;
    for (int m = 0; m < nmat; ++m) {
        a.tile0[m + 1] = a.tile0[m] + (mats[m].out + BM - 1) / BM;
        a.out_m[m] = mats[m].out;
        a.ym[m] = mats[m].y;
        a.bias_m[m] = mats[m].bias;
    }
    if (g) {
        for (int r = 0; r < g->world; ++r) {
            a.ys[r] = g->ys[r];
            a.peer_flags[r] = g->peer_flags[r];
        }
        a.ny = g->world;
        a.y_stride = g->y_stride;
        a.row_offset = g->row_offset;
        a.world = g->world;
        a.rank = g->rank;
        a.epoch = g->epoch;
        a.local_flags = g->local_flags;
        a.done_counter = g->done_counter;
        a.wait = g->wait;
    } else {
        a.ys[0] = mats[0].y;
        a.ny = 1;
        a.y_stride = mats[0].out;
        a.world = 1;
    }
    a.tok_exp = tok_exp;
    a.xsum = xsum;
    a.part = part;
    a.in = in;
    a.T = T;
    a.kb = kb;
    a.total = tiles * kb;
    a.err = err;
    a.tile_cnt = tile_cnt;
    const int G = grid_for(a.total, sm_count);
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(threads_of(TP));
    cfg.dynamicSmemBytes = (size_t)C::SMEM;
    return cudaLaunchKernelEx(&cfg, bgemm_kernel<F, TP>, mw, mx, a);
}

template <int F>
cudaError_t launch_f(const GroupMat* mats, int nmat, const float* x, int in, int T, void* ws, int sm_count, int* err,
                     cudaStream_t stream, const BgemmGather* g) {
    switch (tp_for(T)) {
        case 8: return launch_t<F, 8>(mats, nmat, x, in, T, ws, sm_count, err, stream, g);
        case 16: return launch_t<F, 16>(mats, nmat, x, in, T, ws, sm_count, err, stream, g);
        default: return launch_t<F, 32>(mats, nmat, x, in, T, ws, sm_count, err, stream, g);
    }
}

cudaError_t launch_fmt(int fmt, const GroupMat* mats, int nmat, const float* x, int in, int rows, void* ws,
                       int sm_count, int* err, cudaStream_t stream, const BgemmGather* g) {
    switch (fmt) {
        case kQ8_0: return launch_f<kQ8_0>(mats, nmat, x, in, rows, ws, sm_count, err, stream, g);
        case kQ4_0: return launch_f<kQ4_0>(mats, nmat, x, in, rows, ws, sm_count, err, stream, g);
        case kQ4_1: return launch_f<kQ4_1>(mats, nmat, x, in, rows, ws, sm_count, err, stream, g);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

bool bgemm_shape_ok(int fmt, const void* w, int out, int in, int rows) {
    const long long row_bytes = (long long)((in + kQK - 1) / kQK) * block_bytes(fmt);
    return rows >= MLQ_BGEMM_MIN_ROWS && rows <= kBgemmMaxRows && out > 0 && in % kQK == 0 &&
           reinterpret_cast<uintptr_t>(w) % 16 == 0 && row_bytes % 16 == 0 &&
           (long long)((out + BM - 1) / BM) * (in / kQK) <= kMaxUnits;
}

size_t bgemm_workspace_bytes(int fmt, int in, int rows, int out, int sm_count) {
    const int tp = tp_for(rows);
    const int kb = in / kQK;
    const int total = ((out + BM - 1) / BM) * kb;
    const int G = grid_for(total, sm_count);
    const size_t kbp = (size_t)(kb + BPC - 1) / BPC * BPC;
    size_t b = align256((size_t)2 * tp * in * 2) + align256((size_t)tp * 4);
    if (fmt == kQ4_1) b += align256(kbp * tp * 4);
    b += align256((size_t)((out + BM - 1) / BM) * 4);
    return b + (size_t)G * 2 * tp * BM * 4;
}

size_t bgemm_group_workspace_bytes(int fmt, int in, int rows, const int* out, int nmat, int sm_count) {
    int tiles = 0;
    for (int m = 0; m < nmat; ++m) tiles += (out[m] + BM - 1) / BM;
    return bgemm_workspace_bytes(fmt, in, rows, tiles * BM, sm_count);
}

cudaError_t launch_bgemm(int fmt, const uint8_t* w, const float* x, float* y, int out, int in, int rows,
                         const float* bias, void* ws, int sm_count, int* err, cudaStream_t stream,
                         const BgemmGather* g) {
    const GroupMat m{w, y, out, bias};
    return launch_fmt(fmt, &m, 1, x, in, rows, ws, sm_count, err, stream, g);
}

cudaError_t launch_bgemm_group(int fmt, int nmat, const uint8_t* const* w, float* const* y, const int* out,
                               const float* const* bias, const float* x, int in, int rows, void* ws, int sm_count,
                               int* err, cudaStream_t stream) {
    if (nmat < 1 || nmat > kBgemmMaxGroup) return cudaErrorInvalidValue;
    GroupMat mats[kBgemmMaxGroup];
    long long units = 0;
    for (int m = 0; m < nmat; ++m) {
        mats[m] = GroupMat{w[m], y[m], out[m], bias ? bias[m] : nullptr};
        units += (long long)((out[m] + BM - 1) / BM) * (in / kQK);
    }
    if (units > kMaxUnits) return cudaErrorInvalidValue;
    return launch_fmt(fmt, mats, nmat, x, in, rows, ws, sm_count, err, stream, nullptr);
}

}  // namespace mlq
