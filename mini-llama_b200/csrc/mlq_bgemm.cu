// mlq_bgemm.cu -- batched-decode GEMM on the tensor cores: 2..32 rows of x
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
//   * x is scaled per (token, block) by a power of two s >= max|x_block| and
//     split x/s = xh + xl into two fp16 values (xsplit kernel below): exact
//     to 2^-24 of s, the level of one fp32 rounding of the block's largest
//     value.
//   * One 128 x N x 32 product per block on the tensor cores (two kind::f16
//     MMAs of K = 16) gives D[row][t] = sum q (xh + xl) over the block -- the
//     hi and lo halves of x are the two halves of B (N = 2 x padded tokens)
//     -- in a TMEM accumulator of its own.
//   * CUDA-core "fold" warps read the block's accumulator and add
//     d * (s * D) (+ m * sum(x) for q4_1) to the fp32 total of (row, t).
//     The block scales never enter the tensor-core sums.
//
// CTA = 14 warps, one CTA per SM:
//   warp 0      TMA producer: W chunks (8 blocks x 128 rows, 2-D tensor map
//               over the AoS bytes) and the chunk's x tiles (fp16 [hi; lo],
//               128-B swizzle).
//   warp 1      TMEM allocation; lane 0 issues the MMAs and commits.
//   warps 2-9   decode: two threads per W row, each turning two blocks of an
//               A stage (4 blocks, K = 128) into fp16 codes in its 64-value
//               sub-tile (swizzled, K-major).
//   warps 10-13 fold: thread = W row = TMEM lane (one lane quarter per
//               warp); a block's scale d (and q4_1 minimum m) is read from
//               the W chunk in shared memory.
// A stage's blocks are committed as one TMEM group: one barrier per four
// blocks between the MMA thread and the decode / fold warps.
// Work split ("stream-K"): the matrix is a list of (row tile, block) units;
// CTA c takes the contiguous range [c W / G, (c + 1) W / G).  A row tile a
// CTA covers whole is stored straight to y; the at most two partly covered
// tiles at the ends of its range go to a workspace, and a second kernel adds
// every split tile's parts in CTA order (deterministic) plus the bias.
// Every mbarrier wait is bounded (2 s); no TMA multicast anywhere.
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
constexpr int SB = 4;               // blocks per A stage (K = 128: two 64-value sub-tiles)
constexpr int SPC = BPC / SB;       // A stages per chunk (2)
constexpr int kDecodeWarps = 8;     // warps 2..9: two per row (one 64-value sub-tile each)
constexpr int kFoldWarps = 4;       // warps 10..13: one per TMEM lane quarter
constexpr int kFoldWarp0 = 2 + kDecodeWarps;
constexpr int kThreads = 32 * (2 + kDecodeWarps + kFoldWarps);
constexpr int kSmemMax = 232448 - 1024;  // dynamic shared memory per CTA: 227 KB less the static part
constexpr int kMinBlocksPerCta = 16;

constexpr int cmin(int a, int b) { return a < b ? a : b; }
constexpr int pow2_at_least(int v) { return v <= 32 ? 32 : (v <= 64 ? 64 : (v <= 128 ? 128 : (v <= 256 ? 256 : 512))); }

// TP: padded tokens (8, 16 or 32); the MMA's N is 2 TP (x hi, then x lo).
template <int F, int TP>
struct BCfg {
    static constexpr int BS = Fmt<F>::kBlockBytes;
    static constexpr int N = 2 * TP;
    static constexpr int W_ROW = BPC * BS;             // 272 / 144 / 160 bytes of a row's chunk
    static constexpr int W_ESZ = F == kQ8_0 ? 2 : 1;   // tensor-map element (inner box <= 256 elements)
    static constexpr int W_TILE = BM * W_ROW;
    static constexpr int B_SUB = N * 128;              // [hi; lo] x tile of 64 values (fp16, 128-B rows)
    static constexpr int B_TILE = (KC / 64) * B_SUB;
    // the chunk's x block scales (and q4_1 block sums): [8 blocks][TP] floats each
    static constexpr int SC_BYTES = BPC * TP * 4 * (F == kQ4_1 ? 2 : 1);
    static constexpr int C_STAGE = (W_TILE + B_TILE + SC_BYTES + 1023) / 1024 * 1024;  // W, x tiles, x scales
    // A (fp16 codes) lives in TMEM: an A stage is 4 blocks x 32 values x
    // 2 B / 4 B per column = 64 columns; the accumulator groups (4 blocks x N
    // columns each) take the rest of the 512 columns
    static constexpr int AS = 2;
    static constexpr int A_COLS = SB * kQK / 2;
    static constexpr int ACC_COL0 = AS * A_COLS;
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

struct BgemmArgs {
    float* y;             // [T][out]
    const float* bias;    // [out] or null
    const float* sc;      // [kb][TP]: power-of-two block scale of x (NaN: the block holds NaN/Inf)
    const float* xsum;    // [kb][TP]: block sums of x (q4_1), else null
    float* part;          // [grid][2][TP][BM]: partial sums of partly covered row tiles
    int out, in, T, kb;   // kb = blocks per row
    long long total;      // units = row tiles x kb
    int* err;
};

// The units [f0, f1) of CTA c among G.
__host__ __device__ __forceinline__ long long unit_begin(long long total, int c, int G) {
    return (long long)c * total / G;
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
__device__ __forceinline__ void for_each_chunk(long long f0, long long f1, int kb, Fn&& fn) {
    if (f1 <= f0) return;
    const long long t0 = f0 / kb, t1 = (f1 - 1) / kb;
    for (long long t = t0; t <= t1; ++t) {
        const int b_lo = (int)(f0 > t * kb ? f0 - t * kb : 0);
        const int b_hi = (int)(f1 < (t + 1) * kb ? f1 - t * kb : kb);
        for (int c = b_lo / BPC; c <= (b_hi - 1) / BPC; ++c)
            if (!fn((int)t, c, b_lo, b_hi)) return;
    }
}

template <int F, int TP>
__global__ void __launch_bounds__(kThreads, 1)
    bgemm_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_x, BgemmArgs a) {
    using C = BCfg<F, TP>;
    constexpr int CS = C::CS, AS = C::AS, NG = C::NG, N = C::N;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t c_full[CS], c_empty[CS], a_full[AS], a_empty[AS];
    __shared__ __align__(8) uint64_t g_full[NG], g_empty[NG];
    __shared__ __align__(8) uint64_t drain_bar, end_bar;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
    auto w_st = [&](int s) { return base + (uint32_t)(s * C::C_STAGE); };
    auto x_st = [&](int s) { return w_st(s) + (uint32_t)C::W_TILE; };
    auto sc_st = [&](int s) { return x_st(s) + (uint32_t)C::B_TILE; };  // [8][TP] scales, then (q4_1) [8][TP] sums

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
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(smem_u32(&tmem_base_s), C::TMEM_COLS);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;
    launch_dependents();  // the fix-up kernel may be scheduled; it waits for this grid

    const int G = gridDim.x;
    const long long f0 = unit_begin(a.total, blockIdx.x, G), f1 = unit_begin(a.total, blockIdx.x + 1, G);
    auto aborted = [&]() { return *(volatile int*)&abort_flag != 0; };
    auto fail = [&](int code) {
        report_error(a.err, code);
        abort_flag = 1;
    };
    // valid-block mask of A stage j of chunk c (bit b: block c * 8 + 4 j + b)
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
            // dependent launch), their x tiles and scales after it.
            auto issue_x = [&](int s, int c) {
                const uint32_t fb = smem_u32(&c_full[s]);
#pragma unroll
                for (int q = 0; q < KC / 64; ++q) tma_load_2d(x_st(s) + (uint32_t)(q * C::B_SUB), &tm_x, c * KC + q * 64, 0, fb);
                // x block scales (and sums) of the chunk's 8 blocks: the arrays
                // are padded to whole chunks, so this never reads past them
                bulk_g2s(sc_st(s), a.sc + (long long)c * BPC * TP, (uint32_t)(BPC * TP * 4), fb);
                if constexpr (F == kQ4_1)
                    bulk_g2s(sc_st(s) + (uint32_t)(BPC * TP * 4), a.xsum + (long long)c * BPC * TP, (uint32_t)(BPC * TP * 4), fb);
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
                tma_load_2d(w_st(s), &tm_w, c * (C::W_ROW / C::W_ESZ), t * BM, fb);
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
                if (!mbar_wait(smem_u32(&c_full[cs]), (cseq / CS) & 1u)) {
                    fail(22);
                    return false;
                }
                for (int j = 0; j < SPC; ++j) {
                    const unsigned m = stage_mask(c, j, b_lo, b_hi);
                    if (!m) continue;
                    const int as = (int)(aseq % AS), g = (int)(aseq % NG);
                    if (!mbar_wait(smem_u32(&a_full[as]), (aseq / AS) & 1u) ||
                        !mbar_wait(smem_u32(&g_empty[g]), ((aseq / NG) & 1u) ^ 1u)) {
                        fail(22);
                        return false;
                    }
                    if (aborted()) return false;
                    tc_fence_after();
#pragma unroll
                    for (int b = 0; b < SB; ++b) {
                        if (!(m >> b & 1u)) continue;
                        // A: the block's 16 columns of the A stage in TMEM (8 per K = 16)
                        const uint32_t ta = tmem + (uint32_t)(as * C::A_COLS + b * 16);
                        const uint64_t bd = sw128_desc(x_st(cs) + (uint32_t)((2 * j + (b >> 1)) * C::B_SUB));
                        const uint32_t td = tmem + (uint32_t)(C::ACC_COL0 + (g * SB + b) * N);
#pragma unroll
                        for (int kk = 0; kk < 2; ++kk) {
                            const uint64_t adv = (uint64_t)(((b & 1) * 64 + kk * 32) >> 4);  // B bytes along K / 16
                            mma_f16kind_ta(td, ta + (uint32_t)(kk * 8), bd + adv, idesc, kk);
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
        // two threads per W row: `half` h fills the stage's 64-value sub-tile
        // h (blocks 2h, 2h + 1 of the stage)
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
                const unsigned mine = (m >> (2 * half)) & 3u;
                // the two halves as compile-time cases, so every register index
                // below is a constant
                auto decode_half = [&](auto HALF) {
                    constexpr int half = decltype(HALF)::value;
                    // this thread's two blocks: 2 BS bytes from byte (4 j + 2 half) BS
                    // of the row's chunk (a word boundary), read as the 16-B units
                    // that cover them (rows are 17 / 9 / 10 units apart: the 8
                    // lanes of a load phase hit distinct bank groups)
                    constexpr int NW = 2 * C::BS / 4;
                    const int sb = (SB * j + 2 * half) * C::BS;
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
                    const uint32_t arow = tlane + (uint32_t)(as * C::A_COLS + 2 * half * 16);
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
                __syncwarp();
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
        const int quarter = warp & 3;          // TMEM lanes 32 quarter .. + 31
        const int row = quarter * 32 + lane;   // tile row
        float acc[TP];
#pragma unroll
        for (int t = 0; t < TP; ++t) acc[t] = 0.f;
        uint32_t cseq = 0, aseq = 0;
        int seg_tile = -1;
        auto flush = [&](int t, int b_lo, int b_hi) {
            // the CTA's segment of row tile t ends: y, or its part for the fix-up
            const int o = t * BM + row;
            if (b_lo == 0 && b_hi == a.kb) {
                if (o < a.out) {
                    const float bo = a.bias ? a.bias[o] : 0.f;
#pragma unroll
                    for (int tt = 0; tt < TP; ++tt)
                        if (tt < a.T) a.y[(long long)tt * a.out + o] = a.bias ? __fadd_rn(acc[tt], bo) : acc[tt];
                }
            } else {
                const int slot01 = f0 >= (long long)t * a.kb ? 0 : 1;
                float* p = a.part + ((long long)blockIdx.x * 2 + slot01) * TP * BM;
#pragma unroll
                for (int tt = 0; tt < TP; ++tt) p[tt * BM + row] = acc[tt];
            }
#pragma unroll
            for (int tt = 0; tt < TP; ++tt) acc[tt] = 0.f;
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
                // the group's accumulators, PB blocks per TMEM wait (two while
                // their registers fit); x scales come from the chunk's stage
                constexpr int PB = N <= 32 ? 2 : 1;
                // fold of block b's tokens [t0, t0 + NT): D = hi + lo columns
                auto fold_tokens = [&](int b, int t0, const uint32_t* hi, const uint32_t* lo, int nt) {
                    const uint32_t boff = wrow + (uint32_t)((SB * j + b) * C::BS);
                    const float d = half_bits_to_float(lds_u16(boff));
                    const uint32_t sb = sc_st(cs) + (uint32_t)((SB * j + b) * TP * 4);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        if (4 * q >= nt) break;
                        const float4 s4 = lds_f4(sb + 4u * (t0 + 4 * q));  // the same address in every lane
                        const float sv[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int tt = 4 * q + u;
                            const float dsum = __uint_as_float(hi[tt]) + __uint_as_float(lo[tt]);
                            acc[t0 + tt] = fmaf(dsum * sv[u], d, acc[t0 + tt]);
                        }
                    }
                    if constexpr (F == kQ4_1) {  // + m * (block sum of x)
                        const float mn = half_bits_to_float(lds_u16(boff + 2u));
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            if (4 * q >= nt) break;
                            const float4 m4 = lds_f4(sb + (uint32_t)(BPC * TP * 4) + 4u * (t0 + 4 * q));
                            acc[t0 + 4 * q] = fmaf(mn, m4.x, acc[t0 + 4 * q]);
                            acc[t0 + 4 * q + 1] = fmaf(mn, m4.y, acc[t0 + 4 * q + 1]);
                            acc[t0 + 4 * q + 2] = fmaf(mn, m4.z, acc[t0 + 4 * q + 2]);
                            acc[t0 + 4 * q + 3] = fmaf(mn, m4.w, acc[t0 + 4 * q + 3]);
                        }
                    }
                };
                if constexpr (N <= 32) {
                    // TP <= 16: one load holds a block's hi and lo columns; two
                    // blocks per TMEM wait
#pragma unroll
                    for (int b2 = 0; b2 < SB; b2 += PB) {
                        uint32_t v[PB][N];
#pragma unroll
                        for (int h = 0; h < PB; ++h) {
                            if (!(m >> (b2 + h) & 1u)) continue;
                            const uint32_t ta = tq + (uint32_t)((g * SB + b2 + h) * N);
                            if constexpr (N == 16) tmem_ld16_issue(ta, *reinterpret_cast<uint32_t(*)[16]>(v[h]));
                            else tmem_ld32_issue(ta, *reinterpret_cast<uint32_t(*)[32]>(v[h]));
                        }
                        tmem_wait_ld(*reinterpret_cast<uint32_t(*)[PB * N]>(&v[0][0]));
#pragma unroll
                        for (int h = 0; h < PB; ++h)
                            if (m >> (b2 + h) & 1u) fold_tokens(b2 + h, 0, v[h], v[h] + TP, TP);
                    }
                } else {
                    // TP = 32: sixteen tokens at a time (their hi and lo columns)
#pragma unroll 1
                    for (int b = 0; b < SB; ++b) {
                        if (!(m >> b & 1u)) continue;
                        const uint32_t ta = tq + (uint32_t)((g * SB + b) * N);
#pragma unroll
                        for (int t0 = 0; t0 < TP; t0 += 16) {
                            uint32_t v[32];
                            tmem_ld16_issue(ta + (uint32_t)t0, *reinterpret_cast<uint32_t(*)[16]>(v));
                            tmem_ld16_issue(ta + (uint32_t)(TP + t0), *reinterpret_cast<uint32_t(*)[16]>(v + 16));
                            tmem_wait_ld(v);
                            fold_tokens(b, t0, v, v + 16, 16);
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
}

// x fp32 [T][in] -> the B operand fp16 [2 TP][in] (rows t: hi, TP + t: lo;
// rows >= T zero), per (block, token) the power-of-two scale and (q4_1) the
// block sum.  One warp per (block, token).
template <int TP>
__global__ void bgemm_xsplit_kernel(const float* __restrict__ x, int T, int in, int kb, __half* __restrict__ xb,
                                    float* __restrict__ sc, float* __restrict__ xsum) {
    launch_dependents();  // the GEMM may start streaming its weights
    const long long wid = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= (long long)kb * TP) return;
    const int b = (int)(wid / TP), t = (int)(wid % TP);
    const long long e = (long long)b * kQK + lane;
    const float v = t < T ? x[(long long)t * in + e] : 0.f;
    float mx = fabsf(v);
    int bad = !(mx <= 3.402823466e38f);  // NaN or Inf
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        bad |= __shfl_xor_sync(0xffffffffu, bad, off);
    }
    int ex = 0;
    if (mx > 0.f && !bad) frexpf(mx, &ex);  // mx = f 2^ex, f in [0.5, 1): |v / 2^ex| < 1
    const float xs = ldexpf(v, -ex);        // exact (a power-of-two scaling)
    const __half h = __float2half_rn(xs);
    const __half l = __float2half_rn(xs - __half2float(h));
    xb[(long long)t * in + e] = h;
    xb[(long long)(TP + t) * in + e] = l;
    float s = v;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
        sc[(long long)b * TP + t] = bad ? __int_as_float(0x7fc00000) : ldexpf(1.0f, ex);
        if (xsum) xsum[(long long)b * TP + t] = s;
    }
}

// Split row tiles: y = the parts of every CTA that covers the tile, in CTA
// order, plus the bias.  One thread per (tile, token, row).
__global__ void bgemm_fixup_kernel(BgemmArgs a, int tp, int G) {
    grid_dependency_wait();  // every CTA of the GEMM has stored its parts
    const long long tiles = (a.out + BM - 1) / BM;
    const long long n = tiles * a.T * BM;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const int r = (int)(i % BM);
        const int tt = (int)((i / BM) % a.T);
        const long long t = i / BM / a.T;
        const int o = (int)(t * BM + r);
        if (o >= a.out) continue;
        // CTAs holding the tile's first and last unit
        const long long u0 = t * a.kb, u1 = u0 + a.kb - 1;
        int c0 = (int)(u0 * G / a.total), c1 = (int)(u1 * G / a.total);
        while (c0 + 1 < G && unit_begin(a.total, c0 + 1, G) <= u0) ++c0;
        while (c0 > 0 && unit_begin(a.total, c0, G) > u0) --c0;
        while (c1 + 1 < G && unit_begin(a.total, c1 + 1, G) <= u1) ++c1;
        while (c1 > 0 && unit_begin(a.total, c1, G) > u1) --c1;
        if (c0 == c1) continue;  // one CTA covered it whole and stored y
        float v = 0.f;
        for (int c = c0; c <= c1; ++c) {
            const int slot01 = unit_begin(a.total, c, G) >= u0 ? 0 : 1;
            v = c == c0 ? a.part[(((long long)c * 2 + slot01) * tp + tt) * BM + r]
                        : __fadd_rn(v, a.part[(((long long)c * 2 + slot01) * tp + tt) * BM + r]);
        }
        if (a.bias) v = __fadd_rn(v, a.bias[o]);
        a.y[(long long)tt * a.out + o] = v;
    }
}

int tp_for(int T) { return T <= 8 ? 8 : (T <= 16 ? 16 : 32); }

int grid_for(long long total, int sm_count) {
    long long g = (total + kMinBlocksPerCta - 1) / kMinBlocksPerCta;
    if (g > sm_count) g = sm_count;
    return g < 1 ? 1 : (int)g;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

template <int F, int TP>
cudaError_t launch_t(const uint8_t* w, const float* x, float* y, int out, int in, int T, const float* bias,
                     void* ws, int sm_count, int* err, cudaStream_t stream) {
    using C = BCfg<F, TP>;
    const int kb = in / kQK;
    char* p = static_cast<char*>(ws);
    __half* xb = reinterpret_cast<__half*>(p);
    p += align256((size_t)2 * TP * in * sizeof(__half));
    // scales and sums padded to whole 8-block chunks (the kernel copies a
    // chunk's worth at a time)
    const size_t kbp = (size_t)(kb + BPC - 1) / BPC * BPC;
    float* sc = reinterpret_cast<float*>(p);
    p += align256(kbp * TP * sizeof(float));
    float* xsum = nullptr;
    if (F == kQ4_1) {
        xsum = reinterpret_cast<float*>(p);
        p += align256(kbp * TP * sizeof(float));
    }
    float* part = reinterpret_cast<float*>(p);

    const long long warps = (long long)kb * TP;
    bgemm_xsplit_kernel<TP><<<(int)((warps * 32 + 255) / 256), 256, 0, stream>>>(x, T, in, kb, xb, sc, xsum);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    const long long row_bytes = (long long)kb * C::BS;
    CUtensorMap mw, mx;
    if (!make_map_2d(&mw, F == kQ8_0 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                     const_cast<uint8_t*>(w), (uint64_t)(row_bytes / C::W_ESZ), (uint64_t)out, (uint64_t)row_bytes,
                     (uint32_t)(C::W_ROW / C::W_ESZ), BM, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&mx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xb, (uint64_t)in, (uint64_t)(2 * TP), (uint64_t)in * 2, 64,
                     (uint32_t)(2 * TP), CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;

    static std::atomic<bool> attr_set[64];  // one value per instantiation: racing first calls agree
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(bgemm_kernel<F, TP>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    BgemmArgs a{};
    a.y = y;
    a.bias = bias;
    a.sc = sc;
    a.xsum = xsum;
    a.part = part;
    a.out = out;
    a.in = in;
    a.T = T;
    a.kb = kb;
    a.total = (long long)((out + BM - 1) / BM) * kb;
    a.err = err;
    const int G = grid_for(a.total, sm_count);
    // the GEMM and the fix-up each start while the kernel before them drains
    // (programmatic dependent launch); both wait on the device for the data
    // they need
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = (size_t)C::SMEM;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, bgemm_kernel<F, TP>, mw, mx, a);
    if (e != cudaSuccess) return e;
    const long long n = (long long)((out + BM - 1) / BM) * T * BM;
    const long long nb = (n + 255) / 256;
    cfg.gridDim = dim3((unsigned)(nb < 4 * sm_count ? nb : 4 * sm_count));
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = 0;
    return cudaLaunchKernelEx(&cfg, bgemm_fixup_kernel, a, (int)TP, G);
}

template <int F>
cudaError_t launch_f(const uint8_t* w, const float* x, float* y, int out, int in, int T, const float* bias, void* ws,
                     int sm_count, int* err, cudaStream_t stream) {
    switch (tp_for(T)) {
        case 8: return launch_t<F, 8>(w, x, y, out, in, T, bias, ws, sm_count, err, stream);
        case 16: return launch_t<F, 16>(w, x, y, out, in, T, bias, ws, sm_count, err, stream);
        default: return launch_t<F, 32>(w, x, y, out, in, T, bias, ws, sm_count, err, stream);
    }
}

}  // namespace

bool bgemm_shape_ok(int fmt, const void* w, int out, int in, int rows) {
    const long long row_bytes = (long long)((in + kQK - 1) / kQK) * block_bytes(fmt);
    return rows >= MLQ_BGEMM_MIN_ROWS && rows <= kBgemmMaxRows && out > 0 && in % kQK == 0 &&
           reinterpret_cast<uintptr_t>(w) % 16 == 0 && row_bytes % 16 == 0;
}

size_t bgemm_workspace_bytes(int fmt, int in, int rows, int out, int sm_count) {
    const int tp = tp_for(rows);
    const int kb = in / kQK;
    const long long total = (long long)((out + BM - 1) / BM) * kb;
    const int G = grid_for(total, sm_count);
    const size_t kbp = (size_t)(kb + BPC - 1) / BPC * BPC;
    size_t b = align256((size_t)2 * tp * in * 2) + align256(kbp * tp * 4);
    if (fmt == kQ4_1) b += align256(kbp * tp * 4);
    return b + (size_t)G * 2 * tp * BM * 4;
}

cudaError_t launch_bgemm(int fmt, const uint8_t* w, const float* x, float* y, int out, int in, int rows,
                         const float* bias, void* ws, int sm_count, int* err, cudaStream_t stream) {
    switch (fmt) {
        case kQ8_0: return launch_f<kQ8_0>(w, x, y, out, in, rows, bias, ws, sm_count, err, stream);
        case kQ4_0: return launch_f<kQ4_0>(w, x, y, out, in, rows, bias, ws, sm_count, err, stream);
        case kQ4_1: return launch_f<kQ4_1>(w, x, y, out, in, rows, bias, ws, sm_count, err, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mlq
