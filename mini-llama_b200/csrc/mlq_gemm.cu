// mlq_gemm.cu -- dequant-fused GEMM on the 5th-generation tensor cores
// (tcgen05 + TMEM) for prefill / batched rows of x (MLQ_GEMM_ROWS_RULE in mlq.h).
//
// The reference has no GEMM for quantized weights: forwardBatch loops the
// GEMV one token at a time (src/batch.cc:32-55) and linearQ* loops rows
// (src/quant.cc:453-472).  This kernel computes the same y = x W^T for many
// rows at once with the tensor cores while keeping fp32-level accuracy:
//
//   * W is decoded EXACTLY to fp32 (w = d*q, d*(q-8) or d*q + m, the
//     reference's dequantizeFrom* values), then split w = wh + wl with
//     wh = bf16_rn(w), wl = bf16_rn(w - wh);  x is split the same way.
//   * D = wh*xh + wh*xl + wl*xh in fp32 (TMEM), three kind::f16 MMAs per
//     K-step.  The dropped wl*xl term and the two splits' residues are
//     below 2^-17 of each product, so y matches the fp32 reference to
//     ~1e-5 relative -- far inside the 1e-3 contract.
//
// CTA = 10 warps, one output tile of 128 W rows x NT tokens at a time (NT =
// 16/32/64/128, the narrowest covering the call's rows), persistent over
// tiles:
//   warp 0   TMA producer: packed W chunks (256 values per row, 2-D tensor
//            map over the AoS bytes, no swizzle) and x hi/lo tiles (2-D
//            tensor maps over bf16 [T][K], 128-B swizzle).
//   warp 1   allocates the TMEM columns; lane 0 issues the MMAs and the
//            tcgen05.commit arrivals.
//   warps 2-9 ("row" threads, thread = W row = TMEM lane, two warps per
//            lane quarter): each decodes its row's block of every 64-wide
//            K-step from shared memory, writes the bf16 hi/lo A halves in
//            the 128-B swizzled K-major layout, then runs its share of the
//            epilogue (tcgen05.ld -> y, + bias).
// When the tiles cannot fill the SMs, the K extent is split into ranges of
// whole W chunks (split-K): a work item is (row tile, token tile, K range),
// the epilogue writes partial sums to the workspace and a second kernel adds
// them in range order.  All mbarrier waits are bounded (2 s); no TMA
// multicast anywhere.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <mutex>

#include "mlq.h"
#include "mlq_device.cuh"
#include "mlq_kernels.h"
#include "mlq_tc.cuh"
#include "mlq_tmap.h"

namespace mlq {
namespace {

constexpr int BM = 128;       // W rows per tile = MMA M = TMEM lanes
// Tokens per tile (MMA N, TMEM columns) is a template parameter NT: 16, 32,
// 64 or 128, the smallest that covers the call's rows of x (up to 128), so
// a batched-decode call does not run 128-wide MMAs on 16 real columns.
constexpr int BK = 64;        // K per stage: one 128-byte swizzle row of bf16
constexpr int KW = 256;       // K per packed-W chunk (8 blocks per row)
constexpr int KSUB = KW / BK; // stages per W chunk
// A/B stages: 2 at N = 128 (64 KB each); 4 for narrow tiles, whose B
// half is small, to keep more K-steps of decoded A in flight.
constexpr int ab_stages_for(int nt) { return nt <= 32 ? 4 : 2; }
constexpr int W_STAGES = 2;
constexpr int kRowWarps = 8;  // warps 2..9: two per TMEM lane quarter, one K-step block each
constexpr int kGemmThreads = 32 * (2 + kRowWarps);
constexpr uint32_t tmem_cols_for(int nt) { return nt < 32 ? 32u : (uint32_t)nt; }  // power of 2, >= 32

constexpr int kGemmSmemMax = 232448;  // dynamic shared memory per CTA (227 KB)

template <int F, int NT>
struct GemmCfg {
    static constexpr int BS = Fmt<F>::kBlockBytes;
    static constexpr int W_ROW = (KW / kQK) * BS;  // bytes of one row's chunk: 272 / 144 / 160
    static constexpr int W_ESZ = F == kQ8_0 ? 2 : 1;  // tensor-map element (inner box <= 256 elems)
    static constexpr int W_TILE = BM * W_ROW;
    static constexpr int W_SLOT = (W_TILE + 1023) / 1024 * 1024;
    static constexpr int A_TILE = BM * BK * 2;  // bf16
    static constexpr int B_TILE = NT * BK * 2;
    static constexpr int AB_STAGE = 2 * A_TILE + 2 * B_TILE;  // A hi, A lo, B hi, B lo
    static constexpr int AB_FIT = (kGemmSmemMax - W_STAGES * W_SLOT - 1024) / AB_STAGE;
    static constexpr int AB_STAGES = ab_stages_for(NT) < AB_FIT ? ab_stages_for(NT) : AB_FIT;
    static constexpr int SMEM = AB_STAGES * AB_STAGE + W_STAGES * W_SLOT + 1024;  // + align slack
    static_assert(AB_STAGES >= 2 && SMEM <= kGemmSmemMax, "GEMM stages must fit shared memory");
    static_assert(AB_STAGE % 1024 == 0 && W_SLOT % 1024 == 0, "SW128 atoms need 1024-B aligned tiles");
    static_assert(W_ROW % 16 == 0, "W chunk row must be 16-byte granular");
};

// kind::f16 instruction descriptor of this kernel: D f32, A/B bf16, M = BM.
constexpr uint32_t idesc_for(int nt) { return idesc_f16kind(true, BM, nt); }

template <int NT>
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t accumulate) {
    mma_f16kind(tmem_d, adesc, bdesc, idesc_for(NT), accumulate);
}

// ---- exact decode of one block into bf16 hi/lo pairs --------------------------
// bw[] holds the block's bytes from its first byte (word 0 = its first 4
// bytes).  Writes the 32 values w (the reference's dequantized fp32 values,
// exactly) as 16 bf16x2 words hi[] and lo[] with w = hi + lo to ~2^-17:
//   q4_0:  w = d*(q-8) = fma(128+q, d, -136d)      (128+q by a byte permute
//          into the mantissa of 128.0f; 136d and the product are exact)
//   q4_1:  w = fma(d, q, m)                         (d*q exact, one rounding,
//          the same value as the reference's d*q + m)
//   q8_0:  w = d*q                                  (exact)
__device__ __forceinline__ void split_pair(float w0, float w1, uint32_t& h, uint32_t& l) {
    const __nv_bfloat162 hb = __floats2bfloat162_rn(w0, w1);
    h = *reinterpret_cast<const uint32_t*>(&hb);
    const float h0 = __uint_as_float(h << 16), h1 = __uint_as_float(h & 0xFFFF0000u);
    const __nv_bfloat162 lb = __floats2bfloat162_rn(w0 - h0, w1 - h1);
    l = *reinterpret_cast<const uint32_t*>(&lb);
}

template <int F>
__device__ __forceinline__ void decode_block_bf16(const uint32_t* bw, uint32_t hi[16], uint32_t lo[16]) {
    const float d = half_bits_to_float(bw[0] & 0xFFFFu);
    if constexpr (F == kQ8_0) {
        // bytes 2..33: value e at byte 2+e
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // values 4j..4j+3
            const uint32_t word = __funnelshift_r(bw[j], bw[j + 1], 16) ^ 0x80808080u;
            float w[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                w[u] = __fmul_rn(d, __uint_as_float(__byte_perm(word, 0x4B000000u, 0x7540 + u)) - 8388736.0f);
            split_pair(w[0], w[1], hi[2 * j], lo[2 * j]);
            split_pair(w[2], w[3], hi[2 * j + 1], lo[2 * j + 1]);
        }
    } else {
        constexpr int QS = F == kQ4_0 ? 2 : 4;  // first qs byte
        const float mn = F == kQ4_1 ? half_bits_to_float(bw[0] >> 16) : 0.0f;
        const float c = -136.0f * d;  // q4_0: exact (8-bit x 11-bit)
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // qs word j: values 4j..4j+3 (low nibbles), 16+4j.. (high)
            const uint32_t qw = QS == 2 ? __funnelshift_r(bw[j], bw[j + 1], 16) : bw[1 + j];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t nib = (h ? (qw >> 4) : qw) & 0x0F0F0F0Fu;
                float w[4];
#pragma unroll
                for (int u = 0; u < 4; ++u) {
                    const float f = __uint_as_float(__byte_perm(nib, 0x43000000u, 0x7044 + 0x100 * u));  // 128 + q
                    w[u] = F == kQ4_0 ? __fmaf_rn(f, d, c) : __fmaf_rn(d, f - 128.0f, mn);
                }
                const int e2 = (16 * h + 4 * j) / 2;  // pair index of value 16h + 4j
                split_pair(w[0], w[1], hi[e2], lo[e2]);
                split_pair(w[2], w[3], hi[e2 + 1], lo[e2 + 1]);
            }
        }
    }
}

template <int F, int NT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_xh,
                   const __grid_constant__ CUtensorMap tm_xl, GemmArgs a) {
    using C = GemmCfg<F, NT>;
    constexpr int AB_STAGES = C::AB_STAGES;
    constexpr uint32_t kTmemCols = tmem_cols_for(NT);
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    __shared__ __align__(8) uint64_t ab_full[AB_STAGES], ab_empty[AB_STAGES];
    __shared__ __align__(8) uint64_t w_full[W_STAGES], w_empty[W_STAGES];
    __shared__ __align__(8) uint64_t acc_full, acc_empty;
    __shared__ uint32_t tmem_base_s;
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;  // 1024-B aligned (SW128 atoms)
    auto a_hi = [&](int s) { return base + (uint32_t)(s * C::AB_STAGE); };
    auto a_lo = [&](int s) { return a_hi(s) + C::A_TILE; };
    auto b_hi = [&](int s) { return a_hi(s) + 2 * C::A_TILE; };
    auto b_lo = [&](int s) { return b_hi(s) + C::B_TILE; };
    auto w_st = [&](int s) { return base + (uint32_t)(AB_STAGES * C::AB_STAGE + s * C::W_SLOT); };

    if (threadIdx.x == 0) {
        for (int s = 0; s < AB_STAGES; ++s) {
            mbar_init(smem_u32(&ab_full[s]), 1 + kRowWarps);  // producer (B bytes) + row warps (A)
            mbar_init(smem_u32(&ab_empty[s]), 1);     // tcgen05.commit
        }
        for (int s = 0; s < W_STAGES; ++s) {
            mbar_init(smem_u32(&w_full[s]), 1);
            mbar_init(smem_u32(&w_empty[s]), kRowWarps);
        }
        mbar_init(smem_u32(&acc_full), 1);
        mbar_init(smem_u32(&acc_empty), kRowWarps);
        abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32(&tmem_base_s)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    const int tiles_n = (a.T + NT - 1) / NT;
    const int tiles_m = (a.out + BM - 1) / BM;
    const int ntiles = tiles_m * tiles_n * a.split;  // (row tile, token tile, K range)
    const int KS = (a.in + BK - 1) / BK;
    const int KSR = a.kchunks_per_split * KSUB;      // K-steps per range (whole W chunks)
    // tile -> row tile mt, token tile nt, K-steps [ks0, ks1) of range kr
    auto decompose = [&](int tile, int& mt, int& nt, int& kr, int& ks0, int& ks1) {
        kr = tile % a.split;
        const int mn = tile / a.split;
        mt = mn / tiles_n;
        nt = mn % tiles_n;
        ks0 = kr * KSR;
        ks1 = min(KS, ks0 + KSR);
    };

    if (warp == 0) {
        // ------------------------------ TMA producer ------------------------------
        if (lane == 0) {
            uint32_t g = 0, gc = 0;
            for (int tile = blockIdx.x; tile < ntiles && !*(volatile int*)&abort_flag; tile += gridDim.x) {
                int mt, nt, kr, ks0, ks1;
                decompose(tile, mt, nt, kr, ks0, ks1);
                for (int ks = ks0; ks < ks1; ++ks, ++g) {
                    if (ks % KSUB == 0) {
                        const int sw = (int)(gc % W_STAGES);
                        if (!mbar_wait(smem_u32(&w_empty[sw]), ((gc / W_STAGES) & 1u) ^ 1u)) {
                            report_error(a.err, 12);
                            abort_flag = 1;
                            break;
                        }
                        mbar_arrive_expect_tx(smem_u32(&w_full[sw]), (uint32_t)C::W_TILE);
                        tma_load_2d(w_st(sw), &tm_w, (ks / KSUB) * (C::W_ROW / C::W_ESZ), mt * BM,
                                    smem_u32(&w_full[sw]));
                        ++gc;
                    }
                    const int s = (int)(g % AB_STAGES);
                    if (!mbar_wait(smem_u32(&ab_empty[s]), ((g / AB_STAGES) & 1u) ^ 1u)) {
                        report_error(a.err, 12);
                        abort_flag = 1;
                        break;
                    }
                    mbar_arrive_expect_tx(smem_u32(&ab_full[s]), 2u * C::B_TILE);
                    tma_load_2d(b_hi(s), &tm_xh, ks * BK, nt * NT, smem_u32(&ab_full[s]));
                    tma_load_2d(b_lo(s), &tm_xl, ks * BK, nt * NT, smem_u32(&ab_full[s]));
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------ MMA issuer ------------------------------
        uint32_t tc = 0;
        if (lane == 0) {
            uint32_t g = 0;
            for (int tile = blockIdx.x; tile < ntiles && !*(volatile int*)&abort_flag; tile += gridDim.x, ++tc) {
                if (!mbar_wait(smem_u32(&acc_empty), (tc & 1u) ^ 1u)) {
                    report_error(a.err, 13);
                    abort_flag = 1;
                    break;
                }
                tc_fence_after();
                int mt, nt, kr, ks0, ks1;
                decompose(tile, mt, nt, kr, ks0, ks1);
                for (int ks = ks0; ks < ks1; ++ks, ++g) {
                    const int s = (int)(g % AB_STAGES);
                    if (!mbar_wait(smem_u32(&ab_full[s]), (g / AB_STAGES) & 1u)) {
                        report_error(a.err, 13);
                        abort_flag = 1;
                        break;
                    }
                    tc_fence_after();
                    const uint64_t dah = sw128_desc(a_hi(s)), dal = sw128_desc(a_lo(s));
                    const uint64_t dbh = sw128_desc(b_hi(s)), dbl = sw128_desc(b_lo(s));
#pragma unroll
                    for (int k = 0; k < BK / 16; ++k) {
                        const uint64_t adv = (uint64_t)(k * 32) >> 4;  // 16 bf16 = 32 B along K
                        mma_bf16<NT>(tmem, dah + adv, dbh + adv, (ks != ks0 || k != 0) ? 1u : 0u);
                        mma_bf16<NT>(tmem, dah + adv, dbl + adv, 1u);
                        mma_bf16<NT>(tmem, dal + adv, dbh + adv, 1u);
                    }
                    mma_commit(smem_u32(&ab_empty[s]));  // stage free once these MMAs finish
                }
                if (*(volatile int*)&abort_flag) break;
                mma_commit(smem_u32(&acc_full));  // accumulator complete
            }
            // drain: the last tile's epilogue has read TMEM before it is freed
            if (tc > 0 && !mbar_wait(smem_u32(&acc_empty), (tc - 1) & 1u)) report_error(a.err, 14);
        }
        __syncwarp();
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols)
                     : "memory");
    } else {
        // --------------------- row threads: decode A, epilogue ---------------------
        // Two warps per TMEM lane quarter: `half` 0 decodes block 0 of each
        // 64-wide K-step and reads accumulator columns 0..63, half 1 block 1
        // and columns 64..127.
        const int quarter = warp & 3;          // TMEM lanes 32*quarter .. +31
        const int half = (warp - 2) >> 2;      // 0: warps 2..5, 1: warps 6..9
        const int row = quarter * 32 + lane;   // tile row = TMEM lane
        const uint32_t swz = (uint32_t)(row & 7);
        uint32_t g = 0, gc = 0, tc = 0;
        for (int tile = blockIdx.x; tile < ntiles; tile += gridDim.x, ++tc) {
            int mt, nt, kr, ks0, ks1;
            decompose(tile, mt, nt, kr, ks0, ks1);
            int sw = 0;
            for (int ks = ks0; ks < ks1; ++ks, ++g) {
                if (ks % KSUB == 0) {
                    sw = (int)(gc % W_STAGES);
                    if (!mbar_wait(smem_u32(&w_full[sw]), (gc / W_STAGES) & 1u)) {
                        report_error(a.err, 15);
                        return;
                    }
                }
                const int s = (int)(g % AB_STAGES);
                if (!mbar_wait(smem_u32(&ab_empty[s]), ((g / AB_STAGES) & 1u) ^ 1u)) {
                    report_error(a.err, 15);
                    return;
                }
                // this row's block `half` of the K-step (zero-filled past the matrix)
                const int off = ((ks % KSUB) * 2 + half) * C::BS;  // block's first byte in the row chunk
                const uint32_t src = w_st(sw) + (uint32_t)(row * C::W_ROW + (off & ~3));
                // words covering the block from the 4-B boundary below it (18- and
                // 34-byte blocks start 2 bytes past one half the time); never past
                // the row chunk's end
                constexpr int NW = (C::BS + (C::BS % 4 ? 2 : 0) + 3) / 4;
                uint32_t raw[NW + 1];
#pragma unroll
                for (int j = 0; j < NW; ++j) raw[j] = lds_u32(src + 4 * j);
                raw[NW] = 0;
                uint32_t bw[NW];  // the block's bytes from its first byte
#pragma unroll
                for (int j = 0; j < NW; ++j) bw[j] = (off & 3) ? __funnelshift_r(raw[j], raw[j + 1], (off & 3) * 8) : raw[j];
                uint32_t h[16], l[16];
                decode_block_bf16<F>(bw, h, l);
                const uint32_t dst_hi = a_hi(s) + (uint32_t)row * 128u;
                const uint32_t dst_lo = a_lo(s) + (uint32_t)row * 128u;
#pragma unroll
                for (int c = 0; c < 4; ++c) {  // 16-byte chunks 4*half + c of the 64-value row
                    const uint32_t cs = ((((uint32_t)(4 * half + c)) ^ swz) << 4);
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst_hi + cs), "r"(h[4 * c]),
                                 "r"(h[4 * c + 1]), "r"(h[4 * c + 2]), "r"(h[4 * c + 3])
                                 : "memory");
                    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(dst_lo + cs), "r"(l[4 * c]),
                                 "r"(l[4 * c + 1]), "r"(l[4 * c + 2]), "r"(l[4 * c + 3])
                                 : "memory");
                }
                fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor cores
                __syncwarp();
                if (lane == 0) {
                    mbar_arrive(smem_u32(&ab_full[s]));
                    if (ks % KSUB == KSUB - 1 || ks == ks1 - 1) mbar_arrive(smem_u32(&w_empty[sw]));
                }
                if (ks % KSUB == KSUB - 1 || ks == ks1 - 1) ++gc;
            }
            // epilogue: TMEM -> registers -> y (consecutive rows across lanes)
            if (!mbar_wait(smem_u32(&acc_full), tc & 1u)) {
                report_error(a.err, 16);
                return;
            }
            tc_fence_after();
            const int o = mt * BM + row;
            // this thread's output feature: one bias value for all its columns
            // (split-K: the partials carry none; the reduction adds it)
            const bool has_bias = a.split == 1 && a.bias != nullptr && o < a.out;
            const float bo = has_bias ? a.bias[o] : 0.0f;
            float* const dst = a.split == 1 ? a.y : a.part + (long long)kr * a.T * a.out;
            // 32-column chunks of the accumulator, split between the halves
            constexpr int NCH = NT < 32 ? 1 : NT / 32;
            constexpr int PER = NCH >= 2 ? NCH / 2 : 1;
#pragma unroll 1
            for (int c = half * PER; c < (half + 1) * PER && c < NCH; ++c) {
                uint32_t v[32];
                tmem_ld32(tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 32), v);
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int t = nt * NT + c * 32 + j;
                    if (c * 32 + j >= NT) break;
                    if (o < a.out && t < a.T) {
                        const float yv = __uint_as_float(v[j]);
                        dst[(long long)t * a.out + o] = has_bias ? __fadd_rn(yv, bo) : yv;
                    }
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&acc_empty));
        }
    }
}

// Byte offset of the split-K partials in the workspace: after the x split,
// 256-B aligned.
size_t split_offset(int in, int T) {
    return ((size_t)T * in * 2 * sizeof(__nv_bfloat16) + 255) & ~(size_t)255;
}

// x fp32 [T][K] -> xh = bf16_rn(x), xl = bf16_rn(x - xh), both [T][K].
__global__ void xsplit_kernel(const float* __restrict__ x, long long n, __nv_bfloat16* __restrict__ xh,
                              __nv_bfloat16* __restrict__ xl) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        const float v = x[i];
        const __nv_bfloat16 h = __float2bfloat16_rn(v);
        xh[i] = h;
        xl[i] = __float2bfloat16_rn(v - __bfloat162float(h));
    }
}

// y[i] = sum over the split K ranges of part[r][i] (range order), + bias.
__global__ void splitk_reduce_kernel(const float* __restrict__ part, int split, long long n, int out,
                                     const float* __restrict__ bias, float* __restrict__ y) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n;
         i += (long long)gridDim.x * blockDim.x) {
        float v = part[i];
        for (int r = 1; r < split; ++r) v = __fadd_rn(v, part[(long long)r * n + i]);
        if (bias) v = __fadd_rn(v, bias[i % out]);
        y[i] = v;
    }
}

template <int F, int NT>
cudaError_t launch_gemm_t(const uint8_t* w, const float* x, float* y, int out, int in, int T,
                          const float* bias, void* ws, int split, int sm_count, int* err, cudaStream_t stream) {
    using C = GemmCfg<F, NT>;
    __nv_bfloat16* xh = static_cast<__nv_bfloat16*>(ws);
    __nv_bfloat16* xl = xh + (size_t)T * in;
    const long long n = (long long)T * in;
    xsplit_kernel<<<(int)((n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096), 256, 0, stream>>>(x, n, xh, xl);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;

    const long long row_bytes = (long long)((in + kQK - 1) / kQK) * C::BS;
    CUtensorMap mw, mxh, mxl;
    if (!make_map_2d(&mw, F == kQ8_0 ? CU_TENSOR_MAP_DATA_TYPE_UINT16 : CU_TENSOR_MAP_DATA_TYPE_UINT8,
                     const_cast<uint8_t*>(w), (uint64_t)(row_bytes / C::W_ESZ), (uint64_t)out,
                     (uint64_t)row_bytes, (uint32_t)(C::W_ROW / C::W_ESZ), BM,
                     CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !make_map_2d(&mxh, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xh, (uint64_t)in, (uint64_t)T,
                     (uint64_t)in * 2, BK, NT, CU_TENSOR_MAP_SWIZZLE_128B) ||
        !make_map_2d(&mxl, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, xl, (uint64_t)in, (uint64_t)T,
                     (uint64_t)in * 2, BK, NT, CU_TENSOR_MAP_SWIZZLE_128B))
        return cudaErrorInvalidValue;

    static std::atomic<bool> attr_set[64];  // one value per instantiation: racing first calls agree
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
        e = cudaFuncSetAttribute(gemm_tc_kernel<F, NT>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_set[dev].store(true, std::memory_order_release);
    }
    GemmArgs a{};
    a.y = y;
    a.bias = bias;
    a.out = out;
    a.in = in;
    a.T = T;
    a.err = err;
    const int chunks = (in + KW - 1) / KW;  // W chunks along K
    if (split < 1) split = 1;
    a.kchunks_per_split = (chunks + split - 1) / split;
    a.split = (chunks + a.kchunks_per_split - 1) / a.kchunks_per_split;  // no empty range
    a.part = a.split > 1 ? reinterpret_cast<float*>(static_cast<char*>(ws) + split_offset(in, T)) : nullptr;
    const int ntiles = ((out + BM - 1) / BM) * ((T + NT - 1) / NT) * a.split;
    const int grid = ntiles < sm_count ? ntiles : sm_count;
    gemm_tc_kernel<F, NT><<<grid, kGemmThreads, C::SMEM, stream>>>(mw, mxh, mxl, a);
    e = cudaGetLastError();
    if (e != cudaSuccess || a.split == 1) return e;
    const long long ny = (long long)T * out;
    const long long nb = (ny + 255) / 256;
    splitk_reduce_kernel<<<(int)(nb < 4 * sm_count ? nb : 4 * sm_count), 256, 0, stream>>>(a.part, a.split, ny,
                                                                                         out, bias, y);
    return cudaGetLastError();
}

// Narrowest tile that covers the rows of x (wider calls tile by 128).
template <int F>
cudaError_t launch_gemm_f(const uint8_t* w, const float* x, float* y, int out, int in, int T,
                          const float* bias, void* ws, int split, int sm_count, int* err, cudaStream_t stream) {
    if (T <= 16) return launch_gemm_t<F, 16>(w, x, y, out, in, T, bias, ws, split, sm_count, err, stream);
    if (T <= 32) return launch_gemm_t<F, 32>(w, x, y, out, in, T, bias, ws, split, sm_count, err, stream);
    if (T <= 64) return launch_gemm_t<F, 64>(w, x, y, out, in, T, bias, ws, split, sm_count, err, stream);
    return launch_gemm_t<F, 128>(w, x, y, out, in, T, bias, ws, split, sm_count, err, stream);
}

}  // namespace

bool gemm_shape_ok(int fmt, const void* w, int out, int in, int rows) {
    const long long row_bytes = (long long)((in + kQK - 1) / kQK) * block_bytes(fmt);
    return MLQ_GEMM_ROWS_RULE(rows, out, in) && reinterpret_cast<uintptr_t>(w) % 16 == 0 && row_bytes % 16 == 0 &&
           in % 8 == 0;
}

bool gemm_supported(int fmt, const void* w, int out, int in, int rows) {
    return gemm_shape_ok(fmt, w, out, in, rows) && encode_fn() != nullptr;
}

int gemm_split(int out, int in, int rows, int sm_count) {
    const int nt = rows <= 16 ? 16 : rows <= 32 ? 32 : rows <= 64 ? 64 : 128;
    const long long tiles = (long long)((out + BM - 1) / BM) * ((rows + nt - 1) / nt);
    const int chunks = (in + KW - 1) / KW;
    if (tiles >= sm_count || chunks < 2) return 1;
    long long s = sm_count / tiles;
    if (s > 8) s = 8;  // each range adds a T x out partial to write and read back
    if (s > chunks) s = chunks;
    return s < 1 ? 1 : (int)s;
}

size_t gemm_workspace_bytes(int in, int rows, int out, int split) {
    const size_t xs = split_offset(in, rows);
    return split > 1 ? xs + (size_t)split * rows * out * sizeof(float) : (size_t)rows * in * 2 * sizeof(__nv_bfloat16);
}

cudaError_t launch_gemm(int fmt, const uint8_t* w, const float* x, float* y, int out, int in, int rows,
                        const float* bias, void* ws, int split, int sm_count, int* err, cudaStream_t stream) {
    switch (fmt) {
        case kQ8_0: return launch_gemm_f<kQ8_0>(w, x, y, out, in, rows, bias, ws, split, sm_count, err, stream);
        case kQ4_0: return launch_gemm_f<kQ4_0>(w, x, y, out, in, rows, bias, ws, split, sm_count, err, stream);
        case kQ4_1: return launch_gemm_f<kQ4_1>(w, x, y, out, in, rows, bias, ws, split, sm_count, err, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mlq
