// mlq_gemv.cu -- dequant-fused GEMV for decode (rows of x <= 8 per launch).
//
// Replaces q80LinearKernel / q40LinearKernel / q41LinearKernel
// (src/cuda_quant.cu:78-182 of the reference).  Same arithmetic contract:
// fp32 activations, exact decode of the packed weights, fp32 accumulation;
// only the summation order differs.
//
// Design (HBM-bound streaming, persistent grid of one or two CTAs per SM):
//  * Rows are processed in tiles of RT = 8 consumer warps x RPW rows, each
//    tile over the full K extent in K-tiles of 32 lane-groups (2048 values
//    for q8_0/q4_0, 1024 for q4_1).  A CTA takes a balanced contiguous row
//    range, or -- one token and at least 8 tiles per CTA -- row tiles from a
//    per-launch global queue, so faster SMs do more tiles.
//  * Warp 0 streams the weights: a stage is RT rows x one K-tile, fetched
//    as 2-D tensor-map boxes of 8 rows (or, when the row pitch is not a
//    multiple of 16 B, one 1-D cp.async.bulk per row segment); consumers
//    hand a stage back as soon as its words are in registers.
//  * x tiles: kept resident (every K-tile's tile built once) when they fit
//    next to two weight stages, otherwise riding a ring with the stages.
//    Warps 9.. build them (coalesced 128-bit loads, per-block sums); in the
//    one-token mode all nine non-producer warps build the resident tiles
//    together before the consumers start.
//  * Warps 1..8 consume: lane l decodes lane-group l (2 blocks = 9 or 17
//    words, or 1 q4_1 block = 5 words; odd word counts make the 32 lanes'
//    32-bit shared loads bank-conflict free) of RPW rows, reusing every x
//    value it loads for all RPW rows.
//  * One token (integer mode): x as three int8 slices per value against its
//    block's scale (24-bit block fixed point), codes x slices by DP4A, one
//    fold per block (see the integer-mode section below).
//  * Two to eight tokens (fp32 mode): decode without int->float
//    conversions -- a nibble (or a sign-flipped byte) is dropped into the
//    mantissa of a float constant with one PRMT:
//      q4:  float(0x43000000 | q << 16) = 128 + q (exact)
//      q8:  float(0x4B000000 | (q^0x80)) = 2^23+128+q (exact), minus 2^23+128
//    accumulated with packed FFMA2; the per-block constant is folded back
//    with the block's x-sum S:
//      q4_0:  d * (sum (128+q) x - 136 S)
//      q4_1:  d * (sum (128+q) x - 128 S) + m S
//      q8_0:  d * sum q x
//    The fold costs ~7 bits of the fp32 block sum against S; measured
//    relative errors stay near 1e-6 (the contract allows 1e-3).
//  * Launched with programmatic stream serialization: weights stream while
//    the previous kernel drains; x and y wait for it (griddepcontrol).
//  * Sharded calls store every row into every rank's y (NVLink peer
//    stores) and end with a cross-GPU completion handshake.
//  * Epilogues: an optional bias add in the store (runtime check), or -- a
//    separate instantiation -- a SwiGLU pair: each row tile carries the
//    same rows of the gate and up matrices (two tensor maps), and the store
//    writes silu(gate) * up (the feed-forward input of the reference's
//    ffnForwardDevice, src/forward.cc:573-581).
//  * Every mbarrier wait is bounded (2 s); on expiry the kernel records an
//    error code in *err and returns after its in-flight copies land.
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <cstring>
#include <map>
#include <mutex>

#include "mlq_device.cuh"
#include "mlq_kernels.h"
#include "mlq_tmap.h"

namespace mlq {

// Dynamic row-tile queues: one {next tile, finished CTAs} pair per launch.
// Each CUDA stream that launches a queued GEMV gets a ring of its own
// (kStreamRings rings per device; streams beyond that use static row ranges),
// and its launches take the ring's slots round-robin.  Launches on one stream
// overlap at most pairwise (programmatic dependent launch), so a slot is free
// again long before its ring comes back to it, whatever other streams do.
// Every CTA of a launch counts itself in the pair's second word when its
// producer is done with the queue -- on the normal path and after an abort --
// and the last one puts the pair back to zero (it is zero at module load, and
// mlq_device_error clears the whole array after a kernel reported an error).
constexpr int kStreamRings = 64;
constexpr int kSlotsPerRing = 32;
constexpr int kTileSlots = kStreamRings * kSlotsPerRing;
__device__ unsigned int g_gemv_tile_slots[2 * kTileSlots];

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kXWarp = 1 + kConsumerWarps;  // warps 9.. build the x tiles
// x-loader warps: one; four for eight tokens (a stage's x tile is then
// 64 KB, more than one warp turns around in a consumer's stage time)
constexpr int xw_for(int mt) { return mt >= 8 ? 4 : 1; }
constexpr int threads_for(int mt) { return 32 * (1 + kConsumerWarps + xw_for(mt)); }
constexpr int kMaxStages = 8;

template <int F, int MT, int RPW, bool INT>
struct GemvCfg {
    static constexpr int G = Fmt<F>::kGroupBlocks;
    static constexpr int BS = Fmt<F>::kBlockBytes;
    static constexpr int GB = G * BS;            // bytes per lane-group
    static constexpr int WPG = GB / 4;           // 32-bit words per lane-group (odd)
    static constexpr int KTE = 32 * G * kQK;     // x values per K-tile
    static constexpr int RT = kConsumerWarps * RPW;
    static constexpr int SLOT = 32 * GB + 16;    // one tile row segment + align slack
    static constexpr int W_BYTES = RT * SLOT;
    // x tile of a K-tile: fp32 values (FP mode) or three int8 slices per
    // value, as 6 rows of 32 lanes x 16 B per block of a lane-group (INT mode)
    static constexpr int X_BYTES = INT ? MT * G * 6 * 512 : MT * KTE * 4;
    // per block: x sum (FP mode) or (slice scale, x sum) (INT mode)
    static constexpr int S_BYTES = MT * 32 * G * (INT ? 8 : 4);
    static constexpr int XT_BYTES = X_BYTES + S_BYTES;  // x tile (x + block sums) of a stage
    // 2-D tensor-map layout of a stage's weights: boxes of 8 rows x one
    // K-tile of bytes, as 8-byte elements (a box row is <= 256 elements, so
    // q8_0's 2176-byte K-tile row is split into two regions of 16 groups).
    // Every box destination must be 128-byte aligned (tensor TMA), so the
    // regions are not offset against each other; q8_0's half-warps then
    // share banks (2-way conflicts on its weight loads).
    static constexpr int KTB = 32 * GB;
    static constexpr int NREG = (KTB / 8 > 256) ? 2 : 1;
    static constexpr int BOXB = KTB / NREG;
    static constexpr int BOXW = BOXB / 8;
    static constexpr int REGION = RT * BOXB;
    static_assert(REGION % 128 == 0 && (8 * BOXB) % 128 == 0 && W_BYTES % 128 == 0 &&
                      XT_BYTES % 128 == 0,
                  "tensor TMA destinations must be 128-byte aligned");
    static_assert(NREG * REGION <= W_BYTES, "2-D layout must fit the stage");
    static_assert(BOXB % 16 == 0, "box rows must be 16-byte granular");
    static_assert(WPG % 2 == 1, "lane-group word count must be odd");
    static_assert(SLOT % 16 == 0, "stage alignment");
    static_assert(!INT || MT == 1, "integer mode is the one-token path");
};

// x-tile row ("part") p of block bg holds 4 consecutive x values; the 8
// parts of a block in the order the consumers walk the packed codes:
//   q4:  p = 2j + h  ->  values 16h + 4j .. +3   (qs word j, nibble half h)
//   q8:  p = j       ->  values 4j .. +3         (qs word j)
template <int F>
__device__ __forceinline__ int part_of(int e) {
    if constexpr (F == kQ8_0) {
        return e >> 2;
    } else {
        return (((e & 15) >> 2) << 1) | (e >> 4);
    }
}

// Four packed codes -> four floats.  q4: every byte of `nib` is one code
// q (0..15); dropped into byte 2 under exponent byte 0x43 it gives the float
// 128 + q exactly.
__device__ __forceinline__ void q4_to_f(uint32_t nib, float f[4]) {
    f[0] = __uint_as_float(__byte_perm(nib, 0x43000000u, 0x7044));
    f[1] = __uint_as_float(__byte_perm(nib, 0x43000000u, 0x7144));
    f[2] = __uint_as_float(__byte_perm(nib, 0x43000000u, 0x7244));
    f[3] = __uint_as_float(__byte_perm(nib, 0x43000000u, 0x7344));
}

// Nibble half h of a qs word, one code per byte.
__device__ __forceinline__ uint32_t q4_nibbles(uint32_t qw, int h) {
    return (h ? (qw >> 4) : qw) & 0x0F0F0F0Fu;
}

__device__ __forceinline__ void q8_to_f(uint32_t word, float f[4]) {
    const uint32_t u = word ^ 0x80808080u;
    const float c = 8388736.0f;  // 2^23 + 128
    f[0] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7540)) - c;
    f[1] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7541)) - c;
    f[2] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7542)) - c;
    f[3] = __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7543)) - c;
}

// qs word j (0-based) of block bg inside the lane-group words wv[].
template <int F>
__device__ __forceinline__ uint32_t qs_word(const uint32_t* wv, int bg, int j) {
    if constexpr (F == kQ4_1) {
        return wv[1 + j];
    } else if constexpr (F == kQ4_0) {
        // block 0: bytes 2..17 (misaligned by 2), block 1: bytes 20..35 = words 5..8
        return bg == 0 ? __byte_perm(wv[j], wv[j + 1], 0x5432) : wv[5 + j];
    } else {
        // block 0: bytes 2..33, block 1: bytes 36..67 = words 9..16
        return bg == 0 ? __byte_perm(wv[j], wv[j + 1], 0x5432) : wv[9 + j];
    }
}

template <int F>
__device__ __forceinline__ uint32_t d_bits(const uint32_t* wv, int bg) {
    if constexpr (F == kQ4_1) return wv[0] & 0xFFFFu;
    if constexpr (F == kQ4_0) return bg == 0 ? (wv[0] & 0xFFFFu) : (wv[4] >> 16);
    return bg == 0 ? (wv[0] & 0xFFFFu) : (wv[8] >> 16);
}

// --- integer mode -----------------------------------------------------------
// One token: x is carried as three int8 slices per value, relative to its
// 32-value block's scale s = max|x| / 127:
//     x / s = h + m / 254 + l / 254^2 + e,   h, m, l in [-127, 127], |e| <= 1/(2*254^2)
// i.e. 24-bit block fixed point, |x - s (h + m/254 + l/254^2)| <= 6.1e-8 max|x| --
// the size of one fp32 rounding of the block's largest value.  The codes
// (q4: 0..15, q8: -128..127) then meet the slices in DP4A: four 8-bit
// products summed exactly per instruction, one int32 sum per slice, block
// and row.  The fold per block:
//     sum q x = s * (H + (254 M + L) / 254^2)          (H, M, L the slice sums)
//     q4_0:  d * (that - 8 S),  q4_1:  d * that + m S,  q8_0:  d * that
// with S the block's x sum.
constexpr float kRound = 12582912.0f;        // 1.5 * 2^23: x + kRound rounds x to an integer
constexpr float kInvSlice2 = 1.0f / 64516.0f;  // 1 / 254^2

// Low byte of a kRound-biased float = its integer as a two's-complement byte.
__device__ __forceinline__ uint32_t pack_low_bytes(float a, float b, float c, float d) {
    const uint32_t ab = __byte_perm(__float_as_uint(a), __float_as_uint(b), 0x0040);
    const uint32_t cd = __byte_perm(__float_as_uint(c), __float_as_uint(d), 0x0040);
    return __byte_perm(ab, cd, 0x5410);
}

// Column (16-byte unit) of lane-group g's quad q (q = 2*bg + half) in an
// INT-mode x-tile row: lanes of one 8-lane store phase land in 8 distinct
// bank groups, and every reader lane of a row in a distinct one.
template <int G>
__device__ __forceinline__ uint32_t xcol(int g, int q) {
    return (uint32_t)((g + (4 / G) * q) & 31) * 16u;
}

// INT mode x tile, piece i of K-tile k0 for this lane: 16 values
// [k0 + 16 (32 i + lane), +16) = one half of block (32 i + lane) / 2.
template <int G>
__device__ __forceinline__ void int_piece_load(const float* x, int in, long long k0, int i, int lane,
                                               float v[16]) {
    const long long e0 = k0 + 16LL * (i * 32 + lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e0 + 4 * j < in) q4 = ldg_nc_f4(x + e0 + 4 * j);
        v[4 * j] = q4.x;
        v[4 * j + 1] = q4.y;
        v[4 * j + 2] = q4.z;
        v[4 * j + 3] = q4.w;
    }
}

// The same piece from x staged in shared memory at `xst` (x[0] at xst).
__device__ __forceinline__ void int_piece_load_smem(uint32_t xst, int in, long long k0, int i, int lane,
                                                    float v[16]) {
    const long long e0 = k0 + 16LL * (i * 32 + lane);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        float4 q4 = make_float4(0.f, 0.f, 0.f, 0.f);
        if (e0 + 4 * j < in) q4 = lds_f4(xst + (uint32_t)((e0 + 4 * j) * 4));
        v[4 * j] = q4.x;
        v[4 * j + 1] = q4.y;
        v[4 * j + 2] = q4.z;
        v[4 * j + 3] = q4.w;
    }
}

// Slices of one piece into x tile `xs` (+ scale/sum pair into `ss`).  The two
// lanes holding a block's halves are neighbours (shuffle partners).
template <int G>
__device__ __forceinline__ void int_piece_store(const float v[16], int i, int lane, uint32_t xs,
                                                uint32_t ss) {
    const int gi = i * 32 + lane;
    const int blk = gi >> 1, half = gi & 1;
    const int g = blk / G, bg = blk % G;
    float mx = 0.f, sum = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
        mx = fmaxf(mx, fabsf(v[e]));
        sum += v[e];
    }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    // blocks of (near-)zero magnitude carry no slices
    const float inv = mx > 1e-30f ? __fdiv_rn(127.0f, mx) : 0.0f;
    uint32_t wh[4], wm[4], wl[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float fh[4], fm[4], fl[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const float xv = v[4 * q + u];
            fh[u] = fmaf(xv, inv, kRound);
            const float r = fmaf(xv, inv, -(fh[u] - kRound));  // exact, |r| <= 1/2
            fm[u] = fmaf(r, 254.0f, kRound);
            const float r2 = fmaf(r, 254.0f, -(fm[u] - kRound));
            fl[u] = fmaf(r2, 254.0f, kRound);
        }
        wh[q] = pack_low_bytes(fh[0], fh[1], fh[2], fh[3]);
        wm[q] = pack_low_bytes(fm[0], fm[1], fm[2], fm[3]);
        wl[q] = pack_low_bytes(fl[0], fl[1], fl[2], fl[3]);
    }
    const uint32_t col = xcol<G>(g, 2 * bg + half);
    const uint32_t row = (uint32_t)(bg * 6 + half) * 512u;
    sts_u4(xs + row + col, make_uint4(wh[0], wh[1], wh[2], wh[3]));
    sts_u4(xs + row + 1024u + col, make_uint4(wm[0], wm[1], wm[2], wm[3]));
    sts_u4(xs + row + 2048u + col, make_uint4(wl[0], wl[1], wl[2], wl[3]));
    // scale (NaN/Inf in x poison it, as they would the fp32 sum) and x sum
    if (half == 0) sts_f2(ss + (uint32_t)blk * 8u, make_float2(fmaf(0.0f, sum, mx * (1.0f / 127.0f)), sum));
}

// One K-tile of one lane in integer mode: the lane-group words wv[r] of RPW
// rows against the x tile at xs (slices; xoff[q] this lane's column in quad
// q's rows) and the lane's (scale, x sum) pairs at ss, folded into tot[r].
template <int F, int RPW>
__device__ __forceinline__ void int_ktile(const uint32_t (&wv)[RPW][GemvCfg<F, 1, RPW, true>::WPG], uint32_t xs,
                                          uint32_t ss, const uint32_t (&xoff)[8], float (&tot)[RPW][1]) {
    constexpr int G = Fmt<F>::kGroupBlocks;
#pragma unroll
    for (int bg = 0; bg < G; ++bg) {
        const float2 sc = lds_f2(ss + (uint32_t)bg * 8u);
        uint4 xq[6];  // (slice, half): x slices of this lane's block bg
#pragma unroll
        for (int k = 0; k < 6; ++k) xq[k] = lds_u4(xs + (uint32_t)(bg * 6 + k) * 512u + xoff[2 * bg + (k & 1)]);
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            uint32_t c[8];
            if constexpr (F == kQ8_0) {
#pragma unroll
                for (int j = 0; j < 8; ++j) c[j] = qs_word<F>(wv[r], bg, j);
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const uint32_t qw = qs_word<F>(wv[r], bg, j);
                    c[j] = qw & 0x0F0F0F0Fu;
                    c[4 + j] = (qw >> 4) & 0x0F0F0F0Fu;
                }
            }
            int acc[3];
#pragma unroll
            for (int sl = 0; sl < 3; ++sl) {
                const uint4 lo = xq[2 * sl], hi = xq[2 * sl + 1];
                int v = __dp4a((int)c[0], (int)lo.x, 0);
                v = __dp4a((int)c[1], (int)lo.y, v);
                v = __dp4a((int)c[2], (int)lo.z, v);
                v = __dp4a((int)c[3], (int)lo.w, v);
                v = __dp4a((int)c[4], (int)hi.x, v);
                v = __dp4a((int)c[5], (int)hi.y, v);
                v = __dp4a((int)c[6], (int)hi.z, v);
                v = __dp4a((int)c[7], (int)hi.w, v);
                acc[sl] = v;
            }
            const float qx =
                sc.x * fmaf(__int2float_rn(acc[1] * 254 + acc[2]), kInvSlice2, __int2float_rn(acc[0]));
            const float d = half_bits_to_float(d_bits<F>(wv[r], bg));
            if constexpr (F == kQ4_0) {
                tot[r][0] = fmaf(d, fmaf(-8.0f, sc.y, qx), tot[r][0]);
            } else if constexpr (F == kQ4_1) {
                tot[r][0] = fmaf(d, qx, tot[r][0]);
                tot[r][0] = fmaf(half_bits_to_float(wv[r][0] >> 16), sc.y, tot[r][0]);
            } else {
                tot[r][0] = fmaf(d, qx, tot[r][0]);
            }
        }
    }
}

constexpr int log2_of(int n) { return n <= 1 ? 0 : 1 + log2_of(n / 2); }

// A CTA's producer is done taking tiles from the launch's queue {next, done}:
// count it; the last CTA of the grid puts the pair back to zero.
__device__ __forceinline__ void release_tile_queue(unsigned int* tiles) {
    __threadfence();
    if (atomicAdd(tiles + 1, 1u) == gridDim.x - 1) {
        atomicExch(tiles, 0u);
        atomicExch(tiles + 1, 0u);
    }
}

// Sharded-call completion counter: CTAs that gave up add this bit with their
// count, so the launch's last CTA knows not to publish the epoch.
constexpr unsigned int kDonePoison = 1u << 16;

// What a launch does after the sums: store y (+ bias, when the call has one:
// a runtime check, so plain and bias calls share one kernel), or -- a
// separate instantiation -- store silu(gate) * up for a SwiGLU pair.
// (Measured on the decode step: a separate bias instantiation cost ~3 us per
// step more than the runtime check, and a plain kernel carrying the pair's
// code as runtime branches ~3 us more than without it.)
constexpr int kEpiPlain = 0, kEpiPair = 2;

// The weights' tensor maps: one, or gate and up for a pair.
template <int N>
struct WMaps {
    CUtensorMap m[N];
};

// Sum of v[r][0] over the 32 lanes for every row r < RPW (1, 2 or 4), as a
// reduce-scatter: after it, the lanes of block k of 32/RPW consecutive lanes
// hold row k's total.
template <int RPW, int MT>
__device__ __forceinline__ float reduce_rows(float (&v)[RPW][MT], int lane) {
    float k;
    if constexpr (RPW == 4) {
        const bool up = lane & 16;
        float k0 = up ? v[2][0] : v[0][0], k1 = up ? v[3][0] : v[1][0];
        const float s0 = up ? v[0][0] : v[2][0], s1 = up ? v[1][0] : v[3][0];
        k0 += __shfl_xor_sync(0xffffffffu, s0, 16);
        k1 += __shfl_xor_sync(0xffffffffu, s1, 16);
        const bool up8 = lane & 8;
        k = up8 ? k1 : k0;
        k += __shfl_xor_sync(0xffffffffu, up8 ? k0 : k1, 8);
        k += __shfl_xor_sync(0xffffffffu, k, 4);
    } else if constexpr (RPW == 2) {
        const bool up = lane & 16;
        k = up ? v[1][0] : v[0][0];
        k += __shfl_xor_sync(0xffffffffu, up ? v[0][0] : v[1][0], 16);
        k += __shfl_xor_sync(0xffffffffu, k, 8);
        k += __shfl_xor_sync(0xffffffffu, k, 4);
    } else {
        k = v[0][0];
        k += __shfl_xor_sync(0xffffffffu, k, 16);
        k += __shfl_xor_sync(0xffffffffu, k, 8);
        k += __shfl_xor_sync(0xffffffffu, k, 4);
    }
    k += __shfl_xor_sync(0xffffffffu, k, 2);
    k += __shfl_xor_sync(0xffffffffu, k, 1);
    return k;
}

template <int F, int MT, int RPW, int MINB, bool INT, int EPI>
__global__ void __launch_bounds__(threads_for(MT), MINB)
    gemv_stream_kernel(GemvArgs a, const __grid_constant__ WMaps<EPI == kEpiPair ? 2 : 1> wm) {
    using C = GemvCfg<F, MT, RPW, INT>;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];   // weights released (early)
    __shared__ __align__(8) uint64_t xfull_bar[kMaxStages];   // x tile landed
    __shared__ __align__(8) uint64_t xempty_bar[kMaxStages];  // x tile released
    __shared__ int abort_flag;
    __shared__ float tile_res[2][MT * C::RT];  // per-tile results, double-buffered
    __shared__ __align__(8) uint64_t tile_bar;  // consumer warps' per-tile rendezvous
    __shared__ __align__(8) uint64_t xready_bar;  // INT resident mode: all x tiles built
    __shared__ __align__(8) uint64_t xstage_bar;  // INT resident mode: x staged in shared memory
    __shared__ int stage_row[kMaxStages];         // dynamic mode: first row of each stage's tile (-1: end)

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int S = a.nstages;
    const bool xres = a.x_resident != 0;
    // SwiGLU pair: a tile holds TR rows of each matrix (gate rows in stage
    // rows [0, TR), the same rows of up in [TR, RT)); otherwise RT rows of one
    constexpr bool pair = EPI == kEpiPair;
    constexpr int TR = pair ? C::RT / 2 : C::RT;
    const bool has_bias = !pair && a.bias != nullptr;
    const CUtensorMap& wmap = wm.m[0];
    const CUtensorMap& wmap2 = wm.m[pair ? 1 : 0];

    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 32);
            mbar_init(smem_u32(&empty_bar[s]), kConsumerWarps);
            mbar_init(smem_u32(&xfull_bar[s]), xw_for(MT));
            mbar_init(smem_u32(&xempty_bar[s]), kConsumerWarps);
        }
        mbar_init(smem_u32(&tile_bar), kConsumerWarps);
        mbar_init(smem_u32(&xready_bar), kConsumerWarps + 1);
        mbar_init(smem_u32(&xstage_bar), 1);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    // The next kernel in the stream may come up on SMs this grid frees (a
    // kPdlFirst launch lets it only after its own wait, in the consumers).
    if (a.pdl_mode != kPdlFirst) launch_dependents();
    // the wait for the previous kernel before x is read (none in a run of
    // independent launches: the run's first launch has waited)
    auto dep_wait = [&]() {
        if (a.pdl_mode != kPdlNoWait) grid_dependency_wait();
    };

    // balanced row ranges in units of 8 rows (the 2-D boxes' height)
    const long long units = (a.out + 7) / 8;
    const long long r_begin = 8 * ((long long)blockIdx.x * units / gridDim.x);
    const long long r_end = min((long long)a.out, 8 * ((long long)(blockIdx.x + 1) * units / gridDim.x));
    const int nrows_cta = (int)(r_end - r_begin);
    const int ntiles = (nrows_cta + TR - 1) / TR;
    const uint32_t smem_base = (smem_u32(smem) + 127u) & ~127u;  // TMA boxes: 128-B aligned
    // S weight stages, then the x slots (one per K-tile when resident, else one per stage)
    const uint32_t x_base = smem_base + (uint32_t)S * C::W_BYTES;
    const uintptr_t wbase = reinterpret_cast<uintptr_t>(a.w);
    const uintptr_t wend16 = (wbase + (uintptr_t)a.total_bytes) & ~(uintptr_t)15;
    const uintptr_t w2base = reinterpret_cast<uintptr_t>(a.w2);
    const uintptr_t w2end16 = (w2base + (uintptr_t)a.total_bytes) & ~(uintptr_t)15;

    // Dynamic tiles (one token, resident x, many tiles): CTAs take row tiles
    // from a global queue instead of a fixed row range, so SMs that stream
    // faster do more tiles and all CTAs finish together.
    const bool dyn = INT && xres && a.tiles != nullptr;
    const long long ntiles_all = (a.out + TR - 1) / TR;

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        // x into L2 ahead of the weight stream: the first CTAs each take a
        // 4 KB chunk.  Only a hint -- the x loads proper come after the grid
        // dependency, so a producer kernel still writing x is harmless.
        {
            const long long xbytes = (long long)a.M * a.in * 4;
            const long long nchunk = (xbytes + 4095) / 4096;
            if (lane == 0 && blockIdx.x < nchunk) {
                const long long off = (long long)blockIdx.x * 4096;
                const long long len = min(4096LL, xbytes - off);
                prefetch_l2(reinterpret_cast<const uint8_t*>(a.x) + off, (uint32_t)len);
            }
        }
        uint32_t seq = 0;
        int s = 0;
        uint32_t ph = 0;
        // every weight byte is read once per launch: evict-first in L2
        const uint64_t wpol = l2_evict_first_policy();
        // lane 0 holds the next queue ticket, fetched one tile ahead
        unsigned int ticket = (dyn && lane == 0) ? atomicAdd(a.tiles, 1u) : 0u;
        for (int t = 0; dyn || t < ntiles; ++t) {
            long long row0;
            if (dyn) {
                const unsigned int cur = __shfl_sync(0xffffffffu, ticket, 0);
                if ((long long)cur >= ntiles_all) break;
                if (lane == 0) ticket = atomicAdd(a.tiles, 1u);
                row0 = (long long)cur * TR;
            } else {
                row0 = r_begin + (long long)t * TR;
            }
            const int nrows = (int)min((long long)TR, (dyn ? (long long)a.out : r_end) - row0);
            for (int kt = 0; kt < a.ktiles; ++kt, ++seq) {
                // resident integer mode: one stage in flight until the x tiles
                // are built, so the x loads do not queue behind the weights
                if (INT && xres && seq == 1 && !mbar_wait(smem_u32(&xready_bar), 0u)) {
                    report_error(a.err, 7);
                    abort_flag = 1;
                }
                const uint32_t fb = smem_u32(&full_bar[s]);
                if (!mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u)) {
                    report_error(a.err, 2);
                    abort_flag = 1;
                }
                if (*(volatile int*)&abort_flag) goto producer_drain;
                const uint32_t stage = smem_base + (uint32_t)s * C::W_BYTES;
                if (dyn && lane == 0) stage_row[s] = (int)row0;
                const int groups = min(32, a.gpr - kt * 32);
                const uint32_t seg = (uint32_t)(groups * C::GB);
                if (a.tma2d) {
                    // boxes of 8 rows x K-tile bytes (x2 regions for q8_0); a
                    // pair's second matrix fills the boxes from stage row TR on
                    const int nb = (nrows + 7) / 8;
                    const int nbox = (pair ? 2 * nb : nb) * C::NREG;
                    if (lane == 0) mbar_expect_tx(fb, (uint32_t)(nbox * 8 * C::BOXB));
                    __syncwarp();
                    if (lane < nbox) {
                        const int reg = lane % C::NREG, b = lane / C::NREG;
                        const bool second = pair && b >= nb;
                        const int k = second ? b - nb : b;
                        const int rb = second ? C::RT / 16 + k : k;
                        tma_load_2d_hint(stage + (uint32_t)(reg * C::REGION + rb * 8 * C::BOXB),
                                         second ? &wmap2 : &wmap, kt * C::NREG * C::BOXW + reg * C::BOXW,
                                         (int)(row0 + 8 * k), fb, wpol);
                    }
                } else {
                // lane i streams stage row i's segment (RT <= 32 rows per tile;
                // a pair's second matrix from stage row TR on)
                const bool second = pair && lane >= TR;
                const int ri = second ? lane - TR : lane;
                const bool row_ok = ri < nrows && (pair || lane < TR);
                uintptr_t src = 0, lo = 0, hi = 0;
                uint32_t bytes = 0;
                if (row_ok) {
                    src = (second ? w2base : wbase) + (uintptr_t)((row0 + ri) * a.row_bytes) +
                          (uintptr_t)kt * 32u * C::GB;
                    lo = src & ~(uintptr_t)15;
                    hi = (src + seg + 15) & ~(uintptr_t)15;
                    const uintptr_t end16 = second ? w2end16 : wend16;
                    if (hi > end16) hi = end16;  // never read past the array
                    bytes = hi > lo ? (uint32_t)(hi - lo) : 0u;
                }
                uint32_t tx = bytes;
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) tx += __shfl_xor_sync(0xffffffffu, tx, off);
                if (lane == 0) mbar_expect_tx(fb, tx);
                __syncwarp();
                if (bytes)
                    bulk_g2s_hint(stage + (uint32_t)lane * C::SLOT, reinterpret_cast<const void*>(lo), bytes, fb, wpol);
                if (row_ok) {
                    // bytes past the array's last 16-B boundary: plain copy
                    for (uintptr_t q = (bytes ? hi : lo); q < src + seg; ++q)
                        sts_u8(stage + (uint32_t)lane * C::SLOT + (uint32_t)(q - lo),
                               *reinterpret_cast<const uint8_t*>(q));
                }
                }
                mbar_arrive(fb);
                __syncwarp();
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        if (dyn) {
            // end marker for the consumers: a stage with no bytes and row -1
            if (!mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u)) {
                report_error(a.err, 2);
                abort_flag = 1;
            }
            if (*(volatile int*)&abort_flag) goto producer_drain;
            if (lane == 0) stage_row[s] = -1;
            __syncwarp();
            mbar_arrive(smem_u32(&full_bar[s]));
            if (lane == 0) release_tile_queue(a.tiles);
        }
        return;
    producer_drain:
        // Abort: the stages already issued may still have copies in flight;
        // wait (bounded) for each of them before the CTA's smem goes away.
        for (uint32_t k = (seq >= (uint32_t)S ? seq - (uint32_t)S : 0); k < seq; ++k) {
            const int ks = (int)(k % (uint32_t)S);
            if (!mbar_wait(smem_u32(&full_bar[ks]), (k / (uint32_t)S) & 1u)) {
                report_error(a.err, 3);
                break;
            }
        }
        // an aborting CTA is done with the queue too: it still counts, so the
        // launch's last CTA resets the slot for the next launch that takes it
        if (dyn && lane == 0) release_tile_queue(a.tiles);
        return;
    }

    if (INT && xres) {
        // ------------------- x tiles, built once by warps 1..9 -------------------
        // Resident integer mode: the consumers and the x loader split the
        // pieces of every K-tile between them, then meet on xready_bar.
        // x may be the previous kernel's output: wait for it (weights are
        // read-only, so warp 0 started streaming them without waiting).
        // Staged: one lane copies all of x to shared memory with one bulk
        // copy (one memory round trip) and the warps build the tiles from
        // there; otherwise every warp loads its pieces from global memory.
        const uint32_t xst = x_base + (uint32_t)a.ktiles * C::XT_BYTES;
        bool staged_ok = true;
        if (a.x_staged) {
            if (warp == kXWarp && lane == 0) {
                dep_wait();
                mbar_arrive_expect_tx(smem_u32(&xstage_bar), (uint32_t)a.x_staged);
                bulk_g2s(xst, a.x, (uint32_t)a.x_staged, smem_u32(&xstage_bar));
            }
            if (!mbar_wait(smem_u32(&xstage_bar), 0u)) {
                report_error(a.err, 8);
                abort_flag = 1;
                staged_ok = false;
            }
        } else {
            dep_wait();
        }
        constexpr int NQ = 2 * C::G;
        const int items = staged_ok ? a.ktiles * NQ : 0;
        for (int it = warp - 1; it < items; it += 2 * (kConsumerWarps + 1)) {
            // two pieces in flight per warp
            const int it2 = it + kConsumerWarps + 1;
            float v0[16], v1[16];
            if (a.x_staged) {
                int_piece_load_smem(xst, a.in, (long long)(it / NQ) * C::KTE, it % NQ, lane, v0);
                if (it2 < items) int_piece_load_smem(xst, a.in, (long long)(it2 / NQ) * C::KTE, it2 % NQ, lane, v1);
            } else {
                int_piece_load<C::G>(a.x, a.in, (long long)(it / NQ) * C::KTE, it % NQ, lane, v0);
                if (it2 < items) int_piece_load<C::G>(a.x, a.in, (long long)(it2 / NQ) * C::KTE, it2 % NQ, lane, v1);
            }
            const uint32_t xs0 = x_base + (uint32_t)(it / NQ) * C::XT_BYTES;
            int_piece_store<C::G>(v0, it % NQ, lane, xs0, xs0 + C::X_BYTES);
            if (it2 < items) {
                const uint32_t xs1 = x_base + (uint32_t)(it2 / NQ) * C::XT_BYTES;
                int_piece_store<C::G>(v1, it2 % NQ, lane, xs1, xs1 + C::X_BYTES);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&xready_bar));
        if (warp == kXWarp) return;
    }

    if (warp >= kXWarp) {
        // ------------------------------ x loader ------------------------------
        // Per K-tile: x for MT tokens with coalesced 128-bit loads (all in
        // flight together), per-block sums by shuffles, stored in the order
        // the consumers read.  Resident mode (every K-tile has its own slot):
        // each x tile is built once and kept for all row tiles; otherwise the
        // tiles ride the stage ring, up to S stages ahead of the consumers.
        // x may be the previous kernel's output: wait for it (weights are
        // read-only, so warp 0 started streaming them without waiting)
        dep_wait();
        const int nt = xres ? min(ntiles, 1) : ntiles;
        int s = 0;
        uint32_t ph = 0;
        for (int t = 0; t < nt; ++t) {
            for (int kt = 0; kt < a.ktiles; ++kt) {
                const int slot = xres ? kt : s;
                if (!xres && !mbar_wait(smem_u32(&xempty_bar[s]), ph ^ 1u)) {
                    report_error(a.err, 6);
                    abort_flag = 1;
                }
                if (*(volatile int*)&abort_flag) return;
                const uint32_t xs = x_base + (uint32_t)slot * C::XT_BYTES;
                const uint32_t ss = xs + C::X_BYTES;
                const long long k0 = (long long)kt * C::KTE;
                if constexpr (INT) {
                    // lane takes 16-value pieces 32 i + lane (all loads in flight first)
                    constexpr int NQ = 2 * C::G;
                    float v[NQ][16];
#pragma unroll
                    for (int i = 0; i < NQ; ++i) int_piece_load<C::G>(a.x, a.in, k0, i, lane, v[i]);
#pragma unroll
                    for (int i = 0; i < NQ; ++i) int_piece_store<C::G>(v[i], i, lane, xs, ss);
                } else {
                    constexpr int NV = C::KTE / 128;  // float4 loads per lane per token
#pragma unroll 1
                    for (int m = warp - kXWarp; m < MT; m += xw_for(MT)) {
                        const float* xr = a.x + (long long)m * a.in;
                        float4 v[NV];
#pragma unroll
                        for (int i = 0; i < NV; ++i) {
                            const int e4 = (i * 32 + lane) * 4;
                            v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
                            if (m < a.M && k0 + e4 < a.in) v[i] = ldg_nc_f4(xr + k0 + e4);
                        }
#pragma unroll
                        for (int i = 0; i < NV; ++i) {
                            const int e4 = (i * 32 + lane) * 4;
                            float sum = (v[i].x + v[i].y) + (v[i].z + v[i].w);
                            sum += __shfl_xor_sync(0xffffffffu, sum, 1);
                            sum += __shfl_xor_sync(0xffffffffu, sum, 2);
                            sum += __shfl_xor_sync(0xffffffffu, sum, 4);
                            const int blk = e4 >> 5;
                            const int g = blk / C::G;
                            const int bg = blk % C::G;
                            const int p = part_of<F>(e4 & 31);
                            sts_f4(xs + (uint32_t)(((m * C::G * 8 + bg * 8 + p) * 32 + (g ^ p)) * 16), v[i]);
                            if ((lane & 7) == 0) sts_f32(ss + (uint32_t)((m * 32 * C::G + blk) * 4), sum);
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&xfull_bar[slot]));
                if (!xres && ++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        return;
    }

    // -------------------------------- consumers --------------------------------
    // y (and the peers' y) may still be read by the previous kernel
    dep_wait();
    if (a.pdl_mode == kPdlFirst) launch_dependents();
    // Bias of the first tile's row that this thread stores (one-token stores:
    // the reduce-scatter's row of this lane; tile stores: row c % TR of
    // thread c), loaded after the wait above, so a bias written by the
    // previous kernel in the stream is seen complete.  Later tiles load
    // theirs when they start.
    float bias_first = 0.f;
    if (has_bias && !dyn) {
        const int i = (MT == 1 && a.ny == 1) ? (warp - 1) + (lane >> (5 - log2_of(RPW))) * kConsumerWarps
                                             : (int)(threadIdx.x - 32) % TR;
        if (i < min(TR, nrows_cta)) bias_first = __ldg(a.bias + a.row_offset + r_begin + i);
    }
    if (INT && xres && !mbar_wait(smem_u32(&xready_bar), 0u)) {
        report_error(a.err, 7);
        abort_flag = 1;
    }
    const int wc = warp - 1;
    // FP mode: byte offset of this lane's float4 in x-tile part row p: (lane ^ p) * 16
    // INT mode: this lane's column in quad q's rows
    uint32_t xoff[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) xoff[p] = INT ? xcol<C::G>(lane, p & (2 * C::G - 1)) : (uint32_t)((lane ^ p) * 16);
    // The consumer loop; returns the tiles this warp processed, or -1 when it
    // gave up (a bounded wait ran out here or in another warp of the CTA).
    auto consume = [&]() -> int {
    int s = 0;
    uint32_t ph = 0;
    int t = 0;  // after the loop: the tiles this CTA processed
    for (; dyn || t < ntiles; ++t) {
        long long row0;
        if (dyn) {
            // the tile's first stage names its rows
            if (!mbar_wait(smem_u32(&full_bar[s]), ph)) {
                report_error(a.err, 1);
                abort_flag = 1;
            }
            if (*(volatile int*)&abort_flag) return -1;
            const int r0 = *(volatile int*)&stage_row[s];
            if (r0 < 0) break;
            row0 = r0;
        } else {
            row0 = r_begin + (long long)t * TR;
        }
        const int nrows = (int)min((long long)TR, (dyn ? (long long)a.out : r_end) - row0);
        // bias of the row this thread stores (the first tile's was loaded at
        // the start; a later tile's is loaded here, ahead of its K loop)
        float bias_v = bias_first;
        if (has_bias) {
            if (dyn || t > 0) {
                const int i = (MT == 1 && a.ny == 1) ? wc + (lane >> (5 - log2_of(RPW))) * kConsumerWarps
                                                     : (int)(threadIdx.x - 32) % TR;
                bias_v = i < nrows ? __ldg(a.bias + a.row_offset + row0 + i) : 0.f;
            }
        }
        float tot[RPW][MT];
#pragma unroll
        for (int r = 0; r < RPW; ++r)
#pragma unroll
            for (int m = 0; m < MT; ++m) tot[r][m] = 0.f;
        // shared-memory offset of this lane's group in each of its rows' slots:
        // a row segment's misalignment (its address mod 16) is the same for
        // every K-tile, because a K-tile spans 32 groups = a multiple of 16 B
        uint32_t soff[RPW];
        bool row_on[RPW];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int i = wc + r * kConsumerWarps;  // stage row
            const bool second = pair && i >= TR;
            const int ri = second ? i - TR : i;     // row within the tile
            row_on[r] = ri < nrows;
            if (a.tma2d) {
                constexpr int LPR = 32 / C::NREG;  // lanes per region
                soff[r] = (uint32_t)((lane / LPR) * C::REGION + i * C::BOXB + (lane % LPR) * C::GB);
            } else {
                const uintptr_t rowaddr = (second ? w2base : wbase) + (uintptr_t)((row0 + ri) * a.row_bytes);
                soff[r] = (uint32_t)i * C::SLOT + (uint32_t)(rowaddr & 15) + (uint32_t)lane * C::GB;
            }
        }

        for (int kt = 0; kt < a.ktiles; ++kt) {
            if (!(dyn && kt == 0) && !mbar_wait(smem_u32(&full_bar[s]), ph)) {
                report_error(a.err, 1);
                abort_flag = 1;
            }
            if (*(volatile int*)&abort_flag) return -1;
            const uint32_t stage = smem_base + (uint32_t)s * C::W_BYTES;
            const int xslot = xres ? kt : s;
            const uint32_t xs = x_base + (uint32_t)xslot * C::XT_BYTES;
            const uint32_t ss = xs + C::X_BYTES + (uint32_t)lane * C::G * (INT ? 8 : 4);
            const bool lane_on = lane < a.gpr - kt * 32;

            uint32_t wv[RPW][C::WPG];
#pragma unroll
            for (int r = 0; r < RPW; ++r) {
                // 2-D boxes need no guard: bytes past a row's end arrive as
                // zeros (tensor-map bounds), and rows past the tile hold stale
                // but finite-or-not data that only feeds that row's discarded
                // sum (rows never mix in the reduction)
                if (a.tma2d || (row_on[r] && lane_on)) {
#pragma unroll
                    for (int j = 0; j < C::WPG; ++j) wv[r][j] = lds_u32(stage + soff[r] + 4 * j);
                } else {
#pragma unroll
                    for (int j = 0; j < C::WPG; ++j) wv[r][j] = 0u;
                }
            }

            // weights are in registers now: hand the stage's weight region back
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
            if (!(INT && xres) && !mbar_wait(smem_u32(&xfull_bar[xslot]), xres ? 0u : ph)) {
                report_error(a.err, 1);
                abort_flag = 1;
            }
            if (*(volatile int*)&abort_flag) return -1;

            if constexpr (INT) {
                int_ktile<F, RPW>(wv, xs, ss, xoff, tot);
            } else {
#pragma unroll
            for (int bg = 0; bg < C::G; ++bg) {
                // two packed partial-sum pairs per (row, token): even / odd parts (FFMA2)
                float2 acc0[RPW][MT], acc1[RPW][MT];
#pragma unroll
                for (int r = 0; r < RPW; ++r)
#pragma unroll
                    for (int m = 0; m < MT; ++m) acc0[r][m] = acc1[r][m] = make_float2(0.f, 0.f);

#pragma unroll
                for (int p = 0; p < 8; ++p) {
                    float4 xv[MT];
                    const int row = bg * 8 + p;
#pragma unroll
                    for (int m = 0; m < MT; ++m)
                        xv[m] = lds_f4(xs + (uint32_t)((m * C::G * 8 + row) * 512) + xoff[p]);
#pragma unroll
                    for (int r = 0; r < RPW; ++r) {
                        float f[4];
                        if constexpr (F == kQ8_0) {
                            q8_to_f(qs_word<F>(wv[r], bg, p), f);
                        } else {
                            q4_to_f(q4_nibbles(qs_word<F>(wv[r], bg, p >> 1), p & 1), f);
                        }
#pragma unroll
                        for (int m = 0; m < MT; ++m) {
                            float2& acc = (p & 1) ? acc1[r][m] : acc0[r][m];
                            acc = __ffma2_rn(make_float2(f[0], f[1]), make_float2(xv[m].x, xv[m].y), acc);
                            acc = __ffma2_rn(make_float2(f[2], f[3]), make_float2(xv[m].z, xv[m].w), acc);
                        }
                    }
                }
                // fold the block back: scale, offset constant, q4_1 minimum
                float sx[MT];
#pragma unroll
                for (int m = 0; m < MT; ++m)
                    sx[m] = __uint_as_float(lds_u32(ss + (uint32_t)((m * 32 * C::G + bg) * 4)));
#pragma unroll
                for (int r = 0; r < RPW; ++r) {
                    const float d = half_bits_to_float(d_bits<F>(wv[r], bg));
#pragma unroll
                    for (int m = 0; m < MT; ++m) {
                        const float blk = (acc0[r][m].x + acc0[r][m].y) + (acc1[r][m].x + acc1[r][m].y);
                        // blk = sum (128 + q) x  =>  sum q x = blk - 128 S
                        if constexpr (F == kQ8_0) {
                            tot[r][m] = fmaf(d, blk, tot[r][m]);
                        } else if constexpr (F == kQ4_0) {  // sum (q-8) x = blk - 136 S
                            tot[r][m] = fmaf(d, fmaf(-136.0f, sx[m], blk), tot[r][m]);
                        } else {                            // sum (d q + m) x
                            const float mn = half_bits_to_float(wv[r][0] >> 16);
                            tot[r][m] = fmaf(d, fmaf(-128.0f, sx[m], blk), tot[r][m]);
                            tot[r][m] = fmaf(mn, sx[m], tot[r][m]);
                        }
                    }
                }
            }
            }
            if (!xres) {
                __syncwarp();
                if (lane == 0) mbar_arrive(smem_u32(&xempty_bar[s]));
            }
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }

        if (MT == 1 && a.ny == 1) {
            // One token, one destination: reduce-scatter the RPW row sums
            // across the lanes (RPW-1 + 5 - log2 RPW shuffles instead of 5 RPW)
            // and let the lane that ends up with row r's total store it.
            float v = reduce_rows<RPW>(tot, lane);
            const int r = lane >> (5 - log2_of(RPW));  // row held by this lane
            const int i = wc + r * kConsumerWarps;
            const bool lead = (lane & (31 >> log2_of(RPW))) == 0;
            if constexpr (pair) {
                // the second matrix's row i sits in stage row TR + i, whose
                // total the reduce-scatter leaves 16 lanes further on
                const float u = __shfl_xor_sync(0xffffffffu, v, 16);
                if (lead && i < TR && i < nrows) a.ys[0][a.row_offset + row0 + i] = silu_mul(v, u);
            } else if (lead && i < nrows) {
                const long long o = a.row_offset + row0 + i;
                if (has_bias) v = __fadd_rn(v, bias_v);
                a.ys[0][o] = v;
            }
            continue;
        }
        // reduce the 32 lane partials of every (row, token) into the tile's
        // result buffer, then store it with coalesced writes: RT consecutive
        // floats per token, to this GPU's y and, in a sharded call, to every
        // peer's y over NVLink.
        float* res = tile_res[t & 1];
#pragma unroll
        for (int r = 0; r < RPW; ++r) {
            const int i = wc + r * kConsumerWarps;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
                float v = tot[r][m];
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                v += __shfl_xor_sync(0xffffffffu, v, 8);
                v += __shfl_xor_sync(0xffffffffu, v, 4);
                v += __shfl_xor_sync(0xffffffffu, v, 2);
                v += __shfl_xor_sync(0xffffffffu, v, 1);
                if (lane == ((r * MT + m) & 31)) res[m * C::RT + i] = v;
            }
        }
        // all 8 consumer warps rendezvous (bounded: an mbarrier, not bar.sync,
        // so a warp that left on an abort cannot hang the others)
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&tile_bar));
        if (!mbar_wait(smem_u32(&tile_bar), (uint32_t)t & 1u)) {
            report_error(a.err, 5);
            abort_flag = 1;
            return -1;
        }
        {
            const int c = threadIdx.x - 32;  // 0 .. 255
            const int m = c / TR, i = c % TR;
            if (m < a.M && i < nrows) {
                float v = res[m * C::RT + i];
                if constexpr (pair) {
                    v = silu_mul(v, res[m * C::RT + TR + i]);
                } else if (has_bias) {
                    v = __fadd_rn(v, bias_v);
                }
                const long long off = (long long)m * a.y_stride + a.row_offset + row0 + i;
                for (int d = 0; d < a.ny; ++d) a.ys[d][off] = v;
            }
        }
    }
    return t;
    };
    const int done_tiles = consume();

    if (a.world > 1) {
        // Sharded call: this CTA's rows are in every rank's y.  The last CTA
        // of this rank to finish publishes the epoch to every peer, then
        // waits (bounded) until every rank's slice has landed here.  Every
        // CTA counts itself exactly once, also after giving up (then with
        // kDonePoison), so the counter is back at zero for the next call and
        // a launch with a failed CTA never publishes its epoch: the peers'
        // waits then run out and report code 4 instead of reading a y with
        // missing rows.
        bool ok = done_tiles >= 0;
        if (ok) {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&tile_bar));
        }
        if (threadIdx.x == 32) {
            if (ok && !mbar_wait(smem_u32(&tile_bar), (uint32_t)done_tiles & 1u)) {
                report_error(a.err, 5);
                ok = false;
            }
            if (*(volatile int*)&abort_flag) ok = false;
            // Ordering without system-wide fences per CTA: this CTA's y stores
            // (local and peer) happen before this point (tile_bar, CTA scope);
            // the GPU-scope acquire-release count carries them to the last CTA,
            // whose one system-scope release fence then publishes every CTA's
            // stores ahead of the epoch flags (the fence is cumulative).
            const unsigned int prev = atom_add_acq_rel_gpu(a.done_counter, ok ? 1u : 1u + kDonePoison);
            if ((prev & (kDonePoison - 1u)) == gridDim.x - 1) {
                *a.done_counter = 0u;  // every CTA of this launch has counted
                if (ok && prev < kDonePoison) {
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

// ---------------------------------------------------------------------------
// A run of independent one-row products in one launch.
//
// Launched one by one, each product of a decode step pays a launch's
// start-up: a CTA's first weights land ~2.5 us after it starts, its x tiles
// are built meanwhile, and the next launch's CTAs find the SMs' shared
// memory taken until the last CTA of the previous one leaves.  A run instead:
//  * gemv_run_xprep_kernel slices every op's x once (integer mode, in the
//    x-tile layout the consumers read) into a workspace that stays in L2;
//  * gemv_run_kernel (persistent, two CTAs per SM) takes row tiles of all
//    ops from one queue -- ops with the most K-tiles first, so the long
//    tiles start early -- and each stage brings its weights (2-D tensor map)
//    and, into a ring of x slots, the stage's x tile (one bulk copy).  Its
//    producer streams the first stages' weights before the grid dependency
//    (weights are read-only) and copies x tiles only after it.
// The decode per K-tile is the streaming kernel's integer mode (int_ktile).
// ---------------------------------------------------------------------------
constexpr int kRunThreads = 32 * (1 + kConsumerWarps);

struct RunOpDev {
    float* ys[kMaxWorld];  // row i goes to ys[d][row_offset + i], d < ny
    const float* bias;     // [out] of this op's rows, or null
    int ny, row_offset;
    int out;
    int ktiles;
    int unit0;  // this op's first row tile in the launch's queue order
    int xt0;    // this op's first x tile in the workspace
};

struct RunArgs {
    RunOpDev op[kGemvRunMaxOps];
    int nop;
    int units;               // row tiles of all ops
    const uint8_t* xtiles;   // workspace: XT_BYTES per x tile
    unsigned int* tiles;     // queue {next, done}, or null: strided static tiles
    int nstages, nxslots;
    int* err;
    // Sharded ops (done_counter not null): every CTA counts itself when its
    // stores are done; the last one publishes `epoch` (the highest of the
    // run's sharded ops) to every rank's flags, and with `wait` waits until
    // every rank has published it here (the streaming GEMV's protocol).
    int world, rank;
    uint32_t* peer_flags[kMaxWorld];
    uint32_t* local_flags;
    unsigned int* done_counter;
    uint32_t epoch;
    int wait;
};

struct RunXprepArgs {
    const float* x[kGemvRunMaxOps];
    int in[kGemvRunMaxOps];
    int xt0[kGemvRunMaxOps];
    int nop;
    uint8_t* xtiles;
};

// One CTA per x tile: warp i slices piece i of the tile (int_piece_*), then
// the CTA copies the finished tile out with 16-byte stores.
template <int F>
__global__ void __launch_bounds__(64 * Fmt<F>::kGroupBlocks)
    gemv_run_xprep_kernel(const __grid_constant__ RunXprepArgs a) {
    using C = GemvCfg<F, 1, 4, true>;  // the x-tile layout does not depend on the rows per warp
    __shared__ __align__(16) uint8_t tile[C::XT_BYTES];
    launch_dependents();    // the run kernel may start streaming weights
    grid_dependency_wait();  // x may be the previous kernel's output
    const int t = blockIdx.x;
    int o = 0;
    for (int k = 1; k < a.nop; ++k)
        if (t >= a.xt0[k]) o = k;
    const int kt = t - a.xt0[o];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    float v[16];
    int_piece_load<C::G>(a.x[o], a.in[o], (long long)kt * C::KTE, warp, lane, v);
    const uint32_t xs = smem_u32(tile);
    int_piece_store<C::G>(v, warp, lane, xs, xs + C::X_BYTES);
    __syncthreads();
    const uint4* src = reinterpret_cast<const uint4*>(tile);
    uint4* dst = reinterpret_cast<uint4*>(a.xtiles + (size_t)t * C::XT_BYTES);
    for (int k = threadIdx.x; k < C::XT_BYTES / 16; k += blockDim.x) dst[k] = src[k];
}

template <int F, int RPW>
__global__ void __launch_bounds__(kRunThreads, 2)
    gemv_run_kernel(const __grid_constant__ RunArgs a, const __grid_constant__ WMaps<kGemvRunMaxOps> wm) {
    using C = GemvCfg<F, 1, RPW, true>;
    constexpr int TR = C::RT;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ __align__(8) uint64_t full_bar[kMaxStages];   // a stage's weights landed
    __shared__ __align__(8) uint64_t empty_bar[kMaxStages];  // ... and are in the consumers' registers
    __shared__ __align__(8) uint64_t xfull_bar[kMaxStages];  // an x slot's tile landed
    __shared__ __align__(8) uint64_t xempty_bar[kMaxStages]; // ... and is consumed
    __shared__ int stage_unit[kMaxStages];                   // row tile of each stage (-1: end)
    __shared__ __align__(8) uint64_t done_bar;                // consumer warps' stores issued
    __shared__ int abort_flag;

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int S = a.nstages, NX = a.nxslots;
    if (threadIdx.x == 0) {
        for (int s = 0; s < kMaxStages; ++s) {
            mbar_init(smem_u32(&full_bar[s]), 32);
            mbar_init(smem_u32(&empty_bar[s]), kConsumerWarps);
            mbar_init(smem_u32(&xfull_bar[s]), 1);
            mbar_init(smem_u32(&xempty_bar[s]), kConsumerWarps);
        }
        mbar_init(smem_u32(&done_bar), kConsumerWarps);
        abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    launch_dependents();
    const uint32_t smem_base = (smem_u32(smem) + 127u) & ~127u;
    const uint32_t x_base = smem_base + (uint32_t)S * C::W_BYTES;
    // op of row tile u: ops are laid out in queue order by unit0
    auto op_of = [&](int u) {
        int o = 0;
        for (int k = 1; k < a.nop; ++k)
            if (u >= a.op[k].unit0) o = k;
        return o;
    };

    if (warp == 0) {
        // ------------------------------ producer ------------------------------
        const uint64_t wpol = l2_evict_first_policy();
        uint32_t seq = 0;      // stages issued
        uint32_t xissued = 0;  // x copies issued (stages [0, xissued))
        int s = 0;
        uint32_t ph = 0;
        bool dep = false;
        int pend[kMaxStages];  // (op << 16 | kt) of stages whose x copy waits for the dependency
        auto issue_x = [&](uint32_t k, int o, int kt) {
            const uint32_t xb = smem_u32(&xfull_bar[k % (uint32_t)NX]);
            mbar_arrive_expect_tx(xb, (uint32_t)C::XT_BYTES);
            bulk_g2s(x_base + (k % (uint32_t)NX) * (uint32_t)C::XT_BYTES,
                     a.xtiles + (size_t)(a.op[o].xt0 + kt) * C::XT_BYTES, (uint32_t)C::XT_BYTES, xb);
        };
        // the grid dependency, then the x copies of stages [xissued, end)
        auto flush_pending = [&](uint32_t end) {
            grid_dependency_wait();
            dep = true;
            if (lane == 0)
                for (uint32_t k = xissued; k < end; ++k) issue_x(k, pend[k] >> 16, pend[k] & 0xFFFF);
            xissued = end;
        };
        unsigned int ticket = 0;
        if (lane == 0) ticket = a.tiles ? atomicAdd(a.tiles, 1u) : blockIdx.x;
        for (int n = 1;; ++n) {
            const int u = (int)__shfl_sync(0xffffffffu, ticket, 0);
            if (u >= a.units) break;
            if (lane == 0) ticket = a.tiles ? atomicAdd(a.tiles, 1u) : blockIdx.x + (unsigned int)n * gridDim.x;
            const int o = op_of(u);
            const long long row0 = (long long)(u - a.op[o].unit0) * TR;
            const int nrows = (int)min((long long)TR, (long long)a.op[o].out - row0);
            const int nbox = (nrows + 7) / 8 * C::NREG;
            for (int kt = 0; kt < a.op[o].ktiles; ++kt, ++seq) {
                bool ok = mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u);
                if (ok)
                    ok = mbar_wait(smem_u32(&xempty_bar[seq % (uint32_t)NX]), ((seq / (uint32_t)NX) & 1u) ^ 1u);
                if (!ok) {
                    report_error(a.err, 2);
                    abort_flag = 1;
                }
                if (*(volatile int*)&abort_flag) goto producer_drain;
                const uint32_t stage = smem_base + (uint32_t)s * C::W_BYTES;
                const uint32_t fb = smem_u32(&full_bar[s]);
                if (lane == 0) {
                    stage_unit[s] = u;
                    mbar_expect_tx(fb, (uint32_t)(nbox * 8 * C::BOXB));
                }
                __syncwarp();
                if (lane < nbox) {
                    const int reg = lane % C::NREG, b = lane / C::NREG;
                    tma_load_2d_hint(stage + (uint32_t)(reg * C::REGION + b * 8 * C::BOXB), &wm.m[o],
                                     kt * C::NREG * C::BOXW + reg * C::BOXW, (int)(row0 + 8 * b), fb, wpol);
                }
                mbar_arrive(fb);
                __syncwarp();
                if (dep) {
                    if (lane == 0) issue_x(seq, o, kt);
                    xissued = seq + 1;
                } else {
                    pend[seq] = (o << 16) | kt;
                    // S stages of weights in flight: the x tiles now
                    if (seq + 1 == (uint32_t)S) flush_pending(seq + 1);
                }
                if (++s == S) {
                    s = 0;
                    ph ^= 1u;
                }
            }
        }
        if (!dep) flush_pending(seq);
        // end marker for the consumers: a stage with no bytes and row tile -1
        if (!mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u)) {
            report_error(a.err, 2);
            abort_flag = 1;
        }
        if (*(volatile int*)&abort_flag) goto producer_drain;
        if (lane == 0) stage_unit[s] = -1;
        __syncwarp();
        mbar_arrive(smem_u32(&full_bar[s]));
        if (a.tiles && lane == 0) release_tile_queue(a.tiles);
        return;
    producer_drain:
        // Abort: wait (bounded) for the copies still in flight into this CTA.
        for (uint32_t k = (seq >= (uint32_t)S ? seq - (uint32_t)S : 0); k < seq; ++k) {
            if (!mbar_wait(smem_u32(&full_bar[k % (uint32_t)S]), (k / (uint32_t)S) & 1u)) {
                report_error(a.err, 3);
                break;
            }
        }
        for (uint32_t k = (xissued >= (uint32_t)NX ? xissued - (uint32_t)NX : 0); k < xissued; ++k) {
            if (!mbar_wait(smem_u32(&xfull_bar[k % (uint32_t)NX]), (k / (uint32_t)NX) & 1u)) {
                report_error(a.err, 3);
                break;
            }
        }
        if (a.tiles && lane == 0) release_tile_queue(a.tiles);
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int wc = warp - 1;
    uint32_t xoff[8];
#pragma unroll
    for (int p = 0; p < 8; ++p) xoff[p] = xcol<C::G>(lane, p & (2 * C::G - 1));
    uint32_t soff[RPW];  // this lane's group in each of its rows' box rows
#pragma unroll
    for (int r = 0; r < RPW; ++r) {
        constexpr int LPR = 32 / C::NREG;
        soff[r] = (uint32_t)((lane / LPR) * C::REGION + (wc + r * kConsumerWarps) * C::BOXB + (lane % LPR) * C::GB);
    }
    // The consumer loop; false when it gave up (a bounded wait ran out here
    // or in another warp of the CTA).
    auto consume = [&]() -> bool {
    int s = 0;
    uint32_t ph = 0, seq = 0;
    for (;;) {
        if (!mbar_wait(smem_u32(&full_bar[s]), ph)) {
            report_error(a.err, 1);
            abort_flag = 1;
        }
        if (*(volatile int*)&abort_flag) return false;
        const int u = *(volatile int*)&stage_unit[s];
        if (u < 0) return true;
        const int o = op_of(u);
        const long long row0 = (long long)(u - a.op[o].unit0) * TR;
        const int nrows = (int)min((long long)TR, (long long)a.op[o].out - row0);
        const int kts = a.op[o].ktiles;
        float tot[RPW][1];
#pragma unroll
        for (int r = 0; r < RPW; ++r) tot[r][0] = 0.f;
        for (int kt = 0; kt < kts; ++kt, ++seq) {
            if (kt > 0 && !mbar_wait(smem_u32(&full_bar[s]), ph)) {
                report_error(a.err, 1);
                abort_flag = 1;
            }
            if (*(volatile int*)&abort_flag) return false;
            // 2-D boxes: bytes past a row's end and rows past the matrix
            // arrive as zeros (tensor-map bounds)
            const uint32_t stage = smem_base + (uint32_t)s * C::W_BYTES;
            uint32_t wv[RPW][C::WPG];
#pragma unroll
            for (int r = 0; r < RPW; ++r)
#pragma unroll
                for (int j = 0; j < C::WPG; ++j) wv[r][j] = lds_u32(stage + soff[r] + 4 * j);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&empty_bar[s]));
            const uint32_t xk = seq % (uint32_t)NX;
            if (!mbar_wait(smem_u32(&xfull_bar[xk]), (seq / (uint32_t)NX) & 1u)) {
                report_error(a.err, 1);
                abort_flag = 1;
            }
            if (*(volatile int*)&abort_flag) return false;
            const uint32_t xs = x_base + xk * (uint32_t)C::XT_BYTES;
            int_ktile<F, RPW>(wv, xs, xs + C::X_BYTES + (uint32_t)lane * C::G * 8, xoff, tot);
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&xempty_bar[xk]));
            if (++s == S) {
                s = 0;
                ph ^= 1u;
            }
        }
        // reduce-scatter the RPW row sums; the lead lane of each row stores it
        float v = reduce_rows<RPW>(tot, lane);
        const int r = lane >> (5 - log2_of(RPW));
        const int i = wc + r * kConsumerWarps;
        if ((lane & (31 >> log2_of(RPW))) == 0 && i < nrows) {
            const long long row = row0 + i;
            const float* bias = a.op[o].bias;
            if (bias) v = __fadd_rn(v, bias[row]);
            const long long off = a.op[o].row_offset + row;
            for (int d = 0; d < a.op[o].ny; ++d) a.op[o].ys[d][off] = v;
        }
    }
    };
    const bool ok = consume();

    if (a.done_counter) {
        // Sharded ops in the run: the same completion protocol as a sharded
        // streaming GEMV.  This CTA's stores (local and peer) happen before
        // done_bar (CTA scope); the GPU-scope acquire-release count carries
        // them to the last CTA, whose system-scope release fence publishes
        // every CTA's stores ahead of the epoch flags.  A CTA that gave up
        // counts with kDonePoison, and the launch then never publishes.
        if (ok) {
            __syncwarp();
            if (lane == 0) mbar_arrive(smem_u32(&done_bar));
        }
        if (threadIdx.x == 32) {
            bool good = ok;
            if (good && !mbar_wait(smem_u32(&done_bar), 0u)) {
                report_error(a.err, 5);
                good = false;
            }
            if (*(volatile int*)&abort_flag) good = false;
            const unsigned int prev = atom_add_acq_rel_gpu(a.done_counter, good ? 1u : 1u + kDonePoison);
            if ((prev & (kDonePoison - 1u)) == gridDim.x - 1) {
                *a.done_counter = 0u;  // every CTA of this launch has counted
                if (good && prev < kDonePoison) {
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

// ---------------------------------------------------------------------------
// Fallback for layouts the streaming kernel does not take (odd block count
// per row for q8_0/q4_0, weights or x not 16-B aligned, in % 4 != 0): one
// warp per output row, byte loads, any alignment.  Same arithmetic as above
// but each weight is decoded to its fp32 value w and accumulated as w * x.
// ---------------------------------------------------------------------------
template <int F>
__global__ void __launch_bounds__(256) gemv_generic_kernel(const uint8_t* __restrict__ w,
                                                           const float* __restrict__ x,
                                                           float* __restrict__ y, int out, int in,
                                                           int M, int bpr) {
    constexpr int BS = Fmt<F>::kBlockBytes;
    const int o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    const int lane = threadIdx.x & 31;
    if (o >= out) return;
    const uint8_t* wr = w + (long long)o * bpr * BS;
    for (int m0 = 0; m0 < M; m0 += 8) {
        float acc[8];
#pragma unroll
        for (int m = 0; m < 8; ++m) acc[m] = 0.f;
        for (int b = lane; b < bpr; b += 32) {
            const uint8_t* blk = wr + (long long)b * BS;
            const float d = half_bits_to_float((uint32_t)blk[0] | ((uint32_t)blk[1] << 8));
            float mn = 0.f;
            if constexpr (F == kQ4_1) mn = half_bits_to_float((uint32_t)blk[2] | ((uint32_t)blk[3] << 8));
            const int k0 = b * kQK;
            const int n = min(kQK, in - k0);
            for (int e = 0; e < n; ++e) {
                float wv;
                if constexpr (F == kQ8_0) {
                    wv = d * (float)(int8_t)blk[2 + e];
                } else if constexpr (F == kQ4_0) {
                    const int q = e < 16 ? (blk[2 + e] & 15) : (blk[2 + e - 16] >> 4);
                    wv = d * (float)(q - 8);
                } else {
                    const int q = e < 16 ? (blk[4 + e] & 15) : (blk[4 + e - 16] >> 4);
                    wv = fmaf(d, (float)q, mn);
                }
#pragma unroll
                for (int m = 0; m < 8; ++m)
                    if (m0 + m < M) acc[m] = fmaf(wv, __ldg(x + (long long)(m0 + m) * in + k0 + e), acc[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < 8; ++m) {
            float v = acc[m];
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0 && m0 + m < M) y[(long long)(m0 + m) * out + o] = v;
        }
    }
}

// This device's tile-queue ring (looked up once per device, that device current).
unsigned int* tile_slots(int dev) {
    static std::atomic<unsigned int*> ptrs[64];
    if (dev < 0 || dev >= 64) return nullptr;
    unsigned int* p = ptrs[dev].load(std::memory_order_acquire);
    if (!p) {
        void* q = nullptr;
        if (cudaGetSymbolAddress(&q, g_gemv_tile_slots) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        p = static_cast<unsigned int*>(q);
        ptrs[dev].store(p, std::memory_order_release);
    }
    return p;
}

// The ring of `stream` on device `dev`: rings are handed to streams in the
// order they first launch a queued GEMV; -1 once all kStreamRings are taken
// (that stream's launches then use static row ranges).
struct StreamRings {
    std::mutex mu;
    std::map<cudaStream_t, int> ring;
    std::atomic<unsigned int> seq[kStreamRings];
};

int stream_ring(StreamRings& sr, cudaStream_t stream) {
    std::lock_guard<std::mutex> lock(sr.mu);
    auto it = sr.ring.find(stream);
    if (it != sr.ring.end()) return it->second;
    if ((int)sr.ring.size() >= kStreamRings) return -1;
    const int r = (int)sr.ring.size();
    sr.ring.emplace(stream, r);
    return r;
}

// A queue for one launch on `stream`, or null (static row ranges) when the
// stream is being captured (a graph would replay the same slot) or has no
// ring.
unsigned int* tile_queue(int dev, cudaStream_t stream) {
    static StreamRings rings[64];
    if (dev < 0 || dev >= 64) return nullptr;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(stream, &cs) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    if (cs != cudaStreamCaptureStatusNone) return nullptr;
    unsigned int* base = tile_slots(dev);
    if (!base) return nullptr;
    const int r = stream_ring(rings[dev], stream);
    if (r < 0) return nullptr;
    const unsigned int slot = rings[dev].seq[r].fetch_add(1u, std::memory_order_relaxed) % kSlotsPerRing;
    return base + 2u * ((unsigned int)r * kSlotsPerRing + slot);
}

// MINB: CTAs per SM the kernel's registers and shared memory are sized for;
// cps: CTAs per SM actually launched (cps < MINB leaves room on every SM for
// the next kernel in the stream to start its weight stream early).
template <int F, int MT, int RPW, int MINB, bool INT, int EPI>
cudaError_t launch_stream_t(GemvArgs args, int sm_count, int smem_per_sm, cudaStream_t stream,
                            int cps = MINB) {
    using C = GemvCfg<F, MT, RPW, INT>;
    // Per-CTA budget: the SM's shared memory split MINB ways, minus the 1 KB
    // the driver reserves per CTA, this kernel's static shared memory
    // (barriers + tile results, < 2.5 KB) and the alignment slack.
    const int budget = smem_per_sm / MINB - 1024 - 2560 - 128;
    // Resident x (every K-tile's x tile kept, built once) when it fits next
    // to two weight stages; the fp32 mode also needs a barrier per K-tile.
    const long long xres_bytes = (long long)args.ktiles * C::XT_BYTES;
    // one-token resident mode over three or more K-tiles: x staged in shared
    // memory by one bulk copy (x 16-B aligned, in % 4 == 0: a 16-B multiple)
    // when it fits next to the tiles and two weight stages
    const long long stage_bytes = ((long long)args.in * 4 + 127) / 128 * 128;
    args.x_staged = 0;
    int S, nx;
    if (INT && args.ktiles >= 3 && xres_bytes + stage_bytes + 2LL * C::W_BYTES <= budget) {
        args.x_resident = 1;
        args.x_staged = args.in * 4;
        nx = args.ktiles;
        S = (int)((budget - xres_bytes - stage_bytes) / C::W_BYTES);
    } else if (xres_bytes + 2LL * C::W_BYTES <= budget && (INT || args.ktiles <= kMaxStages)) {
        args.x_resident = 1;
        nx = args.ktiles;
        S = (int)((budget - xres_bytes) / C::W_BYTES);
    } else {
        args.x_resident = 0;
        S = budget / (C::W_BYTES + C::XT_BYTES);
        nx = S;
    }
    if (S > kMaxStages) S = kMaxStages;
    if (!args.x_resident) nx = S;
    if (S < 2) return cudaErrorInvalidConfiguration;
    args.nstages = S;
    const int smem = S * C::W_BYTES + nx * C::XT_BYTES + (args.x_staged ? (int)stage_bytes : 0) +
                     128;  // + the alignment slack
    // Every launch of this instantiation uses at most budget + 128 bytes
    // (stages and x slots are sized to the budget), so the attribute is set
    // to that once per device; concurrent first calls set the same value.
    static std::atomic<bool> attr_done[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_done[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(gemv_stream_kernel<F, MT, RPW, MINB, INT, EPI>,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, budget + 128);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_done[dev].store(true, std::memory_order_release);
    }
    // weights by 2-D tensor map when the row pitch and base (both bases of a
    // pair) allow it
    constexpr bool pair = EPI == kEpiPair;
    WMaps<pair ? 2 : 1> wm;
    std::memset(&wm, 0, sizeof(wm));
    auto map_of = [&](CUtensorMap* m, const uint8_t* base) {
        return reinterpret_cast<uintptr_t>(base) % 16 == 0 &&
               make_map_2d(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, const_cast<uint8_t*>(base),
                           (uint64_t)(args.row_bytes / 8), (uint64_t)args.out, (uint64_t)args.row_bytes,
                           (uint32_t)C::BOXW, 8u, CU_TENSOR_MAP_SWIZZLE_NONE);
    };
    args.tma2d = 0;
    if (args.out > 0 && args.row_bytes % 16 == 0 && map_of(&wm.m[0], args.w) &&
        (!pair || map_of(&wm.m[pair ? 1 : 0], args.w2)))
        args.tma2d = 1;
    // output rows per row tile (a pair's tile holds that many rows of each matrix)
    constexpr int tile_rows = pair ? C::RT / 2 : C::RT;
    const long long units = (args.out + 7) / 8;  // rows are handed out 8 at a time
    const long long want = (long long)sm_count * cps;
    int grid = (int)(units < want ? units : want);
    if (grid < 1) grid = 1;  // a rank holding no rows still runs the handshake
    // Dynamic tiles only pay with many tiles per CTA: with few, whole CTAs
    // would sit idle at the end and each queue ticket's latency shows.
    args.tiles = nullptr;
    if (INT && args.x_resident &&
        (args.out + tile_rows - 1) / tile_rows >= 8LL * grid)
        args.tiles = tile_queue(dev, stream);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads_for(MT));
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_stream_kernel<F, MT, RPW, MINB, INT, EPI>, args, wm);
}

// rows-per-warp choice per format: keeps the lane-group words of all RPW
// rows in registers (q8_0: 17 words per row, so 2 rows; q4: 4 rows).
template <int F>
constexpr int rpw_for() {
    return F == kQ8_0 ? 2 : 4;
}

// One or two tokens per pass: two CTAs per SM (16 consumer warps per SM,
// registers capped at 102); more tokens: one CTA per SM with deeper stages.
// One token takes the integer (DP4A) mode: 24 four-way integer dot products
// and ~12 mask ops per block and row, against ~32 byte-permutes + 16 packed
// FMAs in the fp32 mode, whose decode cost is shared only from two tokens on.
template <int F, int MT, int EPI>
cudaError_t dispatch_mt(const GemvArgs& args, int sm_count, int smem_per_sm, cudaStream_t stream) {
    constexpr int RPW = rpw_for<F>();
    constexpr int MINB = MT <= 2 ? 2 : 1;
    if constexpr (MT == 1) {
        // fewer than one full tile per CTA at two CTAs per SM: one CTA per SM
        // (a full tile each, and the whole shared memory for weight stages)
        const long long streamed_rows = (long long)args.out * (EPI == kEpiPair ? 2 : 1);
        if (streamed_rows < 2LL * sm_count * kConsumerWarps * RPW)
            return launch_stream_t<F, 1, RPW, 1, true, EPI>(args, sm_count, smem_per_sm, stream);
        return launch_stream_t<F, 1, RPW, 2, true, EPI>(args, sm_count, smem_per_sm, stream);
    } else {
        // fp32 mode, measured per token count (q4_0 28672 x 8192): 2 tokens
        // and 8 tokens run best with two rows per warp (fewer live
        // accumulators; 8 tokens also need the four x-loader warps' registers),
        // 4 tokens with four.
        constexpr int RPW_FP = (MT == 4 || RPW < 4) ? RPW : RPW / 2;
        return launch_stream_t<F, MT, RPW_FP, MINB, false, EPI>(args, sm_count, smem_per_sm, stream);
    }
}

int ktiles_of(int fmt, int in) {
    const int bpr = (in + kQK - 1) / kQK;
    const int gpr = bpr / (fmt == kQ4_1 ? 1 : 2);
    return (gpr + 31) / 32;
}

template <int F>
cudaError_t launch_run_t(const GemvRunOp* ops, int nop, void* ws, int sm_count, int smem_per_sm, int* err,
                         cudaStream_t stream) {
    constexpr int RPW = rpw_for<F>();
    using C = GemvCfg<F, 1, RPW, true>;
    if (nop < 1 || nop > kGemvRunMaxOps) return cudaErrorInvalidValue;
    // queue order: most K-tiles first (a stable order otherwise)
    int ord[kGemvRunMaxOps];
    for (int k = 0; k < nop; ++k) ord[k] = k;
    for (int k = 1; k < nop; ++k)
        for (int j = k; j > 0 && ktiles_of(F, ops[ord[j]].in) > ktiles_of(F, ops[ord[j - 1]].in); --j) {
            const int t = ord[j];
            ord[j] = ord[j - 1];
            ord[j - 1] = t;
        }
    RunArgs ra;
    std::memset(&ra, 0, sizeof(ra));
    RunXprepArgs xa;
    std::memset(&xa, 0, sizeof(xa));
    WMaps<kGemvRunMaxOps> wm;
    std::memset(&wm, 0, sizeof(wm));
    int units = 0, xt = 0;
    const GemvRunOp* sharded = nullptr;  // the run's first sharded op
    for (int k = 0; k < nop; ++k) {
        const GemvRunOp& op = ops[ord[k]];
        const long long row_bytes = (long long)((op.in + kQK - 1) / kQK) * Fmt<F>::kBlockBytes;
        if (op.out > 0 &&
            !make_map_2d(&wm.m[k], CU_TENSOR_MAP_DATA_TYPE_UINT64, const_cast<uint8_t*>(op.w),
                         (uint64_t)(row_bytes / 8), (uint64_t)op.out, (uint64_t)row_bytes, (uint32_t)C::BOXW, 8u,
                         CU_TENSOR_MAP_SWIZZLE_NONE))
            return cudaErrorInvalidValue;
        const int kts = ktiles_of(F, op.in);
        RunOpDev& d = ra.op[k];
        for (int r = 0; r < op.ny; ++r) d.ys[r] = op.y[r];
        d.bias = op.bias;
        d.ny = op.ny;
        d.row_offset = op.row_offset;
        d.out = op.out;
        d.ktiles = kts;
        d.unit0 = units;
        d.xt0 = xt;
        if (op.world > 1) {
            if (sharded && !gemv_run_compatible(*sharded, op)) return cudaErrorInvalidValue;
            if (!sharded) {
                sharded = &op;
                ra.epoch = op.epoch;
            }
            if ((int)(op.epoch - ra.epoch) > 0) ra.epoch = op.epoch;
            ra.wait |= op.wait;
        }
        xa.x[k] = op.x;
        xa.in[k] = op.in;
        xa.xt0[k] = xt;
        units += (op.out + C::RT - 1) / C::RT;
        xt += kts;
    }
    if (sharded) {
        ra.world = sharded->world;
        ra.rank = sharded->rank;
        for (int r = 0; r < sharded->world; ++r) ra.peer_flags[r] = sharded->flags[r];
        ra.local_flags = sharded->flags[sharded->rank];
        ra.done_counter = sharded->done_counter;
    }
    ra.nop = xa.nop = nop;
    ra.units = units;
    ra.xtiles = static_cast<const uint8_t*>(ws);
    xa.xtiles = static_cast<uint8_t*>(ws);
    ra.err = err;
    // Two CTAs per SM: S weight stages and NX >= S x slots per CTA (an x
    // slot is held from its copy until the stage is consumed; the first S
    // stages' x copies wait for the grid dependency, so S slots must be free
    // then).
    const int budget = smem_per_sm / 2 - 1024 - 1024 - 128;
    int S = budget / (C::W_BYTES + C::XT_BYTES);
    if (S > kMaxStages) S = kMaxStages;
    if (S < 2) return cudaErrorInvalidConfiguration;
    int NX = (budget - S * C::W_BYTES) / C::XT_BYTES;
    if (NX > kMaxStages) NX = kMaxStages;
    if (NX < S) return cudaErrorInvalidConfiguration;
    ra.nstages = S;
    ra.nxslots = NX;
    const int smem = S * C::W_BYTES + NX * C::XT_BYTES + 128;
    static std::atomic<bool> attr_done[64];
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 64 || !attr_done[dev].load(std::memory_order_acquire)) {
        cudaError_t e = cudaFuncSetAttribute(gemv_run_kernel<F, RPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             budget + 128);
        if (e != cudaSuccess) return e;
        if (dev < 64) attr_done[dev].store(true, std::memory_order_release);
    }
    int grid = 2 * sm_count;
    if (grid > units) grid = units;
    if (grid < 1) grid = 1;  // a rank holding no rows still runs the handshake
    ra.tiles = tile_queue(dev, stream);  // null while capturing: strided static tiles

    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cx = {};
    cx.gridDim = dim3(xt);
    cx.blockDim = dim3(64 * C::G);
    cx.stream = stream;
    cx.attrs = attr;
    cx.numAttrs = 1;
    cudaError_t e = cudaLaunchKernelEx(&cx, gemv_run_xprep_kernel<F>, xa);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(kRunThreads);
    cfg.dynamicSmemBytes = (size_t)smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, gemv_run_kernel<F, RPW>, ra, wm);
}

}  // namespace

bool gemv_run_ok(int fmt, const GemvRunOp& op) {
    if (fmt != kQ8_0 && fmt != kQ4_0 && fmt != kQ4_1) return false;
    if (op.out < 0 || (op.out == 0 && op.world <= 1) || op.in < 1 || (op.out > 0 && !op.w) || !op.x) return false;
    if (op.ny < 1 || op.ny > kMaxWorld || (op.world > 1 && (op.ny != op.world || !op.done_counter))) return false;
    for (int d = 0; d < op.ny; ++d)
        if (!op.y[d]) return false;
    const int bpr = (op.in + kQK - 1) / kQK;
    const long long row_bytes = (long long)bpr * block_bytes(fmt);
    return reinterpret_cast<uintptr_t>(op.w) % 16 == 0 && reinterpret_cast<uintptr_t>(op.x) % 16 == 0 &&
           row_bytes % 16 == 0 && bpr % (fmt == kQ4_1 ? 1 : 2) == 0 && op.in % 4 == 0 && encode_fn() != nullptr;
}

bool gemv_run_compatible(const GemvRunOp& a, const GemvRunOp& b) {
    if (a.world <= 1 || b.world <= 1) return true;
    if (a.world != b.world || a.rank != b.rank || a.done_counter != b.done_counter) return false;
    for (int r = 0; r < a.world; ++r)
        if (a.flags[r] != b.flags[r]) return false;
    return true;
}

size_t gemv_run_workspace_bytes(int fmt, const GemvRunOp* ops, int nop) {
    size_t tiles = 0;
    for (int k = 0; k < nop; ++k) tiles += (size_t)ktiles_of(fmt, ops[k].in);
    const size_t xt = fmt == kQ4_1 ? GemvCfg<kQ4_1, 1, 4, true>::XT_BYTES : GemvCfg<kQ4_0, 1, 4, true>::XT_BYTES;
    return tiles * xt;
}

cudaError_t launch_gemv_run(int fmt, const GemvRunOp* ops, int nop, void* ws, int sm_count, int smem_per_sm,
                            int* err, cudaStream_t stream) {
    switch (fmt) {
        case kQ8_0: return launch_run_t<kQ8_0>(ops, nop, ws, sm_count, smem_per_sm, err, stream);
        case kQ4_0: return launch_run_t<kQ4_0>(ops, nop, ws, sm_count, smem_per_sm, err, stream);
        case kQ4_1: return launch_run_t<kQ4_1>(ops, nop, ws, sm_count, smem_per_sm, err, stream);
    }
    return cudaErrorInvalidValue;
}

int gemv_tokens_per_pass(int rows_left) {
    return rows_left >= 5 ? 8 : (rows_left >= 3 ? 4 : (rows_left == 2 ? 2 : 1));
}

cudaError_t launch_gemv_stream(int fmt, const GemvArgs& args, int mt, int sm_count, int smem_per_sm,
                               cudaStream_t stream) {
    const int epi = args.w2 ? kEpiPair : kEpiPlain;
#define MLQ_STREAM_MT(F, E)                                                            \
    switch (mt) {                                                                      \
        case 1: return dispatch_mt<F, 1, E>(args, sm_count, smem_per_sm, stream);      \
        case 2: return dispatch_mt<F, 2, E>(args, sm_count, smem_per_sm, stream);      \
        case 4: return dispatch_mt<F, 4, E>(args, sm_count, smem_per_sm, stream);      \
        default: return dispatch_mt<F, 8, E>(args, sm_count, smem_per_sm, stream);     \
    }
#define MLQ_STREAM(F)                                                                  \
    if (epi == kEpiPair) MLQ_STREAM_MT(F, kEpiPair)                                    \
    MLQ_STREAM_MT(F, kEpiPlain)
    switch (fmt) {
        case kQ8_0: MLQ_STREAM(kQ8_0)
        case kQ4_0: MLQ_STREAM(kQ4_0)
        case kQ4_1: MLQ_STREAM(kQ4_1)
    }
#undef MLQ_STREAM
#undef MLQ_STREAM_MT
    return cudaErrorInvalidValue;
}

cudaError_t launch_gemv_generic(int fmt, const uint8_t* w, const float* x, float* y, int out,
                                int in, int M, int bpr, cudaStream_t stream) {
    const dim3 block(256);
    const dim3 grid((out + 7) / 8);
    switch (fmt) {
        case kQ8_0: gemv_generic_kernel<kQ8_0><<<grid, block, 0, stream>>>(w, x, y, out, in, M, bpr); break;
        case kQ4_0: gemv_generic_kernel<kQ4_0><<<grid, block, 0, stream>>>(w, x, y, out, in, M, bpr); break;
        case kQ4_1: gemv_generic_kernel<kQ4_1><<<grid, block, 0, stream>>>(w, x, y, out, in, M, bpr); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// Puts every tile-queue pair of the current device back to zero (after a
// kernel gave up mid-launch; the caller has synchronised the device).
cudaError_t reset_tile_queues() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    unsigned int* base = tile_slots(dev);
    if (!base) return cudaErrorInvalidSymbol;
    return cudaMemset(base, 0, sizeof(unsigned int) * 2 * kTileSlots);
}

}  // namespace mlq

namespace mlq {
namespace {

// The deferred half of a sharded call's handshake (one thread): every
// rank's epoch word here at least `epoch`, bounded as the in-kernel wait.
__global__ void gather_wait_kernel(const uint32_t* flags, int world, uint32_t epoch, int* err) {
    // the next kernel (a GEMV, batched-decode or run launch of the next
    // step) may start streaming its weights; it reads x and writes y only
    // after this kernel has completed (griddepcontrol.wait)
    launch_dependents();
    if (threadIdx.x != 0) return;
    const uint64_t t0 = global_ns();
    for (int r = 0; r < world; ++r) {
        while ((int)(ld_acquire_sys(flags + r) - epoch) < 0) {
            if (global_ns() - t0 > kWaitLimitNs) {
                report_error(err, 4);
                return;
            }
            __nanosleep(64);
        }
    }
}

}  // namespace

cudaError_t launch_gather_wait(const uint32_t* local_flags, int world, uint32_t epoch, int* err,
                               cudaStream_t stream) {
    gather_wait_kernel<<<1, 32, 0, stream>>>(local_flags, world, epoch, err);
    return cudaGetLastError();
}

}  // namespace mlq

namespace mlq {
namespace {
__global__ void join_kernel() {}
}  // namespace

cudaError_t launch_join(cudaStream_t stream) {
    join_kernel<<<1, 32, 0, stream>>>();
    return cudaGetLastError();
}
}  // namespace mlq
