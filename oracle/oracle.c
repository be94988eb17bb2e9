/*
 * oracle.c -- CPU restatement of the reference's quantized-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (the mlq library, its
 * Python/C++ host layers) links, loads or calls this file.  Only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * legs use it, as the checker and as the timed CPU baseline.
 *
 * Every function restates one piece of the reference (Haobin-Lee/mini-llama)
 * and cites the file:line it follows.  The restatement is pinned against the
 * reference itself (oracle/_ref, built from the reference's own sources by
 * oracle/Makefile) and against the golden vectors in tests/golden/.
 *
 * Block byte layouts (include/mini_llama/quantized_tensor.h:36-72):
 *   q8_0: { u16 d; i8  qs[32]; }          34 bytes
 *   q4_0: { u16 d; u8  qs[16]; }          18 bytes, element j -> low nibble
 *                                          of qs[j], element 16+j -> high
 *   q4_1: { u16 d; u16 m; u8 qs[16]; }    20 bytes, same nibble order
 * Rows are stored one after another, each row = ceil(cols/32) blocks.
 *
 * Compile with -ffp-contract=off: the reference's scalar build (no -mfma)
 * rounds every multiply and add separately, and so must this file.
 */
#include <math.h>
#include <pthread.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORC_QK 32

enum { ORC_Q4_0 = 2, ORC_Q4_1 = 3, ORC_Q8_0 = 8 }; /* GGUF type ids,
                                                      include/mini_llama/gguf.h:16-22 */

int orc_block_bytes(int fmt) {
    switch (fmt) {
        case ORC_Q8_0: return 34;
        case ORC_Q4_0: return 18;
        case ORC_Q4_1: return 20;
        default: return 0;
    }
}

/* ---------------------------------------------------------------------------
 * fp16 codec.  Encoding follows src/quant.cc:32-70: truncate the mantissa to
 * 10 bits and add one unit when bit 12 of the fp32 mantissa is set (round
 * half up in magnitude, not round-to-nearest-even); subnormal results use the
 * same rule after the shift; exponent overflow and NaN give +-Inf.
 * Decoding follows src/quant.cc:72-101 and is exact.
 * ------------------------------------------------------------------------- */
static uint32_t f2u(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }
static float u2f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

uint16_t orc_fp16_from_f32(float value) {
    uint32_t bits = f2u(value);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int32_t e = (int32_t)((bits >> 23) & 0xffu) - 112; /* rebias 127 -> 15 */
    uint32_t man = bits & 0x7fffffu;
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        uint32_t sh = (man | 0x800000u) >> (1 - e);
        if (sh & 0x1000u) sh += 0x2000u;
        return (uint16_t)(sign | (sh >> 13));
    }
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (man & 0x1000u) {
        man += 0x2000u;
        if (man & 0x800000u) {
            man = 0;
            e += 1;
            if (e >= 31) return (uint16_t)(sign | 0x7c00u);
        }
    }
    return (uint16_t)(sign | ((uint32_t)e << 10) | (man >> 13));
}

float orc_f32_from_fp16(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    if (e == 0) {
        if (man == 0) return u2f(sign);
        /* subnormal: value = man * 2^-24, exactly representable in fp32 */
        int32_t ex = 1;
        while ((man & 0x400u) == 0) { man <<= 1; ex -= 1; }
        man &= 0x3ffu;
        return u2f(sign | ((uint32_t)(ex + 112) << 23) | (man << 13));
    }
    if (e == 31) return u2f(sign | 0x7f800000u | (man << 13));
    return u2f(sign | ((e + 112u) << 23) | (man << 13));
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static void wr16(uint8_t* p, uint16_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }

/* ---------------------------------------------------------------------------
 * Quantizers.  q8_0 follows src/quant.cc:130-190; q4_0 follows
 * src/quant.cc:228-302.  Per block: max|x| over the block's real elements,
 * d = max/127 (q8_0) or max/7 (q4_0) stored as fp16, inverse taken from the
 * STORED scale, q = round-half-away(x*id) (+8 for q4_0) clamped; an all-zero
 * block stores d = 0 and zero code bytes.
 * Padding elements of a partial last block: q8_0 stores 0, q4_0 stores code
 * round(0 + 8) = 8 (when the block is not all zero).
 * ------------------------------------------------------------------------- */
static void quant_q8_0_block(const float* x, int n, uint8_t* blk) {
    memset(blk, 0, 34);
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    if (!(amax > 0.0f)) return;
    uint16_t dh = orc_fp16_from_f32(amax / 127.0f);
    wr16(blk, dh);
    float sd = orc_f32_from_fp16(dh);
    float id = sd == 0.0f ? 0.0f : 1.0f / sd;
    for (int i = 0; i < n; ++i) {
        int q = (int)roundf(x[i] * id);
        if (q > 127) q = 127; else if (q < -127) q = -127;
        blk[2 + i] = (uint8_t)(int8_t)q;
    }
}

static int clamp15(int q) { return q < 0 ? 0 : (q > 15 ? 15 : q); }

static void quant_q4_0_block(const float* x, int n, uint8_t* blk) {
    memset(blk, 0, 18);
    float amax = 0.0f;
    for (int i = 0; i < n; ++i) { float a = fabsf(x[i]); if (a > amax) amax = a; }
    if (!(amax > 0.0f)) return; /* d = 0, qs = 0: the reference leaves the
                                   memset() zeros in place (quant.cc:258-295) */
    uint16_t dh = orc_fp16_from_f32(amax / 7.0f);
    wr16(blk, dh);
    float sd = orc_f32_from_fp16(dh);
    float id = sd == 0.0f ? 0.0f : 1.0f / sd;
    for (int j = 0; j < 16; ++j) {
        float v0 = j < n ? x[j] * id : 0.0f;
        float v1 = j + 16 < n ? x[j + 16] * id : 0.0f;
        int q0 = clamp15((int)roundf(v0 + 8.0f));
        int q1 = clamp15((int)roundf(v1 + 8.0f));
        blk[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* q4_1 has NO quantizer in the reference (tests/test_cuda.cc:115-131 builds
 * blocks by hand).  This one is defined by this project and is therefore
 * parity-unpinned: d = (max-min)/15 and m = min, both stored as fp16 with the
 * reference's encoder; codes use the STORED values:
 * q = clamp(round-half-away((x - m') * (1/d')), 0, 15); d' = 0 gives q = 0.
 * Padding elements get code 0. */
static void quant_q4_1_block(const float* x, int n, uint8_t* blk) {
    memset(blk, 0, 20);
    float mn = x[0], mx = x[0];
    for (int i = 1; i < n; ++i) { if (x[i] < mn) mn = x[i]; if (x[i] > mx) mx = x[i]; }
    uint16_t dh = orc_fp16_from_f32((mx - mn) / 15.0f);
    uint16_t mh = orc_fp16_from_f32(mn);
    wr16(blk, dh);
    wr16(blk + 2, mh);
    float sd = orc_f32_from_fp16(dh);
    float sm = orc_f32_from_fp16(mh);
    float id = sd == 0.0f ? 0.0f : 1.0f / sd;
    for (int j = 0; j < 16; ++j) {
        int q0 = j < n ? clamp15((int)roundf((x[j] - sm) * id)) : 0;
        int q1 = j + 16 < n ? clamp15((int)roundf((x[j + 16] - sm) * id)) : 0;
        blk[4 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* Quantize a row-major [rows, cols] fp32 matrix; rows are independent
 * (src/quant.cc:135-139 takes the row length from shape.back()). */
int orc_quantize(int fmt, const float* src, int64_t rows, int64_t cols, uint8_t* out) {
    int bs = orc_block_bytes(fmt);
    if (!bs || rows <= 0 || cols <= 0) return -1;
    int64_t bpr = (cols + ORC_QK - 1) / ORC_QK;
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t b = 0; b < bpr; ++b) {
            const float* x = src + r * cols + b * ORC_QK;
            int n = (int)((cols - b * ORC_QK) < ORC_QK ? (cols - b * ORC_QK) : ORC_QK);
            uint8_t* blk = out + (r * bpr + b) * bs;
            if (fmt == ORC_Q8_0) quant_q8_0_block(x, n, blk);
            else if (fmt == ORC_Q4_0) quant_q4_0_block(x, n, blk);
            else quant_q4_1_block(x, n, blk);
        }
    }
    return 0;
}

/* ---------------------------------------------------------------------------
 * Element decode, one element at a time, the way dequantQ80/Q40/Q41 do it
 * (src/quant.cc:477-503): w = d*q (q8_0), d*(q-8) (q4_0), d*q + m (q4_1),
 * each a single fp32 multiply (and add) of the decoded fp16 fields.
 * ------------------------------------------------------------------------- */
static inline float decode_elem(int fmt, const uint8_t* blk, int i) {
    float d = orc_f32_from_fp16(rd16(blk));
    if (fmt == ORC_Q8_0) return d * (float)(int8_t)blk[2 + i];
    if (fmt == ORC_Q4_0) {
        int q = i < 16 ? (blk[2 + i] & 0x0F) : (blk[2 + i - 16] >> 4);
        return d * (float)(q - 8);
    }
    float m = orc_f32_from_fp16(rd16(blk + 2));
    int q = i < 16 ? (blk[4 + i] & 0x0F) : (blk[4 + i - 16] >> 4);
    return d * (float)q + m;
}

/* Dequantize to a row-major fp32 [rows, cols] matrix
 * (src/quant.cc:192-223, 304-345, 350-392). */
int orc_dequantize(int fmt, const uint8_t* blocks, int64_t rows, int64_t cols, float* dst) {
    int bs = orc_block_bytes(fmt);
    if (!bs || rows <= 0 || cols <= 0) return -1;
    int64_t bpr = (cols + ORC_QK - 1) / ORC_QK;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t k = 0; k < cols; ++k)
            dst[r * cols + k] = decode_elem(fmt, blocks + (r * bpr + k / ORC_QK) * bs, (int)(k % ORC_QK));
    return 0;
}

/* ---------------------------------------------------------------------------
 * Linear y[r, o] = sum_k w[o, k] * x[r, k], following linearQuantizedImpl
 * (src/quant.cc:401-475): one fp32 accumulator per output, k ascending,
 * sum += w*x with w decoded per element.  Outputs are independent, so the
 * pthread split below (contiguous ranges of the flat index r*out + o, as
 * ThreadPool::submitTask does in src/threadpool.cc:26-57) changes nothing.
 * ------------------------------------------------------------------------- */
typedef struct {
    int fmt;
    const float* x;
    int64_t in;
    const uint8_t* w;
    int64_t out;
    float* y;
    int64_t begin, end;
} lin_job;

static void* lin_worker(void* arg) {
    lin_job* j = (lin_job*)arg;
    int bs = orc_block_bytes(j->fmt);
    int64_t bpr = (j->in + ORC_QK - 1) / ORC_QK;
    for (int64_t f = j->begin; f < j->end; ++f) {
        int64_t r = f / j->out, o = f % j->out;
        const float* xr = j->x + r * j->in;
        const uint8_t* wr = j->w + o * bpr * bs;
        float sum = 0.0f;
        for (int64_t b = 0; b < bpr; ++b) {
            const uint8_t* blk = wr + b * bs;
            int64_t k0 = b * ORC_QK;
            int64_t k1 = k0 + ORC_QK < j->in ? k0 + ORC_QK : j->in;
            for (int64_t k = k0; k < k1; ++k) {
                float w = decode_elem(j->fmt, blk, (int)(k - k0));
                sum += w * xr[k];
            }
        }
        j->y[f] = sum;
    }
    return NULL;
}

int orc_linear(int fmt, const float* x, int64_t xrows, int64_t in, const uint8_t* blocks,
               int64_t out, float* y, int threads) {
    if (!orc_block_bytes(fmt) || xrows <= 0 || in <= 0 || out <= 0) return -1;
    int64_t n = xrows * out;
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if (n < 16 * (int64_t)threads) threads = 1;
    pthread_t th[256];
    lin_job jobs[256];
    int64_t chunk = n / threads, rem = n % threads, start = 0;
    for (int t = 0; t < threads; ++t) {
        int64_t len = chunk + (t < rem ? 1 : 0);
        jobs[t] = (lin_job){fmt, x, in, blocks, out, y, start, start + len};
        start += len;
    }
    for (int t = 1; t < threads; ++t) pthread_create(&th[t], NULL, lin_worker, &jobs[t]);
    lin_worker(&jobs[0]);
    for (int t = 1; t < threads; ++t) pthread_join(th[t], NULL);
    return 0;
}

/* ---------------------------------------------------------------------------
 * Epilogues that follow the linear in the reference's forward path.
 * ------------------------------------------------------------------------- */

/* h[i] = silu(gate[i]) * up[i], as the reference's swiGlu (src/ops.cc:111-145):
 * silu computes val / (1.0 + std::exp(-val)) -- std::exp of a float is the
 * float exp, the sum and quotient are double -- stored as float, then
 * elementwiseMul multiplies two floats. */
int orc_swiglu(const float* gate, const float* up, int64_t n, float* h) {
    if (n < 0) return -1;
    for (int64_t i = 0; i < n; ++i) {
        const float v = gate[i];
        const float s = (float)((double)v / (1.0 + (double)expf(-v)));
        h[i] = s * up[i];
    }
    return 0;
}

/* y[r][c] += bias[c]: the host variants' bias add after the download
 * (src/cuda_quant.cu:326-329), one float add per output. */
int orc_add_bias(float* y, const float* bias, int64_t rows, int64_t cols) {
    if (rows < 0 || cols < 0) return -1;
    for (int64_t r = 0; r < rows; ++r)
        for (int64_t c = 0; c < cols; ++c) y[r * cols + c] = y[r * cols + c] + bias[c];
    return 0;
}
