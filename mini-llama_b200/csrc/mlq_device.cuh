// mlq_device.cuh -- device primitives shared by the mlq kernels (sm_100a).
//
// Block formats (the reference's include/mini_llama/quantized_tensor.h:36-72):
//   q8_0 { u16 d; i8 qs[32]; }          34 B   w = d*q
//   q4_0 { u16 d; u8 qs[16]; }          18 B   w = d*(q-8)
//   q4_1 { u16 d; u16 m; u8 qs[16]; }   20 B   w = d*q + m
// q4 nibble order: element j is the low nibble of qs[j], element 16+j the
// high nibble (src/quant.cc:329-340).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace mlq {

enum Format : int { kQ4_0 = 2, kQ4_1 = 3, kQ8_0 = 8 };

constexpr int kQK = 32;  // values per block

// Static facts per format for the streaming GEMV.  A "group" is the unit one
// lane decodes from shared memory: 2 blocks for q8_0/q4_0, 1 for q4_1, chosen
// so the group is a whole, ODD number of 32-bit words (17, 9, 5).  Lanes then
// read consecutive groups with 32-bit loads that hit 32 distinct banks.
template <int F>
struct Fmt;
template <>
struct Fmt<kQ8_0> {
    static constexpr int kBlockBytes = 34;
    static constexpr int kGroupBlocks = 2;
};
template <>
struct Fmt<kQ4_0> {
    static constexpr int kBlockBytes = 18;
    static constexpr int kGroupBlocks = 2;
};
template <>
struct Fmt<kQ4_1> {
    static constexpr int kBlockBytes = 20;
    static constexpr int kGroupBlocks = 1;
};

__host__ __device__ constexpr int block_bytes(int f) {
    return f == kQ8_0 ? 34 : (f == kQ4_0 ? 18 : (f == kQ4_1 ? 20 : 0));
}

// Exact fp16 -> fp32 of a raw bit pattern (hardware conversion; exact for
// every finite value and for infinities).
__device__ __forceinline__ float half_bits_to_float(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16)));
}

// SwiGLU of one output: silu(g) * u with silu(v) = v / (1 + exp(-v)), in the
// reference's fp32 steps (siluKernel, then elementwiseMulKernel:
// src/cuda_ops.cu:147-160), each rounded on its own.
__device__ __forceinline__ float silu_mul(float g, float u) {
    return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// ---------------------------------------------------------------------------
// Error reporting from kernels.  A kernel that gives up (a bounded wait ran
// out) records a code here and returns; the host reads it back with
// mlq_device_error().  Codes: 1 = pipeline "full" wait, 2 = "empty" wait,
// 3 = drain wait, 4 = peer flag wait, 5 = consumer rendezvous, 6 = x-tile
// "empty" wait, 7 = resident x tiles ready wait, 8 = staged x copy wait,
// 12-16 = GEMM waits, 20-26 = batched-decode GEMM waits.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void report_error(int* err, int code) {
    if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wall-clock bound for every spin in this library.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

// ---------------------------------------------------------------------------
// mbarrier (shared::cta) helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}"
                 ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity), "r"(1000000u)  // suspend-time hint: 1 ms
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete.  Returns false
// when kWaitLimitNs elapses first (the caller then reports and bails out).
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 0 && global_ns() - t0 > kWaitLimitNs) return false;  // clock read rarely
    }
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
    asm volatile(
        "{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
            bar),
        "r"(bytes)
        : "memory");
}

// 1-D bulk copy global -> shared (TMA, no tensor map), completion counted in
// bytes on an mbarrier.  dst/src 16-B aligned, bytes a multiple of 16.
// No multicast: every copy reads this GPU's own memory into this CTA only.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            dst),
        "l"(src), "r"(bytes), "r"(bar)
        : "memory");
}

// 2-D tiled TMA load (tensor map in kernel-parameter space), completion
// counted in bytes on an mbarrier.  No multicast.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            uint32_t bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
        "[%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
        : "memory");
}

// L2 eviction policy for data read once per launch (the GEMV's weight
// stream): its lines go first when L2 needs room, so small data that is
// read again -- x, y, bias, the next launch's inputs -- stays in L2 instead
// of being pushed out by hundreds of MB of weights.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// bulk_g2s with an L2 cache policy (see l2_evict_first_policy).
__device__ __forceinline__ void bulk_g2s_hint(uint32_t dst, const void* src, uint32_t bytes,
                                              uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1], %2, [%3], %4;" ::"r"(dst),
        "l"(src), "r"(bytes), "r"(bar), "l"(policy)
        : "memory");
}

// tma_load_2d with an L2 cache policy (see l2_evict_first_policy).
__device__ __forceinline__ void tma_load_2d_hint(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t bar, uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint "
        "[%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
        : "memory");
}

// Hint: bring [src, src + bytes) into L2 (16-B aligned, bytes % 16 == 0).
__device__ __forceinline__ void prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic
// stream serialization may start before its predecessor in the stream has
// finished; grid_dependency_wait() blocks the calling thread until the
// predecessor has completed and its memory is visible.  launch_dependents()
// lets the next kernel in the stream be scheduled early.
__device__ __forceinline__ void grid_dependency_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Read-only, L1-bypassing 128-bit global load (x tiles: each CTA touches
// them once per stage, the L2 keeps them for the other CTAs).
__device__ __forceinline__ float4 ldg_nc_f4(const float* p) {
    float4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p));
    return v;
}

// GPU-scope acquire-release atomic add (returns the old value).
__device__ __forceinline__ unsigned int atom_add_acq_rel_gpu(unsigned int* p, unsigned int v) {
    unsigned int old;
    asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// System-scope acquire-release fence, then relaxed system-scope flag
// stores: one release for several flags (peer memory).
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_relaxed_sys(uint32_t* p, uint32_t v) {
    asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// System-scope acquire load of a 32-bit flag (written by a peer).
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ uint32_t lds_u16(uint32_t addr) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ uint32_t lds_u32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

__device__ __forceinline__ float4 lds_f4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts_f4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}

__device__ __forceinline__ uint4 lds_u4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr));
    return v;
}

__device__ __forceinline__ float2 lds_f2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
    return v;
}

__device__ __forceinline__ void sts_u4(uint32_t addr, uint4 v) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z),
                 "r"(v.w)
                 : "memory");
}

__device__ __forceinline__ void sts_f2(uint32_t addr, float2 v) {
    asm volatile("st.shared.v2.f32 [%0], {%1,%2};" ::"r"(addr), "f"(v.x), "f"(v.y) : "memory");
}

__device__ __forceinline__ void sts_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}

__device__ __forceinline__ void sts_u8(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u8 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}

}  // namespace mlq
