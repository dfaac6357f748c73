// Device-side building blocks shared by the attention kernels (sm_100a only).
//
// Everything here is a thin, hand-written wrapper over one documented PTX instruction:
// mbarrier phases, TMA tensor loads (no multicast anywhere in this library), ldmatrix,
// warp-level bf16 MMA, and bf16 packing.  Every spin-wait is bounded: after
// kSpinLimit polls it records kErrTimeout in the library's device status word and the
// caller abandons the loop, so a logic error surfaces as a status, never as a hang.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "mllm_b200 kernels target sm_100a only"
#endif

namespace mllm_b200 {

// ---------------------------------------------------------------------------------------
// Device status words.  Every translation unit that includes this header owns one (internal
// linkage, so the library needs no relocatable device code); kernels OR error bits into it and
// the host reads and clears all of them through mllm_attn_device_status().
// ---------------------------------------------------------------------------------------
enum DeviceError : unsigned {
    kErrNone = 0u,
    kErrTimeout = 1u,       // a bounded wait ran out (pipeline logic error)
    kErrBadLength = 2u,     // a device-side length exceeded the capacity given by the host
    kErrSmemAlign = 4u,     // a kernel found its dynamic shared memory less aligned than it needs
};
static __device__ unsigned g_tu_status = 0u;

__device__ __forceinline__ void record_error(unsigned bits) { atomicOr(&g_tu_status, bits); }

// Defines `int read_clear_status_<name>(cudaStream_t, unsigned*)`: copies this translation
// unit's status word to the host and clears it, in stream order (the caller synchronises).
#define MLLM_DEFINE_STATUS_READER(name)                                                             \
    int read_clear_status_##name(cudaStream_t s, unsigned* out) {                                   \
        static const unsigned zero = 0u;                                                            \
        cudaError_t e = cudaMemcpyFromSymbolAsync(out, g_tu_status, sizeof(unsigned), 0,            \
                                                  cudaMemcpyDeviceToHost, s);                       \
        if (e == cudaSuccess)                                                                       \
            e = cudaMemcpyToSymbolAsync(g_tu_status, &zero, sizeof(unsigned), 0,                    \
                                        cudaMemcpyHostToDevice, s);                                 \
        return e == cudaSuccess ? 0 : (int)e;                                                       \
    }

// ~1 s at B200 clocks with the nanosleep back-off below.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false (and records a timeout)
// if the phase did not complete within kSpinLimit polls.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if (i > 64) __nanosleep(128);
    }
    record_error(kErrTimeout);
    return false;
}

// ---------------------------------------------------------------------------------------
// Programmatic dependent launch: a kernel launched with programmatic stream serialisation may
// start while the previous kernel in the stream still runs; pdl_wait() blocks until that
// kernel has completed and its memory is visible (a no-op for an ordinary launch).
// pdl_trigger() lets the next kernel in the stream start launching early.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor), unicast only.  Coordinates are innermost-first; the innermost
// coordinate of every call site is a multiple of 64 bf16 elements (128 B), which satisfies
// the 16-byte rule for tiled copies.
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

// ---------------------------------------------------------------------------------------
// Warp-level tensor-core helpers (ldmatrix + m16n8k16 bf16 MMA, fp32 accumulate)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}

__device__ __forceinline__ void mma_bf16_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---------------------------------------------------------------------------------------
// Scalars
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// max(a, b, c) in one instruction (sm_100 three-input max).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Packed fp32 pair arithmetic (sm_100 f32x2): two IEEE round-to-nearest results per instruction.
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                     float c1) {
    unsigned long long a, b, c, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(c) : "f"(c0), "f"(c1));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1) {
    unsigned long long d, a;
    asm("mov.b64 %0, {%1, %2};" : "=l"(d) : "f"(d0), "f"(d1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("add.rn.f32x2 %0, %0, %1;" : "+l"(d) : "l"(a));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float bf16_to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

// Byte offset of (row, 16-byte chunk) inside a TMA box written with CU_TENSOR_MAP_SWIZZLE_128B:
// rows are 128 B, and the chunk index is XORed with (row mod 8).  Box bases are 1024-B aligned.
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
    return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

}  // namespace mllm_b200
