// Peer-memory plumbing for the tensor-parallel o_proj exchange (mllm_b200/tp.py PeerExchange):
// buffers shared between the ranks' processes through CUDA IPC, 32-bit flags a rank raises in a
// peer's memory, a bounded wait on such a flag, and a kernel that sums rows read from the ranks'
// buffers (over NVLink, by the SMs) and stores the result into every rank's buffer.
//
// One exchange step is: (each rank) the GEMM writes its partial rows into its own shared
// buffer, then mllm_signal_u32 raises a monotonically increasing value in the owner's flag (a
// system-scope release after the GEMM completed); (owner) mllm_wait_u32 on its local flags (an
// acquire; bounded: after about four seconds it records MLLM_ERR_DEVICE_TIMEOUT and returns),
// then mllm_sum_bf16 pulls the partials from every rank and pushes the sum to every rank, then
// flags tell each rank its rows have arrived.  No multicast object or multicast load is involved,
// and no library kernel ever reads or writes a peer's memory.
#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "host_util.h"

namespace mllm_b200 {
namespace {

__global__ void signal_kernel(uint32_t* flag, uint32_t value) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(value) : "memory");
}

// A peer's flag depends on another process's host-side progress (its launches can lag this
// rank's by a scheduling hiccup), so this wait allows about four seconds, not one.
constexpr uint32_t kPeerSpinLimit = 4u * kSpinLimit;

__global__ void wait_kernel(const uint32_t* flag, uint32_t value) {
    for (uint32_t i = 0; i < kPeerSpinLimit; ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if ((int32_t)(v - value) >= 0) return;
        if (i > 64) __nanosleep(256);
    }
    record_error(kErrTimeout);
}

// The same wait bounded by device time (%globaltimer, ns) instead of a poll count.  The poll
// count is capped too (far above any timeout the host accepts), so the loop ends even if the
// timer were to stall.
__device__ __forceinline__ uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}

__global__ void wait_for_kernel(const uint32_t* flag, uint32_t value, uint64_t timeout_ns) {
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < (1u << 31); ++i) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flag) : "memory");
        if ((int32_t)(v - value) >= 0) return;
        if (global_ns() - t0 > timeout_ns) break;
        if (i > 64) __nanosleep(256);
    }
    record_error(kErrTimeout);
}

constexpr int kMaxSum = 8;
struct SumPtrs {
    const uint4* src[kMaxSum];
    uint4* dst[kMaxSum];
};

// Loads 16 bytes that another GPU may have written (before raising the flag this stream
// waited on): volatile, so no stale copy of a line from an earlier call can be used.
__device__ __forceinline__ uint4 ld_volatile_16(const uint4* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

__device__ __forceinline__ void add_bf16x2(float& lo, float& hi, uint32_t w) {
    __nv_bfloat162 v = *reinterpret_cast<__nv_bfloat162*>(&w);
    lo += __low2float(v);
    hi += __high2float(v);
}

// dst_d[i] = sum_s src_s[i] for every destination d: fp32 in the order s = 0, 1, ..., rounded
// once to bf16.  A thread takes kVec 16-byte vectors per round and loads all of them from every
// source before any add, so it keeps kVec * n_src loads in flight (over NVLink for a peer's
// buffer); the result is stored to every destination (a peer's buffer included).  The grid is
// kept to about half the SMs: the o_proj GEMM of the next piece runs beside it.
constexpr int kVec = 4;

template <int NS>
__global__ void __launch_bounds__(256) sum_rows_kernel(SumPtrs p, int n_dst, int64_t n16) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n16; i0 += stride * kVec) {
        uint4 v[kVec][NS];
#pragma unroll
        for (int u = 0; u < kVec; ++u) {
            const int64_t i = i0 + u * stride;
#pragma unroll
            for (int s = 0; s < NS; ++s)
                if (i < n16) v[u][s] = ld_volatile_16(p.src[s] + i);
        }
#pragma unroll
        for (int u = 0; u < kVec; ++u) {
            const int64_t i = i0 + u * stride;
            if (i >= n16) break;
            float f[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] = 0.f;
#pragma unroll
            for (int s = 0; s < NS; ++s) {
                add_bf16x2(f[0], f[1], v[u][s].x);
                add_bf16x2(f[2], f[3], v[u][s].y);
                add_bf16x2(f[4], f[5], v[u][s].z);
                add_bf16x2(f[6], f[7], v[u][s].w);
            }
            uint4 o;
            o.x = pack_bf16x2(f[0], f[1]);
            o.y = pack_bf16x2(f[2], f[3]);
            o.z = pack_bf16x2(f[4], f[5]);
            o.w = pack_bf16x2(f[6], f[7]);
#pragma unroll
            for (int d = 0; d < kMaxSum; ++d)
                if (d < n_dst) p.dst[d][i] = o;
        }
    }
}

}  // namespace

MLLM_DEFINE_STATUS_READER(peer)

}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" int mllm_ipc_alloc(size_t bytes, void** ptr) {
    if (!ptr || bytes == 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "ipc_alloc: bad arguments");
    *ptr = nullptr;
    if (int st = check_cuda(cudaMalloc(ptr, bytes), "ipc_alloc: cudaMalloc")) return st;
    if (int st = check_cuda(cudaMemset(*ptr, 0, bytes), "ipc_alloc: cudaMemset")) return st;
    return ok();
}

extern "C" int mllm_ipc_free(void* ptr) {
    if (!ptr) return ok();
    if (int st = check_cuda(cudaFree(ptr), "ipc_free")) return st;
    return ok();
}

extern "C" int mllm_ipc_get_handle(const void* ptr, void* handle) {
    if (!ptr || !handle) return fail(MLLM_ERR_INVALID_ARGUMENT, "ipc_get_handle: null pointer");
    cudaIpcMemHandle_t h;
    if (int st = check_cuda(cudaIpcGetMemHandle(&h, const_cast<void*>(ptr)), "cudaIpcGetMemHandle")) return st;
    static_assert(sizeof(h) == MLLM_IPC_HANDLE_BYTES, "IPC handle size");
    memcpy(handle, &h, sizeof(h));
    return ok();
}

extern "C" int mllm_ipc_open_handle(const void* handle, void** ptr) {
    if (!ptr || !handle) return fail(MLLM_ERR_INVALID_ARGUMENT, "ipc_open_handle: null pointer");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof(h));
    *ptr = nullptr;
    if (int st = check_cuda(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle"))
        return st;
    return ok();
}

extern "C" int mllm_ipc_close_handle(void* ptr) {
    if (!ptr) return ok();
    if (int st = check_cuda(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle")) return st;
    return ok();
}

extern "C" int mllm_copy_async(void* dst, const void* src, size_t bytes, mllm_stream_t stream) {
    if (bytes == 0) return ok();
    if (!dst || !src) return fail(MLLM_ERR_INVALID_ARGUMENT, "copy_async: null pointer");
    if (int st = check_cuda(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream),
                            "copy_async"))
        return st;
    return ok();
}

extern "C" int mllm_signal_u32(uint32_t* flag, uint32_t value, mllm_stream_t stream) {
    if (!flag || !aligned(flag, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "signal_u32: bad flag pointer");
    signal_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(flag, value);
    if (int st = check_cuda(cudaGetLastError(), "signal_u32 launch")) return st;
    return ok();
}

extern "C" int mllm_wait_u32(const uint32_t* flag, uint32_t value, mllm_stream_t stream) {
    if (!flag || !aligned(flag, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "wait_u32: bad flag pointer");
    wait_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(flag, value);
    if (int st = check_cuda(cudaGetLastError(), "wait_u32 launch")) return st;
    return ok();
}

extern "C" int mllm_wait_u32_timeout(const uint32_t* flag, uint32_t value, uint32_t timeout_us,
                                     mllm_stream_t stream) {
    if (!flag || !aligned(flag, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "wait_u32_timeout: bad flag pointer");
    if (timeout_us < 1 || timeout_us > 60u * 1000u * 1000u)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "wait_u32_timeout: timeout must lie in [1 us, 60 s]");
    wait_for_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(flag, value, (uint64_t)timeout_us * 1000ull);
    if (int st = check_cuda(cudaGetLastError(), "wait_u32_timeout launch")) return st;
    return ok();
}

extern "C" int mllm_sum_bf16(void* const* dsts, int n_dst, const void* const* srcs, int n_src, int64_t count,
                             mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_sum_bf16");
    if (n_src < 1 || n_src > kMaxSum || n_dst < 1 || n_dst > kMaxSum || count < 0 || (count % 8) != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: 1..8 sources and destinations, count a multiple of 8");
    if (count == 0) return ok();
    if (!dsts || !srcs) return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: null pointer arrays");
    SumPtrs p = {};
    for (int i = 0; i < n_src; ++i) {
        if (!srcs[i] || !aligned(srcs[i], 16)) return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: bad source");
        p.src[i] = static_cast<const uint4*>(srcs[i]);
    }
    for (int i = 0; i < n_dst; ++i) {
        if (!dsts[i] || !aligned(dsts[i], 16)) return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: bad destination");
        p.dst[i] = static_cast<uint4*>(dsts[i]);
    }
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;
    const int64_t n16 = count / 8;
    const int blocks = (int)std::max<int64_t>(1, std::min<int64_t>((n16 + 256 * kVec - 1) / (256 * kVec),
                                                                    (int64_t)(num_sms + 1) / 2));
    cudaStream_t s = (cudaStream_t)stream;
    switch (n_src) {
        case 1: sum_rows_kernel<1><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        case 2: sum_rows_kernel<2><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        case 3: sum_rows_kernel<3><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        case 4: sum_rows_kernel<4><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        case 5: sum_rows_kernel<5><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        case 6: sum_rows_kernel<6><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        case 7: sum_rows_kernel<7><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
        default: sum_rows_kernel<8><<<blocks, 256, 0, s>>>(p, n_dst, n16); break;
    }
    if (int st = check_cuda(cudaGetLastError(), "sum_bf16 launch")) return st;
    return ok();
}
