// Peer-memory plumbing for the tensor-parallel o_proj exchange (mllm_b200/tp.py PeerExchange):
// buffers shared between the ranks' processes through CUDA IPC, copies on the copy engines,
// 32-bit flags a rank raises in a peer's memory after its copy, a bounded wait on such a flag,
// and the sum of the ranks' partial rows.
//
// A transfer is: (sender) cudaMemcpyAsync of rows into the owner's buffer, then, on the same
// stream, mllm_signal_u32 of a monotonically increasing value into the owner's flag (a
// system-scope release after the copy completed); (owner) mllm_wait_u32 on its local flag (an
// acquire; bounded: after about four seconds it records MLLM_ERR_DEVICE_TIMEOUT and returns), then
// kernels that read the rows.  The data moves over NVLink on the copy engines, so it overlaps
// the GEMM running on the SMs.  No multicast object or multicast load is involved.
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

constexpr int kMaxSum = 8;
struct SumSources {
    const __nv_bfloat16* p[kMaxSum];
};

// out[i] = sum_s src_s[i] in fp32, in the order s = 0, 1, ..., rounded once to bf16.
__global__ void sum_kernel(__nv_bfloat16* out, SumSources src, int n, int64_t count2) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count2; i += stride) {
        float a = 0.f, b = 0.f;
        for (int s = 0; s < n; ++s) {
            const __nv_bfloat162 v = reinterpret_cast<const __nv_bfloat162*>(src.p[s])[i];
            a += __low2float(v);
            b += __high2float(v);
        }
        reinterpret_cast<__nv_bfloat162*>(out)[i] = __floats2bfloat162_rn(a, b);
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

extern "C" int mllm_sum_bf16(void* out, const void* const* srcs, int n, int64_t count, mllm_stream_t stream) {
    if (n < 1 || n > kMaxSum || count < 0 || (count & 1))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: 1..8 sources and an even element count");
    if (count == 0) return ok();
    if (!out || !srcs || !aligned(out, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: bad output");
    SumSources s = {};
    for (int i = 0; i < n; ++i) {
        if (!srcs[i] || !aligned(srcs[i], 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "sum_bf16: bad source");
        s.p[i] = (const __nv_bfloat16*)srcs[i];
    }
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;
    const int64_t count2 = count / 2;
    const int blocks = (int)std::min<int64_t>((count2 + 255) / 256, (int64_t)num_sms * 8);
    sum_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>((__nv_bfloat16*)out, s, n, count2);
    if (int st = check_cuda(cudaGetLastError(), "sum_bf16 launch")) return st;
    return ok();
}
