// C-ABI plumbing: status strings, per-thread error detail, the device status word, device
// checks and TMA tensor-map encoding through the driver entry point (no -lcuda needed).
#include <cudaTypedefs.h>

#include <cstdio>
#include <mutex>
#include <string>

#include "common.cuh"
#include "host_util.h"

namespace mllm_b200 {

namespace {
thread_local std::string t_last_error;

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
        }
    });
    return fn;
}
}  // namespace

int fail(int status, const std::string& msg) {
    t_last_error = msg;
    return status;
}

int ok() {
    t_last_error.clear();
    return MLLM_OK;
}

int check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return MLLM_OK;
    return fail(MLLM_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

int require_sm100(int* num_sms) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return fail(MLLM_ERR_NO_DEVICE, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
    // Cached per device: attribute queries are cheap but not free on the decode path.
    static int cached_major[64], cached_sms[64];
    static bool cached[64];
    if (dev < 64 && cached[dev]) {
        if (num_sms) *num_sms = cached_sms[dev];
        return cached_major[dev] == 10 ? MLLM_OK
                                       : fail(MLLM_ERR_NO_DEVICE, "current device is not sm_100 (B200)");
    }
    int major = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return fail(MLLM_ERR_NO_DEVICE, "cannot query device attributes");
    if (dev < 64) {
        cached_major[dev] = major;
        cached_sms[dev] = sms;
        cached[dev] = true;
    }
    if (num_sms) *num_sms = sms;
    if (major != 10) return fail(MLLM_ERR_NO_DEVICE, "current device is not sm_100 (B200)");
    return MLLM_OK;
}

int encode_kv_map(CUtensorMap* map, const void* base, int64_t d, int64_t rows, int64_t heads, int64_t batch,
                  int64_t stride_row, int64_t stride_head, int64_t stride_batch, uint32_t box_d,
                  uint32_t box_rows, uint32_t box_heads) {
    auto fn = get_encode_fn();
    if (!fn) return fail(MLLM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    if (!aligned(base, 16)) return fail(MLLM_ERR_INVALID_ARGUMENT, "TMA base address must be 16-byte aligned");
    const int64_t es = 2;  // bf16
    for (int64_t s : {stride_row, stride_head, stride_batch}) {
        if ((s * es) % 16 != 0 || s <= 0)
            return fail(MLLM_ERR_INVALID_ARGUMENT, "cache strides must be positive multiples of 8 elements");
    }
    cuuint64_t dims[4] = {(cuuint64_t)d, (cuuint64_t)rows, (cuuint64_t)heads, (cuuint64_t)batch};
    cuuint64_t strides[3] = {(cuuint64_t)(stride_row * es), (cuuint64_t)(stride_head * es),
                             (cuuint64_t)(stride_batch * es)};
    cuuint32_t box[4] = {box_d, box_rows, box_heads, 1};
    cuuint32_t elem_strides[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                    elem_strides, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d) dims=%lld,%lld,%lld,%lld", (int)r,
                 (long long)d, (long long)rows, (long long)heads, (long long)batch);
        return fail(MLLM_ERR_INVALID_ARGUMENT, buf);
    }
    return MLLM_OK;
}

int encode_u8_map(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int64_t stride_row,
                  uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
    auto fn = get_encode_fn();
    if (!fn) return fail(MLLM_ERR_CUDA, "cuTensorMapEncodeTiled entry point unavailable");
    if (!aligned(base, 16)) return fail(MLLM_ERR_INVALID_ARGUMENT, "TMA base address must be 16-byte aligned");
    if (stride_row <= 0 || stride_row % 16 != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "byte-matrix row stride must be a positive multiple of 16");
    cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)rows, 1, 1};
    cuuint64_t strides[3] = {(cuuint64_t)stride_row, (cuuint64_t)(stride_row * rows), (cuuint64_t)(stride_row * rows)};
    cuuint32_t box[4] = {box_cols, box_rows, 1, 1};
    cuuint32_t elem_strides[4] = {1, 1, 1, 1};
    CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 4, const_cast<void*>(base), dims, strides, box, elem_strides,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        char buf[160];
        snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled (bytes) failed (%d) dims=%lld,%lld", (int)r,
                 (long long)cols, (long long)rows);
        return fail(MLLM_ERR_INVALID_ARGUMENT, buf);
    }
    return MLLM_OK;
}

}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" int mllm_attn_abi_version(void) { return 6; }

extern "C" const char* mllm_attn_status_string(int status) {
    switch (status) {
        case MLLM_OK: return "ok";
        case MLLM_ERR_INVALID_ARGUMENT: return "invalid argument";
        case MLLM_ERR_UNSUPPORTED: return "unsupported configuration";
        case MLLM_ERR_CUDA: return "CUDA error";
        case MLLM_ERR_WORKSPACE: return "workspace missing or too small";
        case MLLM_ERR_NO_DEVICE: return "no sm_100 device";
        case MLLM_ERR_DEVICE_TIMEOUT: return "device wait timed out";
        case MLLM_ERR_DEVICE_LENGTH: return "device length out of range";
        case MLLM_ERR_COMM: return "communicator failed or aborted";
        case MLLM_ERR_COMM_TIMEOUT: return "collective timed out";
        default: return "unknown status";
    }
}

extern "C" const char* mllm_attn_last_error(void) { return t_last_error.c_str(); }

extern "C" int mllm_attn_device_status(mllm_stream_t stream) {
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    constexpr int kReaders = 5;
    unsigned v[kReaders] = {0u, 0u, 0u, 0u, 0u};
    int (*readers[kReaders])(cudaStream_t, unsigned*) = {read_clear_status_decode, read_clear_status_prefill,
                                                         read_clear_status_epilogue, read_clear_status_peer,
                                                         read_clear_status_linear};
    for (int i = 0; i < kReaders; ++i) {
        const int e = readers[i](s, &v[i]);
        if (e != 0) return check_cuda((cudaError_t)e, "read device status");
    }
    if (int st = check_cuda(cudaStreamSynchronize(s), "synchronize")) return st;
    unsigned all = 0u;
    for (int i = 0; i < kReaders; ++i) all |= v[i];
    if (all & kErrTimeout) return fail(MLLM_ERR_DEVICE_TIMEOUT, "a kernel's bounded wait expired");
    if (all & kErrBadLength) return fail(MLLM_ERR_DEVICE_LENGTH, "a device-side length exceeded its capacity");
    if (all & kErrSmemAlign) return fail(MLLM_ERR_CUDA, "a kernel's dynamic shared memory was misaligned (no work done)");
    return ok();
}
