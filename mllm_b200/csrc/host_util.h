// Host-side helpers shared by the C-ABI entry points: error reporting, device checks and
// TMA tensor-map encoding.  Nothing here throws across the C boundary.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

#include <string>
#include <utility>

#include "../../include/mllm_attn.h"

namespace mllm_b200 {

// Records `msg` as this thread's last error and returns `status`.
int fail(int status, const std::string& msg);
// Clears the thread's last error and returns MLLM_OK.
int ok();

// Checks a CUDA runtime result; on failure records it and returns MLLM_ERR_CUDA.
int check_cuda(cudaError_t e, const char* what);

// Returns MLLM_OK if the current device is sm_100 (B200 class), else a failure status.
int require_sm100(int* num_sms = nullptr);

// Launches `kern` with programmatic stream serialisation (the kernel calls pdl_wait() before
// touching data written by the previous kernel in the stream).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// An NVTX range around a host call (the launch side of an entry point), visible to Nsight and
// ncu's NVTX filters.  Header-only NVTX3: without a profiler attached it costs a pointer check.
struct NvtxRange {
    explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
    ~NvtxRange() { nvtxRangePop(); }
    NvtxRange(const NvtxRange&) = delete;
    NvtxRange& operator=(const NvtxRange&) = delete;
};
#define MLLM_NVTX_RANGE(name) ::mllm_b200::NvtxRange mllm_nvtx_range_(name)

// Per-translation-unit device status readers (see MLLM_DEFINE_STATUS_READER).
int read_clear_status_decode(cudaStream_t s, unsigned* out);
int read_clear_status_prefill(cudaStream_t s, unsigned* out);
int read_clear_status_epilogue(cudaStream_t s, unsigned* out);
int read_clear_status_peer(cudaStream_t s, unsigned* out);
int read_clear_status_linear(cudaStream_t s, unsigned* out);

// Encodes a 4-D bf16 tensor map {d (inner), rows, heads, batch} with 128-byte swizzle and a
// {box_d, box_rows, box_heads, 1} box.  Strides are in elements and need not be ordered (a
// weight matrix is viewed as {64 columns, rows, column blocks} with the blocks 128 B apart).
// Returns MLLM_OK or an error.
int encode_kv_map(CUtensorMap* map, const void* base, int64_t d, int64_t rows, int64_t heads, int64_t batch,
                  int64_t stride_row, int64_t stride_head, int64_t stride_batch, uint32_t box_d,
                  uint32_t box_rows, uint32_t box_heads = 1);

// Encodes a 2-D byte tensor map {cols (inner), rows} with row stride `stride_row` bytes and a
// {box_cols, box_rows} box (as a 4-D map with unit outer dimensions, so that the 4-D load helper
// serves it); with swizzle128 the box rows (box_cols <= 128) land with the 128-byte swizzle: 16-byte
// chunk c of box row r at chunk c ^ (r % 8).  Returns MLLM_OK or an error.
int encode_u8_map(CUtensorMap* map, const void* base, int64_t cols, int64_t rows, int64_t stride_row,
                  uint32_t box_cols, uint32_t box_rows, bool swizzle128 = false);

}  // namespace mllm_b200
