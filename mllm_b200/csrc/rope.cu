// RoPE table builder and standalone RoPE apply (the mllm::RoPE facade's device path).
//
// Both follow the reference's fp32 step order (src/core/runtime/RoPE.h):
//   inv_freq[j] = exp(-((2j / D) * ln(theta)))      RoPE.h:43-50  (two fp32 roundings, exp)
//   angle       = float(pos) * inv_freq[j]           RoPE.h:52-54
//   cos/sin     = cos/sin(angle), duplicated over both halves of the row (RoPE.h:56-58)
//   apply       = x*cos + cat(-x2, x1)*sin, each op rounded separately (RoPE.h:77-88)
// The products and the sum use __fmul_rn/__fadd_rn so the compiler cannot contract them
// into an FMA (the reference rounds after each tensor op).
#include "common.cuh"
#include "host_util.h"
#include "rope_math.cuh"

namespace mllm_b200 {
namespace {

__global__ void rope_table_kernel(const int64_t* __restrict__ pos, int64_t n, int head_dim, float log_theta,
                                  float* __restrict__ cos_out, float* __restrict__ sin_out) {
    const int half = head_dim >> 1;
    const int64_t total = n * half;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t row = i / half;
        const int j = (int)(i - row * half);
        float c, s;
        rope_angle_cos_sin(pos[row], j, head_dim, log_theta, c, s);
        float* crow = cos_out + row * head_dim;
        float* srow = sin_out + row * head_dim;
        crow[j] = c;
        crow[j + half] = c;
        srow[j] = s;
        srow[j + half] = s;
    }
}

__global__ void rope_apply_kernel(const __nv_bfloat16* __restrict__ x, int64_t sb, int64_t sh, int64_t ss,
                                  int B, int H, int S, int D, const float* __restrict__ cos,
                                  const float* __restrict__ sin, __nv_bfloat16* __restrict__ out) {
    const int half = D >> 1;
    const int64_t total = (int64_t)B * H * S * half;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        int64_t r = i / half;
        const int j = (int)(i - r * half);
        const int s = (int)(r % S);
        r /= S;
        const int h = (int)(r % H);
        const int b = (int)(r / H);
        const __nv_bfloat16* xr = x + b * sb + h * sh + s * ss;
        const float x1 = __bfloat162float(xr[j]);
        const float x2 = __bfloat162float(xr[j + half]);
        const float* c = cos + (int64_t)s * D;
        const float* sn = sin + (int64_t)s * D;
        float lo, hi;
        rope_rotate_pair(x1, x2, c[j], sn[j], c[j + half], sn[j + half], lo, hi);
        __nv_bfloat16* o = out + (((int64_t)b * H + h) * S + s) * D;
        o[j] = __float2bfloat16_rn(lo);
        o[j + half] = __float2bfloat16_rn(hi);
    }
}

int grid_for(int64_t work, int threads) {
    int64_t g = (work + threads - 1) / threads;
    if (g < 1) g = 1;
    if (g > 148 * 32) g = 148 * 32;
    return (int)g;
}

}  // namespace
}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" int mllm_rope_build_cos_sin(const int64_t* positions, int64_t n, int head_dim, double rope_theta,
                                       float* cos_out, float* sin_out, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_rope_build_cos_sin");
    if (head_dim <= 0 || head_dim % 2 != 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: head_dim must be even.");
    if (n < 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: negative position count");
    if (!(rope_theta > 0.0)) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: rope_theta must be positive");
    if (n == 0) return ok();
    if (!positions || !cos_out || !sin_out) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: null pointer");
    if (int st = require_sm100()) return st;
    const int threads = 256;
    rope_table_kernel<<<grid_for(n * (head_dim / 2), threads), threads, 0, (cudaStream_t)stream>>>(
        positions, n, head_dim, rope_log_theta(rope_theta), cos_out, sin_out);
    if (int st = check_cuda(cudaGetLastError(), "rope_table_kernel launch")) return st;
    return ok();
}

extern "C" int mllm_rope_apply_bf16(const void* x, int64_t sb, int64_t sh, int64_t ss, int batch, int num_heads,
                                    int seq_len, int head_dim, const float* cos, const float* sin, void* out,
                                    mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_rope_apply_bf16");
    if (head_dim <= 0 || head_dim % 2 != 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: head_dim must be even.");
    if (batch < 0 || num_heads < 0 || seq_len < 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: negative size");
    const int64_t total = (int64_t)batch * num_heads * seq_len;
    if (total == 0) return ok();
    if (!x || !cos || !sin || !out) return fail(MLLM_ERR_INVALID_ARGUMENT, "RoPE: null pointer");
    if (int st = require_sm100()) return st;
    const int threads = 256;
    rope_apply_kernel<<<grid_for(total * (head_dim / 2), threads), threads, 0, (cudaStream_t)stream>>>(
        (const __nv_bfloat16*)x, sb, sh, ss, batch, num_heads, seq_len, head_dim, cos, sin, (__nv_bfloat16*)out);
    if (int st = check_cuda(cudaGetLastError(), "rope_apply_kernel launch")) return st;
    return ok();
}
