// Per-element RoPE arithmetic shared by the table builder, RoPE apply and the fused epilogue,
// so all three produce bit-identical angles and rotations.
#pragma once

#include <cmath>

#include "common.cuh"

namespace mllm_b200 {

// ln(theta) rounded to fp32 on the host, as the reference passes the double log through a
// float tensor op (RoPE.h:48-50: `idx / D * log_theta` on a float tensor).
inline float rope_log_theta(double theta) { return static_cast<float>(std::log(theta)); }

// The RoPE angle for column j (< D/2) at integer position `pos`.
__device__ __forceinline__ float rope_angle(int64_t pos, int j, int head_dim, float log_theta) {
    const float idx = (float)(2 * j);
    const float ratio = __fdiv_rn(idx, (float)head_dim);            // idx / D
    const float arg = -__fmul_rn(ratio, log_theta);                 // (.. * log_theta).neg()
    const float inv_freq = expf(arg);                               // .exp()
    return __fmul_rn((float)pos, inv_freq);                         // pos_f32 * inv_freq
}

// cos/sin of the RoPE angle for column j (< D/2) at integer position `pos`.
__device__ __forceinline__ void rope_angle_cos_sin(int64_t pos, int j, int head_dim, float log_theta, float& c,
                                                   float& s) {
    const float angle = rope_angle(pos, j, head_dim, log_theta);
    c = cosf(angle);
    s = sinf(angle);
}

// Rotates the pair (x1 = x[j], x2 = x[j + D/2]):
//   out[j]       = x1*cos[j]       + (-x2)*sin[j]
//   out[j + D/2] = x2*cos[j + D/2] + ( x1)*sin[j + D/2]
// with each multiply and the add rounded separately.
__device__ __forceinline__ void rope_rotate_pair(float x1, float x2, float c_lo, float s_lo, float c_hi,
                                                 float s_hi, float& lo, float& hi) {
    lo = __fadd_rn(__fmul_rn(x1, c_lo), __fmul_rn(-x2, s_lo));
    hi = __fadd_rn(__fmul_rn(x2, c_hi), __fmul_rn(x1, s_hi));
}

}  // namespace mllm_b200
