// Per-row QK-RMSNorm + RoPE arithmetic shared by the fused QKV epilogue and the fused decode
// step, so both write bit-identical q rows and cache rows.
//
// A warp owns one head row; lane L holds the elements d = L + 32*i (i < D/32).  That layout
// gives two things at once:
//   * RMSNorm's fp32 sum of squares in exactly the reference CPU LibTorch order
//     (8-wide vectors with 4 interleaved accumulators: lane L = 8k + j holds accumulator
//     P_k[j]; then ((P0+P1)+P2)+P3 per j, then j = 0..7 in sequence), so the bf16 result is
//     bit-identical to the reference;
//   * both halves of every RoPE pair (d, d + D/2) in the same lane: no shuffles.
// Every fp32 step uses explicit round-to-nearest intrinsics so no FMA contraction occurs.
#pragma once

#include "common.cuh"
#include "rope_math.cuh"

namespace mllm_b200 {

// Sum of squares of a head row in the reference's reduction order (see above); every lane
// returns the total.
template <int NI>
__device__ __forceinline__ float row_sum_squares(const float (&x)[NI], int lane) {
    float p = 0.f;
#pragma unroll
    for (int i = 0; i < NI; ++i) p = __fadd_rn(p, __fmul_rn(x[i], x[i]));
    const int j = lane & 7;
    const float p0 = __shfl_sync(0xffffffffu, p, j);
    const float p1 = __shfl_sync(0xffffffffu, p, j + 8);
    const float p2 = __shfl_sync(0xffffffffu, p, j + 16);
    const float p3 = __shfl_sync(0xffffffffu, p, j + 24);
    const float acc = __fadd_rn(__fadd_rn(__fadd_rn(p0, p1), p2), p3);
    float total = 0.f;
#pragma unroll
    for (int jj = 0; jj < 8; ++jj) total = __fadd_rn(total, __shfl_sync(0xffffffffu, acc, jj));
    return total;
}

// RMSNorm scale 1/sqrt(mean(x^2) + eps) from a row's sum of squares (RMSNorm.h:48-57:
// LibTorch CPU's rsqrt is 1/sqrt).
template <int D>
__device__ __forceinline__ float rms_scale(float sum_squares, float eps) {
    const float var = __fdiv_rn(sum_squares, (float)D);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// The RoPE values lane L needs for its pairs (d, d + D/2), d = L + 32*i, i < D/64: the
// table entries at column d ("lo") and d + D/2 ("hi").  For the reference's tables the two
// halves are equal; a caller-given table is read as given.
template <int D>
struct RopeLane {
    float c_lo[D / 64], s_lo[D / 64], c_hi[D / 64], s_hi[D / 64];
};

// From [D] cos/sin tables (shared memory or global).
template <int D>
__device__ __forceinline__ RopeLane<D> rope_lane_from_tables(const float* cos_, const float* sin_, int lane) {
    RopeLane<D> r;
#pragma unroll
    for (int i = 0; i < D / 64; ++i) {
        const int j = lane + 32 * i;
        r.c_lo[i] = cos_[j];
        r.s_lo[i] = sin_[j];
        r.c_hi[i] = cos_[j + D / 2];
        r.s_hi[i] = sin_[j + D / 2];
    }
    return r;
}

// Computed in registers for one position: lane L evaluates exactly the columns it needs, with
// the steps of rope_angle_cos_sin (so the values equal the table mllm_rope_build_cos_sin builds).
template <int D>
__device__ __forceinline__ RopeLane<D> rope_lane_compute(int64_t pos, int lane, float log_theta) {
    RopeLane<D> r;
#pragma unroll
    for (int i = 0; i < D / 64; ++i) {
        rope_angle_cos_sin(pos, lane + 32 * i, D, log_theta, r.c_lo[i], r.s_lo[i]);
        r.c_hi[i] = r.c_lo[i];
        r.s_hi[i] = r.s_lo[i];
    }
    return r;
}

// One q or k head row: optional RMSNorm (x * rr * w, rounded to bf16 as the reference's
// RMSNorm returns the input dtype; `rr` from rms_scale; gamma_l[i] = w[lane + 32*i] as fp32),
// then RoPE on the pairs (d, d + D/2) (RoPE.h:77-88), rounded to bf16.
template <int D>
__device__ __forceinline__ void qk_norm_rope_row(float (&x)[D / 32], bool norm, const float (&gamma_l)[D / 32],
                                                 float rr, const RopeLane<D>& rope, __nv_bfloat16 (&y)[D / 32]) {
    constexpr int NI = D / 32;
    constexpr int PAIR = NI / 2;   // slot i pairs with slot i + PAIR (distance D/2)
    if (norm) {
#pragma unroll
        for (int i = 0; i < NI; ++i)
            x[i] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(x[i], rr), gamma_l[i])));
    }
#pragma unroll
    for (int i = 0; i < PAIR; ++i) {
        float lo, hi;
        rope_rotate_pair(x[i], x[i + PAIR], rope.c_lo[i], rope.s_lo[i], rope.c_hi[i], rope.s_hi[i], lo, hi);
        y[i] = __float2bfloat16_rn(lo);
        y[i + PAIR] = __float2bfloat16_rn(hi);
    }
}

// Angle tables for one position, written by a group of `nthreads` threads (t = rank in the
// group): column j's cos and sin go to both halves of each table.  The values are those of
// rope_angle_cos_sin, as mllm_rope_build_cos_sin would produce them.
template <int D>
__device__ __forceinline__ void rope_angles_for_position(int64_t pos, int t, int nthreads, float log_theta,
                                                         float* cos_, float* sin_) {
    constexpr int HALF = D / 2;
    for (int j = t; j < HALF; j += nthreads) {
        float c, s;
        rope_angle_cos_sin(pos, j, D, log_theta, c, s);
        cos_[j] = c;
        cos_[j + HALF] = c;
        sin_[j] = s;
        sin_[j + HALF] = s;
    }
}

}  // namespace mllm_b200
