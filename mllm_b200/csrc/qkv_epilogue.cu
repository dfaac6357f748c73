// Fused QKV epilogue: per-head RMSNorm (Qwen3) + RoPE + KV-cache append, one kernel.
//
// Replaces, for each token (b, s):
//   TransformerBlock.h:103-107,130-134  q/k per-head RMSNorm (RMSNorm.h:27-64), fp32, cast bf16
//   Attention.h:157-177                 RoPE on q and k (RoPE.h:68-89), fp32, cast bf16
//   Attention.h:183-208                 KV append -- rows written in place (no torch::cat)
//
// Work split: one warp per (token, head), lane L holding the elements d = L + 32*i; the
// per-row arithmetic (reference reduction order, explicit rounding) is in qkv_math.cuh and is
// shared with the fused decode step.
//
// Memory: each head row is read once (D*2 bytes) and written once (q_out or the cache row).
#include <algorithm>

#include "common.cuh"
#include "host_util.h"
#include "kv_layout.cuh"
#include "qkv_math.cuh"

namespace mllm_b200 {
namespace {

struct EpilogueArgs {
    const __nv_bfloat16* q;
    const __nv_bfloat16* k;
    const __nv_bfloat16* v;
    int64_t q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh;
    int B, S, H, Hkv;
    const int64_t* positions;
    int64_t pos_sb, pos_ss;
    float log_theta;
    const float* rope_cos;
    const float* rope_sin;
    int64_t rope_row_sb, rope_row_ss;
    const __nv_bfloat16* q_gamma;
    const __nv_bfloat16* k_gamma;
    float eps;
    __nv_bfloat16* q_out;
    __nv_bfloat16* k_cache;
    __nv_bfloat16* v_cache;
    int64_t c_sb, c_sh, c_st, capacity;   // paged: block, head and row strides; rows per sequence
    KvLayout lay;                          // contiguous, or the paged cache's block table
    const int32_t* cache_start;   // NULL: uniform_start for every sequence
    int64_t uniform_start;
    // Packed sequences (null: B x S tokens): the call runs as one sequence of all tokens, and
    // cache sequence i takes tokens cu_seqlens[i] .. cu_seqlens[i+1]-1 (n_seqs sequences).
    const int32_t* cu_seqlens;
    int n_seqs;
};

// Cache sequence and row of token (b, s).  Packed: s is the token's packed index; a token outside
// the ranges cu_seqlens describes gets row -1 (recorded as a bad length, its K/V not written).
__device__ __forceinline__ int64_t cache_slot(const EpilogueArgs& a, int b, int s, int& seq) {
    if (a.cu_seqlens == nullptr) {
        seq = b;
        return (a.cache_start ? (int64_t)a.cache_start[b] : a.uniform_start) + s;
    }
    int lo = 0, hi = a.n_seqs - 1;   // the last sequence that starts at or before s
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (a.cu_seqlens[mid] <= s) lo = mid;
        else hi = mid - 1;
    }
    const int first = a.cu_seqlens[lo];
    seq = lo;
    if (first > s || s >= a.cu_seqlens[lo + 1]) return -1;
    return (a.cache_start ? (int64_t)a.cache_start[lo] : a.uniform_start) + (s - first);
}

constexpr int kWarps = 8;

// Locates head `head` (q heads first, then k, then v) of token (b, s).
struct HeadRef {
    const __nv_bfloat16* src;
    const __nv_bfloat16* gamma;
    int kind;  // 0 = q, 1 = k, 2 = v
    int h;
};

__device__ __forceinline__ HeadRef locate_head(const EpilogueArgs& a, int head, int b, int s) {
    HeadRef r;
    if (head < a.H) {
        r.kind = 0;
        r.h = head;
        r.src = a.q + b * a.q_sb + s * a.q_ss + r.h * a.q_sh;
        r.gamma = a.q_gamma;
    } else if (head < a.H + a.Hkv) {
        r.kind = 1;
        r.h = head - a.H;
        r.src = a.k + b * a.k_sb + s * a.k_ss + r.h * a.k_sh;
        r.gamma = a.k_gamma;
    } else {
        r.kind = 2;
        r.h = head - a.H - a.Hkv;
        r.src = a.v + b * a.v_sb + s * a.v_ss + r.h * a.v_sh;
        r.gamma = nullptr;
    }
    return r;
}

// HPW heads per warp.  Every warp issues the loads of all its heads before the block waits
// for the RoPE angles, so several rows per warp are in flight at once (the kernel is
// HBM-bound at prefill sizes and latency-bound at decode sizes).
template <int D, int HPW>
__global__ void __launch_bounds__(kWarps * 32, 6) qkv_epilogue_kernel(EpilogueArgs a) {
    constexpr int NI = D / 32;     // elements per lane
    __shared__ float s_cos[D];
    __shared__ float s_sin[D];
    __shared__ float s_gamma[2][D];   // q / k per-head norm weights (fp32 copies of the bf16 values)
    __shared__ int64_t s_slot;
    __shared__ int s_seq;

    pdl_trigger();   // a decode launched next may start its set-up (it waits for this grid)
    const int token = blockIdx.x;
    const int b = token / a.S;
    const int s = token - b * a.S;
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int total_heads = a.H + 2 * a.Hkv;
    const int head0 = (blockIdx.y * kWarps + (tid >> 5)) * HPW;

    float x[HPW][NI];
#pragma unroll
    for (int t = 0; t < HPW; ++t) {
        if (head0 + t < total_heads) {
            const HeadRef r = locate_head(a, head0 + t, b, s);
#pragma unroll
            for (int i = 0; i < NI; ++i) x[t][i] = __bfloat162float(r.src[lane + 32 * i]);
        }
    }

    // Everything the per-head work needs besides its own row is staged once per block, while
    // the row loads above are in flight: norm weights, the cache slot and the RoPE angles.
    if (a.q_gamma != nullptr) {
        for (int d = tid; d < D; d += blockDim.x) {
            s_gamma[0][d] = __bfloat162float(a.q_gamma[d]);
            s_gamma[1][d] = __bfloat162float(a.k_gamma[d]);
        }
    }
    if (tid == 0) {
        int seq;
        s_slot = cache_slot(a, b, s, seq);
        s_seq = seq;
    }
    // Angles for this token: from the caller's table, or computed (bit-identical to the
    // table that mllm_rope_build_cos_sin would produce for the same position).
    if (a.rope_cos != nullptr) {
        const int64_t row = (int64_t)b * a.rope_row_sb + (int64_t)s * a.rope_row_ss;
        for (int d = tid; d < D; d += blockDim.x) {
            s_cos[d] = a.rope_cos[row * D + d];
            s_sin[d] = a.rope_sin[row * D + d];
        }
    } else {
        rope_angles_for_position<D>(a.positions[(int64_t)b * a.pos_sb + (int64_t)s * a.pos_ss], tid, blockDim.x,
                                    a.log_theta, s_cos, s_sin);
    }
    __syncthreads();

    const int64_t slot = s_slot;
    const int cseq = s_seq;
#pragma unroll
    for (int t = 0; t < HPW; ++t) {
        if (head0 + t >= total_heads) break;
        const HeadRef r = locate_head(a, head0 + t, b, s);
        __nv_bfloat16 y[NI];
        if (r.kind == 2) {
#pragma unroll
            for (int i = 0; i < NI; ++i) y[i] = __float2bfloat16_rn(x[t][i]);   // exact: x came from bf16
        } else {
            // RMSNorm.h:48-63 (var = mean(x^2); x * rsqrt(var + eps) * w; cast to bf16), then
            // RoPE.h:77-88 on the pairs (d, d + D/2).
            float xv[NI];
#pragma unroll
            for (int i = 0; i < NI; ++i) xv[i] = x[t][i];
            const bool norm = r.gamma != nullptr;
            const float rr = norm ? rms_scale<D>(row_sum_squares<NI>(xv, lane), a.eps) : 1.f;
            float gl[NI];
#pragma unroll
            for (int i = 0; i < NI; ++i) gl[i] = norm ? s_gamma[r.kind][lane + 32 * i] : 0.f;
            qk_norm_rope_row<D>(xv, norm, gl, rr, rope_lane_from_tables<D>(s_cos, s_sin, lane), y);
        }
        __nv_bfloat16* dst;
        if (r.kind == 0) {
            dst = a.q_out + (((int64_t)b * a.H + r.h) * a.S + s) * D;
        } else {
            int blk, row;
            if (slot < 0 || slot >= a.capacity || !kv_locate(a.lay, cseq, slot, blk, row)) {
                if (lane == 0) record_error(kErrBadLength);
                continue;
            }
            __nv_bfloat16* base = (r.kind == 1) ? a.k_cache : a.v_cache;
            dst = base + blk * a.c_sb + r.h * a.c_sh + row * a.c_st;
        }
#pragma unroll
        for (int i = 0; i < NI; ++i) dst[lane + 32 * i] = y[i];
    }
}

// Many tokens (prefill): a quarter-warp (8 lanes) per head row, lane j holding the columns
// d = j + 8m (m < D/8).  All four of the reference's accumulators for column class j then sit
// in one lane -- P_k[j] sums x[d]^2 over d = j + 8k + 32i, i.e. m = k + 4i, in order of i -- so
// acc_j = ((P0+P1)+P2)+P3 needs no exchange; only the final sum over j = 0..7, in order, crosses
// lanes (8 shuffles inside the quarter-warp, serving four rows per warp instruction).  The
// reduction order, and every rounding step, is that of qkv_math.cuh, so the results are
// bit-identical to the warp-per-row kernel.  RoPE pairs (d, d + D/2) are m and m + D/16: the
// same lane.  A block takes kQwTokens tokens; 16 quarter-warps per token, RPQ rows each.
constexpr int kQwTokens = 2;

template <int D, int RPQ>
__global__ void __launch_bounds__(256, (D == 128 && RPQ >= 4) ? 2 : 3) qkv_epilogue_qw_kernel(EpilogueArgs a, int ntok) {
    constexpr int NE = D / 8;        // elements per lane per row
    constexpr int HM = NE / 2;       // slot m pairs with slot m + HM (distance D/2)
    constexpr int NI = D / 32;       // accumulation steps per accumulator
    constexpr int kQwPerTok = 32 / kQwTokens;
    __shared__ float s_cos[kQwTokens][D];
    __shared__ float s_sin[kQwTokens][D];
    __shared__ float s_gamma[2][D];
    __shared__ int64_t s_slot[kQwTokens];
    __shared__ int s_seq[kQwTokens];

    pdl_trigger();   // a decode launched next may start its set-up (it waits for this grid)
    const int tid = threadIdx.x;
    const int lane = tid & 31;
    const int j = lane & 7;
    const int qbase = lane & ~7;
    // the 8 lanes of this quarter-warp: the quarter-warps of a warp may take different branches
    // (a v row, a row past the last head), so the norm's exchange names only its own lanes
    const unsigned qmask = 0xFFu << qbase;
    const int qw = tid >> 3;
    const int tl = qw / kQwPerTok;          // token of this quarter-warp within the block
    const int hq = qw % kQwPerTok;          // its rows: heads hq + kQwPerTok * t
    const int token = blockIdx.x * kQwTokens + tl;
    const bool tok_ok = token < ntok;
    const int b = tok_ok ? token / a.S : 0;
    const int s = tok_ok ? token - b * a.S : 0;
    const int total_heads = a.H + 2 * a.Hkv;

    float x[RPQ][NE];
#pragma unroll
    for (int t = 0; t < RPQ; ++t) {
        const int head = hq + kQwPerTok * t;
        if (tok_ok && head < total_heads) {
            const HeadRef r = locate_head(a, head, b, s);
#pragma unroll
            for (int m = 0; m < NE; ++m) x[t][m] = __bfloat162float(r.src[j + 8 * m]);
        }
    }

    // staged once per block while the row loads are in flight
    if (a.q_gamma != nullptr) {
        for (int d = tid; d < D; d += blockDim.x) {
            s_gamma[0][d] = __bfloat162float(a.q_gamma[d]);
            s_gamma[1][d] = __bfloat162float(a.k_gamma[d]);
        }
    }
    if (tid < kQwTokens) {
        const int tk = blockIdx.x * kQwTokens + tid;
        if (tk < ntok) {
            const int bb = tk / a.S, ss = tk - bb * a.S;
            int seq;
            s_slot[tid] = cache_slot(a, bb, ss, seq);
            s_seq[tid] = seq;
        }
    }
    for (int idx = tid; idx < kQwTokens * D; idx += blockDim.x) {
        const int t2 = idx / D, col = idx - t2 * D;
        const int tk = blockIdx.x * kQwTokens + t2;
        if (tk >= ntok) continue;
        const int bb = tk / a.S, ss = tk - bb * a.S;
        if (a.rope_cos != nullptr) {
            const int64_t row = (int64_t)bb * a.rope_row_sb + (int64_t)ss * a.rope_row_ss;
            s_cos[t2][col] = a.rope_cos[row * D + col];
            s_sin[t2][col] = a.rope_sin[row * D + col];
        } else if (col < D / 2) {
            float c, sn;
            rope_angle_cos_sin(a.positions[(int64_t)bb * a.pos_sb + (int64_t)ss * a.pos_ss], col, D, a.log_theta, c,
                               sn);
            s_cos[t2][col] = c;
            s_cos[t2][col + D / 2] = c;
            s_sin[t2][col] = sn;
            s_sin[t2][col + D / 2] = sn;
        }
    }
    __syncthreads();
    if (!tok_ok) return;

    const int64_t slot = s_slot[tl];
    const int cseq = s_seq[tl];
#pragma unroll
    for (int t = 0; t < RPQ; ++t) {
        const int head = hq + kQwPerTok * t;
        if (head >= total_heads) break;
        const HeadRef r = locate_head(a, head, b, s);
        __nv_bfloat16 y[NE];
        if (r.kind == 2) {
#pragma unroll
            for (int m = 0; m < NE; ++m) y[m] = __float2bfloat16_rn(x[t][m]);   // exact: x came from bf16
        } else {
            if (r.gamma != nullptr) {
                // RMSNorm.h:48-63 in the reference's reduction order (see above)
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    float pk = 0.f;
#pragma unroll
                    for (int i = 0; i < NI; ++i) pk = __fadd_rn(pk, __fmul_rn(x[t][k + 4 * i], x[t][k + 4 * i]));
                    acc = k == 0 ? pk : __fadd_rn(acc, pk);
                }
                float total = 0.f;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) total = __fadd_rn(total, __shfl_sync(qmask, acc, qbase + jj));
                const float rr = rms_scale<D>(total, a.eps);
                const float* gw = s_gamma[r.kind];
#pragma unroll
                for (int m = 0; m < NE; ++m)
                    x[t][m] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(__fmul_rn(x[t][m], rr), gw[j + 8 * m])));
            }
            // RoPE.h:77-88 on the pairs (d, d + D/2)
#pragma unroll
            for (int m = 0; m < HM; ++m) {
                const int d = j + 8 * m;
                float lo, hi;
                rope_rotate_pair(x[t][m], x[t][m + HM], s_cos[tl][d], s_sin[tl][d], s_cos[tl][d + D / 2],
                                 s_sin[tl][d + D / 2], lo, hi);
                y[m] = __float2bfloat16_rn(lo);
                y[m + HM] = __float2bfloat16_rn(hi);
            }
        }
        __nv_bfloat16* dst;
        if (r.kind == 0) {
            dst = a.q_out + (((int64_t)b * a.H + r.h) * a.S + s) * D;
        } else {
            int blk, row;
            if (slot < 0 || slot >= a.capacity || !kv_locate(a.lay, cseq, slot, blk, row)) {
                if (j == 0) record_error(kErrBadLength);
                continue;
            }
            __nv_bfloat16* base = (r.kind == 1) ? a.k_cache : a.v_cache;
            dst = base + blk * a.c_sb + r.h * a.c_sh + row * a.c_st;
        }
#pragma unroll
        for (int m = 0; m < NE; ++m) dst[j + 8 * m] = y[m];
    }
}

// ---------------------------------------------------------------------------------------------
// Many tokens, a thread per head row: each thread brings its whole row into registers with
// 16-byte loads (D/8 of them), norms and rotates it there and writes it with 16-byte stores.
//
// One thread per row keeps the reference's reduction entirely in registers: element d of the row
// belongs to accumulator P_k[j] with j = d % 8, k = (d / 8) % 4, visited in order of d / 32, then
// acc_j = ((P0 + P1) + P2) + P3 and the total sums acc_0 .. acc_7 in order -- the order of the
// quarter-warp and warp kernels (qkv_math.cuh), with no exchange between lanes.  Every fp32 step
// is the same explicitly rounded operation (the two scaling products of the norm as one f32x2
// instruction: a product feeding a product, nothing to contract), so the outputs are
// bit-identical to theirs.
//
// A block takes kRowTokens consecutive tokens: their RoPE angles are computed once (position-
// independent factors once per block) into shared memory, then thread t takes rows t, t + 256, ...
// of the block's tokens x heads (three per thread for the Qwen3-8B geometry).  Preconditions
// (checked on the host): every row 16-byte aligned.
// ---------------------------------------------------------------------------------------------
constexpr int kRowTokens = 16;
constexpr int kRowThreads = 256;

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        f[2 * i] = __uint_as_float(w[i] << 16);
        f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
    uint4 v;
    v.x = pack_bf16x2(f[0], f[1]);
    v.y = pack_bf16x2(f[2], f[3]);
    v.z = pack_bf16x2(f[4], f[5]);
    v.w = pack_bf16x2(f[6], f[7]);
    return v;
}

// 8 consecutive fp32 from 16-byte aligned shared memory
__device__ __forceinline__ void load8f(const float* p, float (&f)[8]) {
    const float4 u = reinterpret_cast<const float4*>(p)[0];
    const float4 w = reinterpret_cast<const float4*>(p)[1];
    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
    f[4] = w.x; f[5] = w.y; f[6] = w.z; f[7] = w.w;
}

// (d0, d1) = (a0 * b0, a1 * b1), each product rounded to nearest (one f32x2 instruction)
__device__ __forceinline__ void mul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
    unsigned long long a, b, d;
    asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "f"(a0), "f"(a1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "f"(b0), "f"(b1));
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(d0), "=f"(d1) : "l"(d));
}

// both values rounded to bf16 precision (round to nearest even) and widened back, exactly as
// __bfloat162float(__float2bfloat16_rn(x)) does for each
__device__ __forceinline__ void round_bf16x2(float& x0, float& x1) {
    const uint32_t w = pack_bf16x2(x0, x1);
    x0 = __uint_as_float(w << 16);
    x1 = __uint_as_float(w & 0xffff0000u);
}

template <int D>
__global__ void __launch_bounds__(kRowThreads, 2) qkv_epilogue_row_kernel(EpilogueArgs a, int ntok) {
    constexpr int NC = D / 8;            // 16-byte chunks per row
    constexpr int AS = 2 * D + 4;        // floats per token in the angle table (cos, sin, pad)
    __shared__ __align__(16) float s_ang[kRowTokens * AS];
    __shared__ __align__(16) float s_gamma[2 * D];
    __shared__ float s_inv_freq[D / 2];

    pdl_trigger();   // a decode launched next may start its set-up (it waits for this grid)
    const int tid = threadIdx.x;
    const int th = a.H + 2 * a.Hkv;
    const int t0 = blockIdx.x * kRowTokens;
    const int nt = min(kRowTokens, ntok - t0);
    const bool norm = a.q_gamma != nullptr;
    const bool tables = a.rope_cos != nullptr;

    if (norm) {
        for (int d = tid; d < D; d += kRowThreads) {
            s_gamma[d] = __bfloat162float(a.q_gamma[d]);
            s_gamma[D + d] = __bfloat162float(a.k_gamma[d]);
        }
    }
    if (!tables) {
        for (int jc = tid; jc < D / 2; jc += kRowThreads) s_inv_freq[jc] = rope_angle(1, jc, D, a.log_theta);
    }
    __syncthreads();
    if (tables) {
        for (int idx = tid; idx < nt * D; idx += kRowThreads) {
            const int tl = idx / D, col = idx - tl * D;
            const int token = t0 + tl;
            const int b = token / a.S, s = token - b * a.S;
            const int64_t row = (int64_t)b * a.rope_row_sb + (int64_t)s * a.rope_row_ss;
            s_ang[tl * AS + col] = a.rope_cos[row * D + col];
            s_ang[tl * AS + D + col] = a.rope_sin[row * D + col];
        }
    } else {
        // rope_angle: float(pos) * inv_freq[col], then cos / sin, for the first half only (the
        // second half of a computed table equals the first)
        for (int idx = tid; idx < nt * (D / 2); idx += kRowThreads) {
            const int tl = idx / (D / 2), col = idx - tl * (D / 2);
            const int token = t0 + tl;
            const int b = token / a.S, s = token - b * a.S;
            const float angle =
                __fmul_rn((float)a.positions[(int64_t)b * a.pos_sb + (int64_t)s * a.pos_ss], s_inv_freq[col]);
            s_ang[tl * AS + col] = cosf(angle);
            s_ang[tl * AS + D + col] = sinf(angle);
        }
    }
    __syncthreads();

    const int rows = nt * th;
#pragma unroll 1
    for (int r = tid; r < rows; r += kRowThreads) {
        const int tl = r / th, head = r - tl * th;
        const int token = t0 + tl;
        const int b = token / a.S, s = token - b * a.S;
        const HeadRef hr = locate_head(a, head, b, s);
        __nv_bfloat16* dst;
        if (hr.kind == 0) {
            dst = a.q_out + (((int64_t)b * a.H + hr.h) * a.S + s) * D;
        } else {
            int seq, blk, rw;
            const int64_t slot = cache_slot(a, b, s, seq);
            if (slot < 0 || slot >= a.capacity || !kv_locate(a.lay, seq, slot, blk, rw)) {
                record_error(kErrBadLength);
                continue;
            }
            dst = (hr.kind == 1 ? a.k_cache : a.v_cache) + blk * a.c_sb + hr.h * a.c_sh + rw * a.c_st;
        }
        const uint4* src = reinterpret_cast<const uint4*>(hr.src);
        uint4* out = reinterpret_cast<uint4*>(dst);
        uint4 v[NC];
#pragma unroll
        for (int c = 0; c < NC; ++c) v[c] = src[c];
        if (hr.kind == 2) {
#pragma unroll
            for (int c = 0; c < NC; ++c) out[c] = v[c];
            continue;
        }
        float rr_scale = 1.f;
        if (norm) {
            // P_k[j] over the row's chunks c (k = c % 4) in order of c / 4
            float p[4][8];
#pragma unroll
            for (int c = 0; c < NC; ++c) {
                float x[8];
                unpack8(v[c], x);
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    const float sq = __fmul_rn(x[jj], x[jj]);
                    p[c & 3][jj] = c < 4 ? sq : __fadd_rn(p[c & 3][jj], sq);
                }
            }
            float total = 0.f;
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
                total = __fadd_rn(total, __fadd_rn(__fadd_rn(__fadd_rn(p[0][jj], p[1][jj]), p[2][jj]), p[3][jj]));
            rr_scale = rms_scale<D>(total, a.eps);
        }
        const float* gw = s_gamma + (hr.kind == 0 ? 0 : D);
        const float* cs = s_ang + tl * AS;
        const float* sn = cs + D;
        // RoPE.h:77-88 on the pairs (d, d + D/2): chunks c and c + NC/2
#pragma unroll
        for (int c = 0; c < NC / 2; ++c) {
            float xl[8], xh[8];
            unpack8(v[c], xl);
            unpack8(v[c + NC / 2], xh);
            if (norm) {
                // RMSNorm.h:48-63: x * rsqrt(var + eps) * w, cast to bf16
                float gl[8], gh[8];
                load8f(gw + 8 * c, gl);
                load8f(gw + 8 * c + D / 2, gh);
#pragma unroll
                for (int jj = 0; jj < 8; jj += 2) {
                    mul2(xl[jj], xl[jj + 1], xl[jj], xl[jj + 1], rr_scale, rr_scale);
                    mul2(xl[jj], xl[jj + 1], xl[jj], xl[jj + 1], gl[jj], gl[jj + 1]);
                    mul2(xh[jj], xh[jj + 1], xh[jj], xh[jj + 1], rr_scale, rr_scale);
                    mul2(xh[jj], xh[jj + 1], xh[jj], xh[jj + 1], gh[jj], gh[jj + 1]);
                    round_bf16x2(xl[jj], xl[jj + 1]);
                    round_bf16x2(xh[jj], xh[jj + 1]);
                }
            }
            float cl[8], sl[8], ch[8], sh[8];
            load8f(cs + 8 * c, cl);
            load8f(sn + 8 * c, sl);
            if (tables) {
                load8f(cs + 8 * c + D / 2, ch);
                load8f(sn + 8 * c + D / 2, sh);
            } else {
#pragma unroll
                for (int jj = 0; jj < 8; ++jj) {
                    ch[jj] = cl[jj];
                    sh[jj] = sl[jj];
                }
            }
            float lo[8], hi[8];
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
                rope_rotate_pair(xl[jj], xh[jj], cl[jj], sl[jj], ch[jj], sh[jj], lo[jj], hi[jj]);
            out[c] = pack8(lo);
            out[c + NC / 2] = pack8(hi);
        }
    }
}

}  // namespace

MLLM_DEFINE_STATUS_READER(epilogue)

}  // namespace mllm_b200

using namespace mllm_b200;

namespace {

// Shared by the contiguous and the paged entry point: `lay` is contiguous (cache strides per
// sequence) or paged (strides per block, capacity = rows per sequence).
int epilogue_entry(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh, const void* k, int64_t k_sb,
                   int64_t k_ss, int64_t k_sh, const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh, int batch,
                   int seq_len, int num_heads, int num_kv_heads, int head_dim, const int64_t* positions,
                   int64_t pos_sb, int64_t pos_ss, double rope_theta, const float* rope_cos, const float* rope_sin,
                   int64_t rope_row_sb, int64_t rope_row_ss, const void* q_norm_weight, const void* k_norm_weight,
                   double rms_norm_eps, void* q_out, void* k_cache, void* v_cache, int64_t cache_sb,
                   int64_t cache_sh, int64_t cache_st, int64_t cache_capacity, const KvLayout& lay,
                   const int32_t* cache_start, int64_t uniform_cache_start, mllm_stream_t stream,
                   const int32_t* cu_seqlens = nullptr, int n_seqs = 0) {
    if (batch < 0 || seq_len < 0 || num_heads <= 0 || num_kv_heads <= 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: bad sizes");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128)
        return fail(MLLM_ERR_UNSUPPORTED, "qkv_epilogue: head_dim must be 64 or 128");
    if ((q_norm_weight == nullptr) != (k_norm_weight == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: give both q/k norm weights or neither");
    if ((rope_cos == nullptr) != (rope_sin == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: give both rope tables or neither");
    if (rope_cos == nullptr && positions == nullptr)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: positions or rope tables required");
    if (rope_cos == nullptr && !(rope_theta > 0.0))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: rope_theta must be positive");
    if (batch == 0 || seq_len == 0) return ok();
    if (!q || !k || !v || !q_out || !k_cache || !v_cache)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: null pointer");
    if (cache_capacity <= 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: cache_capacity must be > 0");
    if ((int64_t)batch * seq_len > 0x7fffffffLL) return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue: too many tokens");
    if (int st = require_sm100()) return st;

    EpilogueArgs a;
    a.q = (const __nv_bfloat16*)q;
    a.k = (const __nv_bfloat16*)k;
    a.v = (const __nv_bfloat16*)v;
    a.q_sb = q_sb; a.q_ss = q_ss; a.q_sh = q_sh;
    a.k_sb = k_sb; a.k_ss = k_ss; a.k_sh = k_sh;
    a.v_sb = v_sb; a.v_ss = v_ss; a.v_sh = v_sh;
    a.B = batch; a.S = seq_len; a.H = num_heads; a.Hkv = num_kv_heads;
    a.positions = positions; a.pos_sb = pos_sb; a.pos_ss = pos_ss;
    a.log_theta = rope_cos ? 0.f : rope_log_theta(rope_theta);
    a.rope_cos = rope_cos; a.rope_sin = rope_sin;
    a.rope_row_sb = rope_row_sb; a.rope_row_ss = rope_row_ss;
    a.q_gamma = (const __nv_bfloat16*)q_norm_weight;
    a.k_gamma = (const __nv_bfloat16*)k_norm_weight;
    a.eps = (float)rms_norm_eps;  // the reference adds the double eps to a float tensor
    a.q_out = (__nv_bfloat16*)q_out;
    a.k_cache = (__nv_bfloat16*)k_cache;
    a.v_cache = (__nv_bfloat16*)v_cache;
    a.c_sb = cache_sb; a.c_sh = cache_sh; a.c_st = cache_st; a.capacity = cache_capacity;
    a.lay = lay;
    a.cache_start = cache_start;
    a.uniform_start = uniform_cache_start;
    a.cu_seqlens = cu_seqlens;
    a.n_seqs = n_seqs;

    // Many tokens (prefill): 4 heads per warp keeps 4 rows in flight per warp.  Few tokens
    // (decode): one head per warp spreads the little work over more SMs.
    const int total_heads = num_heads + 2 * num_kv_heads;
    const int64_t tokens = (int64_t)batch * seq_len;
    cudaStream_t st = (cudaStream_t)stream;
    // Many tokens, every row 16-byte aligned: a thread per head row.
    if (tokens >= 1024) {
        bool al = aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(q_out, 16) && aligned(k_cache, 16) &&
                  aligned(v_cache, 16);
        for (int64_t st8 : {q_sb, q_ss, q_sh, k_sb, k_ss, k_sh, v_sb, v_ss, v_sh, cache_sb, cache_sh, cache_st})
            al = al && (st8 % 8 == 0);
        if (al) {
            const unsigned blocks = (unsigned)((tokens + kRowTokens - 1) / kRowTokens);
            if (head_dim == 128) qkv_epilogue_row_kernel<128><<<blocks, kRowThreads, 0, st>>>(a, (int)tokens);
            else qkv_epilogue_row_kernel<64><<<blocks, kRowThreads, 0, st>>>(a, (int)tokens);
            if (int e = check_cuda(cudaGetLastError(), "qkv_epilogue launch")) return e;
            return ok();
        }
    }
    // Many tokens: the quarter-warp kernel (rows per quarter-warp = ceil(heads / 16)).
    const int rpq = (total_heads + 15) / 16;
    if (tokens >= 1024 && rpq <= 4) {
        const unsigned blocks = (unsigned)((tokens + kQwTokens - 1) / kQwTokens);
        const int nt = (int)tokens;
        auto launch = [&](auto kern) { kern<<<blocks, 256, 0, st>>>(a, nt); };
        if (head_dim == 128) {
            if (rpq == 1) launch(qkv_epilogue_qw_kernel<128, 1>);
            else if (rpq == 2) launch(qkv_epilogue_qw_kernel<128, 2>);
            else if (rpq == 3) launch(qkv_epilogue_qw_kernel<128, 3>);
            else launch(qkv_epilogue_qw_kernel<128, 4>);
        } else {
            if (rpq == 1) launch(qkv_epilogue_qw_kernel<64, 1>);
            else if (rpq == 2) launch(qkv_epilogue_qw_kernel<64, 2>);
            else if (rpq == 3) launch(qkv_epilogue_qw_kernel<64, 3>);
            else launch(qkv_epilogue_qw_kernel<64, 4>);
        }
        if (int e = check_cuda(cudaGetLastError(), "qkv_epilogue launch")) return e;
        return ok();
    }
    const int hpw = tokens >= 1024 ? 4 : 1;
    dim3 grid((unsigned)tokens, (unsigned)((total_heads + kWarps * hpw - 1) / (kWarps * hpw)));
    if (grid.y > 65535) return fail(MLLM_ERR_UNSUPPORTED, "qkv_epilogue: too many heads");
    if (head_dim == 128) {
        if (hpw == 4) qkv_epilogue_kernel<128, 4><<<grid, kWarps * 32, 0, st>>>(a);
        else qkv_epilogue_kernel<128, 1><<<grid, kWarps * 32, 0, st>>>(a);
    } else {
        if (hpw == 4) qkv_epilogue_kernel<64, 4><<<grid, kWarps * 32, 0, st>>>(a);
        else qkv_epilogue_kernel<64, 1><<<grid, kWarps * 32, 0, st>>>(a);
    }
    if (int st = check_cuda(cudaGetLastError(), "qkv_epilogue launch")) return st;
    return ok();
}

}  // namespace

extern "C" int mllm_qkv_epilogue_bf16(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                                      const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                                      const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                                      int batch, int seq_len, int num_heads, int num_kv_heads, int head_dim,
                                      const int64_t* positions, int64_t pos_sb, int64_t pos_ss, double rope_theta,
                                      const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                                      int64_t rope_row_ss, const void* q_norm_weight, const void* k_norm_weight,
                                      double rms_norm_eps, void* q_out, void* k_cache, void* v_cache,
                                      int64_t cache_sb, int64_t cache_sh, int64_t cache_st, int64_t cache_capacity,
                                      const int32_t* cache_start, int64_t uniform_cache_start,
                                      mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_qkv_epilogue_bf16");
    return epilogue_entry(q, q_sb, q_ss, q_sh, k, k_sb, k_ss, k_sh, v, v_sb, v_ss, v_sh, batch, seq_len, num_heads,
                          num_kv_heads, head_dim, positions, pos_sb, pos_ss, rope_theta, rope_cos, rope_sin,
                          rope_row_sb, rope_row_ss, q_norm_weight, k_norm_weight, rms_norm_eps, q_out, k_cache,
                          v_cache, cache_sb, cache_sh, cache_st, cache_capacity, KvLayout{}, cache_start,
                          uniform_cache_start, stream);
}

extern "C" int mllm_qkv_epilogue_paged_bf16(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                                            const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                                            const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                                            int batch, int seq_len, int num_heads, int num_kv_heads, int head_dim,
                                            const int64_t* positions, int64_t pos_sb, int64_t pos_ss,
                                            double rope_theta, const float* rope_cos, const float* rope_sin,
                                            int64_t rope_row_sb, int64_t rope_row_ss, const void* q_norm_weight,
                                            const void* k_norm_weight, double rms_norm_eps, void* q_out,
                                            const mllm_paged_kv* kv, const int32_t* cache_start,
                                            int64_t uniform_cache_start, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_qkv_epilogue_paged_bf16");
    KvLayout lay;
    if (int st = paged_layout(kv, 0, head_dim, "qkv_epilogue_paged", &lay)) return st;
    return epilogue_entry(q, q_sb, q_ss, q_sh, k, k_sb, k_ss, k_sh, v, v_sb, v_ss, v_sh, batch, seq_len, num_heads,
                          num_kv_heads, head_dim, positions, pos_sb, pos_ss, rope_theta, rope_cos, rope_sin,
                          rope_row_sb, rope_row_ss, q_norm_weight, k_norm_weight, rms_norm_eps, q_out, kv->k_pool,
                          kv->v_pool, kv->block_stride, kv->head_stride, kv->row_stride,
                          (int64_t)kv->max_blocks_per_seq * kv->block_size, lay, cache_start, uniform_cache_start,
                          stream);
}

// Packed sequences: the tokens run as one sequence (q/k/v rows `total_tokens` apart by the token
// strides, positions[t], Q out [H, total_tokens, D]); only the cache rows follow cu_seqlens.
static int varlen_checks(int total_tokens, const int64_t* positions, const int32_t* cu_seqlens, int batch) {
    if (total_tokens < 0 || batch < 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue_varlen: bad sizes");
    if (total_tokens > 0 && (batch == 0 || cu_seqlens == nullptr || positions == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "qkv_epilogue_varlen: cu_seqlens, positions and batch >= 1 required");
    return MLLM_OK;
}

extern "C" int mllm_qkv_epilogue_varlen_bf16(const void* q, int64_t q_st, int64_t q_sh, const void* k, int64_t k_st,
                                             int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh,
                                             int total_tokens, int num_heads, int num_kv_heads, int head_dim,
                                             const int64_t* positions, double rope_theta, const void* q_norm_weight,
                                             const void* k_norm_weight, double rms_norm_eps, void* q_out,
                                             void* k_cache, void* v_cache, int64_t cache_sb, int64_t cache_sh,
                                             int64_t cache_st, int64_t cache_capacity, const int32_t* cu_seqlens,
                                             int batch, const int32_t* cache_start, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_qkv_epilogue_varlen_bf16");
    if (int st = varlen_checks(total_tokens, positions, cu_seqlens, batch)) return st;
    return epilogue_entry(q, 0, q_st, q_sh, k, 0, k_st, k_sh, v, 0, v_st, v_sh, 1, total_tokens, num_heads,
                          num_kv_heads, head_dim, positions, 0, 1, rope_theta, nullptr, nullptr, 0, 0, q_norm_weight,
                          k_norm_weight, rms_norm_eps, q_out, k_cache, v_cache, cache_sb, cache_sh, cache_st,
                          cache_capacity, KvLayout{}, cache_start, 0, stream, cu_seqlens, batch);
}

extern "C" int mllm_qkv_epilogue_varlen_paged_bf16(const void* q, int64_t q_st, int64_t q_sh, const void* k,
                                                   int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
                                                   int64_t v_sh, int total_tokens, int num_heads, int num_kv_heads,
                                                   int head_dim, const int64_t* positions, double rope_theta,
                                                   const void* q_norm_weight, const void* k_norm_weight,
                                                   double rms_norm_eps, void* q_out, const mllm_paged_kv* kv,
                                                   const int32_t* cu_seqlens, int batch, const int32_t* cache_start,
                                                   mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_qkv_epilogue_varlen_paged_bf16");
    if (int st = varlen_checks(total_tokens, positions, cu_seqlens, batch)) return st;
    KvLayout lay;
    if (int st = paged_layout(kv, 0, head_dim, "qkv_epilogue_varlen_paged", &lay)) return st;
    return epilogue_entry(q, 0, q_st, q_sh, k, 0, k_st, k_sh, v, 0, v_st, v_sh, 1, total_tokens, num_heads,
                          num_kv_heads, head_dim, positions, 0, 1, rope_theta, nullptr, nullptr, 0, 0, q_norm_weight,
                          k_norm_weight, rms_norm_eps, q_out, kv->k_pool, kv->v_pool, kv->block_stride,
                          kv->head_stride, kv->row_stride, (int64_t)kv->max_blocks_per_seq * kv->block_size, lay,
                          cache_start, 0, stream, cu_seqlens, batch);
}
