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
// Many tokens: the rows of KT consecutive tokens of one sequence (a "group": KT = kStTokens, or
// kStTokensFew when few heads share the GPU) move between HBM and shared memory as TMA tensor
// boxes, and a thread per q/k row transforms them in place.
//
// A persistent block takes groups in turn.  Per group:
//   1. One thread loads the group's q, k and v rows: per tensor and 64-column half, one box of
//      {64 columns, KT tokens, all heads} (128-byte swizzle), all completing on the
//      stage's mbarrier -- six copies for the whole group at head_dim 128.
//   2. The block computes the group's RoPE angles once.
//   3. A thread per q/k row norms and rotates its row in place: a first pass sums the squares,
//      a second scales, rounds and rotates the pairs (d, d + D/2).  Row r of a box holds head
//      r / KT of token r % KT, and its 16-byte chunk c sits at chunk c ^ (r % 8) of
//      its 128 bytes, so the 32 rows a warp reads at once fall in different bank groups.
//   4. One thread stores the boxes: q to q_out ([B, H, S, D], the same box shape, rows past the
//      sequence end clipped by the TMA unit), k and v to the cache when the group's KT cache rows
//      are consecutive rows of one sequence or block.  Otherwise (a group that ends a sequence,
//      crosses a packed sequence or a cache block, or holds a refused row) the threads write the
//      group's valid cache rows with 16-byte stores.
// Three or four blocks per SM overlap one another's copies with their arithmetic.  (Two stages per
// block, the next group's copies issued before the current group is computed, measured slower:
// the second stage's shared memory leaves room for two blocks per SM only.)
//
// One thread per row keeps the reference's reduction entirely in registers: element d of the row
// belongs to accumulator P_k[j] with j = d % 8, k = (d / 8) % 4, visited in order of d / 32, then
// acc_j = ((P0 + P1) + P2) + P3 and the total sums acc_0 .. acc_7 in order -- the order of the
// quarter-warp and warp kernels (qkv_math.cuh), with no exchange between lanes.  Every fp32 step
// is the same explicitly rounded operation: products two at a time (one f32x2 multiply rounds each
// lane as the scalar multiply does), and every sum a scalar __fadd_rn / __fsub_rn, so that no
// product is contracted into its sum.  The outputs are bit-identical to the other kernels'.
// ---------------------------------------------------------------------------------------------
constexpr int kStTokens = 4;        // tokens per group
constexpr int kStTokensFew = 16;    // tokens per group when fewer than 16 q+k heads share the GPU
constexpr int kStMaxThreads = 192;   // a thread per row up to 48 q+k heads; more heads loop
constexpr int kStMinBlocks = 3;      // at least three blocks per SM: at most 113 registers a thread

// A pair of fp32 values in one 64-bit register, element 0 in the low half.
typedef unsigned long long f32x2;

__device__ __forceinline__ f32x2 f2_make(float lo, float hi) {
    f32x2 r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}
__device__ __forceinline__ void f2_split(f32x2 v, float& lo, float& hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 f2_mul(f32x2 a, f32x2 b) {
    f32x2 d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
// the two bf16 of a 32-bit word (element 0 in the low half), widened exactly
__device__ __forceinline__ f32x2 f2_from_bf16x2(uint32_t w) {
    return f2_make(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}
// both rounded to bf16 (nearest even), element 0 in the low half
__device__ __forceinline__ uint32_t f2_to_bf16x2(f32x2 v) {
    float lo, hi;
    f2_split(v, lo, hi);
    return pack_bf16x2(lo, hi);
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                             int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

// Shared memory of the TMA kernel for head dimension D, H q heads and Hkv kv heads: the boxes
// (q, k, v; per tensor one region per 64-column half, each a multiple of 1 KB), then the angles,
// gamma, inv_freq, the per-token cache rows (3 ints per token) and the mbarrier.
template <int D, int KT>
struct TmaEpiSmem {
    static constexpr int kHalves = D / 64;
    // floats per token in the angle table (cos | sin | 4 of padding): the rows a warp transforms
    // belong to four tokens, whose table reads then fall in different bank groups
    static constexpr int kAng = 2 * D + 4;
    __host__ __device__ static uint32_t region(int heads) { return ((uint32_t)KT * heads * 128 + 1023) & ~1023u; }
    __host__ __device__ static uint32_t stage_bytes(int H, int Hkv) { return kHalves * (region(H) + 2 * region(Hkv)); }
    __host__ __device__ static size_t bytes(int H, int Hkv) {
        return 1024 + (size_t)stage_bytes(H, Hkv) + (size_t)KT * kAng * 4 + 2 * D * 4 + (D / 2) * 4 + KT * 3 * 4 +
               16;
    }
};

template <int D, int KT>
__global__ void __launch_bounds__(kStMaxThreads, kStMinBlocks) qkv_epilogue_tma_kernel(
    const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
    const __grid_constant__ CUtensorMap tmV, const __grid_constant__ CUtensorMap tmQo,
    const __grid_constant__ CUtensorMap tmKc, const __grid_constant__ CUtensorMap tmVc, EpilogueArgs a) {
    using L = TmaEpiSmem<D, KT>;
    constexpr int HALVES = L::kHalves;
    constexpr int NC = D / 8;                     // 16-byte chunks per row
    extern __shared__ unsigned char tma_smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(tma_smem_raw) + 1023) &
                                                         ~uintptr_t(1023));
    const int H = a.H, Hkv = a.Hkv, qk = H + Hkv;
    const uint32_t rq = L::region(H), rkv = L::region(Hkv);
    const uint32_t stage_bytes = L::stage_bytes(H, Hkv);
    float* s_ang = reinterpret_cast<float*>(sm + stage_bytes);
    float* s_gamma = s_ang + KT * L::kAng;
    float* s_inv_freq = s_gamma + 2 * D;
    int* s_rows = reinterpret_cast<int*>(s_inv_freq + D / 2);   // [KT][3]: seq, block, row (-1: none)
    uint64_t* s_bar = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(s_rows + KT * 3) + 7) & ~uintptr_t(7));

    pdl_trigger();   // a decode launched next may start its set-up (it waits for this grid)
    const int tid = threadIdx.x;
    const int nthr = blockDim.x;
    const int groups_per_seq = (a.S + KT - 1) / KT;
    const int ngroups = a.B * groups_per_seq;
    const bool norm = a.q_gamma != nullptr;
    const bool tables = a.rope_cos != nullptr;
    // box base of tensor `ten` (0 q, 1 k, 2 v), 64-column half `x`
    auto box = [&](int ten, int x) -> unsigned char* {
        unsigned char* b = sm;
        if (ten == 0) return b + x * rq;
        b += HALVES * rq;
        if (ten == 1) return b + x * rkv;
        return b + HALVES * rkv + x * rkv;
    };
    auto group_of = [&](int g, int& b, int& s0, int& nt) {
        b = g / groups_per_seq;
        s0 = (g - b * groups_per_seq) * KT;
        nt = min(KT, a.S - s0);
    };
    // cache rows of the group's tokens (-1 block: not written, the error recorded)
    auto prep = [&](int g) {
        int b, s0, nt;
        group_of(g, b, s0, nt);
        if (tid < KT) {
            int* o = s_rows + tid * 3;
            o[0] = -1; o[1] = -1; o[2] = -1;
            if (tid < nt) {
                int seq, blk, rw;
                const int64_t slot = cache_slot(a, b, s0 + tid, seq);
                if (slot < 0 || slot >= a.capacity || !kv_locate(a.lay, seq, slot, blk, rw)) {
                    record_error(kErrBadLength);
                } else {
                    o[0] = seq; o[1] = blk; o[2] = rw;
                }
            }
        }
    };
    // one thread: the group's boxes
    auto issue = [&](int g) {
        int b, s0, nt;
        group_of(g, b, s0, nt);
        mbar_arrive_expect_tx(s_bar, (uint32_t)(KT * (H + 2 * Hkv) * D * 2));
#pragma unroll
        for (int x = 0; x < HALVES; ++x) {
            tma_load_4d(box(0, x), &tmQ, s_bar, x * 64, s0, 0, b);
            tma_load_4d(box(1, x), &tmK, s_bar, x * 64, s0, 0, b);
            tma_load_4d(box(2, x), &tmV, s_bar, x * 64, s0, 0, b);
        }
    };

    if (tid == 0) {
        tma_prefetch_desc(&tmQ);
        tma_prefetch_desc(&tmK);
        tma_prefetch_desc(&tmV);
        tma_prefetch_desc(&tmQo);
        tma_prefetch_desc(&tmKc);
        tma_prefetch_desc(&tmVc);
        mbar_init(s_bar, 1);
        mbar_fence_init();
    }
    if (norm) {
        for (int d = tid; d < D; d += nthr) {
            s_gamma[d] = __bfloat162float(a.q_gamma[d]);
            s_gamma[D + d] = __bfloat162float(a.k_gamma[d]);
        }
    }
    if (!tables) {
        for (int jc = tid; jc < D / 2; jc += nthr) s_inv_freq[jc] = rope_angle(1, jc, D, a.log_theta);
    }
    __syncthreads();   // barriers initialised

    int it = 0;
    for (int g = blockIdx.x; g < ngroups; g += gridDim.x, ++it) {
        int b, s0, nt;
        group_of(g, b, s0, nt);
        // shared memory is free once the previous group's stores have read it; then this group's
        // copies go out
        if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncthreads();
        prep(g);
        if (tid == 0) issue(g);

        // RoPE angles of this group's tokens
        if (tables) {
            for (int idx = tid; idx < nt * D; idx += nthr) {
                const int tl = idx / D, col = idx - tl * D;
                const int64_t row = (int64_t)b * a.rope_row_sb + (int64_t)(s0 + tl) * a.rope_row_ss;
                s_ang[tl * L::kAng + col] = a.rope_cos[row * D + col];
                s_ang[tl * L::kAng + D + col] = a.rope_sin[row * D + col];
            }
        } else {
            // rope_angle: float(pos) * inv_freq[col], then cos / sin, for the first half only (the
            // second half of a computed table equals the first)
            for (int idx = tid; idx < nt * (D / 2); idx += nthr) {
                const int tl = idx / (D / 2), col = idx - tl * (D / 2);
                const float angle = __fmul_rn(
                    (float)a.positions[(int64_t)b * a.pos_sb + (int64_t)(s0 + tl) * a.pos_ss], s_inv_freq[col]);
                float sn, cs;
                // one argument reduction for both; the GPU tests check that the rows equal those of
                // the warp kernel, which calls cosf and sinf (rope_angle_cos_sin)
                sincosf(angle, &sn, &cs);
                s_ang[tl * L::kAng + col] = cs;
                s_ang[tl * L::kAng + D + col] = sn;
            }
        }
        // this group's boxes landed (one thread waits; a timeout stops the whole block, its error
        // recorded), and the angles and cache rows are visible
        const bool landed = tid != 0 || mbar_wait(s_bar, it & 1);
        if (!__syncthreads_and(landed)) break;

        // a thread per q/k row, in place; rows r = head * KT + token of the q boxes, then the k boxes
        for (int r = tid; r < KT * qk; r += nthr) {
            const bool is_q = r < KT * H;
            const int rr = is_q ? r : r - KT * H;
            const int tl = rr % KT;
            if (tl >= nt) continue;
            unsigned char* base0 = box(is_q ? 0 : 1, 0);
            const uint32_t region = is_q ? rq : rkv;
            const uint32_t swz = (uint32_t)(rr & 7);
            // chunk c of the row: half c / 8, physical chunk (c % 8) ^ (row % 8)
            auto chunk = [&](int c) -> uint4* {
                return reinterpret_cast<uint4*>(base0 + (c >> 3) * region + rr * 128 + ((((uint32_t)c & 7u) ^ swz) << 4));
            };
            f32x2 rr2 = f2_make(1.f, 1.f);
            if (norm) {
                // P_k[j] over the row's chunks c (k = c % 4) in order of c / 4: the squares two
                // at a time, each accumulated with a scalar add
                float p[4][8];
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    const uint4 w = *chunk(c);
                    const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const f32x2 x = f2_from_bf16x2(ww[i]);
                        float s0q, s1q;
                        f2_split(f2_mul(x, x), s0q, s1q);
                        p[c & 3][2 * i] = c < 4 ? s0q : __fadd_rn(p[c & 3][2 * i], s0q);
                        p[c & 3][2 * i + 1] = c < 4 ? s1q : __fadd_rn(p[c & 3][2 * i + 1], s1q);
                    }
                }
                float total = 0.f;
#pragma unroll
                for (int jj = 0; jj < 8; ++jj)
                    total = __fadd_rn(total, __fadd_rn(__fadd_rn(__fadd_rn(p[0][jj], p[1][jj]), p[2][jj]), p[3][jj]));
                const float rsc = rms_scale<D>(total, a.eps);
                rr2 = f2_make(rsc, rsc);
            }
            const float* gw = s_gamma + (is_q ? 0 : D);
            const float* cs = s_ang + tl * L::kAng;
            const float* sn = cs + D;
            // 8 consecutive fp32 of a table (16-byte aligned), as four pairs
            auto pairs8 = [](const float* q, f32x2 (&o)[4]) {
                const ulonglong2 u = reinterpret_cast<const ulonglong2*>(q)[0];
                const ulonglong2 v = reinterpret_cast<const ulonglong2*>(q)[1];
                o[0] = u.x; o[1] = u.y; o[2] = v.x; o[3] = v.y;
            };
            // RoPE.h:77-88 on the pairs (d, d + D/2): chunks c and c + NC/2
#pragma unroll
            for (int c = 0; c < NC / 2; ++c) {
                uint4* pl = chunk(c);
                uint4* ph = chunk(c + NC / 2);
                const uint4 wl = *pl, wh = *ph;
                const uint32_t wwl[4] = {wl.x, wl.y, wl.z, wl.w};
                const uint32_t wwh[4] = {wh.x, wh.y, wh.z, wh.w};
                f32x2 gl[4], gh[4], cl[4], sl[4], ch[4], sh[4];
                if (norm) {
                    pairs8(gw + 8 * c, gl);
                    pairs8(gw + 8 * c + D / 2, gh);
                }
                pairs8(cs + 8 * c, cl);
                pairs8(sn + 8 * c, sl);
                if (tables) {
                    pairs8(cs + 8 * c + D / 2, ch);
                    pairs8(sn + 8 * c + D / 2, sh);
                } else {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        ch[i] = cl[i];
                        sh[i] = sl[i];
                    }
                }
                uint32_t ol[4], oh[4];
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    f32x2 xl = f2_from_bf16x2(wwl[i]);
                    f32x2 xh = f2_from_bf16x2(wwh[i]);
                    if (norm) {
                        // RMSNorm.h:48-63: x * rsqrt(var + eps) * w, cast to bf16
                        xl = f2_from_bf16x2(f2_to_bf16x2(f2_mul(f2_mul(xl, rr2), gl[i])));
                        xh = f2_from_bf16x2(f2_to_bf16x2(f2_mul(f2_mul(xh, rr2), gh[i])));
                    }
                    // out[d] = x[d]*cos[d] + (-x[d+D/2])*sin[d], out[d+D/2] = x[d+D/2]*cos[d+D/2] +
                    // x[d]*sin[d+D/2]
                    float a0, a1, b0, b1, c0, c1, d0, d1;
                    f2_split(f2_mul(xl, cl[i]), a0, a1);
                    f2_split(f2_mul(xh, sl[i]), b0, b1);
                    f2_split(f2_mul(xh, ch[i]), c0, c1);
                    f2_split(f2_mul(xl, sh[i]), d0, d1);
                    ol[i] = pack_bf16x2(__fsub_rn(a0, b0), __fsub_rn(a1, b1));
                    oh[i] = pack_bf16x2(__fadd_rn(c0, d0), __fadd_rn(c1, d1));
                }
                *pl = make_uint4(ol[0], ol[1], ol[2], ol[3]);
                *ph = make_uint4(oh[0], oh[1], oh[2], oh[3]);
            }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");   // the rows, for the TMA stores
        __syncthreads();

        // the group's cache rows: one box per half when they are KT consecutive rows of one block
        const int* crow = s_rows;
        bool boxed = nt == KT;
        for (int t = 0; t < KT && boxed; ++t)
            boxed = crow[3 * t + 1] >= 0 && crow[3 * t] == crow[0] && crow[3 * t + 1] == crow[1] &&
                    crow[3 * t + 2] == crow[2] + t;
        if (tid == 0) {
#pragma unroll
            for (int x = 0; x < HALVES; ++x) {
                tma_store_4d(&tmQo, box(0, x), x * 64, s0, 0, b);
                if (boxed) {
                    tma_store_4d(&tmKc, box(1, x), x * 64, crow[2], 0, crow[1]);
                    tma_store_4d(&tmVc, box(2, x), x * 64, crow[2], 0, crow[1]);
                }
            }
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
        if (!boxed) {
            // 16-byte stores of the valid rows: index = ((ten * Hkv + h) * KT + t) * NC + c
            const int total = 2 * Hkv * KT * NC;
            for (int i = tid; i < total; i += nthr) {
                const int c = i % NC, t = (i / NC) % KT, hrow = i / (NC * KT);   // hrow = ten * Hkv + h
                const int ten = hrow >= Hkv ? 1 : 0, h = hrow - ten * Hkv;
                if (t >= nt || crow[3 * t + 1] < 0) continue;
                const int rr = h * KT + t;
                const uint4 val = *reinterpret_cast<const uint4*>(box(1 + ten, c >> 3) + rr * 128 +
                                                                   ((((uint32_t)c & 7u) ^ (uint32_t)(rr & 7)) << 4));
                __nv_bfloat16* dst = (ten == 0 ? a.k_cache : a.v_cache) + (int64_t)crow[3 * t + 1] * a.c_sb +
                                     (int64_t)h * a.c_sh + (int64_t)crow[3 * t + 2] * a.c_st + 8 * c;
                *reinterpret_cast<uint4*>(dst) = val;
            }
        }
    }
    if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");   // smem stays until read
    __syncthreads();
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
    // Many tokens, every row 16-byte aligned: TMA boxes of a group of tokens x all heads.
    if (tokens >= 1024 && num_heads <= 256) {
        bool al = aligned(q, 16) && aligned(k, 16) && aligned(v, 16) && aligned(q_out, 16) && aligned(k_cache, 16) &&
                  aligned(v_cache, 16);
        for (int64_t st8 : {q_ss, q_sh, k_ss, k_sh, v_ss, v_sh, cache_sb, cache_sh, cache_st})
            al = al && st8 > 0 && (st8 % 8 == 0);
        for (int64_t st8 : {q_sb, k_sb, v_sb}) al = al && (batch == 1 || (st8 > 0 && st8 % 8 == 0));
        int sms = 0;
        if (int e = require_sm100(&sms)) return e;
        // tokens per group: 4 with many heads; 16 when few heads share a GPU (a tensor-parallel
        // rank's share), so that a group still gives its block several warps of rows
        const bool wide = num_heads + num_kv_heads < 16;
        const int kt_tokens = wide ? kStTokensFew : kStTokens;
        const size_t smem = head_dim == 128
            ? (wide ? TmaEpiSmem<128, kStTokensFew>::bytes(num_heads, num_kv_heads)
                    : TmaEpiSmem<128, kStTokens>::bytes(num_heads, num_kv_heads))
            : (wide ? TmaEpiSmem<64, kStTokensFew>::bytes(num_heads, num_kv_heads)
                    : TmaEpiSmem<64, kStTokens>::bytes(num_heads, num_kv_heads));
        const int64_t cache_rows = lay.table ? lay.block_size : cache_capacity;
        if (al && smem <= 200 * 1024 && seq_len >= kt_tokens && cache_rows >= kt_tokens) {
            // tensor maps {D, rows, heads, batch}: q/k/v by token (batch stride arbitrary for B = 1),
            // q_out [B, H, S, D], the cache by (sequence or block, kv head, row)
            const int64_t S = seq_len, D = head_dim;
            auto bstride = [&](int64_t sb, int64_t ss) { return batch == 1 ? S * ss : sb; };
            const int64_t cache_batch = lay.table ? lay.num_blocks : (cu_seqlens ? n_seqs : batch);
            CUtensorMap mq, mk, mv, mqo, mkc, mvc;
            const uint32_t kt = (uint32_t)kt_tokens;
            if (int e = encode_kv_map(&mq, q, D, S, num_heads, batch, q_ss, q_sh, bstride(q_sb, q_ss), 64, kt,
                                      (uint32_t)num_heads))
                return e;
            if (int e = encode_kv_map(&mk, k, D, S, num_kv_heads, batch, k_ss, k_sh, bstride(k_sb, k_ss), 64, kt,
                                      (uint32_t)num_kv_heads))
                return e;
            if (int e = encode_kv_map(&mv, v, D, S, num_kv_heads, batch, v_ss, v_sh, bstride(v_sb, v_ss), 64, kt,
                                      (uint32_t)num_kv_heads))
                return e;
            if (int e = encode_kv_map(&mqo, q_out, D, S, num_heads, batch, D, S * D, (int64_t)num_heads * S * D, 64,
                                      kt, (uint32_t)num_heads))
                return e;
            if (int e = encode_kv_map(&mkc, k_cache, D, cache_rows, num_kv_heads, cache_batch, cache_st, cache_sh,
                                      cache_sb, 64, kt, (uint32_t)num_kv_heads))
                return e;
            if (int e = encode_kv_map(&mvc, v_cache, D, cache_rows, num_kv_heads, cache_batch, cache_st, cache_sh,
                                      cache_sb, 64, kt, (uint32_t)num_kv_heads))
                return e;
            const int threads = std::min(kStMaxThreads, (kt_tokens * (num_heads + num_kv_heads) + 31) / 32 * 32);
            const int64_t groups = (int64_t)batch * ((seq_len + kt_tokens - 1) / kt_tokens);
            auto launch = [&](auto kern) {
                if (int e = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                            (int)smem),
                                       "qkv_epilogue smem"))
                    return e;
                // persistent: as many blocks as fit on the GPU at once (registers and shared memory),
                // queried once per device, head dimension, group size, block size and shared-memory size
                struct Fit { int dev = -1, d = 0, kt = 0, threads = 0; size_t smem = 0; int per_sm = 0; };
                static thread_local Fit fits[8];
                int dev = 0;
                if (int e = check_cuda(cudaGetDevice(&dev), "qkv_epilogue device")) return e;
                int per_sm = 0;
                for (const Fit& f : fits)
                    if (f.dev == dev && f.d == head_dim && f.kt == kt_tokens && f.threads == threads && f.smem == smem)
                        per_sm = f.per_sm;
                if (per_sm == 0) {
                    if (int e = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, threads, smem),
                                           "qkv_epilogue occupancy"))
                        return e;
                    static thread_local int next = 0;
                    fits[next] = Fit{dev, head_dim, kt_tokens, threads, smem, per_sm};
                    next = (next + 1) % 8;
                }
                const unsigned blocks = (unsigned)std::min<int64_t>(groups, (int64_t)sms * std::max(per_sm, 1));
                kern<<<blocks, threads, smem, st>>>(mq, mk, mv, mqo, mkc, mvc, a);
                return check_cuda(cudaGetLastError(), "qkv_epilogue launch");
            };
            const int e = head_dim == 128 ? (wide ? launch(qkv_epilogue_tma_kernel<128, kStTokensFew>)
                                                  : launch(qkv_epilogue_tma_kernel<128, kStTokens>))
                                          : (wide ? launch(qkv_epilogue_tma_kernel<64, kStTokensFew>)
                                                  : launch(qkv_epilogue_tma_kernel<64, kStTokens>));
            if (e) return e;
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
