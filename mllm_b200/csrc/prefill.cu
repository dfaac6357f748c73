// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces src/core/runtime/Attention.h:220-316 for a block of new query rows against the KV
// cache: no repeat_interleave (each q head reads its kv head's tiles directly), no [S, total]
// fp32 score tensor in HBM (scores live in tensor memory), no materialised mask (the causal
// bound is applied per element while the scores are read out of TMEM).
//
// One CTA computes one 128-row query tile of one (sequence, query head):
//   warp 0        TMA producer: Q tile once, then K/V tiles of 128 cache rows into a
//                 2-stage shared-memory ring (128-byte swizzle, 16-byte-aligned coordinates)
//   warp 1        TMEM allocator + single-thread MMA issuer:
//                   S_j = Q K_j^T   tcgen05.mma kind::f16, M=128 N=128, fp32 into TMEM
//                                   (two S buffers, so S_{j+1} runs while softmax reads S_j)
//                   O  += P_j V_j   tcgen05.mma, A = P_j from shared memory, B = V (MN-major)
//   warps 2..5    softmax: thread r owns query row r (TMEM lane r).  Per tile it loads its
//                 S row with tcgen05.ld, applies scale and the causal bound, runs the online
//                 softmax in the exp2 domain, rescales the O row in TMEM only when its running
//                 max grew by more than 2^8 (the stale max is exact: the final 1/l uses it
//                 too), and writes P_j as bf16 into the swizzled P tile.  At the end it reads
//                 O from TMEM and writes bf16 O / l straight into [B, S, H*D].
// Numerics follow the reference: bf16 Q/K/V, fp32 scores scaled by 1/sqrt(D), fp32
// softmax, P rounded to bf16 for the P.V product, fp32 accumulation.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "host_util.h"
#include "tcgen05.cuh"

namespace mllm_b200 {
namespace {

constexpr int kBM = 128;            // query rows per CTA
constexpr int kBN = 128;            // cache rows per tile
constexpr int kThreads = 192;       // 6 warps
constexpr int kBox = kBN * 128;     // one 128-row x 64-column bf16 box (16 KB)
constexpr uint32_t kTmemCols = 512; // S0 [0,128)  S1 [128,256)  O [256, 256 + D)
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows > 2^8

template <int D>
struct PrefillCfg {
    static constexpr int kBoxes = D / 64;
    static constexpr int kQBytes = kBoxes * kBox;
    static constexpr int kKVBytes = kBoxes * kBox;     // one K (or V) tile
    static constexpr int kStages = (D == 128) ? 2 : 4;
    static constexpr int kStageBytes = 2 * kKVBytes;
    static constexpr int kPBytes = 2 * kBox;           // 128 rows x 128 bf16 columns
    static constexpr int kBarBytes = 256;
    static constexpr int kSmemBytes = kQBytes + kStages * kStageBytes + kPBytes + kBarBytes + 1024;
};

struct PrefillArgs {
    __nv_bfloat16* out;   // [B, q_len, H*D]
    int B, H, Hkv, n_rep, q_len, kv_len, n_mblocks;
    float scale_log2;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, PrefillArgs a) {
    using Cfg = PrefillCfg<D>;
    constexpr int ST = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* sKV = sQ + Cfg::kQBytes;
    uint8_t* sP = sKV + ST * Cfg::kStageBytes;
    uint64_t* bars = reinterpret_cast<uint64_t*>(sP + Cfg::kPBytes);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;
    uint64_t* kv_empty = kv_full + ST;
    uint64_t* s_full = kv_empty + ST;   // [2]
    uint64_t* s_free = s_full + 2;      // [2]
    uint64_t* p_full = s_free + 2;
    uint64_t* pv_done = p_full + 1;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const int mb = a.n_mblocks - 1 - (int)blockIdx.x;  // longest (most causal work) tiles first
    const int h = blockIdx.y;
    const int b = blockIdx.z;
    const int g = h / a.n_rep;
    const int m0 = mb * kBM;
    const int q_last = min(m0 + kBM - 1, a.q_len - 1);
    const int pos_offset = a.kv_len - a.q_len;          // absolute position of query row 0
    const int nb = (pos_offset + q_last) / kBN + 1;     // cache tiles this query tile can see

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < ST; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&s_free[i], 128);
        }
        mbar_init(p_full, 128);
        mbar_init(pv_done, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        // ------------------------------- TMA producer -------------------------------
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(q_full, Cfg::kQBytes);
#pragma unroll
            for (int bx = 0; bx < Cfg::kBoxes; ++bx) tma_load_4d(sQ + bx * kBox, &tmQ, q_full, bx * 64, m0, h, b);
            for (int j = 0; j < nb; ++j) {
                const int stage = j % ST;
                if (!mbar_wait(&kv_empty[stage], ((j / ST) & 1) ^ 1)) break;
                mbar_arrive_expect_tx(&kv_full[stage], Cfg::kStageBytes);
                uint8_t* sk = sKV + stage * Cfg::kStageBytes;
                uint8_t* sv = sk + Cfg::kKVBytes;
#pragma unroll
                for (int bx = 0; bx < Cfg::kBoxes; ++bx) {
                    tma_load_4d(sk + bx * kBox, &tmK, &kv_full[stage], bx * 64, j * kBN, g, b);
                    tma_load_4d(sv + bx * kBox, &tmV, &kv_full[stage], bx * 64, j * kBN, g, b);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_bf16_f32(kBM, kBN, false);
            constexpr uint32_t idesc_o = idesc_bf16_f32(kBM, D, true);
            const uint32_t q_addr = smem_u32(sQ);
            const uint32_t p_addr = smem_u32(sP);
            bool alive = mbar_wait(q_full, 0);
            auto issue_s = [&](int j) -> bool {
                const int stage = j % ST, sb = j & 1;
                if (!mbar_wait(&kv_full[stage], (j / ST) & 1)) return false;
                if (!mbar_wait(&s_free[sb], ((j >> 1) & 1) ^ 1)) return false;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(sKV + stage * Cfg::kStageBytes);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t off = (ks >> 2) * kBox + (ks & 3) * 32;
                    tc_mma_ss(tmem + sb * kBN, smem_desc_sw128(q_addr + off, 16, 1024),
                              smem_desc_sw128(k_addr + off, 16, 1024), idesc_s, ks > 0 ? 1u : 0u);
                }
                tc_commit(&s_full[sb]);
                return true;
            };
            if (alive) alive = issue_s(0);
            for (int j = 0; j < nb && alive; ++j) {
                if (j + 1 < nb && !issue_s(j + 1)) break;
                if (!mbar_wait(p_full, j & 1)) break;
                tc_fence_after();
                const int stage = j % ST;
                const uint32_t v_addr = smem_u32(sKV + stage * Cfg::kStageBytes + Cfg::kKVBytes);
#pragma unroll
                for (int ks = 0; ks < kBN / 16; ++ks) {
                    const uint32_t pa = p_addr + (ks >> 2) * kBox + (ks & 3) * 32;
                    tc_mma_ss(tmem + 2 * kBN, smem_desc_sw128(pa, 16, 1024),
                              smem_desc_sw128(v_addr + ks * 16 * 128, kBox, 1024), idesc_o,
                              (j > 0 || ks > 0) ? 1u : 0u);
                }
                tc_commit(pv_done);
                // release the stage only if the producer will refill it (no arrival may land
                // on this CTA's barriers after its last wait)
                if (j + ST < nb) tc_commit(&kv_empty[stage]);
            }
        }
    } else {
        // --------------------------------- softmax ---------------------------------
        const int quad = warp & 3;
        const int row = quad * 32 + lane;
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        const int p_row = pos_offset + m0 + row;  // last cache row this query may see
        float m_run = -INFINITY, l_run = 0.f;
        bool alive = true;
        for (int j = 0; j < nb; ++j) {
            const int sb = j & 1;
            if (!mbar_wait(&s_full[sb], (j >> 1) & 1)) { alive = false; break; }
            tc_fence_after();
            float s[kBN];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c)
                tmem_ld32(t_lane + sb * kBN + c * 32, *reinterpret_cast<float(*)[32]>(&s[c * 32]));
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&s_free[sb]);

            // Causal bound: only tiles reaching past the CTA's first query position need it
            // (warp-uniform test).  Reductions use 8 independent accumulators so the 128-long
            // max / sum chains do not serialise on instruction latency.
            constexpr int kAcc = 8;
            float mx[kAcc];
#pragma unroll
            for (int i = 0; i < kAcc; ++i) mx[i] = -INFINITY;
            if ((j + 1) * kBN - 1 > pos_offset + m0) {
                const int lim = p_row - j * kBN;   // columns <= lim are visible
#pragma unroll
                for (int c = 0; c < kBN; ++c) {
                    s[c] = (c <= lim) ? s[c] : -INFINITY;
                    mx[c % kAcc] = fmaxf(mx[c % kAcc], s[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < kBN; ++c) mx[c % kAcc] = fmaxf(mx[c % kAcc], s[c]);
            }
#pragma unroll
            for (int w = kAcc / 2; w >= 1; w >>= 1)
#pragma unroll
                for (int i = 0; i < w; ++i) mx[i] = fmaxf(mx[i], mx[i + w]);
            const float mt = mx[0] * a.scale_log2;   // scale > 0: max of scaled = scaled max
            const float m_new = fmaxf(m_run, mt);
            const bool grow = (m_new - m_run) > kRescaleThreshold;   // true on the first tile
            float m_use = grow ? m_new : m_run;
            if (m_use == -INFINITY) m_use = 0.f;
            const float alpha = grow ? ex2_approx(m_run - m_use) : 1.f;
            const float neg_m = -m_use;
            float sum[kAcc];
#pragma unroll
            for (int i = 0; i < kAcc; ++i) sum[i] = 0.f;
#pragma unroll
            for (int c = 0; c < kBN; ++c) {
                s[c] = ex2_approx(fmaf(s[c], a.scale_log2, neg_m));
                sum[c % kAcc] += s[c];
            }
#pragma unroll
            for (int w = kAcc / 2; w >= 1; w >>= 1)
#pragma unroll
                for (int i = 0; i < w; ++i) sum[i] += sum[i + w];
            l_run = l_run * alpha + sum[0];
            m_run = m_use;

            if (j > 0) {
                // P buffer and O are still in use by P_{j-1} V_{j-1} until it completes.
                if (!mbar_wait(pv_done, (j - 1) & 1)) { alive = false; break; }
                tc_fence_after();
                if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
                    for (int c = 0; c < D / 32; ++c) {
                        float o[32];
                        tmem_ld32(t_lane + 2 * kBN + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i) o[i] *= alpha;
                        tmem_st32(t_lane + 2 * kBN + c * 32, o);
                    }
                    tmem_wait_st();
                }
            }
            // P row -> swizzled K-major tile (two 64-column boxes)
#pragma unroll
            for (int cc = 0; cc < kBN / 8; ++cc) {
                uint4 v;
                v.x = pack_bf16x2(s[cc * 8 + 0], s[cc * 8 + 1]);
                v.y = pack_bf16x2(s[cc * 8 + 2], s[cc * 8 + 3]);
                v.z = pack_bf16x2(s[cc * 8 + 4], s[cc * 8 + 5]);
                v.w = pack_bf16x2(s[cc * 8 + 6], s[cc * 8 + 7]);
                *reinterpret_cast<uint4*>(sP + (cc >> 3) * kBox + swz128(row, cc & 7)) = v;
            }
            fence_proxy_async_smem();
            tc_fence_before();
            mbar_arrive(p_full);
        }
        if (alive && mbar_wait(pv_done, (nb - 1) & 1)) {
            tc_fence_after();
            const float inv_l = 1.f / l_run;
            const bool valid = (m0 + row) < a.q_len;
            __nv_bfloat16* orow =
                a.out + (((int64_t)b * a.q_len + (m0 + row)) * a.H + h) * (int64_t)D;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                float o[32];
                tmem_ld32(t_lane + 2 * kBN + c * 32, o);
                tmem_wait_ld();
                if (valid) {
#pragma unroll
                    for (int i = 0; i < 32; i += 8) {
                        uint4 v;
                        v.x = pack_bf16x2(o[i + 0] * inv_l, o[i + 1] * inv_l);
                        v.y = pack_bf16x2(o[i + 2] * inv_l, o[i + 3] * inv_l);
                        v.z = pack_bf16x2(o[i + 4] * inv_l, o[i + 5] * inv_l);
                        v.w = pack_bf16x2(o[i + 6] * inv_l, o[i + 7] * inv_l);
                        *reinterpret_cast<uint4*>(orow + c * 32 + i) = v;
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kTmemCols);
    }
}

}  // namespace
}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" int mllm_prefill_attention_bf16(const void* q, const void* k_cache, const void* v_cache, int64_t cache_sb,
                                           int64_t cache_sh, int64_t cache_st, int batch, int num_heads,
                                           int num_kv_heads, int head_dim, int q_len, int kv_len, float softmax_scale,
                                           void* out, mllm_stream_t stream) {
    if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || q_len < 0 || kv_len < 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: bad sizes");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128)
        return fail(MLLM_ERR_UNSUPPORTED, "prefill_attention: head_dim must be 64 or 128");
    if (kv_len < q_len) return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: kv_len < q_len");
    if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: softmax_scale must be positive");
    if (batch == 0 || q_len == 0) return ok();
    if (!q || !k_cache || !v_cache || !out) return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: null pointer");
    if (!aligned(q, 16) || !aligned(out, 16))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: q/out must be 16-byte aligned");
    if (batch > 65535 || num_heads > 65535) return fail(MLLM_ERR_UNSUPPORTED, "prefill_attention: grid too large");
    if (int st = require_sm100()) return st;

    const int64_t D = head_dim;
    CUtensorMap tmQ, tmK, tmV;
    if (int st = encode_kv_map(&tmQ, q, D, q_len, num_heads, batch, D, (int64_t)q_len * D,
                               (int64_t)num_heads * q_len * D, 64, kBM))
        return st;
    if (int st = encode_kv_map(&tmK, k_cache, D, kv_len, num_kv_heads, batch, cache_st, cache_sh, cache_sb, 64, kBN))
        return st;
    if (int st = encode_kv_map(&tmV, v_cache, D, kv_len, num_kv_heads, batch, cache_st, cache_sh, cache_sb, 64, kBN))
        return st;

    PrefillArgs a;
    a.out = (__nv_bfloat16*)out;
    a.B = batch;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.n_rep = num_heads / num_kv_heads;
    a.q_len = q_len;
    a.kv_len = kv_len;
    a.n_mblocks = (q_len + kBM - 1) / kBM;
    a.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
    dim3 grid(a.n_mblocks, num_heads, batch);
    cudaStream_t s = (cudaStream_t)stream;
    if (head_dim == 128) {
        const int smem = PrefillCfg<128>::kSmemBytes;
        if (int st = check_cuda(cudaFuncSetAttribute(prefill_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     smem),
                                "prefill smem attribute"))
            return st;
        prefill_kernel<128><<<grid, kThreads, smem, s>>>(tmQ, tmK, tmV, a);
    } else {
        const int smem = PrefillCfg<64>::kSmemBytes;
        if (int st = check_cuda(cudaFuncSetAttribute(prefill_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     smem),
                                "prefill smem attribute"))
            return st;
        prefill_kernel<64><<<grid, kThreads, smem, s>>>(tmQ, tmK, tmV, a);
    }
    if (int st = check_cuda(cudaGetLastError(), "prefill_kernel launch")) return st;
    return ok();
}
