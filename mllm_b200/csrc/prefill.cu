// Causal GQA prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
// Replaces src/core/runtime/Attention.h:220-316 for a block of new query rows against the KV
// cache: no repeat_interleave (each q head reads its kv head's tiles directly), no [S, total]
// fp32 score tensor in HBM (scores live in tensor memory), no materialised mask (the causal
// bound is applied per element while the scores are read out of TMEM).
//
// One CTA computes TWO 128-row query tiles (256 consecutive rows) of one (sequence, q head);
// both tiles share every K/V tile the CTA loads.
//   warp 0        TMA producer: both Q tiles once, then K/V tiles of 128 cache rows into a
//                 shared-memory ring (128-byte swizzle; innermost coordinates multiples of 64).
//                 K and V of a stage have their own full/empty barriers: K(j) is free once the
//                 S products of tile j are done, a whole iteration before V(j) is, so the next
//                 K tile is loaded early instead of waiting for the previous P.V
//   warp 1        TMEM allocator + single-thread MMA issuer (tcgen05.mma kind::f16, M=128):
//                   S_i   = Q_i K_j^T    A, B from shared memory, fp32 into TMEM columns S_i
//                   O_i  += P_i V_j      A = P_i from TMEM (written over S_i), B = V (MN-major)
//                 per tile j it issues PV_0(j), S_0(j+1), PV_1(j), S_1(j+1): while one softmax
//                 group works on its tile, the tensor pipe runs the other tile's products.
//                 Each product's k-steps are fully unrolled with constant descriptor offsets:
//                 one thread feeds the tensor pipe, and a rolled loop could not keep a 64-cycle
//                 128 x 128 x 16 instruction queued back to back
//   warps 4-7     softmax of query tile 0, warps 8-11 of tile 1 (warp w reaches TMEM lanes
//                 32*(w%4)..+31); they run with 216 registers each (setmaxnreg).  Thread r
//                 owns row r: it loads its 128 scores from TMEM with back-to-back loads and a
//                 single wait, takes the row max (causal bound applied
//                 per element on diagonal tiles), rescales the O row in TMEM only when the max
//                 grows by more than 2^8 (the stale max stays exact because the final 1/l uses
//                 it too), forms P = exp2(S*scale - m) in bf16 and writes it back over the
//                 consumed S columns for the next P.V.
//                 Seeing S_i(j+1) complete also proves P_i(j) V_j completed (one issuing
//                 thread, in-order tensor pipe), so O_i may be rescaled without another wait.
//                 At the end the group reads O from TMEM and writes bf16 O / l into [B,S,H*D].
// Numerics follow the reference: bf16 Q/K/V, fp32 scores scaled by 1/sqrt(D), fp32
// softmax, P rounded to bf16 for the P.V product, fp32 accumulation.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "host_util.h"
#include "kv_layout.cuh"
#include "tcgen05.cuh"

namespace mllm_b200 {
namespace {

constexpr int kBM = 128;            // query rows per tile
constexpr int kQTiles = 2;          // query tiles per CTA
constexpr int kBN = 128;            // cache rows per K/V tile
constexpr int kThreads = 384;       // 3 warpgroups: {producer, MMA, 2 idle}, softmax tile 0, tile 1
// Register split (setmaxnreg): the kernel launches at 168 registers per thread (384 x 168 =
// 64,512, three warps per SM sub-partition).  The producer/MMA warpgroup gives registers back
// and the two softmax warpgroups take them: 128 x 72 + 256 x 216 = 64,512, and per sub-partition
// 72 + 216 + 216 = 504 = 3 x 168, so the increase can always be satisfied.  72 keeps the fully
// unrolled MMA issue loops free of spills, 216 the softmax.
constexpr uint32_t kLaunchRegs = 168;
constexpr uint32_t kLowRegs = 72;
constexpr uint32_t kHighRegs = 216;
static_assert(128 * kLowRegs + 256 * kHighRegs <= kThreads * kLaunchRegs, "register split exceeds the launch");
static_assert(kLowRegs + 2 * kHighRegs <= 3 * kLaunchRegs, "register split exceeds a sub-partition");
constexpr int kBox = kBN * 128;     // one 128-row x 64-column bf16 box (16 KB)
constexpr uint32_t kTmemCols = 512; // S_0 [0,128) S_1 [128,256) O_0 [256,384) O_1 [384,512)
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows > 2^8

template <int D>
struct PrefillCfg {
    static constexpr int kBoxes = D / 64;
    static constexpr int kQBytes = kBoxes * kBox;      // one 128-row Q tile
    static constexpr int kKVBytes = kBoxes * kBox;     // one K (or V) tile
    static constexpr int kStages = (D == 128) ? 2 : 4;
    static constexpr int kStageBytes = 2 * kKVBytes;
    static constexpr int kBarBytes = 256;
    static constexpr int kSmemBytes = kQTiles * kQBytes + kStages * kStageBytes + kBarBytes + 1024;
    // q_full, k/v full/empty per stage, s_full/p_full/o_done per query tile, the TMEM slot
    static_assert((1 + 4 * kStages + 3 * kQTiles) * 8 + 4 <= kBarBytes, "barrier area too small");
};

struct PrefillArgs {
    __nv_bfloat16* out;   // [B, q_len, H*D]; packed: [total_q, H*D]
    int B, H, Hkv, n_rep, q_len, kv_len, n_mblocks;
    float scale_log2;
    KvLayout lay;         // contiguous, or the paged cache's block table
    // Packed sequences of different lengths (null: every sequence has q_len / kv_len).  Query
    // rows of sequence b are rows cu_q[b] .. cu_q[b+1]-1 of Q [H, total_q, D] and of out;
    // q_len is then the largest length the grid covers.
    const int32_t* cu_q;
    const int32_t* kv_lens;
    int total_q;
    int64_t max_rows;     // cache rows a sequence may address
    // Grid order.  0: grid (n_mblocks, H, B), each (head, sequence)'s blocks heaviest first,
    // one (head, sequence) after another, so that a sequence's K/V stays in L2 while its blocks
    // run.  1: grid (H, B, n_mblocks), the heaviest block of every (head, sequence) before any
    // lighter one (longest-first over the whole launch), for launches whose K/V fits in L2 anyway
    // and whose few waves would otherwise end on the heavy blocks of the last heads.
    int heavy_first;
};

__device__ __forceinline__ uint32_t col_s(int i) { return (uint32_t)(i * kBN); }
__device__ __forceinline__ uint32_t col_o(int i) { return (uint32_t)(2 * kBN + i * 128); }

template <int D>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, PrefillArgs a) {
    using Cfg = PrefillCfg<D>;
    constexpr int ST = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;                                  // [kQTiles][kQBytes]
    uint8_t* sKV = sQ + kQTiles * Cfg::kQBytes;          // [ST][K | V]
    uint64_t* bars = reinterpret_cast<uint64_t*>(sKV + ST * Cfg::kStageBytes);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;        // [ST] K tile landed
    uint64_t* k_empty = k_full + ST;    // [ST] S products that read the K tile are complete
    uint64_t* v_full = k_empty + ST;    // [ST] V tile landed
    uint64_t* v_empty = v_full + ST;    // [ST] P.V products that read the V tile are complete
    uint64_t* s_full = v_empty + ST;    // [2]  S_i(j) complete
    uint64_t* p_full = s_full + 2;      // [2]  P_i(j) written (128 arrivals)
    uint64_t* o_done = p_full + 2;      // [2]  last P_i V complete
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_done + 2);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // longest (most causal work) blocks first; see PrefillArgs::heavy_first for the two orders
    const int mb = a.n_mblocks - 1 - (int)(a.heavy_first ? blockIdx.z : blockIdx.x);
    const int h = a.heavy_first ? (int)blockIdx.x : (int)blockIdx.y;
    const int b = a.heavy_first ? (int)blockIdx.y : (int)blockIdx.z;
    const int g = h / a.n_rep;
    const int m0 = mb * (kQTiles * kBM);
    int q_len = a.q_len, kv_len = a.kv_len;
    if (a.cu_q != nullptr) {
        // CTA-uniform values: the whole block leaves before any barrier or TMEM allocation.
        const int r0 = a.cu_q[b], r1 = a.cu_q[b + 1];
        q_len = r1 - r0;
        kv_len = a.kv_lens[b];
        if (r0 < 0 || r1 > a.total_q || q_len < 0 || q_len > a.q_len || kv_len < q_len || kv_len > a.max_rows) {
            if (threadIdx.x == 0) record_error(kErrBadLength);
            return;
        }
        if (m0 >= q_len) return;                         // shorter than the longest sequence
    }
    const int pos_offset = kv_len - q_len;               // absolute position of query row 0
    int n_tiles[kQTiles];                                // cache tiles each query tile can see
#pragma unroll
    for (int i = 0; i < kQTiles; ++i) {
        const int r0 = m0 + i * kBM;
        n_tiles[i] = (r0 < q_len) ? (pos_offset + min(r0 + kBM - 1, q_len - 1)) / kBN + 1 : 0;
    }
    const int n_max = max(n_tiles[0], n_tiles[1]);

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int s = 0; s < ST; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_done[i], 1);
        }
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
    // Each role's code sits inside the branch that sets its register budget, so the compiler
    // allocates every region with the budget it actually runs under.
    if (warp < 4) {
      asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kLowRegs));
      if (warp == 0) {
        // ------------------------------- TMA producer -------------------------------
        if (lane == 0) {
            tma_prefetch_desc(&tmQ);
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            mbar_arrive_expect_tx(q_full, kQTiles * Cfg::kQBytes);
            // packed sequences: one map over all rows, this sequence's rows from cu_q[b].  The
            // tile loop stays rolled: unrolled, its two row coordinates spill at 72 registers.
            const int q_first = a.cu_q ? a.cu_q[b] : 0;
            const int q_bcoord = a.cu_q ? 0 : b;
#pragma unroll 1
            for (int i = 0; i < kQTiles; ++i)
#pragma unroll
                for (int bx = 0; bx < Cfg::kBoxes; ++bx)
                    tma_load_4d(sQ + i * Cfg::kQBytes + bx * kBox, &tmQ, q_full, bx * 64, q_first + m0 + i * kBM, h,
                                q_bcoord);
            for (int j = 0; j < n_max; ++j) {
                const int stage = j % ST;
                const uint32_t phase = ((j / ST) & 1) ^ 1;
                uint8_t* sk = sKV + stage * Cfg::kStageBytes;
                uint8_t* sv = sk + Cfg::kKVBytes;
                // cache rows j*kBN .. +kBN: one block of a paged cache (block_size % kBN == 0)
                int kblk, krow;
                kv_locate(a.lay, b, (int64_t)j * kBN, kblk, krow);   // a bad table entry reads block 0
                if (!mbar_wait(&k_empty[stage], phase)) break;
                mbar_arrive_expect_tx(&k_full[stage], Cfg::kKVBytes);
#pragma unroll
                for (int bx = 0; bx < Cfg::kBoxes; ++bx)
                    tma_load_4d(sk + bx * kBox, &tmK, &k_full[stage], bx * 64, krow, g, kblk);
                if (!mbar_wait(&v_empty[stage], phase)) break;
                mbar_arrive_expect_tx(&v_full[stage], Cfg::kKVBytes);
#pragma unroll
                for (int bx = 0; bx < Cfg::kBoxes; ++bx)
                    tma_load_4d(sv + bx * kBox, &tmV, &v_full[stage], bx * 64, krow, g, kblk);
            }
        }
      } else if (warp == 1) {
        // ------------------------------- MMA issuer -------------------------------
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_bf16_f32(kBM, kBN, false);
            constexpr uint32_t idesc_o = idesc_bf16_f32(kBM, D, true);
            // Descriptors differ only in their start-address field (bits 0..13, in 16-byte
            // units), so each k-step adds the byte offset >> 4 to a base descriptor.
            constexpr uint32_t desc_hi = smem_desc_hi_sw128(1024);   // every operand: 8-row groups 1 KB apart
            auto issue_s = [&](int i, int j) {
                const uint32_t qd = smem_desc_lo(smem_u32(sQ + i * Cfg::kQBytes), 16);
                const uint32_t kd = smem_desc_lo(smem_u32(sKV + (j % ST) * Cfg::kStageBytes), 16);
#pragma unroll
                for (int ks = 0; ks < D / 16; ++ks) {
                    const uint32_t off = (uint32_t)(((ks >> 2) * kBox + (ks & 3) * 32) >> 4);
                    tc_mma_ss_w(tmem + col_s(i), qd + off, kd + off, desc_hi, idesc_s, ks > 0 ? 1u : 0u);
                }
                tc_commit(&s_full[i]);
            };
            // A stage's K or V is released only if the producer will refill it (no arrival may
            // land on this CTA's barriers after its last wait).
            bool alive = mbar_wait(q_full, 0) && (n_max == 0 || mbar_wait(&k_full[0], 0));
            if (alive) {
                tc_fence_after();
                for (int i = 0; i < kQTiles; ++i)
                    if (n_tiles[i] > 0) issue_s(i, 0);
                if (ST < n_max) tc_commit(&k_empty[0]);
            }
            for (int j = 0; j < n_max && alive; ++j) {
                const int stage = j % ST;
                const uint32_t v_addr = smem_u32(sKV + stage * Cfg::kStageBytes + Cfg::kKVBytes);
                bool v_ready = false, k_next_ready = false;
                for (int i = 0; i < kQTiles && alive; ++i) {
                    if (j >= n_tiles[i]) continue;
                    if (!mbar_wait(&p_full[i], j & 1)) { alive = false; break; }
                    if (!v_ready) {
                        if (!mbar_wait(&v_full[stage], (j / ST) & 1)) { alive = false; break; }
                        v_ready = true;
                    }
                    tc_fence_after();
                    const uint32_t vd = smem_desc_lo(v_addr, kBox);
#pragma unroll
                    for (int ks = 0; ks < kBN / 16; ++ks)
                        tc_mma_ts_w(tmem + col_o(i), tmem + col_s(i) + ks * 8, vd + (uint32_t)((ks * 16 * 128) >> 4),
                                    desc_hi, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
                    if (j + 1 < n_tiles[i]) {
                        if (!k_next_ready) {
                            if (!mbar_wait(&k_full[(j + 1) % ST], ((j + 1) / ST) & 1)) { alive = false; break; }
                            tc_fence_after();
                            k_next_ready = true;
                        }
                        issue_s(i, j + 1);   // overwrites P_i(j) only after the P.V above read it
                    } else {
                        tc_commit(&o_done[i]);
                    }
                }
                if (!alive) break;
                if (j + ST < n_max) tc_commit(&v_empty[stage]);
                if (k_next_ready && j + 1 + ST < n_max) tc_commit(&k_empty[(j + 1) % ST]);
            }
        }
      }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kHighRegs));
        // --------------------------------- softmax ---------------------------------
        const int qt = (warp - 4) >> 2;          // query tile of this warp group
        const int quad = warp & 3;               // TMEM lane quadrant of this warp
        const int row = quad * 32 + lane;
        const int n = n_tiles[qt];
        const uint32_t t_lane = tmem + ((uint32_t)(quad * 32) << 16);
        const uint32_t t_s = t_lane + col_s(qt);
        const uint32_t t_o = t_lane + col_o(qt);
        const int q_row = m0 + qt * kBM + row;
        const int p_row = pos_offset + q_row;    // last cache row this query may see
        const int p_tile_min = pos_offset + m0 + qt * kBM;
        constexpr int kAcc = 8;
        float m_run = -INFINITY, l_run = 0.f;
        bool alive = true;
        for (int j = 0; j < n; ++j) {
            if (!mbar_wait(&s_full[qt], j & 1)) { alive = false; break; }
            tc_fence_after();
            float sv[kBN];
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c)
                tmem_ld32(t_s + c * 32, *reinterpret_cast<float(*)[32]>(&sv[c * 32]));
            tmem_wait_ld();
            if ((j + 1) * kBN - 1 > p_tile_min) {   // diagonal tile (warp-uniform): causal bound
                const int lim = p_row - j * kBN;     // columns <= lim are visible
#pragma unroll
                for (int c = 0; c < kBN; ++c) sv[c] = (c <= lim) ? sv[c] : -INFINITY;
            }
            // row max: 4 independent chains of three-input max (two new scores per step)
            float mx[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) mx[i] = fmaxf(sv[2 * i], sv[2 * i + 1]);
#pragma unroll
            for (int c = 8; c < kBN; c += 8)
#pragma unroll
                for (int i = 0; i < 4; ++i) mx[i] = fmax3(mx[i], sv[c + 2 * i], sv[c + 2 * i + 1]);
            mx[0] = fmax3(mx[0], mx[1], fmaxf(mx[2], mx[3]));
            const float mt = mx[0] * a.scale_log2;   // scale > 0: max of scaled = scaled max
            const float m_new = fmaxf(m_run, mt);
            const bool grow = (m_new - m_run) > kRescaleThreshold;   // true on the first tile
            float m_use = grow ? m_new : m_run;
            if (m_use == -INFINITY) m_use = 0.f;
            const float alpha = grow ? ex2_approx(m_run - m_use) : 1.f;
            if (j > 0 && __any_sync(0xffffffffu, grow)) {
                // P_i(j-1) V_{j-1} is complete (S_i(j) completed after it): rescale O in place.
#pragma unroll
                for (int c = 0; c < D / 32; ++c) {
                    float o[32];
                    tmem_ld32(t_o + c * 32, o);
                    tmem_wait_ld();
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] *= alpha;
                    tmem_st32(t_o + c * 32, o);
                }
            }
            // P = exp2(S * scale - m) in bf16, written over the consumed S columns
            // P = exp2(S * scale - m): packed fp32 pairs for the scale/subtract and the row sum
            const float neg_m = -m_use;
            float sum[kAcc];
#pragma unroll
            for (int i = 0; i < kAcc; ++i) sum[i] = 0.f;
#pragma unroll
            for (int c = 0; c < kBN / 32; ++c) {
                uint32_t pk[16];
#pragma unroll
                for (int e = 0; e < 32; e += 2) {
                    float x0, x1;
                    fma2(x0, x1, sv[c * 32 + e], sv[c * 32 + e + 1], a.scale_log2, a.scale_log2, neg_m, neg_m);
                    const float p0 = ex2_approx(x0);
                    const float p1 = ex2_approx(x1);
                    add2(sum[(e >> 1) % 4 * 2], sum[(e >> 1) % 4 * 2 + 1], p0, p1);
                    pk[e >> 1] = pack_bf16x2(p0, p1);
                }
                tmem_st16(t_s + c * 16, pk);
            }
            tmem_wait_st();
            add2(sum[0], sum[1], sum[2], sum[3]);
            add2(sum[4], sum[5], sum[6], sum[7]);
            add2(sum[0], sum[1], sum[4], sum[5]);
            l_run = l_run * alpha + (sum[0] + sum[1]);
            m_run = m_use;
            tc_fence_before();
            mbar_arrive(&p_full[qt]);
        }
        if (n > 0 && alive && mbar_wait(&o_done[qt], 0)) {
            tc_fence_after();
            const float inv_l = 1.f / l_run;
            const bool valid = q_row < q_len;
            const int64_t out_first = a.cu_q ? (int64_t)a.cu_q[b] : (int64_t)b * a.q_len;
            __nv_bfloat16* orow = a.out + ((out_first + q_row) * a.H + h) * (int64_t)D;
#pragma unroll
            for (int c = 0; c < D / 32; ++c) {
                float o[32];
                tmem_ld32(t_o + c * 32, o);
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

MLLM_DEFINE_STATUS_READER(prefill)

}  // namespace mllm_b200

using namespace mllm_b200;

namespace {

// Packed sequences of different lengths (the varlen entry points): per-sequence query row
// ranges and cache lengths in device memory, `max_rows` the cache rows one sequence may address.
struct PackedSeqs {
    const int32_t* cu_q = nullptr;
    const int32_t* kv_lens = nullptr;
    int total_q = 0;
    int64_t max_rows = 0;
};

// Shared by the contiguous and the paged entry points: the K/V maps cover map_rows rows of
// map_batch sequences (contiguous) or blocks (paged), and `lay` says which.  With `packed`,
// q_len is the longest sequence's length and kv_len is unused.
int prefill_entry(const void* q, const void* k_cache, const void* v_cache, int64_t cache_sb, int64_t cache_sh,
                  int64_t cache_st, int64_t map_rows, int64_t map_batch, const KvLayout& lay, int batch,
                  int num_heads, int num_kv_heads, int head_dim, int q_len, int kv_len, float softmax_scale,
                  void* out, mllm_stream_t stream, const PackedSeqs& packed = PackedSeqs{}) {
    const bool varlen = packed.cu_q != nullptr;
    if (varlen) kv_len = q_len;   // host-side checks below; the device checks each sequence
    if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || q_len < 0 || kv_len < 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: bad sizes");
    if (varlen && (packed.total_q < 0 || packed.kv_lens == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention_varlen: bad total_q or null kv_lens");
    if (varlen && packed.total_q > (int64_t)batch * q_len)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention_varlen: total_q exceeds batch * max_q_len");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128)
        return fail(MLLM_ERR_UNSUPPORTED, "prefill_attention: head_dim must be 64 or 128");
    if (kv_len < q_len) return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: kv_len < q_len");
    if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: softmax_scale must be positive");
    if (batch == 0 || q_len == 0 || (varlen && packed.total_q == 0)) return ok();
    if (!q || !k_cache || !v_cache || !out) return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: null pointer");
    if (!aligned(q, 16) || !aligned(out, 16))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention: q/out must be 16-byte aligned");
    if (batch > 65535 || num_heads > 65535) return fail(MLLM_ERR_UNSUPPORTED, "prefill_attention: grid too large");
    if (int st = require_sm100()) return st;

    const int64_t D = head_dim;
    CUtensorMap tmQ, tmK, tmV;
    // Q [batch, H, q_len, D], or packed Q [H, total_q, D] as one sequence of total_q rows
    const int64_t q_rows = varlen ? packed.total_q : q_len;
    const int64_t q_batch = varlen ? 1 : batch;
    if (int st = encode_kv_map(&tmQ, q, D, q_rows, num_heads, q_batch, D, q_rows * D, (int64_t)num_heads * q_rows * D,
                               64, kBM))
        return st;
    if (int st = encode_kv_map(&tmK, k_cache, D, map_rows, num_kv_heads, map_batch, cache_st, cache_sh, cache_sb, 64,
                               kBN))
        return st;
    if (int st = encode_kv_map(&tmV, v_cache, D, map_rows, num_kv_heads, map_batch, cache_st, cache_sh, cache_sb, 64,
                               kBN))
        return st;

    PrefillArgs a;
    a.lay = lay;
    a.out = (__nv_bfloat16*)out;
    a.B = batch;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.n_rep = num_heads / num_kv_heads;
    a.q_len = q_len;
    a.kv_len = kv_len;
    a.n_mblocks = (q_len + kQTiles * kBM - 1) / (kQTiles * kBM);
    a.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
    a.cu_q = packed.cu_q;
    a.kv_lens = packed.kv_lens;
    a.total_q = packed.total_q;
    a.max_rows = packed.max_rows;
    // Heavy blocks of all heads first when the launch's K/V (read by every block of a head)
    // fits in half the L2: then nothing is lost by interleaving the heads, and a launch of few
    // waves does not end on the heaviest blocks of its last heads.  Packed sequences keep the
    // per-sequence order (their K/V working sets are large and uneven).
    const double kv_bytes = 4.0 * batch * num_kv_heads * (double)kv_len * head_dim;
    a.heavy_first = (!varlen && kv_bytes <= 64.0 * (1 << 20) && a.n_mblocks <= 65535) ? 1 : 0;
    dim3 grid = a.heavy_first ? dim3(num_heads, batch, a.n_mblocks) : dim3(a.n_mblocks, num_heads, batch);
    cudaStream_t s = (cudaStream_t)stream;
    // The kernel moves registers between warpgroups with setmaxnreg; that is only safe if the
    // compiled kernel launches with the register count the split was sized for (otherwise the
    // increase could never be satisfied).  Checked once per kernel.
    auto check_regs = [](const void* fn) -> int {
        cudaFuncAttributes attr;
        if (int st = check_cuda(cudaFuncGetAttributes(&attr, fn), "prefill attributes")) return st;
        if ((uint32_t)attr.numRegs < kLaunchRegs)
            return fail(MLLM_ERR_UNSUPPORTED, "prefill_kernel compiled with fewer registers than its register split needs");
        return MLLM_OK;
    };
    static int regs_ok_128 = -1, regs_ok_64 = -1;
    if (head_dim == 128) {
        if (regs_ok_128 < 0) regs_ok_128 = check_regs((const void*)prefill_kernel<128>);
        if (regs_ok_128 != MLLM_OK) return fail(regs_ok_128, "prefill_kernel<128>: register split check failed");
    } else {
        if (regs_ok_64 < 0) regs_ok_64 = check_regs((const void*)prefill_kernel<64>);
        if (regs_ok_64 != MLLM_OK) return fail(regs_ok_64, "prefill_kernel<64>: register split check failed");
    }
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

}  // namespace

extern "C" int mllm_prefill_attention_bf16(const void* q, const void* k_cache, const void* v_cache, int64_t cache_sb,
                                           int64_t cache_sh, int64_t cache_st, int batch, int num_heads,
                                           int num_kv_heads, int head_dim, int q_len, int kv_len, float softmax_scale,
                                           void* out, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_prefill_attention_bf16");
    // the K/V maps stop at kv_len: rows past it read as zero
    return prefill_entry(q, k_cache, v_cache, cache_sb, cache_sh, cache_st, kv_len, batch, KvLayout{}, batch,
                         num_heads, num_kv_heads, head_dim, q_len, kv_len, softmax_scale, out, stream);
}

extern "C" int mllm_prefill_attention_paged_bf16(const void* q, const mllm_paged_kv* kv, int batch, int num_heads,
                                                 int num_kv_heads, int head_dim, int q_len, int kv_len,
                                                 float softmax_scale, void* out, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_prefill_attention_paged_bf16");
    KvLayout lay;
    if (int st = paged_layout(kv, kv_len, head_dim, "prefill_attention_paged", &lay)) return st;
    return prefill_entry(q, kv->k_pool, kv->v_pool, kv->block_stride, kv->head_stride, kv->row_stride,
                         kv->block_size, kv->num_blocks, lay, batch, num_heads, num_kv_heads, head_dim, q_len,
                         kv_len, softmax_scale, out, stream);
}

extern "C" int mllm_prefill_attention_varlen_bf16(const void* q, const void* k_cache, const void* v_cache,
                                                  int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                                  int64_t cache_capacity, const int32_t* cu_q_lens,
                                                  const int32_t* kv_lens, int batch, int num_heads, int num_kv_heads,
                                                  int head_dim, int total_q, int max_q_len, float softmax_scale,
                                                  void* out, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_prefill_attention_varlen_bf16");
    if (cu_q_lens == nullptr) return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention_varlen: cu_q_lens is NULL");
    if (cache_capacity <= 0 || cache_capacity > 0x7fffffffLL)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention_varlen: bad cache_capacity");
    PackedSeqs p;
    p.cu_q = cu_q_lens;
    p.kv_lens = kv_lens;
    p.total_q = total_q;
    p.max_rows = cache_capacity;
    return prefill_entry(q, k_cache, v_cache, cache_sb, cache_sh, cache_st, cache_capacity, batch, KvLayout{}, batch,
                         num_heads, num_kv_heads, head_dim, max_q_len, 0, softmax_scale, out, stream, p);
}

extern "C" int mllm_prefill_attention_varlen_paged_bf16(const void* q, const mllm_paged_kv* kv,
                                                        const int32_t* cu_q_lens, const int32_t* kv_lens, int batch,
                                                        int num_heads, int num_kv_heads, int head_dim, int total_q,
                                                        int max_q_len, float softmax_scale, void* out,
                                                        mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_prefill_attention_varlen_paged_bf16");
    if (cu_q_lens == nullptr) return fail(MLLM_ERR_INVALID_ARGUMENT, "prefill_attention_varlen: cu_q_lens is NULL");
    KvLayout lay;
    if (int st = paged_layout(kv, 0, head_dim, "prefill_attention_varlen_paged", &lay)) return st;
    PackedSeqs p;
    p.cu_q = cu_q_lens;
    p.kv_lens = kv_lens;
    p.total_q = total_q;
    p.max_rows = (int64_t)kv->max_blocks_per_seq * kv->block_size;
    return prefill_entry(q, kv->k_pool, kv->v_pool, kv->block_stride, kv->head_stride, kv->row_stride,
                         kv->block_size, kv->num_blocks, lay, batch, num_heads, num_kv_heads, head_dim, max_q_len, 0,
                         softmax_scale, out, stream, p);
}
