// Split-K flash-decode over the bf16 KV cache (one new query token per sequence).
//
// Replaces src/core/runtime/Attention.h:183-316 at S == 1: instead of torch::cat-ing the
// cache, repeat_interleave-ing it n_rep times and upcasting it to fp32, each KV-head row is
// streamed from HBM exactly once and shared by its whole GQA group of query heads.
//
// Structure (per CTA, persistent over a list of work items):
//   work item  = (sequence b, kv head g, chunk c of CH cache rows); a CTA's first item is its
//                block index, later ones come from a counter in the workspace (the CTAs that
//                run fastest take more items, so they all finish together); the producer lane
//                claims them one item ahead and publishes the CTA's sequence in shared memory
//   warp 4     = producer: one elected lane issues TMA tile loads (64 rows x head_dim of K
//                and of V, 128-byte swizzled) into an NSTAGE ring guarded by mbarriers
//   warps 0-3  = consumers: each owns 16 of the 64 rows of every tile.
//                S = Q K^T   with mma.sync m16n8k16 (A = the n_rep <= 8 query heads of the
//                            group as MMA rows, B = K rows via ldmatrix), fp32 accumulate
//                online softmax in registers (exp2 domain, running max / sum per head)
//                O += P V    (A = P rounded to bf16, B = V via ldmatrix.trans)
//   item end   : the four warps' (m, l, O) are merged through shared memory; a sequence
//                covered by one chunk writes bf16 O / l directly, otherwise the chunk's
//                unnormalised partial goes to the workspace and decode_combine_kernel
//                merges the chunks.
// The tensor-core MMAs only keep the instruction count far below the memory time: the
// kernel is bound by HBM bandwidth (2 * head_dim * 2 bytes per cached row per kv head).
//
// Rows past a sequence's length inside its last tile are masked to -inf in S and zeroed in
// the V tile (the cache beyond the length may hold any bit pattern).
//
// Fused decode step (kFused, mllm_decode_step_bf16): the QKV epilogue of the new token runs
// inside the split kernel instead of as a launch of its own.  A sixth warp does it: for each
// work item it computes QK-RMSNorm + RoPE of the group's query rows (angles and norm weights in
// registers, each lane evaluating only the columns it holds) into a shared-memory slot that
// the consumers pick up when they reach the item; it can run a whole item ahead.  Doing this
// in the consumers put it on the critical path of every item boundary, and doing it in the
// TMA producer let the stage ring drain -- with equal items every CTA reaches its boundaries
// at the same moments, so either idled HBM.  The item that owns a sequence's
// last chunk also computes the new token's K (norm + RoPE) and V rows, writes them to cache
// row L-1, and leaves the V row and the row's scores for the consumers' merge, which folds the
// row into the softmax; every item's TMA range stops before row L-1, so no CTA of the launch
// reads a row the launch is writing.  The row arithmetic is qkv_math.cuh's, so the cache rows
// are bit-identical to the epilogue kernel's.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "host_util.h"
#include "kv_layout.cuh"
#include "qkv_math.cuh"

namespace mllm_b200 {
namespace {

constexpr int kTile = 64;         // cache rows per pipeline stage
constexpr int kConsumerWarps = 4;
constexpr int kThreads = (kConsumerWarps + 1) * 32;   // consumers + TMA producer
constexpr int kThreadsFused = kThreads + 32;          // + the fused step's epilogue warp
constexpr int kMaxGroup = 8;      // query heads per kv head handled as MMA rows
constexpr int kBoxBytes = kTile * 128;  // one 64-row x 64-column bf16 TMA box
constexpr int kRing = 8;          // entries of a CTA's published item sequence

template <int D>
struct DecodeCfg {
    static constexpr int kBoxes = D / 64;                 // TMA boxes per tile row-block
    static constexpr int kTileBytes = kTile * D * 2;      // K (or V) bytes per stage
    static constexpr int kStages = (D == 128) ? 3 : 6;
    static constexpr int kStageBytes = 2 * kTileBytes;
    static constexpr int kRedFloats = (kConsumerWarps - 1) * kMaxGroup * D;
    static constexpr int kSmemBytes =
        kStages * kStageBytes + kRedFloats * 4 + 2 * kConsumerWarps * kMaxGroup * 4 + 2 * kStages * 8 + 1024;
    // fused step: the transformed q rows of the next item (one slot), the new V row and the new
    // row's scores (two slots, by active-item parity) and four barriers
    static constexpr int kFusedBytes = kMaxGroup * D * 2 + 2 * D * 2 + 2 * kMaxGroup * 4 + 4 * 8;
    static constexpr int kSmemBytesFused = kSmemBytes + kFusedBytes;
    static_assert(2 * (kSmemBytesFused + 1024) <= 233472, "two CTAs per SM no longer fit");
};

struct DecodeArgs {
    const __nv_bfloat16* q;     // [B, H, D]
    const int32_t* kv_lens;     // [B], or NULL: every sequence has max_len rows
    __nv_bfloat16* out;         // [B, H*D]
    float* part_o;              // [B*Hkv*nch, n_rep, D]
    float* part_ml;             // [B*Hkv*nch, n_rep, 2]
    unsigned* item_counter;     // items handed out past the first grid-size ones (zero between calls),
                                // or NULL: the static strided schedule
    int B, H, Hkv, n_rep, max_len, chunk, nch, items;
    float scale_log2;
    KvLayout lay;                // contiguous, or the paged cache's block table
    // fused step only: the new token's projections, RoPE, norm weights and the cache to append to
    const __nv_bfloat16* q_in;   // q head h of sequence b at q_in + b*q_sb + h*q_sh
    const __nv_bfloat16* k_in;
    const __nv_bfloat16* v_in;
    int64_t q_sb, q_sh, k_sb, k_sh, v_sb, v_sh;
    const int64_t* positions;    // positions[b * pos_sb] (when no table is given)
    int64_t pos_sb;
    float log_theta;
    const float* rope_cos;       // optional [rows, D] tables, row b * rope_row_sb
    const float* rope_sin;
    int64_t rope_row_sb;
    const __nv_bfloat16* q_gamma;   // optional per-head QK-RMSNorm weights [D]
    const __nv_bfloat16* k_gamma;
    float eps;
    __nv_bfloat16* k_cache;
    __nv_bfloat16* v_cache;
    int64_t c_sb, c_sh, c_st;    // per sequence (contiguous) or per block (paged)
};

template <int D, bool kFused>
__global__ void __launch_bounds__(kFused ? kThreadsFused : kThreads, 2)
    decode_split_kernel(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                        DecodeArgs a) {
    using Cfg = DecodeCfg<D>;
    constexpr int NS = Cfg::kStages;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    float* red_o = reinterpret_cast<float*>(smem + NS * Cfg::kStageBytes);
    float* red_m = red_o + Cfg::kRedFloats;
    float* red_l = red_m + kConsumerWarps * kMaxGroup;
    uint64_t* full = reinterpret_cast<uint64_t*>(red_l + kConsumerWarps * kMaxGroup);
    uint64_t* empty = full + NS;
    // fused step only
    uint64_t* f_qfull = empty + NS;      // the next item's q rows (and new-row data) are ready
    uint64_t* f_qfree = f_qfull + 1;     // every consumer warp has loaded its q fragments
    uint64_t* f_vsfree = f_qfree + 1;    // [2] the merge has used slot p's new-row data
    float* f_snew = reinterpret_cast<float*>(f_vsfree + 2);                        // [2][kMaxGroup]
    __nv_bfloat16* f_q = reinterpret_cast<__nv_bfloat16*>(f_snew + 2 * kMaxGroup);  // [kMaxGroup][D]
    __nv_bfloat16* f_vnew = f_q + kMaxGroup * D;                                     // [2][D]

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // The CTA's item sequence: entry k at slot k % kRing, valid once s_pub[slot] == k.  The
    // producer lane writes it; the consumers report the entry they work on in s_cons.
    __shared__ int s_items[kRing];
    __shared__ int s_pub[kRing];
    __shared__ int s_cons;

    if (threadIdx.x == 0) {
        for (int i = 0; i < kRing; ++i) s_pub[i] = -1;
        s_items[0] = blockIdx.x;
        s_pub[0] = 0;
        s_cons = 0;
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        if constexpr (kFused) {
            mbar_init(f_qfull, 1);
            mbar_init(f_qfree, kConsumerWarps);
            mbar_init(&f_vsfree[0], 1);
            mbar_init(&f_vsfree[1], 1);
        }
        mbar_fence_init();
    }
    __syncthreads();
    pdl_wait();      // q and the cache rows may come from the kernel launched just before
    pdl_trigger();   // the combine kernel may start launching (it waits for this grid)

    auto item_range = [&](int item, int& b, int& g, int& c, int& t0, int& t1, int& L) {
        c = item % a.nch;
        const int bg = item / a.nch;
        g = bg % a.Hkv;
        b = bg / a.Hkv;
        int len = a.kv_lens ? a.kv_lens[b] : a.max_len;
        if (len < (kFused ? 1 : 0) || len > a.max_len) {
            if (threadIdx.x == 0 && c == 0 && g == 0) record_error(kErrBadLength);
            len = len < 1 ? 0 : a.max_len;
        }
        L = len;
        t0 = c * a.chunk;
        // the fused step's new row L-1 is not loaded: its item takes it from shared memory
        t1 = min(t0 + a.chunk, kFused ? L - 1 : L);
    };
    // Entry k of the CTA's item sequence, once the producer lane has published it (bounded).
    auto item_at = [&](int k) -> int {
        const int slot = k & (kRing - 1);
        for (uint32_t i = 0; i < kSpinLimit; ++i) {
            if (*reinterpret_cast<volatile int*>(&s_pub[slot]) == k) {
                __threadfence_block();
                return *reinterpret_cast<volatile int*>(&s_items[slot]);
            }
            if (i > 64) __nanosleep(64);
        }
        record_error(kErrTimeout);
        return INT_MAX;   // ends the caller's loop
    };

    if (kFused && warp == kConsumerWarps + 1) {
        // --------------------- the new token's epilogue (whole warp) ---------------------
        constexpr int NI = D / 32;
        const bool norm = a.q_gamma != nullptr;
        float gq[NI], gk[NI];   // norm weights at this lane's columns d = lane + 32 i
#pragma unroll
        for (int i = 0; i < NI; ++i) {
            gq[i] = norm ? __bfloat162float(a.q_gamma[lane + 32 * i]) : 0.f;
            gk[i] = norm ? __bfloat162float(a.k_gamma[lane + 32 * i]) : 0.f;
        }
        int n_act = 0;   // active items so far (items with tiles or with the new row)
        for (int k = 0;; ++k) {
            const int item = item_at(k);
            if (item >= a.items) break;
            int b, g, c, t0, t1, L;
            item_range(item, b, g, c, t0, t1, L);
            const int nch_b = (L + a.chunk - 1) / a.chunk;
            const bool last = c == nch_b - 1;
            if (t1 <= t0 && !last) continue;   // nothing to load, no new row: the consumers skip it too
            const int p = n_act & 1;
            if (n_act >= 1 && !mbar_wait(f_qfree, (n_act - 1) & 1)) break;
            if (n_act >= 2 && !mbar_wait(&f_vsfree[p], ((n_act - 2) >> 1) & 1)) break;
            // every row's loads go out first (q rows, and the new K/V rows for the last chunk),
            // so the item costs one memory round trip; the angles are computed meanwhile
            __nv_bfloat16 rq[kMaxGroup][NI], rk[NI], rv[NI];   // indices fixed after unrolling
#pragma unroll
            for (int r = 0; r < kMaxGroup; ++r) {
                if (r < a.n_rep) {
                    const __nv_bfloat16* src = a.q_in + (int64_t)b * a.q_sb + (int64_t)(g * a.n_rep + r) * a.q_sh;
#pragma unroll
                    for (int i = 0; i < NI; ++i) rq[r][i] = src[lane + 32 * i];
                }
            }
            if (last) {
                const __nv_bfloat16* ksrc = a.k_in + (int64_t)b * a.k_sb + (int64_t)g * a.k_sh;
                const __nv_bfloat16* vsrc = a.v_in + (int64_t)b * a.v_sb + (int64_t)g * a.v_sh;
#pragma unroll
                for (int i = 0; i < NI; ++i) {
                    rk[i] = ksrc[lane + 32 * i];
                    rv[i] = vsrc[lane + 32 * i];
                }
            }
            const RopeLane<D> rope = a.rope_cos != nullptr
                ? rope_lane_from_tables<D>(a.rope_cos + (int64_t)b * a.rope_row_sb * D,
                                           a.rope_sin + (int64_t)b * a.rope_row_sb * D, lane)
                : rope_lane_compute<D>(a.positions[(int64_t)b * a.pos_sb], lane, a.log_theta);
            __nv_bfloat16 yk[NI];
            if (last) {
                // the new K row (norm + RoPE) and V row, appended to cache row L-1
                float xk[NI];
#pragma unroll
                for (int i = 0; i < NI; ++i) xk[i] = __bfloat162float(rk[i]);
                const float rr = norm ? rms_scale<D>(row_sum_squares<NI>(xk, lane), a.eps) : 1.f;
                qk_norm_rope_row<D>(xk, norm, gk, rr, rope, yk);
                int blk, row;
                const bool at = kv_locate(a.lay, b, L - 1, blk, row);
                const int64_t crow = (int64_t)blk * a.c_sb + (int64_t)g * a.c_sh + (int64_t)row * a.c_st;
#pragma unroll
                for (int i = 0; i < NI; ++i) {
                    const __nv_bfloat16 yv = rv[i];
                    if (at) {
                        a.k_cache[crow + lane + 32 * i] = yk[i];
                        a.v_cache[crow + lane + 32 * i] = yv;
                    }
                    f_vnew[p * D + lane + 32 * i] = yv;
                }
            }
#pragma unroll
            for (int r = 0; r < kMaxGroup; ++r) {
                if (r >= a.n_rep) break;
                float xq[NI];
#pragma unroll
                for (int i = 0; i < NI; ++i) xq[i] = __bfloat162float(rq[r][i]);
                const float rr = norm ? rms_scale<D>(row_sum_squares<NI>(xq, lane), a.eps) : 1.f;
                __nv_bfloat16 yq[NI];
                qk_norm_rope_row<D>(xq, norm, gq, rr, rope, yq);
#pragma unroll
                for (int i = 0; i < NI; ++i) f_q[r * D + lane + 32 * i] = yq[i];
                if (last) {
                    // the new row's score for this head, fp32 over the bf16 rows: lanes sum
                    // their columns in order, then a butterfly over the warp
                    float acc = 0.f;
#pragma unroll
                    for (int i = 0; i < NI; ++i) acc = fmaf(__bfloat162float(yq[i]), __bfloat162float(yk[i]), acc);
#pragma unroll
                    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
                    if (lane == 0) f_snew[p * kMaxGroup + r] = acc * a.scale_log2;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(f_qfull);
            ++n_act;
        }
        return;
    }
    if (warp == kConsumerWarps) {
        // ------------------------------ producer ------------------------------
        if (lane == 0) {
            tma_prefetch_desc(&tmK);
            tma_prefetch_desc(&tmV);
            int stage = 0;
            uint32_t phase = 0;
            bool alive = true;
            for (int k = 0; alive; ++k) {
                const int item = *reinterpret_cast<volatile int*>(&s_items[k & (kRing - 1)]);   // published by this lane
                if (item >= a.items) break;
                // claim and publish entry k + 1 now, one item ahead of the other warps; never
                // more than kRing - 2 entries ahead of the consumers, whose entry's slot is live
                for (uint32_t i = 0; k + 1 - *reinterpret_cast<volatile int*>(&s_cons) > kRing - 2; ++i) {
                    if (i >= kSpinLimit) { record_error(kErrTimeout); alive = false; break; }
                    if (i > 64) __nanosleep(64);
                }
                if (!alive) break;
                const int nxt = a.item_counter ? (int)gridDim.x + (int)atomicAdd(a.item_counter, 1u)
                                               : item + (int)gridDim.x;
                s_items[(k + 1) & (kRing - 1)] = nxt < a.items ? nxt : a.items;
                __threadfence_block();
                *reinterpret_cast<volatile int*>(&s_pub[(k + 1) & (kRing - 1)]) = k + 1;
                int b, g, c, t0, t1, L;
                item_range(item, b, g, c, t0, t1, L);
                for (int t = t0; t < t1; t += kTile) {
                    if (!mbar_wait(&empty[stage], phase ^ 1)) { alive = false; break; }
                    mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
                    uint8_t* kdst = smem + stage * Cfg::kStageBytes;
                    uint8_t* vdst = kdst + Cfg::kTileBytes;
                    int blk, row;
                    kv_locate(a.lay, b, t, blk, row);   // a bad table entry reads block 0 (and is recorded)
#pragma unroll
                    for (int bx = 0; bx < Cfg::kBoxes; ++bx) {
                        tma_load_4d(kdst + bx * kBoxBytes, &tmK, &full[stage], bx * 64, row, g, blk);
                        tma_load_4d(vdst + bx * kBoxBytes, &tmV, &full[stage], bx * 64, row, g, blk);
                    }
                    if (++stage == NS) { stage = 0; phase ^= 1; }
                }
            }
        }
        return;
    }

    // -------------------------------- consumers --------------------------------
    const int grp = lane >> 2;   // MMA row = query head within the group
    const int tig = lane & 3;    // thread in group
    int stage = 0;
    uint32_t phase = 0;
    constexpr int KS = D / 16;   // k-steps of S = Q K^T
    constexpr int NB = D / 8;    // n-blocks of O
    bool alive = true;
    int n_act = 0;               // fused: active items so far (matches the producer's count)

    for (int k = 0; alive; ++k) {
        if (threadIdx.x == 0) *reinterpret_cast<volatile int*>(&s_cons) = k;
        const int item = item_at(k);
        if (item >= a.items) break;
        int b, g, c, t0, t1, L;
        item_range(item, b, g, c, t0, t1, L);
        const int nch_b = (L + a.chunk - 1) / a.chunk;
        // the fused step's last chunk owns the new row, even when no cached row is left for it
        const bool last = kFused && c == nch_b - 1;
        if (t1 <= t0 && !last) {
            if (L == 0 && c == 0) {  // empty sequence: the reference would produce no row; emit zeros
                for (int i = threadIdx.x; i < a.n_rep * D; i += kConsumerWarps * 32)
                    a.out[(int64_t)b * a.H * D + (int64_t)g * a.n_rep * D + i] = __float2bfloat16_rn(0.f);
            }
            continue;
        }
        const bool row_ok = grp < a.n_rep;

        // Q fragments (A operand): rows = heads of the group, cols = head_dim.
        uint32_t qa[KS][2];
        const __nv_bfloat16* qrow;
        const int slot = n_act & 1;   // fused: this item's new-row data slot
        if constexpr (kFused) {
            // the producer warp computed this item's q rows (and new-row data) into the slot
            if (!mbar_wait(f_qfull, n_act & 1)) { alive = false; break; }
            qrow = f_q + (row_ok ? grp : 0) * D;
        } else {
            qrow = a.q + ((int64_t)b * a.H + (int64_t)g * a.n_rep + (row_ok ? grp : 0)) * D;
        }
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const uint32_t lo = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + tig * 2);
            const uint32_t hi = *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + tig * 2 + 8);
            qa[ks][0] = row_ok ? lo : 0u;
            qa[ks][1] = row_ok ? hi : 0u;
        }
        if constexpr (kFused) {
            __syncwarp();
            if (lane == 0) mbar_arrive(f_qfree);
            ++n_act;
        }
        float o[NB][4];
#pragma unroll
        for (int j = 0; j < NB; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        float m_run = -INFINITY, l_run = 0.f;

        for (int t = t0; t < t1; t += kTile) {
            if (!mbar_wait(&full[stage], phase)) { alive = false; break; }
            uint8_t* kst = smem + stage * Cfg::kStageBytes;
            uint8_t* vst = kst + Cfg::kTileBytes;
            const uint32_t kbase = smem_u32(kst);
            const uint32_t vbase = smem_u32(vst);
            const int row0 = warp * 16;  // this warp's rows within the tile

            // ---- S = Q K^T over this warp's 16 rows (two n-blocks of 8 rows) ----
            float sacc[2][4];
#pragma unroll
            for (int nb = 0; nb < 2; ++nb) sacc[nb][0] = sacc[nb][1] = sacc[nb][2] = sacc[nb][3] = 0.f;
            {
                const int mi = lane >> 3, ri = lane & 7;
                const int row = row0 + 8 * (mi >> 1) + ri;
#pragma unroll
                for (int ks = 0; ks < KS; ++ks) {
                    const int cc = 2 * ks + (mi & 1);       // 16-byte chunk along head_dim
                    const uint32_t addr = kbase + (cc >> 3) * kBoxBytes + swz128(row, cc & 7);
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4(addr, r0, r1, r2, r3);
                    mma_bf16_16816(sacc[0], qa[ks][0], 0u, qa[ks][1], 0u, r0, r1);
                    mma_bf16_16816(sacc[1], qa[ks][0], 0u, qa[ks][1], 0u, r2, r3);
                }
            }

            // ---- mask, online softmax (rows = heads; this thread: head grp, 4 rows) ----
            const int valid_rows = t1 - t;  // rows of this tile inside the sequence chunk
            float s[4];
            float mt = -INFINITY;
#pragma unroll
            for (int nb = 0; nb < 2; ++nb) {
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int r = row0 + nb * 8 + tig * 2 + e;
                    const float v = (r < valid_rows) ? sacc[nb][e] * a.scale_log2 : -INFINITY;
                    s[nb * 2 + e] = v;
                    mt = fmaxf(mt, v);
                }
            }
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 1));
            mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, 2));
            const float m_new = fmaxf(m_run, mt);
            const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
            const float alpha = ex2_approx(m_run - m_use);
            float p[4];
            float psum = 0.f;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                p[i] = ex2_approx(s[i] - m_use);
                psum += p[i];
            }
            l_run = l_run * alpha + psum;
            m_run = m_new;
#pragma unroll
            for (int j = 0; j < NB; ++j) {
                o[j][0] *= alpha;
                o[j][1] *= alpha;
            }
            const uint32_t pa0 = pack_bf16x2(p[0], p[1]);
            const uint32_t pa2 = pack_bf16x2(p[2], p[3]);

            // ---- rows past the sequence end: zero this warp's V rows (any bit pattern may sit there)
            if (valid_rows < row0 + 16) {
                for (int i = lane; i < 16 * (D / 8); i += 32) {
                    const int r = row0 + i / (D / 8);
                    const int cc = i % (D / 8);
                    if (r >= valid_rows)
                        *reinterpret_cast<uint4*>(vst + (cc >> 3) * kBoxBytes + r * 128 + (cc & 7) * 16) =
                            make_uint4(0u, 0u, 0u, 0u);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }

            // ---- O += P V ----
            {
                const int mi = lane >> 3, ri = lane & 7;
                const int row = row0 + 8 * (mi & 1) + ri;
#pragma unroll
                for (int j = 0; j < NB; j += 2) {
                    const int cc = j + (mi >> 1);           // 8-column block of head_dim
                    const uint32_t addr = vbase + (cc >> 3) * kBoxBytes + swz128(row, cc & 7);
                    uint32_t r0, r1, r2, r3;
                    ldsm_x4_trans(addr, r0, r1, r2, r3);
                    mma_bf16_16816(o[j], pa0, 0u, pa2, 0u, r0, r1);
                    mma_bf16_16816(o[j + 1], pa0, 0u, pa2, 0u, r2, r3);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[stage]);
            if (++stage == NS) { stage = 0; phase ^= 1; }
        }
        if (!alive) break;

        // ---- merge the four warps' states for this item ----
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
        l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
        if (warp > 0 && row_ok) {
            float* dst = red_o + ((warp - 1) * kMaxGroup + grp) * D;
#pragma unroll
            for (int j = 0; j < NB; ++j)
                *reinterpret_cast<float2*>(dst + j * 8 + tig * 2) = make_float2(o[j][0], o[j][1]);
            if (tig == 0) {
                red_m[warp * kMaxGroup + grp] = m_run;
                red_l[warp * kMaxGroup + grp] = l_run;
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        if (warp == 0 && row_ok) {
            float M = m_run;
#pragma unroll
            for (int w = 1; w < kConsumerWarps; ++w) M = fmaxf(M, red_m[w * kMaxGroup + grp]);
            const float s_new = last ? f_snew[slot * kMaxGroup + grp] : -INFINITY;   // the fused step's new row
            M = fmaxf(M, s_new);
            const float Mu = (M == -INFINITY) ? 0.f : M;
            float sc[kConsumerWarps];
            sc[0] = ex2_approx(m_run - Mu);
            float Ltot = l_run * sc[0];
#pragma unroll
            for (int w = 1; w < kConsumerWarps; ++w) {
                sc[w] = ex2_approx(red_m[w * kMaxGroup + grp] - Mu);
                Ltot += red_l[w * kMaxGroup + grp] * sc[w];
            }
            // the new row enters like a tile row: fp32 p in the sum, p rounded to bf16 for P.V
            const float p_new = last ? ex2_approx(s_new - Mu) : 0.f;
            const float p_new_bf = __bfloat162float(__float2bfloat16_rn(p_new));
            Ltot += p_new;
            const int head = g * a.n_rep + grp;
            if (nch_b == 1) {
                const float inv = (Ltot > 0.f) ? 1.f / Ltot : 0.f;
                __nv_bfloat16* orow = a.out + ((int64_t)b * a.H + head) * D;
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    float x0 = o[j][0] * sc[0], x1 = o[j][1] * sc[0];
#pragma unroll
                    for (int w = 1; w < kConsumerWarps; ++w) {
                        const float2 r = *reinterpret_cast<const float2*>(red_o + ((w - 1) * kMaxGroup + grp) * D +
                                                                          j * 8 + tig * 2);
                        x0 += r.x * sc[w];
                        x1 += r.y * sc[w];
                    }
                    if (last) {
                        x0 += p_new_bf * __bfloat162float(f_vnew[slot * D + j * 8 + tig * 2]);
                        x1 += p_new_bf * __bfloat162float(f_vnew[slot * D + j * 8 + tig * 2 + 1]);
                    }
                    *reinterpret_cast<uint32_t*>(orow + j * 8 + tig * 2) = pack_bf16x2(x0 * inv, x1 * inv);
                }
            } else {
                const int64_t pidx = (int64_t)item * a.n_rep + grp;
                float* prow = a.part_o + pidx * D;
#pragma unroll
                for (int j = 0; j < NB; ++j) {
                    float x0 = o[j][0] * sc[0], x1 = o[j][1] * sc[0];
#pragma unroll
                    for (int w = 1; w < kConsumerWarps; ++w) {
                        const float2 r = *reinterpret_cast<const float2*>(red_o + ((w - 1) * kMaxGroup + grp) * D +
                                                                          j * 8 + tig * 2);
                        x0 += r.x * sc[w];
                        x1 += r.y * sc[w];
                    }
                    if (last) {
                        x0 += p_new_bf * __bfloat162float(f_vnew[slot * D + j * 8 + tig * 2]);
                        x1 += p_new_bf * __bfloat162float(f_vnew[slot * D + j * 8 + tig * 2 + 1]);
                    }
                    *reinterpret_cast<float2*>(prow + j * 8 + tig * 2) = make_float2(x0, x1);
                }
                if (tig == 0) {
                    a.part_ml[pidx * 2 + 0] = M;
                    a.part_ml[pidx * 2 + 1] = Ltot;
                }
            }
        }
        if constexpr (kFused) {
            if (warp == 0) {   // warp 0 alone read the slot's new-row data
                __syncwarp();
                if (lane == 0) mbar_arrive(&f_vsfree[slot]);
            }
        }
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
    }
}

// Merges the per-chunk partials of every (sequence, query head) whose cache spans more
// than one chunk.  One CTA per (query head, sequence) -- B x H CTAs, enough to fill the GPU even
// when a GPU holds one kv head -- and thread d owns column d.  By the time this runs the partials
// have usually left L2 (the split kernel streamed the whole cache through it after writing them),
// so thread d first issues its column's loads for the first kCombineBatch chunks; meanwhile the
// block takes the chunks' maximum and the weights exp2(m_c - M), and sum_c l_c w_c, by
// reductions in a fixed order (deterministic), and only then are the columns summed, in chunk
// order.
constexpr int kMaxChunks = 128;
constexpr int kCombineBatch = 8;   // chunks per batch of loads in flight
constexpr int kCombineThreads = 128;
static_assert(kMaxChunks <= kCombineThreads, "a thread per chunk for the weights");

template <int D>
__global__ void __launch_bounds__(kCombineThreads) decode_combine_kernel(DecodeArgs a) {
    __shared__ float s_w[kMaxChunks];   // chunk weights exp2(m_c - M)
    __shared__ float s_red[2][kCombineThreads / 32];
    pdl_wait();      // partials come from the split kernel launched just before
    const int g = blockIdx.x / a.n_rep, r = blockIdx.x - g * a.n_rep, b = blockIdx.y;
    // the split grid has finished handing out items: ready the counter for the next call
    if (blockIdx.x == 0 && b == 0 && threadIdx.x == 0 && a.item_counter != nullptr) *a.item_counter = 0u;
    int L = a.kv_lens ? a.kv_lens[b] : a.max_len;
    L = L < 0 ? 0 : (L > a.max_len ? a.max_len : L);
    const int nch_b = (L + a.chunk - 1) / a.chunk;
    if (nch_b <= 1) return;  // written directly by the split kernel
    const int64_t item0 = ((int64_t)b * a.Hkv + g) * a.nch;
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int64_t step = (int64_t)a.n_rep * D;   // next chunk, same head
    const float* col = a.part_o + (item0 * a.n_rep + r) * D + t;
    // the first batch of this thread's column loads, before anything else
    float v[kCombineBatch];
    const int nb0 = nch_b < kCombineBatch ? nch_b : kCombineBatch;
#pragma unroll
    for (int c = 0; c < kCombineBatch; ++c) v[c] = (t < D && c < nb0) ? col[c * step] : 0.f;
    // chunk t's (m, l) of this row
    float m = -INFINITY, l = 0.f;
    if (t < nch_b) {
        const float2 ml = *reinterpret_cast<const float2*>(a.part_ml + ((item0 + t) * a.n_rep + r) * 2);
        m = ml.x;
        l = ml.y;
    }
    float mx = m;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) s_red[0][warp] = mx;
    __syncthreads();
    float M = s_red[0][0];
#pragma unroll
    for (int w = 1; w < kCombineThreads / 32; ++w) M = fmaxf(M, s_red[0][w]);
    const float Mu = (M == -INFINITY) ? 0.f : M;
    const float wgt = (t < nch_b) ? ex2_approx(m - Mu) : 0.f;
    if (t < nch_b) s_w[t] = wgt;
    float lw = l * wgt;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    if (lane == 0) s_red[1][warp] = lw;
    __syncthreads();
    float Lt = s_red[1][0];
#pragma unroll
    for (int w = 1; w < kCombineThreads / 32; ++w) Lt += s_red[1][w];
    const float inv = (Lt > 0.f) ? 1.f / Lt : 0.f;
    if (t >= D) return;
    float acc = 0.f;
    for (int c0 = 0; c0 < nch_b; c0 += kCombineBatch) {
        if (c0 > 0) {   // the next batch (sequences of more than kCombineBatch chunks)
#pragma unroll
            for (int c = 0; c < kCombineBatch; ++c) v[c] = (c0 + c < nch_b) ? col[(c0 + c) * step] : 0.f;
        }
#pragma unroll
        for (int c = 0; c < kCombineBatch; ++c)
            if (c0 + c < nch_b) acc += v[c] * s_w[c0 + c];
    }
    a.out[((int64_t)b * a.H + (int64_t)g * a.n_rep + r) * D + t] = __float2bfloat16_rn(acc * inv);
}

// Chunking of the cache rows into work items, with chunks of at least 256 rows (amortises the
// per-item merge).
constexpr int kMinChunk = 256;
constexpr double kCombineTiles = 4.0;   // the combine launch after a split grid, in tile-times
// An item's set-up (its q rows, the first K/V tiles' latency) and its share of the merge, in
// tile-times: fitted on the Qwen3-14B ragged batch (64 sequences of U[256, 32768] rows), where it
// picks the fastest measured chunk counts with one and with eight kv heads.
constexpr double kItemTiles = 2.0;

int max_chunks(int max_len) { return std::min(kMaxChunks, std::max(1, (max_len + kMinChunk - 1) / kMinChunk)); }

// Picks the chunk count per sequence for a grid of `grid` persistent CTAs, in units of one
// CTA's time per 64-row tile.  One chunk per (sequence, kv head): every CTA takes at most
// ceil(items / grid) items under the static schedule, no partials, no combine.  Several: the
// CTAs take items from the counter, so the work (tiles plus kItemTiles per item)
// spreads evenly over the grid, and the step ends about one item after the average CTA, plus
// the combine launch (about four tile-times, measured).  Each item costs kItemTiles beyond its
// tiles.
void plan_chunks(int B, int Hkv, int max_len, int grid, int& chunk, int& nch) {
    const int64_t pairs = (int64_t)B * Hkv;
    const int64_t tiles = (max_len + kTile - 1) / kTile;
    double best = 1e30;
    int best_n = 1;
    const int n_max = (int)std::min<int64_t>(max_chunks(max_len), tiles);
    for (int n = 1; n <= n_max; ++n) {
        const int64_t chunk_tiles = (tiles + n - 1) / n;
        const int64_t n_eff = (tiles + chunk_tiles - 1) / chunk_tiles;   // chunks actually used
        const int64_t items = pairs * n_eff;
        const double cost = n_eff == 1
            ? (double)((items + grid - 1) / grid) * ((double)chunk_tiles + kItemTiles)
            : (double)items * ((double)chunk_tiles + kItemTiles) / grid + (double)chunk_tiles + kCombineTiles;
        if (cost < best - 1e-9) {
            best = cost;
            best_n = (int)n_eff;
        }
    }
    const int64_t chunk_tiles = (tiles + best_n - 1) / best_n;
    chunk = (int)(chunk_tiles * kTile);
    nch = (max_len + chunk - 1) / chunk;
}

// The workspace starts with a 256-byte header holding the item counter, then the partials.
constexpr size_t kHeaderBytes = 256;

size_t workspace_bytes_for(int B, int H, int Hkv, int D, int max_len) {
    const int n_rep = H / Hkv;
    const size_t parts = (size_t)B * Hkv * max_chunks(max_len) * n_rep;
    const size_t bytes = kHeaderBytes + parts * D * 4 + parts * 2 * 4;
    return (bytes + 255) & ~size_t(255);
}

// Plans the chunks, places the partials in `workspace` and launches the split kernel (and,
// when a sequence spans several chunks, the combine kernel), both with programmatic
// dependent launch.  `a` arrives with its per-call fields set.
template <int D, bool kFused>
int launch_decode_d(DecodeArgs& a, const CUtensorMap& tmK, const CUtensorMap& tmV, int num_sms, void* workspace,
                    cudaStream_t s) {
    plan_chunks(a.B, a.Hkv, a.max_len, 2 * num_sms, a.chunk, a.nch);
    const size_t parts = (size_t)a.B * a.Hkv * a.nch * a.n_rep;
    // items past the first grid-size ones come from the counter when the combine kernel runs
    // after this launch (it resets the counter); a single-chunk call keeps the static schedule
    a.item_counter = a.nch > 1 ? reinterpret_cast<unsigned*>(workspace) : nullptr;
    a.part_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + kHeaderBytes);
    a.part_ml = a.part_o + parts * D;
    a.items = a.B * a.Hkv * a.nch;
    const int grid = std::min(a.items, 2 * num_sms);
    auto kern = decode_split_kernel<D, kFused>;
    const int smem = kFused ? DecodeCfg<D>::kSmemBytesFused : DecodeCfg<D>::kSmemBytes;
    if (int st = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem),
                            "decode smem attribute"))
        return st;
    if (int st = check_cuda(launch_pdl(kern, dim3(grid), dim3(kFused ? kThreadsFused : kThreads), smem, s, tmK, tmV, a),
                            "decode_split_kernel launch"))
        return st;
    if (a.nch > 1) {
        if (int st = check_cuda(launch_pdl(decode_combine_kernel<D>, dim3(a.Hkv * a.n_rep, a.B), dim3(kCombineThreads),
                                           0, s, a),
                                "decode_combine_kernel launch")) {
            // The split grid is queued and takes items from the counter, which only the combine
            // resets: zero it in stream order so the workspace's next call starts clean.
            (void)cudaMemsetAsync(workspace, 0, kHeaderBytes, s);
            return st;
        }
    }
    return MLLM_OK;
}

template <bool kFused>
int launch_decode(DecodeArgs& a, int head_dim, const CUtensorMap& tmK, const CUtensorMap& tmV, int num_sms,
                  void* workspace, cudaStream_t s) {
    return head_dim == 128 ? launch_decode_d<128, kFused>(a, tmK, tmV, num_sms, workspace, s)
                           : launch_decode_d<64, kFused>(a, tmK, tmV, num_sms, workspace, s);
}

}  // namespace

MLLM_DEFINE_STATUS_READER(decode)

}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" size_t mllm_decode_attention_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                                       int max_kv_len) {
    if (batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || max_kv_len <= 0 ||
        head_dim <= 0)
        return 0;
    return workspace_bytes_for(batch, num_heads, num_kv_heads, head_dim, max_kv_len);
}

extern "C" int mllm_decode_attention_plan(int batch, int num_heads, int num_kv_heads, int head_dim, int max_kv_len,
                                          int* chunk_rows, int* chunks, int* launches) {
    if (batch <= 0 || num_heads <= 0 || num_kv_heads <= 0 || num_heads % num_kv_heads || max_kv_len <= 0 ||
        (head_dim != 64 && head_dim != 128))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention_plan: bad sizes");
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;
    int chunk = 0, nch = 0;
    plan_chunks(batch, num_kv_heads, max_kv_len, 2 * num_sms, chunk, nch);
    if (chunk_rows) *chunk_rows = chunk;
    if (chunks) *chunks = nch;
    if (launches) *launches = nch > 1 ? 2 : 1;
    return ok();
}

extern "C" int mllm_decode_attention_bf16(const void* q, const void* k_cache, const void* v_cache,
                                          int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                          const int32_t* kv_lens, int batch, int num_heads, int num_kv_heads,
                                          int head_dim, int max_kv_len, float softmax_scale, void* out,
                                          void* workspace, size_t workspace_bytes, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_decode_attention_bf16");
    if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_kv_len <= 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: bad sizes");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128)
        return fail(MLLM_ERR_UNSUPPORTED, "decode_attention: head_dim must be 64 or 128");
    const int n_rep = num_heads / num_kv_heads;
    if (n_rep > kMaxGroup) return fail(MLLM_ERR_UNSUPPORTED, "decode_attention: GQA group larger than 8");
    if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: softmax_scale must be positive");
    if (batch == 0) return ok();
    if (!q || !k_cache || !v_cache || !out)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: null pointer");
    if (!aligned(q, 4) || !aligned(out, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: q/out misaligned");
    const size_t need = workspace_bytes_for(batch, num_heads, num_kv_heads, head_dim, max_kv_len);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
        return fail(MLLM_ERR_WORKSPACE, "decode_attention: workspace missing, misaligned or smaller than "
                                        "mllm_decode_attention_workspace_size()");
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;

    CUtensorMap tmK, tmV;
    if (int st = encode_kv_map(&tmK, k_cache, head_dim, max_kv_len, num_kv_heads, batch, cache_st, cache_sh, cache_sb,
                               64, kTile))
        return st;
    if (int st = encode_kv_map(&tmV, v_cache, head_dim, max_kv_len, num_kv_heads, batch, cache_st, cache_sh, cache_sb,
                               64, kTile))
        return st;

    DecodeArgs a = {};
    a.q = (const __nv_bfloat16*)q;
    a.kv_lens = kv_lens;
    a.out = (__nv_bfloat16*)out;
    a.B = batch;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.n_rep = n_rep;
    a.max_len = max_kv_len;
    a.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
    if (int st = launch_decode<false>(a, head_dim, tmK, tmV, num_sms, workspace, (cudaStream_t)stream)) return st;
    return ok();
}

extern "C" int mllm_decode_attention_paged_bf16(const void* q, const mllm_paged_kv* kv, const int32_t* kv_lens,
                                                int batch, int num_heads, int num_kv_heads, int head_dim,
                                                int max_kv_len, float softmax_scale, void* out, void* workspace,
                                                size_t workspace_bytes, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_decode_attention_paged_bf16");
    if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_kv_len <= 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: bad sizes");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128)
        return fail(MLLM_ERR_UNSUPPORTED, "decode_attention: head_dim must be 64 or 128");
    const int n_rep = num_heads / num_kv_heads;
    if (n_rep > kMaxGroup) return fail(MLLM_ERR_UNSUPPORTED, "decode_attention: GQA group larger than 8");
    if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: softmax_scale must be positive");
    if (batch == 0) return ok();
    if (!q || !out) return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: null pointer");
    KvLayout lay;
    if (int st = paged_layout(kv, max_kv_len, head_dim, "decode_attention_paged", &lay)) return st;
    if (!aligned(q, 4) || !aligned(out, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention: q/out misaligned");
    const size_t need = workspace_bytes_for(batch, num_heads, num_kv_heads, head_dim, max_kv_len);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
        return fail(MLLM_ERR_WORKSPACE, "decode_attention: workspace missing, misaligned or smaller than "
                                        "mllm_decode_attention_workspace_size()");
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;

    CUtensorMap tmK, tmV;
    if (int st = encode_kv_map(&tmK, kv->k_pool, head_dim, kv->block_size, num_kv_heads, kv->num_blocks,
                               kv->row_stride, kv->head_stride, kv->block_stride, 64, kTile))
        return st;
    if (int st = encode_kv_map(&tmV, kv->v_pool, head_dim, kv->block_size, num_kv_heads, kv->num_blocks,
                               kv->row_stride, kv->head_stride, kv->block_stride, 64, kTile))
        return st;

    DecodeArgs a = {};
    a.lay = lay;
    a.q = (const __nv_bfloat16*)q;
    a.kv_lens = kv_lens;
    a.out = (__nv_bfloat16*)out;
    a.B = batch;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.n_rep = n_rep;
    a.max_len = max_kv_len;
    a.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
    if (int st = launch_decode<false>(a, head_dim, tmK, tmV, num_sms, workspace, (cudaStream_t)stream)) return st;
    return ok();
}

// ---------------------------------------------------------------------------------------------
// Decode without a caller workspace.
//
// Some callers cannot allocate device memory at the moment they run decode: a runtime whose
// memory is carved up once at start-up by its own arena (and forbids later cudaMalloc), a
// kernel-launch hook running inside another framework's allocator lock, or code on a path
// where an allocation would be a synchronising call.  This entry point serves them: the
// split-K partials live in a fixed scratch array that is part of this library's device image,
// so nothing is allocated per call.  The array is kNoAllocScratchBytes (16 MiB) per device and
// stays resident on every GPU that loads the library until the process exits.
// ---------------------------------------------------------------------------------------------
#include <cstdio>
#include <mutex>

namespace mllm_b200 {
namespace {

constexpr size_t kNoAllocScratchBytes = size_t(16) << 20;

// Device-resident scratch shared by every call of mllm_decode_attention_noalloc_bf16 on a device.
static __device__ __align__(256) unsigned char g_decode_noalloc_scratch[kNoAllocScratchBytes];

constexpr int kMaxDevices = 64;

// The array's address belongs to one CUDA context: after cudaDeviceReset, or once the primary
// context is released and created again, the module is loaded anew and may sit elsewhere.  So
// the cached address is keyed by the context's unique ID (cuCtxGetId), and looked up again
// whenever the current context is a different one.
struct ScratchAddr {
    unsigned long long ctx_id;   // 0: not cached
    void* ptr;
};
std::mutex g_noalloc_mutex;
ScratchAddr g_noalloc_addr[kMaxDevices] = {};

using PfnCtxGetCurrent = CUresult (*)(CUcontext*);
using PfnCtxGetId = CUresult (*)(CUcontext, unsigned long long*);

// ID of the calling thread's current context; false if there is none yet (or the driver has no
// cuCtxGetId), in which case the caller looks the address up every time.
bool current_ctx_id(unsigned long long* id) {
    static PfnCtxGetCurrent get_current = nullptr;
    static PfnCtxGetId get_id = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<PfnCtxGetCurrent>(p);
        p = nullptr;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<PfnCtxGetId>(p);
    });
    if (!get_current || !get_id) return false;
    CUcontext ctx = nullptr;
    if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
    return get_id(ctx, id) == CUDA_SUCCESS && *id != 0;
}

// Device address of the scratch array in the current context.  The first call in a context
// looks it up with cudaGetSymbolAddress (host code cannot use the array's name as a device
// address; that lookup also creates the primary context if there is none yet).
int noalloc_scratch(void** out) {
    int dev = 0;
    if (int st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice")) return st;
    if (dev < 0 || dev >= kMaxDevices) return fail(MLLM_ERR_UNSUPPORTED, "decode_attention_noalloc: device index too large");
    unsigned long long id = 0;
    bool have_id = current_ctx_id(&id);
    std::lock_guard<std::mutex> lock(g_noalloc_mutex);
    ScratchAddr& c = g_noalloc_addr[dev];
    if (have_id && c.ctx_id == id && c.ptr != nullptr) {
        *out = c.ptr;
        return MLLM_OK;
    }
    void* p = nullptr;
    if (int st = check_cuda(cudaGetSymbolAddress(&p, g_decode_noalloc_scratch), "cudaGetSymbolAddress(scratch)"))
        return st;
    if (!have_id) have_id = current_ctx_id(&id);
    c.ctx_id = have_id ? id : 0ull;
    c.ptr = p;
    *out = p;
    return MLLM_OK;
}

}  // namespace
}  // namespace mllm_b200

extern "C" int mllm_decode_attention_noalloc_bf16(const void* q, const void* k_cache, const void* v_cache,
                                                  int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                                  const int32_t* kv_lens, int batch, int num_heads,
                                                  int num_kv_heads, int head_dim, int max_kv_len,
                                                  float softmax_scale, void* out, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_decode_attention_noalloc_bf16");
    if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_kv_len <= 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention_noalloc: bad sizes");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128)
        return fail(MLLM_ERR_UNSUPPORTED, "decode_attention_noalloc: head_dim must be 64 or 128");
    const int n_rep = num_heads / num_kv_heads;
    if (n_rep > kMaxGroup) return fail(MLLM_ERR_UNSUPPORTED, "decode_attention_noalloc: GQA group larger than 8");
    if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention_noalloc: softmax_scale must be positive");
    if (batch == 0) return ok();
    if (!q || !k_cache || !v_cache || !out)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention_noalloc: null pointer");
    if (!aligned(q, 4) || !aligned(out, 4))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_attention_noalloc: q/out misaligned");
    const size_t need = workspace_bytes_for(batch, num_heads, num_kv_heads, head_dim, max_kv_len);
    if (need > kNoAllocScratchBytes) {
        char buf[256];
        snprintf(buf, sizeof(buf),
                 "decode_attention_noalloc: this batch needs %zu bytes of split-K scratch but the static "
                 "scratch holds %zu; use mllm_decode_attention_bf16 with a caller workspace",
                 need, kNoAllocScratchBytes);
        return fail(MLLM_ERR_WORKSPACE, buf);
    }
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;
    void* scratch = nullptr;
    if (int st = noalloc_scratch(&scratch)) return st;

    CUtensorMap tmK, tmV;
    if (int st = encode_kv_map(&tmK, k_cache, head_dim, max_kv_len, num_kv_heads, batch, cache_st, cache_sh, cache_sb,
                               64, kTile))
        return st;
    if (int st = encode_kv_map(&tmV, v_cache, head_dim, max_kv_len, num_kv_heads, batch, cache_st, cache_sh, cache_sb,
                               64, kTile))
        return st;

    // The scratch begins with the work-item counter: zero from the start (static storage), reset
    // by the combine kernel of every call that takes items from it, and reset in stream order
    // when the combine cannot be launched.  Every partial the combine reads is written earlier
    // in the same call.  So nothing needs clearing between calls.
    DecodeArgs a = {};
    a.q = (const __nv_bfloat16*)q;
    a.kv_lens = kv_lens;
    a.out = (__nv_bfloat16*)out;
    a.B = batch;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.n_rep = n_rep;
    a.max_len = max_kv_len;
    a.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
    if (int st = launch_decode<false>(a, head_dim, tmK, tmV, num_sms, scratch, (cudaStream_t)stream)) return st;
    return ok();
}

// ---------------------------------------------------------------------------------------------
// Fused decode step: the QKV epilogue of one new token per sequence (QK-RMSNorm, RoPE, KV
// append) and the decode attention over the cache including that token, in one launch of the
// split kernel (plus the combine kernel when a sequence spans several chunks).
// ---------------------------------------------------------------------------------------------
namespace {

// Shared by mllm_decode_step_bf16 and its paged form.  The cache is addressed per sequence
// (contiguous: map_rows = max_kv_len rows, map_batch = batch) or per block (paged: map_rows =
// block_size, map_batch = num_blocks), with `lay` saying which.
int decode_step_entry(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb, int64_t k_sh,
                      const void* v, int64_t v_sb, int64_t v_sh, const int64_t* positions, int64_t pos_sb,
                      double rope_theta, const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                      const void* q_norm_weight, const void* k_norm_weight, double rms_norm_eps, void* k_cache,
                      void* v_cache, int64_t cache_sb, int64_t cache_sh, int64_t cache_st, int64_t map_rows,
                      int64_t map_batch, const KvLayout& lay, const int32_t* kv_lens, int batch, int num_heads,
                      int num_kv_heads, int head_dim, int max_kv_len, float softmax_scale, void* out,
                      void* workspace, size_t workspace_bytes, mllm_stream_t stream) {
    if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_kv_len <= 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: bad sizes");
    if (num_heads % num_kv_heads != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "Attention: num_heads must be divisible by num_kv_heads.");
    if (head_dim != 64 && head_dim != 128) return fail(MLLM_ERR_UNSUPPORTED, "decode_step: head_dim must be 64 or 128");
    const int n_rep = num_heads / num_kv_heads;
    if (n_rep > kMaxGroup) return fail(MLLM_ERR_UNSUPPORTED, "decode_step: GQA group larger than 8");
    if (!(softmax_scale > 0.f) || !std::isfinite(softmax_scale))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: softmax_scale must be positive");
    if ((q_norm_weight == nullptr) != (k_norm_weight == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: give both q/k norm weights or neither");
    if ((rope_cos == nullptr) != (rope_sin == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: give both rope tables or neither");
    if (rope_cos == nullptr && positions == nullptr)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: positions or rope tables required");
    if (rope_cos == nullptr && !(rope_theta > 0.0))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: rope_theta must be positive");
    if (batch == 0) return ok();
    if (!q || !k || !v || !k_cache || !v_cache || !out)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: null pointer");
    if (!aligned(out, 4)) return fail(MLLM_ERR_INVALID_ARGUMENT, "decode_step: out misaligned");
    const size_t need = workspace_bytes_for(batch, num_heads, num_kv_heads, head_dim, max_kv_len);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
        return fail(MLLM_ERR_WORKSPACE, "decode_step: workspace missing, misaligned or smaller than "
                                        "mllm_decode_attention_workspace_size()");
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;

    CUtensorMap tmK, tmV;
    if (int st = encode_kv_map(&tmK, k_cache, head_dim, map_rows, num_kv_heads, map_batch, cache_st, cache_sh,
                               cache_sb, 64, kTile))
        return st;
    if (int st = encode_kv_map(&tmV, v_cache, head_dim, map_rows, num_kv_heads, map_batch, cache_st, cache_sh,
                               cache_sb, 64, kTile))
        return st;

    DecodeArgs a = {};
    a.lay = lay;
    a.kv_lens = kv_lens;
    a.out = (__nv_bfloat16*)out;
    a.B = batch;
    a.H = num_heads;
    a.Hkv = num_kv_heads;
    a.n_rep = n_rep;
    a.max_len = max_kv_len;
    a.scale_log2 = (float)((double)softmax_scale * 1.4426950408889634);
    a.q_in = (const __nv_bfloat16*)q;
    a.k_in = (const __nv_bfloat16*)k;
    a.v_in = (const __nv_bfloat16*)v;
    a.q_sb = q_sb; a.q_sh = q_sh;
    a.k_sb = k_sb; a.k_sh = k_sh;
    a.v_sb = v_sb; a.v_sh = v_sh;
    a.positions = positions;
    a.pos_sb = pos_sb;
    a.log_theta = rope_cos ? 0.f : rope_log_theta(rope_theta);
    a.rope_cos = rope_cos;
    a.rope_sin = rope_sin;
    a.rope_row_sb = rope_row_sb;
    a.q_gamma = (const __nv_bfloat16*)q_norm_weight;
    a.k_gamma = (const __nv_bfloat16*)k_norm_weight;
    a.eps = (float)rms_norm_eps;   // the reference adds the double eps to a float tensor
    a.k_cache = (__nv_bfloat16*)k_cache;
    a.v_cache = (__nv_bfloat16*)v_cache;
    a.c_sb = cache_sb; a.c_sh = cache_sh; a.c_st = cache_st;
    if (int st = launch_decode<true>(a, head_dim, tmK, tmV, num_sms, workspace, (cudaStream_t)stream)) return st;
    return ok();
}

}  // namespace

extern "C" int mllm_decode_step_bf16(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb,
                                     int64_t k_sh, const void* v, int64_t v_sb, int64_t v_sh,
                                     const int64_t* positions, int64_t pos_sb, double rope_theta,
                                     const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                                     const void* q_norm_weight, const void* k_norm_weight, double rms_norm_eps,
                                     void* k_cache, void* v_cache, int64_t cache_sb, int64_t cache_sh,
                                     int64_t cache_st, const int32_t* kv_lens, int batch, int num_heads,
                                     int num_kv_heads, int head_dim, int max_kv_len, float softmax_scale, void* out,
                                     void* workspace, size_t workspace_bytes, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_decode_step_bf16");
    return decode_step_entry(q, q_sb, q_sh, k, k_sb, k_sh, v, v_sb, v_sh, positions, pos_sb, rope_theta, rope_cos,
                             rope_sin, rope_row_sb, q_norm_weight, k_norm_weight, rms_norm_eps, k_cache, v_cache,
                             cache_sb, cache_sh, cache_st, max_kv_len, batch, KvLayout{}, kv_lens, batch, num_heads,
                             num_kv_heads, head_dim, max_kv_len, softmax_scale, out, workspace, workspace_bytes,
                             stream);
}

extern "C" int mllm_decode_step_paged_bf16(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb,
                                           int64_t k_sh, const void* v, int64_t v_sb, int64_t v_sh,
                                           const int64_t* positions, int64_t pos_sb, double rope_theta,
                                           const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                                           const void* q_norm_weight, const void* k_norm_weight,
                                           double rms_norm_eps, const mllm_paged_kv* kv, const int32_t* kv_lens,
                                           int batch, int num_heads, int num_kv_heads, int head_dim, int max_kv_len,
                                           float softmax_scale, void* out, void* workspace, size_t workspace_bytes,
                                           mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_decode_step_paged_bf16");
    KvLayout lay;
    if (int st = paged_layout(kv, max_kv_len, head_dim, "decode_step_paged", &lay)) return st;
    return decode_step_entry(q, q_sb, q_sh, k, k_sb, k_sh, v, v_sb, v_sh, positions, pos_sb, rope_theta, rope_cos,
                             rope_sin, rope_row_sb, q_norm_weight, k_norm_weight, rms_norm_eps, kv->k_pool,
                             kv->v_pool, kv->block_stride, kv->head_stride, kv->row_stride, kv->block_size,
                             kv->num_blocks, lay, kv_lens, batch, num_heads, num_kv_heads, head_dim, max_kv_len,
                             softmax_scale, out, workspace, workspace_bytes, stream);
}
