// Projection GEMM for decode-sized token counts (tokens <= 256): the Linear::Forward calls on
// either side of the attention step (Linear.h:33-68: q/k/v before it, o_proj after it), with
// up to four weights in one launch so q, k and v come out of one kernel as one [T, q|k|v] row
// block without concatenating the weights.
//
// At these sizes the GEMM is a stream over the weights (T x K activations are a few hundred KB
// and stay in L2), so the kernel is built to keep HBM busy:
//   * a CTA owns one 128-row tile of one weight and a contiguous range of its 64-column k-blocks;
//     the tile is the MMA's M side and the tokens its N side (D[128 x NT] = W[128 x K] X^T), so
//     one tcgen05.mma per 16 k covers all tokens, fp32 accumulators in tensor memory;
//   * warp 0 streams weight and activation k-blocks through a ring of shared-memory stages with
//     TMA (no multicast); the weight tiles of the first stages are requested before the
//     programmatic-launch wait, since no earlier kernel writes them;
//   * the k range of a tile is split over up to 8 CTAs, chosen so the grid fills two CTAs per
//     SM in one wave; each CTA writes its fp32 partial to the caller's workspace and the last
//     CTA of a tile to finish (a per-tile counter) adds the partials in split order -- a fixed
//     order, so the result does not depend on scheduling -- rounds once to bf16 and resets the
//     counter.  (Thread-block clusters with a distributed-shared-memory reduction were tried
//     first: only about 33 clusters of 4 are resident at once, so a 48-tile q|k|v grid ran in
//     two waves.)
// Every mbarrier wait is bounded (common.cuh).
#include <cuda_fp8.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "host_util.h"
#include "tcgen05.cuh"

namespace mllm_b200 {
namespace {

constexpr int kTileRows = 128;               // weight rows per tile (the MMA's M)
constexpr int kAtomK = 64;                   // k per 128-byte swizzle atom of bf16
constexpr int kThreads = 128;
constexpr int kMaxWeights = 4;
constexpr int kMaxTokens = 256;
constexpr int kMaxSplits = 8;
constexpr int kRedBatch = 4;                 // tokens per warp per reduction batch
// The workspace starts with a fixed block of tile counters, so calls of different shapes can
// share one workspace: a call's partials never overlap another call's counters.  Splitting only
// happens when the tiles fit in one CTA per SM, far below this.
constexpr int kMaxCounters = 1024;

// A stage holds NB consecutive k-atoms of the tile's 128 weight rows and of the NT token rows.
// Weights arrive as 16 boxes of 8 rows x NB atoms: the tensor map views W as {64 k, rows,
// k-atoms} with the atoms 128 B apart, so one box reads NB x 128 contiguous bytes of each of its
// rows back to back (rows are K x 2 bytes apart; a box of 128 rows x one atom would touch 128
// DRAM pages for 128 bytes each).  In shared memory a box is [atom][8 rows][128 B], i.e. each
// atom's 8-row group is one 1 KB swizzle block, and the 16 boxes follow each other: atom a's
// row group g sits at g * NB KB + a KB, which the MMA reads as a K-major SW128 operand with an
// 8-row-group stride of NB KB.  Tokens arrive as one box of NT rows x NB atoms, [atom][NT rows]
// [128 B] (8-row-group stride 1 KB).
template <int NT>
struct LinCfg {
    static constexpr int kNB = NT <= 64 ? 4 : 2;              // atoms per stage
    static constexpr int kWBytes = kTileRows * kNB * 128;
    static constexpr int kXBytes = NT * kNB * 128;
    static constexpr int kStageBytes = kWBytes + kXBytes;
    static constexpr int kStages = (200 * 1024) / kStageBytes; // 2 or 3, one CTA per SM
    static constexpr int kSmem = kStages * kStageBytes + 1024;
    static_assert(kStages >= 2, "at least two stages");
};

struct LinearMaps {
    CUtensorMap w[kMaxWeights];
    CUtensorMap x;
};

struct LinearArgs {
    int tile_begin[kMaxWeights + 1];   // first tile of weight i (prefix sums of rows / 128)
    int64_t out_col[kMaxWeights];      // first output column of weight i
    int units;                         // stages of kNB atoms covering K (the last may be partial)
    int tokens;
    __nv_bfloat16* out;
    int64_t out_stride;
    unsigned* counters;                // [tiles], zero between calls
    float* partial;                    // [tiles][splits][tokens][128]
};

// The last CTA of a tile sums its split partials: out = ((p0 + p1) + p2) + ... in fp32, one
// rounding.  Lane l owns rows 4l..4l+3 (one float4 per partial); warp w takes tokens w, w+4, ...
// in batches of BATCH tokens whose loads (BATCH x MS float4 per thread) all go out before any
// add, so a batch costs one round trip to L2.
template <int BATCH, int MS>
__device__ __forceinline__ void reduce_partials(const float* base, __nv_bfloat16* orow, int64_t ostride, int T,
                                                int splits, int warp) {
    for (int t0 = warp; t0 < T; t0 += 4 * BATCH) {
        float4 v[BATCH][MS];
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
            const int t = t0 + 4 * b;
#pragma unroll
            for (int sp = 0; sp < MS; ++sp)
                if (t < T && sp < splits)
                    v[b][sp] = __ldcg(reinterpret_cast<const float4*>(base + ((size_t)sp * T + t) * kTileRows));
        }
#pragma unroll
        for (int b = 0; b < BATCH; ++b) {
            const int t = t0 + 4 * b;
            if (t >= T) break;
            float4 acc = v[b][0];
#pragma unroll
            for (int sp = 1; sp < MS; ++sp)
                if (sp < splits) {
                    acc.x = __fadd_rn(acc.x, v[b][sp].x);
                    acc.y = __fadd_rn(acc.y, v[b][sp].y);
                    acc.z = __fadd_rn(acc.z, v[b][sp].z);
                    acc.w = __fadd_rn(acc.w, v[b][sp].w);
                }
            __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y);
            __nv_bfloat162 hi = __floats2bfloat162_rn(acc.z, acc.w);
            uint2 pk;
            pk.x = *reinterpret_cast<uint32_t*>(&lo);
            pk.y = *reinterpret_cast<uint32_t*>(&hi);
            *reinterpret_cast<uint2*>(orow + (int64_t)t * ostride) = pk;
        }
    }
}

template <int NT>
__global__ void __launch_bounds__(kThreads, 1)
    linear_kernel(const __grid_constant__ LinearMaps maps, const LinearArgs a) {
    using Cfg = LinCfg<NT>;
    constexpr int ST = Cfg::kStages;
    constexpr int NB = Cfg::kNB;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t full[ST], empty[ST], done;
    __shared__ uint32_t tmem_base;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int splits = (int)gridDim.x;
    const int split = (int)blockIdx.x;
    const int tile = (int)blockIdx.y;
    // which weight the tile belongs to, with constant indices only (no local-memory copy of `a`)
    int wi = 0, tb = 0;
    int64_t ocol = 0;
#pragma unroll
    for (int i = 1; i < kMaxWeights; ++i) wi += tile >= a.tile_begin[i] ? 1 : 0;
#pragma unroll
    for (int i = 0; i < kMaxWeights; ++i)
        if (i == wi) {
            tb = a.tile_begin[i];
            ocol = a.out_col[i];
        }
    const int wrow = (tile - tb) * kTileRows;
    const int u0 = (int)((int64_t)split * a.units / splits);
    const int nk = (int)((int64_t)(split + 1) * a.units / splits) - u0;   // >= 1 (splits <= units)
    auto stage_w = [&](int s) { return smem + s * Cfg::kStageBytes; };
    auto stage_x = [&](int s) { return smem + s * Cfg::kStageBytes + Cfg::kWBytes; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < ST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(&done, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(&tmem_base, NT);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    if (warp == 0 && lane == 0) {
        // ---------------------------- TMA producer ----------------------------
        const CUtensorMap* wm = &maps.w[wi];
        tma_prefetch_desc(wm);
        tma_prefetch_desc(&maps.x);
        auto load_w = [&](int i, int s) {
#pragma unroll 4
            for (int g = 0; g < kTileRows / 8; ++g)
                tma_load_4d(stage_w(s) + g * NB * 1024, wm, &full[s], 0, wrow + 8 * g, (u0 + i) * NB, 0);
        };
        const int pre = nk < ST ? nk : ST;
        for (int i = 0; i < pre; ++i) {
            mbar_arrive_expect_tx(&full[i], Cfg::kStageBytes);
            load_w(i, i);
        }
        pdl_wait();   // the activations may be the previous kernel's output
        for (int i = 0; i < pre; ++i) tma_load_4d(stage_x(i), &maps.x, &full[i], 0, 0, (u0 + i) * NB, 0);
        int i = pre;
        for (; i < nk; ++i) {
            const int s = i % ST;
            if (!mbar_wait(&empty[s], ((i / ST) - 1) & 1)) break;
            mbar_arrive_expect_tx(&full[s], Cfg::kStageBytes);
            load_w(i, s);
            tma_load_4d(stage_x(s), &maps.x, &full[s], 0, 0, (u0 + i) * NB, 0);
        }
        // every copy issued has landed before the stages are reused or the CTA exits (a no-op
        // unless a wait above gave up)
        for (int j = (i > ST ? i - ST : 0); j < i; ++j) mbar_wait(&full[j % ST], (j / ST) & 1);
    } else if (warp == 1 && lane == 0) {
        // ---------------------------- MMA issuer ----------------------------
        constexpr uint32_t idesc = idesc_bf16_f32(kTileRows, NT, false);
        constexpr uint32_t w_hi = smem_desc_hi_sw128(NB * 1024);   // row groups NB KB apart
        constexpr uint32_t x_hi = smem_desc_hi_sw128(1024);
        for (int i = 0; i < nk; ++i) {
            const int s = i % ST;
            if (!mbar_wait(&full[s], (i / ST) & 1)) break;
            tc_fence_after();
            const uint32_t wd = smem_desc_lo(smem_u32(stage_w(s)), 16);
            const uint32_t xd = smem_desc_lo(smem_u32(stage_x(s)), 16);
#pragma unroll
            for (int at = 0; at < NB; ++at)
#pragma unroll
                for (int ks = 0; ks < kAtomK / 16; ++ks)   // 16 k = 32 bytes along the swizzled row
                    tc_mma_ss_w2(tmem, wd + (uint32_t)((at * 1024 + ks * 32) >> 4), w_hi,
                                 xd + (uint32_t)((at * NT * 128 + ks * 32) >> 4), x_hi, idesc,
                                 (i > 0 || at > 0 || ks > 0) ? 1u : 0u);
            tc_commit(&empty[s]);
        }
        tc_commit(&done);   // also after a bailout, so the MMAs issued so far have completed
    }
    __syncwarp();

    // ------------------------------ epilogue (all 4 warps) ------------------------------
    mbar_wait(&done, 0);
    tc_fence_after();
    pdl_trigger();
    pdl_wait();   // the previous kernel may still read the output rows
    const int T = a.tokens;
    const int row = warp * 32 + lane;   // weight row within the tile == tensor-memory lane
    const int64_t ostride = a.out_stride;
    __nv_bfloat16* outp = a.out + ocol + wrow;
    const uint32_t t_lane = tmem + ((uint32_t)(warp * 32) << 16);
    float* mine = a.partial + ((size_t)(tile * splits + split) * T) * kTileRows;
#pragma unroll 1
    for (int c = 0; c < T; c += 32) {
        float r[32];
        tmem_ld32(t_lane + (uint32_t)c, r);
        tmem_wait_ld();
        if (splits == 1) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (c + j < T) outp[(int64_t)(c + j) * ostride + row] = __float2bfloat16_rn(r[j]);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (c + j < T) mine[(c + j) * kTileRows + row] = r[j];
        }
    }
    if (splits > 1) {
        __shared__ int s_last;
        __threadfence();
        __syncthreads();
        if (threadIdx.x == 0) s_last = atomicAdd(&a.counters[tile], 1u) == (unsigned)(splits - 1);
        __syncthreads();
        if (s_last) {
            // the last CTA of the tile adds the partials (reduce_partials)
            __threadfence();
            const float* base = a.partial + (size_t)tile * splits * T * kTileRows + 4 * lane;
            __nv_bfloat16* orow = outp + 4 * lane;
            // the same registers hold 8 tokens' partials when a tile has at most 4 splits (one
            // round of loads for 32 tokens), else 4 tokens' of up to 8 splits
            if (splits <= kMaxSplits / 2)
                reduce_partials<2 * kRedBatch, kMaxSplits / 2>(base, orow, ostride, T, splits, warp);
            else
                reduce_partials<kRedBatch, kMaxSplits>(base, orow, ostride, T, splits, warp);
            if (threadIdx.x == 0) a.counters[tile] = 0u;   // ready for the next call in the stream
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, NT);
}

struct LinearPlan {
    int tiles = 0, units = 0, splits = 1, nt = 32;
    size_t partial_offset = 0, workspace_bytes = 0;
};

template <int NT>
constexpr int units_for(int64_t in_features) {
    return (int)((in_features / kAtomK + LinCfg<NT>::kNB - 1) / LinCfg<NT>::kNB);
}

// Splits: as many as fill one CTA per SM in one wave, at most 8, at most one per stage unit,
// and few enough that the partials (written and read once) stay below about a quarter of the
// weight bytes (splits * tokens <= K / 8).
void plan_linear(int tokens, int num_weights, const int64_t* out_features, int64_t in_features, int num_sms,
                 LinearPlan* p) {
    p->tiles = 0;
    for (int i = 0; i < num_weights; ++i) p->tiles += (int)(out_features[i] / kTileRows);
    p->nt = tokens <= 32 ? 32 : tokens <= 64 ? 64 : tokens <= 128 ? 128 : 256;
    p->units = p->nt <= 64 ? units_for<32>(in_features) : units_for<128>(in_features);
    int64_t splits = std::min<int64_t>(kMaxSplits, (int64_t)num_sms / std::max(1, p->tiles));
    splits = std::min<int64_t>(splits, p->units);
    splits = std::min<int64_t>(splits, in_features / (8 * (int64_t)std::max(1, tokens)));
    p->splits = (int)std::max<int64_t>(1, splits);
    if (p->tiles > kMaxCounters) p->splits = 1;
    p->partial_offset = kMaxCounters * sizeof(unsigned);   // the same for every shape (see kMaxCounters)
    p->workspace_bytes = p->splits > 1 ? p->partial_offset + (size_t)p->tiles * p->splits * tokens * kTileRows * 4 : 0;
}

int check_linear_args(int tokens, int64_t in_features, int num_weights, const void* const* weights,
                      const int64_t* weight_strides, const int64_t* out_features, int64_t* total) {
    if (tokens < 0 || tokens > kMaxTokens)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: tokens must be in [0, 256]");
    if (num_weights < 1 || num_weights > kMaxWeights || !out_features)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: 1 to 4 weights with their row counts");
    if (in_features <= 0 || in_features % kAtomK != 0 || in_features > (int64_t)1 << 30)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: in_features must be a positive multiple of 64");
    *total = 0;
    for (int i = 0; i < num_weights; ++i) {
        if (out_features[i] <= 0 || out_features[i] % kTileRows != 0 || out_features[i] > (1 << 24))
            return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: each weight needs a positive multiple of 128 rows");
        if (weights && (!weights[i] || !weight_strides || weight_strides[i] < in_features))
            return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: null weight or row stride below in_features");
        *total += out_features[i];
    }
    return MLLM_OK;
}

int sm_count_or_default() {
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && sms > 0)
        return sms;
    cudaGetLastError();
    return 148;
}

template <int NT>
int launch_linear(const LinearMaps& maps, const LinearArgs& a, const LinearPlan& p, cudaStream_t s) {
    using Cfg = LinCfg<NT>;
    auto kern = linear_kernel<NT>;
    if (int st = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem),
                            "linear: shared memory attribute"))
        return st;
    return check_cuda(launch_pdl(kern, dim3(p.splits, p.tiles, 1), dim3(kThreads, 1, 1), (size_t)Cfg::kSmem, s,
                                 maps, a),
                      "linear launch");
}

// ---------------------------------------------------------------------------------------------
// FP8 weights with 128 x 128 block scales (e4m3, weight_scale_inv [N/128][K/128] fp32): the
// reference dequantizes every such projection on every step (QwenRunner.cpp:103-122:
// w.to(bf16) * scale.to(bf16), a bf16 tensor product) and multiplies in bf16 (Linear.h:33-68).
// This kernel streams the fp8 bytes -- half the bf16 weight -- and dequantizes each 128-row x
// 128-k block on chip (from shared memory into tensor memory) with exactly that arithmetic: fp8 -> fp32 (exact), times the
// bf16-rounded scale (an exact product of a 4-bit and an 8-bit significand), one rounding to bf16.
// The tensor cores then see the same bf16 operand the reference's GEMM sees.
//
// Roles (384 threads, the k range of a 128-row tile split over CTAs):
//   warp 0 (lane 0): TMA of the fp8 tile blocks, 128 rows x 128 bytes (128-byte swizzle), into
//     ring A in shared memory;
//   warp 2 (lane 0): TMA of the activations' two 64-k atoms of each block into ring X;
//   warps 4-11: dequantize -- thread (warp % 4, lane) owns tile row 32 * (warp % 4) + lane (its
//     tensor-memory lane), warps 4-7 the block's first 64 k, warps 8-11 the last 64; each writes its
//     row's bf16 values into a tensor-memory stage with tcgen05.st;
//   warp 1 (lane 0): tensor-memory allocation and tcgen05.mma kind::f16 with A = the dequantized
//     block in tensor memory (TS form) and B = the activations in shared memory, fp32 accumulators
//     in tensor memory columns [0, NT);
//   warps 4-7: the epilogue (tensor-memory lane quarters 0-3), split partials as linear_kernel.
// ---------------------------------------------------------------------------------------------
constexpr int kF8Unit = 128;                 // k per unit: one scale block, two bf16 atoms
constexpr int kF8Threads = 384;
constexpr int kF8ConvWarp0 = 4;
constexpr int kF8ConvWarps = 8;
constexpr int kF8MaxTokens = 128;

// At 32 tokens two CTAs share an SM (five fp8 stages and three dequantized stages each, 105 KB of
// shared memory and 256 tensor-memory columns; at most 85 registers at 384 threads): the
// dequantizing warps of two tiles interleave and the tile x split grid fits one wave.  Wider token
// tiles keep one CTA per SM.  The dequantizing issue, not the fp8 stream, sets the pace.
constexpr int f8_ctas_per_sm(int nt) { return nt == 32 ? 2 : 1; }

template <int NT>
struct F8Cfg {
    static constexpr int kABytes = kTileRows * kF8Unit;          // fp8 block
    static constexpr int kBXBytes = NT * kF8Unit * 2;            // activations of one block
    static constexpr int kAStages = NT == 32 ? 5 : (NT == 64 ? 8 : 6);
    static constexpr int kBStages = 3;                           // dequantized (tensor memory) + activations
    static constexpr int kRings = kBStages * kBXBytes + kAStages * kABytes;
    static constexpr int kSmem = kRings + 256;   // + barriers; the kernel has no static shared memory
    // tensor memory: accumulators [0, NT), then kBStages dequantized blocks of 64 columns (128 bf16
    // of k per row); the allocation is the next power of two
    static constexpr uint32_t kACol = NT;
    static constexpr uint32_t kTmemUsed = NT + kBStages * 64;
    static constexpr uint32_t kTmemCols = kTmemUsed <= 256 ? 256 : 512;
    static_assert(f8_ctas_per_sm(NT) * kTmemCols <= 512, "tensor memory of the resident CTAs");
    static_assert(f8_ctas_per_sm(NT) * (kSmem + 1024) <= 228 * 1024, "shared memory of the resident CTAs");
};

struct F8Args {
    int units;                 // K / 128
    int tokens;
    __nv_bfloat16* out;
    int64_t out_stride;
    const float* scale;        // [N/128][scale_stride]
    int64_t scale_stride;
    unsigned* counters;
    float* partial;
};

// 8 e4m3 bytes -> 8 bf16 (16 bytes), each bf16(float(w) * s)
__device__ __forceinline__ uint4 dequant8(uint2 w, float s) {
    const uint32_t in[2] = {w.x, w.y};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const __nv_fp8x2_storage_t pair = (__nv_fp8x2_storage_t)((in[i] >> (16 * h)) & 0xffffu);
            const __half2_raw hr = __nv_cvt_fp8x2_to_halfraw2(pair, __NV_E4M3);
            __half2 hv;
            hv = *reinterpret_cast<const __half2*>(&hr);
            const float2 f = __half22float2(hv);
            // both products in one f32x2 multiply (each lane rounded as __fmul_rn; no sum follows,
            // so nothing can be contracted), then rounded to bf16
            unsigned long long xy, ss, pr;
            asm("mov.b64 %0, {%1, %2};" : "=l"(xy) : "f"(f.x), "f"(f.y));
            asm("mov.b64 %0, {%1, %1};" : "=l"(ss) : "f"(s));
            asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(pr) : "l"(xy), "l"(ss));
            float p0, p1;
            asm("mov.b64 {%0, %1}, %2;" : "=f"(p0), "=f"(p1) : "l"(pr));
            o[2 * i + h] = pack_bf16x2(p0, p1);
        }
    }
    return make_uint4(o[0], o[1], o[2], o[3]);
}

template <int NT>
__global__ void __launch_bounds__(kF8Threads, f8_ctas_per_sm(NT))
    linear_fp8_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                      const F8Args a) {
    using Cfg = F8Cfg<NT>;
    constexpr int SA = Cfg::kAStages;
    constexpr int SB = Cfg::kBStages;
    // All shared memory is dynamic, so that its base is the CTA's shared window (1024-aligned) and
    // two CTAs fit per SM without alignment slack: ring X (swizzled, 1024-aligned stages), ring A
    // (swizzled), then the barriers.  A base found misaligned is recorded and the CTA leaves before it touches
    // a barrier or tensor memory.
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if ((smem_u32(smem_raw) & 1023u) != 0u) {
        if (threadIdx.x == 0) record_error(kErrSmemAlign);
        return;
    }
    uint8_t* smem = smem_raw;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kRings);
    uint64_t* a_full = bars;
    uint64_t* a_empty = a_full + SA;
    uint64_t* b_full = a_empty + SA;
    uint64_t* b_empty = b_full + SB;
    uint64_t* done_bar = b_empty + SB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
    int* last_slot = reinterpret_cast<int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int splits = (int)gridDim.x;
    const int split = (int)blockIdx.x;
    const int tile = (int)blockIdx.y;
    const int wrow = tile * kTileRows;
    const int u0 = (int)((int64_t)split * a.units / splits);
    const int nk = (int)((int64_t)(split + 1) * a.units / splits) - u0;   // >= 1 (splits <= units)
    // ring X first (1024-aligned swizzle blocks), then ring A
    auto stage_bx = [&](int s) { return smem + s * Cfg::kBXBytes; };
    auto stage_a = [&](int s) { return smem + SB * Cfg::kBXBytes + s * Cfg::kABytes; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < SA; ++s) {
            mbar_init(&a_full[s], 1);
            mbar_init(&a_empty[s], kF8ConvWarps);
        }
        for (int s = 0; s < SB; ++s) {
            mbar_init(&b_full[s], 1 + kF8ConvWarps);   // the activation load + every dequantizing warp
            mbar_init(&b_empty[s], 1);
        }
        mbar_init(done_bar, 1);
        mbar_fence_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, Cfg::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // The next kernel in the stream may launch once every CTA of this grid has started: its CTAs
    // take the SMs this grid's CTAs leave, and it waits (griddepcontrol.wait) for this grid to
    // complete before it reads anything this grid writes.  (linear_kernel, one CTA per SM and a
    // shorter ramp, measured 1 % slower with this and triggers in its epilogue instead.)
    pdl_trigger();

    if (warp == 0 && lane == 0) {
        // ------------------------------- fp8 weight blocks -------------------------------
        // The first SA blocks stream before this grid waits for the previous kernel in the stream
        // (as linear_kernel does): the weights must not be that kernel's output.
        tma_prefetch_desc(&wmap);
        int i = 0;
        for (; i < nk && i < SA; ++i) {
            mbar_arrive_expect_tx(&a_full[i], Cfg::kABytes);
            tma_load_4d(stage_a(i), &wmap, &a_full[i], (u0 + i) * kF8Unit, wrow, 0, 0);
        }
        pdl_wait();
        for (; i < nk; ++i) {
            const int s = i % SA;
            if (i >= SA && !mbar_wait(&a_empty[s], ((i / SA) - 1) & 1)) break;
            mbar_arrive_expect_tx(&a_full[s], Cfg::kABytes);
            tma_load_4d(stage_a(s), &wmap, &a_full[s], (u0 + i) * kF8Unit, wrow, 0, 0);
        }
        for (int j = (i > SA ? i - SA : 0); j < i; ++j) mbar_wait(&a_full[j % SA], (j / SA) & 1);
    } else if (warp == 2 && lane == 0) {
        // ------------------------------- activations -------------------------------
        tma_prefetch_desc(&xmap);
        pdl_wait();   // the activations may be the previous kernel's output
        int i = 0;
        for (; i < nk; ++i) {
            const int s = i % SB;
            if (i >= SB && !mbar_wait(&b_empty[s], ((i / SB) - 1) & 1)) break;
            mbar_arrive_expect_tx(&b_full[s], Cfg::kBXBytes);
            tma_load_4d(stage_bx(s), &xmap, &b_full[s], 0, 0, (u0 + i) * 2, 0);
        }
        for (int j = (i > SB ? i - SB : 0); j < i; ++j) mbar_wait(&b_full[j % SB], (j / SB) & 1);
    } else if (warp >= kF8ConvWarp0) {
        // ------------------------------- dequantize -------------------------------
        // thread (warp % 4, lane): tile row r = 32 * (warp % 4) + lane, which is its tensor-memory
        // lane; warps 4-7 take k [0, 64) of each block, warps 8-11 k [64, 128)
        const int quad = warp & 3, khalf = (warp - kF8ConvWarp0) >> 2;
        const int r = quad * 32 + lane;
        const uint32_t t_row = tmem + ((uint32_t)(quad * 32) << 16) + Cfg::kACol + (uint32_t)(khalf * 32);
        const float* srow = a.scale + (int64_t)tile * a.scale_stride;
        for (int i = 0; i < nk; ++i) {
            const int sa = i % SA, sb = i % SB;
            if (!mbar_wait(&a_full[sa], (i / SA) & 1)) break;
            if (i >= SB && !mbar_wait(&b_empty[sb], ((i / SB) - 1) & 1)) break;
            // QwenRunner.cpp:103-122: scale.to(bf16), then the bf16 product
            const float sc = __bfloat162float(__float2bfloat16_rn(srow[u0 + i]));
            // the row's 64 fp8 bytes: 16-byte chunks 4 khalf .. + 3, chunk c at (c ^ (r % 8)) in
            // the swizzled block (the 32 rows a warp reads fall in 8 different bank groups)
            const uint8_t* src = stage_a(sa) + r * kF8Unit;
            uint4 w[4];
#pragma unroll
            for (int q = 0; q < 4; ++q)
                w[q] = *reinterpret_cast<const uint4*>(src + ((((uint32_t)(4 * khalf + q)) ^ (uint32_t)(r & 7)) << 4));
            float o[32];   // 64 bf16 of k, two per tensor-memory column
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 lo = dequant8(make_uint2(w[q].x, w[q].y), sc);
                const uint4 hi = dequant8(make_uint2(w[q].z, w[q].w), sc);
                o[8 * q + 0] = __uint_as_float(lo.x); o[8 * q + 1] = __uint_as_float(lo.y);
                o[8 * q + 2] = __uint_as_float(lo.z); o[8 * q + 3] = __uint_as_float(lo.w);
                o[8 * q + 4] = __uint_as_float(hi.x); o[8 * q + 5] = __uint_as_float(hi.y);
                o[8 * q + 6] = __uint_as_float(hi.z); o[8 * q + 7] = __uint_as_float(hi.w);
            }
            tc_fence_after();   // after the MMA that read this stage (b_empty) completed
            tmem_st32(t_row + (uint32_t)(sb * 64), o);
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&b_full[sb]);
                mbar_arrive(&a_empty[sa]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // -------------------------------- MMA issuer --------------------------------
        // D [128 rows, NT] += A [128 rows, 128 k] (tensor memory, stage sb) x B [128 k, NT tokens]
        constexpr uint32_t idesc = idesc_bf16_f32(kTileRows, NT, false);
        constexpr uint32_t x_hi = smem_desc_hi_sw128(1024);
        for (int i = 0; i < nk; ++i) {
            const int s = i % SB;
            if (!mbar_wait(&b_full[s], (i / SB) & 1)) break;
            tc_fence_after();
            const uint32_t xd = smem_desc_lo(smem_u32(stage_bx(s)), 16);
#pragma unroll
            for (int ks = 0; ks < kF8Unit / 16; ++ks)
                tc_mma_ts_w(tmem, tmem + Cfg::kACol + (uint32_t)(s * 64 + ks * 8),
                            xd + (uint32_t)((((ks >> 2) * NT * 128) + (ks & 3) * 32) >> 4), x_hi, idesc,
                            (i > 0 || ks > 0) ? 1u : 0u);
            tc_commit(&b_empty[s]);
        }
        tc_commit(done_bar);
    }
    __syncwarp();

    // --------------------------- epilogue (warps 4-7) ---------------------------
    if (warp >= 4 && warp < 8) {
        const int ew = warp - 4;                 // tensor-memory lane quarter
        mbar_wait(done_bar, 0);
        tc_fence_after();
        const int T = a.tokens;
        const int row = ew * 32 + lane;
        const int64_t ostride = a.out_stride;
        __nv_bfloat16* outp = a.out + wrow;
        const uint32_t t_lane = tmem + ((uint32_t)(ew * 32) << 16);
        float* mine = a.partial + ((size_t)(tile * splits + split) * T) * kTileRows;
#pragma unroll 1
        for (int c = 0; c < T; c += 32) {
            float r[32];
            tmem_ld32(t_lane + (uint32_t)c, r);
            tmem_wait_ld();
            if (splits == 1) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (c + j < T) outp[(int64_t)(c + j) * ostride + row] = __float2bfloat16_rn(r[j]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (c + j < T) mine[(c + j) * kTileRows + row] = r[j];
            }
        }
        if (splits > 1) {
            __threadfence();
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (ew == 0 && lane == 0) *last_slot = atomicAdd(&a.counters[tile], 1u) == (unsigned)(splits - 1);
            asm volatile("bar.sync 2, 128;" ::: "memory");
            if (*last_slot) {
                __threadfence();
                const float* base = a.partial + (size_t)tile * splits * T * kTileRows + 4 * lane;
                __nv_bfloat16* orow = outp + 4 * lane;
                // one token per batch keeps the kernel's registers low
                reduce_partials<1, kMaxSplits>(base, orow, ostride, T, splits, ew);
                if (ew == 0 && lane == 0) a.counters[tile] = 0u;
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, Cfg::kTmemCols);
}

struct F8Plan {
    int tiles = 0, units = 0, splits = 1, nt = 32;
    size_t partial_offset = 0, workspace_bytes = 0;
};

void plan_linear_fp8(int tokens, int64_t out_features, int64_t in_features, int num_sms, F8Plan* p) {
    p->tiles = (int)(out_features / kTileRows);
    p->nt = tokens <= 32 ? 32 : tokens <= 64 ? 64 : 128;
    p->units = (int)(in_features / kF8Unit);
    // splits: the fewest that minimise (waves of CTAs) x (units per CTA), at most 8, at most one
    // per unit, and few enough that the partials stay below about a quarter of the weight bytes
    const int64_t cap = std::max<int64_t>(1, std::min<int64_t>({(int64_t)kMaxSplits, (int64_t)p->units,
                                                                in_features / (8 * (int64_t)std::max(1, tokens))}));
    const int64_t slots = (int64_t)num_sms * f8_ctas_per_sm(p->nt);   // CTAs resident at once
    double best = 1e30;
    p->splits = 1;
    for (int64_t sp = 1; sp <= cap; ++sp) {
        const int64_t waves = ((int64_t)p->tiles * sp + slots - 1) / slots;
        const double cost = (double)waves * (double)((p->units + sp - 1) / sp);
        if (cost < best - 1e-9) {
            best = cost;
            p->splits = (int)sp;
        }
    }
    if (p->tiles > kMaxCounters) p->splits = 1;
    p->partial_offset = kMaxCounters * sizeof(unsigned);
    p->workspace_bytes = p->splits > 1 ? p->partial_offset + (size_t)p->tiles * p->splits * tokens * kTileRows * 4 : 0;
}

int check_linear_fp8_args(int tokens, int64_t in_features, int64_t out_features) {
    if (tokens < 0 || tokens > kF8MaxTokens)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: tokens must be in [0, 128]");
    if (in_features <= 0 || in_features % kF8Unit != 0 || in_features > (int64_t)1 << 30)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: in_features must be a positive multiple of 128");
    if (out_features <= 0 || out_features % kTileRows != 0 || out_features > (1 << 24))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: out_features must be a positive multiple of 128");
    return MLLM_OK;
}

template <int NT>
int launch_linear_fp8(const CUtensorMap& wmap, const CUtensorMap& xmap, const F8Args& a, const F8Plan& p,
                      cudaStream_t s) {
    using Cfg = F8Cfg<NT>;
    auto kern = linear_fp8_kernel<NT>;
    if (int st = check_cuda(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem),
                            "linear_fp8: shared memory attribute"))
        return st;
    return check_cuda(launch_pdl(kern, dim3(p.splits, p.tiles, 1), dim3(kF8Threads, 1, 1), (size_t)Cfg::kSmem, s,
                                 wmap, xmap, a),
                      "linear_fp8 launch");
}

}  // namespace

MLLM_DEFINE_STATUS_READER(linear)

}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" size_t mllm_linear_workspace_size(int tokens, int num_weights, const int64_t* out_features,
                                             int64_t in_features) {
    int64_t total = 0;
    if (check_linear_args(tokens, in_features, num_weights, nullptr, nullptr, out_features, &total) != MLLM_OK) {
        ok();
        return 0;
    }
    LinearPlan p;
    plan_linear(tokens, num_weights, out_features, in_features, sm_count_or_default(), &p);
    return p.workspace_bytes;
}

extern "C" int mllm_linear_bf16(const void* x, int64_t x_stride, int tokens, int64_t in_features, int num_weights,
                                const void* const* weights, const int64_t* weight_strides,
                                const int64_t* out_features, void* out, int64_t out_stride, void* workspace,
                                size_t workspace_bytes, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_linear_bf16");
    int64_t total = 0;
    if (!weights) return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: weights must be given");
    if (int st = check_linear_args(tokens, in_features, num_weights, weights, weight_strides, out_features, &total))
        return st;
    if (tokens == 0) return ok();
    if (!x || !out || x_stride < in_features || out_stride < total)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: bad activation or output pointer/stride");
    if (!aligned(out, 16) || out_stride % 8 != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: output must be 16-byte aligned with a stride multiple of 8");
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;
    LinearPlan p;
    plan_linear(tokens, num_weights, out_features, in_features, num_sms, &p);
    if (p.tiles > 65535) return fail(MLLM_ERR_INVALID_ARGUMENT, "linear: too many output rows");
    if (p.workspace_bytes > 0 && (!workspace || workspace_bytes < p.workspace_bytes || !aligned(workspace, 256)))
        return fail(MLLM_ERR_INVALID_ARGUMENT,
                    "linear: workspace missing, not 256-byte aligned or smaller than mllm_linear_workspace_size");

    const int nb = p.nt <= 64 ? LinCfg<32>::kNB : LinCfg<128>::kNB;
    LinearMaps maps;
    memset(&maps, 0, sizeof(maps));
    LinearArgs a = {};
    int tile = 0;
    int64_t col = 0;
    for (int i = 0; i < kMaxWeights; ++i) {
        a.tile_begin[i] = tile;
        if (i < num_weights) {
            // {64 k, rows, k-atoms}: box 8 rows x NB atoms (see LinCfg)
            if (int st = encode_kv_map(&maps.w[i], weights[i], kAtomK, out_features[i], in_features / kAtomK, 1,
                                       weight_strides[i], kAtomK, weight_strides[i] * out_features[i], kAtomK, 8,
                                       (uint32_t)nb))
                return st;
            a.out_col[i] = col;
            col += out_features[i];
            tile += (int)(out_features[i] / kTileRows);
        }
    }
    a.tile_begin[kMaxWeights] = tile;   // unused weights begin at the end: no tile selects them
    if (int st = encode_kv_map(&maps.x, x, kAtomK, tokens, in_features / kAtomK, 1, x_stride, kAtomK,
                               x_stride * tokens, kAtomK, (uint32_t)p.nt, (uint32_t)nb))
        return st;
    a.units = p.units;
    a.tokens = tokens;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.out_stride = out_stride;
    a.counters = static_cast<unsigned*>(workspace);
    a.partial = p.workspace_bytes ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.partial_offset)
                                  : nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    int st;
    switch (p.nt) {
        case 32: st = launch_linear<32>(maps, a, p, s); break;
        case 64: st = launch_linear<64>(maps, a, p, s); break;
        case 128: st = launch_linear<128>(maps, a, p, s); break;
        default: st = launch_linear<256>(maps, a, p, s); break;
    }
    return st ? st : ok();
}

extern "C" size_t mllm_linear_fp8_workspace_size(int tokens, int64_t out_features, int64_t in_features) {
    if (check_linear_fp8_args(tokens, in_features, out_features) != MLLM_OK) {
        ok();
        return 0;
    }
    F8Plan p;
    plan_linear_fp8(tokens, out_features, in_features, sm_count_or_default(), &p);
    return p.workspace_bytes;
}

extern "C" int mllm_linear_fp8_bf16(const void* x, int64_t x_stride, int tokens, int64_t in_features,
                                    const void* weight, int64_t weight_stride, int64_t out_features,
                                    const float* weight_scale_inv, int64_t scale_stride, void* out,
                                    int64_t out_stride, void* workspace, size_t workspace_bytes,
                                    mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_linear_fp8_bf16");
    if (int st = check_linear_fp8_args(tokens, in_features, out_features)) return st;
    if (tokens == 0) return ok();
    if (!x || !weight || !weight_scale_inv || !out)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: null pointer");
    if (x_stride < in_features || out_stride < out_features || weight_stride < in_features ||
        scale_stride < in_features / kF8Unit)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: a row stride is below the row length");
    if (!aligned(out, 16) || out_stride % 8 != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: output must be 16-byte aligned with a stride multiple of 8");
    if (!aligned(weight, 16) || weight_stride % 16 != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: weight rows must be 16-byte aligned");
    int num_sms = 0;
    if (int st = require_sm100(&num_sms)) return st;
    F8Plan p;
    plan_linear_fp8(tokens, out_features, in_features, num_sms, &p);
    if (p.tiles > 65535) return fail(MLLM_ERR_INVALID_ARGUMENT, "linear_fp8: too many output rows");
    if (p.workspace_bytes > 0 && (!workspace || workspace_bytes < p.workspace_bytes || !aligned(workspace, 256)))
        return fail(MLLM_ERR_INVALID_ARGUMENT,
                    "linear_fp8: workspace missing, not 256-byte aligned or smaller than mllm_linear_fp8_workspace_size");
    CUtensorMap wmap, xmap;
    if (int st = encode_u8_map(&wmap, weight, in_features, out_features, weight_stride, kF8Unit, kTileRows, true))
        return st;
    // activations {64 k, tokens, k-atoms}: box NT rows x 2 atoms (one 128-k unit)
    if (int st = encode_kv_map(&xmap, x, kAtomK, tokens, in_features / kAtomK, 1, x_stride, kAtomK,
                               x_stride * tokens, kAtomK, (uint32_t)p.nt, 2))
        return st;
    F8Args a = {};
    a.units = p.units;
    a.tokens = tokens;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.out_stride = out_stride;
    a.scale = weight_scale_inv;
    a.scale_stride = scale_stride;
    a.counters = static_cast<unsigned*>(workspace);
    a.partial = p.workspace_bytes ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + p.partial_offset)
                                  : nullptr;
    cudaStream_t s = (cudaStream_t)stream;
    int st;
    switch (p.nt) {
        case 32: st = launch_linear_fp8<32>(wmap, xmap, a, p, s); break;
        case 64: st = launch_linear_fp8<64>(wmap, xmap, a, p, s); break;
        default: st = launch_linear_fp8<128>(wmap, xmap, a, p, s); break;
    }
    return st ? st : ok();
}
