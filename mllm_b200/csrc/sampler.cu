// Token sampling on the device: Sampler::Sample (src/core/runtime/Sampler.cpp:49-232) for a
// batch of logit rows, with no host round trip.
//
// The reference applies the repetition penalty with one `.item()` per previous token
// (Sampler.cpp:12-46, a device sync each when the logits live on the GPU), then takes a greedy
// argmax or samples (softmax / temperature, top-k, top-p, multinomial).  Here one CTA of
// kThreads threads takes one row:
//   penalty   in place, like the reference: every previous-token entry adds one to a per-token
//             counter (caller workspace); the first entry to take a token's count applies the
//             penalty that many times, re-rounding to the logits' dtype after each application
//             as the reference's tensor write does.  Only the touched counters are reset, so
//             the workspace needs no clearing.
//   greedy    argmax with the first index winning ties and NaN above every number (the
//             documented torch::argmax behaviour).
//   sampling  fp32 softmax of logits / temperature; top-k keeps the scores >= the k-th largest
//             (found by a 32-step bisection over the ordered bit patterns of the scores); top-p
//             then keeps the largest scores whose renormalised mass, accumulated from the top,
//             stays <= top_p, always keeping the top one (again by bisection); one uniform draw
//             from a Philox-4x32-10 stream (seed, row, offset) picks the token by a block-wide
//             prefix sum in vocabulary order.  Ties at a top-k or top-p cut are all kept (the
//             reference's sort breaks them arbitrarily).
#include <cmath>

#include "common.cuh"
#include "host_util.h"

namespace mllm_b200 {
namespace {

constexpr int kThreads = 1024;
constexpr int kWarps = kThreads / 32;

struct SampleArgs {
    void* logits;
    bool bf16;
    int64_t row_stride;
    int vocab;
    const int64_t* prev;
    int64_t prev_stride;
    const int32_t* prev_counts;
    int32_t* counts;          // [batch, vocab] scratch
    float temperature;
    int top_k;
    float top_p;
    bool greedy;
    float penalty;
    uint64_t seed, offset;
    int64_t* out;
};

__device__ __forceinline__ float load_logit(const SampleArgs& a, int64_t i) {
    return a.bf16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(a.logits)[i])
                  : reinterpret_cast<const float*>(a.logits)[i];
}

__device__ __forceinline__ void store_logit(const SampleArgs& a, int64_t i, float v) {
    if (a.bf16)
        reinterpret_cast<__nv_bfloat16*>(a.logits)[i] = __float2bfloat16_rn(v);
    else
        reinterpret_cast<float*>(a.logits)[i] = v;
}

// Ordered key of a float: larger float -> larger unsigned key (NaN above +inf).
__device__ __forceinline__ uint32_t float_key(float f) {
    if (f != f) return 0xFFFFFFFFu;
    const uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Block-wide reductions over kThreads threads (scratch: kWarps words).
template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, Op op, T* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    v = scratch[lane < kWarps ? lane : 0];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Philox-4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3",
// SC 2011): ten rounds of the multiply-xor bijection with the paper's round constants.
__device__ __forceinline__ uint32_t philox_first(uint32_t c0, uint32_t c1, uint32_t c2, uint32_t c3, uint32_t k0,
                                                 uint32_t k1) {
    constexpr uint32_t kM0 = 0xD2511F53u, kM1 = 0xCD9E8D57u, kW0 = 0x9E3779B9u, kW1 = 0xBB67AE85u;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
        const uint32_t hi0 = __umulhi(kM0, c0), lo0 = kM0 * c0;
        const uint32_t hi1 = __umulhi(kM1, c2), lo1 = kM1 * c2;
        c0 = hi1 ^ c1 ^ k0;
        c1 = lo1;
        c2 = hi0 ^ c3 ^ k1;
        c3 = lo0;
        k0 += kW0;
        k1 += kW1;
    }
    return c0;
}

__global__ void __launch_bounds__(kThreads, 1) sample_kernel(SampleArgs a) {
    __shared__ float sf[kWarps];
    __shared__ uint32_t su[kWarps];
    __shared__ int si[kWarps];
    __shared__ float s_chunk[kThreads];
    const int b = blockIdx.x;
    const int t = threadIdx.x;
    const int V = a.vocab;
    const int64_t row = (int64_t)b * a.row_stride;

    // ---------------- repetition penalty (Sampler.cpp:12-46), in place ----------------
    if (a.penalty > 1.0f && a.prev_counts != nullptr) {
        const int n = max(0, a.prev_counts[b]);
        const int64_t* hist = a.prev + (int64_t)b * a.prev_stride;
        int32_t* cnt = a.counts + (int64_t)b * V;
        for (int i = t; i < n; i += kThreads) {
            const int64_t tok = hist[i];
            if (tok >= 0 && tok < V) cnt[tok] = 0;
        }
        __syncthreads();
        for (int i = t; i < n; i += kThreads) {
            const int64_t tok = hist[i];
            if (tok >= 0 && tok < V) atomicAdd(&cnt[tok], 1);
        }
        __syncthreads();
        for (int i = t; i < n; i += kThreads) {
            const int64_t tok = hist[i];
            if (tok < 0 || tok >= V) continue;
            const int c = atomicExch(&cnt[tok], 0);   // one entry per token takes the whole count
            float v = load_logit(a, row + tok);
            for (int k = 0; k < c; ++k) {
                v = (v < 0.0f) ? __fmul_rn(v, a.penalty) : __fdiv_rn(v, a.penalty);
                if (a.bf16) v = __bfloat162float(__float2bfloat16_rn(v));   // the tensor write rounds
            }
            if (c > 0) store_logit(a, row + tok, v);
        }
        __syncthreads();
    }

    // ---------------- greedy: argmax (Sampler.cpp:128-140) ----------------
    // key order: NaN above everything, larger value, then smaller index
    uint32_t bk = 0;
    int bi = V;
    float m = -INFINITY;
    for (int i = t; i < V; i += kThreads) {
        const float v = load_logit(a, row + i);
        const uint32_t k = float_key(v);
        if (bi == V || k > bk) { bk = k; bi = i; }
        m = fmaxf(m, v);
    }
    const uint32_t best_key = block_reduce(bk, [](uint32_t x, uint32_t y) { return x > y ? x : y; }, su);
    const int best_idx = block_reduce(bk == best_key ? bi : V, [](int x, int y) { return x < y ? x : y; }, si);
    if (a.greedy) {
        if (t == 0) a.out[b] = best_idx;
        return;
    }

    // ---------------- sampling (Sampler.cpp:142-231) ----------------
    const float inv_t = 1.0f / a.temperature;
    const float mx = block_reduce(m, [](float x, float y) { return fmaxf(x, y); }, sf) * inv_t;
    float z = 0.f;
    for (int i = t; i < V; i += kThreads) z += __expf(load_logit(a, row + i) * inv_t - mx);
    const float Z = block_reduce(z, [](float x, float y) { return x + y; }, sf);
    auto prob = [&](int i) { return __expf(load_logit(a, row + i) * inv_t - mx) / Z; };
    auto key_at = [&](int i) { return float_key(load_logit(a, row + i)); };

    // top-k: the k-th largest key; keep keys >= it
    uint32_t kmin = 0;
    if (a.top_k > 0 && a.top_k < V) {
        uint32_t lo = 0, hi = 0xFFFFFFFFu;   // largest key with count(key >= .) >= k
        for (int it = 0; it < 33 && lo < hi; ++it) {
            const uint32_t mid = lo + (uint32_t)(((uint64_t)hi - lo + 1) >> 1);
            int c = 0;
            for (int i = t; i < V; i += kThreads) c += key_at(i) >= mid;
            c = block_reduce(c, [](int x, int y) { return x + y; }, si);
            if (c >= a.top_k) lo = mid; else hi = mid - 1;
        }
        kmin = lo;
    }
    // top-p over the kept set: the smallest key c whose mass of keys >= c is <= top_p (renormalised)
    float km = 0.f;
    for (int i = t; i < V; i += kThreads) km += key_at(i) >= kmin ? prob(i) : 0.f;
    const float kept_mass = block_reduce(km, [](float x, float y) { return x + y; }, sf);
    uint32_t pmin = kmin;
    if (a.top_p < 1.0f) {
        uint32_t lo = kmin, hi = 0xFFFFFFFFu;   // smallest key with mass(key >= .) <= top_p
        for (int it = 0; it < 33 && lo < hi; ++it) {
            const uint32_t mid = lo + (uint32_t)(((uint64_t)hi - lo) >> 1);
            float s = 0.f;
            for (int i = t; i < V; i += kThreads) {
                const uint32_t k = key_at(i);
                s += (k >= kmin && k >= mid) ? prob(i) : 0.f;
            }
            s = block_reduce(s, [](float x, float y) { return x + y; }, sf) / kept_mass;
            if (s <= a.top_p) hi = mid; else lo = mid + 1;
        }
        pmin = lo > best_key ? best_key : lo;   // the top token is always kept
    }
    // multinomial: one uniform draw over the kept mass, located by a prefix sum in vocab order
    const int chunk = (V + kThreads - 1) / kThreads;
    const int c0 = t * chunk, c1 = min(V, c0 + chunk);
    float cs = 0.f;
    for (int i = c0; i < c1; ++i) cs += key_at(i) >= pmin ? prob(i) : 0.f;
    s_chunk[t] = cs;
    __syncthreads();
    if (t == 0) {
        float acc = 0.f;
        for (int i = 0; i < kThreads; ++i) { const float v = s_chunk[i]; s_chunk[i] = acc; acc += v; }
        const uint32_t r = philox_first((uint32_t)a.offset, (uint32_t)(a.offset >> 32), (uint32_t)b, 0u,
                                        (uint32_t)a.seed, (uint32_t)(a.seed >> 32));
        sf[0] = (float)(r >> 8) * (1.0f / 16777216.0f) * acc;   // u in [0, total)
        si[0] = best_idx;                                         // fallback: rounding at the very end
    }
    __syncthreads();
    const float u = sf[0];
    const float start = s_chunk[t];
    const float next = (t + 1 < kThreads) ? s_chunk[t + 1] : INFINITY;
    if (u >= start && u < next && c0 < c1) {
        float acc = start;
        int pick = -1;
        for (int i = c0; i < c1; ++i) {
            if (key_at(i) < pmin) continue;
            pick = i;
            acc += prob(i);
            if (u < acc) break;
        }
        if (pick >= 0) si[0] = pick;
    }
    __syncthreads();
    if (t == 0) a.out[b] = si[0];
}

}  // namespace
}  // namespace mllm_b200

using namespace mllm_b200;

extern "C" size_t mllm_sample_workspace_size(int batch, int vocab) {
    if (batch <= 0 || vocab <= 0) return 0;
    return ((size_t)batch * vocab * sizeof(int32_t) + 255) & ~size_t(255);
}

extern "C" int mllm_sample(void* logits, int logits_bf16, int64_t row_stride, int batch, int vocab,
                           const int64_t* prev_tokens, int64_t prev_stride, const int32_t* prev_counts,
                           float temperature, int top_k, float top_p, int use_greedy, float repetition_penalty,
                           uint64_t seed, uint64_t offset, int64_t* out_tokens, void* workspace,
                           size_t workspace_bytes, mllm_stream_t stream) {
    MLLM_NVTX_RANGE("mllm_sample");
    // the reference's checks (Sampler.cpp:59-81)
    if (vocab <= 0) return fail(MLLM_ERR_INVALID_ARGUMENT, "Sampler received empty logits.");
    if (!std::isfinite(temperature)) return fail(MLLM_ERR_INVALID_ARGUMENT, "Sampler temperature must be finite.");
    if (!std::isfinite(top_p) || top_p <= 0.0f) return fail(MLLM_ERR_INVALID_ARGUMENT, "Sampler top_p must be in (0, 1].");
    if (batch < 0 || row_stride < vocab) return fail(MLLM_ERR_INVALID_ARGUMENT, "sample: bad sizes");
    if ((prev_tokens == nullptr) != (prev_counts == nullptr))
        return fail(MLLM_ERR_INVALID_ARGUMENT, "sample: give both prev_tokens and prev_counts or neither");
    if (batch == 0) return ok();
    if (!logits || !out_tokens) return fail(MLLM_ERR_INVALID_ARGUMENT, "sample: null pointer");
    const bool penalise = repetition_penalty > 1.0f && prev_counts != nullptr;
    if (penalise && (!workspace || workspace_bytes < mllm_sample_workspace_size(batch, vocab)))
        return fail(MLLM_ERR_WORKSPACE, "sample: the repetition penalty needs mllm_sample_workspace_size() bytes");
    if (int st = require_sm100()) return st;
    SampleArgs a;
    a.logits = logits;   // the penalty is applied in place, as in the reference
    a.bf16 = logits_bf16 != 0;
    a.row_stride = row_stride;
    a.vocab = vocab;
    a.prev = prev_tokens;
    a.prev_stride = prev_stride;
    a.prev_counts = prev_counts;
    a.counts = reinterpret_cast<int32_t*>(workspace);
    a.temperature = temperature;
    a.top_k = top_k;
    a.top_p = top_p < 1.0f ? top_p : 1.0f;
    a.greedy = use_greedy != 0 || temperature <= 0.0f;
    a.penalty = repetition_penalty;
    a.seed = seed;
    a.offset = offset;
    a.out = out_tokens;
    sample_kernel<<<batch, kThreads, 0, (cudaStream_t)stream>>>(a);
    if (int st = check_cuda(cudaGetLastError(), "sample launch")) return st;
    return ok();
}
