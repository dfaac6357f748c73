/*
 * mllm_attn.h -- C ABI of the B200 (sm_100a) attention path for the mLLM runtime.
 *
 * The mLLM runtime (pym2282/mLLM) runs attention as a chain of LibTorch calls inside
 * `mllm::TransformerBlock::Forward` / `mllm::Attention::ForwardProjected`.  This library
 * replaces that chain with three kernel families behind plain C entry points:
 *
 *   mllm_qkv_epilogue_bf16      per-head QK-RMSNorm + RoPE + KV-cache append, one kernel
 *   mllm_prefill_attention_bf16 causal GQA attention over the cache (tcgen05 / TMEM / TMA)
 *   mllm_decode_attention_bf16  split-K flash-decode over the cache (HBM-bound)
 *   mllm_decode_step_bf16       the epilogue of one new token per sequence fused into decode
 *   mllm_*_paged_bf16           the same four over a paged KV cache (block tables)
 *   mllm_*_varlen_*             epilogue and prefill over packed sequences of different
 *                               lengths (several prompts in one launch each)
 *   mllm_sample                 Sampler::Sample on the device (penalty, greedy / top-k / top-p)
 *
 * plus the RoPE table builder and RoPE apply that back the `mllm::RoPE` facade.
 *
 * Conventions
 *   - All tensor arguments are raw DEVICE pointers (e.g. `tensor.data_ptr()` of a CUDA
 *     LibTorch tensor) on the current CUDA device; sizes and strides are in ELEMENTS.
 *   - `head_dim` is the innermost, contiguous dimension of every tensor.
 *   - Every call is asynchronous on `stream` (NULL = the legacy default stream) and
 *     returns an mllm_status; no C++ exception crosses this boundary.  Argument errors are
 *     detected on the host before anything is launched.
 *   - The attention, sampling and projection entry points never allocate device memory;
 *     callers pass workspaces.  Only mllm_ipc_alloc (the shared buffers of the tensor-parallel
 *     exchange) and the communicator set-up of mllm_comm_* allocate, once, at set-up.
 *   - Not thread-safe per stream, like the reference runtime (one Generate at a time).
 */
#ifndef MLLM_ATTN_H_
#define MLLM_ATTN_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define MLLM_API __attribute__((visibility("default")))
#else
#define MLLM_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream (the header needs no CUDA include). */
typedef struct CUstream_st* mllm_stream_t;

typedef enum mllm_status {
    MLLM_OK = 0,
    MLLM_ERR_INVALID_ARGUMENT = 1, /* shape, stride, alignment or pointer rejected on the host */
    MLLM_ERR_UNSUPPORTED = 2,      /* valid request this library does not implement (e.g. head_dim) */
    MLLM_ERR_CUDA = 3,             /* a CUDA runtime / driver call failed */
    MLLM_ERR_WORKSPACE = 4,        /* workspace missing or smaller than *_workspace_size() */
    MLLM_ERR_NO_DEVICE = 5,        /* current device is not sm_100 */
    MLLM_ERR_DEVICE_TIMEOUT = 6,   /* a kernel's bounded wait expired (see mllm_attn_device_status) */
    MLLM_ERR_DEVICE_LENGTH = 7,    /* a device-side length exceeded its host-given capacity */
    MLLM_ERR_COMM = 8,             /* a communicator failed (NCCL error, a peer lost) or was aborted */
    MLLM_ERR_COMM_TIMEOUT = 9      /* a collective ran past its deadline; the communicator was aborted */
} mllm_status;

/* Version of this ABI (bumped on any signature change). */
MLLM_API int mllm_attn_abi_version(void);

/* Static description of a status code. */
MLLM_API const char* mllm_attn_status_string(int status);

/* Detail message of the last failing call on this host thread ("" if none). */
MLLM_API const char* mllm_attn_last_error(void);

/* Reads and clears the device-side status word of the current device (synchronises
 * `stream`).  Returns MLLM_OK, MLLM_ERR_DEVICE_TIMEOUT or MLLM_ERR_DEVICE_LENGTH. */
MLLM_API int mllm_attn_device_status(mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * RoPE table.  Replaces mllm::RoPE::BuildCosSin (src/core/runtime/RoPE.h:29-59):
 *   inv_freq[j] = exp(-(2j / D) * ln(theta)),  angle = float(pos) * inv_freq[j],
 *   cos/sin[s, j] = cos/sin[s, j + D/2] = cos/sin(angle)          all in fp32.
 * positions: int64 [n]; cos_out / sin_out: fp32 [n, head_dim] (row-major). */
MLLM_API int mllm_rope_build_cos_sin(const int64_t* positions, int64_t n, int head_dim, double rope_theta,
                            float* cos_out, float* sin_out, mllm_stream_t stream);

/* RoPE apply.  Replaces mllm::RoPE::Apply (src/core/runtime/RoPE.h:68-89) for bf16 input:
 *   out = bf16(x*cos + cat(-x2, x1)*sin), each product and the sum rounded in fp32.
 * x: bf16 [B, H, S, D] with element strides (x_stride_b, x_stride_h, x_stride_s);
 * cos/sin: fp32 [S, D]; out: bf16 [B, H, S, D] contiguous. */
MLLM_API int mllm_rope_apply_bf16(const void* x, int64_t x_stride_b, int64_t x_stride_h, int64_t x_stride_s,
                         int batch, int num_heads, int seq_len, int head_dim, const float* cos,
                         const float* sin, void* out, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Fused QKV epilogue.  Replaces, in one kernel:
 *   - the Qwen3 per-head RMSNorm of q and k   (src/core/runtime/TransformerBlock.h:103-107,
 *     130-134 via RMSNorm::Forward, src/core/runtime/RMSNorm.h:27-64), when the norm weights
 *     are given;
 *   - RoPE on q and k                          (src/core/runtime/Attention.h:157-177);
 *   - the KV-cache append                      (src/core/runtime/Attention.h:183-208): rows
 *     are written in place instead of torch::cat-ing the whole cache.
 *
 * Inputs (token (b, s), head h, element d; all bf16, d contiguous):
 *   q + b*q_sb + s*q_ss + h*q_sh      h < num_heads        (projected q, pre-norm)
 *   k + b*k_sb + s*k_ss + h*k_sh      h < num_kv_heads
 *   v + b*v_sb + s*v_ss + h*v_sh      h < num_kv_heads
 * RoPE angle source, per token:
 *   rope_cos/rope_sin != NULL: fp32 tables of row length head_dim (the BuildCosSin layout);
 *       token (b, s) uses row  b*rope_row_sb + s*rope_row_ss;
 *   else: computed in-kernel from positions[b*pos_sb + s*pos_ss] and rope_theta with the
 *       same fp32 steps as mllm_rope_build_cos_sin (bit-identical to that table).
 * q_norm_weight / k_norm_weight: bf16 [head_dim] (both given, or both NULL for Llama).
 * Outputs:
 *   q_out: bf16 [batch, num_heads, seq_len, head_dim] contiguous (post-norm, post-RoPE)
 *   k_cache/v_cache row for (b, h, slot = cache_start[b] + s) at
 *       cache + b*cache_sb + h*cache_sh + slot*cache_st
 *   cache_start: int32 device [batch], or NULL for a batch-uniform start row
 *       `uniform_cache_start`; slots must lie below cache_capacity (checked on the device:
 *       out-of-range rows are skipped and MLLM_ERR_DEVICE_LENGTH is recorded). */
MLLM_API int mllm_qkv_epilogue_bf16(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                           const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                           const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                           int batch, int seq_len, int num_heads, int num_kv_heads, int head_dim,
                           const int64_t* positions, int64_t pos_sb, int64_t pos_ss, double rope_theta,
                           const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                           int64_t rope_row_ss,
                           const void* q_norm_weight, const void* k_norm_weight, double rms_norm_eps,
                           void* q_out,
                           void* k_cache, void* v_cache, int64_t cache_sb, int64_t cache_sh,
                           int64_t cache_st, int64_t cache_capacity, const int32_t* cache_start,
                           int64_t uniform_cache_start, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Causal GQA prefill.  Replaces src/core/runtime/Attention.h:220-316 (repeat_interleave
 * GQA expand, fp32 scores * scale, triu causal mask, fp32 softmax, bf16 P, P.V, merge heads)
 * for q_len >= 1 new rows against kv_len >= q_len cached rows; query row s sits at absolute
 * position kv_len - q_len + s and sees cache rows 0 .. kv_len - q_len + s.
 *   q:   bf16 [batch, num_heads, q_len, head_dim] contiguous (mllm_qkv_epilogue_bf16 q_out)
 *   k_cache/v_cache: row (b, kvh, t) at cache + b*cache_sb + kvh*cache_sh + t*cache_st;
 *        strides multiples of 8 elements, base 16-byte aligned (TMA); at least kv_len rows.
 *   out: bf16 [batch, q_len, num_heads*head_dim]  (the o_proj input layout)
 * q head h reads kv head h / (num_heads / num_kv_heads).  head_dim 64 or 128. */
MLLM_API int mllm_prefill_attention_bf16(const void* q, const void* k_cache, const void* v_cache,
                                int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                int batch, int num_heads, int num_kv_heads, int head_dim,
                                int q_len, int kv_len, float softmax_scale, void* out,
                                mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Split-K flash-decode.  Replaces src/core/runtime/Attention.h:183-316 at S == 1 (the
 * decode step of LlamaRunner.cpp:204-232 / QwenRunner.cpp:301-324), generalised to a
 * per-sequence cache length (ragged batches).
 *   q:      bf16 [batch, num_heads, head_dim] contiguous
 *   caches: as for prefill; max_kv_len = rows addressable per (b, kv head)
 *   kv_lens: int32 device [batch], the number of valid rows of each sequence (new token
 *            included); values are clamped to [0, max_kv_len] on the device and an
 *            out-of-range value records MLLM_ERR_DEVICE_LENGTH.  NULL: every sequence has
 *            max_kv_len rows (the batch-uniform cache of the reference runners).
 *   out:    bf16 [batch, num_heads*head_dim]
 *   workspace: device scratch of at least mllm_decode_attention_workspace_size() bytes,
 *            256-byte aligned.  Its first 256 bytes hold the counter from which the persistent
 *            CTAs take work items: they must be zero before the first call, and every call
 *            leaves them zero, so one workspace serves any number of calls of any shape in one
 *            stream (not concurrent calls).  The rest needs no initialisation. */
MLLM_API size_t mllm_decode_attention_workspace_size(int batch, int num_heads, int num_kv_heads, int head_dim,
                                            int max_kv_len);

/* How a decode call of this shape on the current device is split: rows per chunk, chunks per
 * (sequence, kv head) and kernel launches per call (1: one chunk each, no combine; 2: the split
 * kernel and the combine).  Any output pointer may be NULL.  Applies to every decode entry point
 * (plain, paged, fused step, no-alloc). */
MLLM_API int mllm_decode_attention_plan(int batch, int num_heads, int num_kv_heads, int head_dim, int max_kv_len,
                                        int* chunk_rows, int* chunks, int* launches);

MLLM_API int mllm_decode_attention_bf16(const void* q, const void* k_cache, const void* v_cache,
                               int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                               const int32_t* kv_lens, int batch, int num_heads, int num_kv_heads,
                               int head_dim, int max_kv_len, float softmax_scale, void* out,
                               void* workspace, size_t workspace_bytes, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Split-K flash-decode that allocates nothing and takes no workspace.  It has no counterpart
 * in the reference: it exists for callers that cannot allocate device memory when they run
 * decode (a runtime whose device memory is carved up once by its own arena, code running
 * under another framework's allocator lock, or a path where an allocation would be a
 * synchronising call).
 *   Arguments and results are those of mllm_decode_attention_bf16 without the workspace.
 *   The split-K partials live in one 16 MiB scratch array compiled into this library; each
 *   GPU that loads the library keeps that array resident until the process exits.  A batch
 *   whose mllm_decode_attention_workspace_size() exceeds 16 MiB is rejected with
 *   MLLM_ERR_WORKSPACE (C2-sized work -- 32 sequences x 8 kv heads x 4096 rows at
 *   head_dim 128 -- needs about 8.1 MiB).
 *   The first call in each CUDA context of a device (the first call of the process, and the
 *   first after cudaDeviceReset or after the primary context was released and made again)
 *   looks up the array's device address (cudaGetSymbolAddress) and caches it under the
 *   context's ID; make that first call before any CUDA stream capture begins.
 *   All calls on a device share the array, which keeps the previous call's contents.  Its
 *   first 256 bytes are the work-item counter of the decode workspace: zero from the start
 *   (static storage) and set back to zero by every call that uses it -- by the combine kernel,
 *   or, when a call fails after its split kernel was launched, by a memset queued behind it;
 *   the partials after it are always written earlier in a call than they are read, so nothing
 *   needs clearing.  Only a failed CUDA context (after which nothing in it is usable) can
 *   leave the counter dirty.  Calls that overlap on the GPU -- concurrent streams, or several
 *   host threads -- race on it: serialise them. */
MLLM_API int mllm_decode_attention_noalloc_bf16(const void* q, const void* k_cache, const void* v_cache,
                                                int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                                const int32_t* kv_lens, int batch, int num_heads,
                                                int num_kv_heads, int head_dim, int max_kv_len,
                                                float softmax_scale, void* out, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Fused decode step.  Replaces, for one new token per sequence, the whole attention step
 * between the projections and o_proj: TransformerBlock.h:103-107,130-134 (per-head QK-norm),
 * Attention.h:157-208 (RoPE + KV append) and Attention.h:183-316 at S == 1 -- i.e.
 * mllm_qkv_epilogue_bf16 with seq_len 1 followed by mllm_decode_attention_bf16, as one
 * launch of the split kernel (plus its combine kernel when a sequence spans several chunks).
 * The cache rows it writes are bit-identical to mllm_qkv_epilogue_bf16's; the attention
 * output equals mllm_decode_attention_bf16's up to fp32 summation order.
 *   q: bf16 head h of sequence b at q + b*q_sb + h*q_sh (head_dim contiguous); k, v likewise
 *      for the kv heads (strided views of the q/k/v projections)
 *   positions: int64 device, RoPE position of sequence b at positions[b*pos_sb] (pos_sb = 0:
 *      one position for the batch), used when rope_cos/rope_sin are NULL; otherwise fp32
 *      tables with sequence b's row at rope_row_sb*b ([rows, head_dim], halves duplicated)
 *   q_norm_weight / k_norm_weight: bf16 [head_dim] (both, or both NULL for Llama)
 *   kv_lens: int32 device [batch]: rows of each sequence INCLUDING the new token, which is
 *      written to row kv_lens[b] - 1; every value must lie in [1, max_kv_len] (a value outside
 *      records MLLM_ERR_DEVICE_LENGTH; a zero length yields a zero output row).  NULL: every
 *      sequence has max_kv_len rows.
 *   caches, max_kv_len, out, workspace: as for mllm_decode_attention_bf16 (same
 *      workspace size). */
MLLM_API int mllm_decode_step_bf16(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb,
                                   int64_t k_sh, const void* v, int64_t v_sb, int64_t v_sh,
                                   const int64_t* positions, int64_t pos_sb, double rope_theta,
                                   const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                                   const void* q_norm_weight, const void* k_norm_weight, double rms_norm_eps,
                                   void* k_cache, void* v_cache, int64_t cache_sb, int64_t cache_sh,
                                   int64_t cache_st, const int32_t* kv_lens, int batch, int num_heads,
                                   int num_kv_heads, int head_dim, int max_kv_len, float softmax_scale, void* out,
                                   void* workspace, size_t workspace_bytes, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Paged KV cache (the serving format; no counterpart in the reference, whose KVCache is one
 * contiguous tensor per layer grown by torch::cat, KVCache.h:9-28 / Attention.h:189-207).
 * Rows of all sequences live in fixed-size blocks of one pool per layer, and each sequence
 * owns a list of blocks, so sequences of any length share the memory without padding to the
 * longest (the natural step toward the batched Generate the reference lacks,
 * QwenRunner.cpp:459-473).
 *   k_pool / v_pool: bf16; row r of block n for kv head h at
 *       pool + n*block_stride + h*head_stride + r*row_stride    (elements; row_stride and
 *       head_stride multiples of 8, pool 16-byte aligned)
 *   block_size: rows per block, a multiple of 128 (one attention tile never straddles blocks)
 *   block_table: int32 device; block i of sequence b is block_table[b*table_stride + i], and
 *       cache row t of sequence b is row t % block_size of block block_table[b*table_stride +
 *       t / block_size].  Entries must lie in [0, num_blocks); a bad entry records
 *       MLLM_ERR_DEVICE_LENGTH and reads block 0 instead (writes to it are skipped).
 *   max_blocks_per_seq: entries per sequence; rows beyond max_blocks_per_seq*block_size are
 *       rejected like rows beyond a contiguous cache's capacity.
 * Rows of a sequence's last block beyond its length may hold any finite value for prefill
 * (they are masked) and any bits at all for decode; a freshly allocated block should be
 * zero-filled.
 * The paged entry points take the same arguments as their contiguous counterparts with the
 * cache pointers, strides and capacity replaced by the descriptor. */
typedef struct mllm_paged_kv {
    void* k_pool;
    void* v_pool;
    int64_t block_stride;
    int64_t head_stride;
    int64_t row_stride;
    int32_t num_blocks;
    int32_t block_size;
    const int32_t* block_table;
    int64_t table_stride;
    int32_t max_blocks_per_seq;
} mllm_paged_kv;

MLLM_API int mllm_qkv_epilogue_paged_bf16(const void* q, int64_t q_sb, int64_t q_ss, int64_t q_sh,
                                          const void* k, int64_t k_sb, int64_t k_ss, int64_t k_sh,
                                          const void* v, int64_t v_sb, int64_t v_ss, int64_t v_sh,
                                          int batch, int seq_len, int num_heads, int num_kv_heads, int head_dim,
                                          const int64_t* positions, int64_t pos_sb, int64_t pos_ss,
                                          double rope_theta, const float* rope_cos, const float* rope_sin,
                                          int64_t rope_row_sb, int64_t rope_row_ss, const void* q_norm_weight,
                                          const void* k_norm_weight, double rms_norm_eps, void* q_out,
                                          const mllm_paged_kv* kv, const int32_t* cache_start,
                                          int64_t uniform_cache_start, mllm_stream_t stream);

MLLM_API int mllm_prefill_attention_paged_bf16(const void* q, const mllm_paged_kv* kv, int batch, int num_heads,
                                               int num_kv_heads, int head_dim, int q_len, int kv_len,
                                               float softmax_scale, void* out, mllm_stream_t stream);

MLLM_API int mllm_decode_attention_paged_bf16(const void* q, const mllm_paged_kv* kv, const int32_t* kv_lens,
                                              int batch, int num_heads, int num_kv_heads, int head_dim,
                                              int max_kv_len, float softmax_scale, void* out, void* workspace,
                                              size_t workspace_bytes, mllm_stream_t stream);

MLLM_API int mllm_decode_step_paged_bf16(const void* q, int64_t q_sb, int64_t q_sh, const void* k, int64_t k_sb,
                                         int64_t k_sh, const void* v, int64_t v_sb, int64_t v_sh,
                                         const int64_t* positions, int64_t pos_sb, double rope_theta,
                                         const float* rope_cos, const float* rope_sin, int64_t rope_row_sb,
                                         const void* q_norm_weight, const void* k_norm_weight, double rms_norm_eps,
                                         const mllm_paged_kv* kv, const int32_t* kv_lens, int batch,
                                         int num_heads, int num_kv_heads, int head_dim, int max_kv_len,
                                         float softmax_scale, void* out, void* workspace, size_t workspace_bytes,
                                         mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Packed sequences of different lengths (variable-length prefill).  Several prompts, or
 * prompt chunks, go through the epilogue and the attention in one launch each, instead of one
 * call per sequence: the runners' Forward takes one [B, S] batch, so the reference prefills
 * prompts of different lengths one Generate call at a time (QwenRunner.cpp:420-545).
 * Sequence b owns the packed token rows cu_seqlens[b] .. cu_seqlens[b+1]-1 (int32 device
 * [batch + 1], non-decreasing, cu_seqlens[0] = 0, cu_seqlens[batch] = total tokens); empty
 * sequences are allowed.  Cache sequence b of a contiguous cache, or block-table row b of a
 * paged one, receives sequence b's rows.
 *
 * Epilogue (mllm_qkv_epilogue_bf16 / _paged_bf16 for packed tokens):
 *   q/k/v: token t's head h at q + t*q_st + h*q_sh (likewise k, v); bf16, head_dim contiguous.
 *   positions: int64 device [total_tokens], each token's RoPE position (required).
 *   cache_start: int32 device [batch] (NULL: 0), the cache row of sequence b's first new token.
 *   q_out: bf16 [num_heads, total_tokens, head_dim] -- the layout the varlen prefill reads.
 *   A token outside the ranges cu_seqlens describes, or a row past the cache, records
 *   MLLM_ERR_DEVICE_LENGTH and its K/V row is not written.
 *
 * Attention (mllm_prefill_attention_bf16 / _paged_bf16 for packed sequences):
 *   q: bf16 [num_heads, total_q, head_dim] (the varlen epilogue's q_out).
 *   cu_q_lens: as cu_seqlens above, over total_q rows.
 *   kv_lens: int32 device [batch], the cache rows of sequence b after its new rows were
 *       appended (kv_lens[b] >= its q_len); query row s of sequence b sits at position
 *       kv_lens[b] - q_len + s and sees cache rows 0 .. that position.
 *   max_q_len: the longest sequence's q_len, or more (it sizes the grid; a longer one is an
 *       error).
 *   out: bf16 [total_q, num_heads * head_dim].
 *   Cache rows past kv_lens[b] that share a 128-row tile with the last visible row are read
 *   and masked: they must hold finite values (a freshly allocated cache or block should be
 *   zero-filled).  A sequence whose range, q_len or kv_len is inconsistent (or kv_len beyond
 *   cache_capacity, or beyond max_blocks_per_seq * block_size) records MLLM_ERR_DEVICE_LENGTH
 *   and its output rows are not written. */
MLLM_API int mllm_qkv_epilogue_varlen_bf16(const void* q, int64_t q_st, int64_t q_sh, const void* k, int64_t k_st,
                                           int64_t k_sh, const void* v, int64_t v_st, int64_t v_sh, int total_tokens,
                                           int num_heads, int num_kv_heads, int head_dim, const int64_t* positions,
                                           double rope_theta, const void* q_norm_weight, const void* k_norm_weight,
                                           double rms_norm_eps, void* q_out, void* k_cache, void* v_cache,
                                           int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                           int64_t cache_capacity, const int32_t* cu_seqlens, int batch,
                                           const int32_t* cache_start, mllm_stream_t stream);

MLLM_API int mllm_qkv_epilogue_varlen_paged_bf16(const void* q, int64_t q_st, int64_t q_sh, const void* k,
                                                 int64_t k_st, int64_t k_sh, const void* v, int64_t v_st,
                                                 int64_t v_sh, int total_tokens, int num_heads, int num_kv_heads,
                                                 int head_dim, const int64_t* positions, double rope_theta,
                                                 const void* q_norm_weight, const void* k_norm_weight,
                                                 double rms_norm_eps, void* q_out, const mllm_paged_kv* kv,
                                                 const int32_t* cu_seqlens, int batch, const int32_t* cache_start,
                                                 mllm_stream_t stream);

MLLM_API int mllm_prefill_attention_varlen_bf16(const void* q, const void* k_cache, const void* v_cache,
                                                int64_t cache_sb, int64_t cache_sh, int64_t cache_st,
                                                int64_t cache_capacity, const int32_t* cu_q_lens,
                                                const int32_t* kv_lens, int batch, int num_heads, int num_kv_heads,
                                                int head_dim, int total_q, int max_q_len, float softmax_scale,
                                                void* out, mllm_stream_t stream);

MLLM_API int mllm_prefill_attention_varlen_paged_bf16(const void* q, const mllm_paged_kv* kv,
                                                      const int32_t* cu_q_lens, const int32_t* kv_lens, int batch,
                                                      int num_heads, int num_kv_heads, int head_dim, int total_q,
                                                      int max_q_len, float softmax_scale, void* out,
                                                      mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Token sampling on the device.  Replaces src/core/runtime/Sampler.cpp:49-232
 * (Sampler::Sample) for `batch` logit rows at once, with no host round trip (the reference's
 * repetition penalty, Sampler.cpp:12-46, reads and writes one logit per previous token with a
 * device sync each).
 *   logits: bf16 (logits_bf16 != 0) or fp32, row b at logits + b*row_stride, `vocab` entries.
 *       The repetition penalty is applied IN PLACE, as the reference does to its argument: each
 *       occurrence of a token in the history divides a non-negative logit by the penalty or
 *       multiplies a negative one, the result rounded to the logits' dtype each time.
 *   prev_tokens / prev_counts: int64 / int32 device; row b's history is prev_counts[b] tokens at
 *       prev_tokens + b*prev_stride (both NULL: no history).  Out-of-range ids are ignored.
 *   temperature, top_k, top_p, use_greedy, repetition_penalty: as Sampler::Sample, with its
 *       argument errors (non-finite temperature; top_p outside (0, 1]; empty logits).  Greedy
 *       (use_greedy, or temperature <= 0) is the argmax, first index winning ties, NaN above
 *       every number.  Otherwise: softmax(logits / temperature) in fp32; top_k > 0 keeps the
 *       scores >= the top_k-th largest; top_p < 1 keeps the largest scores whose renormalised
 *       mass, summed from the top, stays <= top_p, always keeping the top one; one draw picks the
 *       token.  Ties at a top-k/top-p cut are all kept.
 *   seed, offset: the draw of row b is the first output of Philox-4x32-10 with key `seed` and
 *       counter (offset, b, 0); advance `offset` for every call.
 *   out_tokens: int64 device [batch].
 *   workspace: mllm_sample_workspace_size(batch, vocab) bytes when the penalty applies (> 1
 *       with a history); contents need not be initialised. */
MLLM_API size_t mllm_sample_workspace_size(int batch, int vocab);

MLLM_API int mllm_sample(void* logits, int logits_bf16, int64_t row_stride, int batch, int vocab,
                         const int64_t* prev_tokens, int64_t prev_stride, const int32_t* prev_counts,
                         float temperature, int top_k, float top_p, int use_greedy, float repetition_penalty,
                         uint64_t seed, uint64_t offset, int64_t* out_tokens, void* workspace,
                         size_t workspace_bytes, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Projections for decode-sized token counts.  Replaces Linear::Forward (Linear.h:33-68,
 * F::linear(x, w) = x w^T in bf16) for the attention step's q/k/v projections
 * (TransformerBlock.h:82-96, Attention.h:52-54: three calls become one launch) and o_proj
 * (Attention.h:322-325) when tokens <= 256.
 *   x: bf16 [tokens, in_features], row stride x_stride (elements, multiple of 8; 16-byte aligned);
 *       in_features a multiple of 64
 *   weights[i]: bf16 [out_features[i], in_features], row stride weight_strides[i] (multiple of
 *       8; 16-byte aligned); 1 <= num_weights <= 4; out_features[i] a multiple of 128
 *   out: bf16 [tokens, out_stride], 16-byte aligned, out_stride a multiple of 8; weight i's
 *       rows land in columns [c_i, c_i + out_features[i]), c_i = out_features[0..i) summed
 *   workspace: mllm_linear_workspace_size(...) bytes (0 when no split is needed), 256-byte
 *       aligned.  Its first 4096 bytes are tile counters, which must be zero before the first
 *       use and which every call leaves at zero, so one workspace serves any number of calls of
 *       any shapes in one stream (not concurrent calls); the rest needs no initialisation
 * fp32 accumulation on the tensor cores, one rounding to bf16 per output.  The k range of a
 * 128-row tile may be split over up to 8 CTAs whose fp32 partials are added in split order,
 * so results are deterministic.  0 <= tokens <= 256.
 * The launch may start while the previous kernel in the stream is finishing (programmatic
 * dependent launch) and streams its first weight tiles before it waits for that kernel: the
 * weights must not be written by the kernel launched just before this call in the same stream
 * (x may be).  The same holds for mllm_linear_fp8_bf16. */
MLLM_API size_t mllm_linear_workspace_size(int tokens, int num_weights, const int64_t* out_features,
                                           int64_t in_features);

MLLM_API int mllm_linear_bf16(const void* x, int64_t x_stride, int tokens, int64_t in_features, int num_weights,
                              const void* const* weights, const int64_t* weight_strides,
                              const int64_t* out_features, void* out, int64_t out_stride, void* workspace,
                              size_t workspace_bytes, mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * FP8 projections.  Replaces, for a weight stored as e4m3 with one fp32 scale per 128 x 128
 * block (`weight_scale_inv`, the FP8 checkpoint layout QwenRunner loads, QwenRunner.cpp:148-283),
 * the reference's dequantize-then-multiply: DequantizeFP8 (QwenRunner.cpp:103-122,
 * bf16(fp8 * bf16(scale)), run on every layer of every step) followed by Linear::Forward
 * (Linear.h:33-68).  The fp8 bytes are streamed from HBM (half the bf16 weight) and dequantized
 * on chip with exactly that rounding; the tensor cores then multiply the same bf16
 * operand (fp32 accumulation, one rounding per output, split-k partials added in a fixed order).
 *   x: bf16 [tokens, in_features], row stride x_stride (multiple of 8, 16-byte aligned)
 *   weight: e4m3 [out_features, in_features], row stride weight_stride bytes (multiple of 16,
 *       16-byte aligned); in_features and out_features multiples of 128
 *   weight_scale_inv: fp32 [out_features/128, >= in_features/128], row stride scale_stride
 *   out: bf16 [tokens, out_stride], 16-byte aligned, out_stride a multiple of 8
 *   workspace: mllm_linear_fp8_workspace_size(...) bytes (0 when no split is needed), 256-byte
 *       aligned, with the same counter convention as mllm_linear_bf16's workspace (one workspace
 *       may serve both)
 * 0 <= tokens <= 128 (decode-sized batches; larger batches dequantize and call a GEMM). */
MLLM_API size_t mllm_linear_fp8_workspace_size(int tokens, int64_t out_features, int64_t in_features);
MLLM_API int mllm_linear_fp8_bf16(const void* x, int64_t x_stride, int tokens, int64_t in_features,
                                  const void* weight, int64_t weight_stride, int64_t out_features,
                                  const float* weight_scale_inv, int64_t scale_stride, void* out,
                                  int64_t out_stride, void* workspace, size_t workspace_bytes,
                                  mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Peer-memory plumbing for the tensor-parallel o_proj exchange (no reference counterpart: the
 * reference runs on one device, QwenRunner.cpp:236,328).  mllm_b200/tp.py's PeerExchange
 * sums the ranks' o_proj partials with these: flags raised in a peer's memory, a bounded
 * wait, and a sum kernel that reads every rank's partial rows over NVLink and stores the sum
 * into every rank's output rows.
 *   mllm_ipc_alloc/free: cudaMalloc'd, zero-filled device memory to share (setup, not per call)
 *   mllm_ipc_get_handle / open_handle / close_handle: CUDA IPC of such an allocation's base;
 *       the handle is MLLM_IPC_HANDLE_BYTES bytes
 *   mllm_copy_async: device-to-device copy (either side may be a peer's opened allocation)
 *   mllm_signal_u32: after the stream's earlier work, store `value` to *flag with system-scope
 *       release (flag may be a peer's memory)
 *   mllm_wait_u32: the stream's later work waits until (int32)(*flag - value) >= 0; gives up
 *       after about four seconds and records MLLM_ERR_DEVICE_TIMEOUT (mllm_attn_device_status)
 *   mllm_wait_u32_timeout: the same wait, giving up after timeout_us microseconds of device
 *       time (1 us .. 60 s), for callers that want a short deadline
 *   mllm_sum_bf16: dsts[d][i] = sum over s of srcs[s][i] for every d < n_dst, fp32 in the order
 *       s = 0, 1, ..., one rounding to bf16; 1..8 sources and destinations (either may be a
 *       peer's opened allocation), 16-byte aligned, count a multiple of 8 */
#define MLLM_IPC_HANDLE_BYTES 64
MLLM_API int mllm_ipc_alloc(size_t bytes, void** ptr);
MLLM_API int mllm_ipc_free(void* ptr);
MLLM_API int mllm_ipc_get_handle(const void* ptr, void* handle);
MLLM_API int mllm_ipc_open_handle(const void* handle, void** ptr);
MLLM_API int mllm_ipc_close_handle(void* ptr);
MLLM_API int mllm_copy_async(void* dst, const void* src, size_t bytes, mllm_stream_t stream);
MLLM_API int mllm_signal_u32(uint32_t* flag, uint32_t value, mllm_stream_t stream);
MLLM_API int mllm_wait_u32(const uint32_t* flag, uint32_t value, mllm_stream_t stream);
MLLM_API int mllm_wait_u32_timeout(const uint32_t* flag, uint32_t value, uint32_t timeout_us, mllm_stream_t stream);
MLLM_API int mllm_sum_bf16(void* const* dsts, int n_dst, const void* const* srcs, int n_src, int64_t count,
                           mllm_stream_t stream);

/* ----------------------------------------------------------------------------------------
 * Communicators for the tensor-parallel exchange.  No counterpart in the reference, which runs
 * every layer on one device (QwenRunner.cpp:236,328): sharding attention by KV-head group makes
 * o_proj (Attention.h:322-325) a sum of per-rank partials, and these carry that sum over NVLink
 * with NCCL, one process per GPU.  The C++ drop-in's tensor-parallel mode
 * (b200::TensorParallel) and mllm_b200/tp.py call them.
 *   mllm_comm_unique_id: fills MLLM_COMM_ID_BYTES bytes on one rank; the caller hands them to
 *       every rank (its own side channel: a store, a file, MPI)
 *   mllm_comm_init: every rank, on its own current device: a NON-BLOCKING NCCL communicator
 *       (ncclConfig_t.blocking = 0) plus a watchdog thread.  Set-up, tear-down and every
 *       collective are bounded by timeout_s seconds.
 *   mllm_comm_all_reduce_bf16: recv[i] = sum over ranks of send[i] (bf16, in place allowed),
 *       enqueued on `stream` after its earlier work; the o_proj exchange
 *   mllm_comm_all_gather_bf16: recv = the ranks' send buffers (send_count elements each)
 *       concatenated in rank order
 *   Failure detection: the watchdog tracks each collective by an event recorded behind it and
 *   polls every 5 ms.  An asynchronous NCCL error (a peer failed or left) or a collective still
 *   running timeout_s after it was enqueued aborts the communicator (ncclCommAbort ends its
 *   kernels); from then on every call returns MLLM_ERR_COMM or MLLM_ERR_COMM_TIMEOUT and the
 *   caller builds a new communicator.  mllm_comm_status polls once and reports that state;
 *   mllm_comm_abort aborts on request (the host learned by itself that a peer is gone);
 *   mllm_comm_in_flight counts the tracked collectives not yet complete.  Collectives enqueued
 *   while `stream` is captured into a CUDA graph are not tracked.
 *   mllm_comm_destroy: finalises (bounded) and frees a healthy communicator; frees an aborted
 *   one.  Stops the watchdog.  Must not race with other calls on the communicator. */
#define MLLM_COMM_ID_BYTES 128
typedef struct mllm_comm* mllm_comm_t;
MLLM_API int mllm_comm_unique_id(void* id);
MLLM_API int mllm_comm_init(const void* id, int nranks, int rank, double timeout_s, mllm_comm_t* comm);
MLLM_API int mllm_comm_all_reduce_bf16(mllm_comm_t comm, const void* send, void* recv, size_t count,
                                       mllm_stream_t stream);
MLLM_API int mllm_comm_all_gather_bf16(mllm_comm_t comm, const void* send, void* recv, size_t send_count,
                                       mllm_stream_t stream);
MLLM_API int mllm_comm_status(mllm_comm_t comm);
MLLM_API int mllm_comm_in_flight(mllm_comm_t comm);
MLLM_API int mllm_comm_abort(mllm_comm_t comm);
MLLM_API int mllm_comm_destroy(mllm_comm_t comm);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* MLLM_ATTN_H_ */
