// Where cache row t of sequence b lives.  A contiguous cache ([B, Hkv, capacity, D] with the
// caller's strides) indexes (b, t) directly; a paged cache (mllm_paged_kv) looks the block up in
// the sequence's block table: row t % block_size of block table[b][t / block_size].  The TMA
// tensor maps of both have the same four dimensions {D, rows, kv heads, sequence or block}, so
// every kernel addresses a tile as (column, row, kv head, blk) with (blk, row) from kv_locate.
#pragma once

#include <string>

#include "common.cuh"
#include "host_util.h"

namespace mllm_b200 {

struct KvLayout {
    const int32_t* table = nullptr;   // null: contiguous cache
    int64_t table_stride = 0;
    int block_size = 0;
    int num_blocks = 0;
    int max_blocks = 0;
};

// Fills (blk, row) for cache row t of sequence b.  A block-table entry outside [0, num_blocks)
// (or a row past the table) records kErrBadLength and yields block 0 with `false`, so a load can
// still be issued (reading finite garbage instead of faulting) while a write is skipped.
__device__ __forceinline__ bool kv_locate(const KvLayout& lay, int b, int64_t t, int& blk, int& row) {
    if (lay.table == nullptr) {
        blk = b;
        row = (int)t;
        return true;
    }
    const int64_t i = t / lay.block_size;
    row = (int)(t - i * lay.block_size);
    const int e = (i < lay.max_blocks) ? lay.table[(int64_t)b * lay.table_stride + i] : -1;
    if (e < 0 || e >= lay.num_blocks) {
        record_error(kErrBadLength);
        blk = 0;
        return false;
    }
    blk = e;
    return true;
}

// Host side: checks a paged-cache descriptor for a call that addresses `rows` rows per sequence
// of `head_dim` columns (the pool strides' 16-byte rule is checked by the tensor-map encoder),
// and fills the device layout.
inline int paged_layout(const mllm_paged_kv* kv, int64_t rows, int head_dim, const char* who, KvLayout* out) {
    const std::string w(who);
    if (kv == nullptr) return fail(MLLM_ERR_INVALID_ARGUMENT, w + ": paged cache descriptor is NULL");
    if (!kv->k_pool || !kv->v_pool || !kv->block_table)
        return fail(MLLM_ERR_INVALID_ARGUMENT, w + ": paged cache pools and block table must be given");
    if (kv->block_size <= 0 || kv->block_size % 128 != 0)
        return fail(MLLM_ERR_INVALID_ARGUMENT, w + ": block_size must be a positive multiple of 128");
    if (kv->num_blocks <= 0 || kv->max_blocks_per_seq <= 0 || kv->table_stride < kv->max_blocks_per_seq)
        return fail(MLLM_ERR_INVALID_ARGUMENT, w + ": bad num_blocks, max_blocks_per_seq or table_stride");
    if (kv->row_stride < head_dim || kv->head_stride < head_dim || kv->block_stride < head_dim)
        return fail(MLLM_ERR_INVALID_ARGUMENT, w + ": bad pool strides");
    if (rows > (int64_t)kv->max_blocks_per_seq * kv->block_size)
        return fail(MLLM_ERR_INVALID_ARGUMENT, w + ": rows exceed max_blocks_per_seq * block_size");
    out->table = kv->block_table;
    out->table_stride = kv->table_stride;
    out->block_size = kv->block_size;
    out->num_blocks = kv->num_blocks;
    out->max_blocks = kv->max_blocks_per_seq;
    return MLLM_OK;
}

}  // namespace mllm_b200
