// Argument block of the paged round attention kernel (attention.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "runtime.h"

namespace plm {

struct AttnArgs {
  int dtype;                   // PLM_BF16 or PLM_F16: q, the caches and the output
  const void* q;               // [rows][num_heads][head_dim] (after RoPE)
  const void* k_cache;         // [num_pages][num_kv_heads][page_size][head_dim]
  const void* v_cache;
  const int32_t* block_table;  // [max_pages] logical page -> physical page
  int max_pages;
  int num_pages;
  int page_size;
  int page_shift;              // log2(page_size): page sizes are powers of two
  const int64_t* offset;       // device scalar: logical KV index of query row 0
  int rows;
  const int32_t* depth;        // [rows] relative to offset
  const int32_t* own_start;    // [rows]
  int num_heads, num_kv_heads, head_dim;
  float scale_log2;            // head_dim^-1/2 * log2(e)
  void* out;                   // [rows][num_heads * head_dim]; may be null when row_tiles is set
  void* row_tiles;             // non-null: the output written as row tiles of tile_rows rows instead (common.cuh)
  int tile_rows;
  int splits;                  // KV splits = cluster size, a power of two <= 8
  // non-null: keys at logical indices >= offset (the forward's own rows) are read from these [rows][kv_heads]
  // [head_dim] planes (the round scratch) instead of the paged cache
  const void* scratch_k;
  const void* scratch_v;
  int* err;
};

// Split count that fills about two CTAs per SM for `max_keys` keys.
int attention_splits(int num_heads, int q_tiles, int num_sms, int64_t max_keys);
int attention_launch(plm_ctx* ctx, AttnArgs a, cudaStream_t stream, bool pdl);

}  // namespace plm
