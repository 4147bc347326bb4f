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
  int splits;                  // KV splits: 1 to 8 in one cluster, or 16 in two clusters with part/arrive set
  // non-null: keys at logical indices >= offset (the forward's own rows) are read from these [rows][kv_heads]
  // [head_dim] planes (the round scratch) instead of the paged cache
  const void* scratch_k;
  const void* scratch_v;
  // non-null (with splits = 16): two clusters of 8 splits per (head, query tile). When the keys give all 16 splits four
  // tiles each, every split stores its partial to `part` and waits (bounded) for the others, so every cluster of the
  // launch must be resident at once (attention_two_clusters_fit); otherwise the second cluster leaves at once and the
  // first combines through distributed shared memory. part holds [num_heads][q_tiles][16] x 64 rows x
  // (head_dim + 2) floats, arrive [num_heads][q_tiles][2] counters that are zero between launches.
  float* part;
  int* arrive;
  int* err;
};

// Split count that fills about two CTAs per SM for `max_keys` keys: at most 8 (one cluster), or with
// `global_combine` 16 (two clusters) when the keys can give every split four tiles.
int attention_splits(int num_heads, int q_tiles, int num_sms, int64_t max_keys, bool global_combine = false);
// Whether every cluster of a two-cluster launch (heads x q_tiles x 2 clusters of 8) is resident at once.
bool attention_two_clusters_fit(int num_heads, int q_tiles, int head_dim, int dtype);
// Sizes of the merge buffers of a two-cluster launch.
size_t attention_part_floats(int num_heads, int q_tiles, int head_dim);
size_t attention_arrive_ints(int num_heads, int q_tiles);
int attention_launch(plm_ctx* ctx, AttnArgs a, cudaStream_t stream, bool pdl);

}  // namespace plm
