// Argument block of the KV commit kernel (commit.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace plm {

struct CommitArgs {
  const void* scratch;         // [layers][2][scratch_rows][num_kv_heads][head_dim]: the round's K and V rows
  int scratch_rows;
  void* kv_cache;              // [layers][2][num_pages][num_kv_heads][page_size][head_dim]
  int64_t plane_elems;         // elements of one (layer, K|V) plane of the cache
  int layers, num_kv_heads, head_dim, page_size, num_pages, max_pages;
  const int32_t* block_table;  // [max_pages] logical page -> physical page
  const int64_t* commit;       // device [2]: first logical index, rows to commit
  int* err;
};

int commit_validate(const CommitArgs& a);
int commit_launch(const CommitArgs& a, cudaStream_t stream, bool pdl);

}  // namespace plm
