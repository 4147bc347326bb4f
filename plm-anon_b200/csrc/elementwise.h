// Argument blocks of the row-wise kernels (elementwise.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace plm {

enum PrologueMode : int { kPrologueSteady = 0, kPrologueRound0 = 1, kProloguePrefill = 2 };

struct PrologueArgs {
  int dtype;                   // PLM_BF16 or PLM_F16: the model's storage dtype
  int mode;
  int k;
  int vocab, aux, num_aux_tokens, hidden;
  float eps;
  const int64_t* offset;       // device scalar: logical KV index of row 0
  const int64_t* base;         // device scalar: output position of verify row 0
  const int64_t* anchor;
  const int64_t* pending;      // [k - 1]
  const int64_t* rel_positions;  // [rows] (nullable: r)
  const int64_t* rel_aux;      // [rows] (-1: no auxiliary cell)
  const int64_t* aux_buf;
  int64_t aux_len;
  const int64_t* prompt;       // prefill: prompt token ids
  int64_t prompt_cap;
  const void* embed;
  const void* aux_vocab;
  const void* mask_aux;
  const void* norm_weight;     // layer 0 input_layernorm
  const int32_t* block_table;
  int max_pages, num_pages, page_size, max_pos;
  void* residual;              // [rows][hidden]
  void* normed;                // [rows][hidden]
  int32_t* positions;          // [rows]
  int64_t* slots;              // [rows]
  int round_scratch;           // nonzero: row r's K/V go to row r of the round scratch (slots[r] = r), not to a page
  // The PTP scheme (nullable): auxiliary rows blend rows of this float32 table [ptp_rows][hidden] at the request's
  // uniform aux_u[base + rel_aux] instead of taking an auxiliary-vocabulary row
  const float* ptp_embedding;
  int ptp_rows;
  const float* aux_u;
  int* counters;               // zeroed at the start of the forward (the layer blocks' phase counters; may be null)
  int n_counters;
  int* err;
};

struct AddNormArgs {
  const void* x;
  void* residual;
  void* normed;
  const void* weight;
  int hidden;
  float eps;
  int gather_row;  // -1: none
  void* gathered;
  const float* partials = nullptr;  // non-null: x = bf16(sum of n_partials fp32 slices, split order)
  int n_partials = 0;
  int64_t partial_stride = 0;       // floats between slices
  void* row_tiles = nullptr;        // non-null: the normed rows also as row tiles of `tile_rows` rows (common.cuh)
  int tile_rows = 0;
  const float* corr = nullptr;      // non-null: x[r] = round(x[r] + corr[r - corr_from]) for rows r >= corr_from
  int corr_from = 0;
  int corr_ld = 0;
  int dtype = 0;                    // PLM_BF16 or PLM_F16
};

struct KvAppendArgs {
  int dtype;      // PLM_BF16 or PLM_F16
  const void* k;  // [rows][num_kv_heads][head_dim]
  const void* v;
  void* k_cache;  // [num_pages][num_kv_heads][page_size][head_dim]
  void* v_cache;
  const int32_t* block_table;
  int max_pages, num_pages, page_size;
  const int64_t* offset;
  int rows, num_kv_heads, head_dim;
  int* err;
};

int prologue_launch(const PrologueArgs& a, int rows, cudaStream_t stream, bool pdl);
int add_norm_launch(const AddNormArgs& a, int rows, cudaStream_t stream, bool pdl);
int kv_append_launch(const KvAppendArgs& a, cudaStream_t stream, bool pdl);

}  // namespace plm
