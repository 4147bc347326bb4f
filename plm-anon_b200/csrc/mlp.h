// One persistent launch per layer for everything between attention and the next layer's input norm (mlp.cu): the
// o projection, the residual-add RMSNorm after it, gate_up with SiLU(gate) * up, and down written as fp32 k-split
// partials, which the residual-add RMSNorm after the block sums in split order.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace plm {

constexpr int kMlpMaxRows = 128;        // widest row tile of the block kernel; wider forwards use separate launches
constexpr int kMlpMaxDownSplits = 16;   // k-splits of down (partials summed by the norm that follows)
constexpr int kMlpMaxOSplits = 16;      // k-splits of o (partials summed by the block's own norm rows)

// Work assignment of one block launch: every CTA of the grid runs a list of units: its o (tile, k-split) units,
// its norm rows, its gate_up tiles, then its down (tile, k-split) units. Host-built once per model shape; `sched`
// and `sched_off` are device arrays.
struct MlpSchedule {
  int grid = 0;              // CTAs (one per SM)
  int gate_tiles = 0;        // intermediate / 64
  int down_tiles = 0;        // ceil(hidden / 128)
  int down_splits = 0;       // k-splits of down
  int o_tiles = 0;           // ceil(hidden / 128)
  int o_splits = 0;          // k-splits of o
  int* sched = nullptr;      // unit codes, CTA after CTA
  int* sched_off = nullptr;  // [grid + 1] offsets into sched
};

// Kernel parameters of one launch (pointers are device addresses).
struct BlockParams {
  const uint8_t* wo_tiles;    // o weight packed by pack_weight_tiles (128-row tiles), k = q_size
  const uint8_t* wg_tiles;    // gate_up weight packed with gate_offset = intermediate
  const uint8_t* wd_tiles;    // down weight packed (128-row tiles), k = intermediate
  const uint8_t* attn_tiles;  // attention output as row tiles (common.cuh) of gemm_token_tile(rows) rows
  uint8_t* x_tiles;           // the normed rows, written by the block's norm rows, read by gate_up
  uint8_t* act_tiles;         // SiLU(gate) * up, written by gate_up, read by down
  const int* sched;
  const int* sched_off;
  float* partials;            // [splits][rows][hidden]: o partials, then (after the norm) down partials
  void* residual;             // [>= rows][hidden] model dtype, updated by the norm rows
  const void* norm_weight;    // post-attention RMSNorm weight [hidden]
  float eps;
  int* ctr;                   // this layer's counters, zero at the start of the forward: [0] o units stored,
                              // [1] rows normed, [2] gate_up tiles stored
  int rows, hidden, intermediate, q_size;
  int o_splits, down_splits, o_units;
  // Weights the kernel after this block reads first (the next layer's qkv, or the head of lm_head): each CTA
  // prefetches its slice into L2 once its own weight copies are issued, while the down phase and the norm after it
  // leave HBM idle. May be null.
  const uint8_t* next_weights;
  long long next_bytes;
  int* err;
};

// Assignment of units to `grid` CTAs (deterministic); see mlp.cu.
std::vector<int> mlp_schedule_units(const MlpSchedule& s, int hidden, int intermediate, int q_size,
                                    std::vector<int>* offsets);
// The schedule's sizes for a shape (host only, nothing allocated); PLM_ERR_UNSUPPORTED for shapes the block
// does not take.
int mlp_schedule_plan(int num_sms, int hidden, int intermediate, int q_size, MlpSchedule* out);
int mlp_schedule_create(int num_sms, int hidden, int intermediate, int q_size, MlpSchedule* out);
void mlp_schedule_destroy(MlpSchedule* s);
// One launch of the block for `p.rows` (1..kMlpMaxRows) rows; fills the schedule fields of `p`.
int mlp_block_launch(const MlpSchedule& s, BlockParams p, int dtype, cudaStream_t stream, bool pdl);

}  // namespace plm
