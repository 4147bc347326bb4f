// The Llama MLP block of the round as one persistent launch (mlp.cu): gate_up with SiLU(gate) * up, then down
// written as fp32 k-split partials, which the residual-add RMSNorm after it sums in split order.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <vector>

namespace plm {

constexpr int kMlpMaxRows = 128;        // widest row tile of the block kernel; wider forwards use two launches
constexpr int kMlpMaxDownSplits = 16;   // k-splits of down (partials summed by the norm that follows)

// Work assignment of one block launch: every CTA of the grid runs a list of units, its gate_up tiles first, then
// (down tile, k-split) units. Host-built once per model shape; `sched` and `sched_off` are device arrays.
struct MlpSchedule {
  int grid = 0;            // CTAs (one per SM)
  int gate_tiles = 0;      // intermediate / 64
  int down_tiles = 0;      // ceil(hidden / 128)
  int down_splits = 0;     // k-splits of down
  int* sched = nullptr;    // unit codes, CTA after CTA
  int* sched_off = nullptr;  // [grid + 1] offsets into sched
};

struct MlpBlockArgs {
  int dtype;
  const void* gate_up_tiles;  // the gate_up weight packed by pack_weight_tiles with gate_offset = intermediate
  const void* down_tiles;     // the down weight packed by pack_weight_tiles (128-row tiles)
  const void* x_tiles;        // the normed input as row tiles (common.cuh) of gemm_token_tile(rows) rows, k = hidden
  void* act_tiles;            // SiLU(gate) * up written as row tiles of the same height, k = intermediate
  float* partials;            // [down_splits][rows][hidden]
  int rows, hidden, intermediate;
  int* gate_done;          // this layer's counter: +1 per gate_up tile stored, so epoch * (intermediate / 64)
                           // once a forward's act is complete
  const int* epoch;        // MLP block forwards run so far, this one included
  int* err;
};

// Balanced assignment of units to `grid` CTAs by k-block count (deterministic); see mlp.cu.
std::vector<int> mlp_schedule_units(int grid, int gate_tiles, int gate_kb, int down_tiles, int down_splits,
                                    int down_kb, std::vector<int>* offsets);
int mlp_schedule_create(int num_sms, int hidden, int intermediate, MlpSchedule* out);
void mlp_schedule_destroy(MlpSchedule* s);
// One launch of the block for `rows` (1..kMlpMaxRows) rows.
int mlp_block_launch(const MlpSchedule& s, const MlpBlockArgs& a, cudaStream_t stream, bool pdl);

}  // namespace plm
