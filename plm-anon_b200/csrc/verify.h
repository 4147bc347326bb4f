// Kernel-side argument blocks of the verify decode / acceptance / bookkeeping kernel (voronoi.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace plm {

enum AcceptRule : int { kRuleNucleus = 0, kRuleFloor = 1 };

// Each verify row is decoded by a cluster of kVerifyCluster CTAs of kVerifyThreads threads (the oracle mirrors the
// partition: oracle/voronoi.py CLUSTER and THREADS).
constexpr int kVerifyCluster = 8;
constexpr int kVerifyThreads = 256;
// Diagnostic phase record per verify row: statistics, rule, slice select, merge copy, merge sort, table staging,
// quota/spread/prior, condense and fit of rounds 0 and 1, final cluster barrier, argmin (slots 13..15 unused).
constexpr int kPhaseSlots = 16;
enum BookMode : int { kBookNone = 0, kBookSteady = 1, kBookRound0 = 2, kBookFirstToken = 3 };
// Words of the request stop block (plm_bookkeeping.stop).
enum StopWord : int { kStopBudget = 0, kStopEos = 1, kStopWindow = 2, kStopDone = 3, kStopWords = 4 };

struct Bookkeeping {
  int mode;
  int k;                     // verify rows of a steady round
  const float* best_val;     // [n_tiles][rows] lm_head per-tile maxima of every row
  const int32_t* best_idx;   // [n_tiles][rows] their first indices
  int n_tiles;
  int rows;                  // rows of the forward (W)
  int64_t* out;              // [out_cap] output tokens
  int64_t out_cap;
  int64_t* base;             // next output position
  int64_t* offset;           // KV length committed
  int64_t* anchor;           // last confirmed token
  int64_t* pending;          // [k - 1] proposals to verify next round
  int64_t* round_sequence;   // [seq_cap] accepted count per steady round
  int64_t seq_cap;
  int64_t* sequence_step;
  int64_t prompt_len;        // first-token mode: the offset round 0 starts at
  int64_t* stop;             // nullable [kStopWords]: budget, end-of-text id, end-of-text window, done flag
  int64_t* commit;           // nullable [2]: first logical KV index and count of the round rows to commit
};

struct VerifyArgs {
  const float* logits;       // [n_rows][logits_stride] fp32 (model-dtype values)
  int vocab;
  int64_t logits_stride;
  const void* table;         // [vocab][aux] Voronoi cost table, model dtype
  int aux;
  const int64_t* aux_buf;    // auxiliary cell stream
  int64_t aux_len;
  const int64_t* aux_base;   // device scalar added to every row's stream index (nullable: 0)
  int aux_row_offset;
  const int64_t* pending;    // [n_accept] proposals tested by the relaxed rule
  int n_accept;
  int rule;                  // AcceptRule
  float threshold;           // nucleus mass (<= 0: exact match) or floor probability
  int top_m, shortlist, rounds, sweeps;
  float eps[4];              // fp32 epsilon of each fit round
  float anneal[4];           // fp32 per-sweep temperature factor of each round
  int64_t* verify;           // [n_rows] decoded tokens
  int32_t* flags;            // [n_rows] relaxed-rule verdicts (nullable)
  int32_t* dbg_tokens;       // [n_rows][top_m] (nullable)
  int32_t* dbg_counts;       // [n_rows][top_m]
  float* dbg_bias;           // [n_rows][top_m]
  float* dbg_stats;          // [n_rows][4] max, sum of exp, normaliser, unit
  int32_t* dbg_sigma;        // [n_rows] shortlist index of the decoded token
  int64_t* dbg_phase_ns;     // [n_rows][kPhaseSlots] ns from kernel start to the end of each phase (nullable)
  int tokens_given;          // nonzero: verify[] already holds the rows' tokens (inverse-CDF decode); only the
                             // relaxed rule's verdicts and the bookkeeping run
  Bookkeeping book;
  int* counter;              // arrival counter (zero between launches)
  int* err;
};

int verify_validate(const VerifyArgs& a, int n_rows);
int verify_launch(const VerifyArgs& a, int dtype, int n_rows, cudaStream_t stream, bool pdl);

}  // namespace plm
