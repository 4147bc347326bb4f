// Verify decode, acceptance and round bookkeeping (compiled with -fmad=false: bit-exact with the CPU oracle).
//
// One CTA of 1024 threads per verify row. For its row of fp32 logits the CTA computes
//   1. the softmax statistics (maximum, sum of exp, normaliser = max + log sum) and, when the round uses a relaxed
//      rule, the rule's verdict for the row's pending proposal (plm/decoder.py:71-82);
//   2. the exact top-m shortlist by a 4-pass radix select on order-preserving keys (ties: lower index first), its
//      largest-remainder quota (plm/iterate.py:248-273, 214-223), the cost spread and the prior (275-290);
//   3. `rounds` x (condense each auxiliary item to its `shortlist` cheapest targets, then an annealed Sinkhorn fit of
//      `sweeps` sweeps) (83-159, 292-312), with the per-target load accumulated in a fixed order (per-warp bins
//      filled by lane groups in ascending lane order, then summed over warps) instead of float atomics;
//   4. sigma(cell) = argmin_m C[m, cell] + b[m] for the single auxiliary cell the row reads, and the token
//      tokens[sigma] (auxiliary.py:67-75, iterate.py:345-346).
// The last CTA to finish (arrival counter) then runs the round's bookkeeping (plm/decoder.py:351-365 for a steady
// round, 275-310 for round 0, and the first token after the prefill, 384): accepted count, output tokens, the
// per-round accepted-count record, the next pending proposals from the lm_head's per-tile argmax partials, anchor,
// base and offset (the implicit KV commit).
//
// Every floating-point step is a separate IEEE operation in a fixed order and exp/log come from plm_math.h; the
// numpy oracle (oracle/voronoi.py) performs the same operations.
#include <climits>

#include "common.cuh"
#include "plm_math.h"
#include "runtime.h"
#include "verify.h"

namespace plm {
using namespace plm_math;

namespace {

constexpr int kVThreads = 1024;
constexpr int kMaxTopM = 128;
constexpr int kTieBuffer = 1024;
constexpr int kMaxItemsPerThread = 4;  // aux vocabulary up to 4096
constexpr size_t kRowSmemLimit = 210 * 1024;

struct VerifySmem {
  uint32_t hist[256];
  int ties[kTieBuffer];
  int sel_idx[kMaxTopM];
  int tok[kMaxTopM];
  float val[kMaxTopM];
  float prob[kMaxTopM];
  int cnt[kMaxTopM];
  float frac[kMaxTopM];
  int counts[kMaxTopM];
  float bias[kMaxTopM];
  float offset[kMaxTopM];
  float corr[kMaxTopM];
  float share[kMaxTopM];
  float diff[64];
  float red_f[32];
  int red_i[32];
  int64_t new_pending[32];
  int need, tie_total, cnt_gt, cnt_tie, remaining, last, nc;
  uint32_t prefix;
  float psum, unit;
  int64_t picked;
};

constexpr size_t kFitScratchBytes = (32 * 128 + 32 * 32) * sizeof(float);

__device__ __forceinline__ float block_sum_f(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < int(blockDim.x >> 5) ? red[lane] : 0.0f;
    w = warp_sum(w);
    if (lane == 0) red[0] = w;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_max_f(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < int(blockDim.x >> 5) ? red[lane] : -INFINITY;
    w = warp_max(w);
    if (lane == 0) red[0] = w;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

template <typename T>
__device__ __forceinline__ float table_at(const T* table, int tok, int aux, int item) {
  return to_f32<T>(table[size_t(tok) * aux + item]);
}

// Canonical shortlist order: larger key first, then lower index.
__device__ __forceinline__ bool before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

template <typename T, int SL>
__global__ void __launch_bounds__(kVThreads, 1) verify_decode_kernel(const VerifyArgs a) {
  extern __shared__ __align__(16) uint8_t vsmem[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int r = blockIdx.x;
  const int V = a.vocab, A = a.aux, M = a.top_m;
  const bool row_in_smem = size_t(V) * 4 <= kRowSmemLimit;
  const size_t union_bytes = ((row_in_smem ? size_t(V) * 4 : 0) > kFitScratchBytes ? size_t(V) * 4 : kFitScratchBytes);
  float* row_buf = reinterpret_cast<float*>(vsmem);
  float* bins = reinterpret_cast<float*>(vsmem);      // fit phase (row no longer needed)
  float* wsh = bins + 32 * 128;
  VerifySmem* s = reinterpret_cast<VerifySmem*>(vsmem + ((union_bytes + 15) & ~size_t(15)));
  const T* table = reinterpret_cast<const T*>(a.table);

  grid_dependency_wait();
  allow_dependents();
  const uint64_t t_start = global_timer_ns();
  auto phase = [&](int k) {
    if (a.dbg_phase_ns != nullptr && tid == 0) a.dbg_phase_ns[r * 8 + k] = int64_t(global_timer_ns() - t_start);
  };

  // ---------------- 1. softmax statistics and the acceptance rule ----------------
  const float* grow = a.logits + size_t(r) * a.logits_stride;
  const float* row = grow;
  if (row_in_smem) {
    for (int i = tid; i < V; i += kVThreads) row_buf[i] = grow[i];
    __syncthreads();
    row = row_buf;
  }
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kVThreads) mx = fmaxf(mx, row[i]);
  mx = block_max_f(mx, s->red_f);
  float acc = 0.0f;
  for (int i = tid; i < V; i += kVThreads) acc = acc + plm_expf(row[i] - mx);
  const float total = block_sum_f(acc, s->red_f);
  const float normaliser = mx + plm_logf(total);
  phase(0);

  int flag = 0;
  if (r < a.n_accept && (a.rule == kRuleFloor || a.threshold > 0.0f)) {
    int64_t pt = a.pending[r];
    const bool ok = pt >= 0 && pt < V;
    if (!ok) {
      if (tid == 0) record_error(a.err, kErrBadIndex);
      pt = 0;
    }
    if (a.rule == kRuleFloor) {
      flag = ok && ((row[pt] - normaliser) > plm_logf(a.threshold));
    } else {
      const float own = plm_expf(row[pt] - mx) / total;
      float mass = 0.0f, pmax = -INFINITY;
      for (int i = tid; i < V; i += kVThreads) {
        const float pi = plm_expf(row[i] - mx) / total;
        pmax = fmaxf(pmax, pi);
        if (pi > own) mass = mass + pi;
      }
      mass = block_sum_f(mass, s->red_f);
      pmax = block_max_f(pmax, s->red_f);
      flag = ok && ((mass < a.threshold) || (own >= pmax && a.threshold > 0.0f));
    }
  }

  phase(1);
  // ---------------- 2a. exact top-M by radix select ----------------
  uint32_t prefix = 0, pmask = 0;
  int need = M;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += kVThreads) s->hist[i] = 0;
    __syncthreads();
    // warp-aggregated: one shared-memory atomic per distinct digit per warp (most keys share the leading byte)
    for (int base = 0; base < V; base += kVThreads) {
      const int i = base + tid;
      const uint32_t u = i < V ? orderable_key(row[i]) : 0u;
      const bool match = i < V && (u & pmask) == prefix;
      const uint32_t digit = match ? (u >> shift) & 255u : 256u;
      const unsigned grp = __match_any_sync(0xffffffffu, digit);
      if (match && lane == __ffs(grp) - 1) atomicAdd(&s->hist[digit], uint32_t(__popc(grp)));
    }
    __syncthreads();
    if (warp == 0) {
      uint32_t c[8], local = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = s->hist[255 - 8 * lane - j];
        local += c[j];
      }
      uint32_t incl = local;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      const uint32_t excl = incl - local;
      if (excl < uint32_t(need) && uint32_t(need) <= incl) {
        uint32_t cum = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (cum + c[j] >= uint32_t(need)) {
            const uint32_t chosen = uint32_t(255 - 8 * lane - j);
            s->need = need - int(cum);
            s->tie_total = int(c[j]);
            s->prefix = prefix | (chosen << shift);
            break;
          }
          cum += c[j];
        }
      }
    }
    __syncthreads();
    prefix = s->prefix;
    need = s->need;
    pmask |= 255u << shift;
  }
  const uint32_t thr = prefix;
  const int take_ties = need;
  const int tie_total = s->tie_total;
  const int n_gt = M - take_ties;

  if (tid == 0) {
    s->cnt_gt = 0;
    s->cnt_tie = 0;
  }
  __syncthreads();
  for (int i = tid; i < V; i += kVThreads) {
    const uint32_t u = orderable_key(row[i]);
    if (u > thr) {
      const int pos = atomicAdd(&s->cnt_gt, 1);
      if (pos < M) s->sel_idx[pos] = i;
    } else if (u == thr && tie_total <= kTieBuffer) {
      const int pos = atomicAdd(&s->cnt_tie, 1);
      if (pos < kTieBuffer) s->ties[pos] = i;
    }
  }
  __syncthreads();
  if (tie_total <= kTieBuffer) {
    for (int e = tid; e < tie_total; e += kVThreads) {
      const int idx = s->ties[e];
      int rank = 0;
      for (int f = 0; f < tie_total; ++f) rank += s->ties[f] < idx ? 1 : 0;
      if (rank < take_ties) s->sel_idx[n_gt + rank] = idx;
    }
  } else {
    // Many equal values at the boundary (a flat row): take the lowest indices by an ordered scan.
    int taken = 0;
    for (int base = 0; base < V && taken < take_ties; base += kVThreads) {
      const int i = base + tid;
      const bool is_tie = i < V && orderable_key(row[i]) == thr;
      const unsigned bal = __ballot_sync(0xffffffffu, is_tie);
      if (lane == 0) s->red_i[warp] = __popc(bal);
      __syncthreads();
      int woff = 0, chunk = 0;
      for (int w = 0; w < 32; ++w) {
        if (w < warp) woff += s->red_i[w];
        chunk += s->red_i[w];
      }
      const int rank = taken + woff + __popc(bal & ((1u << lane) - 1u));
      if (is_tie && rank < take_ties) s->sel_idx[n_gt + rank] = i;
      __syncthreads();
      taken += chunk;
    }
  }
  __syncthreads();
  if (tid < M) {
    const int idx = s->sel_idx[tid];
    const uint32_t k0 = orderable_key(row[idx]);
    int rank = 0;
    for (int f = 0; f < M; ++f) {
      const int j = s->sel_idx[f];
      rank += before(orderable_key(row[j]), j, k0, idx) ? 1 : 0;
    }
    s->tok[rank] = idx;
    s->val[rank] = row[idx];
  }
  __syncthreads();

  phase(2);
  // ---------------- 2b. quota, spread, prior ----------------
  if (tid < M) s->prob[tid] = plm_expf(s->val[tid] - normaliser);
  __syncthreads();
  if (warp == 0) {
    float p = 0.0f;
    for (int m = lane; m < M; m += 32) p = p + s->prob[m];
    p = warp_sum(p);
    if (lane == 0) s->psum = p;
  }
  __syncthreads();
  if (tid < M) {
    const float w = s->prob[tid] / s->psum;
    const float ex = w * float(A);
    const int c = int(floorf(ex));
    s->cnt[tid] = c;
    s->frac[tid] = ex - float(c);
  }
  __syncthreads();
  if (warp == 0) {
    int c = 0;
    for (int m = lane; m < M; m += 32) c += s->cnt[m];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) c += __shfl_xor_sync(0xffffffffu, c, off);
    if (lane == 0) s->remaining = A - c;
  }
  const int ncols = A < 64 ? A : 64;
  if (tid < ncols) {
    float hi = -INFINITY, lo = INFINITY;
    for (int m = 0; m < M; ++m) {
      const float v = table_at(table, s->tok[m], A, tid);
      hi = fmaxf(hi, v);
      lo = fminf(lo, v);
    }
    s->diff[tid] = round_to<T>(hi - lo);
  }
  __syncthreads();
  if (tid < M) {
    const float f = s->frac[tid];
    int rank = 0;
    for (int j = 0; j < M; ++j) {
      const float g = s->frac[j];
      rank += (g > f || (g == f && j < tid)) ? 1 : 0;
    }
    s->counts[tid] = s->cnt[tid] + (rank < s->remaining ? 1 : 0);
  }
  if (warp == 0) {
    float u = 0.0f;
    for (int c = lane; c < ncols; c += 32) u = u + s->diff[c];
    u = warp_sum(u);
    if (lane == 0) s->unit = u / float(ncols);
  }
  __syncthreads();
  const float unit = s->unit;
  if (tid < M) {
    const int c = s->counts[tid];
    const float share = fmaxf(float(c) / float(A), 1e-9f);
    s->bias[tid] = c > 0 ? (-0.1f * unit) * plm_logf(share) : 1000.0f * unit;
  }
  __syncthreads();

  phase(3);
  // ---------------- 3. condense + annealed fit, `rounds` times ----------------
  const int threads_used = A < kVThreads ? A : kVThreads;
  const int ipt = A / threads_used;
  const int nw = threads_used / 32;
  const bool warp_active = warp < nw;
  for (int rd = 0; rd < a.rounds; ++rd) {
    if (tid < M) s->offset[tid] = s->bias[tid];
    __syncthreads();
    int32_t keys[kMaxItemsPerThread][SL];
#pragma unroll
    for (int j = 0; j < kMaxItemsPerThread; ++j) {
      if (j < ipt && warp_active) {
        const int item = j * threads_used + tid;
#pragma unroll
        for (int q = 0; q < SL; ++q) keys[j][q] = INT_MAX;
        for (int m = 0; m < M; ++m) {
          const float cost = table_at(table, s->tok[m], A, item) + s->offset[m];
          int32_t key = condense_key(cost, m);
          if (key < keys[j][SL - 1]) {
            keys[j][SL - 1] = key;
#pragma unroll
            for (int q = SL - 1; q > 0; --q) {
              if (keys[j][q] < keys[j][q - 1]) {
                const int32_t t = keys[j][q];
                keys[j][q] = keys[j][q - 1];
                keys[j][q - 1] = t;
              }
            }
          }
        }
      }
    }
    if (rd == 0) phase(4);
    if (tid < M) {
      s->share[tid] = plm_logf(fmaxf(float(s->counts[tid]), 1e-9f));
      s->corr[tid] = 0.0f;
    }
    for (int i = tid; i < 32 * 128; i += kVThreads) bins[i] = 0.0f;
    float temperature = a.eps[rd] * unit;
    const float bound = 0.25f * unit;
    __syncthreads();
    for (int it = 0; it < a.sweeps; ++it) {
#pragma unroll
      for (int j = 0; j < kMaxItemsPerThread; ++j) {
        if (j < ipt && warp_active) {
          float e[SL];
          int tg[SL];
          float wmax = -INFINITY;
#pragma unroll
          for (int q = 0; q < SL; ++q) {
            tg[q] = keys[j][q] & 0x7F;
            const float cost = condensed_cost(keys[j][q]) + s->corr[tg[q]];
            e[q] = (-cost) / temperature;
            wmax = fmaxf(wmax, e[q]);
          }
          float ws = 0.0f;
#pragma unroll
          for (int q = 0; q < SL; ++q) {
            e[q] = plm_expf(e[q] - wmax);
            ws = ws + e[q];
          }
#pragma unroll
          for (int q = 0; q < SL; ++q) {
            e[q] = e[q] / ws;
            wsh[warp * 32 + lane] = e[q];
            __syncwarp();
            const unsigned grp = __match_any_sync(0xffffffffu, tg[q]);
            if (lane == __ffs(grp) - 1) {
              float g = 0.0f;
              for (unsigned mm = grp; mm != 0; mm &= mm - 1) g = g + wsh[warp * 32 + __ffs(mm) - 1];
              bins[warp * 128 + tg[q]] = bins[warp * 128 + tg[q]] + g;
            }
            __syncwarp();
          }
        }
      }
      __syncthreads();
      if (tid < M) {
        float load = 0.0f;
        for (int w = 0; w < nw; ++w) {
          load = load + bins[w * 128 + tid];
          bins[w * 128 + tid] = 0.0f;
        }
        float step = temperature * (plm_logf(fmaxf(load, 0.01f)) - s->share[tid]);
        step = fminf(fmaxf(step, -bound), bound);
        const float c = s->corr[tid] + 1.9f * step;
        s->corr[tid] = s->counts[tid] > 0 ? c : 0.0f;
      }
      temperature = temperature * a.anneal[rd];
      __syncthreads();
    }
    if (tid < M) s->bias[tid] = s->offset[tid] + s->corr[tid];
    __syncthreads();
    if (rd == 0) phase(5);
  }
  phase(6);

  // ---------------- 4. the row's auxiliary cell ----------------
  if (warp == 0) {
    const int64_t index = (a.aux_base != nullptr ? *a.aux_base : 0) + a.aux_row_offset + r;
    int64_t cell = 0;
    if (index < 0 || index >= a.aux_len) {
      if (lane == 0) record_error(a.err, kErrBadIndex);
    } else {
      cell = a.aux_buf[index];
      if (cell < 0) {
        if (lane == 0) record_error(a.err, kErrBadIndex);
        cell = 0;
      }
      if (cell > A - 1) cell = A - 1;
    }
    float best = INFINITY;
    int bm = INT_MAX;
    for (int m = lane; m < M; m += 32) {
      const float v = table_at(table, s->tok[m], A, int(cell)) + s->bias[m];
      if (v < best || (v == best && m < bm)) {
        best = v;
        bm = m;
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int om = __shfl_xor_sync(0xffffffffu, bm, off);
      if (ob < best || (ob == best && om < bm)) {
        best = ob;
        bm = om;
      }
    }
    if (lane == 0) {
      if (bm < 0 || bm >= M) bm = 0;
      a.verify[r] = s->tok[bm];
      if (a.flags != nullptr) a.flags[r] = flag;
      if (a.dbg_sigma != nullptr) a.dbg_sigma[r] = bm;
      if (a.dbg_phase_ns != nullptr) a.dbg_phase_ns[r * 8 + 7] = int64_t(global_timer_ns() - t_start);
      if (a.dbg_stats != nullptr) {
        a.dbg_stats[r * 4 + 0] = mx;
        a.dbg_stats[r * 4 + 1] = total;
        a.dbg_stats[r * 4 + 2] = normaliser;
        a.dbg_stats[r * 4 + 3] = unit;
      }
    }
  }
  if (tid < M) {
    if (a.dbg_tokens != nullptr) a.dbg_tokens[r * M + tid] = s->tok[tid];
    if (a.dbg_counts != nullptr) a.dbg_counts[r * M + tid] = s->counts[tid];
    if (a.dbg_bias != nullptr) a.dbg_bias[r * M + tid] = s->bias[tid];
  }

  // ---------------- 5. bookkeeping by the last CTA ----------------
  const Bookkeeping& b = a.book;
  if (b.mode == kBookNone) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(a.counter, 1);
    s->last = old == int(gridDim.x) - 1 ? 1 : 0;
  }
  __syncthreads();
  if (s->last == 0) return;
  __threadfence();
  if (tid == 0) *a.counter = 0;
  const int K = b.k;

  if (b.mode == kBookFirstToken) {
    for (int64_t i = tid; i < b.out_cap; i += kVThreads) b.out[i] = -1;
    __syncthreads();
    if (tid == 0) {
      const int64_t first = __ldcg(a.verify);
      b.out[0] = first;
      *b.base = 1;
      *b.anchor = first;
      for (int i = 0; i < K - 1; ++i) b.pending[i] = 0;
      *b.offset = b.prompt_len;
    }
    return;
  }

  if (tid == 0) {
    int nc = 0;
    if (b.mode == kBookSteady) {
      while (nc < K - 1) {
        const bool accepted = __ldcg(a.verify + nc) == b.pending[nc] || __ldcg(a.flags + nc) != 0;
        if (!accepted) break;
        ++nc;
      }
    }
    s->nc = nc;
    s->picked = __ldcg(a.verify + nc);
  }
  __syncthreads();
  const int nc = s->nc;
  // Next pending proposals: rows 1..K-1 of the selected block (steady) or rows 2..K (round 0).
  if (warp < K - 1) {
    const int prow = b.mode == kBookSteady ? K + nc * K + 1 + warp : 2 + warp;
    float best = -INFINITY;
    int bi = INT_MAX;
    if (prow < b.rows) {
      for (int t = lane; t < b.n_tiles; t += 32) {
        const float v = __ldcg(b.best_val + size_t(t) * b.rows + prow);
        const int ix = __ldcg(b.best_idx + size_t(t) * b.rows + prow);
        if (v > best || (v == best && ix < bi)) {
          best = v;
          bi = ix;
        }
      }
    } else if (lane == 0) {
      record_error(a.err, kErrBadShape);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, off);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (lane == 0) s->new_pending[warp] = bi == INT_MAX ? 0 : bi;
  }
  __syncthreads();
  if (tid == 0) {
    const int64_t base = *b.base;
    const int64_t picked = s->picked;
    for (int j = 0; j < K; ++j) {
      const int64_t slot = base + j;
      if (slot < 0 || slot >= b.out_cap) {
        if (j <= nc) record_error(a.err, kErrBadIndex);
        continue;
      }
      if (j < nc) b.out[slot] = j < K - 1 ? b.pending[j] : __ldcg(a.verify + K - 1);
      else if (j == nc) b.out[slot] = picked;
    }
    if (b.mode == kBookSteady) {
      const int64_t step = *b.sequence_step;
      b.round_sequence[step < b.seq_cap - 1 ? step : b.seq_cap - 1] = nc;
      *b.sequence_step = step + 1;
    }
    for (int i = 0; i < K - 1; ++i) b.pending[i] = s->new_pending[i];
    *b.anchor = picked;
    *b.base = base + nc + 1;
    *b.offset = *b.offset + nc + 1;
  }
}

template <typename T, int SL>
int launch_verify(const VerifyArgs& a, int n_rows, cudaStream_t stream, bool pdl) {
  const bool row_in_smem = size_t(a.vocab) * 4 <= kRowSmemLimit;
  const size_t row_bytes = row_in_smem ? size_t(a.vocab) * 4 : 0;
  const size_t union_bytes = (row_bytes > kFitScratchBytes ? row_bytes : kFitScratchBytes);
  const size_t smem = ((union_bytes + 15) & ~size_t(15)) + sizeof(VerifySmem);
  auto kernel = verify_decode_kernel<T, SL>;
  static size_t attr_bytes = 0;
  if (attr_bytes < smem) {
    int st = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)),
                        "cudaFuncSetAttribute(verify smem)");
    if (st != PLM_OK) return st;
    attr_bytes = smem;
  }
  return check_cuda(launch(kernel, dim3(n_rows), dim3(kVThreads), smem, stream, pdl, a), "verify_decode_kernel");
}

}  // namespace

int verify_launch(const VerifyArgs& a, int dtype, int n_rows, cudaStream_t stream, bool pdl) {
  if (dtype != PLM_BF16) return fail(PLM_ERR_UNSUPPORTED, "verify decode: only bf16 tables are built");
  switch (a.shortlist) {
    case 1: return launch_verify<__nv_bfloat16, 1>(a, n_rows, stream, pdl);
    case 2: return launch_verify<__nv_bfloat16, 2>(a, n_rows, stream, pdl);
    case 4: return launch_verify<__nv_bfloat16, 4>(a, n_rows, stream, pdl);
    case 8: return launch_verify<__nv_bfloat16, 8>(a, n_rows, stream, pdl);
  }
  return fail(PLM_ERR_UNSUPPORTED, "verify decode: shortlist %d (1, 2, 4 or 8)", a.shortlist);
}

int verify_validate(const VerifyArgs& a, int n_rows) {
  if (n_rows < 1 || n_rows > 32) return fail(PLM_ERR_INVALID, "verify decode: %d rows (1..32)", n_rows);
  if (a.logits == nullptr || a.table == nullptr || a.verify == nullptr || a.aux_buf == nullptr)
    return fail(PLM_ERR_INVALID, "verify decode: null operand");
  if (a.top_m < 1 || a.top_m > kMaxTopM || (a.top_m & (a.top_m - 1)) != 0)
    return fail(PLM_ERR_UNSUPPORTED, "verify decode: top_m %d must be a power of two <= %d", a.top_m, kMaxTopM);
  if (a.vocab < a.top_m) return fail(PLM_ERR_INVALID, "verify decode: vocab %d < top_m %d", a.vocab, a.top_m);
  if (a.aux < 32 || a.aux > kVThreads * kMaxItemsPerThread || (a.aux & (a.aux - 1)) != 0)
    return fail(PLM_ERR_UNSUPPORTED, "verify decode: aux vocabulary %d must be a power of two in [32, 4096]", a.aux);
  if (a.shortlist > a.top_m) return fail(PLM_ERR_INVALID, "verify decode: shortlist > top_m");
  if (a.rounds < 0 || a.rounds > 4 || a.sweeps < 0) return fail(PLM_ERR_INVALID, "verify decode: rounds/sweeps");
  if (a.n_accept > 0 && a.pending == nullptr) return fail(PLM_ERR_INVALID, "verify decode: pending missing");
  if (a.book.mode != kBookNone) {
    const Bookkeeping& b = a.book;
    if (a.counter == nullptr || b.out == nullptr || b.base == nullptr || b.offset == nullptr ||
        b.anchor == nullptr || b.pending == nullptr)
      return fail(PLM_ERR_INVALID, "verify decode: bookkeeping state missing");
    if (b.k < 1 || b.k > 32) return fail(PLM_ERR_INVALID, "verify decode: k=%d", b.k);
    if (b.mode == kBookSteady && (n_rows != b.k || a.flags == nullptr || b.round_sequence == nullptr ||
                                  b.sequence_step == nullptr || b.seq_cap < 1))
      return fail(PLM_ERR_INVALID, "verify decode: steady bookkeeping needs k rows, flags and the round record");
    if ((b.mode == kBookRound0 || b.mode == kBookFirstToken) && n_rows != 1)
      return fail(PLM_ERR_INVALID, "verify decode: round-0 / first-token bookkeeping decodes one row");
    if (b.mode != kBookFirstToken && (b.best_val == nullptr || b.best_idx == nullptr || b.n_tiles < 1))
      return fail(PLM_ERR_INVALID, "verify decode: proposal argmax partials missing");
  }
  return PLM_OK;
}

}  // namespace plm

using namespace plm;

extern "C" int plm_verify_decode(plm_ctx* ctx, const plm_verify_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_verify_decode: null argument");
  VerifyArgs a = {};
  a.logits = d->logits;
  a.vocab = d->vocab;
  a.logits_stride = d->logits_stride > 0 ? d->logits_stride : d->vocab;
  a.table = d->table;
  a.aux = d->aux;
  a.aux_buf = d->aux_buf;
  a.aux_len = d->aux_len;
  a.aux_base = d->aux_base;
  a.aux_row_offset = d->aux_row_offset;
  a.pending = d->pending;
  a.n_accept = d->n_accept;
  a.rule = d->rule;
  a.threshold = d->threshold;
  a.top_m = d->top_m;
  a.shortlist = d->shortlist;
  a.rounds = d->rounds;
  a.sweeps = d->sweeps;
  for (int r = 0; r < 4; ++r) {
    // plm/iterate.py:333-336: epsilon for the first fit, epsilon * refocus after; the per-sweep anneal factor is
    // (endpoint / epsilon) ** (1 / sweeps) in double precision, handed to the kernel as fp32.
    const double eps = r == 0 ? d->epsilon : d->epsilon * d->refocus;
    a.eps[r] = float(eps);
    a.anneal[r] = float(pow(d->endpoint / eps, 1.0 / double(d->sweeps > 1 ? d->sweeps : 1)));
  }
  a.verify = d->verify;
  a.flags = d->flags;
  a.dbg_tokens = d->dbg_tokens;
  a.dbg_counts = d->dbg_counts;
  a.dbg_bias = d->dbg_bias;
  a.dbg_stats = d->dbg_stats;
  a.dbg_sigma = d->dbg_sigma;
  a.dbg_phase_ns = d->dbg_phase_ns;
  const plm_bookkeeping& b = d->book;
  a.book = Bookkeeping{b.mode,       b.k,     b.best_val, b.best_idx,       b.n_tiles, b.rows,
                       b.out,        b.out_cap, b.base,   b.offset,         b.anchor,  b.pending,
                       b.round_sequence, b.seq_cap, b.sequence_step, b.prompt_len};
  a.counter = ctx->counters + (ctx->n_counters - 1);
  a.err = ctx->err;
  int st = verify_validate(a, d->n_rows);
  if (st != PLM_OK) return st;
  return verify_launch(a, d->dtype, d->n_rows, static_cast<cudaStream_t>(stream), true);
}
