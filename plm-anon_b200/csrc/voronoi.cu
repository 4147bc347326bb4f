// Verify decode, acceptance and round bookkeeping (compiled with -fmad=false: bit-exact with the CPU oracle).
//
// Each verify row is decoded by a cluster of kCluster CTAs of kThreads threads; rank q of the cluster owns the
// vocabulary slice [q * L, (q + 1) * L), L = ceil(V / kCluster), and the auxiliary items [q * A / kCluster, ...).
//   1. softmax statistics: the row maximum (exact), the sum of exp(x - max) of each slice in the block order of
//      oracle.exact.block_sum with 256 threads, slice sums added in rank order; normaliser = max + log(sum). The
//      relaxed acceptance rule of the row's pending proposal (plm/decoder.py:71-82) uses the same partitioned sums.
//   2. the exact top-m shortlist: a 4-pass radix select on order-preserving keys inside each slice (ties: lower index
//      first), then every rank merges the kCluster sorted candidate lists (read through distributed shared memory)
//      by ranking each candidate against the other lists with binary searches. Quota (largest remainder, equal
//      remainders by shortlist position), spread and prior (plm/iterate.py:248-290) are computed by every rank
//      identically.
//   3. `rounds` x (condense each owned item to its `shortlist` cheapest targets, then `sweeps` annealed Sinkhorn
//      sweeps, plm/iterate.py:83-159, 292-312). A sweep's per-target load is summed without atomics: inside a rank,
//      one warp sums a target's entries (owned items ascending) in lane_sum order — lane l adds entries l, l + 32, ...
//      sequentially, then an xor butterfly; every rank stores its partials into every rank's shared memory and
//      arrives on the receiver's mbarrier (one wait per sweep, double-buffered by sweep parity); the kCluster partials
//      are added in rank order.
//   4. sigma(cell) = argmin_m C[m, cell] + b[m] for the row's auxiliary cell and its token (plm/auxiliary.py:67-75).
// The last cluster to finish runs the round's bookkeeping (plm/decoder.py:351-365 steady, 275-310 round 0, 384 first
// token after the prefill): accepted count, output tokens, the accepted-count record, the next pending proposals
// from the lm_head's per-tile argmax partials, anchor, base and offset (the implicit KV commit).
// Every floating-point step is a separate IEEE operation in a fixed order and exp/log come from plm_math.h; the numpy
// oracle (oracle/voronoi.py) performs the same operations.
#include <climits>
#include <map>
#include <mutex>

#include "common.cuh"
#include "plm_math.h"
#include "runtime.h"
#include "verify.h"

namespace plm {
using namespace plm_math;

namespace {

constexpr int kCluster = kVerifyCluster;
constexpr int kThreads = kVerifyThreads;
constexpr int kWarps = kThreads / 32;
constexpr int kMaxTopM = 128;
constexpr int kMaxSlice = 8192;                 // vocabulary up to kCluster * kMaxSlice
constexpr int kMaxOwned = 512;                  // auxiliary items per rank (A <= 4096)
constexpr int kWords = kMaxOwned / 32;
constexpr int kTieBuffer = 1024;
constexpr int kMaxEntries = kMaxOwned * 8;
constexpr int kTargetsPerWarp = kMaxTopM / kWarps;
constexpr int kPrefilterBins = 2048;  // the top 11 bits of the orderable key
constexpr int kCandBuffer = kCluster * kMaxTopM;  // prefiltered candidates held in all_key / all_idx
static_assert(kTargetsPerWarp == 16, "the transposed butterfly reduces 16 targets per warp");

struct VerifySmem {
  float slice[kMaxSlice];
  uint32_t hist[kPrefilterBins];  // radix histograms (256 bins) and the prefilter's (2048)
  int ties[kTieBuffer];
  uint32_t cand_key[kMaxTopM];  // this rank's sorted candidates, read by every rank of the cluster
  int cand_idx[kMaxTopM];
  uint32_t all_key[kCluster * kMaxTopM];  // every rank's candidates, copied locally for the merge
  int all_idx[kCluster * kMaxTopM];
  int sel_pos[kMaxTopM];
  uint32_t sel_key[kMaxTopM];
  uint32_t sort_key[kMaxTopM];
  int sort_idx[kMaxTopM];
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
  alignas(16) float recv[2][kCluster][kMaxTopM];  // every rank's per-target load partial, double-buffered by sweep parity
  alignas(16) float mine[kMaxTopM];  // this rank's partials of the sweep, staged for the 16-byte pushes
  uint64_t recv_bar[2];  // completes when all kCluster ranks have stored their partials of a sweep
  float diff[64];
  float spread_hi[kThreads / 64][64];
  float spread_lo[kThreads / 64][64];
  uint32_t bitmap[kMaxTopM][kWords];  // owned items holding each target
  int list_begin[kMaxTopM + 1];
  int pos_of[kMaxEntries];  // an entry's (owned item * SL + slot) position in target order, items ascending
  int32_t keybuf[kMaxEntries];  // condensed keys of the owned items
  float wbuf[kMaxEntries];  // the sweep's weights in target order
  float red_f[32];
  int red_i[32];
  float xchg[4];  // per-rank scalars read by the cluster: max, sum, mass, max probability
  int cand_n;
  int64_t new_pending[32];
  int need, tie_total, cnt_gt, cnt_tie, remaining, last, nc;
  int pre_bin, pre_count, n_buf;
  int warp_tot[kWarps];
  uint32_t prefix;
  float psum, unit;
  int64_t picked;
};

__device__ __forceinline__ float block_sum_f(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float w = lane < kWarps ? red[lane] : 0.0f;
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
    float w = lane < kWarps ? red[lane] : -INFINITY;
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

// warp_sum (xor 16, 8, 4, 2, 1) of 16 values per lane at once: after the step with distance d a lane keeps the half
// of its targets selected by its bit d and adds the partner's copy, so every kept value equals warp_sum's partial at
// that lane. Lane l returns target l >> 1's sum.
__device__ __forceinline__ float transposed_warp_sum(const float (&p)[16], int lane) {
  float q8[8], q4[4], q2[2];
  const bool b16 = lane & 16, b8 = lane & 8, b4 = lane & 4, b2 = lane & 2;
#pragma unroll
  for (int i = 0; i < 8; ++i) q8[i] = (b16 ? p[i + 8] : p[i]) + __shfl_xor_sync(0xffffffffu, b16 ? p[i] : p[i + 8], 16);
#pragma unroll
  for (int i = 0; i < 4; ++i) q4[i] = (b8 ? q8[i + 4] : q8[i]) + __shfl_xor_sync(0xffffffffu, b8 ? q8[i] : q8[i + 4], 8);
#pragma unroll
  for (int i = 0; i < 2; ++i) q2[i] = (b4 ? q4[i + 2] : q4[i]) + __shfl_xor_sync(0xffffffffu, b4 ? q4[i] : q4[i + 2], 4);
  const float q1 = (b2 ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? q2[0] : q2[1], 2);
  return q1 + __shfl_xor_sync(0xffffffffu, q1, 1);
}

// Canonical order: larger key first, then lower index.
__device__ __forceinline__ bool before(uint32_t ka, int ia, uint32_t kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// The canonical top-`want` of n elements whose (key, index) `get(pos, key, index)` returns, written sorted to
// out_key / out_idx. Radix select on the key (4 passes of 8 bits, warp-aggregated histogram); elements above the
// threshold key are taken, equal keys lowest index first. Beyond kTieBuffer equal keys at the threshold (a flat
// row), equal keys must appear at ascending positions in ascending index order (true for a vocabulary slice).
// Returns the count.
template <typename Get>
__device__ int select_top(Get get, int n, int want, VerifySmem* s, uint32_t* out_key, int* out_idx) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (want > n) want = n;
  if (want <= 0) return 0;
  uint32_t prefix = 0, pmask = 0;
  int need = want;
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += kThreads) s->hist[i] = 0;
    __syncthreads();
    for (int base = 0; base < n; base += kThreads) {
      const int i = base + tid;
      uint32_t u = 0;
      int idx = 0;
      if (i < n) get(i, u, idx);
      const bool match = i < n && (u & pmask) == prefix;
      const uint32_t digit = match ? (u >> shift) & 255u : 256u;
      // most keys of a row share their leading bytes: one atomic when the whole warp agrees, else one per lane
      const uint32_t d0 = __shfl_sync(0xffffffffu, digit, 0);
      if (__all_sync(0xffffffffu, digit == d0)) {
        if (lane == 0 && d0 != 256u) atomicAdd(&s->hist[d0], 32u);
      } else if (match) {
        atomicAdd(&s->hist[digit], 1u);
      }
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
            s->need = need - int(cum);
            s->tie_total = int(c[j]);
            s->prefix = prefix | (uint32_t(255 - 8 * lane - j) << shift);
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
  const int take_ties = need, tie_total = s->tie_total, n_gt = want - take_ties;
  if (tid == 0) {
    s->cnt_gt = 0;
    s->cnt_tie = 0;
  }
  __syncthreads();
  for (int i = tid; i < n; i += kThreads) {
    uint32_t u;
    int idx;
    get(i, u, idx);
    if (u > thr) {
      const int pos = atomicAdd(&s->cnt_gt, 1);
      if (pos < want) s->sel_pos[pos] = i;
    } else if (u == thr && tie_total <= kTieBuffer) {
      const int pos = atomicAdd(&s->cnt_tie, 1);
      if (pos < kTieBuffer) s->ties[pos] = i;
    }
  }
  __syncthreads();
  if (tie_total <= kTieBuffer) {
    for (int e = tid; e < tie_total; e += kThreads) {
      const int pe = s->ties[e];
      uint32_t ue;
      int ie;
      get(pe, ue, ie);
      int rank = 0;
      for (int f = 0; f < tie_total; ++f) {
        uint32_t uf;
        int i_f;
        get(s->ties[f], uf, i_f);
        rank += i_f < ie ? 1 : 0;
      }
      if (rank < take_ties) s->sel_pos[n_gt + rank] = pe;
    }
  } else {
    // many equal keys at the boundary (a flat row): ordered scan over positions
    int taken = 0;
    for (int base = 0; base < n && taken < take_ties; base += kThreads) {
      const int i = base + tid;
      uint32_t u = 0;
      int idx = 0;
      if (i < n) get(i, u, idx);
      const bool is_tie = i < n && u == thr;
      const unsigned bal = __ballot_sync(0xffffffffu, is_tie);
      if (lane == 0) s->red_i[warp] = __popc(bal);
      __syncthreads();
      int woff = 0, chunk = 0;
      for (int w = 0; w < kWarps; ++w) {
        if (w < warp) woff += s->red_i[w];
        chunk += s->red_i[w];
      }
      const int rank = taken + woff + __popc(bal & ((1u << lane) - 1u));
      if (is_tie && rank < take_ties) s->sel_pos[n_gt + rank] = i;
      __syncthreads();
      taken += chunk;
    }
  }
  __syncthreads();
  if (tid < want) {  // the selected (key, index) pairs, gathered once for the rank sort
    uint32_t k0;
    int i0;
    get(s->sel_pos[tid], k0, i0);
    s->sort_key[tid] = k0;
    s->sort_idx[tid] = i0;
  }
  __syncthreads();
  for (int m = tid; m < want; m += kThreads) {
    const uint32_t k0 = s->sort_key[m];
    const int i0 = s->sort_idx[m];
    int rank = 0;
#pragma unroll 8
    for (int f = 0; f < want; ++f) rank += before(s->sort_key[f], s->sort_idx[f], k0, i0) ? 1 : 0;
    out_key[rank] = k0;
    out_idx[rank] = i0;
  }
  __syncthreads();
  return want;
}

template <typename T, int SL>
__global__ void __launch_bounds__(kThreads, 1) verify_decode_kernel(const VerifyArgs a) {
  extern __shared__ __align__(16) uint8_t vsmem[];
  VerifySmem* s = reinterpret_cast<VerifySmem*>(vsmem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t rank = cluster_rank();
  const int r = blockIdx.x / kCluster;  // verify row
  const int V = a.vocab, A = a.aux, M = a.top_m;
  const int slice_len = (V + kCluster - 1) / kCluster;
  const int v0 = min(V, int(rank) * slice_len), v1 = min(V, v0 + slice_len);
  const int n_slice = v1 - v0;
  const int owned = A / kCluster;
  const int item0 = int(rank) * owned;
  const int words = (owned + 31) / 32;
  const T* table = reinterpret_cast<const T*>(a.table);

  if (tid == 0) {  // published to the cluster by the first cluster_sync below
    mbar_init(&s->recv_bar[0], kCluster);  // one arrival per sending rank
    mbar_init(&s->recv_bar[1], kCluster);
    fence_barrier_init();
  }
  grid_dependency_wait();
  allow_dependents();
  const uint64_t t_start = global_timer_ns();
  auto phase = [&](int k) {
    if (a.dbg_phase_ns != nullptr && tid == 0 && rank == 0)
      a.dbg_phase_ns[r * kPhaseSlots + k] = int64_t(global_timer_ns() - t_start);
  };

  // ---------------- 1. statistics of the row ----------------
  const float* grow = a.logits + size_t(r) * a.logits_stride;
  for (int i = tid; i < n_slice; i += kThreads) s->slice[i] = grow[v0 + i];
  __syncthreads();
  float mx = -INFINITY;
  for (int i = tid; i < n_slice; i += kThreads) mx = fmaxf(mx, s->slice[i]);
  mx = block_max_f(mx, s->red_f);
  if (tid == 0) s->xchg[0] = mx;
  cluster_sync();
  {
    float part[kCluster];
#pragma unroll
    for (int q = 0; q < kCluster; ++q) part[q] = ld_dsmem_f32(cluster_map(&s->xchg[0], uint32_t(q)));
#pragma unroll
    for (int q = 0; q < kCluster; ++q) mx = fmaxf(mx, part[q]);
  }
  float acc = 0.0f;
  for (int i = tid; i < n_slice; i += kThreads) acc = acc + plm_expf(s->slice[i] - mx);
  acc = block_sum_f(acc, s->red_f);
  if (tid == 0) s->xchg[1] = acc;
  cluster_sync();
  float total = 0.0f;
  {
    float part[kCluster];
#pragma unroll
    for (int q = 0; q < kCluster; ++q) part[q] = ld_dsmem_f32(cluster_map(&s->xchg[1], uint32_t(q)));
#pragma unroll
    for (int q = 0; q < kCluster; ++q) total = total + part[q];
  }
  const float normaliser = mx + plm_logf(total);
  phase(0);

  int flag = 0;
  if (r < a.n_accept && (a.rule == kRuleFloor || a.threshold > 0.0f)) {  // uniform over the cluster
    int64_t pt = a.pending[r];
    const bool ok = pt >= 0 && pt < V;
    if (!ok) {
      if (tid == 0 && rank == 0) record_error(a.err, kErrBadIndex);
      pt = 0;
    }
    const float own_logit = grow[pt];
    if (a.rule == kRuleFloor) {
      flag = ok && ((own_logit - normaliser) > plm_logf(a.threshold));
    } else {
      const float own = plm_expf(own_logit - mx) / total;
      float mass = 0.0f, pmax = -INFINITY;
      for (int i = tid; i < n_slice; i += kThreads) {
        const float pi = plm_expf(s->slice[i] - mx) / total;
        pmax = fmaxf(pmax, pi);
        if (pi > own) mass = mass + pi;
      }
      mass = block_sum_f(mass, s->red_f);
      pmax = block_max_f(pmax, s->red_f);
      if (tid == 0) {
        s->xchg[2] = mass;
        s->xchg[3] = pmax;
      }
      cluster_sync();
      float masses[kCluster], pmaxes[kCluster];
#pragma unroll
      for (int q = 0; q < kCluster; ++q) {
        masses[q] = ld_dsmem_f32(cluster_map(&s->xchg[2], uint32_t(q)));
        pmaxes[q] = ld_dsmem_f32(cluster_map(&s->xchg[3], uint32_t(q)));
      }
      float total_mass = 0.0f;
#pragma unroll
      for (int q = 0; q < kCluster; ++q) {
        total_mass = total_mass + masses[q];
        pmax = fmaxf(pmax, pmaxes[q]);
      }
      flag = ok && ((total_mass < a.threshold) || (own >= pmax && a.threshold > 0.0f));
    }
  }
  phase(1);

  // With tokens_given the rows' tokens were decoded before this launch (the PTP scheme's inverse CDF): only the
  // relaxed rule's verdicts and the bookkeeping remain.
  if (a.tokens_given) {
    if (rank == 0 && tid == 0 && a.flags != nullptr) a.flags[r] = flag;
  } else {
  // ---------------- 2a. exact top-M: per slice, then merged over the cluster ----------------
  // Prefilter: a histogram of the keys' top 11 bits finds the bin holding the slice's want-th largest key; the
  // elements at or above that bin (usually a few hundred) are compacted into all_key / all_idx and the exact top-want
  // is taken among them (rank counting when they fit one per thread, else the radix select). A flat row whose
  // candidates overflow the buffer takes the radix select over the whole slice.
  {
    auto get_slice = [&](int i, uint32_t& u, int& idx) {
      u = orderable_key(s->slice[i]);
      idx = v0 + i;
    };
    const int want = min(M, n_slice);
    for (int i = tid; i < kPrefilterBins; i += kThreads) s->hist[i] = 0;
    if (tid == 0) s->n_buf = 0;
    __syncthreads();
    for (int i = tid; i < n_slice; i += kThreads) atomicAdd(&s->hist[orderable_key(s->slice[i]) >> 21], 1u);
    __syncthreads();
    if (want > 0) {  // thread t scans bins 2047 - 8t downwards; a block scan over threads finds the boundary bin
      constexpr int kPer = kPrefilterBins / kThreads;
      uint32_t c[kPer], local = 0;
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        c[j] = s->hist[kPrefilterBins - 1 - kPer * tid - j];
        local += c[j];
      }
      uint32_t incl = local;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t o = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += o;
      }
      if (lane == 31) s->warp_tot[warp] = int(incl);
      __syncthreads();
      uint32_t before_warp = 0;
      for (int w = 0; w < warp; ++w) before_warp += uint32_t(s->warp_tot[w]);
      incl += before_warp;
      const uint32_t excl = incl - local;
      if (excl < uint32_t(want) && uint32_t(want) <= incl) {
        uint32_t cum = excl;
#pragma unroll
        for (int j = 0; j < kPer; ++j) {
          if (cum + c[j] >= uint32_t(want)) {
            s->pre_bin = kPrefilterBins - 1 - kPer * tid - j;
            s->pre_count = int(cum + c[j]);
            break;
          }
          cum += c[j];
        }
      }
    }
    __syncthreads();
    const bool prefiltered = want > 0 && s->pre_count <= kCandBuffer;
    if (prefiltered) {
      const uint32_t bin = uint32_t(s->pre_bin);
      for (int base = 0; base < n_slice; base += kThreads) {
        const int i = base + tid;
        const uint32_t u = i < n_slice ? orderable_key(s->slice[i]) : 0u;
        const bool take = i < n_slice && (u >> 21) >= bin;
        const unsigned bal = __ballot_sync(0xffffffffu, take);
        int pos0 = 0;
        if (lane == 0 && bal != 0u) pos0 = atomicAdd(&s->n_buf, __popc(bal));
        pos0 = __shfl_sync(0xffffffffu, pos0, 0);
        if (take) {
          const int pos = pos0 + __popc(bal & ((1u << lane) - 1u));
          s->all_key[pos] = u;
          s->all_idx[pos] = v0 + i;
        }
      }
      __syncthreads();
      const int nb = s->n_buf;
      if (nb <= kThreads) {
        if (tid < nb) {
          const uint32_t k0 = s->all_key[tid];
          const int i0 = s->all_idx[tid];
          int rk = 0;
          for (int f = 0; f < nb; ++f) rk += before(s->all_key[f], s->all_idx[f], k0, i0) ? 1 : 0;
          if (rk < want) {
            s->cand_key[rk] = k0;
            s->cand_idx[rk] = i0;
          }
        }
        __syncthreads();
      } else {
        auto get_buf = [&](int i, uint32_t& u, int& idx) {
          u = s->all_key[i];
          idx = s->all_idx[i];
        };
        select_top(get_buf, nb, want, s, s->cand_key, s->cand_idx);
      }
    } else if (want > 0) {
      select_top(get_slice, n_slice, want, s, s->cand_key, s->cand_idx);
    }
    if (tid == 0) s->cand_n = want;
  }
  phase(2);
  cluster_sync();
  {
    constexpr int kPer = kCluster * kMaxTopM / kThreads;
    uint32_t keyv[kPer];
    int idxv[kPer], nq[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kThreads;
      const uint32_t q = uint32_t(e / kMaxTopM);
      const int j = e % kMaxTopM;
      nq[u] = int(ld_dsmem_u32(cluster_map(&s->cand_n, q)));
      keyv[u] = ld_dsmem_u32(cluster_map(&s->cand_key[j], q));
      idxv[u] = int(ld_dsmem_u32(cluster_map(&s->cand_idx[j], q)));
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int e = tid + u * kThreads;
      const bool real = (e % kMaxTopM) < nq[u];
      s->all_key[e] = real ? keyv[u] : 0u;  // below every finite value's key: padding never wins
      s->all_idx[e] = real ? idxv[u] : INT_MAX;
    }
  }
  __syncthreads();
  phase(3);
  // Top-M of the kCluster sorted lists by pairwise merges in log2(kCluster) levels: the elementwise better of list a
  // and list b reversed holds the top kMaxTopM of both as a bitonic sequence, which a half-cleaner cascade sorts.
  for (int width = 1; width < kCluster; width <<= 1) {
    const int merges = kCluster / (2 * width);
    for (int e = tid; e < merges * kMaxTopM; e += kThreads) {
      const int la = (e / kMaxTopM) * 2 * width * kMaxTopM, lb = la + width * kMaxTopM, i = e % kMaxTopM;
      const uint32_t kb = s->all_key[lb + kMaxTopM - 1 - i];
      const int ib = s->all_idx[lb + kMaxTopM - 1 - i];
      if (before(kb, ib, s->all_key[la + i], s->all_idx[la + i])) {
        s->all_key[la + i] = kb;
        s->all_idx[la + i] = ib;
      }
    }
    __syncthreads();
    for (int j = kMaxTopM / 2; j > 0; j >>= 1) {
      for (int e = tid; e < merges * kMaxTopM / 2; e += kThreads) {
        const int h = e % (kMaxTopM / 2);
        const int i = (e / (kMaxTopM / 2)) * 2 * width * kMaxTopM + (h / j) * 2 * j + h % j;
        const uint32_t k0 = s->all_key[i], k1 = s->all_key[i + j];
        const int i0 = s->all_idx[i], i1 = s->all_idx[i + j];
        if (before(k1, i1, k0, i0)) {
          s->all_key[i] = k1;
          s->all_idx[i] = i1;
          s->all_key[i + j] = k0;
          s->all_idx[i + j] = i0;
        }
      }
      __syncthreads();
    }
  }
  if (tid < M) {
    s->sel_key[tid] = s->all_key[tid];
    s->tok[tid] = s->all_idx[tid];
  }
  __syncthreads();
  phase(4);
  if (tid < M) s->val[tid] = grow[s->tok[tid]];
  // The rank's owned columns of the shortlist's table rows, staged once for both rounds' condense (the vocabulary
  // slice is no longer needed); [m][owned item]
  // with 16-byte cp.async copies where rows and columns are 16-byte aligned; they land while the quota, spread and
  // prior are computed
  __syncthreads();
  T* tcol = reinterpret_cast<T*>(s->slice);
  const bool staged = size_t(owned) * size_t(M) * sizeof(T) <= sizeof(s->slice);
  constexpr int kChunk = 16 / int(sizeof(T));
  const bool staged_async = staged && A % kChunk == 0 && owned % kChunk == 0 &&
                            (reinterpret_cast<uintptr_t>(table) & 15u) == 0;
  if (staged_async) {
    const int per_row = owned / kChunk;
    for (int e = tid; e < M * per_row; e += kThreads) {
      const int m = e / per_row, c = e - m * per_row;
      cp_async_16(tcol + m * owned + c * kChunk, table + size_t(s->tok[m]) * A + item0 + c * kChunk);
    }
    cp_async_commit();
  } else if (staged) {
    for (int e = tid; e < M * owned; e += kThreads) {
      const int m = e / owned, li = e - m * owned;
      tcol[e] = table[size_t(s->tok[m]) * A + item0 + li];
    }
  }
  phase(5);

  // ---------------- 2b. quota, spread, prior (every rank identically) ----------------
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
  {  // max and min (exact in any order) over quarters of the shortlist, then combined
    const int c = tid & 63, quarter = tid >> 6;
    float hi = -INFINITY, lo = INFINITY;
    if (c < ncols) {
      for (int m = quarter; m < M; m += kThreads / 64) {
        const float v = table_at(table, s->tok[m], A, c);
        hi = fmaxf(hi, v);
        lo = fminf(lo, v);
      }
    }
    s->spread_hi[quarter][c] = hi;
    s->spread_lo[quarter][c] = lo;
  }
  __syncthreads();
  if (tid < ncols) {
    float hi = s->spread_hi[0][tid], lo = s->spread_lo[0][tid];
#pragma unroll
    for (int q = 1; q < kThreads / 64; ++q) {
      hi = fmaxf(hi, s->spread_hi[q][tid]);
      lo = fminf(lo, s->spread_lo[q][tid]);
    }
    s->diff[tid] = round_to<T>(hi - lo);
  }
  __syncthreads();
  if (tid < M) {
    const float f = s->frac[tid];
    int rk = 0;
    for (int j = 0; j < M; ++j) {
      const float g = s->frac[j];
      rk += (g > f || (g == f && j < tid)) ? 1 : 0;
    }
    s->counts[tid] = s->cnt[tid] + (rk < s->remaining ? 1 : 0);
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
  if (staged_async) cp_async_wait<0>();
  __syncthreads();
  phase(6);

  // ---------------- 3. condense + annealed fit, `rounds` times ----------------
  // condense: one thread per owned item; keys land in shared memory. fit: two threads per item, slots split in
  // halves (HALF each); per-target loads by one warp per target in lane_sum order over the target's entries.
  constexpr int HALF = SL > 1 ? SL / 2 : 1;
  constexpr int kPairs = kThreads / 2;
  constexpr int kPairIters = kMaxOwned / kPairs;
  const int pair = tid >> 1, side = tid & 1;
  const bool side_active = SL > 1 || side == 0;
  int sweep = 0;  // sweeps so far over all rounds: recv buffer = sweep & 1, its mbarrier phase = (sweep >> 1) & 1
  for (int rd = 0; rd < a.rounds; ++rd) {
    if (tid < M) s->offset[tid] = s->bias[tid];
    for (int i = tid; i < kMaxTopM * kWords; i += kThreads) (&s->bitmap[0][0])[i] = 0u;
    __syncthreads();
    for (int li0 = 0; li0 < owned; li0 += kPairs) {
      const int li = li0 + pair;
      int32_t keys[SL];
#pragma unroll
      for (int q = 0; q < SL; ++q) keys[q] = INT_MAX;
      if (li < owned) {  // this thread's half of the targets; the SL smallest keys, ascending
        const int half = (M + 1) / 2;
        const int m_end = side ? M : half;
        // batches of 8 targets; each key enters the sorted list through a branch-free min/max chain (the largest
        // falls off the end), so lanes never diverge and consecutive keys pipeline through the chain
        for (int m8 = side ? half : 0; m8 < m_end; m8 += 8) {
          int32_t kb[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int m = m8 + u;
            kb[u] = INT_MAX;
            if (m < m_end) {
              const float tv = staged ? to_f32<T>(tcol[m * owned + li]) : table_at(table, s->tok[m], A, item0 + li);
              kb[u] = condense_key(tv + s->offset[m], m);
            }
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            int32_t x = kb[u];
#pragma unroll
            for (int q = 0; q < SL; ++q) {
              const int32_t lo = min(keys[q], x);
              x = max(keys[q], x);
              keys[q] = lo;
            }
          }
        }
      }
      // the pair's two sorted lists: the elementwise smaller of mine and the partner's reversed is the SL smallest
      // of both as a bitonic sequence, sorted by a half-cleaner cascade
      int32_t other[SL];
#pragma unroll
      for (int q = 0; q < SL; ++q) other[q] = __shfl_xor_sync(0xffffffffu, keys[q], 1);
#pragma unroll
      for (int q = 0; q < SL; ++q) keys[q] = min(keys[q], other[SL - 1 - q]);
#pragma unroll
      for (int j = SL / 2; j > 0; j >>= 1) {
#pragma unroll
        for (int q = 0; q < SL; ++q) {
          if ((q & j) == 0 && keys[q + j] < keys[q]) {
            const int32_t t = keys[q];
            keys[q] = keys[q + j];
            keys[q + j] = t;
          }
        }
      }
      if (li < owned && side == 0) {
#pragma unroll
        for (int q = 0; q < SL; ++q) {
          s->keybuf[li * SL + q] = keys[q];
          atomicOr(&s->bitmap[keys[q] & 0x7F][li >> 5], 1u << (li & 31));
        }
      }
    }
    __syncthreads();
    if (rd == 0) phase(7);
    if (rd == 1) phase(9);
    if (warp == 0) {  // list offsets: exclusive scan of the per-target counts
      int run = 0;
      for (int m0 = 0; m0 < kMaxTopM; m0 += 32) {
        const int m = m0 + lane;
        int c = 0;
        for (int w = 0; w < words; ++w) c += __popc(s->bitmap[m][w]);
        int incl = c;
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const int o = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += o;
        }
        s->list_begin[m] = run + incl - c;
        run += __shfl_sync(0xffffffffu, incl, 31);
      }
      if (lane == 0) s->list_begin[kMaxTopM] = run;
    }
    __syncthreads();
    for (int e = tid; e < owned * SL; e += kThreads) {  // each entry at its target's offset + owned items below it
      const int li = e / SL;
      const int m = s->keybuf[e] & 0x7F;
      int below = 0;
      for (int w = 0; w < (li >> 5); ++w) below += __popc(s->bitmap[m][w]);
      below += __popc(s->bitmap[m][li >> 5] & ((1u << (li & 31)) - 1u));
      s->pos_of[e] = s->list_begin[m] + below;
    }
    if (tid < M) {
      s->share[tid] = plm_logf(fmaxf(float(s->counts[tid]), 1e-9f));
      s->corr[tid] = 0.0f;
    }
    float temperature = a.eps[rd] * unit;
    const float bound = 0.25f * unit;
    __syncthreads();
    // For this round's sweeps: where the thread's weights go in target order, and the warp's targets
    // t * kWarps + warp (interleaved, so the shortlist's popular head is spread over the warps) with their ranges.
    int wpos[kPairIters][HALF];
#pragma unroll
    for (int j = 0; j < kPairIters; ++j) {
      const int li = pair + j * kPairs;
#pragma unroll
      for (int u = 0; u < HALF; ++u) wpos[j][u] = li < owned && side_active ? s->pos_of[li * SL + side * HALF + u] : 0;
    }
    int tb[kTargetsPerWarp], tn[kTargetsPerWarp];
    int chunks = 0;
#pragma unroll
    for (int t = 0; t < kTargetsPerWarp; ++t) {
      const int m = t * kWarps + warp;
      tb[t] = s->list_begin[m];
      tn[t] = s->list_begin[m + 1] - tb[t];
      chunks = max(chunks, (tn[t] + 31) / 32);
    }
    for (int it = 0; it < a.sweeps; ++it, ++sweep) {
      const int parity = sweep & 1;
      // weights: the pair's two threads hold slots [0, HALF) and [HALF, SL); max and the sequential sum over the
      // slots cross the pair by shuffles, so the order is that of one thread doing all slots
#pragma unroll
      for (int j = 0; j < kPairIters; ++j) {
        if (j * kPairs >= owned) break;  // uniform over the block
        const int li = pair + j * kPairs;
        const bool valid = li < owned;
        float e[HALF];
        float wmax = -INFINITY;
#pragma unroll
        for (int u = 0; u < HALF; ++u) {
          e[u] = -INFINITY;
          if (valid && side_active) {
            const int32_t key = s->keybuf[li * SL + side * HALF + u];
            const float cost = condensed_cost(key) + s->corr[key & 0x7F];
            e[u] = (-cost) / temperature;
            wmax = fmaxf(wmax, e[u]);
          }
        }
        if (SL > 1) wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, 1));
        float part = 0.0f;
#pragma unroll
        for (int u = 0; u < HALF; ++u) {
          e[u] = plm_expf(e[u] - wmax);
          if (side == 0) part = part + e[u];
        }
        float ws = part;
        if (SL > 1) {
          const float first = __shfl_sync(0xffffffffu, part, (lane & ~1));
          if (side == 1) {
            ws = first;
#pragma unroll
            for (int u = 0; u < HALF; ++u) ws = ws + e[u];
          }
          ws = __shfl_sync(0xffffffffu, ws, lane | 1);
        }
        if (valid && side_active) {
#pragma unroll
          for (int u = 0; u < HALF; ++u) s->wbuf[wpos[j][u]] = e[u] / ws;
        }
      }
      __syncthreads();
      // this rank's partial per target, the warp's targets read from wbuf in target order: lane l sums the target's
      // entries l, l + 32, ... sequentially (an absent entry adds 0, and 0 + w is w), then the xor butterfly of
      // warp_sum for all the warp's targets at once: each step hands half of the lane's targets to its partner
      // Each rank then pushes its partials into recv[parity][rank] of every rank and arrives on the receiver's
      // recv_bar[parity]; a rank's next push into the same buffer needs everyone's partials of the sweep in between,
      // so a buffer is never overwritten before its reader is done with it.
      {
        float p[kTargetsPerWarp];
#pragma unroll
        for (int t = 0; t < kTargetsPerWarp; ++t) p[t] = lane < tn[t] ? s->wbuf[tb[t] + lane] : 0.0f;
        // entries l + 32, l + 64, ... chunk by chunk, the loads of all the warp's targets of a chunk in flight together;
        // each target still adds its entries in order (past its end it adds 0, which leaves the nonnegative sum as is)
        for (int c = 1; c < chunks; ++c) {
          const int i = lane + 32 * c;
#pragma unroll
          for (int t = 0; t < kTargetsPerWarp; ++t) p[t] = p[t] + (i < tn[t] ? s->wbuf[tb[t] + i] : 0.0f);
        }
        const float total = transposed_warp_sum(p, lane);
        if ((lane & 1) == 0) s->mine[(lane >> 1) * kWarps + warp] = total;
      }
      __syncthreads();
      // pushed with 16-byte stores (thread q * 32 + c sends targets [4c, 4c + 4) to rank q), then one release arrival
      // per receiving rank once the whole CTA has stored
      if (tid < kCluster * (kMaxTopM / 4) && (tid & 31) * 4 < M) {
        const int c4 = (tid & 31) * 4;
        st_dsmem_f32x4(cluster_map(&s->recv[parity][rank][c4], uint32_t(tid >> 5)),
                       *reinterpret_cast<const float4*>(&s->mine[c4]));
      }
      __syncthreads();
      if (tid < kCluster) mbar_arrive_remote(cluster_map(&s->recv_bar[parity], uint32_t(tid)));
      if (tid < M) {
        mbar_wait_cluster(&s->recv_bar[parity], uint32_t(sweep >> 1) & 1u, a.err, kErrTimeoutPeer);
        float load = 0.0f;
#pragma unroll
        for (int q = 0; q < kCluster; ++q) load = load + s->recv[parity][q][tid];
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
    if (rd == 0) phase(8);
    if (rd == 1) phase(10);
  }
  cluster_sync();  // no rank leaves while another still reads its shared memory
  phase(11);

  // ---------------- 4. the row's auxiliary cell ----------------
  if (rank == 0 && warp == 0) {
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
      if (a.dbg_stats != nullptr) {
        a.dbg_stats[r * 4 + 0] = mx;
        a.dbg_stats[r * 4 + 1] = total;
        a.dbg_stats[r * 4 + 2] = normaliser;
        a.dbg_stats[r * 4 + 3] = unit;
      }
      if (a.dbg_phase_ns != nullptr) a.dbg_phase_ns[r * kPhaseSlots + 12] = int64_t(global_timer_ns() - t_start);
    }
  }
  if (rank == 0 && tid < M) {
    if (a.dbg_tokens != nullptr) a.dbg_tokens[r * M + tid] = s->tok[tid];
    if (a.dbg_counts != nullptr) a.dbg_counts[r * M + tid] = s->counts[tid];
    if (a.dbg_bias != nullptr) a.dbg_bias[r * M + tid] = s->bias[tid];
  }

  }  // !a.tokens_given

  // ---------------- 5. bookkeeping by the last cluster ----------------
  const Bookkeeping& b = a.book;
  if (b.mode == kBookNone || rank != 0) return;
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(a.counter, 1);
    s->last = old == int(gridDim.x / kCluster) - 1 ? 1 : 0;
  }
  __syncthreads();
  if (s->last == 0) return;
  __threadfence();
  if (tid == 0) *a.counter = 0;
  const int K = b.k;
  // A request that has already stopped: the round was queued behind the one that ended it and commits nothing.
  if (b.mode == kBookSteady && b.stop != nullptr && __ldcg(b.stop + kStopDone) != 0) {
    if (tid == 0 && b.commit != nullptr) b.commit[1] = 0;
    return;
  }

  if (b.mode == kBookFirstToken) {
    for (int64_t i = tid; i < b.out_cap; i += kThreads) b.out[i] = -1;
    __syncthreads();
    if (tid == 0) {
      const int64_t first = __ldcg(a.verify);
      b.out[0] = first;
      *b.base = 1;
      *b.anchor = first;
      for (int i = 0; i < K - 1; ++i) b.pending[i] = 0;
      *b.offset = b.prompt_len;
      if (b.stop != nullptr) b.stop[kStopDone] = 0;
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
  // next pending proposals: rows 1..K-1 of the selected block (steady) or rows 2..K (round 0)
  for (int i = warp; i < K - 1; i += kWarps) {
    const int prow = b.mode == kBookSteady ? K + nc * K + 1 + i : 2 + i;
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
    if (lane == 0) s->new_pending[i] = bi == INT_MAX ? 0 : bi;
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
      if (j < nc) b.out[slot] = b.pending[j];
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
    const int64_t committed = *b.offset;
    if (b.commit != nullptr) {  // verify rows 0 .. nc go to logical indices offset .. offset + nc
      b.commit[0] = committed;
      b.commit[1] = nc + 1;
    }
    *b.offset = committed + nc + 1;
    if (b.mode == kBookSteady && b.stop != nullptr) {
      // The stop test of the reference's host loop (plm/decoder.py:414-439) on the tokens this round confirmed.
      const int64_t next = base + nc + 1;
      bool done = next >= b.stop[kStopBudget];
      const int64_t eos = b.stop[kStopEos];
      if (eos >= 0) {
        const int64_t end = min(min(next, b.stop[kStopWindow]), b.out_cap);
        for (int64_t j = max(base, int64_t(0)); j < end; ++j) done = done || b.out[j] == eos;
      }
      if (done) b.stop[kStopDone] = 1;
    }
  }
}

template <typename T, int SL>
int launch_verify(const VerifyArgs& a, int n_rows, cudaStream_t stream, bool pdl) {
  const size_t smem = sizeof(VerifySmem);
  auto kernel = verify_decode_kernel<T, SL>;
  const int st =
      raise_smem_limit(reinterpret_cast<const void*>(kernel), int(smem), "cudaFuncSetAttribute(verify smem)");
  if (st != PLM_OK) return st;
  return check_cuda(launch_cluster(kernel, dim3(kCluster * n_rows), dim3(kThreads), smem, stream, pdl, kCluster, 1, a),
                    "verify_decode_kernel");
}

}  // namespace

int verify_launch(const VerifyArgs& a, int dtype, int n_rows, cudaStream_t stream, bool pdl) {
  if (dtype != PLM_BF16 && dtype != PLM_F16) return fail(PLM_ERR_INVALID, "verify decode: dtype %d", dtype);
  if (dtype == PLM_F16) {
    switch (a.shortlist) {
      case 1: return launch_verify<__half, 1>(a, n_rows, stream, pdl);
      case 2: return launch_verify<__half, 2>(a, n_rows, stream, pdl);
      case 4: return launch_verify<__half, 4>(a, n_rows, stream, pdl);
      case 8: return launch_verify<__half, 8>(a, n_rows, stream, pdl);
    }
  }
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
  if (a.tokens_given) {  // rule verdicts and bookkeeping only: no Voronoi table, cells or shortlist
    if (a.logits == nullptr || a.verify == nullptr) return fail(PLM_ERR_INVALID, "verify decode: null operand");
    if (a.vocab < 1 || a.vocab > kCluster * kMaxSlice)
      return fail(PLM_ERR_UNSUPPORTED, "verify decode: vocab %d (1..%d)", a.vocab, kCluster * kMaxSlice);
  } else {
  if (a.logits == nullptr || a.table == nullptr || a.verify == nullptr || a.aux_buf == nullptr)
    return fail(PLM_ERR_INVALID, "verify decode: null operand");
  if (a.top_m < 1 || a.top_m > kMaxTopM || (a.top_m & (a.top_m - 1)) != 0)
    return fail(PLM_ERR_UNSUPPORTED, "verify decode: top_m %d must be a power of two <= %d", a.top_m, kMaxTopM);
  if (a.vocab < a.top_m || a.vocab > kCluster * kMaxSlice)
    return fail(PLM_ERR_UNSUPPORTED, "verify decode: vocab %d (top_m..%d)", a.vocab, kCluster * kMaxSlice);
  if (a.aux < 32 || a.aux > kCluster * kMaxOwned || (a.aux & (a.aux - 1)) != 0)
    return fail(PLM_ERR_UNSUPPORTED, "verify decode: aux vocabulary %d must be a power of two in [32, %d]", a.aux,
                kCluster * kMaxOwned);
  if (a.shortlist > a.top_m) return fail(PLM_ERR_INVALID, "verify decode: shortlist > top_m");
  if (a.rounds < 0 || a.rounds > 4 || a.sweeps < 0) return fail(PLM_ERR_INVALID, "verify decode: rounds/sweeps");
  }
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
                       b.round_sequence, b.seq_cap, b.sequence_step, b.prompt_len, b.stop, b.commit};
  a.counter = ctx->counters + (ctx->n_counters - 1);
  a.err = ctx->err;
  int st = verify_validate(a, d->n_rows);
  if (st != PLM_OK) return st;
  return verify_launch(a, d->dtype, d->n_rows, static_cast<cudaStream_t>(stream), true);
}

// ---------------------------------------------------------------------------------------------------------------
// plm_verify_decode_static: the same kernel with no context and no allocation. Its scratch (the bookkeeping arrival
// counter, the device error word when the caller gives none, and the per-row decoded tokens and verdicts when the
// caller gives no buffers for them) is this file-scope array of kStaticScratchBytes. Callers that cannot allocate
// device memory use it: a host runtime bound over a foreign-function interface whose device memory belongs to its
// own allocator, or a decode loop that must not stall, since cudaMalloc / cudaFree synchronise the device.
// ---------------------------------------------------------------------------------------------------------------
namespace {

constexpr int kStaticScratchBytes = 1024;
constexpr int kStaticRows = 32;          // per-row slots; the kernel decodes at most 32 rows per launch
constexpr int kStaticTokensOffset = 256; // int64 tokens [kStaticRows]
constexpr int kStaticFlagsOffset = 512;  // int32 verdicts [kStaticRows]
static_assert(kStaticTokensOffset + 8 * kStaticRows <= kStaticFlagsOffset, "static scratch layout");
static_assert(kStaticFlagsOffset + 4 * kStaticRows <= kStaticScratchBytes, "static scratch layout");

// Word 0: arrival counter. It is zero at module load, and every launch leaves it at zero: each cluster's rank 0
// arrives exactly once (a wait that runs out of time still reaches the arrival), and the last to arrive resets it.
// Word 1: device error word when the caller passes none. Errors recorded there cannot be read back through the
// C ABI; callers that need them pass their own zeroed int32.
static __device__ __align__(256) unsigned char g_verify_static_scratch[kStaticScratchBytes];

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);

// The context's process-unique id (cuCtxGetId), or 0 when there is no current context or the driver lacks the call.
unsigned long long current_context_id() {
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (get_current == nullptr || get_id == nullptr || get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return 0;
  return get_id(ctx, &id) == CUDA_SUCCESS ? id : 0;
}

// Device address of the scratch in the current context, resolved by cudaGetSymbolAddress the first time a context
// calls. The cache is keyed on the context's process-unique id, so a context created after cudaDeviceReset (which
// reloads the module elsewhere) resolves its own address instead of reusing a stale one.
int static_scratch(unsigned char** out) {
  static std::mutex mu;
  static std::map<unsigned long long, unsigned char*> resolved;
  unsigned long long id = current_context_id();
  if (id != 0) {
    std::lock_guard<std::mutex> lock(mu);
    const auto it = resolved.find(id);
    if (it != resolved.end()) {
      *out = it->second;
      return PLM_OK;
    }
  }
  void* addr = nullptr;
  const int st = check_cuda(cudaGetSymbolAddress(&addr, g_verify_static_scratch),
                            "plm_verify_decode_static: cudaGetSymbolAddress(scratch)");
  if (st != PLM_OK) return st;
  *out = static_cast<unsigned char*>(addr);
  id = current_context_id();  // the call above made the device's primary context current if none was
  if (id != 0) {
    std::lock_guard<std::mutex> lock(mu);
    resolved[id] = *out;
  }
  return PLM_OK;
}

}  // namespace

extern "C" int plm_verify_decode_static(const plm_verify_desc* d, int32_t* device_error, void* stream) {
  if (d == nullptr) return fail(PLM_ERR_INVALID, "plm_verify_decode_static: null descriptor");
  if (d->n_rows > kStaticRows)
    return fail(PLM_ERR_INVALID, "plm_verify_decode_static: %d rows exceed the static scratch's %d row slots (%d bytes)",
                d->n_rows, kStaticRows, kStaticScratchBytes);
  unsigned char* scratch = nullptr;
  int st = static_scratch(&scratch);
  if (st != PLM_OK) return st;
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
  for (int r = 0; r < 4; ++r) {  // as plm_verify_decode (plm/iterate.py:333-336)
    const double eps = r == 0 ? d->epsilon : d->epsilon * d->refocus;
    a.eps[r] = float(eps);
    a.anneal[r] = float(pow(d->endpoint / eps, 1.0 / double(d->sweeps > 1 ? d->sweeps : 1)));
  }
  a.verify = d->verify != nullptr ? d->verify : reinterpret_cast<int64_t*>(scratch + kStaticTokensOffset);
  a.flags = d->flags != nullptr ? d->flags : reinterpret_cast<int32_t*>(scratch + kStaticFlagsOffset);
  a.dbg_tokens = d->dbg_tokens;
  a.dbg_counts = d->dbg_counts;
  a.dbg_bias = d->dbg_bias;
  a.dbg_stats = d->dbg_stats;
  a.dbg_sigma = d->dbg_sigma;
  a.dbg_phase_ns = d->dbg_phase_ns;
  const plm_bookkeeping& b = d->book;
  a.book = Bookkeeping{b.mode,       b.k,     b.best_val, b.best_idx,       b.n_tiles, b.rows,
                       b.out,        b.out_cap, b.base,   b.offset,         b.anchor,  b.pending,
                       b.round_sequence, b.seq_cap, b.sequence_step, b.prompt_len, b.stop, b.commit};
  a.counter = reinterpret_cast<int*>(scratch);
  a.err = device_error != nullptr ? device_error : reinterpret_cast<int*>(scratch) + 1;
  st = verify_validate(a, d->n_rows);
  if (st != PLM_OK) return st;
  return verify_launch(a, d->dtype, d->n_rows, static_cast<cudaStream_t>(stream), true);
}
