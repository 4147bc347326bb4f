// Inverse-CDF verify decode of the PTP scheme, the linear-interpolation auxiliary scheme of the reference's
// gated-LoRA model (plm/auxiliary.py:104-113): for each row, the softmax at temperature 1 over the vocabulary, its
// top_k largest probabilities put in token-id order and renormalised, and the token of the first bin whose right
// edge exceeds the row's uniform u (the last edge is 1).
//
// One CTA of 1024 threads per row; the row's probabilities stay in shared memory (vocab <= kIcdfMaxVocab).
//   1. the maximum and the sum of exp(x - max) (block reductions), then p = e / sum;
//   2. the top_k-th largest p by a radix select over the float bits, 8 bits a pass (p >= 0, so the bits order like
//      the values); histogram updates are aggregated per warp and bin;
//   3. the chosen ids in ascending order by a block-wide compaction over the vocabulary in id order: every p above
//      the threshold, then the lowest ids among those equal to it;
//   4. one thread renormalises in float32, forms the right edges as a running sum in double rounded to float32 (a
//      float32 cumulative sum as torch computes it on the CPU), and takes the first edge above u.
#include <cmath>

#include "common.cuh"
#include "icdf.h"
#include "runtime.h"

namespace plm {
namespace {

constexpr int kIcdfThreads = 1024;
constexpr int kIcdfWarps = kIcdfThreads / 32;


__device__ __forceinline__ float block_max(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = red[0];
  for (int w = 1; w < kIcdfWarps; ++w) m = fmaxf(m, red[w]);
  return m;
}

__device__ __forceinline__ float block_sum(float v, float* red) {
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < kIcdfWarps; ++w) s += red[w];
  return s;
}

// Exclusive prefix count of `flag` over the CTA in thread order; `*total` gets the CTA's count.
__device__ __forceinline__ int block_exclusive_count(bool flag, int* red, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const unsigned ballot = __ballot_sync(0xffffffffu, flag);
  const int below = __popc(ballot & ((1u << lane) - 1u));
  __syncthreads();  // the previous call's totals have been read
  if (lane == 0) red[warp] = __popc(ballot);
  __syncthreads();
  int before = 0, all = 0;
  for (int w = 0; w < kIcdfWarps; ++w) {
    const int c = red[w];
    if (w < warp) before += c;
    all += c;
  }
  *total = all;
  return before + below;
}

__global__ void __launch_bounds__(kIcdfThreads, 1) icdf_decode_kernel(const IcdfArgs a) {
  extern __shared__ __align__(16) float p[];  // [vocab]
  __shared__ float fred[kIcdfWarps];
  __shared__ int ired[kIcdfWarps];
  __shared__ unsigned hist[256];
  __shared__ int chosen_id[kIcdfMaxTopK];
  __shared__ float chosen_p[kIcdfMaxTopK];
  __shared__ unsigned s_prefix;
  __shared__ int s_need;

  const int row = blockIdx.x, tid = threadIdx.x, lane = tid & 31;
  const int V = a.vocab, K = a.top_k;
  grid_dependency_wait();  // the logits may come from the previous kernel
  const float* x = a.logits + size_t(row) * size_t(a.ld);

  // 1. softmax at temperature 1
  float m = -INFINITY;
  for (int i = tid; i < V; i += kIcdfThreads) m = fmaxf(m, x[i]);
  m = block_max(m, fred);
  float s = 0.f;
  for (int i = tid; i < V; i += kIcdfThreads) {
    const float e = expf(x[i] - m);
    p[i] = e;
    s += e;
  }
  s = block_sum(s, fred);
  for (int i = tid; i < V; i += kIcdfThreads) p[i] = p[i] / s;
  __syncthreads();

  // 2. radix select: after the pass over bits [shift, shift + 8), `prefix` holds the top bits of the K-th largest
  // bit pattern and `need` how many of the patterns that share them are still to be taken from the top
  unsigned prefix = 0u, mask = 0u;
  int need = K;
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int b = tid; b < 256; b += kIcdfThreads) hist[b] = 0u;
    __syncthreads();
    for (int i0 = 0; i0 < V; i0 += kIcdfThreads) {  // every lane runs every step: the match below needs all 32
      const int i = i0 + tid;
      const unsigned bits = i < V ? __float_as_uint(p[i]) : 0u;
      const bool in = i < V && (bits & mask) == prefix;
      const unsigned bin = (bits >> shift) & 255u;
      const unsigned peers = __match_any_sync(0xffffffffu, in ? bin : 256u + unsigned(lane));
      if (in && lane == __ffs(peers) - 1) atomicAdd(&hist[bin], unsigned(__popc(peers)));
    }
    __syncthreads();
    if (tid == 0) {
      int above = 0, b = 255;
      for (; b > 0; --b) {
        if (above + int(hist[b]) >= need) break;
        above += int(hist[b]);
      }
      s_prefix = prefix | (unsigned(b) << shift);
      s_need = need - above;
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
    mask |= 255u << shift;
  }
  const unsigned threshold = prefix;

  // 3. the chosen ids in ascending order
  int taken = 0, ties = 0;
  for (int i0 = 0; i0 < V; i0 += kIcdfThreads) {
    const int i = i0 + tid;
    const unsigned bits = i < V ? __float_as_uint(p[i]) : 0u;
    const bool above = i < V && bits > threshold, tie = i < V && bits == threshold;
    int tie_count = 0, take_count = 0;
    const int tie_rank = ties + block_exclusive_count(tie, ired, &tie_count);
    const bool take = above || (tie && tie_rank < need);
    const int pos = taken + block_exclusive_count(take, ired, &take_count);
    if (take && pos < K) {
      chosen_id[pos] = i;
      chosen_p[pos] = p[i];
    }
    ties += tie_count;
    taken += take_count;
  }
  __syncthreads();

  // 4. renormalise, right edges, the bin of u
  if (tid == 0) {
    if (taken != K) record_error(a.err, kErrBadIndex);
    const int k = taken < K ? taken : K;
    float total = 0.f;
    for (int j = 0; j < k; ++j) total += chosen_p[j];
    float u = 0.f;
    if (a.u_base == nullptr) {
      u = a.u[row];
    } else {  // the round's uniforms: the request's stream from the round's first output position
      const int64_t index = *a.u_base + row;
      if (index < 0 || index >= a.u_len) record_error(a.err, kErrBadIndex);
      else u = a.u[index];
    }
    double run = 0.0;
    int bin = -1;
    for (int j = 0; j < k; ++j) {
      run += double(chosen_p[j] / total);
      const float edge = j == k - 1 ? 1.0f : float(run);
      if (bin < 0 && edge > u) bin = j;
      if (a.edges_out != nullptr) a.edges_out[size_t(row) * K + j] = edge;
      if (a.ids_out != nullptr) a.ids_out[size_t(row) * K + j] = chosen_id[j];
    }
    if (bin < 0) bin = k - 1;  // u >= 1: the last bin
    a.tokens[row] = k > 0 ? int64_t(chosen_id[bin]) : 0;
  }
}

}  // namespace

int icdf_launch(const IcdfArgs& a, cudaStream_t stream, bool pdl) {
  const int smem = a.vocab * int(sizeof(float));
  int st = raise_smem_limit(reinterpret_cast<const void*>(icdf_decode_kernel), smem,
                            "cudaFuncSetAttribute(icdf smem)");
  if (st != PLM_OK) return st;
  return check_cuda(launch(icdf_decode_kernel, dim3(a.n_rows), dim3(kIcdfThreads), size_t(smem), stream, pdl, a),
                    "icdf_decode_kernel");
}

}  // namespace plm

using namespace plm;

extern "C" int plm_icdf_decode(plm_ctx* ctx, const plm_icdf_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_icdf_decode: null argument");
  if (!d->logits || !d->u || !d->tokens) return fail(PLM_ERR_INVALID, "plm_icdf_decode: null operand");
  if (d->n_rows < 1 || d->vocab < 1 || d->vocab > kIcdfMaxVocab || d->ld < d->vocab)
    return fail(PLM_ERR_UNSUPPORTED, "plm_icdf_decode: %d rows over a vocabulary of %d (ld %lld; at most %d)",
                d->n_rows, d->vocab, (long long)d->ld, kIcdfMaxVocab);
  if (d->top_k < 1 || d->top_k > kIcdfMaxTopK || d->top_k > d->vocab)
    return fail(PLM_ERR_UNSUPPORTED, "plm_icdf_decode: top_k %d (1..%d, at most the vocabulary)", d->top_k,
                kIcdfMaxTopK);
  IcdfArgs a = {d->logits, d->ld, d->u, d->n_rows, d->vocab, d->top_k, d->tokens, d->ids_out, d->edges_out,
                nullptr, 0, ctx->err};
  return icdf_launch(a, static_cast<cudaStream_t>(stream), true);
}
