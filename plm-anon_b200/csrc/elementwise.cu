// Row-wise kernels of the round: the prologue (ids, auxiliary cells, embeddings, rotary positions, KV slots)
// fused with the first RMSNorm, the residual-add RMSNorm between sublayers, and a standalone paged KV append.
#include "common.cuh"
#include "elementwise.h"
#include "runtime.h"

namespace plm {
namespace {

constexpr int kRowThreads = 256;
constexpr int kVec = 8;      // 16-byte vectors of bf16
constexpr int kMaxVecs = 2;  // vectors per thread: hidden <= kRowThreads * kVec * kMaxVecs = 4096
constexpr int kMaxNormPartials = 16;  // k-split partials an add_norm may sum
constexpr int kNormThreads = 256;     // add_norm: at most, one or two quads of 4 elements a thread
constexpr int kNormQuads = 2;         // hidden <= 4 * kNormThreads * kNormQuads * (cluster of 2) = 4096

// The row's 16-byte vectors owned by this thread: vector j is elements [8 (tid + j 256), ... + 8).
template <typename T>
__device__ __forceinline__ void load_row(const T* __restrict__ src, int hidden, uint4 (&out)[kMaxVecs]) {
#pragma unroll
  for (int j = 0; j < kMaxVecs; ++j) {
    const int c = threadIdx.x + j * kRowThreads;
    out[j] = c * kVec < hidden ? reinterpret_cast<const uint4*>(src)[c] : make_uint4(0, 0, 0, 0);
  }
}

template <typename T>
__device__ __forceinline__ float elem(const uint4& v, int e) {
  return to_f32<T>(reinterpret_cast<const T*>(&v)[e]);
}

__device__ __forceinline__ float block_sum_rows(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float r = 0.f;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) r += red[w];
  return r;
}

// One CTA per row. Writes residual (the embedding, model dtype) and normed = RMSNorm(embedding) * w.
//   ids: steady round [anchor, pending..., V x k^2]; round 0 [anchor, V x (W-1)]; prefill chunk prompt[offset + r].
//   Rows whose id lies in [V, V + num_aux_tokens) take auxiliary_vocabulary[min(cell, A - 1)] (mask_auxiliary if
//   the cell is the sentinel A), all others embed_tokens[clamp(id, 0, V - 1)] (plm/decoder.py:264-268, 331-349;
//   plm/auxiliary.py:50-54). The row's rotary position is offset + rel_positions[r] and its KV slot the physical
//   slot of logical index offset + r through the block table (plm/decoder.py:340, 347), or for a round's rows
//   (round_scratch) row r of the round scratch, from which the commit copies the accepted rows into the pages.
template <typename T>
__global__ void __launch_bounds__(kRowThreads) embed_norm_kernel(const PrologueArgs a) {
  __shared__ float red[32];
  __shared__ int64_t s_id, s_cell;
  __shared__ float s_u;
  const int r = blockIdx.x, tid = threadIdx.x;
  grid_dependency_wait();
  if (r == 0 && a.counters != nullptr)
    for (int i = tid; i < a.n_counters; i += kRowThreads) a.counters[i] = 0;
  const int64_t offset = *a.offset;
  if (tid == 0) {
    int64_t id = a.vocab, cell = a.aux;  // proposal placeholder; masked sentinel cell
    int64_t position = offset + (a.rel_positions != nullptr ? a.rel_positions[r] : r);
    if (a.mode == kProloguePrefill) {
      const int64_t p = offset + r;
      if (p < 0 || p >= a.prompt_cap) {
        record_error(a.err, kErrBadIndex);
        id = 0;
      } else {
        id = a.prompt[p];
      }
    } else {
      if (r == 0) id = *a.anchor;
      else if (a.mode == kPrologueSteady && r < a.k) id = a.pending[r - 1];
      const int64_t rel_aux = a.rel_aux[r];
      s_u = 0.f;  // the PTP scheme's value of rows without an auxiliary value (plm/decoder.py:107-108)
      if (rel_aux >= 0) {
        const int64_t index = *a.base + rel_aux;
        if (index < 0 || index >= a.aux_len) {
          record_error(a.err, kErrBadIndex);
          cell = 0;
        } else if (a.ptp_embedding != nullptr) {
          s_u = a.aux_u[index];
        } else {
          cell = a.aux_buf[index];
        }
      }
    }
    if (position < 0 || position >= a.max_pos) {
      record_error(a.err, kErrBadIndex);
      position = 0;
    }
    a.positions[r] = int32_t(position);
    const int64_t logical = offset + r;
    const int64_t lp = logical / a.page_size;
    const int page = (logical >= 0 && lp < a.max_pages) ? a.block_table[lp] : -1;
    if (a.round_scratch) {
      a.slots[r] = r;  // a round's rows are candidates: their K/V wait in the round scratch for the commit
    } else if (page < 0 || page >= a.num_pages) {
      record_error(a.err, kErrBadIndex);
      a.slots[r] = -1;
    } else {
      a.slots[r] = int64_t(page) * a.page_size + logical % a.page_size;
    }
    s_id = id;
    s_cell = cell;
  }
  __syncthreads();
  const int64_t id = s_id;
  const bool aux_row = id >= a.vocab && id < int64_t(a.vocab) + a.num_aux_tokens;
  const T* src;
  if (aux_row) {
    const int64_t cell = s_cell;
    if (cell == a.aux) {
      src = reinterpret_cast<const T*>(a.mask_aux);
    } else {
      const int64_t c = cell < 0 ? 0 : (cell > a.aux - 1 ? a.aux - 1 : cell);
      src = reinterpret_cast<const T*>(a.aux_vocab) + size_t(c) * a.hidden;
    }
  } else {
    const int64_t tok = id < 0 ? 0 : (id > a.vocab - 1 ? a.vocab - 1 : id);
    src = reinterpret_cast<const T*>(a.embed) + size_t(tok) * a.hidden;
  }
  T* __restrict__ res = reinterpret_cast<T*>(a.residual) + size_t(r) * a.hidden;
  T* __restrict__ nrm = reinterpret_cast<T*>(a.normed) + size_t(r) * a.hidden;
  const T* __restrict__ w = reinterpret_cast<const T*>(a.norm_weight);
  uint4 e[kMaxVecs], wv[kMaxVecs];
  if (aux_row && a.ptp_embedding != nullptr) {
    // LinearInterpolationAuxiliary.embed (plm/auxiliary.py:96-102): u scaled to [0, n - 1], the two neighbouring
    // float32 rows weighted by the fraction, each step rounded on its own (no fused multiply-add), then cast to the
    // model dtype (plm/decoder.py:264-268).
    const int last = a.ptp_rows - 1;
    const float scaled = __fmul_rn(s_u, float(last));
    const float below = floorf(scaled);
    const int lo = max(0, min(last, int(below)));
    const int hi = min(lo + 1, last);
    const float frac = __fsub_rn(scaled, below);
    const float keep = __fsub_rn(1.0f, frac);
    const float* rlo = a.ptp_embedding + size_t(lo) * a.hidden;
    const float* rhi = a.ptp_embedding + size_t(hi) * a.hidden;
#pragma unroll
    for (int j = 0; j < kMaxVecs; ++j) {
      const int c = tid + j * kRowThreads;
      if (c * kVec >= a.hidden) continue;
      T* ev = reinterpret_cast<T*>(&e[j]);
#pragma unroll
      for (int q = 0; q < kVec; ++q)
        ev[q] = from_f32<T>(__fadd_rn(__fmul_rn(rlo[c * kVec + q], keep), __fmul_rn(rhi[c * kVec + q], frac)));
    }
  } else {
    load_row<T>(src, a.hidden, e);
  }
  load_row<T>(w, a.hidden, wv);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxVecs; ++j) {
    const int c = tid + j * kRowThreads;
    if (c * kVec < a.hidden) {
      reinterpret_cast<uint4*>(res)[c] = e[j];
#pragma unroll
      for (int q = 0; q < kVec; ++q) ss += elem<T>(e[j], q) * elem<T>(e[j], q);
    }
  }
  ss = block_sum_rows(ss, red);
  allow_dependents();  // the first qkv projection is let in once the rows' sums are known, as after add_norm
  const float rstd = rsqrtf(ss / float(a.hidden) + a.eps);
#pragma unroll
  for (int j = 0; j < kMaxVecs; ++j) {
    const int c = tid + j * kRowThreads;
    if (c * kVec < a.hidden) {
      uint4 o;
      T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int q = 0; q < kVec; ++q) ov[q] = from_f32<T>(round_to<T>(elem<T>(e[j], q) * rstd) * elem<T>(wv[j], q));
      reinterpret_cast<uint4*>(nrm)[c] = o;
    }
  }
}

// A cluster of CS CTAs per row (CS = 4, or 2 when hidden is not a multiple of 16): residual <- x + residual;
// normed <- RMSNorm(x + residual) * w (vLLM fused_add_rms_norm: the sum is formed in fp32, stored rounded as the new
// residual, and normalised unrounded). CTA q of the row's cluster owns columns [q hidden / CS, (q + 1) hidden / CS),
// in quads of 4 elements, one or two per thread, so each SM takes in a CS-th of the row's k-split partials. The
// CTAs' sums of squares are exchanged through distributed shared memory and added in rank order. With gather_row >= 0
// the normed row `gather_row` is also copied to `gathered` (the prefill's last prompt row).
template <typename T, int CS>
__global__ void __launch_bounds__(kNormThreads) add_norm_kernel(const AddNormArgs a) {
  __shared__ float red[kNormThreads / 32];
  __shared__ float row_ss[CS];  // every CTA's sum of squares, pushed by the CTA itself
  const uint32_t rank = cluster_rank();
  const int r = blockIdx.x / CS, tid = threadIdx.x, nthreads = blockDim.x;
  const int quads = a.hidden / (4 * CS), q0 = int(rank) * quads;  // this CTA's quads [q0, q0 + quads)
  cluster_arrive_relaxed();  // paired with the wait before the push: every CTA of the cluster has started by then
  const T* __restrict__ x = reinterpret_cast<const T*>(a.x) + size_t(r) * a.hidden;
  T* __restrict__ res = reinterpret_cast<T*>(a.residual) + size_t(r) * a.hidden;
  T* __restrict__ nrm = reinterpret_cast<T*>(a.normed) + size_t(r) * a.hidden;
  T* gathered = (r == a.gather_row && a.gathered != nullptr) ? reinterpret_cast<T*>(a.gathered) : nullptr;
  uint2 wv[kNormQuads], rv[kNormQuads], xv[kNormQuads];
  // The norm weight is never written: loaded before the dependency wait.
#pragma unroll
  for (int j = 0; j < kNormQuads; ++j) {
    const int q = tid + j * nthreads;
    if (q < quads) wv[j] = reinterpret_cast<const uint2*>(a.weight)[q0 + q];
  }
  grid_dependency_wait();
  // Every load of the CTA's columns is issued before any store.
#pragma unroll
  for (int j = 0; j < kNormQuads; ++j) {
    const int q = tid + j * nthreads;
    if (q < quads) rv[j] = reinterpret_cast<const uint2*>(res)[q0 + q];
  }
  if (a.partials != nullptr) {
    // The projection's k-split partials, summed in split order from 0 and rounded to the model dtype: the values the
    // GEMM's own reduction and store would have produced. The loads of every split of a quad go out before the sum.
    const float* __restrict__ pp = a.partials + size_t(r) * a.hidden;
#pragma unroll
    for (int j = 0; j < kNormQuads; ++j) {
      const int q = tid + j * nthreads;
      xv[j] = make_uint2(0, 0);
      if (q >= quads) continue;
      float4 p[kMaxNormPartials];
#pragma unroll
      for (int sp = 0; sp < kMaxNormPartials; ++sp)
        if (sp < a.n_partials) p[sp] = reinterpret_cast<const float4*>(pp + size_t(sp) * a.partial_stride)[q0 + q];
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int sp = 0; sp < kMaxNormPartials; ++sp) {
        if (sp < a.n_partials) {
          acc[0] += p[sp].x;
          acc[1] += p[sp].y;
          acc[2] += p[sp].z;
          acc[3] += p[sp].w;
        }
      }
      T* xo = reinterpret_cast<T*>(&xv[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) xo[e] = from_f32<T>(acc[e]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kNormQuads; ++j) {
      const int q = tid + j * nthreads;
      if (q < quads) xv[j] = reinterpret_cast<const uint2*>(x)[q0 + q];
    }
  }
  if (a.corr != nullptr && r >= a.corr_from) {
    // a gated-LoRA adapter's output on this row, added to the projection's rounded output and rounded again
    const float* __restrict__ cr = a.corr + size_t(r - a.corr_from) * a.corr_ld;
#pragma unroll
    for (int j = 0; j < kNormQuads; ++j) {
      const int q = tid + j * nthreads;
      if (q >= quads) continue;
      const float4 add = reinterpret_cast<const float4*>(cr)[q0 + q];
      const float av[4] = {add.x, add.y, add.z, add.w};
      T* xo = reinterpret_cast<T*>(&xv[j]);
#pragma unroll
      for (int e = 0; e < 4; ++e) xo[e] = from_f32<T>(to_f32<T>(xo[e]) + av[e]);
    }
  }
  float v[kNormQuads][4];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kNormQuads; ++j) {
    const int q = tid + j * nthreads;
    if (q >= quads) continue;
    const T* x4 = reinterpret_cast<const T*>(&xv[j]);
    const T* r4 = reinterpret_cast<const T*>(&rv[j]);
    uint2 o;
    T* o4 = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[j][e] = to_f32<T>(x4[e]) + to_f32<T>(r4[e]);
      o4[e] = from_f32<T>(v[j][e]);
      ss += v[j][e] * v[j][e];
    }
    reinterpret_cast<uint2*>(res)[q0 + q] = o;
  }
  // CTA sum (lanes by butterfly, warps in order), pushed into slot `rank` of every CTA of the cluster; after the
  // cluster barrier each CTA adds the CS sums in rank order.
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  cluster_wait();
  if (tid < CS) {
    float t = 0.f;
    for (int w = 0; w < (nthreads + 31) / 32; ++w) t += red[w];
    st_dsmem_f32(cluster_map(&row_ss[rank], uint32_t(tid)), t);
  }
  cluster_sync();
  float total = 0.f;
#pragma unroll
  for (int c = 0; c < CS; ++c) total += row_ss[c];
  // The next kernel (the qkv projection's clusters) is let in only now: launched at this kernel's start, its
  // clusters were placed while the layer block still held most SMs, and one launch in three ran half again as long.
  allow_dependents();
  const float rstd = rsqrtf(total / float(a.hidden) + a.eps);
  uint8_t* tiles = static_cast<uint8_t*>(a.row_tiles);
#pragma unroll
  for (int j = 0; j < kNormQuads; ++j) {
    const int q = tid + j * nthreads;
    if (q >= quads) continue;
    const T* w4 = reinterpret_cast<const T*>(&wv[j]);
    uint2 o;
    T* o4 = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int e = 0; e < 4; ++e) o4[e] = from_f32<T>(round_to<T>(v[j][e] * rstd) * to_f32<T>(w4[e]));
    const int g = q0 + q;  // quad of the row: elements [4 g, 4 g + 4), half (g & 1) of 8-element chunk g / 2
    reinterpret_cast<uint2*>(nrm)[g] = o;
    if (gathered != nullptr) reinterpret_cast<uint2*>(gathered)[g] = o;
    if (tiles != nullptr) {
      const int c = g >> 1;
      *reinterpret_cast<uint2*>(tiles + row_tile_chunk(c >> 3, r, c & 7, a.tile_rows) * 16 + (g & 1) * 8) = o;
    }
  }
}

// Scatter K and V rows [rows][kv_heads][head_dim] to logical KV indices offset + r through the block table
// (the write vLLM's reshape_and_cache_flash performs at plm/decoder.py:347's slots). One warp per (row, kv head),
// 16-byte stores.
template <typename T>
__global__ void kv_append_kernel(const KvAppendArgs a) {
  grid_dependency_wait();
  allow_dependents();
  const int warp_global = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp_global >= a.rows * a.num_kv_heads) return;
  const int r = warp_global / a.num_kv_heads, g = warp_global % a.num_kv_heads;
  const int64_t logical = *a.offset + r;
  const int64_t lp = logical / a.page_size;
  const int page = (logical >= 0 && lp < a.max_pages) ? a.block_table[lp] : -1;
  if (page < 0 || page >= a.num_pages) {
    if (lane == 0) record_error(a.err, kErrBadIndex);
    return;
  }
  const size_t dst = ((size_t(page) * a.num_kv_heads + g) * a.page_size + size_t(logical % a.page_size)) * a.head_dim;
  const size_t src = (size_t(r) * a.num_kv_heads + g) * a.head_dim;
  const int vecs = a.head_dim / 8;  // 16-byte vectors of 8 elements
  for (int c = lane; c < vecs; c += 32) {
    reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.k_cache) + dst)[c] =
        reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.k) + src)[c];
    reinterpret_cast<uint4*>(reinterpret_cast<T*>(a.v_cache) + dst)[c] =
        reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(a.v) + src)[c];
  }
}

}  // namespace

int prologue_launch(const PrologueArgs& a, int rows, cudaStream_t stream, bool pdl) {
  if (a.hidden > kRowThreads * kVec * kMaxVecs || a.hidden % kVec != 0)
    return fail(PLM_ERR_UNSUPPORTED, "prologue: hidden %d (a multiple of 8, at most 4096)", a.hidden);
  if (a.dtype == PLM_F16)
    return check_cuda(launch(embed_norm_kernel<__half>, dim3(rows), dim3(kRowThreads), 0, stream, pdl, a),
                      "embed_norm_kernel");
  return check_cuda(launch(embed_norm_kernel<__nv_bfloat16>, dim3(rows), dim3(kRowThreads), 0, stream, pdl, a),
                    "embed_norm_kernel");
}

template <int CS>
int launch_add_norm(const AddNormArgs& a, int rows, cudaStream_t stream, bool pdl) {
  const int quads = a.hidden / (4 * CS);
  const int threads = min(kNormThreads, (quads + 31) / 32 * 32);
  auto kernel = a.dtype == PLM_F16 ? add_norm_kernel<__half, CS> : add_norm_kernel<__nv_bfloat16, CS>;
  return check_cuda(launch_cluster(kernel, dim3(rows * CS), dim3(threads), 0, stream, pdl, CS, 1, a),
                    "add_norm_kernel");
}

int add_norm_launch(const AddNormArgs& a, int rows, cudaStream_t stream, bool pdl) {
  if (a.hidden > kRowThreads * kVec * kMaxVecs || a.hidden % kVec != 0)
    return fail(PLM_ERR_UNSUPPORTED, "add_norm: hidden %d (a multiple of 8, at most 4096)", a.hidden);
  if (a.n_partials > kMaxNormPartials) return fail(PLM_ERR_UNSUPPORTED, "add_norm: %d partials", a.n_partials);
  return a.hidden % 16 == 0 ? launch_add_norm<4>(a, rows, stream, pdl) : launch_add_norm<2>(a, rows, stream, pdl);
}

int kv_append_launch(const KvAppendArgs& a, cudaStream_t stream, bool pdl) {
  if (a.head_dim % 8 != 0) return fail(PLM_ERR_UNSUPPORTED, "kv_append: head_dim %d", a.head_dim);
  const int warps = a.rows * a.num_kv_heads;
  const int blocks = (warps * 32 + 255) / 256;
  if (a.dtype == PLM_F16)
    return check_cuda(launch(kv_append_kernel<__half>, dim3(blocks), dim3(256), 0, stream, pdl, a),
                      "kv_append_kernel");
  return check_cuda(launch(kv_append_kernel<__nv_bfloat16>, dim3(blocks), dim3(256), 0, stream, pdl, a),
                    "kv_append_kernel");
}

}  // namespace plm

using namespace plm;

extern "C" int plm_kv_append(plm_ctx* ctx, const plm_kv_append_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_kv_append: null argument");
  if (d->dtype != PLM_BF16 && d->dtype != PLM_F16) return fail(PLM_ERR_INVALID, "plm_kv_append: dtype %d", d->dtype);
  if (!d->k || !d->v || !d->k_cache || !d->v_cache || !d->block_table || !d->offset || d->rows < 1)
    return fail(PLM_ERR_INVALID, "plm_kv_append: null operand or no rows");
  KvAppendArgs a = {d->dtype,     d->k,         d->v,         d->k_cache,  d->v_cache,  d->block_table,
                    d->max_pages, d->num_pages, d->page_size, d->offset,   d->rows,     d->num_kv_heads,
                    d->head_dim,  ctx->err};
  return kv_append_launch(a, static_cast<cudaStream_t>(stream), true);
}

extern "C" int plm_add_rmsnorm(plm_ctx* ctx, const plm_add_rmsnorm_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_add_rmsnorm: null argument");
  if (d->dtype != PLM_BF16 && d->dtype != PLM_F16) return fail(PLM_ERR_INVALID, "plm_add_rmsnorm: dtype %d", d->dtype);
  if (!d->residual || !d->normed || !d->weight || d->rows < 1 || d->hidden < 1)
    return fail(PLM_ERR_INVALID, "plm_add_rmsnorm: null operand");
  if (d->partials == nullptr && d->x == nullptr) return fail(PLM_ERR_INVALID, "plm_add_rmsnorm: null operand");
  if (d->partials != nullptr &&
      (d->n_partials < 1 || d->n_partials > kMaxNormPartials || d->partial_stride < int64_t(d->rows) * d->hidden))
    return fail(PLM_ERR_INVALID, "plm_add_rmsnorm: %d partials with stride %lld", d->n_partials,
                (long long)d->partial_stride);
  if (d->corr != nullptr && (d->corr_from < 0 || d->corr_ld < d->hidden || d->corr_ld % 4 != 0 || d->hidden % 8 != 0))
    return fail(PLM_ERR_INVALID, "plm_add_rmsnorm: corrections from row %d with stride %d", d->corr_from,
                d->corr_ld);
  AddNormArgs a = {d->x,      d->residual,   d->normed,       d->weight,       d->hidden,
                   d->eps,    d->gather_row, d->gathered,     d->partials,     d->n_partials,
                   d->partial_stride};
  a.corr = d->corr;
  a.corr_from = d->corr_from;
  a.corr_ld = d->corr_ld;
  a.dtype = d->dtype;
  return add_norm_launch(a, d->rows, static_cast<cudaStream_t>(stream), true);
}
