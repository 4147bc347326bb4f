// Paged attention of the round's query rows under the round mask (replaces FlexAttention with the block mask of
// plm/mask.py:23-29 as vLLM's backend calls it: vllm/v1/attention/backends/flex_attention.py:1070-1205).
//
// Grid (head, KV split, 64-row query tile), 4 warps; warp w owns query rows [16w, 16w + 16) of the tile.
// Keys are visited in tiles of 64: each tile's K and V rows are gathered page by page through the block table
// with 16-byte cp.async into XOR-swizzled shared memory (double buffered), S = Q K^T and O += P V run on tensor
// cores (mma.m16n8k16 bf16, fp32 accumulation; P is rounded to bf16 for the second product), and the softmax is
// online in base 2. The KV splits of one (head, query tile) form a thread-block cluster whose partial results are
// combined through distributed shared memory. Key kv is visible to row r (logical query offset + r) iff
//     kv < offset + rows  and  (kv < offset  or  kv - offset <= depth[r]
//                                 or  (kv - offset >= own_start[r]  and  kv <= offset + r)),
// which is RoundMaskView for a round (depth / own_start from round_layout) and plain causal attention for a
// prefill chunk (depth[r] = r).
#include <type_traits>

#include "attention.h"
#include "common.cuh"
#include "runtime.h"

namespace plm {
namespace {

constexpr int kKeysPerTile = 64;
constexpr int kAttnThreads = 128;
constexpr int kQRowsPerCta = 64;
constexpr int kStages = 3;           // K/V tiles in flight per CTA (two CTAs still share an SM)
constexpr int kMaxPageSlice = 1024;  // block-table entries staged per CTA (keys per CTA <= 1023 pages)
constexpr int kClusterMax = 8;      // KV splits of one cluster; a launch with merge buffers has two per head

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}
// m16n8k16 tensor-core product with fp32 accumulation, operands in the model dtype T (bf16 or f16).
template <typename T>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
// 2^x by the special-function unit (relative error ~2^-22; -inf gives +0): the softmax's exponentials.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Two floats rounded to the model dtype, packed low element first.
template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const T l = from_f32<T>(lo), h = from_f32<T>(hi);
  return uint32_t(*reinterpret_cast<const uint16_t*>(&l)) | (uint32_t(*reinterpret_cast<const uint16_t*>(&h)) << 16);
}

// Byte offset of (row, 16-byte chunk) in a swizzled tile with HD/8 chunks per row.
template <int HD>
__device__ __forceinline__ int swz(int row, int chunk) {
  return row * (HD * 2) + ((chunk ^ (row & 7)) << 4);
}

template <int HD, typename T>
__global__ void __launch_bounds__(kAttnThreads, 1) round_attention_kernel(const AttnArgs a) {
  constexpr int CH = HD / 8;
  constexpr int TILE_BYTES = kKeysPerTile * HD * 2;
  constexpr int NT = kKeysPerTile / 8;  // key n-tiles per tile
  constexpr int KS = HD / 16;           // k-steps over the head dim
  extern __shared__ __align__(128) uint8_t smem[];
  auto kbuf = [&](int slot) { return smem + (2 * slot) * TILE_BYTES; };  // ring slot: K tile, then V tile
  auto vbuf = [&](int slot) { return smem + (2 * slot + 1) * TILE_BYTES; };

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int head = blockIdx.x, split = blockIdx.y, qt = blockIdx.z;
  const int group = head / (a.num_heads / a.num_kv_heads);

  // Before the dependency wait: everything the previous kernel does not write. The offset comes from an earlier
  // kernel (the last round's commit, or a copy before a prefill), the block table and the layout are static, and
  // the context keys [0, offset) were written by earlier rounds; only the query rows and the round's own K/V come
  // from the QKV projection this kernel follows.
  const int64_t offset = *a.offset;
  const int64_t seq_len = offset + a.rows;
  const int n_tiles = int((seq_len + kKeysPerTile - 1) / kKeysPerTile);
  // With two clusters per head (a.part set) the second one works only when every one of the 16 splits keeps at least
  // four tiles; otherwise its CTAs leave at once and the first cluster's 8 splits cover all keys and combine
  // through distributed shared memory.
  const int S = a.part != nullptr && 4 * a.splits > n_tiles ? kClusterMax : a.splits;
  if (split >= S) return;
  // Tiles spread evenly over the splits, the larger shares first: the last split holds the masked tiles of the
  // round's own keys, so it gets the smaller share.
  const int t0 = n_tiles - int(int64_t(S - split) * n_tiles / S);
  const int t1 = n_tiles - int(int64_t(S - split - 1) * n_tiles / S);
  const int n_local = t1 - t0;
  int* pages = reinterpret_cast<int*>(smem + 2 * kStages * TILE_BYTES);
  const int64_t lp0 = (int64_t(t0) * kKeysPerTile) >> a.page_shift;
  const int n_pages = n_local > 0 ? int(((int64_t(t1) * kKeysPerTile - 1) >> a.page_shift) - lp0 + 1) : 0;
  const bool staged_pages = n_pages <= kMaxPageSlice;
  for (int i = tid; i < (staged_pages ? n_pages : 0); i += kAttnThreads) {
    const int64_t lp = lp0 + i;
    pages[i] = lp < a.max_pages ? a.block_table[lp] : -1;
  }
  const int r0 = qt * kQRowsPerCta + warp * 16 + gq, r1 = r0 + 8;
  const int dep0 = r0 < a.rows ? a.depth[r0] : -1, own0 = r0 < a.rows ? a.own_start[r0] : (1 << 30);
  const int dep1 = r1 < a.rows ? a.depth[r1] : -1, own1 = r1 < a.rows ? a.own_start[r1] : (1 << 30);
  __syncthreads();

  const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(a.k_cache);
  const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(a.v_cache);
  // Thread tid always copies 16-byte chunk tid % CH of tile rows tid / CH + u * RSTEP: its page lookups are issued
  // together, then 32-bit-cheap address arithmetic from per-thread constants; a bad page is recorded once per tile.
  constexpr int ITER = (kKeysPerTile * CH) / kAttnThreads;
  constexpr int RSTEP = kAttnThreads / CH;
  const int my_chunk = tid % CH, my_row0 = tid / CH;
  const size_t head_off = size_t(group) * a.page_size * HD + size_t(my_chunk) * 8;  // elements
  const size_t page_stride = size_t(a.num_kv_heads) * a.page_size * HD;            // elements per page
  // The forward's own keys (logical index >= offset) come from the round scratch when the rows are a round's
  // candidates (scratch_k set): row kv - offset, kv heads contiguous.
  const __nv_bfloat16* sk = reinterpret_cast<const __nv_bfloat16*>(a.scratch_k);
  const __nv_bfloat16* sv = reinterpret_cast<const __nv_bfloat16*>(a.scratch_v);
  const size_t scratch_off = size_t(group) * HD + size_t(my_chunk) * 8;
  // Tile t (absolute) into ring slot buf; one commit group per call. A tile wholly inside the context takes the
  // branch-free path (every key through the block table); only the tiles holding the forward's own keys test each
  // key against the offset.
  auto issue = [&](int t, int buf) {
    const int64_t kv0 = int64_t(t) * kKeysPerTile + my_row0;
    const bool context_tile = sk == nullptr || int64_t(t + 1) * kKeysPerTile <= offset;
    int pg[ITER];
#pragma unroll
    for (int u = 0; u < ITER; ++u) {
      const int64_t kv = kv0 + u * RSTEP;
      const int64_t lp = kv >> a.page_shift;
      pg[u] = kv >= seq_len ? -2 : staged_pages ? pages[lp - lp0] : (lp < a.max_pages ? a.block_table[lp] : -1);
    }
    bool bad = false;
    if (context_tile) {
#pragma unroll
      for (int u = 0; u < ITER; ++u) {
        const int row = my_row0 + u * RSTEP;
        const bool valid = pg[u] >= 0 && pg[u] < a.num_pages;
        bad |= pg[u] != -2 && !valid;
        const size_t src =
            valid ? size_t(pg[u]) * page_stride + head_off + size_t((kv0 + u * RSTEP) & (a.page_size - 1)) * HD : 0;
        cp_async_16(kbuf(buf) + swz<HD>(row, my_chunk), kc + src, valid);
        cp_async_16(vbuf(buf) + swz<HD>(row, my_chunk), vc + src, valid);
      }
    } else {
#pragma unroll
      for (int u = 0; u < ITER; ++u) {
        const int row = my_row0 + u * RSTEP;
        const int64_t kv = kv0 + u * RSTEP;
        const bool own = kv >= offset && kv < seq_len;
        const bool valid = own || (pg[u] >= 0 && pg[u] < a.num_pages);
        bad |= !own && pg[u] != -2 && !valid;
        const __nv_bfloat16* ks =
            own ? sk + size_t(kv - offset) * size_t(a.num_kv_heads) * HD + scratch_off
                : kc + (valid ? size_t(pg[u]) * page_stride + head_off + size_t(kv & (a.page_size - 1)) * HD : 0);
        const __nv_bfloat16* vs =
            own ? sv + size_t(kv - offset) * size_t(a.num_kv_heads) * HD + scratch_off
                : vc + (valid ? size_t(pg[u]) * page_stride + head_off + size_t(kv & (a.page_size - 1)) * HD : 0);
        cp_async_16(kbuf(buf) + swz<HD>(row, my_chunk), ks, valid);
        cp_async_16(vbuf(buf) + swz<HD>(row, my_chunk), vs, valid);
      }
    }
    if (bad) record_error(a.err, kErrBadIndex);
  };
  // Pipeline prologue: kStages - 1 commit groups. Tiles lying wholly in the context go out before the wait.
  int64_t whole = offset / kKeysPerTile - t0;  // tiles of this CTA whose last key lies below offset
  whole = whole < 0 ? 0 : (whole > n_local ? n_local : whole);
  const int ctx_tiles = int(whole);
  int issued = 0;
  for (; issued < kStages - 1 && issued < ctx_tiles; ++issued) {
    issue(t0 + issued, issued);
    cp_async_commit();
  }

  grid_dependency_wait();
  allow_dependents();

  for (; issued < kStages - 1; ++issued) {
    if (issued < n_local) issue(t0 + issued, issued);
    cp_async_commit();
  }

  // ---- query fragments (A operand, rows r0 and r0 + 8 of this warp) ----
  const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q);
  const size_t q_stride = size_t(a.num_heads) * HD;
  uint32_t qf[KS][4];
#pragma unroll
  for (int kk = 0; kk < KS; ++kk) {
    const int col = kk * 16 + 2 * tq;
    auto ld = [&](int rr, int c) -> uint32_t {
      if (rr >= a.rows) return 0u;
      return *reinterpret_cast<const uint32_t*>(q + size_t(rr) * q_stride + size_t(head) * HD + c);
    };
    qf[kk][0] = ld(r0, col);
    qf[kk][1] = ld(r1, col);
    qf[kk][2] = ld(r0, col + 8);
    qf[kk][3] = ld(r1, col + 8);
  }

  float o[HD / 8][4];
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float scale = a.scale_log2;

  for (int i = 0; i < n_local; ++i) {
    const int t = t0 + i, buf = i % kStages;
    cp_async_wait<kStages - 2>();  // tile i has landed (one group is committed per tile, empty ones included)
    __syncthreads();               // ... for every thread, and slot (i - 1) % kStages is free again
    if (i + kStages - 1 < n_local) issue(t + kStages - 1, (i + kStages - 1) % kStages);
    cp_async_commit();
    const uint8_t* kb = kbuf(buf);
    const uint8_t* vb = vbuf(buf);

    float s[NT][4];
#pragma unroll
    for (int j = 0; j < NT; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < KS; ++kk) {
#pragma unroll
      for (int jj = 0; jj < NT / 2; ++jj) {
        const int mi = lane >> 3, rr = lane & 7;
        const int row = jj * 16 + (mi >> 1) * 8 + rr;
        const int chunk = kk * 2 + (mi & 1);
        uint32_t b[4];
        ldmatrix_x4(b, kb + swz<HD>(row, chunk));
        mma_16816<T>(s[2 * jj], qf[kk], b[0], b[1]);
        mma_16816<T>(s[2 * jj + 1], qf[kk], b[2], b[3]);
      }
    }
    // Mask the tiles that reach the forward's own keys. Key kbase + c relative to the offset, in 32 bits: visible
    // iff rel < rows and (a context key, or within the row's depth, or inside its own block up to its own
    // position). Bitwise operators, so no branch per key.
    const int64_t kbase = int64_t(t) * kKeysPerTile;
    if (kbase + kKeysPerTile > offset) {
      const int rel_base = int(kbase - offset) + 2 * tq;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int rel = rel_base + j * 8 + (e & 1);
          const int rr = e < 2 ? r0 : r1;
          const int dep = e < 2 ? dep0 : dep1, own = e < 2 ? own0 : own1;
          const bool vis = (rel < a.rows) & ((rel < 0) | (rel <= dep) | ((rel >= own) & (rel <= rr)));
          s[j][e] = vis ? s[j][e] : -INFINITY;
        }
      }
    }
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
    // Maxima are kept in raw score units and each exponent is ex2(s * scale - m * scale), one FMA. A row with no
    // visible key yet keeps m = -inf: its exponents come out 0 and its correction 1.
    const float ns0 = n0 == -INFINITY ? 0.f : n0 * scale, ns1 = n1 == -INFINITY ? 0.f : n1 * scale;
    const float c0 = n0 == -INFINITY ? 1.f : ex2(fmaf(m0, scale, -ns0));
    const float c1 = n1 == -INFINITY ? 1.f : ex2(fmaf(m1, scale, -ns1));
    m0 = n0;
    m1 = n1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int j = 0; j < NT; ++j) {
      s[j][0] = ex2(fmaf(s[j][0], scale, -ns0));
      s[j][1] = ex2(fmaf(s[j][1], scale, -ns0));
      s[j][2] = ex2(fmaf(s[j][2], scale, -ns1));
      s[j][3] = ex2(fmaf(s[j][3], scale, -ns1));
      ps0 += s[j][0] + s[j][1];
      ps1 += s[j][2] + s[j][3];
    }
    l0 = l0 * c0 + ps0;
    l1 = l1 * c1 + ps1;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      o[j][0] *= c0;
      o[j][1] *= c0;
      o[j][2] *= c1;
      o[j][3] *= c1;
    }
    // O += P V
#pragma unroll
    for (int kk = 0; kk < kKeysPerTile / 16; ++kk) {
      uint32_t pa[4];
      pa[0] = pack2<T>(s[2 * kk][0], s[2 * kk][1]);
      pa[1] = pack2<T>(s[2 * kk][2], s[2 * kk][3]);
      pa[2] = pack2<T>(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[3] = pack2<T>(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int nn = 0; nn < HD / 16; ++nn) {
        const int mi = lane >> 3, rr = lane & 7;
        const int row = kk * 16 + (mi & 1) * 8 + rr;
        const int chunk = nn * 2 + (mi >> 1);
        uint32_t b[4];
        ldmatrix_x4_trans(b, vb + swz<HD>(row, chunk));
        mma_16816<T>(o[2 * nn], pa, b[0], b[1]);
        mma_16816<T>(o[2 * nn + 1], pa, b[2], b[3]);
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is reused by the split combine below

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);

  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  const size_t out_stride = size_t(a.num_heads) * HD;
  // Element (row, col) of the output: row-major, or inside the row tiles (the 16-byte chunk of its k-block, then
  // the position within the chunk; writers store at most one chunk's worth at a time).
  uint8_t* tiles = static_cast<uint8_t*>(a.row_tiles);
  auto out_at = [&](int row, int col) -> __nv_bfloat16* {
    if (tiles != nullptr)
      return reinterpret_cast<__nv_bfloat16*>(tiles + row_tile_chunk(col >> 6, row, (col >> 3) & 7, a.tile_rows) * 16) +
             (col & 7);
    return out + size_t(row) * out_stride + col;
  };
  if (a.splits == 1) {
    const float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      const int col = head * HD + j * 8 + 2 * tq;
      if (r0 < a.rows)
        *reinterpret_cast<uint32_t*>(out_at(r0, col)) = pack2<T>(o[j][0] * inv0, o[j][1] * inv0);
      if (r1 < a.rows)
        *reinterpret_cast<uint32_t*>(out_at(r1, col)) = pack2<T>(o[j][2] * inv1, o[j][3] * inv1);
    }
    return;
  }

  if (S > kClusterMax) {
    // ---- both clusters of the head active: split partials combined through global memory ----
    // Each CTA stores its unnormalised partial (O, then (m, l) per row), signals a per-(head, query tile) counter and
    // waits until all S splits have stored theirs (the host enables this only when every cluster of the launch is
    // resident at once); split s then combines rows [s * 64 / S, (s + 1) * 64 / S) over the splits in split order,
    // loading every split's (m, l) and 16 bytes of O together, and the last CTA done reading resets the counters.
    constexpr int PSTRIDE = kQRowsPerCta * (HD + 2);
    float* const head_part = a.part + size_t(head * int(gridDim.z) + qt) * S * PSTRIDE;
    float* const mine = head_part + size_t(split) * PSTRIDE;
    const int lr0 = warp * 16 + gq, lr1 = lr0 + 8;
#pragma unroll
    for (int j = 0; j < HD / 8; ++j) {
      const int col = j * 8 + 2 * tq;
      __stcg(reinterpret_cast<float2*>(mine + lr0 * HD + col), make_float2(o[j][0], o[j][1]));
      __stcg(reinterpret_cast<float2*>(mine + lr1 * HD + col), make_float2(o[j][2], o[j][3]));
    }
    if (tq == 0) {  // maxima in log2 units
      __stcg(reinterpret_cast<float2*>(mine + kQRowsPerCta * HD + lr0 * 2), make_float2(m0 * scale, l0));
      __stcg(reinterpret_cast<float2*>(mine + kQRowsPerCta * HD + lr1 * 2), make_float2(m1 * scale, l1));
    }
    __syncthreads();
    int* const ctr = a.arrive + 2 * (head * int(gridDim.z) + qt);
    int* const flag = reinterpret_cast<int*>(smem);
    if (tid == 0) {
      signal_stored(ctr);
      int ok = 1;
      if (ld_acquire_gpu(ctr) < S) {
        const uint64_t start = global_timer_ns();
        while (ld_acquire_gpu(ctr) < S) {
          if (global_timer_ns() - start > kWaitLimitNs) {
            record_error(a.err, kErrTimeoutFlag);
            ok = 0;
            break;
          }
        }
      }
      *flag = ok;
    }
    __syncthreads();
    if (*flag != 0) {
      const int rpc = kQRowsPerCta / S;
      const int row_begin = split * rpc;
      constexpr int Q4 = HD / 4;
      const int live = max(0, min(rpc, a.rows - (qt * kQRowsPerCta + row_begin)));
      for (int idx = tid; idx < live * Q4; idx += kAttnThreads) {
        const int lr = idx / Q4, c = (idx % Q4) * 4;
        const float* ml = head_part + kQRowsPerCta * HD + (row_begin + lr) * 2;
        const float* src = head_part + (row_begin + lr) * HD + c;
        float2 mls[2 * kClusterMax];
        float4 v[2 * kClusterMax];
#pragma unroll
        for (int sp = 0; sp < 2 * kClusterMax; ++sp) {
          mls[sp] = __ldcg(reinterpret_cast<const float2*>(ml + size_t(sp) * PSTRIDE));
          v[sp] = __ldcg(reinterpret_cast<const float4*>(src + size_t(sp) * PSTRIDE));
        }
        float mmax = -INFINITY;
#pragma unroll
        for (int sp = 0; sp < 2 * kClusterMax; ++sp) mmax = fmaxf(mmax, mls[sp].x);
        float lsum = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int sp = 0; sp < 2 * kClusterMax; ++sp) {
          const float w = mls[sp].x != -INFINITY ? exp2f(mls[sp].x - mmax) : 0.f;
          lsum += w * mls[sp].y;
          acc.x += w * v[sp].x;
          acc.y += w * v[sp].y;
          acc.z += w * v[sp].z;
          acc.w += w * v[sp].w;
        }
        const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
        uint32_t* dst = reinterpret_cast<uint32_t*>(out_at(qt * kQRowsPerCta + row_begin + lr, head * HD + c));
        dst[0] = pack2<T>(acc.x * inv, acc.y * inv);
        dst[1] = pack2<T>(acc.z * inv, acc.w * inv);
      }
    }
    __syncthreads();
    if (tid == 0 && atomicAdd(ctr + 1, 1) == S - 1) {
      ctr[0] = 0;
      ctr[1] = 0;
    }
    return;
  }

  // ---- split partials, combined over the cluster of the (head, query tile) ----
  // Each CTA leaves its unnormalised partial (O, m, l) in its own shared memory (the K/V buffers are free now);
  // after a cluster barrier rank r combines rows [r * 64 / S, (r + 1) * 64 / S) over all ranks in rank order through
  // distributed shared memory; a second barrier keeps every partial alive until all rows are combined.
  float* po = reinterpret_cast<float*>(smem);                              // [64][HD]
  float* pml = reinterpret_cast<float*>(smem + kQRowsPerCta * HD * 4);     // [64][2]
  float* wts = pml + kQRowsPerCta * 2;                                     // [64 / S rows][S] weights, then 1/L
  const int lr0 = warp * 16 + gq, lr1 = lr0 + 8;
#pragma unroll
  for (int j = 0; j < HD / 8; ++j) {
    const int col = j * 8 + 2 * tq;
    *reinterpret_cast<float2*>(po + lr0 * HD + col) = make_float2(o[j][0], o[j][1]);
    *reinterpret_cast<float2*>(po + lr1 * HD + col) = make_float2(o[j][2], o[j][3]);
  }
  if (tq == 0) {  // the combine works with maxima in log2 units
    *reinterpret_cast<float2*>(pml + lr0 * 2) = make_float2(m0 * scale, l0);
    *reinterpret_cast<float2*>(pml + lr1 * 2) = make_float2(m1 * scale, l1);
  }
  cluster_sync();
  const uint32_t rank = cluster_rank();
  const int rpc = (kQRowsPerCta + S - 1) / S;  // rows per rank; the last rank's share ends at the tile's edge
  const int row_begin = int(rank) * rpc;
  const int own_rows = max(0, min(rpc, kQRowsPerCta - row_begin));
  if (tid < own_rows) {
    const int row = row_begin + tid;
    float ms[kClusterMax], ls[kClusterMax], mmax = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < kClusterMax; ++sp) {
      ms[sp] = -INFINITY;
      ls[sp] = 0.f;
      if (sp < S) {
        const float2 ml = ld_dsmem_f32x2(cluster_map(pml + row * 2, uint32_t(sp)));
        ms[sp] = ml.x;
        ls[sp] = ml.y;
        mmax = fmaxf(mmax, ml.x);
      }
    }
    float lsum = 0.f;
#pragma unroll
    for (int sp = 0; sp < kClusterMax; ++sp) {
      const float w = (sp < S && ms[sp] != -INFINITY) ? exp2f(ms[sp] - mmax) : 0.f;
      if (sp < S) wts[tid * (S + 1) + sp] = w;
      lsum += w * ls[sp];
    }
    wts[tid * (S + 1) + S] = lsum > 0.f ? 1.f / lsum : 0.f;
  }
  __syncthreads();
  // 16-byte remote loads, two of the thread's row chunks x every rank in flight at a time; rows past a.rows are
  // skipped
  constexpr int Q4 = HD / 4;  // float4 per row
  const int live = max(0, min(own_rows, a.rows - (qt * kQRowsPerCta + row_begin)));
  for (int idx0 = tid; idx0 < live * Q4; idx0 += 2 * kAttnThreads) {
    float4 part[2][kClusterMax];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int idx = idx0 + u * kAttnThreads;
      const int lr = idx / Q4, c = (idx % Q4) * 4;
      const uint32_t off = uint32_t((row_begin + lr) * HD + c) * 4u;
#pragma unroll
      for (int sp = 0; sp < kClusterMax; ++sp)
        part[u][sp] = (sp < S && idx < live * Q4) ? ld_dsmem_f32x4(cluster_map(po, uint32_t(sp)) + off)
                                                   : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int idx = idx0 + u * kAttnThreads;
      if (idx >= live * Q4) continue;
      const int lr = idx / Q4, c = (idx % Q4) * 4;
      float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int sp = 0; sp < kClusterMax; ++sp) {
        if (sp < S) {
          const float w = wts[lr * (S + 1) + sp];
          acc.x += w * part[u][sp].x;
          acc.y += w * part[u][sp].y;
          acc.z += w * part[u][sp].z;
          acc.w += w * part[u][sp].w;
        }
      }
      const int grow = qt * kQRowsPerCta + row_begin + lr;
      const float inv = wts[lr * (S + 1) + S];
      uint32_t* dst = reinterpret_cast<uint32_t*>(out_at(grow, head * HD + c));
      dst[0] = pack2<T>(acc.x * inv, acc.y * inv);
      dst[1] = pack2<T>(acc.z * inv, acc.w * inv);
    }
  }
  cluster_sync();
}

template <int HD, typename T>
int launch_attention(const AttnArgs& a, int q_tiles, cudaStream_t stream, bool pdl) {
  constexpr int SMEM = 2 * kStages * kKeysPerTile * HD * 2 + kMaxPageSlice * 4;
  auto kernel = round_attention_kernel<HD, T>;
  const int st = raise_smem_limit(reinterpret_cast<const void*>(kernel), SMEM, "cudaFuncSetAttribute(attention smem)");
  if (st != PLM_OK) return st;
  // Two clusters per head take the load-balancing placement: spread over distinct SMs, some of the 32 clusters
  // started well after the others while the previous kernel still held SMs. One cluster per head stays spread.
  return check_cuda(launch_cluster_pref(kernel, dim3(a.num_heads, a.splits, q_tiles), dim3(kAttnThreads), SMEM, stream,
                                        pdl, 1, a.splits < kClusterMax ? a.splits : kClusterMax, a.part != nullptr, a),
                    "round_attention_kernel");
}

}  // namespace

int attention_splits(int num_heads, int q_tiles, int num_sms, int64_t max_keys, bool global_combine) {
  const int ctas = num_heads * q_tiles;
  const int max_tiles = int((max_keys + kKeysPerTile - 1) / kKeysPerTile);
  int splits = 1;
  while (splits < 8 && ctas * splits < 2 * num_sms && 2 * splits <= max_tiles) splits *= 2;
  if (global_combine && splits == 8 && ctas * 16 <= 2 * num_sms && 4 * 16 <= max_tiles) splits = 16;
  return splits;
}

namespace {
template <int HD, typename T>
bool two_clusters_fit(int num_heads, int q_tiles) {
  constexpr int SMEM = 2 * kStages * kKeysPerTile * HD * 2 + kMaxPageSlice * 4;
  auto kernel = round_attention_kernel<HD, T>;
  if (raise_smem_limit(reinterpret_cast<const void*>(kernel), SMEM, "cudaFuncSetAttribute(attention smem)") != PLM_OK)
    return false;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_heads, 2 * kClusterMax, q_tiles);
  cfg.blockDim = dim3(kAttnThreads);
  cfg.dynamicSmemBytes = SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = kClusterMax;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return clusters >= num_heads * q_tiles * 2;
}
}  // namespace

bool attention_two_clusters_fit(int num_heads, int q_tiles, int head_dim, int dtype) {
  if (head_dim == 128)
    return dtype == PLM_F16 ? two_clusters_fit<128, __half>(num_heads, q_tiles)
                            : two_clusters_fit<128, __nv_bfloat16>(num_heads, q_tiles);
  if (head_dim == 64)
    return dtype == PLM_F16 ? two_clusters_fit<64, __half>(num_heads, q_tiles)
                            : two_clusters_fit<64, __nv_bfloat16>(num_heads, q_tiles);
  return false;
}

size_t attention_part_floats(int num_heads, int q_tiles, int head_dim) {
  return size_t(num_heads) * q_tiles * 2 * kClusterMax * kQRowsPerCta * (head_dim + 2);
}

size_t attention_arrive_ints(int num_heads, int q_tiles) { return size_t(num_heads) * q_tiles * 2; }

int attention_launch(plm_ctx* ctx, AttnArgs a, cudaStream_t stream, bool pdl) {
  if (a.head_dim != 64 && a.head_dim != 128) return fail(PLM_ERR_UNSUPPORTED, "attention: head_dim %d", a.head_dim);
  if (a.num_kv_heads <= 0 || a.num_heads % a.num_kv_heads != 0)
    return fail(PLM_ERR_INVALID, "attention: %d heads over %d kv heads", a.num_heads, a.num_kv_heads);
  if (a.rows < 1 || a.rows > 1024) return fail(PLM_ERR_INVALID, "attention: rows %d", a.rows);
  if (a.page_size < 1 || a.page_size > 4096 || (a.page_size & (a.page_size - 1)) != 0)
    return fail(PLM_ERR_UNSUPPORTED, "attention: page size %d (a power of two <= 4096)", a.page_size);
  a.page_shift = __builtin_ctz(unsigned(a.page_size));
  if (!a.q || !a.k_cache || !a.v_cache || !a.block_table || !a.offset || !a.depth || !a.own_start ||
      (!a.out && !a.row_tiles) || (a.row_tiles && (a.tile_rows < a.rows || a.tile_rows % 16 != 0)))
    return fail(PLM_ERR_INVALID, "attention: null operand");
  const int q_tiles = (a.rows + kQRowsPerCta - 1) / kQRowsPerCta;
  if (a.splits < 1) a.splits = 1;
  if (a.part != nullptr ? a.splits != 2 * kClusterMax || a.arrive == nullptr : a.splits > kClusterMax)
    return fail(PLM_ERR_UNSUPPORTED, "attention: %d splits (at most %d, or %d with merge buffers)", a.splits,
                kClusterMax, 2 * kClusterMax);
  a.err = ctx->err;
  if (a.dtype == PLM_F16)
    return a.head_dim == 128 ? launch_attention<128, __half>(a, q_tiles, stream, pdl)
                             : launch_attention<64, __half>(a, q_tiles, stream, pdl);
  return a.head_dim == 128 ? launch_attention<128, __nv_bfloat16>(a, q_tiles, stream, pdl)
                           : launch_attention<64, __nv_bfloat16>(a, q_tiles, stream, pdl);
}

}  // namespace plm

using namespace plm;

extern "C" int plm_attention(plm_ctx* ctx, const plm_attention_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_attention: null argument");
  if (d->dtype != PLM_BF16 && d->dtype != PLM_F16) return fail(PLM_ERR_INVALID, "plm_attention: dtype %d", d->dtype);
  AttnArgs a = {};
  a.dtype = d->dtype;
  a.q = d->q;
  a.k_cache = d->k_cache;
  a.v_cache = d->v_cache;
  a.block_table = d->block_table;
  a.max_pages = d->max_pages;
  a.num_pages = d->num_pages;
  a.page_size = d->page_size;
  a.offset = d->offset;
  a.rows = d->rows;
  a.depth = d->depth;
  a.own_start = d->own_start;
  a.num_heads = d->num_heads;
  a.num_kv_heads = d->num_kv_heads;
  a.head_dim = d->head_dim;
  a.scale_log2 = float(1.4426950408889634 / sqrt(double(d->head_dim)));
  a.out = d->out;
  const int q_tiles = (d->rows + kQRowsPerCta - 1) / kQRowsPerCta;
  a.splits = d->splits > 0 ? d->splits : attention_splits(d->num_heads, q_tiles, ctx->num_sms, d->max_keys);
  if (a.splits == 2 * kClusterMax) {  // two clusters per head: the context's merge buffers, grown to this shape
    if (!attention_two_clusters_fit(d->num_heads, q_tiles, d->head_dim, d->dtype))
      return fail(PLM_ERR_UNSUPPORTED, "plm_attention: 16 splits need every cluster resident at once");
    const size_t nf = attention_part_floats(d->num_heads, q_tiles, d->head_dim);
    const size_t na = attention_arrive_ints(d->num_heads, q_tiles);
    if (ctx->attn_part_floats < nf || ctx->attn_arrive_ints < na) {
      int st = check_cuda(cudaDeviceSynchronize(), "plm_attention: synchronize before growing the merge buffers");
      if (st != PLM_OK) return st;
      cudaFree(ctx->attn_part);
      cudaFree(ctx->attn_arrive);
      ctx->attn_part = nullptr;
      ctx->attn_arrive = nullptr;
      ctx->attn_part_floats = ctx->attn_arrive_ints = 0;
      st = check_cuda(cudaMalloc(&ctx->attn_part, nf * sizeof(float)), "plm_attention: merge buffers");
      if (st == PLM_OK) st = check_cuda(cudaMalloc(&ctx->attn_arrive, na * sizeof(int)), "plm_attention: counters");
      if (st == PLM_OK) st = check_cuda(cudaMemset(ctx->attn_arrive, 0, na * sizeof(int)), "plm_attention: counters");
      if (st != PLM_OK) return st;
      ctx->attn_part_floats = nf;
      ctx->attn_arrive_ints = na;
    }
    a.part = ctx->attn_part;
    a.arrive = ctx->attn_arrive;
  }
  return attention_launch(ctx, a, static_cast<cudaStream_t>(stream), true);
}
