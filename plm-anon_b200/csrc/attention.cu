// Paged attention of the round's query rows under the round mask (replaces FlexAttention with the block mask of
// plm/mask.py:23-29 as vLLM's backend calls it: vllm/v1/attention/backends/flex_attention.py:1070-1205).
//
// Grid (head, KV split, 128-row query tile), 4 warps; thread t owns query row t of the tile, which is TMEM lane t.
// A CTA walks its keys in chunks of up to 128 (two 64-key tiles):
//   - every thread gathers 16-byte pieces of the chunk's K and V rows through the block table with cp.async into
//     shared memory, in the 128-byte-swizzled layout the tensor cores read (a double-buffered ring);
//   - one thread issues S = Q K^T (tcgen05.mma, M = 128 query rows, N = the chunk's keys, K = head_dim) into TMEM;
//   - each thread loads its row of S from TMEM, applies the scale and the mask, and forms the online softmax in
//     base 2: P = 2^(S - m) rounded to bf16 is written to shared memory, the running sum l in fp32; when the row
//     maximum grows, the row of O in TMEM is rescaled first;
//   - one thread issues O += P V (tcgen05.mma, N = head_dim, K = the chunk's keys; V is read MN-major) into TMEM.
// The KV splits of one (head, query tile) form a thread-block cluster whose unnormalised partials (O, m, l) are
// combined through distributed shared memory. Key kv is visible to row r (logical query offset + r) iff
//     kv < offset + rows  and  (kv < offset  or  kv - offset <= depth[r]
//                                 or  (kv - offset >= own_start[r]  and  kv <= offset + r)),
// which is RoundMaskView for a round (depth / own_start from round_layout) and plain causal attention for a
// prefill chunk (depth[r] = r).
#include "attention.h"
#include "common.cuh"
#include "runtime.h"

namespace plm {
namespace {

constexpr int kKeysPerTile = 64;
constexpr int kTilesPerChunk = 2;
constexpr int kChunkKeys = kKeysPerTile * kTilesPerChunk;
constexpr int kAttnThreads = 128;
constexpr int kQRowsPerCta = 128;
constexpr int kMaxPageSlice = 1024;  // block-table entries staged per CTA (keys per CTA <= 1023 pages)
constexpr uint32_t kAttnTmemCols = 256;  // S: columns [0, 128); O: columns [128, 128 + head_dim)
constexpr uint32_t kTmemO = 128;

// 2^x by the special-function unit (relative error ~2^-22; -inf gives +0): the softmax's exponentials.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

template <int HD>
struct AttnSmem {
  static constexpr int KB = HD / 64;                    // 64-element k-blocks of a head row
  static constexpr int Q_BYTES = KB * kQRowsPerCta * 128;
  static constexpr int KV_BLOCK = kChunkKeys * 128;     // one k-block of a chunk's K (or V) rows
  static constexpr int K_BYTES = KB * KV_BLOCK;
  static constexpr int BUF_BYTES = 2 * K_BYTES;         // K then V
  static constexpr int P_BYTES = kTilesPerChunk * kQRowsPerCta * 128;
  static constexpr int Q_OFF = 0;
  static constexpr int RING_OFF = Q_OFF + Q_BYTES;
  static constexpr int P_OFF = RING_OFF + 2 * BUF_BYTES;
  static constexpr int PAGES_OFF = P_OFF + P_BYTES;
  static constexpr int BAR_OFF = PAGES_OFF + kMaxPageSlice * 4;
  static constexpr int SMEM = 1024 + BAR_OFF + 64;
  // the split combine reuses the ring: O partial [128][HD] fp32, then (m, l) [128][2], then the weights
  static_assert(kQRowsPerCta * HD * 4 + kQRowsPerCta * 2 * 4 + kQRowsPerCta * 9 * 4 <= 2 * BUF_BYTES, "combine");
  static_assert(SMEM <= 227 * 1024, "shared memory");
  static_assert(Q_BYTES % 1024 == 0 && KV_BLOCK % 1024 == 0 && P_BYTES % 1024 == 0, "1024-byte swizzle atoms");
};

// Byte offset of 16-byte chunk c (of 8 per 128-byte row) of row `row` in a 128-byte-swizzled operand block.
__device__ __forceinline__ uint32_t swz128(int row, int c) { return uint32_t(row * 128 + ((c ^ (row & 7)) << 4)); }

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 1) round_attention_kernel(const AttnArgs a) {
  using L = AttnSmem<HD>;
  constexpr int PIECES = HD / 8;                       // 16-byte pieces of a head row
  constexpr int RSTEP = kAttnThreads / PIECES;         // rows one pass of the CTA covers
  constexpr int ITER = kKeysPerTile / RSTEP;           // rows per thread per 64-key tile
  constexpr uint32_t IDESC_S = umma_idesc_f16(128, kChunkKeys, true);
  constexpr uint32_t IDESC_S_HALF = umma_idesc_f16(128, kKeysPerTile, true);
  constexpr uint32_t IDESC_O = umma_idesc_f16(128, HD, true) | kUmmaBMajorMN;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem + L::Q_OFF;
  uint8_t* p_s = smem + L::P_OFF;
  int* pages = reinterpret_cast<int*>(smem + L::PAGES_OFF);
  uint64_t* s_bar = reinterpret_cast<uint64_t*>(smem + L::BAR_OFF);
  uint64_t* o_bar = s_bar + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_bar + 1);
  auto k_buf = [&](int b) { return smem + L::RING_OFF + b * L::BUF_BYTES; };
  auto v_buf = [&](int b) { return smem + L::RING_OFF + b * L::BUF_BYTES + L::K_BYTES; };

  const int tid = threadIdx.x, warp = tid >> 5;
  const int head = blockIdx.x, split = blockIdx.y, qt = blockIdx.z;
  const int group = head / (a.num_heads / a.num_kv_heads);

  if (tid == 0) {
    mbar_init(s_bar, 1);
    mbar_init(o_bar, 1);
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, kAttnTmemCols);

  // Before the dependency wait: everything the previous kernel does not write. The offset comes from an earlier
  // kernel (the last round's commit, or a copy before a prefill), the block table and the layout are static, and
  // the context keys [0, offset) were written by earlier rounds; only the query rows and the round's own K/V come
  // from the QKV projection this kernel follows.
  const int64_t offset = *a.offset;
  const int64_t seq_len = offset + a.rows;
  const int n_tiles = int((seq_len + kKeysPerTile - 1) / kKeysPerTile);
  // Tiles spread evenly over the splits, the larger shares first: the last split holds the masked tiles of the
  // round's own keys, so it gets the smaller share.
  const int t0 = n_tiles - int(int64_t(a.splits - split) * n_tiles / a.splits);
  const int t1 = n_tiles - int(int64_t(a.splits - split - 1) * n_tiles / a.splits);
  const int n_local = t1 - t0;
  const int n_chunks = (n_local + kTilesPerChunk - 1) / kTilesPerChunk;
  const int64_t lp0 = (int64_t(t0) * kKeysPerTile) >> a.page_shift;
  const int n_pages = n_local > 0 ? int(((int64_t(t1) * kKeysPerTile - 1) >> a.page_shift) - lp0 + 1) : 0;
  const bool staged_pages = n_pages <= kMaxPageSlice;
  for (int i = tid; i < (staged_pages ? n_pages : 0); i += kAttnThreads) {
    const int64_t lp = lp0 + i;
    pages[i] = lp < a.max_pages ? a.block_table[lp] : -1;
  }
  const int row = qt * kQRowsPerCta + tid;  // this thread's query row
  const bool live = row < a.rows;
  const int dep = live ? a.depth[row] : -1, own = live ? a.own_start[row] : (1 << 30);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_lane = uint32_t(warp * 32) << 16;  // this warp's TMEM lane slice

  const __nv_bfloat16* kc = reinterpret_cast<const __nv_bfloat16*>(a.k_cache);
  const __nv_bfloat16* vc = reinterpret_cast<const __nv_bfloat16*>(a.v_cache);
  // Thread tid copies 16-byte piece tid % PIECES of tile rows tid / PIECES + u * RSTEP: its page lookups are issued
  // together, then per-thread constant address arithmetic; a bad page is recorded once per tile.
  const int my_piece = tid % PIECES, my_row0 = tid / PIECES;
  const size_t head_off = size_t(group) * a.page_size * HD + size_t(my_piece) * 8;  // elements
  const size_t page_stride = size_t(a.num_kv_heads) * a.page_size * HD;            // elements per page
  const uint32_t dst_piece = uint32_t((my_piece >> 3) * L::KV_BLOCK);
  // Tile t (absolute) into half `half` of ring buffer `buf`; `context_only`: only when the whole tile lies below
  // offset (issued before the dependency wait), else only when it does not (after it).
  auto issue_tile = [&](int t, int buf, int half) {
    const int64_t kv0 = int64_t(t) * kKeysPerTile + my_row0;
    int pg[ITER];
#pragma unroll
    for (int u = 0; u < ITER; ++u) {
      const int64_t kv = kv0 + u * RSTEP;
      const int64_t lp = kv >> a.page_shift;
      pg[u] = kv >= seq_len ? -2 : staged_pages ? pages[lp - lp0] : (lp < a.max_pages ? a.block_table[lp] : -1);
    }
    bool bad = false;
#pragma unroll
    for (int u = 0; u < ITER; ++u) {
      const int r = half * kKeysPerTile + my_row0 + u * RSTEP;  // key row inside the chunk
      const bool valid = pg[u] >= 0 && pg[u] < a.num_pages;
      bad |= pg[u] != -2 && !valid;
      const size_t src =
          valid ? size_t(pg[u]) * page_stride + head_off + size_t((kv0 + u * RSTEP) & (a.page_size - 1)) * HD : 0;
      const uint32_t dst = dst_piece + swz128(r, my_piece & 7);
      cp_async_16(k_buf(buf) + dst, kc + src, valid);
      cp_async_16(v_buf(buf) + dst, vc + src, valid);
    }
    if (bad) record_error(a.err, kErrBadIndex);
  };
  auto tile_in_context = [&](int t) { return int64_t(t + 1) * kKeysPerTile <= offset; };
  auto issue_chunk = [&](int c, int mode) {  // mode 0: context tiles only, 1: the others, 2: all
    for (int h = 0; h < kTilesPerChunk; ++h) {
      const int t = t0 + c * kTilesPerChunk + h;
      if (t >= t1) break;
      const bool ctx_tile = tile_in_context(t);
      if (mode == 2 || (mode == 0) == ctx_tile) issue_tile(t, c & 1, h);
    }
  };
  if (n_chunks > 0) issue_chunk(0, 0);

  grid_dependency_wait();
  allow_dependents();

  // Q rows of the tile (rows past a.rows zero-filled), then the rest of chunk 0: commit group 0. Chunk 1: group 1.
  {
    const __nv_bfloat16* q = reinterpret_cast<const __nv_bfloat16*>(a.q);
    const size_t q_stride = size_t(a.num_heads) * HD;
    for (int idx = tid; idx < kQRowsPerCta * PIECES; idx += kAttnThreads) {
      const int r = idx / PIECES, pc = idx % PIECES;
      const int gr = qt * kQRowsPerCta + r;
      const bool ok = gr < a.rows;
      const size_t src = ok ? size_t(gr) * q_stride + size_t(head) * HD + size_t(pc) * 8 : 0;
      cp_async_16(q_s + (pc >> 3) * (kQRowsPerCta * 128) + swz128(r, pc & 7), q + src, ok);
    }
  }
  if (n_chunks > 0) issue_chunk(0, 1);
  cp_async_commit();
  if (n_chunks > 1) issue_chunk(1, 2);
  cp_async_commit();

  const float scale = a.scale_log2;
  float m_run = -INFINITY, l_run = 0.f;
  for (int c = 0; c < n_chunks; ++c) {
    const int buf = c & 1;
    const int tiles = min(kTilesPerChunk, t1 - (t0 + c * kTilesPerChunk));
    const int n_keys = tiles * kKeysPerTile;
    const int64_t key0 = int64_t(t0 + c * kTilesPerChunk) * kKeysPerTile;
    cp_async_wait<1>();          // chunk c (and Q) landed for this thread
    fence_proxy_async_shared();  // ... and is visible to the tensor cores
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t q_addr = smem_u32(q_s), k_addr = smem_u32(k_buf(buf));
#pragma unroll
      for (int kk = 0; kk < HD / 16; ++kk) {
        const uint64_t ad = umma_desc_sw128(q_addr + (kk >> 2) * (kQRowsPerCta * 128) + (kk & 3) * 32);
        const uint64_t bd = umma_desc_sw128(k_addr + (kk >> 2) * L::KV_BLOCK + (kk & 3) * 32);
        umma_f16(tmem, ad, bd, n_keys == kChunkKeys ? IDESC_S : IDESC_S_HALF, kk > 0 ? 1u : 0u);
      }
      umma_commit(s_bar);
    }
    __syncwarp();
    mbar_wait(s_bar, uint32_t(c & 1), a.err, kErrTimeoutDone);
    tc_fence_after();

    // This thread's row of S: scale, mask, row maximum.
    uint32_t sr[kChunkKeys];
    tmem_ld_32cols_async(tmem + t_lane + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
    tmem_ld_32cols_async(tmem + t_lane + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
    if (n_keys > kKeysPerTile) {
      tmem_ld_32cols_async(tmem + t_lane + 64, *reinterpret_cast<uint32_t(*)[32]>(sr + 64));
      tmem_ld_32cols_async(tmem + t_lane + 96, *reinterpret_cast<uint32_t(*)[32]>(sr + 96));
    }
    tmem_ld_wait();
    const bool need_mask = key0 + n_keys > offset;
    float mx = -INFINITY;
#pragma unroll
    for (int j = 0; j < kChunkKeys; ++j) {  // in place: sr[j] becomes the scaled, masked score
      const float v = __uint_as_float(sr[j]) * scale;
      bool vis = live && j < n_keys;
      if (need_mask && vis) {
        const int64_t kv = key0 + j;
        vis = kv < seq_len;
        if (vis && kv >= offset) {
          const int64_t rel = kv - offset;
          vis = rel <= dep || (rel >= own && rel <= row);
        }
      }
      const float sv = vis ? v : -INFINITY;
      sr[j] = __float_as_uint(sv);
      mx = fmaxf(mx, sv);
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = m_new == -INFINITY ? 1.f : ex2(m_run - m_new);
    m_run = m_new;
    // before P is overwritten, the previous chunk's P V must have read it
    if (c > 0) {
      mbar_wait(o_bar, uint32_t((c - 1) & 1), a.err, kErrTimeoutDone);
      tc_fence_after();
    }
    // P = 2^(S - m) for this row, rounded to bf16, into the row's 128-byte rows of the P operand
    float psum = 0.f;
#pragma unroll
    for (int j8 = 0; j8 < kChunkKeys / 8; ++j8) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p0 = m_new == -INFINITY ? 0.f : ex2(__uint_as_float(sr[8 * j8 + 2 * e]) - m_new);
        const float p1 = m_new == -INFINITY ? 0.f : ex2(__uint_as_float(sr[8 * j8 + 2 * e + 1]) - m_new);
        psum += p0 + p1;
        w[e] = pack_bf16(p0, p1);
      }
      if (j8 * 8 < n_keys)
        *reinterpret_cast<uint4*>(p_s + (j8 >> 3) * (kQRowsPerCta * 128) + swz128(tid, j8 & 7)) =
            make_uint4(w[0], w[1], w[2], w[3]);
    }
    l_run = l_run * alpha + psum;
    // Rescale this row of O when its maximum grew (the whole warp joins the TMEM round trip if any lane needs it).
    if (c > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll
      for (int c32 = 0; c32 < HD / 32; ++c32) {
        uint32_t o[32];
        tmem_ld_32cols_async(tmem + t_lane + kTmemO + c32 * 32, o);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
        tmem_st_32cols(tmem + t_lane + kTmemO + c32 * 32, o);
      }
    }
    fence_proxy_async_shared();  // P is read by the tensor cores next
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      const uint32_t p_addr = smem_u32(p_s), v_addr = smem_u32(v_buf(buf));
      for (int kk = 0; kk < n_keys / 16; ++kk) {
        const uint64_t ad = umma_desc_sw128(p_addr + (kk >> 2) * (kQRowsPerCta * 128) + (kk & 3) * 32);
        const uint64_t bd = umma_desc_sw128_mn(v_addr + kk * 16 * 128, L::KV_BLOCK, 1024);
        umma_f16(tmem + kTmemO, ad, bd, IDESC_O, (c > 0 || kk > 0) ? 1u : 0u);
      }
      umma_commit(o_bar);
    }
    __syncwarp();
    // The ring buffer of chunk c is free once its P V has completed: chunk c + 2 goes there.
    if (c + 2 < n_chunks) {
      mbar_wait(o_bar, uint32_t(c & 1), a.err, kErrTimeoutDone);
      issue_chunk(c + 2, 2);
    }
    cp_async_commit();
  }
  if (n_chunks > 0) mbar_wait(o_bar, uint32_t((n_chunks - 1) & 1), a.err, kErrTimeoutDone);
  cp_async_wait<0>();
  tc_fence_after();

  // This thread's row of O (unnormalised) from TMEM.
  float o[HD];
#pragma unroll
  for (int c32 = 0; c32 < HD / 32; ++c32) tmem_ld_32cols_async(tmem + t_lane + kTmemO + c32 * 32,
                                                               *reinterpret_cast<uint32_t(*)[32]>(o + c32 * 32));
  tmem_ld_wait();
  if (n_chunks == 0) {
#pragma unroll
    for (int i = 0; i < HD; ++i) o[i] = 0.f;
  }
  tc_fence_before();
  __syncthreads();  // every thread has its row: TMEM and the ring are free
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kAttnTmemCols);
  }

  __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(a.out);
  const size_t out_stride = size_t(a.num_heads) * HD;
  // Eight consecutive output elements (one 16-byte chunk) of row `r`, columns col .. col + 7 of the head output:
  // row-major, or inside the row tiles (the 16-byte chunk of its k-block).
  uint8_t* tiles = static_cast<uint8_t*>(a.row_tiles);
  auto out_chunk = [&](int r, int col) -> uint4* {
    if (tiles != nullptr) return reinterpret_cast<uint4*>(tiles) + row_tile_chunk(col >> 6, r, (col >> 3) & 7, a.tile_rows);
    return reinterpret_cast<uint4*>(out + size_t(r) * out_stride + col);
  };
  if (a.splits == 1) {
    if (live) {
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
#pragma unroll
      for (int j = 0; j < HD / 8; ++j)
        *out_chunk(row, head * HD + 8 * j) =
            make_uint4(pack_bf16(o[8 * j] * inv, o[8 * j + 1] * inv), pack_bf16(o[8 * j + 2] * inv, o[8 * j + 3] * inv),
                       pack_bf16(o[8 * j + 4] * inv, o[8 * j + 5] * inv), pack_bf16(o[8 * j + 6] * inv, o[8 * j + 7] * inv));
    }
    return;
  }

  // ---- split partials, combined over the cluster of the (head, query tile) ----
  // Each CTA leaves its unnormalised partial (O, m, l) in its own shared memory (the ring is free now); after a
  // cluster barrier rank q combines its share of the live rows over all ranks in rank order through distributed
  // shared memory; a second barrier keeps every partial alive until all rows are combined.
  float* po = reinterpret_cast<float*>(smem + L::RING_OFF);         // [128][HD]
  float* pml = po + kQRowsPerCta * HD;                              // [128][2]
  float* wts = pml + kQRowsPerCta * 2;                              // [rows of this rank][S + 1]
  if (live) {
#pragma unroll
    for (int j = 0; j < HD / 4; ++j)
      *reinterpret_cast<float4*>(po + tid * HD + 4 * j) = make_float4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
    *reinterpret_cast<float2*>(pml + tid * 2) = make_float2(m_run, l_run);
  }
  cluster_sync();
  const int S = a.splits;
  const uint32_t rank = cluster_rank();
  const int live_rows = max(0, min(kQRowsPerCta, a.rows - qt * kQRowsPerCta));
  const int rpc = (live_rows + S - 1) / S;
  const int row_begin = min(live_rows, int(rank) * rpc);
  const int my_rows = max(0, min(rpc, live_rows - row_begin));
  if (tid < my_rows) {
    const int r = row_begin + tid;
    float ms[8], ls[8], mmax = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < 8; ++sp) {
      ms[sp] = -INFINITY;
      ls[sp] = 0.f;
      if (sp < S) {
        const float2 ml = ld_dsmem_f32x2(cluster_map(pml + r * 2, uint32_t(sp)));
        ms[sp] = ml.x;
        ls[sp] = ml.y;
        mmax = fmaxf(mmax, ml.x);
      }
    }
    float lsum = 0.f;
#pragma unroll
    for (int sp = 0; sp < 8; ++sp) {
      const float w = (sp < S && ms[sp] != -INFINITY) ? exp2f(ms[sp] - mmax) : 0.f;
      if (sp < S) wts[tid * (S + 1) + sp] = w;
      lsum += w * ls[sp];
    }
    wts[tid * (S + 1) + S] = lsum > 0.f ? 1.f / lsum : 0.f;
  }
  __syncthreads();
  // 16-byte remote loads of eight output elements, every rank's piece in flight before any is summed
  constexpr int Q8 = HD / 8;
  for (int idx = tid; idx < my_rows * Q8; idx += kAttnThreads) {
    const int lr = idx / Q8, c8 = (idx % Q8) * 8;
    const uint32_t off = uint32_t((row_begin + lr) * HD + c8) * 4u;
    float4 lo[8], hi[8];
#pragma unroll
    for (int sp = 0; sp < 8; ++sp) {
      if (sp < S) {
        const uint32_t base = cluster_map(po, uint32_t(sp)) + off;
        lo[sp] = ld_dsmem_f32x4(base);
        hi[sp] = ld_dsmem_f32x4(base + 16);
      }
    }
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int sp = 0; sp < 8; ++sp) {
      if (sp < S) {
        const float w = wts[lr * (S + 1) + sp];
        acc[0] += w * lo[sp].x;
        acc[1] += w * lo[sp].y;
        acc[2] += w * lo[sp].z;
        acc[3] += w * lo[sp].w;
        acc[4] += w * hi[sp].x;
        acc[5] += w * hi[sp].y;
        acc[6] += w * hi[sp].z;
        acc[7] += w * hi[sp].w;
      }
    }
    const float inv = wts[lr * (S + 1) + S];
    *out_chunk(qt * kQRowsPerCta + row_begin + lr, head * HD + c8) =
        make_uint4(pack_bf16(acc[0] * inv, acc[1] * inv), pack_bf16(acc[2] * inv, acc[3] * inv),
                   pack_bf16(acc[4] * inv, acc[5] * inv), pack_bf16(acc[6] * inv, acc[7] * inv));
  }
  cluster_sync();
}

template <int HD>
int launch_attention(const AttnArgs& a, int q_tiles, cudaStream_t stream, bool pdl) {
  constexpr int SMEM = AttnSmem<HD>::SMEM;
  auto kernel = round_attention_kernel<HD>;
  const int st = raise_smem_limit(reinterpret_cast<const void*>(kernel), SMEM, "cudaFuncSetAttribute(attention smem)");
  if (st != PLM_OK) return st;
  return check_cuda(launch_ex(kernel, dim3(a.num_heads, a.splits, q_tiles), dim3(kAttnThreads), SMEM, stream, pdl,
                              a.splits, a),
                    "round_attention_kernel");
}

}  // namespace

int attention_splits(int num_heads, int q_tiles, int num_sms, int64_t max_keys) {
  // One CTA per SM (shared memory and tensor memory): double the splits while the grid still fits in one wave and
  // every split keeps at least two tiles.
  const int ctas = num_heads * q_tiles;
  const int max_tiles = int((max_keys + kKeysPerTile - 1) / kKeysPerTile);
  int splits = 1;
  while (splits < 8 && ctas * 2 * splits <= num_sms && 2 * splits <= max_tiles / 2) splits *= 2;
  return splits;
}

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
  if (a.splits > 8 || (a.splits & (a.splits - 1)) != 0)
    return fail(PLM_ERR_UNSUPPORTED, "attention: %d splits (a power of two <= 8)", a.splits);
  a.err = ctx->err;
  return a.head_dim == 128 ? launch_attention<128>(a, q_tiles, stream, pdl)
                           : launch_attention<64>(a, q_tiles, stream, pdl);
}

}  // namespace plm

using namespace plm;

extern "C" int plm_attention(plm_ctx* ctx, const plm_attention_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_attention: null argument");
  if (d->dtype != PLM_BF16) return fail(PLM_ERR_UNSUPPORTED, "plm_attention: only bf16 is built");
  AttnArgs a = {};
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
  return attention_launch(ctx, a, static_cast<cudaStream_t>(stream), true);
}
