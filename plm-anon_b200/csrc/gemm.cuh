// Skinny weight-streaming GEMM for the round: Y[rows, n_out] = X[rows, k] . W[n_out, k]^T, fp32 accumulation.
//
// The round has only W = k + k^2 query rows (56 at k = 7), so every weight byte is used by one MMA and the
// kernel is bound by HBM bandwidth on the weight stream. The operands are swapped: a 128-row weight tile is the
// MMA's M side (TMEM lanes = output features) and the round rows are its N side (TMEM columns = rows), so one
// tcgen05.mma.kind::f16 of 128 x NTOK x 16 covers the whole round. Weight tiles (128 rows x 64 k, 16 KB) and
// row tiles (NTOK rows x 64 k) are staged by TMA with the 128-byte swizzle into a STAGES-deep ring; one thread
// issues TMA (warp 0), one thread issues MMAs (warp 1), and the four warps read the accumulator back with
// tcgen05.ld.
//
// Work is split over (output tile, k-split). The k-splits of a tile run as one thread-block cluster: each CTA keeps
// its fp32 partial tile in its own shared memory and, after a cluster barrier, reduces one slice of the token
// columns over all ranks in rank order through distributed shared memory, so the result does not depend on timing
// and no global scratch is involved. Each CTA then runs the fused epilogue on its slice:
//   kEpiStore    plain store in the model dtype;
//   kEpiSiluMul  the gate_up projection with SiLU(gate) * up fused (tile = 64 gate rows + the matching 64 up rows);
//   kEpiQkvRope  the qkv projection with neox RoPE on q and k, q written out, k and v scattered into the paged cache;
//   kEpiLogits   the lm_head: verify rows as fp32 logits, proposal rows reduced to a per-tile (max, first index);
//   kEpiTable    the Voronoi cost table, table[v][a] = -(aux_vocab[a] . lm_head[v]);
//   kEpiPartial  each k-split's fp32 partial straight to global memory, no cluster reduction (the next kernel sums
//                the splits in order).
// Weight loads are issued before griddepcontrol.wait, so under programmatic dependent launch they overlap the
// tail of the previous kernel; everything that reads activations comes after it.
#pragma once

#include <type_traits>

#include "common.cuh"

namespace plm {

constexpr int kMaxPartialSplits = 16;  // k-splits a kEpiPartial launch may write out

enum GemmEpilogueKind : int {
  kEpiStore = 0,
  kEpiSiluMul = 1,
  kEpiQkvRope = 2,
  kEpiLogits = 3,
  kEpiTable = 4,
  kEpiPartial = 5,
};

struct QkvEpilogue {
  void* q_out;               // [rows][num_heads * head_dim]
  void* k_cache;             // K plane: [num_pages][num_kv_heads][page_size][head_dim]
  void* v_cache;             // V plane, same layout
  const int32_t* positions;  // [rows] rotary position of each row
  const int64_t* slots;      // [rows] physical slot = page * page_size + index within the page
  const void* cos_sin;       // [max_pos][head_dim]: cos in [0, hd/2), sin in [hd/2, hd), model dtype
  int num_heads, num_kv_heads, head_dim, page_size;
  int64_t num_slots;         // num_pages * page_size
  int max_pos;
};

struct LogitsEpilogue {
  float* verify_logits;  // [n_verify][vocab]: fp32 copies of the model-dtype logits
  float* best_val;       // [n_tiles][rows]: per-tile maximum of each proposal row
  int32_t* best_idx;     // [n_tiles][rows]: its first index
  int n_verify;
  int vocab;
};

struct TableEpilogue {
  void* table;  // [vocab][aux] model dtype
  int aux;
  int a0;       // aux item of this launch's row 0
};

struct GemmArgs {
  int n_out;
  int k;
  int rows;
  int n_tiles;
  int splits;
  int kb_per_split;
  int gate_offset;  // kEpiSiluMul: first row of the up half inside W (the intermediate size)
  void* out;
  int ldo;
  int* err;
  QkvEpilogue qkv;
  LogitsEpilogue logits;
  TableEpilogue table;
  const float* corr;  // kEpiQkvRope / kEpiSiluMul: fp32 corrections of rows >= corr_from (gated-LoRA adapters)
  int corr_from;
  int corr_ld;
  // non-null: the weight as packed 128-row tiles (pack.cu: [tile][k-block] 16 KB shared-memory images), loaded with
  // one untiled bulk copy per k-block instead of the tensor map
  const uint8_t* w_packed;
};

constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 128;
constexpr int kStagePad = 132;  // fp32 staging row stride (16-byte rows for vector loads of a column's features)

template <int NTOK>
struct GemmShape {
  static constexpr int A_BYTES = 128 * kGemmBK * 2;
  static constexpr int B_BYTES = NTOK * kGemmBK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr uint32_t TMEM_COLS = NTOK <= 32 ? 32 : NTOK <= 64 ? 64 : NTOK <= 128 ? 128 : 256;
  static_assert(NTOK % 16 == 0 && NTOK >= 16 && NTOK <= 256, "token tile must be a multiple of 16 in [16, 256]");
  static_assert(STAGE_BYTES % 1024 == 0, "stages must keep 1024-byte alignment for the 128-byte swizzle");
};

// Bytes before the barriers: the TMA ring, or after the main loop the fp32 staging tile plus (with a split) the
// reduced slice of at most half the columns, whichever is larger. Splits are only used for NTOK <= 128.
template <int NTOK, int STAGES>
constexpr int gemm_bar_offset() {
  constexpr int ring = STAGES * GemmShape<NTOK>::STAGE_BYTES;
  constexpr int staging = (NTOK <= 128 ? NTOK + NTOK / 2 : NTOK) * kStagePad * 4;
  return ((ring > staging ? ring : staging) + 7) & ~7;
}

// The QKV epilogue's per-column data: positions and slots in an area of their own (read while the MMAs run), the
// rotary rows of those positions in the ring's space past the staging tile (copied once the ring is consumed), where
// that space holds NTOK rows of head_dim <= 128.
template <int NTOK>
constexpr int gemm_rowdata_bytes() {
  return (NTOK * 12 + 15) & ~15;
}
template <int NTOK>
constexpr int gemm_staging_end() {
  return ((NTOK <= 128 ? NTOK + NTOK / 2 : NTOK) * kStagePad * 4 + 15) & ~15;
}
template <int NTOK, int STAGES>
constexpr bool gemm_rope_staged() {
  return gemm_bar_offset<NTOK, STAGES>() - gemm_staging_end<NTOK>() >= NTOK * 128 * 2;
}

template <int NTOK, int STAGES>
constexpr int gemm_smem_bytes() {
  return gemm_bar_offset<NTOK, STAGES>() + 1024 /*alignment slack*/ + 256 /*barriers, flags*/ +
         gemm_rowdata_bytes<NTOK>();
}

template <typename T, int NTOK, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
    skinny_gemm_kernel(const __grid_constant__ CUtensorMap map_w, const __grid_constant__ CUtensorMap map_x,
                       const GemmArgs args) {
  using Shape = GemmShape<NTOK>;
  constexpr uint32_t IDESC = umma_idesc_f16(128, NTOK, std::is_same<T, __nv_bfloat16>::value);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + gemm_bar_offset<NTOK, STAGES>());
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* done_bar = empty_bar + STAGES;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  int* flags = reinterpret_cast<int*>(tmem_slot + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tile = blockIdx.x, split = blockIdx.y;
  const int total_kb = args.k / kGemmBK;
  const int kb_begin = split * total_kb / args.splits;  // k-blocks spread evenly: no split is empty
  const int kb_end = (split + 1) * total_kb / args.splits;
  const int nk = kb_end - kb_begin;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full_bar + s, 1);
      mbar_init(empty_bar + s, 1);
    }
    mbar_init(done_bar, 1);
    flags[0] = 0;  // abort
    flags[1] = 0;  // this CTA reduces the tile
    flags[2] = 0;  // k-blocks issued by the producer
    flags[3] = 0;  // k-blocks consumed by the MMA issuer
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, Shape::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  allow_dependents();

  // Role warps are kept converged: lane 0 waits and issues, the other lanes park in __shfl_sync, so no lane spins
  // in a barrier wait beside the issuing lane.
  auto warp_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    int ok = 1;
    if (lane == 0) ok = mbar_wait(bar, parity, args.err, code) ? 1 : 0;
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
  };
  if (warp == 0) {
    // ---------------- TMA producer warp ----------------
    uint64_t pol_w = 0, pol_x = 0;
    if (lane == 0) {
      tma_prefetch_map(&map_w);
      tma_prefetch_map(&map_x);
      pol_w = l2_policy_evict_first();
      pol_x = l2_policy_evict_last();
    }
    auto load_w = [&](int s, int kb) {
      uint8_t* a = smem + s * Shape::STAGE_BYTES;
      if (args.w_packed != nullptr) {
        bulk_load(a, args.w_packed + (size_t(tile) * (args.k / kGemmBK) + kb) * Shape::A_BYTES, Shape::A_BYTES,
                  full_bar + s, pol_w);
        return;
      }
      if (EPI == kEpiSiluMul) {
        // 64 gate rows then the 64 up rows of the same intermediate features.
        tma_load_2d(a, &map_w, full_bar + s, kb * kGemmBK, tile * 64, pol_w);
        tma_load_2d(a + 64 * 128, &map_w, full_bar + s, kb * kGemmBK, args.gate_offset + tile * 64, pol_w);
      } else {
        tma_load_2d(a, &map_w, full_bar + s, kb * kGemmBK, tile * 128, pol_w);
      }
    };
    auto load_x = [&](int s, int kb) {
      uint8_t* b = smem + s * Shape::STAGE_BYTES + Shape::A_BYTES;
      tma_load_2d(b, &map_x, full_bar + s, kb * kGemmBK, 0, pol_x);
    };
    const int pre = nk < STAGES ? nk : STAGES;
    if (lane == 0) {
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(full_bar + i, Shape::STAGE_BYTES);
        load_w(i, kb_begin + i);
      }
    }
    grid_dependency_wait();  // the row operand is written by the previous kernel
    if (lane == 0)
      for (int i = 0; i < pre; ++i) load_x(i, kb_begin + i);
    int issued = pre;
    for (int i = STAGES; i < nk; ++i) {
      const int s = i % STAGES;
      if (!warp_wait(empty_bar + s, ((i / STAGES) - 1) & 1, kErrTimeoutEmpty)) {
        // Stages already issued still land; they are drained before the CTA reuses shared memory.
        if (lane == 0) flags[0] = 1;
        break;
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(full_bar + s, Shape::STAGE_BYTES);
        load_w(s, kb_begin + i);
        load_x(s, kb_begin + i);
      }
      issued = i + 1;
    }
    if (lane == 0) flags[2] = issued;
  } else if (warp == 1) {
    // ---------------- MMA warp ----------------
    int consumed = 0;
    for (int i = 0; i < nk; ++i) {
      const int s = i % STAGES;
      if (!warp_wait(full_bar + s, (i / STAGES) & 1, kErrTimeoutFull)) {
        if (lane == 0) flags[0] = 1;
        break;
      }
      tc_fence_after();
      if (lane == 0) {
        const uint32_t a_addr = smem_u32(smem + s * Shape::STAGE_BYTES);
        const uint32_t b_addr = a_addr + Shape::A_BYTES;
#pragma unroll
        for (int kk = 0; kk < kGemmBK / 16; ++kk) {
          umma_f16(tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), IDESC,
                   (i > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(empty_bar + s);
      }
      __syncwarp();
      consumed = i + 1;
    }
    if (lane == 0) {
      flags[3] = consumed;
      umma_commit(done_bar);
    }
    __syncwarp();
  }
  grid_dependency_wait();

  // This CTA's token columns after the split reduction: [c_begin, c_end) of the tile.
  const int S = args.splits;
  const uint32_t rank = S > 1 ? cluster_rank() : 0;
  const int cs = (args.rows + S - 1) / S;
  const int c_begin = min(args.rows, int(rank) * cs), c_end = min(args.rows, c_begin + cs);
  constexpr bool kRopeStaged = EPI == kEpiQkvRope && gemm_rope_staged<NTOK, STAGES>();
  const bool rope_staged = kRopeStaged && args.qkv.head_dim <= 128;
  int* const rd_pos = reinterpret_cast<int*>(smem + gemm_bar_offset<NTOK, STAGES>() + 256);  // [NTOK]
  int64_t* const rd_slot = reinterpret_cast<int64_t*>(rd_pos + NTOK);                       // [NTOK]
  T* const rd_cs = reinterpret_cast<T*>(smem + gemm_staging_end<NTOK>());                    // [NTOK][head_dim]
  if (rope_staged && warp >= 2) {  // warps without a role fetch the columns' positions and slots meanwhile
    for (int i = tid - 64; i < c_end - c_begin; i += kGemmThreads - 64) {
      rd_pos[i] = __ldg(args.qkv.positions + c_begin + i);
      rd_slot[i] = __ldg(args.qkv.slots + c_begin + i);
    }
  }

  // ---------------- accumulator -> this CTA's staging tile (fp32, [token][feature]) ----------------
  const bool mma_ok = warp_wait(done_bar, 0, kErrTimeoutDone);
  tc_fence_after();
  float* stage = reinterpret_cast<float*>(smem);
  const int row = warp * 32 + lane;  // feature lane inside the 128-wide tile
  const uint32_t t_warp = tmem + (uint32_t(warp * 32) << 16);
  const int rows = args.rows;
  float* partial = EPI == kEpiPartial ? reinterpret_cast<float*>(args.out) + size_t(split) * rows * args.ldo : nullptr;
  const int part_feats = min(128, args.n_out - tile * 128);
  for (int c0 = 0; c0 < rows; c0 += 32) {
    float v[32];
    tmem_ld_32cols(t_warp + c0, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      if (c0 + j >= rows) continue;
      if (EPI == kEpiPartial) {  // a warp's 32 lanes write 32 consecutive features of one row
        if (row < part_feats) partial[size_t(c0 + j) * args.ldo + tile * 128 + row] = v[j];
      } else {
        stage[(c0 + j) * kStagePad + row] = v[j];
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (rope_staged && flags[0] == 0) {
    // The rotary rows of the columns' positions, copied into the consumed ring while the split reduction runs.
    const int hd = args.qkv.head_dim, chunks = hd / 8;
    const T* cs_tab = reinterpret_cast<const T*>(args.qkv.cos_sin);
    for (int idx = tid; idx < (c_end - c_begin) * chunks; idx += kGemmThreads) {
      const int r = idx / chunks, ch = idx % chunks;
      const int pos = rd_pos[r];
      const bool valid = pos >= 0 && pos < args.qkv.max_pos;
      cp_async_16(rd_cs + r * hd + ch * 8, cs_tab + (valid ? size_t(pos) * hd + ch * 8 : 0), valid);
    }
    cp_async_commit();
  }
  if (flags[0] != 0 && tid == 0) {
    // Aborted: let every TMA copy this CTA issued but never consumed land before shared memory is reused.
    for (int i = flags[3]; i < flags[2]; ++i)
      if (!mbar_wait(full_bar + (i % STAGES), (i / STAGES) & 1, args.err, kErrTimeoutFull)) break;
  }
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, Shape::TMEM_COLS);
  }
  const bool ok = mma_ok && flags[0] == 0;
  if (EPI == kEpiPartial) return;  // launched without a cluster: nothing left to reduce here

  // ---------------- split reduction over the cluster ----------------
  // The `splits` CTAs of a tile form one cluster. After the barrier, rank r sums the partial tiles of all ranks,
  // in rank order, for its slice of token columns [c_begin, c_end), reading peers' staging tiles through
  // distributed shared memory; a second barrier keeps every staging tile alive until all slices are read.
  float* red = stage;
  if (S > 1) {
    red = stage + rows * kStagePad;
    cluster_sync();
    uint32_t peer[8];
#pragma unroll
    for (int s = 0; s < 8; ++s) peer[s] = s < S ? cluster_map(stage, uint32_t(s)) : 0u;
    // 16-byte remote loads: thread tid takes features [4 (tid % 32), +4) of local columns tid / 32, + 4, ...; the
    // loads of kPullCols of its columns from every rank are issued before any is summed.
    constexpr int kPullCols = 4;
    const int ncols_red = c_end - c_begin;
    const int fq = (tid & 31) * 4, cq = tid >> 5;
    for (int i0 = cq; i0 < ncols_red; i0 += 4 * kPullCols) {
      float4 part[kPullCols][8];
#pragma unroll
      for (int i = 0; i < kPullCols; ++i) {
        const int lc = i0 + 4 * i;
        const uint32_t off = uint32_t((c_begin + lc) * kStagePad + fq) * 4u;
#pragma unroll
        for (int s = 0; s < 8; ++s)
          part[i][s] = (s < S && lc < ncols_red) ? ld_dsmem_f32x4(peer[s] + off) : make_float4(0.f, 0.f, 0.f, 0.f);
      }
#pragma unroll
      for (int i = 0; i < kPullCols; ++i) {
        const int lc = i0 + 4 * i;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int s = 0; s < 8; ++s) {
          if (s < S) {
            acc.x += part[i][s].x;
            acc.y += part[i][s].y;
            acc.z += part[i][s].z;
            acc.w += part[i][s].w;
          }
        }
        if (lc < ncols_red) *reinterpret_cast<float4*>(red + lc * kStagePad + fq) = acc;
      }
    }
    cluster_sync();
  } else {
    __syncthreads();
  }
  if (!ok) return;
  if (kRopeStaged) {
    cp_async_wait<0>();
    __syncthreads();
  }
  // From here `red` holds the finished tile for token columns [c_begin, c_end), local column c - c_begin.

  // ---------------- fused epilogues ----------------
  const int ncols = c_end - c_begin;
  if (EPI == kEpiStore) {
    T* out = reinterpret_cast<T*>(args.out);
    const int n0 = tile * 128;
    const int feats = min(128, args.n_out - n0);
    for (int idx = tid; idx < ncols * 128; idx += kGemmThreads) {
      const int lc = idx >> 7, f = idx & 127;
      if (f < feats) out[size_t(c_begin + lc) * args.ldo + n0 + f] = from_f32<T>(red[lc * kStagePad + f]);
    }
  } else if (EPI == kEpiSiluMul) {
    T* out = reinterpret_cast<T*>(args.out);
    const int j0 = tile * 64;
    for (int idx = tid; idx < ncols * 64; idx += kGemmThreads) {
      const int lc = idx >> 6, f = idx & 63;
      float g = round_to<T>(red[lc * kStagePad + f]);
      float u = round_to<T>(red[lc * kStagePad + 64 + f]);
      const int c = c_begin + lc;
      if (args.corr != nullptr && c >= args.corr_from) {  // the adapter's output joins before the activation
        const float* cr = args.corr + size_t(c - args.corr_from) * args.corr_ld;
        g = round_to<T>(g + cr[j0 + f]);
        u = round_to<T>(u + cr[args.gate_offset + j0 + f]);
      }
      const float act = g / (1.0f + expf(-g)) * u;
      out[size_t(c_begin + lc) * args.ldo + j0 + f] = from_f32<T>(act);
    }
  } else if (EPI == kEpiQkvRope) {
    // Thread tid owns feature tile * 128 + tid of every row of the slice, so what depends on the feature alone (its
    // head, rotary partner, plane) is worked out once, and a power-of-two page splits a slot with a shift and a
    // mask instead of a 64-bit division. The row data (positions, slots, the rotary table) is read-only during the
    // launch and is read through the non-coherent path.
    static_assert(kGemmThreads == 128, "one feature per thread");
    const QkvEpilogue& q = args.qkv;
    const int hd = q.head_dim, half = hd >> 1;
    const int q_size = q.num_heads * hd, kv_size = q.num_kv_heads * hd;
    const int f = tid, F = tile * 128 + f;
    const int d = F % hd;
    const bool rope = F < q_size + kv_size, is_q = F < q_size, is_k = !is_q && rope;
    const int dh = d < half ? d : d - half;
    const int fp = d < half ? f + half : f - half;
    const int g = is_q ? 0 : (is_k ? F - q_size : F - q_size - kv_size) / hd;
    const bool pow2_page = (q.page_size & (q.page_size - 1)) == 0;
    const int page_shift = __ffs(q.page_size) - 1;
    const T* cs_tab = reinterpret_cast<const T*>(q.cos_sin);
    T* plane = reinterpret_cast<T*>(is_k ? q.k_cache : q.v_cache);
    // the last tile may run past n_out when (heads + 2 kv_heads) * head_dim is not a multiple of 128
    for (int lc = 0; lc < (F < args.n_out ? ncols : 0); ++lc) {
      const int c = c_begin + lc;
      const float* cr = (args.corr != nullptr && c >= args.corr_from)
                            ? args.corr + size_t(c - args.corr_from) * args.corr_ld : nullptr;
      float x = round_to<T>(red[lc * kStagePad + f]);
      if (cr != nullptr) x = round_to<T>(x + cr[F]);  // the adapter's output joins before the rotary embedding
      float y = x;
      if (rope) {
        const int pos = rope_staged ? rd_pos[lc] : __ldg(q.positions + c);
        if (pos < 0 || pos >= q.max_pos) {
          record_error(args.err, kErrBadIndex);
          continue;
        }
        float xp = round_to<T>(red[lc * kStagePad + fp]);
        if (cr != nullptr) xp = round_to<T>(xp + cr[tile * 128 + fp]);
        const T* cs_row = rope_staged ? rd_cs + lc * hd : cs_tab + size_t(pos) * hd;
        const float cv = to_f32<T>(cs_row[dh]);
        const float sv = to_f32<T>(cs_row[half + dh]);
        y = d < half ? x * cv - xp * sv : x * cv + xp * sv;
      }
      if (is_q) {
        reinterpret_cast<T*>(q.q_out)[size_t(c) * q_size + F] = from_f32<T>(y);
      } else {
        const int64_t slot = rope_staged ? rd_slot[lc] : __ldg(q.slots + c);
        if (slot < 0 || slot >= q.num_slots) {
          record_error(args.err, kErrBadIndex);
          continue;
        }
        const int64_t page = pow2_page ? slot >> page_shift : slot / q.page_size;
        const int64_t within = pow2_page ? slot & (q.page_size - 1) : slot % q.page_size;
        plane[((page * q.num_kv_heads + g) * q.page_size + within) * hd + d] = from_f32<T>(y);
      }
    }
  } else if (EPI == kEpiLogits) {
    const LogitsEpilogue& L = args.logits;
    const int n0 = tile * 128;
    const int nv_end = min(c_end, L.n_verify);
    for (int idx = tid; idx < max(0, nv_end - c_begin) * 128; idx += kGemmThreads) {
      const int lc = idx >> 7, f = idx & 127;
      if (n0 + f < L.vocab)
        L.verify_logits[size_t(c_begin + lc) * L.vocab + n0 + f] = round_to<T>(red[lc * kStagePad + f]);
    }
    for (int c = max(c_begin, L.n_verify) + warp; c < c_end; c += kGemmThreads / 32) {
      const int lc = c - c_begin;
      float best = -INFINITY;
      int bi = 0x7fffffff;
      for (int f = lane; f < 128; f += 32) {
        const int v = n0 + f;
        if (v < L.vocab) {
          const float x = round_to<T>(red[lc * kStagePad + f]);
          if (x > best || (x == best && v < bi)) {
            best = x;
            bi = v;
          }
        }
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
      if (lane == 0) {
        L.best_val[size_t(tile) * rows + c] = best;
        L.best_idx[size_t(tile) * rows + c] = bi;
      }
    }
  } else if (EPI == kEpiTable) {
    const TableEpilogue& tb = args.table;
    T* table = reinterpret_cast<T*>(tb.table);
    const int n0 = tile * 128;
    const int feats = min(128, args.n_out - n0);
    for (int idx = tid; idx < ncols * 128; idx += kGemmThreads) {
      const int f = idx / ncols, lc = idx % ncols;
      if (f < feats)
        table[size_t(n0 + f) * tb.aux + tb.a0 + c_begin + lc] = from_f32<T>(-round_to<T>(red[lc * kStagePad + f]));
    }
  }
}

}  // namespace plm
