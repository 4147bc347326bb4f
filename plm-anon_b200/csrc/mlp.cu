// Everything between attention and the next layer's input norm as ONE persistent launch per layer:
//   o partials[s] = attn[:, K_s] . Wo[:, K_s]^T          (o_proj, fp32 k-split partials)
//   residual, x   = residual-add RMSNorm of sum_s o partials[s]   (vLLM fused_add_rms_norm)
//   act           = SiLU(x . Wg^T) * (x . Wu^T)          (gate_up_proj -> SiluAndMul)
//   partials[s]   = act[:, K_s] . Wd[:, K_s]^T           (down_proj, fp32 k-split partials; the residual-add RMSNorm
//                                                         launched after the block sums them)
// The products and the norm are those of the separate launches it replaces (skinny_gemm_kernel with the kEpiPartial
// and kEpiSiluMul epilogues, add_norm_kernel); a gate_up tile is accumulated by one CTA over the whole k range
// instead of a cluster of k-splits, and the norm's sum of squares is reduced in another order, so fp32 sums are
// formed in another order.
//
// Why one launch: at 56 rows the layer streams 109 MB of these weights and the row operands are tiny, so the time
// is HBM time plus whatever stalls the weight stream. With separate launches the stream stops at every kernel
// boundary. Here one CTA per SM runs a fixed list of units (o units, norm rows, gate_up tiles, down units) through
// ONE continuous ring, so the weights of a CTA's next units stream while the phase before finishes. Only the row
// operands wait, each phase on one counter of this layer that the units of the phase before increment: the norm
// rows on the o units, gate_up on the norm rows, down on the gate_up tiles.
//
// Every operand is one contiguous bulk copy per ring stage of two k-blocks: the weights come from packed copies
// (pack.cu, 32 KB per stage), the row operands as row tiles (common.cuh: the attention output written by the
// attention kernel, x by the norm rows, act by the SiLU epilogue). A stage therefore costs the SM's copy engine two
// operations for 32 KB of weights; with 64-k stages and tensor-map boxes it took four, which paced the ring below
// HBM speed.
//
// Warp roles (352 threads): warp 0 issues the weight copies (never waits on another kernel or CTA, only on free ring
// stages), warp 10 issues the row-operand copies (after the previous kernel, or after a phase counter), warp 1
// issues tcgen05.mma into one of two TMEM accumulators, warps 2-9 run the epilogues (the fp32 partial store, SiLU *
// up over all 256 epilogue threads) and the norm rows, so the epilogue of one unit overlaps the MMAs of the next.
// A ring stage completes when both producers' copies have landed (its full barrier expects two arrivals).
//
// Progress: every CTA is resident at once (one CTA per SM, grid = SM count); every CTA runs its units in phase
// order (o, norm, gate_up, down) and a unit only waits for units of earlier phases, so every wait ends. Each wait
// is still bounded (one second); on expiry the kernel records kErrTimeoutFlag / a stage timeout in the device error
// word, every role stops, copies in flight are drained and TMEM is freed.
#include <algorithm>
#include <cstring>
#include <vector>

#include "gemm.cuh"
#include "mlp.h"
#include "runtime.h"

namespace plm {

constexpr int kMlpEpiWarps = 8;                      // warps 2..9: two per TMEM lane slice (column halves)
constexpr int kMlpThreads = (3 + kMlpEpiWarps) * 32;  // + weight producer, MMA issuer, row producer (warp 10)
constexpr int kMlpRowWarp = 2 + kMlpEpiWarps;
constexpr int kMlpStageKb = 2;                        // k-blocks of 64 per ring stage
constexpr int kMlpSmemBudget = 226 * 1024;            // one CTA per SM

template <int NTOK>
struct MlpShape {
  static constexpr int W_BLOCK = 128 * kGemmBK * 2;  // one packed weight block: 128 rows x 64 k
  static constexpr int X_BLOCK = NTOK * kGemmBK * 2;  // one row tile k-block: NTOK rows x 64 k
  static constexpr int W_BYTES = kMlpStageKb * W_BLOCK;
  static constexpr int X_BYTES = kMlpStageKb * X_BLOCK;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int GU_BYTES = 2 * NTOK * 64 * 2;  // gate and up halves of one gate_up tile, model dtype
  static constexpr int STAGES_FIT = (kMlpSmemBudget - GU_BYTES - 1024 - 256) / STAGE;
  static constexpr int STAGES = STAGES_FIT > 8 ? 8 : STAGES_FIT;
  static constexpr int ACC_COLS = (NTOK + 31) / 32 * 32;  // TMEM columns per accumulator (reads are 32 wide)
  static constexpr uint32_t TMEM_COLS = 2 * ACC_COLS <= 64 ? 64 : 2 * ACC_COLS <= 128 ? 128 : 256;
  static constexpr int BAR_OFFSET = STAGES * STAGE + GU_BYTES;
  static constexpr int SMEM = 1024 + BAR_OFFSET + 256;
  static_assert(X_BLOCK % 1024 == 0 && STAGE % 1024 == 0, "operands keep the 1024-byte alignment of the swizzle");
  static_assert(STAGES >= 3, "ring too shallow");
  static_assert((2 * STAGES + 5) * 8 + 28 <= 256, "barrier area");
  static_assert(SMEM <= 227 * 1024, "shared memory");
};

// Unit code: bits 28..29 = kind, bits 12..27 = tile (the row for a norm unit), bits 0..11 = k-split.
enum BlockUnitKind : int { kUnitGate = 0, kUnitDown = 1, kUnitO = 2, kUnitNorm = 3 };
__host__ __device__ constexpr int block_unit(int kind, int tile, int split) {
  return (kind << 28) | (tile << 12) | split;
}

template <typename T, int NTOK>
__device__ __forceinline__ void block_norm_row(const BlockParams& p, int r, int et, float* red, volatile int* abort_flag);

template <typename T, int NTOK>
__global__ void __launch_bounds__(kMlpThreads, 1) mlp_block_kernel(const BlockParams p) {
  using S = MlpShape<NTOK>;
  constexpr uint32_t IDESC = umma_idesc_f16(128, NTOK, std::is_same<T, __nv_bfloat16>::value);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  T* gu = reinterpret_cast<T*>(smem + S::STAGES * S::STAGE);  // [2][NTOK][64]: gate rows, then up rows
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + S::BAR_OFFSET);
  uint64_t* empty_bar = full_bar + S::STAGES;
  uint64_t* acc_full = empty_bar + S::STAGES;  // [2]
  uint64_t* acc_empty = acc_full + 2;          // [2]
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* verdict = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [2] accumulator ready, by unit parity
  int* counts = reinterpret_cast<int*>(tmem_slot + 4);  // stages issued: [0] weights, [1] rows; [2] consumed

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int u_begin = p.sched_off[blockIdx.x], u_end = p.sched_off[blockIdx.x + 1];
  const int gate_kb = p.hidden / kGemmBK, down_kb = p.intermediate / kGemmBK, o_kb = p.q_size / kGemmBK;
  int* const err = p.err;

  if (tid == 0) {
    for (int s = 0; s < S::STAGES; ++s) {
      mbar_init(full_bar + s, 2);  // the weight copy and the row copy
      mbar_init(empty_bar + s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full + b, 1);
      mbar_init(acc_empty + b, kMlpEpiWarps);  // one arrival per epilogue warp
    }
    mbar_init(done_bar, 1);
    *abort_flag = 0;
    counts[0] = 0;
    counts[1] = 0;
    counts[2] = 0;
    fence_barrier_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, S::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  allow_dependents();

  // Bounded wait of lane 0 on an mbarrier phase that also gives up once another role has aborted; the verdict is
  // broadcast to the warp, whose other lanes park in __shfl_sync.
  auto warp_wait = [&](uint64_t* bar, uint32_t parity, int code) -> bool {
    int ok = 1;
    if (lane == 0) {
      if (!mbar_try_wait(bar, parity)) {
        const uint64_t start = global_timer_ns();
        while (true) {
          bool got = false;
          for (int i = 0; i < 64 && !got; ++i) got = mbar_try_wait(bar, parity);
          if (got) break;
          if (*abort_flag) {
            ok = 0;
            break;
          }
          if (global_timer_ns() - start > kWaitLimitNs) {
            record_error(err, code);
            *abort_flag = 1;
            ok = 0;
            break;
          }
        }
      }
    }
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
  };
  // k-block range of a unit, in whole stages (split boundaries fall on even k-blocks). Both producers walk a unit's
  // stages starting at stage (tile % stages) and wrapping around, so that the CTAs that read the same row operand
  // (every gate_up tile reads all of x; the tiles of a down or o split read the same k-blocks) do not request the
  // same k-block at the same moment; the MMA accumulates the stages in arrival order.
  auto unit_range = [&](int code, int& kb0, int& kb1) {
    const int kind = (code >> 28) & 3, split = code & 0xfff;
    if (kind == kUnitGate) {
      kb0 = 0;
      kb1 = gate_kb;
    } else if (kind == kUnitNorm) {
      kb0 = kb1 = 0;
    } else {
      const int pairs = (kind == kUnitDown ? down_kb : o_kb) / kMlpStageKb;
      const int splits = kind == kUnitDown ? p.down_splits : p.o_splits;
      kb0 = kMlpStageKb * (split * pairs / splits);
      kb1 = kMlpStageKb * ((split + 1) * pairs / splits);
    }
  };

  if (warp == 0) {
    // ---------------- weight producer ----------------
    uint64_t pol_w = 0;
    if (lane == 0) pol_w = l2_policy_evict_first();
    int it = 0;
    bool ok = true;
    for (int u = u_begin; u < u_end && ok; ++u) {
      const int code = p.sched[u];
      const int kind = (code >> 28) & 3, tile = (code >> 12) & 0xffff;
      if (kind == kUnitNorm) continue;
      int kb0, kb1;
      unit_range(code, kb0, kb1);
      const uint8_t* wbase = kind == kUnitGate ? p.wg_tiles + size_t(tile) * gate_kb * S::W_BLOCK
                             : kind == kUnitDown ? p.wd_tiles + size_t(tile) * down_kb * S::W_BLOCK
                                                 : p.wo_tiles + size_t(tile) * o_kb * S::W_BLOCK;
      const int n_st = (kb1 - kb0) / kMlpStageKb;
      for (int i = 0; i < n_st; ++i, ++it) {
        const int kb = kb0 + kMlpStageKb * ((i + tile) % n_st);  // rotated k order (see unit_range)
        const int s = it % S::STAGES;
        if (it >= S::STAGES && !warp_wait(empty_bar + s, ((it / S::STAGES) - 1) & 1, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          // two consecutive packed blocks of the tile: the stage's swizzled shared-memory image (pack.cu)
          mbar_arrive_expect_tx(full_bar + s, S::W_BYTES);
          bulk_load(smem + s * S::STAGE, wbase + size_t(kb) * S::W_BLOCK, S::W_BYTES, full_bar + s, pol_w);
          counts[0] = it + 1;
        }
      }
    }
    if (lane == 0 && p.next_weights != nullptr) {
      // This CTA's slice (4 KB aligned) of the weights the next kernel reads first, into L2 in 64 KB prefetches.
      const long long per = ((p.next_bytes / gridDim.x) + 4095) & ~4095LL;
      const long long b0 = per * blockIdx.x;
      const long long n = p.next_bytes - b0 < per ? p.next_bytes - b0 : per;
      for (long long off = 0; off < n; off += 65536)
        bulk_prefetch_l2(p.next_weights + b0 + off, uint32_t(n - off < 65536 ? n - off : 65536));
    }
  } else if (warp == kMlpRowWarp) {
    // ---------------- row-operand producer ----------------
    uint64_t pol_x = 0;
    if (lane == 0) pol_x = l2_policy_evict_last();
    grid_dependency_wait();  // the attention output is written by the previous kernel
    // Waits once for a counter of this grid (norm rows, gate_up tiles). On a timeout the copies are still issued
    // (stale data, error recorded) so that their stages can be drained.
    auto wait_counter = [&](const int* counter, int target) {
      if (lane == 0) {
        if (ld_acquire_gpu(counter) < target) {
          const uint64_t start = global_timer_ns();
          while (ld_acquire_gpu(counter) < target) {
            if (*abort_flag) break;
            if (global_timer_ns() - start > kWaitLimitNs) {
              record_error(err, kErrTimeoutFlag);
              *abort_flag = 1;
              break;
            }
          }
        }
        fence_proxy_async_global();  // the bulk reads below come after the acquire
      }
      __syncwarp();
    };
    int it = 0;
    bool ok = true, x_ready = false, act_ready = false;
    for (int u = u_begin; u < u_end && ok; ++u) {
      const int code = p.sched[u];
      const int kind = (code >> 28) & 3, tile = (code >> 12) & 0xffff;
      if (kind == kUnitNorm) continue;
      if (kind == kUnitGate && !x_ready) {
        wait_counter(p.ctr + 1, p.rows);  // every row normed
        x_ready = true;
      }
      if (kind == kUnitDown && !act_ready) {
        wait_counter(p.ctr + 2, p.intermediate / 64);  // every gate_up tile stored
        act_ready = true;
      }
      int kb0, kb1;
      unit_range(code, kb0, kb1);
      const uint8_t* rows_src = kind == kUnitGate ? p.x_tiles : kind == kUnitDown ? p.act_tiles : p.attn_tiles;
      const int n_st = (kb1 - kb0) / kMlpStageKb;
      for (int i = 0; i < n_st; ++i, ++it) {
        const int kb = kb0 + kMlpStageKb * ((i + tile) % n_st);  // rotated k order (see unit_range)
        const int s = it % S::STAGES;
        if (it >= S::STAGES && !warp_wait(empty_bar + s, ((it / S::STAGES) - 1) & 1, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(full_bar + s, S::X_BYTES);
          bulk_load(smem + s * S::STAGE + S::W_BYTES, rows_src + size_t(kb) * S::X_BLOCK, S::X_BYTES, full_bar + s,
                    pol_x);
          counts[1] = it + 1;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    int it = 0, n = 0;
    bool ok = true;
    for (int u = u_begin; u < u_end && ok; ++u) {
      const int code = p.sched[u];
      if (((code >> 28) & 3) == kUnitNorm) continue;
      int kb0, kb1;
      unit_range(code, kb0, kb1);
      const int buf = n & 1;
      if (n >= 2 && !warp_wait(acc_empty + buf, ((n >> 1) - 1) & 1, kErrTimeoutDone)) break;
      tc_fence_after();
      const uint32_t d_tmem = tmem + uint32_t(buf * S::ACC_COLS);
      for (int kb = kb0; kb < kb1; kb += kMlpStageKb, ++it) {  // stage order does not matter here
        const int s = it % S::STAGES;
        if (!warp_wait(full_bar + s, (it / S::STAGES) & 1, kErrTimeoutFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + s * S::STAGE);
          const uint32_t b_addr = a_addr + S::W_BYTES;
#pragma unroll
          for (int kk = 0; kk < kMlpStageKb * (kGemmBK / 16); ++kk) {
            const uint32_t a_k = a_addr + (kk >> 2) * S::W_BLOCK + (kk & 3) * 32;
            const uint32_t b_k = b_addr + (kk >> 2) * S::X_BLOCK + (kk & 3) * 32;
            umma_f16(d_tmem, umma_desc_sw128(a_k), umma_desc_sw128(b_k), IDESC, (kb > kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(empty_bar + s);
          counts[2] = it + 1;
        }
        __syncwarp();
      }
      if (!ok) break;
      if (lane == 0) umma_commit(acc_full + buf);
      __syncwarp();
      ++n;
    }
    if (lane == 0) umma_commit(done_bar);  // arrives once every MMA issued above has completed
    __syncwarp();
  } else if (warp < kMlpRowWarp) {
    // ---------------- epilogue warps 2..9 ----------------
    // Warp w reads TMEM lane slice w % 4 (features slice*32 .. +31 of the tile) for the column (row) blocks
    // half*32, half*32 + 64, ... with half = (w - 2) / 4, so the eight warps cover the accumulator once.
    grid_dependency_wait();  // the outputs may still be read by earlier kernels of the stream
    const int et = tid - 64;            // 0..255
    const int slice = warp & 3;
    const int half = (warp - 2) >> 2;
    const int feat = slice * 32 + lane;
    const int rows = p.rows, hidden = p.hidden;
    int n = 0;  // MMA units seen (the TMEM buffer parity)
    for (int u = u_begin; u < u_end; ++u) {
      const int code = p.sched[u];
      const int kind = (code >> 28) & 3, tile = (code >> 12) & 0xffff, split = code & 0xfff;
      if (kind == kUnitNorm) {
        if (tile < rows) block_norm_row<T, NTOK>(p, tile, et, reinterpret_cast<float*>(gu), abort_flag);
        continue;
      }
      const int buf = n & 1;
      // One warp waits for the accumulator and publishes the verdict, so that all epilogue warps take the same
      // path through the named barriers below.
      if (warp == 2) {
        const bool ready = warp_wait(acc_full + buf, (n >> 1) & 1, kErrTimeoutDone);
        if (lane == 0) verdict[n & 1] = ready ? 1 : 0;
      }
      named_barrier_sync(1, kMlpEpiWarps * 32);
      if (verdict[n & 1] == 0) break;
      tc_fence_after();
      const uint32_t t_acc = tmem + (uint32_t(slice * 32) << 16) + uint32_t(buf * S::ACC_COLS);
      if (kind != kUnitGate) {  // o or down: the fp32 partial of this k-split
        float* part = p.partials + size_t(split) * rows * hidden;
        const int f = tile * 128 + feat;
        for (int c0 = half * 32; c0 < rows; c0 += 64) {
          float v[32];
          tmem_ld_32cols(t_acc + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < rows && f < hidden) part[size_t(c0 + j) * hidden + f] = v[j];
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + buf);
        if (kind == kUnitO) {  // the norm rows wait for every o partial
          named_barrier_sync(3, kMlpEpiWarps * 32);
          if (et == 0) signal_stored(p.ctr + 0);
        }
      } else {
        // TMEM lanes 0..63 are the gate rows, 64..127 the up rows of the same 64 intermediate features: each warp
        // stages its values (rounded to the model dtype, as the separate launch does) ...
        T* dst_stage = gu + (slice >= 2 ? NTOK * 64 : 0);
        const int f64 = feat & 63;
        for (int c0 = half * 32; c0 < rows; c0 += 64) {
          float v[32];
          tmem_ld_32cols(t_acc + c0, v);
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < rows) dst_stage[(c0 + j) * 64 + f64] = from_f32<T>(v[j]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(acc_empty + buf);
        named_barrier_sync(2, kMlpEpiWarps * 32);  // gate and up staged
        // ... then all 256 threads form SiLU(gate) * up, eight features (one 16-byte chunk of the act row tile)
        // per thread and step.
        uint4* act_chunks = reinterpret_cast<uint4*>(p.act_tiles);
        for (int idx = et; idx < rows * 8; idx += kMlpEpiWarps * 32) {
          const int r = idx >> 3, c = idx & 7;
          const uint4 gv = *reinterpret_cast<const uint4*>(gu + r * 64 + c * 8);
          const uint4 uv = *reinterpret_cast<const uint4*>(gu + NTOK * 64 + r * 64 + c * 8);
          const T* g8 = reinterpret_cast<const T*>(&gv);
          const T* u8 = reinterpret_cast<const T*>(&uv);
          uint4 out;
          T* o8 = reinterpret_cast<T*>(&out);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const float g = to_f32<T>(g8[q]);
            o8[q] = from_f32<T>(g / (1.0f + expf(-g)) * to_f32<T>(u8[q]));
          }
          act_chunks[row_tile_chunk(tile, r, c, NTOK)] = out;
        }
        named_barrier_sync(3, kMlpEpiWarps * 32);  // every feature of the tile is stored
        if (et == 0) signal_stored(p.ctr + 2);
      }
      ++n;
    }
  }

  // ---------------- teardown ----------------
  __syncthreads();
  if (tid == 0) {
    // Every MMA this CTA issued has completed (and, after an abort, every copy in flight has landed) before shared
    // memory and TMEM are released.
    mbar_wait(done_bar, 0, err, kErrTimeoutDone);
    if (*abort_flag) {
      // A stage one producer issued and the other did not gets the missing arrival (no bytes) so that its phase
      // completes once the copy that was issued has landed.
      const int issued = max(counts[0], counts[1]);
      for (int i = counts[2]; i < issued; ++i) {
        if ((i < counts[0]) != (i < counts[1])) mbar_arrive(full_bar + (i % S::STAGES));
        if (!mbar_wait(full_bar + (i % S::STAGES), (i / S::STAGES) & 1, err, kErrTimeoutFull)) break;
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, S::TMEM_COLS);
  }
}

// One row of the residual-add RMSNorm after the o projection (the arithmetic of add_norm_kernel in
// elementwise.cu, vLLM fused_add_rms_norm): x = the o partials summed in split order and rounded to bf16,
// v = x + residual in fp32, residual <- bf16(v), normed = bf16(bf16(v * rstd) * w), written as row tiles for the
// gate_up units. Run by the 256 epilogue threads once every o unit of the grid has signalled.
template <typename T, int NTOK>
__device__ __forceinline__ void block_norm_row(const BlockParams& p, int r, int et, float* red,
                                               volatile int* abort_flag) {
  constexpr int kThreads = kMlpEpiWarps * 32;
  constexpr int kMaxChunks = 2;  // hidden <= 8 * 256 * 2
  // The norm weight is never written: loaded before the wait for the o partials, so that no load follows the row's
  // barrier.
  uint4 wv[kMaxChunks];
#pragma unroll
  for (int j = 0; j < kMaxChunks; ++j) {
    const int c = et + j * kThreads;
    if (c < p.hidden / 8) wv[j] = reinterpret_cast<const uint4*>(p.norm_weight)[c];
  }
  if (et == 0) {
    const int target = p.o_units;
    if (ld_acquire_gpu(p.ctr + 0) < target) {
      const uint64_t start = global_timer_ns();
      while (ld_acquire_gpu(p.ctr + 0) < target) {
        if (*abort_flag) break;
        if (global_timer_ns() - start > kWaitLimitNs) {
          record_error(p.err, kErrTimeoutFlag);
          *abort_flag = 1;
          break;
        }
      }
    }
  }
  named_barrier_sync(4, kThreads);  // the partials of every o unit are visible from here on
  const int chunks = p.hidden / 8;
  T* res = reinterpret_cast<T*>(p.residual) + size_t(r) * p.hidden;
  float v[kMaxChunks][8];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxChunks; ++j) {
    const int c = et + j * kThreads;
    if (c >= chunks) continue;
    // The loads of kBatch splits are issued before they are summed (in split order from 0): one L2 round trip per
    // batch instead of one per split.
    const uint4 rv = reinterpret_cast<const uint4*>(res)[c];
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    constexpr int kBatch = 10;
    for (int sp0 = 0; sp0 < p.o_splits; sp0 += kBatch) {
      float4 lo[kBatch], hi[kBatch];
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (sp0 + b < p.o_splits) {
          const float4* src =
              reinterpret_cast<const float4*>(p.partials + (size_t(sp0 + b) * p.rows + r) * p.hidden) + 2 * c;
          lo[b] = src[0];
          hi[b] = src[1];
        }
      }
#pragma unroll
      for (int b = 0; b < kBatch; ++b) {
        if (sp0 + b < p.o_splits) {
          acc[0] += lo[b].x;
          acc[1] += lo[b].y;
          acc[2] += lo[b].z;
          acc[3] += lo[b].w;
          acc[4] += hi[b].x;
          acc[5] += hi[b].y;
          acc[6] += hi[b].z;
          acc[7] += hi[b].w;
        }
      }
    }
    const T* r8 = reinterpret_cast<const T*>(&rv);
    uint4 nr;
    T* n8 = reinterpret_cast<T*>(&nr);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      v[j][q] = round_to<T>(acc[q]) + to_f32<T>(r8[q]);
      n8[q] = from_f32<T>(v[j][q]);
      ss += v[j][q] * v[j][q];
    }
    reinterpret_cast<uint4*>(res)[c] = nr;
  }
  ss = warp_sum(ss);
  if ((et & 31) == 0) red[et >> 5] = ss;
  named_barrier_sync(5, kThreads);
  float total = 0.f;
#pragma unroll
  for (int i = 0; i < kMlpEpiWarps; ++i) total += red[i];
  const float rstd = rsqrtf(total / float(p.hidden) + p.eps);
  uint4* tiles = reinterpret_cast<uint4*>(p.x_tiles);
#pragma unroll
  for (int j = 0; j < kMaxChunks; ++j) {
    const int c = et + j * kThreads;
    if (c >= chunks) continue;
    const T* w8 = reinterpret_cast<const T*>(&wv[j]);
    uint4 o;
    T* o8 = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int q = 0; q < 8; ++q) o8[q] = from_f32<T>(round_to<T>(v[j][q] * rstd) * to_f32<T>(w8[q]));
    tiles[row_tile_chunk(c >> 3, r, c & 7, NTOK)] = o;
  }
  named_barrier_sync(6, kThreads);  // the row is stored (and red[] may be reused)
  if (et == 0) signal_stored(p.ctr + 1);
}

// ------------------------------------------------------------------------------------------------------------------
// Host side.

std::vector<int> mlp_schedule_units(const MlpSchedule& s, int hidden, int intermediate, int q_size,
                                    std::vector<int>* offsets) {
  // Phase by phase, in the order every CTA runs them:
  //   o units: unit j on CTA grid - 1 - (j % grid), so the CTAs without a gate_up tile take them first;
  //   norm rows: row r on CTA (gate_tiles + r) % grid, so the rows every forward has (the low ones) start on the
  //     CTAs without a gate_up tile;
  //   gate_up tiles: tile t on the CTA with the fewest gate k-blocks (CTA t when there are at most grid tiles);
  //   down units: they load their act operand only once every gate_up tile is stored, so they are balanced on
  //     their own: each goes to the CTA with the fewest down k-blocks, then less gate work, then the lowest index.
  const int grid = s.grid;
  std::vector<std::vector<int>> lists(grid);
  const int o_units = s.o_tiles * s.o_splits;
  for (int j = 0; j < o_units; ++j)
    lists[grid - 1 - (j % grid)].push_back(block_unit(kUnitO, j % s.o_tiles, j / s.o_tiles));
  for (int r = 0; r < kMlpMaxRows; ++r) lists[(s.gate_tiles + r) % grid].push_back(block_unit(kUnitNorm, r, 0));
  std::vector<long> gate_load(grid, 0), down_load(grid, 0);
  const int gate_kb = hidden / kGemmBK, down_kb = intermediate / kGemmBK;
  for (int t = 0; t < s.gate_tiles; ++t) {
    int c = 0;
    for (int i = 1; i < grid; ++i)
      if (gate_load[i] < gate_load[c]) c = i;
    lists[c].push_back(block_unit(kUnitGate, t, 0));
    gate_load[c] += gate_kb;
  }
  const int pairs = down_kb / kMlpStageKb;  // as unit_range in the kernel
  for (int sp = 0; sp < s.down_splits; ++sp) {
    const int kb = kMlpStageKb * ((sp + 1) * pairs / s.down_splits - sp * pairs / s.down_splits);
    for (int t = 0; t < s.down_tiles; ++t) {
      int c = 0;
      for (int i = 1; i < grid; ++i)
        if (down_load[i] < down_load[c] || (down_load[i] == down_load[c] && gate_load[i] < gate_load[c])) c = i;
      lists[c].push_back(block_unit(kUnitDown, t, sp));
      down_load[c] += kb;
    }
  }
  (void)q_size;
  std::vector<int> flat;
  offsets->assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    flat.insert(flat.end(), lists[c].begin(), lists[c].end());
    offsets->push_back(int(flat.size()));
  }
  return flat;
}

int mlp_schedule_plan(int num_sms, int hidden, int intermediate, int q_size, MlpSchedule* out) {
  *out = MlpSchedule{};
  constexpr int kPair = kMlpStageKb * kGemmBK;
  if (num_sms < 1 || hidden < kPair || intermediate < kPair || q_size < kPair || hidden % kPair != 0 ||
      intermediate % kPair != 0 || q_size % kPair != 0 || hidden > 8 * 256 * 2 || intermediate / 64 >= (1 << 16))
    return fail(PLM_ERR_UNSUPPORTED, "layer block: %d SMs, hidden %d, intermediate %d, q_size %d", num_sms, hidden,
                intermediate, q_size);
  out->grid = num_sms;
  out->gate_tiles = intermediate / 64;
  out->down_tiles = (hidden + 127) / 128;
  out->down_splits = std::min(kMlpMaxDownSplits, intermediate / kPair);
  out->o_tiles = (hidden + 127) / 128;
  out->o_splits = std::max(1, std::min({kMlpMaxOSplits, q_size / kPair, num_sms / out->o_tiles}));
  return PLM_OK;
}

int mlp_schedule_create(int num_sms, int hidden, int intermediate, int q_size, MlpSchedule* out) {
  MlpSchedule s;
  int plan = mlp_schedule_plan(num_sms, hidden, intermediate, q_size, &s);
  *out = MlpSchedule{};
  if (plan != PLM_OK) return plan;
  std::vector<int> offsets;
  std::vector<int> units = mlp_schedule_units(s, hidden, intermediate, q_size, &offsets);
  int st = check_cuda(cudaMalloc(&s.sched, units.size() * sizeof(int)), "block schedule");
  if (st == PLM_OK) st = check_cuda(cudaMalloc(&s.sched_off, offsets.size() * sizeof(int)), "block schedule");
  if (st == PLM_OK)
    st = check_cuda(cudaMemcpy(s.sched, units.data(), units.size() * sizeof(int), cudaMemcpyHostToDevice),
                    "block schedule upload");
  if (st == PLM_OK)
    st = check_cuda(cudaMemcpy(s.sched_off, offsets.data(), offsets.size() * sizeof(int), cudaMemcpyHostToDevice),
                    "block schedule upload");
  if (st != PLM_OK) {
    mlp_schedule_destroy(&s);
    return st;
  }
  *out = s;
  return PLM_OK;
}

void mlp_schedule_destroy(MlpSchedule* s) {
  if (s->sched) cudaFree(s->sched);
  if (s->sched_off) cudaFree(s->sched_off);
  *s = MlpSchedule{};
}

namespace {

template <typename T, int NTOK>
int launch_block(const MlpSchedule& s, const BlockParams& p, cudaStream_t stream, bool pdl) {
  using S = MlpShape<NTOK>;
  auto kernel = mlp_block_kernel<T, NTOK>;
  int st = raise_smem_limit(reinterpret_cast<const void*>(kernel), S::SMEM, "cudaFuncSetAttribute(block smem)");
  if (st != PLM_OK) return st;
  int per_sm = 0;
  st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kMlpThreads, S::SMEM),
                  "block occupancy");
  if (st != PLM_OK) return st;
  if (per_sm < 1) return fail(PLM_ERR_UNSUPPORTED, "layer block: %d bytes of shared memory do not fit", S::SMEM);
  return check_cuda(launch(kernel, dim3(s.grid), dim3(kMlpThreads), S::SMEM, stream, pdl, p),
                    "mlp_block_kernel launch");
}

}  // namespace

template <typename T>
int launch_block_rows(const MlpSchedule& s, const BlockParams& p, cudaStream_t stream, bool pdl) {
  switch (gemm_token_tile(p.rows)) {  // the row tiles' height
    case 16: return launch_block<T, 16>(s, p, stream, pdl);
    case 32: return launch_block<T, 32>(s, p, stream, pdl);
    case 48: return launch_block<T, 48>(s, p, stream, pdl);
    case 64: return launch_block<T, 64>(s, p, stream, pdl);
    case 80: return launch_block<T, 80>(s, p, stream, pdl);
    case 96: return launch_block<T, 96>(s, p, stream, pdl);
    case 112: return launch_block<T, 112>(s, p, stream, pdl);
    case 128: return launch_block<T, 128>(s, p, stream, pdl);
  }
  return fail(PLM_ERR_UNSUPPORTED, "layer block: %d rows", p.rows);
}

int mlp_block_launch(const MlpSchedule& s, BlockParams p, int dtype, cudaStream_t stream, bool pdl) {
  if (dtype != PLM_BF16 && dtype != PLM_F16) return fail(PLM_ERR_INVALID, "layer block: dtype %d", dtype);
  if (s.sched == nullptr || s.grid < 1) return fail(PLM_ERR_INVALID, "layer block: no schedule");
  if (p.rows < 1 || p.rows > kMlpMaxRows) return fail(PLM_ERR_UNSUPPORTED, "layer block: %d rows", p.rows);
  if ((p.hidden + 127) / 128 != s.down_tiles || p.intermediate / 64 != s.gate_tiles)
    return fail(PLM_ERR_INVALID, "layer block: shape differs from its schedule");
  if (!p.wo_tiles || !p.wg_tiles || !p.wd_tiles || !p.attn_tiles || !p.x_tiles || !p.act_tiles || !p.partials ||
      !p.residual || !p.norm_weight || !p.ctr)
    return fail(PLM_ERR_INVALID, "layer block: null operand");
  p.sched = s.sched;
  p.sched_off = s.sched_off;
  p.o_splits = s.o_splits;
  p.down_splits = s.down_splits;
  p.o_units = s.o_tiles * s.o_splits;
  return dtype == PLM_F16 ? launch_block_rows<__half>(s, p, stream, pdl)
                          : launch_block_rows<__nv_bfloat16>(s, p, stream, pdl);
}

}  // namespace plm

using namespace plm;

extern "C" int plm_block_schedule(int32_t num_sms, int32_t hidden, int32_t intermediate, int32_t q_size,
                                  int32_t* units, int32_t capacity, int32_t* offsets, int32_t* n_units) {
  if (!offsets || !n_units || (capacity > 0 && !units))
    return fail(PLM_ERR_INVALID, "plm_block_schedule: null argument");
  MlpSchedule s;
  int st = mlp_schedule_plan(num_sms, hidden, intermediate, q_size, &s);
  if (st != PLM_OK) return st;
  std::vector<int> off;
  const std::vector<int> flat = mlp_schedule_units(s, hidden, intermediate, q_size, &off);
  *n_units = int32_t(flat.size());
  if (capacity < int32_t(flat.size()))
    return fail(PLM_ERR_INVALID, "plm_block_schedule: %zu units, capacity %d", flat.size(), capacity);
  std::copy(flat.begin(), flat.end(), units);
  std::copy(off.begin(), off.end(), offsets);
  return PLM_OK;
}
