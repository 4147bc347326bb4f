// The Llama MLP block of one forward as ONE persistent launch:
//   act = SiLU(x . Wg^T) * (x . Wu^T)            (vLLM LlamaMLP: gate_up_proj -> SiluAndMul)
//   partials[s] = act[:, K_s] . Wd[:, K_s]^T      (down_proj, fp32 k-split partials)
// The products are the ones the two skinny_gemm_kernel launches it replaces compute (gemm.cuh, epilogues
// kEpiSiluMul and kEpiPartial); a gate_up tile is accumulated by one CTA over the whole k range instead of a
// cluster of k-splits, so fp32 sums are formed in another order.
//
// Why one launch: at 56 rows the block streams 101 MB of weights per layer and the row operands are tiny, so the
// time is HBM time plus whatever stalls the weight stream. With two launches the stream stops at the boundary:
// the down launch can start loading only when the gate_up grid has drained. Here one CTA per SM runs a fixed list
// of units (its gate_up tiles, then down (tile, k-split) units) through ONE continuous ring, so the weights of its
// down units stream while the gate_up phase finishes. Only the act operand of the down units waits: on one counter
// per layer that every gate_up tile increments once stored (by whichever CTA computed it).
//
// Every operand is one contiguous bulk copy per ring stage of two k-blocks: the weights come from packed copies
// (pack.cu, 32 KB per stage), x and act as row tiles (common.cuh: x written by the residual-add RMSNorm before this
// kernel, act by this kernel's SiLU epilogue). A stage therefore costs the SM's copy engine two operations for
// 32 KB of weights; with 64-k stages and tensor-map boxes it took four, which paced the ring below HBM speed.
//
// Warp roles (352 threads): warp 0 issues the weight copies (never waits on another kernel or CTA, only on free ring
// stages), warp 10 issues the row-operand copies (x after the previous kernel, act after the gate_up counter),
// warp 1 issues tcgen05.mma into one of two TMEM accumulators, warps 2-9 drain the other accumulator (SiLU * up
// over all 256 epilogue threads, or the fp32 partial store), so the epilogue of one unit overlaps the MMAs of the
// next. A ring stage completes when both producers' copies have landed (its full barrier expects two arrivals).
//
// Progress: every CTA is resident at once (one CTA per SM, grid = SM count), gate_up units wait on nothing but the
// previous kernel, and down units wait only on gate_up tiles, so every wait ends. Each wait is still bounded (one
// second); on expiry the kernel records kErrTimeoutFlag / a stage timeout in the device error word, every role
// stops, copies in flight are drained and TMEM is freed.
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

// Unit code: bit 30 = down (else gate_up), bits 12..29 = tile, bits 0..11 = k-split.
__host__ __device__ constexpr int mlp_unit(int down, int tile, int split) {
  return (down << 30) | (tile << 12) | split;
}

template <typename T, int NTOK>
__global__ void __launch_bounds__(kMlpThreads, 1)
    mlp_block_kernel(const uint8_t* __restrict__ wg_tiles, const uint8_t* __restrict__ x_tiles,
                     const uint8_t* __restrict__ wd_tiles, uint8_t* __restrict__ act_tiles,
                     const int* __restrict__ sched, const int* __restrict__ sched_off, float* __restrict__ partials,
                     int* gate_done, const int* epoch, int rows, int hidden, int intermediate, int down_splits,
                     int* err) {
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
  const int u_begin = sched_off[blockIdx.x], u_end = sched_off[blockIdx.x + 1];
  const int gate_kb = hidden / kGemmBK, down_kb = intermediate / kGemmBK;

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
  // (every gate_up tile reads all of x; the 16 tiles of a down split read the same act k-blocks) do not request
  // the same k-block at the same moment; the MMA accumulates the stages in arrival order.
  auto unit_range = [&](int code, int& kb0, int& kb1) {
    if (code >> 30) {
      const int split = code & 0xfff, pairs = down_kb / kMlpStageKb;
      kb0 = kMlpStageKb * (split * pairs / down_splits);
      kb1 = kMlpStageKb * ((split + 1) * pairs / down_splits);
    } else {
      kb0 = 0;
      kb1 = gate_kb;
    }
  };

  if (warp == 0) {
    // ---------------- weight producer ----------------
    uint64_t pol_w = 0;
    if (lane == 0) pol_w = l2_policy_evict_first();
    int it = 0;
    bool ok = true;
    for (int u = u_begin; u < u_end && ok; ++u) {
      const int code = sched[u];
      const bool down = (code >> 30) != 0;
      const int tile = (code >> 12) & 0x3ffff;
      int kb0, kb1;
      unit_range(code, kb0, kb1);
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
          const uint8_t* src = down ? wd_tiles + (size_t(tile) * down_kb + kb) * S::W_BLOCK
                                    : wg_tiles + (size_t(tile) * gate_kb + kb) * S::W_BLOCK;
          mbar_arrive_expect_tx(full_bar + s, S::W_BYTES);
          bulk_load(smem + s * S::STAGE, src, S::W_BYTES, full_bar + s, pol_w);
          counts[0] = it + 1;
        }
      }
    }
  } else if (warp == kMlpRowWarp) {
    // ---------------- row-operand producer ----------------
    uint64_t pol_x = 0;
    if (lane == 0) pol_x = l2_policy_evict_last();
    grid_dependency_wait();  // x and the epoch are written by earlier kernels of the stream
    int it = 0;
    bool ok = true, act_ready = false;
    for (int u = u_begin; u < u_end && ok; ++u) {
      const int code = sched[u];
      const bool down = (code >> 30) != 0;
      const int tile = (code >> 12) & 0x3ffff;
      int kb0, kb1;
      unit_range(code, kb0, kb1);
      if (down && !act_ready) {
        // Every gate_up tile of this forward is stored once the layer's counter reaches epoch * tiles. On a
        // timeout the copies are still issued (stale data, error recorded) so that their stages can be drained.
        if (lane == 0) {
          const int target = *reinterpret_cast<const volatile int*>(epoch) * (intermediate / 64);
          if (ld_acquire_gpu(gate_done) < target) {
            const uint64_t start = global_timer_ns();
            while (ld_acquire_gpu(gate_done) < target) {
              if (*abort_flag) break;
              if (global_timer_ns() - start > kWaitLimitNs) {
                record_error(err, kErrTimeoutFlag);
                *abort_flag = 1;
                break;
              }
            }
          }
          fence_proxy_async_global();  // the bulk reads of act below come after the acquire
        }
        __syncwarp();
        act_ready = true;
      }
      const uint8_t* rows_src = down ? act_tiles : x_tiles;
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
    for (int u = u_begin; u < u_end && ok; ++u, ++n) {
      int kb0, kb1;
      unit_range(sched[u], kb0, kb1);
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
    }
    if (lane == 0) umma_commit(done_bar);  // arrives once every MMA issued above has completed
    __syncwarp();
  } else if (warp < kMlpRowWarp) {
    // ---------------- epilogue warps 2..9 ----------------
    // Warp w reads TMEM lane slice w % 4 (features slice*32 .. +31 of the tile) for the column (row) blocks
    // half*32, half*32 + 64, ... with half = (w - 2) / 4, so the eight warps cover the accumulator once.
    grid_dependency_wait();  // act and the partials may still be read by earlier kernels of the stream
    const int et = tid - 64;            // 0..255
    const int slice = warp & 3;
    const int half = (warp - 2) >> 2;
    const int feat = slice * 32 + lane;
    int n = 0;
    for (int u = u_begin; u < u_end; ++u, ++n) {
      const int code = sched[u];
      const bool down = (code >> 30) != 0;
      const int tile = (code >> 12) & 0x3ffff, split = code & 0xfff;
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
      if (down) {
        float* part = partials + size_t(split) * rows * hidden;
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
        uint4* act_chunks = reinterpret_cast<uint4*>(act_tiles);
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
        __threadfence();
        named_barrier_sync(3, kMlpEpiWarps * 32);  // every feature of the tile is stored
        if (et == 0) red_release_gpu_add(gate_done, 1);
      }
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

// ------------------------------------------------------------------------------------------------------------------
// Host side.

std::vector<int> mlp_schedule_units(int grid, int gate_tiles, int gate_kb, int down_tiles, int down_splits,
                                    int down_kb, std::vector<int>* offsets) {
  // Gate_up tiles go to the CTAs with the fewest gate k-blocks so far. The down units can only load their act
  // operand once every gate_up tile is stored, so they are balanced on their own: each goes to the CTA with the
  // fewest down k-blocks so far, preferring CTAs with less gate work, then the lowest index (deterministic).
  // Within a CTA its gate_up units precede its down units.
  std::vector<std::vector<int>> lists(grid);
  std::vector<long> gate_load(grid, 0), down_load(grid, 0);
  auto least = [&](bool down) {
    int best = 0;
    for (int c = 1; c < grid; ++c) {
      const bool better = down ? (down_load[c] < down_load[best] ||
                                  (down_load[c] == down_load[best] && gate_load[c] < gate_load[best]))
                               : gate_load[c] < gate_load[best];
      if (better) best = c;
    }
    return best;
  };
  for (int t = 0; t < gate_tiles; ++t) {
    const int c = least(false);
    lists[c].push_back(mlp_unit(0, t, 0));
    gate_load[c] += gate_kb;
  }
  for (int sp = 0; sp < down_splits; ++sp) {
    const int pairs = down_kb / kMlpStageKb;  // as unit_range in the kernel
    const int kb = kMlpStageKb * ((sp + 1) * pairs / down_splits - sp * pairs / down_splits);
    for (int t = 0; t < down_tiles; ++t) {
      const int c = least(true);
      lists[c].push_back(mlp_unit(1, t, sp));
      down_load[c] += kb;
    }
  }
  std::vector<int> flat;
  offsets->assign(1, 0);
  for (int c = 0; c < grid; ++c) {
    flat.insert(flat.end(), lists[c].begin(), lists[c].end());
    offsets->push_back(int(flat.size()));
  }
  return flat;
}

int mlp_schedule_create(int num_sms, int hidden, int intermediate, MlpSchedule* out) {
  *out = MlpSchedule{};
  if (hidden % (kMlpStageKb * kGemmBK) != 0 || intermediate % (kMlpStageKb * kGemmBK) != 0 ||
      intermediate / 64 >= (1 << 18))
    return fail(PLM_ERR_UNSUPPORTED, "mlp block: hidden %d, intermediate %d (multiples of 128)", hidden, intermediate);
  MlpSchedule s;
  s.grid = num_sms;
  s.gate_tiles = intermediate / 64;
  s.down_tiles = (hidden + 127) / 128;
  s.down_splits = std::min(kMlpMaxDownSplits, intermediate / (kMlpStageKb * kGemmBK));
  std::vector<int> offsets;
  std::vector<int> units = mlp_schedule_units(s.grid, s.gate_tiles, hidden / kGemmBK, s.down_tiles, s.down_splits,
                                              intermediate / kGemmBK, &offsets);
  int st = check_cuda(cudaMalloc(&s.sched, units.size() * sizeof(int)), "mlp schedule");
  if (st == PLM_OK) st = check_cuda(cudaMalloc(&s.sched_off, offsets.size() * sizeof(int)), "mlp schedule");
  if (st == PLM_OK)
    st = check_cuda(cudaMemcpy(s.sched, units.data(), units.size() * sizeof(int), cudaMemcpyHostToDevice),
                    "mlp schedule upload");
  if (st == PLM_OK)
    st = check_cuda(cudaMemcpy(s.sched_off, offsets.data(), offsets.size() * sizeof(int), cudaMemcpyHostToDevice),
                    "mlp schedule upload");
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
int launch_block(const MlpSchedule& s, const MlpBlockArgs& a, cudaStream_t stream, bool pdl) {
  using S = MlpShape<NTOK>;
  auto kernel = mlp_block_kernel<T, NTOK>;
  static bool attr_set = false;
  if (!attr_set) {
    int st = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::SMEM),
                        "cudaFuncSetAttribute(mlp block smem)");
    if (st != PLM_OK) return st;
    int per_sm = 0;
    st = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kMlpThreads, S::SMEM),
                    "mlp block occupancy");
    if (st != PLM_OK) return st;
    if (per_sm < 1) return fail(PLM_ERR_UNSUPPORTED, "mlp block: %d bytes of shared memory do not fit", S::SMEM);
    attr_set = true;
  }
  return check_cuda(launch(kernel, dim3(s.grid), dim3(kMlpThreads), S::SMEM, stream, pdl,
                           static_cast<const uint8_t*>(a.gate_up_tiles), static_cast<const uint8_t*>(a.x_tiles),
                           static_cast<const uint8_t*>(a.down_tiles), static_cast<uint8_t*>(a.act_tiles),
                           (const int*)s.sched, (const int*)s.sched_off,
                           a.partials, a.gate_done, a.epoch, a.rows, a.hidden,
                           a.intermediate, s.down_splits, a.err),
                    "mlp_block_kernel launch");
}

}  // namespace

int mlp_block_launch(const MlpSchedule& s, const MlpBlockArgs& a, cudaStream_t stream, bool pdl) {
  if (a.dtype != PLM_BF16) return fail(PLM_ERR_UNSUPPORTED, "mlp block: only bf16 is built");
  if (s.sched == nullptr || s.grid < 1) return fail(PLM_ERR_INVALID, "mlp block: no schedule");
  if (a.rows < 1 || a.rows > kMlpMaxRows) return fail(PLM_ERR_UNSUPPORTED, "mlp block: %d rows", a.rows);
  if (a.hidden / 128 > s.down_tiles || a.intermediate / 64 != s.gate_tiles)
    return fail(PLM_ERR_INVALID, "mlp block: shape differs from its schedule");
  if (!a.act_tiles || !a.partials || !a.gate_done || !a.epoch || !a.gate_up_tiles || !a.down_tiles || !a.x_tiles)
    return fail(PLM_ERR_INVALID, "mlp block: null operand");
  switch (gemm_token_tile(a.rows)) {  // the row maps' box height
    case 16: return launch_block<__nv_bfloat16, 16>(s, a, stream, pdl);
    case 32: return launch_block<__nv_bfloat16, 32>(s, a, stream, pdl);
    case 48: return launch_block<__nv_bfloat16, 48>(s, a, stream, pdl);
    case 64: return launch_block<__nv_bfloat16, 64>(s, a, stream, pdl);
    case 80: return launch_block<__nv_bfloat16, 80>(s, a, stream, pdl);
    case 96: return launch_block<__nv_bfloat16, 96>(s, a, stream, pdl);
    case 112: return launch_block<__nv_bfloat16, 112>(s, a, stream, pdl);
    case 128: return launch_block<__nv_bfloat16, 128>(s, a, stream, pdl);
  }
  return fail(PLM_ERR_UNSUPPORTED, "mlp block: %d rows", a.rows);
}

}  // namespace plm
