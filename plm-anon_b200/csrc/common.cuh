// Shared device helpers for the PLM round kernels (sm_100a only).
//
// Everything here is a thin wrapper over one PTX instruction: mbarriers, TMA tensor loads (never with
// cluster multicast), tcgen05 (TMEM allocation, MMA, commit, loads), programmatic dependent launch and the
// bounded waits every spin in this library goes through. A wait that runs out of time records an error
// code in the caller's device error word and returns false; nothing here traps or spins forever.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace plm {

// Error codes written to the device error word (first writer wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,      // MMA issuer waited too long for a TMA stage
  kErrTimeoutEmpty = 2,     // TMA producer waited too long for a free stage
  kErrTimeoutDone = 3,      // epilogue waited too long for the MMA chain
  kErrBadIndex = 4,         // an index (page, slot, token, aux cell) out of range was skipped
  kErrTimeoutSplit = 5,     // split reduction saw an inconsistent arrival count
  kErrBadShape = 6,         // a kernel was launched with a shape it cannot handle
  kErrTimeoutPeer = 7,      // a cluster peer's st.async data did not arrive
  kErrTimeoutFlag = 8,      // an operand another CTA of the grid produces was not signalled in time
};

// One second: far above any legitimate wait in a round (a whole round takes about a millisecond).
constexpr uint64_t kWaitLimitNs = 1000000000ull;

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------------------------------------------
// Programmatic dependent launch. Kernels launched with the programmatic-serialisation attribute may start while
// their predecessor is still running; `grid_dependency_wait` blocks until every predecessor has completed and its
// memory is visible. Only reads of data that no kernel of the stream writes (weights) may precede it.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ----------------------------------------------------------------------------------------------------------------
// mbarriers
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait on a phase parity. Returns false (and records `code`) after kWaitLimitNs.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_error(err, code);
      return false;
    }
  }
}

// The same bounded wait with cluster-scope acquire: for data that peers of the cluster deliver with st.async.
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (mbar_try_wait_cluster(bar, parity)) return true;
  const uint64_t start = global_timer_ns();
  while (true) {
    for (int i = 0; i < 64; ++i)
      if (mbar_try_wait_cluster(bar, parity)) return true;
    if (global_timer_ns() - start > kWaitLimitNs) {
      record_error(err, code);
      return false;
    }
  }
}

// ----------------------------------------------------------------------------------------------------------------
// Hand-off between CTAs of one grid through global counters. The threads that store the data synchronise on a CTA
// barrier, then one of them calls signal_stored: a gpu-scope acquire-release fence and a relaxed add (the release
// pattern), whose cumulativity covers the stores the barrier ordered before it. The reader polls with acquire
// loads, synchronises its own threads on a barrier, and before reading the data with the async proxy (TMA, bulk
// copies) orders that read after the acquire with fence.proxy.async.global.
__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Acquire-release add returning the previous value: the release (after a fence) covers the stores the calling CTA
// ordered before it with a barrier, the acquire the loads that follow it.
__device__ __forceinline__ int atom_add_acq_rel_gpu(int* p, int v) {
  int old;
  asm volatile("fence.acq_rel.gpu;\n\tatom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v)
               : "memory");
  return old;
}
__device__ __forceinline__ void signal_stored(int* counter) {
  asm volatile("fence.acq_rel.gpu;\n\tred.relaxed.gpu.global.add.s32 [%0], 1;" ::"l"(counter) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}
// Barrier over `count` threads (a multiple of 32) of the CTA; ids 1..15 (0 is __syncthreads).
__device__ __forceinline__ void named_barrier_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// 16-byte asynchronous global -> shared copies (both addresses 16-byte aligned); `valid` false zero-fills.
__device__ __forceinline__ void cp_async_16(void* smem_dst, const void* src, bool valid = true) {
  const int size = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(src), "r"(size)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ----------------------------------------------------------------------------------------------------------------
// TMA (tiled tensor loads, no multicast). The innermost coordinate is always a multiple of 64 bf16 elements.
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global to shared memory,
// completing on `bar` like the tiled loads (no multicast).
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* src, uint32_t bytes, uint64_t* bar,
                                          uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// Row operands packed for bulk loads ("row tiles"): k-block kb (64 elements) of rows [0, ntok) is ntok x 128
// contiguous bytes, row r's 16-byte chunk c stored at chunk c ^ (r % 8) of its 128-byte row (the 128-byte swizzle
// the MMA descriptors expect); k-blocks follow each other, so any run of k-blocks is one contiguous copy.
// Returns the index of that 16-byte chunk.
__host__ __device__ __forceinline__ size_t row_tile_chunk(int kb, int r, int c, int ntok) {
  return (size_t(kb) * ntok + r) * 8 + size_t(c ^ (r & 7));
}

// Bulk prefetch of `bytes` (a multiple of 16, 16-byte aligned) from global memory into L2; nothing waits for it.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ----------------------------------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA (kind::f16, both operands from shared memory), commit and loads.
__device__ __forceinline__ void tmem_alloc(uint32_t* smem_slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_slot)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D(tmem, fp32) (+)= A(smem desc) * B(smem desc)^T, M x N x 16, bf16 or f16 inputs per `idesc`.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on `bar` when every previously issued tcgen05.mma of this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Instruction descriptor for kind::f16 with fp32 accumulation, both operands K-major.
//   bits 4-5 D format (1 = f32), 7-9 A format, 10-12 B format (0 = f16, 1 = bf16),
//   17-22 N >> 3, 24-28 M >> 4.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n, bool bf16) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | (uint32_t(n >> 3) << 17) |
         (uint32_t(m >> 4) << 24);
}

// Shared-memory matrix descriptor for a K-major tile stored as 128-byte rows with the 128-byte swizzle
// (what TMA writes with CU_TENSOR_MAP_SWIZZLE_128B): stride between 8-row groups 1024 B, version 1.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= uint64_t((smem_addr >> 4) & 0x3FFF);
  d |= uint64_t(1) << 16;            // leading byte offset (unused for swizzled K-major), 16 B
  d |= uint64_t(1024 >> 4) << 32;    // stride byte offset: 8 rows x 128 B
  d |= uint64_t(1) << 46;            // descriptor version for sm_100
  d |= uint64_t(2) << 61;            // SWIZZLE_128B
  return d;
}

// 32 lanes x 32 columns of fp32 from TMEM: thread i of the warp receives lane (lane_base + i), columns
// col .. col+31. The warp may only address the 32-lane slice (warp_id % 4) * 32.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// ----------------------------------------------------------------------------------------------------------------
// Thread-block clusters: rank, barrier and distributed shared memory loads (no TMA, no multicast).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of every CTA of the cluster must execute this (it is a hardware barrier, like __syncthreads).
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The two halves of a cluster barrier, for work between them: every thread arrives, then later waits. An arrival
// without release orders nothing; the wait returns once every thread of every CTA of the cluster has arrived, so a
// CTA that passed it knows that all CTAs of its cluster have started.
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait.aligned;" ::: "memory"); }
// Shared-memory address of `local` (an address in this CTA's shared memory) in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_map(const void* local, uint32_t rank) {
  uint32_t out;
  asm("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(local)), "r"(rank));
  return out;
}
// Plain 16-byte store into a cluster peer's shared memory (`addr` from cluster_map).
__device__ __forceinline__ void st_dsmem_f32x4(uint32_t addr, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_dsmem_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
// One arrival on a cluster peer's mbarrier (`remote_bar` from cluster_map) with release semantics at cluster scope:
// this thread's earlier writes, and those ordered before it by a CTA barrier, are visible to the peer's waiters.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t remote_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote_bar) : "memory");
}
// Distributed shared memory loads are plain (not volatile): they read peers' shared memory that a cluster_sync (a
// compiler memory barrier) has published, so the compiler may batch independent loads.
__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t ld_dsmem_u32(uint32_t addr) {
  uint32_t v;
  asm("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ float2 ld_dsmem_f32x2(uint32_t addr) {
  float2 v;
  asm("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}
__device__ __forceinline__ float4 ld_dsmem_f32x4(uint32_t addr) {
  float4 v;
  asm("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// ----------------------------------------------------------------------------------------------------------------
// Element helpers: the model's storage dtype is bf16 or f16; arithmetic is fp32.
template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }

template <typename T>
__device__ __forceinline__ T from_f32(float x);
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

// Round an fp32 value to the storage dtype and back (what storing and re-reading a tensor does).
template <typename T>
__device__ __forceinline__ float round_to(float x) { return to_f32<T>(from_f32<T>(x)); }

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, off));
  return v;
}

}  // namespace plm
