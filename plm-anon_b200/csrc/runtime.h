// Host-side runtime shared by the C-ABI entry points: the context, error reporting, TMA descriptor encoding and
// launches with programmatic dependent launch enabled.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstddef>
#include <cstdint>
#include <string>

#include "../../include/plm_native.h"

struct plm_ctx {
  int device = 0;
  int num_sms = 148;
  int max_smem_optin = 0;
  int smem_per_sm = 0;
  int* err = nullptr;           // device error word
  int* counters = nullptr;      // arrival counters, zero between launches
  int n_counters = 0;
  float* attn_part = nullptr;   // plm_attention's two-cluster merge buffers, grown on demand
  size_t attn_part_floats = 0;
  int* attn_arrive = nullptr;   // zero between launches
  size_t attn_arrive_ints = 0;
};

namespace plm {

// Records a message for plm_last_error() and returns `status`.
int fail(int status, const char* fmt, ...);
// Returns PLM_OK or records the CUDA error (with `what`) and returns PLM_ERR_CUDA.
int check_cuda(cudaError_t e, const char* what);

// Encodes a 2-D tiled TMA descriptor over a row-major [outer][inner] tensor of 2-byte elements with the 128-byte
// swizzle. Returns PLM_OK or an error status.
int encode_map_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer);


// Raises `kernel`'s dynamic shared memory limit to at least `bytes` on the current device. The attribute belongs to
// a (function, device) pair, so each device a process launches on gets its own call; later calls that need no more
// than an earlier one return at once. Thread-safe.
int raise_smem_limit(const void* kernel, int bytes, const char* what);

// Launch with optional programmatic dependent launch and an optional cluster of cluster_x * cluster_y CTAs. With
// `pack`, the hardware may place several CTAs of one cluster on an SM (load-balancing scheduling) instead of
// spreading them over distinct SMs.
template <typename... KArgs, typename... Args>
cudaError_t launch_cluster_pref(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                                bool pdl, int cluster_x, int cluster_y, bool pack, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[3];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_x * cluster_y > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = unsigned(cluster_x);
    attr[n].val.clusterDim.y = unsigned(cluster_y);
    attr[n].val.clusterDim.z = 1;
    ++n;
    if (pack) {
      attr[n].id = cudaLaunchAttributeClusterSchedulingPolicyPreference;
      attr[n].val.clusterSchedulingPolicyPreference = cudaClusterSchedulingPolicyLoadBalancing;
      ++n;
    }
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                           bool pdl, int cluster_x, int cluster_y, Args&&... args) {
  return launch_cluster_pref(kernel, grid, block, smem, stream, pdl, cluster_x, cluster_y, false,
                             std::forward<Args>(args)...);
}

// Cluster of `cluster_y` CTAs along y.
template <typename... KArgs, typename... Args>
cudaError_t launch_ex(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                      int cluster_y, Args&&... args) {
  return launch_cluster(kernel, grid, block, smem, stream, pdl, 1, cluster_y, std::forward<Args>(args)...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl,
                   Args&&... args) {
  return launch_cluster(kernel, grid, block, smem, stream, pdl, 1, 1, std::forward<Args>(args)...);
}

// Cluster size (1..8) for the k-split of a weight-streaming GEMM over `slots` resident CTAs (SMs x CTAs per SM).
int gemm_cluster_splits(int tiles, int total_kb, int slots);

// Internal GEMM launch used by plm_gemm and by the round engine (`map_w` encoded once per weight).
// With `w_packed` the weight comes from its packed tiles (pack.cu) instead of map_w, which the kernel then only
// prefetches.
int gemm_launch(plm_ctx* ctx, const plm_gemm_desc& d, const CUtensorMap* map_w, const CUtensorMap* map_x,
                cudaStream_t stream, bool pdl, const void* w_packed = nullptr);
int gemm_weight_map(CUtensorMap* map, const plm_gemm_desc& d);
int gemm_row_map(CUtensorMap* map, const plm_gemm_desc& d);
int gemm_token_tile(int rows);
// Split count for a PLM_EPI_PARTIAL launch of this shape (1..16): fills the resident CTA slots in one wave.
int gemm_partial_splits(plm_ctx* ctx, int n_out, int k, int rows);

// Tiled weight copies (pack.cu): bytes of the packed copy, and the packing launch on `stream`.
size_t packed_tiles_bytes(int n_out, int k, int gate_offset);
int pack_weight_tiles(const void* w, int n_out, int k, int gate_offset, void* dst, cudaStream_t stream);

}  // namespace plm
