// Tiled copies of weight matrices for the weight-streaming kernels.
//
// A row-major [n_out][k] weight read as 128-row x 64-k TMA boxes costs the HBM one 128-byte piece from each of 128
// rows that lie k * 2 bytes apart. Packed, tile t / k-block kb is ONE contiguous 16 KB block that already holds the
// shared-memory image the MMA reads: 128 rows of 128 bytes, 16-byte chunk c of row r stored at chunk c ^ (r % 8)
// (the 128-byte swizzle that the tensor maps of gemm.cu request), so one untiled bulk copy loads a stage.
//
// Block order: [tile][k-block][128 x 64]. Rows past n_out are zero. With gate_offset > 0 (the gate_up weight of a
// SiLU * up tile) tile t holds gate rows t*64 .. t*64+63 followed by up rows gate_offset + t*64 .. +63, as the
// SiLU epilogue expects.
#include "runtime.h"

namespace plm {
namespace {

__global__ void __launch_bounds__(128) pack_tiles_kernel(const uint4* __restrict__ w, int n_out, int k,
                                                         int gate_offset, uint4* __restrict__ dst) {
  const int total_kb = k / 64;
  const int tile = blockIdx.x / total_kb, kb = blockIdx.x % total_kb;
  const int r = threadIdx.x;
  int src_row;
  if (gate_offset > 0)
    src_row = r < 64 ? tile * 64 + r : gate_offset + tile * 64 + (r - 64);
  else
    src_row = tile * 128 + r;
  uint4* out = dst + size_t(blockIdx.x) * 1024 + r * 8;  // 16 KB block = 1024 chunks; row r = 8 chunks
  const bool valid = src_row < n_out;
  const uint4* in = w + (size_t(src_row) * k + size_t(kb) * 64) / 8;
#pragma unroll
  for (int c = 0; c < 8; ++c) out[c ^ (r & 7)] = valid ? in[c] : make_uint4(0, 0, 0, 0);
}

}  // namespace

size_t packed_tiles_bytes(int n_out, int k, int gate_offset) {
  const size_t tiles = gate_offset > 0 ? size_t(gate_offset / 64) : size_t((n_out + 127) / 128);
  return tiles * size_t(k / 64) * 16384;
}

int pack_weight_tiles(const void* w, int n_out, int k, int gate_offset, void* dst, cudaStream_t stream) {
  if (k % 64 != 0 || (gate_offset > 0 && (gate_offset % 64 != 0 || n_out != 2 * gate_offset)))
    return fail(PLM_ERR_INVALID, "pack: n_out %d, k %d, gate_offset %d", n_out, k, gate_offset);
  if ((reinterpret_cast<uintptr_t>(w) & 15) != 0 || (reinterpret_cast<uintptr_t>(dst) & 15) != 0)
    return fail(PLM_ERR_INVALID, "pack: operands must be 16-byte aligned");
  const int tiles = gate_offset > 0 ? gate_offset / 64 : (n_out + 127) / 128;
  const int blocks = tiles * (k / 64);
  pack_tiles_kernel<<<blocks, 128, 0, stream>>>(static_cast<const uint4*>(w), n_out, k, gate_offset,
                                                static_cast<uint4*>(dst));
  return check_cuda(cudaGetLastError(), "pack_tiles_kernel");
}

}  // namespace plm
