// Context lifetime, error reporting and TMA descriptor encoding for libplm_native.so.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "runtime.h"

namespace {
thread_local char g_last_error[1024] = "";

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// Arrival counters of a context (zero between launches).
constexpr int kCounters = 64;
}  // namespace

namespace plm {

int fail(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

int check_cuda(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PLM_OK;
  return fail(e == cudaErrorMemoryAllocation ? PLM_ERR_NOMEM : PLM_ERR_CUDA, "%s: %s (%s)", what,
              cudaGetErrorName(e), cudaGetErrorString(e));
}

int raise_smem_limit(const void* kernel, int bytes, const char* what) {
  int dev = 0;
  int st = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (st != PLM_OK) return st;
  static std::mutex mu;
  static std::map<std::pair<const void*, int>, int> raised;  // (kernel, device) -> the limit set so far
  std::lock_guard<std::mutex> lock(mu);
  const auto key = std::make_pair(kernel, dev);
  const auto it = raised.find(key);
  if (it != raised.end() && it->second >= bytes) return PLM_OK;
  st = check_cuda(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes), what);
  if (st == PLM_OK) raised[key] = bytes;
  return st;
}

int encode_map_2d(CUtensorMap* map, const void* base, int dtype, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return fail(PLM_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || (row_stride_bytes & 15) != 0)
    return fail(PLM_ERR_INVALID, "TMA operand must be 16-byte aligned (base %p, row stride %llu)", base,
                (unsigned long long)row_stride_bytes);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  const CUtensorMapDataType t = dtype == PLM_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = fn(map, t, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(PLM_ERR_INVALID, "cuTensorMapEncodeTiled failed (%d) for [%llu x %llu] box [%u x %u]", int(r),
                (unsigned long long)outer, (unsigned long long)inner, box_outer, box_inner);
  return PLM_OK;
}

int gemm_cluster_splits(int tiles, int total_kb, int slots) {
  // Splits of a tile run as one cluster (at most 8 CTAs). Estimated time in k-block units: waves over the
  // `slots` resident CTAs times (k-blocks per split + a fixed cost of kGemmOverheadKb for pipeline fill and the
  // epilogue). The cheapest split count wins; ties keep fewer splits (less reduction work).
  constexpr int kGemmOverheadKb = 4;
  int best = 1;
  long best_cost = -1;
  for (int s = 1; s <= 8 && s <= total_kb; ++s) {
    const int per = (total_kb + s - 1) / s;  // the largest split (k-blocks are spread evenly)
    const long waves = (long(tiles) * s + slots - 1) / slots;
    const long cost = waves * (per + kGemmOverheadKb);
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace plm

using namespace plm;

extern "C" {

int plm_abi_version(void) { return PLM_ABI_VERSION; }

int plm_last_error(char* buf, size_t n) {
  if (buf == nullptr || n == 0) return PLM_ERR_INVALID;
  strncpy(buf, g_last_error, n - 1);
  buf[n - 1] = '\0';
  return PLM_OK;
}

int plm_ctx_create(plm_ctx** out) {
  if (out == nullptr) return fail(PLM_ERR_INVALID, "plm_ctx_create: null output");
  *out = nullptr;
  plm_ctx* c = new plm_ctx();
  int st = check_cuda(cudaGetDevice(&c->device), "cudaGetDevice");
  if (st == PLM_OK) st = check_cuda(cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, c->device),
                                    "cudaDeviceGetAttribute(sm count)");
  if (st == PLM_OK)
    st = check_cuda(cudaDeviceGetAttribute(&c->max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, c->device),
                    "cudaDeviceGetAttribute(smem)");
  if (st == PLM_OK)
    st = check_cuda(cudaDeviceGetAttribute(&c->smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, c->device),
                    "cudaDeviceGetAttribute(smem per SM)");
  if (st == PLM_OK) {
    int major = 0, minor = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, c->device);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, c->device);
    if (major != 10 || minor != 0)
      st = fail(PLM_ERR_UNSUPPORTED, "libplm_native is built for sm_100a only; device %d is sm_%d%d", c->device,
                major, minor);
  }
  if (st == PLM_OK) st = check_cuda(cudaMalloc(&c->err, sizeof(int)), "cudaMalloc(error word)");
  if (st == PLM_OK) st = check_cuda(cudaMemset(c->err, 0, sizeof(int)), "cudaMemset(error word)");
  if (st == PLM_OK) st = check_cuda(cudaMalloc(&c->counters, kCounters * sizeof(int)), "cudaMalloc(counters)");
  if (st == PLM_OK) st = check_cuda(cudaMemset(c->counters, 0, kCounters * sizeof(int)), "cudaMemset(counters)");
  if (st == PLM_OK) c->n_counters = kCounters;
  if (st == PLM_OK) st = check_cuda(cudaDeviceSynchronize(), "plm_ctx_create");
  if (st != PLM_OK) {
    plm_ctx_destroy(c);
    return st;
  }
  *out = c;
  return PLM_OK;
}

int plm_ctx_destroy(plm_ctx* ctx) {
  if (ctx == nullptr) return PLM_OK;
  cudaFree(ctx->err);
  cudaFree(ctx->counters);
  cudaFree(ctx->attn_part);
  cudaFree(ctx->attn_arrive);
  delete ctx;
  return PLM_OK;
}

int plm_ctx_check(plm_ctx* ctx, int32_t* device_error) {
  if (ctx == nullptr || device_error == nullptr) return fail(PLM_ERR_INVALID, "plm_ctx_check: null argument");
  int st = check_cuda(cudaDeviceSynchronize(), "plm_ctx_check: synchronize");
  if (st != PLM_OK) return st;
  int v = 0;
  st = check_cuda(cudaMemcpy(&v, ctx->err, sizeof(int), cudaMemcpyDeviceToHost), "plm_ctx_check: read");
  if (st != PLM_OK) return st;
  *device_error = v;
  if (v != 0) {
    st = check_cuda(cudaMemset(ctx->err, 0, sizeof(int)), "plm_ctx_check: clearing the error word");
    // A launch that stopped early may have left arrival counters mid-count.
    if (st == PLM_OK)
      st = check_cuda(cudaMemset(ctx->counters, 0, ctx->n_counters * sizeof(int)), "plm_ctx_check: counters");
    if (st == PLM_OK) st = check_cuda(cudaDeviceSynchronize(), "plm_ctx_check: synchronize");
  }
  return st;
}

}  // extern "C"
