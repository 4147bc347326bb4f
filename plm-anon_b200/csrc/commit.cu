// KV commit and compaction of a round (north star item 5; the explicit form of the reference's implicit commit,
// plm/decoder.py:351-365, with the KV move idiom of eagle3/tree.py:263-279).
//
// A round's forward writes the K and V of all its W = k + k^2 rows into a per-handle scratch area instead of the
// paged cache: the rows are only candidates until the verify decode has decided how many of them the request keeps.
// Once it has, this kernel copies the accepted verify rows 0 .. nc (the bookkeeping leaves their first logical index
// and count in a two-word commit record) into the permanent pages at logical indices offset .. offset + nc through
// the block table. The other rows, among them the selected proposal block whose inputs were auxiliary embeddings at
// other row indices, stay in scratch, which the next round overwrites: they never enter the committed context, so
// the cache holds exactly what the reference's does below the committed offset.
//
// Grid (layer x {K, V}, scratch row); a CTA copies one row of one plane (num_kv_heads x head_dim elements) with
// 16-byte loads and stores, or returns at once when its row is not committed.
#include <cuda_bf16.h>

#include "commit.h"
#include "common.cuh"
#include "runtime.h"

namespace plm {
namespace {

constexpr int kCommitThreads = 256;

__global__ void __launch_bounds__(kCommitThreads) commit_kernel(const CommitArgs a) {
  grid_dependency_wait();  // the commit record comes from the bookkeeping of the kernel before
  allow_dependents();
  const int plane = blockIdx.x, j = blockIdx.y;
  const int64_t first = a.commit[0], count = a.commit[1];
  if (j >= count) return;
  const int64_t logical = first + j;
  const int64_t lp = logical / a.page_size;
  const int page = (logical >= 0 && lp < a.max_pages) ? a.block_table[lp] : -1;
  if (page < 0 || page >= a.num_pages || count > a.scratch_rows) {
    if (threadIdx.x == 0) record_error(a.err, kErrBadIndex);
    return;
  }
  const int within = int(logical % a.page_size);
  const int chunks_per_head = a.head_dim / 8;
  const int chunks = a.num_kv_heads * chunks_per_head;
  const uint4* src = reinterpret_cast<const uint4*>(a.scratch) +
                     (size_t(plane) * a.scratch_rows + j) * size_t(chunks);
  uint4* dst = reinterpret_cast<uint4*>(a.kv_cache) + size_t(plane) * (a.plane_elems / 8);
  for (int i = threadIdx.x; i < chunks; i += kCommitThreads) {
    const int g = i / chunks_per_head, c = i % chunks_per_head;
    dst[((size_t(page) * a.num_kv_heads + g) * a.page_size + within) * chunks_per_head + c] = src[i];
  }
}

}  // namespace

int commit_validate(const CommitArgs& a) {
  if (!a.scratch || !a.kv_cache || !a.block_table || !a.commit)
    return fail(PLM_ERR_INVALID, "commit: null operand");
  if (a.layers < 1 || a.num_kv_heads < 1 || a.head_dim < 8 || a.head_dim % 8 != 0 || a.page_size < 1 ||
      a.num_pages < 1 || a.max_pages < 1 || a.scratch_rows < 1 || a.scratch_rows > 4096)
    return fail(PLM_ERR_INVALID, "commit: layers %d, kv heads %d, head_dim %d, page %d, pages %d/%d, rows %d",
                a.layers, a.num_kv_heads, a.head_dim, a.page_size, a.num_pages, a.max_pages, a.scratch_rows);
  if (a.plane_elems != int64_t(a.num_pages) * a.num_kv_heads * a.page_size * a.head_dim)
    return fail(PLM_ERR_INVALID, "commit: plane of %lld elements does not match the pool",
                (long long)a.plane_elems);
  if ((reinterpret_cast<uintptr_t>(a.scratch) | reinterpret_cast<uintptr_t>(a.kv_cache)) & 15)
    return fail(PLM_ERR_INVALID, "commit: scratch and cache must be 16-byte aligned");
  return PLM_OK;
}

int commit_launch(const CommitArgs& a, cudaStream_t stream, bool pdl) {
  int st = commit_validate(a);
  if (st != PLM_OK) return st;
  return check_cuda(launch(commit_kernel, dim3(2 * a.layers, a.scratch_rows), dim3(kCommitThreads), 0, stream, pdl, a),
                    "commit_kernel");
}

}  // namespace plm

using namespace plm;

extern "C" int plm_commit(plm_ctx* ctx, const plm_commit_desc* d, void* stream) {
  if (ctx == nullptr || d == nullptr) return fail(PLM_ERR_INVALID, "plm_commit: null argument");
  if (d->dtype != PLM_BF16 && d->dtype != PLM_F16) return fail(PLM_ERR_INVALID, "plm_commit: dtype %d", d->dtype);
  CommitArgs a = {};
  a.scratch = d->scratch;
  a.scratch_rows = d->scratch_rows;
  a.kv_cache = d->kv_cache;
  a.plane_elems = d->plane_elems;
  a.layers = d->layers;
  a.num_kv_heads = d->num_kv_heads;
  a.head_dim = d->head_dim;
  a.page_size = d->page_size;
  a.num_pages = d->num_pages;
  a.max_pages = d->max_pages;
  a.block_table = d->block_table;
  a.commit = d->commit;
  a.err = ctx->err;
  return commit_launch(a, static_cast<cudaStream_t>(stream), true);
}
