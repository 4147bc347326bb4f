// Host side of the skinny GEMM: operand validation, TMA descriptors, split planning and the
// (dtype, token tile, epilogue) dispatch. Entry point plm_gemm replaces plm/fast_gemm.py:82-97 (triton_linear).
#include "gemm.cuh"
#include "runtime.h"

namespace plm {

int gemm_token_tile(int rows) {
  if (rows <= 0) return -1;
  if (rows <= 16) return 16;
  if (rows <= 32) return 32;
  if (rows <= 48) return 48;
  if (rows <= 64) return 64;
  if (rows <= 80) return 80;
  if (rows <= 96) return 96;
  if (rows <= 112) return 112;
  if (rows <= 128) return 128;
  if (rows <= 256) return 256;
  return -1;
}

namespace {

// Pipeline depth: a ring of about 72 KB, so that three CTAs share an SM and one CTA's prologue and epilogue overlap
// the others' weight streaming (at least 2 stages).
template <int NTOK, int EPI>
constexpr int stages_for() {
  constexpr int by_budget = (72 * 1024) / GemmShape<NTOK>::STAGE_BYTES;
  return by_budget < 2 ? 2 : by_budget;
}

int tiles_for(int kind, int n_out, int gate_offset) {
  return kind == PLM_EPI_SILU_MUL ? gate_offset / 64 : (n_out + 127) / 128;
}

GemmArgs make_args(plm_ctx* ctx, const plm_gemm_desc& d, int tiles, int splits, int kb_per, const void* w_packed) {
  GemmArgs a = {};
  a.n_out = d.n_out;
  a.k = d.k;
  a.rows = d.rows;
  a.n_tiles = tiles;
  a.splits = splits;
  a.kb_per_split = kb_per;
  a.gate_offset = d.epi.gate_offset;
  a.out = d.out;
  a.ldo = d.ldo;
  a.err = ctx->err;
  const plm_gemm_epilogue& e = d.epi;
  a.qkv = QkvEpilogue{e.q_out,     e.k_cache,      e.v_cache,  e.positions, e.slots,     e.cos_sin,
                      e.num_heads, e.num_kv_heads, e.head_dim, e.page_size, e.num_slots, e.max_pos};
  a.logits = LogitsEpilogue{e.verify_logits, e.best_val, e.best_idx, e.n_verify, e.vocab};
  a.table = TableEpilogue{e.table, e.aux, e.a0};
  a.corr = e.corr;
  a.corr_from = e.corr_from;
  a.corr_ld = e.corr_ld;
  a.w_packed = static_cast<const uint8_t*>(w_packed);
  return a;
}

template <typename T, int NTOK, int EPI>
int launch_one(plm_ctx* ctx, const plm_gemm_desc& d, const CUtensorMap* map_w, const CUtensorMap* map_x,
               cudaStream_t stream, bool pdl, const void* w_packed) {
  constexpr int STAGES = stages_for<NTOK, EPI>();
  constexpr int SMEM = gemm_smem_bytes<NTOK, STAGES>();
  auto kernel = skinny_gemm_kernel<T, NTOK, STAGES, EPI>;
  {
    const int st = raise_smem_limit(reinterpret_cast<const void*>(kernel), SMEM, "cudaFuncSetAttribute(gemm smem)");
    if (st != PLM_OK) return st;
  }
  const int tiles = tiles_for(EPI, d.n_out, d.epi.gate_offset);
  const int total_kb = d.k / kGemmBK;
  const int per_sm = ctx->smem_per_sm > 0 ? ctx->smem_per_sm / (SMEM + 1024) : 1;
  int splits = d.splits > 0 ? d.splits : gemm_cluster_splits(tiles, total_kb, ctx->num_sms * (per_sm > 0 ? per_sm : 1));
  if (EPI == kEpiPartial) {  // splits written out, not reduced: no cluster, up to kMaxPartialSplits
    if (splits < 1 || splits > kMaxPartialSplits || splits > total_kb)
      return fail(PLM_ERR_UNSUPPORTED, "plm_gemm: %d partial splits (1..%d, at most k/64)", splits, kMaxPartialSplits);
  } else {
    if (splits > 8 || splits > total_kb)
      return fail(PLM_ERR_UNSUPPORTED, "plm_gemm: %d splits (at most 8 and at most k/64)", splits);
    if (NTOK > 128) splits = 1;  // the staging area holds no reduced slice for the widest tiles
  }
  const int kb_per = (total_kb + splits - 1) / splits;
  GemmArgs args = make_args(ctx, d, tiles, splits, kb_per, w_packed);
  return check_cuda(launch_ex(kernel, dim3(tiles, splits), dim3(kGemmThreads), SMEM, stream, pdl,
                              EPI == kEpiPartial ? 1 : splits, *map_w,
                              *map_x, args),
                    "skinny_gemm_kernel launch");
}

template <typename T, int NTOK>
int launch_epi(plm_ctx* ctx, const plm_gemm_desc& d, const CUtensorMap* mw, const CUtensorMap* mx,
               cudaStream_t s, bool pdl, const void* wp) {
  switch (d.epi.kind) {
    case PLM_EPI_STORE: return launch_one<T, NTOK, kEpiStore>(ctx, d, mw, mx, s, pdl, wp);
    case PLM_EPI_SILU_MUL: return launch_one<T, NTOK, kEpiSiluMul>(ctx, d, mw, mx, s, pdl, wp);
    case PLM_EPI_QKV_ROPE: return launch_one<T, NTOK, kEpiQkvRope>(ctx, d, mw, mx, s, pdl, wp);
    case PLM_EPI_LOGITS: return launch_one<T, NTOK, kEpiLogits>(ctx, d, mw, mx, s, pdl, wp);
    case PLM_EPI_TABLE: return launch_one<T, NTOK, kEpiTable>(ctx, d, mw, mx, s, pdl, wp);
    case PLM_EPI_PARTIAL: return launch_one<T, NTOK, kEpiPartial>(ctx, d, mw, mx, s, pdl, wp);
  }
  return fail(PLM_ERR_INVALID, "plm_gemm: unknown epilogue %d", d.epi.kind);
}

template <typename T>
int launch_dtype(plm_ctx* ctx, const plm_gemm_desc& d, const CUtensorMap* mw, const CUtensorMap* mx,
                 cudaStream_t s, bool pdl, const void* wp) {
  switch (gemm_token_tile(d.rows)) {
    case 16: return launch_epi<T, 16>(ctx, d, mw, mx, s, pdl, wp);
    case 32: return launch_epi<T, 32>(ctx, d, mw, mx, s, pdl, wp);
    case 48: return launch_epi<T, 48>(ctx, d, mw, mx, s, pdl, wp);
    case 64: return launch_epi<T, 64>(ctx, d, mw, mx, s, pdl, wp);
    case 80: return launch_epi<T, 80>(ctx, d, mw, mx, s, pdl, wp);
    case 96: return launch_epi<T, 96>(ctx, d, mw, mx, s, pdl, wp);
    case 112: return launch_epi<T, 112>(ctx, d, mw, mx, s, pdl, wp);
    case 128: return launch_epi<T, 128>(ctx, d, mw, mx, s, pdl, wp);
    case 256: return launch_epi<T, 256>(ctx, d, mw, mx, s, pdl, wp);
  }
  return fail(PLM_ERR_UNSUPPORTED, "plm_gemm: %d rows (1..256 supported)", d.rows);
}

int validate(const plm_gemm_desc& d) {
  if (d.dtype != PLM_BF16 && d.dtype != PLM_F16) return fail(PLM_ERR_INVALID, "plm_gemm: dtype %d", d.dtype);
  if (d.w == nullptr || d.x == nullptr) return fail(PLM_ERR_INVALID, "plm_gemm: null operand");
  if (d.k <= 0 || d.k % 64 != 0) return fail(PLM_ERR_INVALID, "plm_gemm: k=%d must be a positive multiple of 64", d.k);
  if (d.rows < 1 || d.rows > 256 || d.x_rows < d.rows)
    return fail(PLM_ERR_INVALID, "plm_gemm: rows=%d x_rows=%d", d.rows, d.x_rows);
  if (d.n_out < 1) return fail(PLM_ERR_INVALID, "plm_gemm: n_out=%d", d.n_out);
  const plm_gemm_epilogue& e = d.epi;
  switch (e.kind) {
    case PLM_EPI_STORE:
      if (d.out == nullptr || d.ldo < d.n_out) return fail(PLM_ERR_INVALID, "plm_gemm: store needs out, ldo >= n_out");
      break;
    case PLM_EPI_PARTIAL:
      if (d.out == nullptr || d.ldo < d.n_out) return fail(PLM_ERR_INVALID, "plm_gemm: partial needs out, ldo >= n_out");
      if (d.splits < 1) return fail(PLM_ERR_INVALID, "plm_gemm: partial needs an explicit split count");
      break;
    case PLM_EPI_SILU_MUL:
      if (e.gate_offset <= 0 || e.gate_offset % 64 != 0 || d.n_out != 2 * e.gate_offset)
        return fail(PLM_ERR_INVALID, "plm_gemm: silu needs n_out = 2 * gate_offset, gate_offset % 64 == 0");
      if (d.out == nullptr || d.ldo < e.gate_offset) return fail(PLM_ERR_INVALID, "plm_gemm: silu needs out");
      break;
    case PLM_EPI_QKV_ROPE:
      if (e.head_dim != 64 && e.head_dim != 128) return fail(PLM_ERR_UNSUPPORTED, "plm_gemm: head_dim %d", e.head_dim);
      if (e.num_heads <= 0 || e.num_kv_heads <= 0 || d.n_out != (e.num_heads + 2 * e.num_kv_heads) * e.head_dim)
        return fail(PLM_ERR_INVALID, "plm_gemm: qkv n_out must be (heads + 2 kv_heads) * head_dim");
      if (!e.q_out || !e.k_cache || !e.v_cache || !e.positions || !e.slots || !e.cos_sin || e.page_size <= 0)
        return fail(PLM_ERR_INVALID, "plm_gemm: qkv epilogue operands missing");
      break;
    case PLM_EPI_LOGITS:
      if (e.vocab <= 0 || e.vocab > d.n_out || e.n_verify < 0 || e.n_verify > d.rows)
        return fail(PLM_ERR_INVALID, "plm_gemm: logits vocab=%d n_verify=%d", e.vocab, e.n_verify);
      if ((e.n_verify > 0 && !e.verify_logits) || (e.n_verify < d.rows && (!e.best_val || !e.best_idx)))
        return fail(PLM_ERR_INVALID, "plm_gemm: logits outputs missing");
      break;
    case PLM_EPI_TABLE:
      if (!e.table || e.aux <= 0 || e.a0 < 0 || e.a0 + d.rows > e.aux)
        return fail(PLM_ERR_INVALID, "plm_gemm: table aux=%d a0=%d rows=%d", e.aux, e.a0, d.rows);
      break;
    default:
      return fail(PLM_ERR_INVALID, "plm_gemm: unknown epilogue %d", e.kind);
  }
  return PLM_OK;
}

}  // namespace

int gemm_weight_map(CUtensorMap* map, const plm_gemm_desc& d) {
  const uint32_t box_rows = d.epi.kind == PLM_EPI_SILU_MUL ? 64 : 128;
  return encode_map_2d(map, d.w, d.dtype, uint64_t(d.k), uint64_t(d.n_out), uint64_t(d.k) * 2, 64, box_rows);
}

int gemm_row_map(CUtensorMap* map, const plm_gemm_desc& d) {
  const int ntok = gemm_token_tile(d.rows);
  if (ntok < 0) return fail(PLM_ERR_UNSUPPORTED, "plm_gemm: %d rows", d.rows);
  return encode_map_2d(map, d.x, d.dtype, uint64_t(d.k), uint64_t(d.x_rows), uint64_t(d.k) * 2, 64, uint32_t(ntok));
}

template <int NTOK>
int partial_splits_for(plm_ctx* ctx, int n_out, int k) {
  constexpr int SMEM = gemm_smem_bytes<NTOK, stages_for<NTOK, kEpiPartial>()>();
  const int per_sm = ctx->smem_per_sm > 0 ? ctx->smem_per_sm / (SMEM + 1024) : 1;
  const int slots = ctx->num_sms * (per_sm > 0 ? per_sm : 1);
  const int tiles = (n_out + 127) / 128, total_kb = k / kGemmBK;
  // waves x (k-blocks per split + a fixed cost of 3) plus a quarter k-block per split for the consumer's extra reads
  int best = 1;
  double best_cost = -1;
  for (int s = 1; s <= kMaxPartialSplits && s <= total_kb; ++s) {
    const int per = (total_kb + s - 1) / s;
    const double waves = double((tiles * s + slots - 1) / slots);
    const double cost = waves * (per + 3) + 0.25 * s;
    if (best_cost < 0 || cost < best_cost) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

int gemm_partial_splits(plm_ctx* ctx, int n_out, int k, int rows) {
  switch (gemm_token_tile(rows)) {
    case 16: return partial_splits_for<16>(ctx, n_out, k);
    case 32: return partial_splits_for<32>(ctx, n_out, k);
    case 48: return partial_splits_for<48>(ctx, n_out, k);
    case 64: return partial_splits_for<64>(ctx, n_out, k);
    case 80: return partial_splits_for<80>(ctx, n_out, k);
    case 96: return partial_splits_for<96>(ctx, n_out, k);
    case 112: return partial_splits_for<112>(ctx, n_out, k);
    case 128: return partial_splits_for<128>(ctx, n_out, k);
    case 256: return partial_splits_for<256>(ctx, n_out, k);
  }
  return 1;
}

int gemm_launch(plm_ctx* ctx, const plm_gemm_desc& d, const CUtensorMap* map_w, const CUtensorMap* map_x,
                cudaStream_t stream, bool pdl, const void* w_packed) {
  int st = validate(d);
  if (st != PLM_OK) return st;
  if (w_packed != nullptr && (d.epi.kind == PLM_EPI_LOGITS || d.epi.kind == PLM_EPI_TABLE ||
                              (reinterpret_cast<uintptr_t>(w_packed) & 15) != 0))
    return fail(PLM_ERR_INVALID, "gemm: packed weights for the projections only, 16-byte aligned");
  if (d.dtype == PLM_F16) return launch_dtype<__half>(ctx, d, map_w, map_x, stream, pdl, w_packed);
  return launch_dtype<__nv_bfloat16>(ctx, d, map_w, map_x, stream, pdl, w_packed);
}

}  // namespace plm

using namespace plm;

extern "C" int plm_gemm_tiles(int32_t kind, int32_t n_out, int32_t gate_offset, int32_t* tiles) {
  if (tiles == nullptr) return fail(PLM_ERR_INVALID, "plm_gemm_tiles: null output");
  *tiles = tiles_for(kind, n_out, gate_offset);
  return PLM_OK;
}

extern "C" int plm_gemm(plm_ctx* ctx, const plm_gemm_desc* desc, void* stream) {
  if (ctx == nullptr || desc == nullptr) return fail(PLM_ERR_INVALID, "plm_gemm: null argument");
  int st = validate(*desc);
  if (st != PLM_OK) return st;
  CUtensorMap mw, mx;
  st = gemm_weight_map(&mw, *desc);
  if (st != PLM_OK) return st;
  st = gemm_row_map(&mx, *desc);
  if (st != PLM_OK) return st;
  return gemm_launch(ctx, *desc, &mw, &mx, static_cast<cudaStream_t>(stream), true);
}
