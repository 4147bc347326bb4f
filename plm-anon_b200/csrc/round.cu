// The round engine behind the C ABI: one handle = one request stream on one GPU (batch 1, like the reference's
// RoundDecoder, plm/decoder.py:85-467). The handle owns the paged KV pool, the block table, the activation buffers,
// the round layouts, the loop-carried state (out, base, offset, anchor, pending, round_sequence) and the Voronoi
// cost table; the weights are borrowed device pointers.
//
// plm_round / plm_round0 / plm_prefill only enqueue kernels on the caller's stream (programmatic dependent launch
// between consecutive kernels, no host synchronisation), so a caller can capture plm_round into a CUDA graph and
// replay it once per round, as the reference replays its captured steady round (decoder.py:312-324, 414-439).
#include <cuda_bf16.h>

#include <algorithm>
#include <array>
#include <cstring>
#include <map>
#include <vector>

#include "attention.h"
#include "commit.h"
#include "elementwise.h"
#include "icdf.h"
#include "mlp.h"
#include "runtime.h"
#include "verify.h"

namespace plm {
namespace {

constexpr int kUnreachable = 1 << 30;  // plm/mask.py:14
constexpr int kMaxPrefillRows = 256;

constexpr int kPartialSlices = 16;  // the most k-splits gemm_partial_splits chooses

template <typename Tp>
int dev_alloc(Tp** p, size_t count, const char* what) {
  return check_cuda(cudaMalloc(reinterpret_cast<void**>(p), std::max<size_t>(count, 1) * sizeof(Tp)), what);
}

}  // namespace
}  // namespace plm

struct plm_handle {
  plm_ctx* ctx = nullptr;
  plm_model_desc m = {};
  plm_round_desc rd = {};
  int W = 0;                 // rows of a round: k + k^2
  int R = 0;                 // activation row capacity
  // weights (borrowed)
  const void *embed = nullptr, *lm_head = nullptr, *final_norm = nullptr, *aux_vocab = nullptr, *mask_aux = nullptr,
             *cos_sin = nullptr;
  std::vector<const void*> qkv, o, gate_up, down, in_norm, post_norm;
  void* table = nullptr;
  bool own_table = false;
  std::vector<CUtensorMap> map_qkv, map_o, map_gate_up, map_down;
  CUtensorMap map_lm;
  std::map<std::pair<const void*, int>, CUtensorMap> row_maps;
  // activations
  void *x_norm = nullptr, *residual = nullptr, *y = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr,
       *gathered = nullptr;
  int32_t* positions = nullptr;
  int64_t* slots = nullptr;
  float* partials = nullptr;  // [kPartialSlices][R][hidden] fp32 k-split partials of the o and down projections
  float* verify_logits = nullptr;
  float* best_val = nullptr;
  int32_t* best_idx = nullptr;
  int lm_tiles = 0;
  int64_t* verify = nullptr;
  int32_t* flags = nullptr;
  // layouts
  int64_t *st_relpos = nullptr, *st_relaux = nullptr, *r0_relpos = nullptr, *r0_relaux = nullptr;
  int32_t *st_depth = nullptr, *st_own = nullptr, *r0_depth = nullptr, *r0_own = nullptr, *causal_depth = nullptr,
          *causal_own = nullptr;
  // paged KV
  void* kv = nullptr;
  size_t plane_elems = 0;
  int32_t* block_table = nullptr;
  // a round's candidate rows: K/V of all W rows of the last round0 / steady forward, [layer][K|V][W][kv_heads][hd],
  // and the commit record [first logical index, rows] the bookkeeping leaves for the commit kernel
  void* round_kv = nullptr;
  int64_t* commit = nullptr;
  // loop state
  int64_t *out = nullptr, *base = nullptr, *offset = nullptr, *anchor = nullptr, *pending = nullptr,
          *round_sequence = nullptr, *sequence_step = nullptr, *aux_buf = nullptr, *prompt = nullptr,
          *chunk_offsets = nullptr;
  int64_t* stop = nullptr;      // [kStopWords] the request stop block the steady bookkeeping reads and sets
  int64_t stop_host[4] = {};    // the values plm_set_stop last queued (the copy's host source stays valid)
  int64_t prompt_len = 0;
  int attn_splits_round = 1;
  float* attn_part = nullptr;  // the round attention's split partials when its splits are combined in memory
  int* attn_arrive = nullptr;
  // MLP block kernel: schedule, per-layer gate_up counters and the forward counter they are compared with
  plm::MlpSchedule mlp;
  int* block_ctr = nullptr;  // [layers][4] phase counters of the layer blocks, zeroed by every forward's prologue
  void* block_tiles = nullptr;  // per layer: packed o, gate_up, down (pack.cu)
  void *attn_tiles = nullptr, *x_tiles = nullptr, *act_tiles = nullptr;  // row operands as row tiles (common.cuh)
  size_t block_o_bytes = 0, block_gate_up_bytes = 0, block_layer_bytes = 0;
  // The PTP scheme of the gated-LoRA model (ptp_embedding null: the logit-Voronoi scheme of every PLM)
  const float* ptp_embedding = nullptr;
  int ptp_rows = 0, ptp_top_k = 0, lora_rank = 0;
  float* aux_u = nullptr;  // [aux_len] the request's uniforms
  // per layer and projection (qkv, o, gate_up, down): the adapter's shards, each a down map (rank rows of the stacked
  // A) and an up map (its output rows of B); empty when the projection has no adapter
  struct LoraShard {
    const void* a = nullptr;
    const void* b = nullptr;
    CUtensorMap map_a, map_b;
    int out0 = 0, width = 0;  // the shard's output columns
  };
  std::vector<std::array<std::vector<LoraShard>, 4>> lora;
  void* lora_hidden = nullptr;  // [3][R][rank] model dtype: x A_s^T of the gated rows, per shard
  float* lora_corr = nullptr;   // [R][widest output] fp32: the adapter's output of the gated rows
};

namespace plm {
namespace {

void* kv_plane(plm_handle* h, int layer, int which) {
  return static_cast<__nv_bfloat16*>(h->kv) + (size_t(layer) * 2 + which) * h->plane_elems;
}
void* round_plane(plm_handle* h, int layer, int which) {
  return static_cast<__nv_bfloat16*>(h->round_kv) +
         (size_t(layer) * 2 + which) * size_t(h->W) * h->m.num_kv_heads * h->m.head_dim;
}

int row_map(plm_handle* h, const void* buffer, int k, int rows, const CUtensorMap** out, int x_rows = 0) {
  const int ntok = gemm_token_tile(rows);
  if (ntok < 0) return fail(PLM_ERR_UNSUPPORTED, "row map: %d rows", rows);
  auto key = std::make_pair(buffer, ntok);
  auto it = h->row_maps.find(key);
  if (it == h->row_maps.end()) {
    plm_gemm_desc d = {};
    d.dtype = h->m.dtype;
    d.x = buffer;
    d.k = k;
    d.rows = rows;
    d.x_rows = x_rows > 0 ? x_rows : buffer == h->gathered ? 16 : h->R;
    CUtensorMap map;
    int st = gemm_row_map(&map, d);
    if (st != PLM_OK) return st;
    it = h->row_maps.emplace(key, map).first;
  }
  *out = &it->second;
  return PLM_OK;
}

int gemm(plm_handle* h, const void* w, const CUtensorMap* mw, int n_out, int k, const void* x, int rows,
         const plm_gemm_epilogue& epi, void* out, int ldo, cudaStream_t s, int splits = 0, int x_rows = 0,
         const void* w_packed = nullptr) {
  plm_gemm_desc d = {};
  d.dtype = h->m.dtype;
  d.w = w;
  d.n_out = n_out;
  d.k = k;
  d.x = x;
  d.x_rows = x_rows > 0 ? x_rows : x == h->gathered ? 16 : h->R;
  d.rows = rows;
  d.out = out;
  d.ldo = ldo;
  d.splits = splits;
  d.epi = epi;
  const CUtensorMap* mx = nullptr;
  int st = row_map(h, x, k, rows, &mx, x_rows);
  if (st != PLM_OK) return st;
  return gemm_launch(h->ctx, d, mw, mx, s, true, w_packed);
}

// The packed copy of layer l's o (which 0), gate_up (1) or down (2) weight when the handle holds one: the separate
// launches read it too, so the caller's originals are not read after plm_create.
const void* packed_weight(const plm_handle* h, int l, int which) {
  if (h->block_tiles == nullptr) return nullptr;
  const uint8_t* w = static_cast<const uint8_t*>(h->block_tiles) + size_t(l) * h->block_layer_bytes;
  return which == 0 ? w : which == 1 ? w + h->block_o_bytes : w + h->block_o_bytes + h->block_gate_up_bytes;
}

// Layer `l`'s block (mlp.cu): o projection, the residual-add RMSNorm after it, gate_up + SiLU and down as k-split
// partials, over `rows` rows whose attention output is in the row tiles. The block's phase counters must be zero
// (every forward's prologue zeroes them).
int layer_block_launch(plm_handle* h, int l, int rows, cudaStream_t s) {
  const plm_model_desc& m = h->m;
  BlockParams b = {};
  const uint8_t* w = static_cast<const uint8_t*>(h->block_tiles) + size_t(l) * h->block_layer_bytes;
  b.wo_tiles = w;
  b.wg_tiles = w + h->block_o_bytes;
  b.wd_tiles = w + h->block_o_bytes + h->block_gate_up_bytes;
  b.attn_tiles = static_cast<const uint8_t*>(h->attn_tiles);
  b.x_tiles = static_cast<uint8_t*>(h->x_tiles);
  b.act_tiles = static_cast<uint8_t*>(h->act_tiles);
  b.partials = h->partials;
  b.residual = h->residual;
  b.norm_weight = h->post_norm[l];
  b.eps = m.rms_eps;
  b.ctr = h->block_ctr + 4 * l;
  b.rows = rows;
  b.hidden = m.hidden;
  b.intermediate = m.intermediate;
  b.q_size = m.num_heads * m.head_dim;
  // the next kernel's first weights: the next layer's qkv, or after the last layer the head of lm_head (as much as
  // the idle tail of the block and the norm after it can bring in)
  constexpr long long kLmHeadPrefetch = 32ll << 20;
  if (l + 1 < m.num_layers) {
    b.next_weights = static_cast<const uint8_t*>(h->qkv[l + 1]);
    b.next_bytes = (long long)(m.num_heads + 2 * m.num_kv_heads) * m.head_dim * m.hidden * 2;
  } else {
    b.next_weights = static_cast<const uint8_t*>(h->lm_head);
    b.next_bytes = std::min<long long>((long long)m.vocab * m.hidden * 2, kLmHeadPrefetch) & ~15LL;
  }
  b.err = h->ctx->err;
  return mlp_block_launch(h->mlp, b, m.dtype, s, true);
}

// The Llama forward of `rows` rows whose logical KV indices start at *offset_ptr (vLLM llama.py:253-314):
// prologue (+ layer-0 input norm), then per layer qkv(+RoPE, KV scatter) -> attention -> o -> add+norm ->
// gate_up(+SiLU) -> down -> add+norm (the next layer's input norm, or the final norm).
// The gated-LoRA correction of projection `proj` (0 qkv, 1 o, 2 gate_up, 3 down) of layer `l` on rows
// [from, rows) of `x` ([R][k] model dtype): per shard s, hidden_s = round(x A_s^T) into the hidden slices, then
// hidden_s B_s^T in fp32 into the shard's columns of lora_corr (row r - from, stride n_total)
// (plm/gated_lora.py:45-57). The projection's own epilogue (or the norm after it) adds it. Returns the stride,
// or 0 when the projection has no adapter (nothing launched).
int lora_correction(plm_handle* h, int l, int proj, const void* x, int k, int from, int rows, int n_total,
                    cudaStream_t s, int* corr_ld) {
  *corr_ld = 0;
  if (h->ptp_embedding == nullptr || h->lora_rank == 0 || from >= rows || h->lora[l][proj].empty()) return PLM_OK;
  const int g_rows = rows - from;
  const int rank = h->lora_rank;
  const void* xg = static_cast<const __nv_bfloat16*>(x) + size_t(from) * k;
  int st = PLM_OK;
  const std::vector<plm_handle::LoraShard>& shards = h->lora[l][proj];
  for (size_t sh = 0; sh < shards.size() && st == PLM_OK; ++sh) {
    const plm_handle::LoraShard& z = shards[sh];
    void* hidden = static_cast<__nv_bfloat16*>(h->lora_hidden) + sh * size_t(h->R) * rank;
    plm_gemm_epilogue store = {};
    store.kind = PLM_EPI_STORE;
    st = gemm(h, z.a, &z.map_a, rank, k, xg, g_rows, store, hidden, rank, s, 0, h->R - from);
    plm_gemm_epilogue part = {};
    part.kind = PLM_EPI_PARTIAL;
    if (st == PLM_OK)
      st = gemm(h, z.b, &z.map_b, z.width, rank, hidden, g_rows, part, h->lora_corr + z.out0, n_total, s, 1);
  }
  if (st == PLM_OK) *corr_ld = n_total;
  return st;
}

// A round's forward (round0 or steady mode) writes its rows' K/V into the round scratch, and attention reads the
// forward's own keys from there; a prefill writes straight into the pages (every prompt row is committed).
int forward(plm_handle* h, int mode, int rows, const int64_t* offset_ptr, const int64_t* relpos, const int64_t* relaux,
            const int32_t* depth, const int32_t* own, int attn_splits, int gather_row, cudaStream_t s) {
  const bool round_rows = mode != kProloguePrefill;
  // the first row a gated-LoRA adapter acts on: row k of a steady round, row 1 of round 0, none in a prefill
  // (plm/decoder.py:298, 317, 381)
  const int gated_from = mode == kPrologueSteady ? h->rd.k : mode == kPrologueRound0 ? 1 : rows;
  const plm_model_desc& m = h->m;
  const int hidden = m.hidden, hd = m.head_dim;
  const int q_size = m.num_heads * hd, kv_size = m.num_kv_heads * hd;
  PrologueArgs p = {};
  p.dtype = m.dtype;
  p.mode = mode;
  p.k = h->rd.k;
  p.vocab = m.vocab;
  p.aux = m.aux_vocab;
  p.num_aux_tokens = m.num_aux_tokens;
  p.hidden = hidden;
  p.eps = m.rms_eps;
  p.offset = offset_ptr;
  p.base = h->base;
  p.anchor = h->anchor;
  p.pending = h->pending;
  p.rel_positions = relpos;
  p.rel_aux = relaux;
  p.aux_buf = h->aux_buf;
  p.aux_len = h->rd.aux_len;
  p.prompt = h->prompt;
  p.prompt_cap = int64_t(h->rd.max_pages) * h->rd.page_size;
  p.embed = h->embed;
  p.aux_vocab = h->aux_vocab;
  p.mask_aux = h->mask_aux;
  p.norm_weight = h->in_norm[0];
  p.block_table = h->block_table;
  p.max_pages = h->rd.max_pages;
  p.num_pages = h->rd.num_pages;
  p.page_size = h->rd.page_size;
  p.max_pos = m.max_pos;
  p.residual = h->residual;
  p.normed = h->x_norm;
  p.positions = h->positions;
  p.slots = h->slots;
  p.round_scratch = round_rows ? 1 : 0;
  p.ptp_embedding = h->ptp_embedding;
  p.ptp_rows = h->ptp_rows;
  p.aux_u = h->aux_u;
  const bool layer_block = h->mlp.sched != nullptr && rows <= kMlpMaxRows;
  p.counters = h->block_ctr;
  p.n_counters = h->block_ctr != nullptr ? 4 * m.num_layers : 0;
  p.err = h->ctx->err;
  int st = prologue_launch(p, rows, s, true);
  if (st != PLM_OK) return st;

  for (int l = 0; l < m.num_layers; ++l) {
    plm_gemm_epilogue e = {};
    e.kind = PLM_EPI_QKV_ROPE;
    e.q_out = h->q;
    e.positions = h->positions;
    e.slots = h->slots;
    e.cos_sin = h->cos_sin;
    e.num_heads = m.num_heads;
    e.num_kv_heads = m.num_kv_heads;
    e.head_dim = hd;
    if (round_rows) {  // the round scratch as a cache of one-row pages: slot r is row r
      e.k_cache = round_plane(h, l, 0);
      e.v_cache = round_plane(h, l, 1);
      e.page_size = 1;
      e.num_slots = h->W;
    } else {
      e.k_cache = kv_plane(h, l, 0);
      e.v_cache = kv_plane(h, l, 1);
      e.page_size = h->rd.page_size;
      e.num_slots = int64_t(h->rd.num_pages) * h->rd.page_size;
    }
    e.max_pos = m.max_pos;
    st = lora_correction(h, l, 0, h->x_norm, hidden, gated_from, rows, q_size + 2 * kv_size, s, &e.corr_ld);
    if (st != PLM_OK) return st;
    if (e.corr_ld > 0) {
      e.corr = h->lora_corr;
      e.corr_from = gated_from;
    }
    st = gemm(h, h->qkv[l], &h->map_qkv[l], q_size + 2 * kv_size, hidden, h->x_norm, rows, e, nullptr, 0, s);
    if (st != PLM_OK) return st;

    AttnArgs a = {};
    a.dtype = m.dtype;
    a.q = h->q;
    a.k_cache = kv_plane(h, l, 0);
    a.v_cache = kv_plane(h, l, 1);
    a.block_table = h->block_table;
    a.max_pages = h->rd.max_pages;
    a.num_pages = h->rd.num_pages;
    a.page_size = h->rd.page_size;
    a.offset = offset_ptr;
    a.rows = rows;
    a.depth = depth;
    a.own_start = own;
    a.num_heads = m.num_heads;
    a.num_kv_heads = m.num_kv_heads;
    a.head_dim = hd;
    a.scale_log2 = float(1.4426950408889634 / sqrt(double(hd)));
    if (layer_block) {  // the block reads the attention output as row tiles
      a.row_tiles = h->attn_tiles;
      a.tile_rows = gemm_token_tile(rows);
    } else {
      a.out = h->attn;
    }
    a.splits = attn_splits;
    if (attn_splits > 8) {  // the round's attention with two clusters of splits per head
      a.part = h->attn_part;
      a.arrive = h->attn_arrive;
    }
    if (round_rows) {
      a.scratch_k = round_plane(h, l, 0);
      a.scratch_v = round_plane(h, l, 1);
    }
    st = attention_launch(h->ctx, a, s, true);
    if (st != PLM_OK) return st;

    // o and down write their k-split partials; the residual-add RMSNorm that follows each sums them in split order
    plm_gemm_epilogue part = {};
    part.kind = PLM_EPI_PARTIAL;
    const int64_t slice = int64_t(rows) * hidden;
    int s_d = 0, down_ld = 0;
    if (layer_block) {  // o, its norm, gate_up and down in one launch
      st = layer_block_launch(h, l, rows, s);
      if (st != PLM_OK) return st;
      s_d = h->mlp.down_splits;
    } else {
      int ld = 0;
      st = lora_correction(h, l, 1, h->attn, q_size, gated_from, rows, hidden, s, &ld);
      if (st != PLM_OK) return st;
      const int s_o = gemm_partial_splits(h->ctx, hidden, q_size, rows);
      st = gemm(h, h->o[l], &h->map_o[l], hidden, q_size, h->attn, rows, part, h->partials, hidden, s, s_o, 0,
                packed_weight(h, l, 0));
      if (st != PLM_OK) return st;
      AddNormArgs n1 = {nullptr, h->residual, h->x_norm, h->post_norm[l], hidden, m.rms_eps, -1, nullptr,
                        h->partials, s_o, slice};
      n1.dtype = m.dtype;
      if (ld > 0) {
        n1.corr = h->lora_corr;
        n1.corr_from = gated_from;
        n1.corr_ld = ld;
      }
      st = add_norm_launch(n1, rows, s, true);
      if (st != PLM_OK) return st;
      plm_gemm_epilogue silu = {};
      silu.kind = PLM_EPI_SILU_MUL;
      silu.gate_offset = m.intermediate;
      st = lora_correction(h, l, 2, h->x_norm, hidden, gated_from, rows, 2 * m.intermediate, s, &silu.corr_ld);
      if (st != PLM_OK) return st;
      if (silu.corr_ld > 0) {
        silu.corr = h->lora_corr;
        silu.corr_from = gated_from;
      }
      st = gemm(h, h->gate_up[l], &h->map_gate_up[l], 2 * m.intermediate, hidden, h->x_norm, rows, silu, h->act,
                m.intermediate, s, 0, 0, packed_weight(h, l, 1));
      if (st != PLM_OK) return st;
      st = lora_correction(h, l, 3, h->act, m.intermediate, gated_from, rows, hidden, s, &down_ld);
      if (st != PLM_OK) return st;
      s_d = gemm_partial_splits(h->ctx, hidden, m.intermediate, rows);
      st = gemm(h, h->down[l], &h->map_down[l], hidden, m.intermediate, h->act, rows, part, h->partials, hidden, s,
                s_d, 0, packed_weight(h, l, 2));
      if (st != PLM_OK) return st;
    }
    const bool last = l + 1 == m.num_layers;
    AddNormArgs n2 = {nullptr,  h->residual,           h->x_norm, last ? h->final_norm : h->in_norm[l + 1],
                      hidden,   m.rms_eps,             last ? gather_row : -1, last ? h->gathered : nullptr,
                      h->partials, s_d, slice};
    n2.dtype = m.dtype;
    if (down_ld > 0) {
      n2.corr = h->lora_corr;
      n2.corr_from = gated_from;
      n2.corr_ld = down_ld;
    }
    st = add_norm_launch(n2, rows, s, true);
    if (st != PLM_OK) return st;
  }
  return PLM_OK;
}

int lm_head(plm_handle* h, const void* x, int rows, int n_verify, cudaStream_t s) {
  plm_gemm_epilogue e = {};
  e.kind = PLM_EPI_LOGITS;
  e.verify_logits = h->verify_logits;
  e.best_val = h->best_val;
  e.best_idx = h->best_idx;
  e.n_verify = n_verify;
  e.vocab = h->m.vocab;
  return gemm(h, h->lm_head, &h->map_lm, h->m.vocab, h->m.hidden, x, rows, e, nullptr, 0, s);
}

int verify(plm_handle* h, int n_rows, int mode, const int64_t* aux_base, cudaStream_t s) {
  VerifyArgs a = {};
  if (h->ptp_embedding != nullptr) {
    // The PTP scheme decodes by inverse CDF at the request's uniforms (plm/auxiliary.py:104-113); the verify kernel
    // then adds only the relaxed rule's verdicts and the bookkeeping.
    IcdfArgs ic = {};
    ic.logits = h->verify_logits;
    ic.ld = h->m.vocab;
    ic.u = h->aux_u;
    ic.n_rows = n_rows;
    ic.vocab = h->m.vocab;
    ic.top_k = h->ptp_top_k;
    ic.tokens = h->verify;
    ic.u_base = aux_base;
    ic.u_len = h->rd.aux_len;
    ic.err = h->ctx->err;
    const int st = icdf_launch(ic, s, true);
    if (st != PLM_OK) return st;
    a.tokens_given = 1;
  }
  a.logits = h->verify_logits;
  a.vocab = h->m.vocab;
  a.logits_stride = h->m.vocab;
  a.table = h->table;
  a.aux = h->m.aux_vocab;
  a.aux_buf = h->aux_buf;
  a.aux_len = h->rd.aux_len;
  a.aux_base = aux_base;
  a.aux_row_offset = 0;
  a.pending = h->pending;
  a.n_accept = mode == kBookSteady ? h->rd.k - 1 : 0;
  a.rule = h->rd.rule;
  a.threshold = h->rd.threshold;
  a.top_m = h->m.top_m;
  a.shortlist = h->m.shortlist;
  a.rounds = h->m.rounds;
  a.sweeps = h->m.sweeps;
  for (int r = 0; r < 4; ++r) {
    const double eps = r == 0 ? h->m.epsilon : h->m.epsilon * h->m.refocus;
    a.eps[r] = float(eps);
    a.anneal[r] = float(pow(h->m.endpoint / eps, 1.0 / double(h->m.sweeps > 1 ? h->m.sweeps : 1)));
  }
  a.verify = h->verify;
  a.flags = h->flags;
  a.book.mode = mode;
  a.book.k = h->rd.k;
  a.book.best_val = h->best_val;
  a.book.best_idx = h->best_idx;
  a.book.n_tiles = h->lm_tiles;
  a.book.rows = h->W;
  a.book.out = h->out;
  a.book.out_cap = h->rd.out_capacity;
  a.book.base = h->base;
  a.book.offset = h->offset;
  a.book.anchor = h->anchor;
  a.book.pending = h->pending;
  a.book.round_sequence = h->round_sequence;
  a.book.seq_cap = h->rd.seq_capacity;
  a.book.sequence_step = h->sequence_step;
  a.book.prompt_len = h->prompt_len;
  a.book.stop = h->stop;
  a.book.commit = h->commit;
  a.counter = h->ctx->counters + (h->ctx->n_counters - 1);
  a.err = h->ctx->err;
  int st = verify_validate(a, n_rows);
  if (st != PLM_OK) return st;
  // Launched without programmatic dependent launch: started early, its clusters were placed while lm_head's CTAs
  // still held the SMs and the decode's critical path grew by ~9 us.
  return verify_launch(a, h->m.dtype, n_rows, s, false);
}

// The accepted verify rows of the round just decided, from the round scratch into the pages (commit.cu).
int commit_rows(plm_handle* h, cudaStream_t s) {
  CommitArgs c = {};
  c.scratch = h->round_kv;
  c.scratch_rows = h->W;
  c.kv_cache = h->kv;
  c.plane_elems = int64_t(h->plane_elems);
  c.layers = h->m.num_layers;
  c.num_kv_heads = h->m.num_kv_heads;
  c.head_dim = h->m.head_dim;
  c.page_size = h->rd.page_size;
  c.num_pages = h->rd.num_pages;
  c.max_pages = h->rd.max_pages;
  c.block_table = h->block_table;
  c.commit = h->commit;
  c.err = h->ctx->err;
  return commit_launch(c, s, true);
}

int upload_layout(const std::vector<int64_t>& v, int64_t* dst) {
  return check_cuda(cudaMemcpy(dst, v.data(), v.size() * sizeof(int64_t), cudaMemcpyHostToDevice), "layout upload");
}
int upload_layout32(const std::vector<int32_t>& v, int32_t* dst) {
  return check_cuda(cudaMemcpy(dst, v.data(), v.size() * sizeof(int32_t), cudaMemcpyHostToDevice), "layout upload");
}

// plm/mask.py:42-65 for block sizes `blocks`.
void round_layout(const std::vector<int>& blocks, std::vector<int64_t>& relpos, std::vector<int64_t>& relaux,
                  std::vector<int32_t>& depth, std::vector<int32_t>& own) {
  const int n = int(blocks.size());
  relpos.clear();
  relaux.clear();
  depth.clear();
  own.clear();
  for (int d = 0; d < n; ++d) {
    relpos.push_back(d);
    relaux.push_back(-1);
    depth.push_back(d);
    own.push_back(kUnreachable);
  }
  int start = n;
  for (int d = 0; d < n; ++d) {
    for (int j = 0; j < blocks[d]; ++j) {
      relpos.push_back(d + j);
      relaux.push_back(d + j);
      depth.push_back(d);
      own.push_back(start);
    }
    start += blocks[d];
  }
}

int validate_create(const plm_model_desc* m, const plm_weight_ptrs* w, const plm_round_desc* r) {
  if (m->dtype != PLM_BF16 && m->dtype != PLM_F16) return fail(PLM_ERR_INVALID, "plm_create: dtype %d", m->dtype);
  if (m->num_layers < 1 || m->hidden % 64 != 0 || m->intermediate % 64 != 0 || m->head_dim % 64 != 0)
    return fail(PLM_ERR_INVALID, "plm_create: hidden / intermediate / head_dim must be multiples of 64");
  if ((m->num_heads * m->head_dim) % 64 != 0 || m->num_heads % m->num_kv_heads != 0)
    return fail(PLM_ERR_INVALID, "plm_create: heads %d / kv heads %d", m->num_heads, m->num_kv_heads);
  const plm_ptp_desc* ptp = w->ptp;
  if (ptp == nullptr && (m->vocab < m->top_m || m->aux_vocab < 32))
    return fail(PLM_ERR_INVALID, "plm_create: vocab / aux vocabulary");
  if (ptp != nullptr) {
    if (!ptp->embedding || ptp->num_embeddings < 1 || ptp->top_k < 1 || ptp->top_k > kIcdfMaxTopK ||
        ptp->top_k > m->vocab || m->vocab > kIcdfMaxVocab || ptp->rank < 0 || ptp->rank % 64 != 0 ||
        ptp->rank > 256)
      return fail(PLM_ERR_INVALID, "plm_create: PTP scheme (embeddings %d, top_k %d, rank %d, vocab %d)",
                  ptp->num_embeddings, ptp->top_k, ptp->rank, m->vocab);
  }
  if (r->k < 1 || r->k + r->k * r->k > 256 || r->k > 32)
    return fail(PLM_ERR_UNSUPPORTED, "plm_create: k=%d (round width must be <= 256)", r->k);
  if (r->page_size < 1 || r->num_pages < 1 || r->max_pages < 1)
    return fail(PLM_ERR_INVALID, "plm_create: paging");
  if (r->max_prefill < 1 || r->max_prefill > kMaxPrefillRows)
    return fail(PLM_ERR_INVALID, "plm_create: max_prefill %d (1..%d)", r->max_prefill, kMaxPrefillRows);
  if (!w->embed || !w->lm_head || !w->final_norm || !w->cos_sin || !w->qkv || !w->o || !w->gate_up || !w->down ||
      !w->input_norm || !w->post_norm || (ptp == nullptr && (!w->aux_vocab || !w->mask_aux)))
    return fail(PLM_ERR_INVALID, "plm_create: missing weight pointer");
  return PLM_OK;
}

}  // namespace
}  // namespace plm

using namespace plm;

extern "C" {

int plm_destroy(plm_handle* h) {
  if (h == nullptr) return PLM_OK;
  void* bufs[] = {h->x_norm, h->residual, h->y, h->q, h->attn, h->act, h->gathered, h->partials, h->positions,
                  h->slots,
                  h->verify_logits, h->best_val, h->best_idx, h->verify, h->flags, h->st_relpos, h->st_relaux,
                  h->r0_relpos, h->r0_relaux, h->st_depth, h->st_own, h->r0_depth, h->r0_own, h->causal_depth,
                  h->causal_own, h->kv, h->block_table, h->out, h->base, h->offset, h->anchor, h->pending,
                  h->round_sequence, h->sequence_step, h->aux_buf, h->prompt, h->chunk_offsets, h->stop, h->round_kv,
                  h->commit, h->aux_u, h->lora_hidden, h->lora_corr, h->block_ctr,
                  h->block_tiles, h->attn_tiles, h->x_tiles, h->act_tiles, h->attn_part, h->attn_arrive};
  for (void* b : bufs) cudaFree(b);
  mlp_schedule_destroy(&h->mlp);
  if (h->own_table) cudaFree(h->table);
  plm_ctx_destroy(h->ctx);
  delete h;
  return PLM_OK;
}

int plm_create(const plm_model_desc* m, const plm_weight_ptrs* w, const plm_round_desc* rd, plm_handle** out) {
  if (!m || !w || !rd || !out) return fail(PLM_ERR_INVALID, "plm_create: null argument");
  *out = nullptr;
  int st = validate_create(m, w, rd);
  if (st != PLM_OK) return st;
  plm_handle* h = new plm_handle();
  h->m = *m;
  h->rd = *rd;
  if (h->rd.seq_capacity < 1) h->rd.seq_capacity = 1 << 17;  // plm/decoder.py:86
  if (h->rd.aux_len < 1) h->rd.aux_len = 8192;               // plm/decoder.py:28
  const int K = rd->k;
  h->W = K + K * K;
  h->R = kMaxPrefillRows;
  st = plm_ctx_create(&h->ctx);
  auto guard = [&](int s) {
    if (s != PLM_OK) plm_destroy(h);
    return s;
  };
  if (st != PLM_OK) return guard(st);
  h->embed = w->embed;
  h->lm_head = w->lm_head;
  h->final_norm = w->final_norm;
  h->aux_vocab = w->aux_vocab;
  h->mask_aux = w->mask_aux;
  h->cos_sin = w->cos_sin;
  const int L = m->num_layers;
  h->qkv.assign(w->qkv, w->qkv + L);
  h->o.assign(w->o, w->o + L);
  h->gate_up.assign(w->gate_up, w->gate_up + L);
  h->down.assign(w->down, w->down + L);
  h->in_norm.assign(w->input_norm, w->input_norm + L);
  h->post_norm.assign(w->post_norm, w->post_norm + L);

  const int hidden = m->hidden, hd = m->head_dim, I = m->intermediate;
  const int q_size = m->num_heads * hd, kv_size = m->num_kv_heads * hd;
  // weight descriptors, once
  h->map_qkv.resize(L);
  h->map_o.resize(L);
  h->map_gate_up.resize(L);
  h->map_down.resize(L);
  for (int l = 0; l < L && st == PLM_OK; ++l) {
    plm_gemm_desc d = {};
    d.dtype = m->dtype;
    d.w = h->qkv[l], d.n_out = q_size + 2 * kv_size, d.k = hidden, d.epi.kind = PLM_EPI_QKV_ROPE;
    st = gemm_weight_map(&h->map_qkv[l], d);
    d.w = h->o[l], d.n_out = hidden, d.k = q_size, d.epi.kind = PLM_EPI_STORE;
    if (st == PLM_OK) st = gemm_weight_map(&h->map_o[l], d);
    d.w = h->gate_up[l], d.n_out = 2 * I, d.k = hidden, d.epi.kind = PLM_EPI_SILU_MUL;
    if (st == PLM_OK) st = gemm_weight_map(&h->map_gate_up[l], d);
    d.w = h->down[l], d.n_out = hidden, d.k = I, d.epi.kind = PLM_EPI_STORE;
    if (st == PLM_OK) st = gemm_weight_map(&h->map_down[l], d);
  }
  if (st == PLM_OK) {
    plm_gemm_desc d = {};
    d.dtype = m->dtype;
    d.w = h->lm_head, d.n_out = m->vocab, d.k = hidden, d.epi.kind = PLM_EPI_LOGITS;
    st = gemm_weight_map(&h->map_lm, d);
  }
  if (st != PLM_OK) return guard(st);

  const size_t R = size_t(h->R);
  const size_t widest = size_t(std::max(std::max(hidden, q_size), I));
  (void)widest;
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->x_norm), R * hidden, "x_norm");
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->residual), R * hidden, "residual");
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->y), R * hidden, "y");
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->q), R * q_size, "q");
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->attn), R * q_size, "attn");
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->act), R * I, "act");
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->gathered), size_t(16) * hidden, "gathered");
  if (st == PLM_OK) st = dev_alloc(&h->partials, size_t(kPartialSlices) * R * hidden, "projection partials");
  if (st == PLM_OK) st = dev_alloc(&h->positions, R, "positions");
  if (st == PLM_OK) st = dev_alloc(&h->slots, R, "slots");
  h->lm_tiles = (m->vocab + 127) / 128;
  if (st == PLM_OK) st = dev_alloc(&h->verify_logits, size_t(K) * m->vocab, "verify logits");
  if (st == PLM_OK) st = dev_alloc(&h->best_val, size_t(h->lm_tiles) * h->W, "argmax partials");
  if (st == PLM_OK) st = dev_alloc(&h->best_idx, size_t(h->lm_tiles) * h->W, "argmax partials");
  if (st == PLM_OK) st = dev_alloc(&h->verify, 32, "verify");
  if (st == PLM_OK) st = dev_alloc(&h->flags, 32, "flags");
  // the PTP scheme: its table, the uniform stream and the adapters' maps and buffers
  const bool adapters = w->ptp != nullptr && w->ptp->rank > 0;
  if (st == PLM_OK && w->ptp != nullptr) {
    const plm_ptp_desc& pd = *w->ptp;
    h->ptp_embedding = pd.embedding;
    h->ptp_rows = pd.num_embeddings;
    h->ptp_top_k = pd.top_k;
    h->lora_rank = pd.rank;
    st = dev_alloc(&h->aux_u, size_t(h->rd.aux_len), "uniform stream");
    if (st == PLM_OK) st = check_cuda(cudaMemset(h->aux_u, 0, size_t(h->rd.aux_len) * 4), "uniform stream");
    h->lora.assign(L, {});
    const void* const* const As[4] = {pd.qkv_a, pd.o_a, pd.gate_up_a, pd.down_a};
    const void* const* const Bs[4] = {pd.qkv_b, pd.o_b, pd.gate_up_b, pd.down_b};
    const int ins[4] = {hidden, q_size, hidden, I};
    const std::vector<int> outs[4] = {{q_size, kv_size, kv_size}, {hidden}, {I, I}, {hidden}};
    for (int l = 0; l < L && adapters && st == PLM_OK; ++l) {
      for (int pj = 0; pj < 4 && st == PLM_OK; ++pj) {
        if (As[pj] == nullptr || Bs[pj] == nullptr || As[pj][l] == nullptr || Bs[pj][l] == nullptr) continue;
        int out0 = 0;
        for (size_t sh = 0; sh < outs[pj].size() && st == PLM_OK; ++sh) {
          plm_handle::LoraShard z;
          z.a = static_cast<const __nv_bfloat16*>(As[pj][l]) + sh * size_t(pd.rank) * ins[pj];
          z.b = static_cast<const __nv_bfloat16*>(Bs[pj][l]) + size_t(out0) * pd.rank;
          z.out0 = out0;
          z.width = outs[pj][sh];
          plm_gemm_desc d = {};
          d.dtype = m->dtype;
          d.w = z.a, d.n_out = pd.rank, d.k = ins[pj], d.epi.kind = PLM_EPI_STORE;
          st = gemm_weight_map(&z.map_a, d);
          d.w = z.b, d.n_out = z.width, d.k = pd.rank, d.epi.kind = PLM_EPI_PARTIAL;
          if (st == PLM_OK) st = gemm_weight_map(&z.map_b, d);
          h->lora[l][pj].push_back(z);
          out0 += z.width;
        }
      }
    }
    const size_t widest_out = size_t(std::max({q_size + 2 * kv_size, 2 * I, hidden}));
    if (st == PLM_OK && adapters)
      st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->lora_hidden), size_t(3) * R * pd.rank, "adapter rows");
    if (st == PLM_OK && adapters) st = dev_alloc(&h->lora_corr, R * widest_out, "adapter corrections");
  }
  // The layer block fuses o, its norm, gate_up and down; a model with adapters runs them as separate launches.
  if (st == PLM_OK && rd->separate_mlp == 0 && !adapters && hidden % 128 == 0 && I % 128 == 0 && q_size % 128 == 0 &&
      hidden <= 4096) {
    st = mlp_schedule_create(h->ctx->num_sms, hidden, I, q_size, &h->mlp);
    // row tiles of up to kMlpMaxRows rows, zeroed once (rows past a forward's count are read but never stored)
    const size_t tile_elems[3] = {size_t(kMlpMaxRows) * q_size, size_t(kMlpMaxRows) * hidden, size_t(kMlpMaxRows) * I};
    void** tiles[3] = {&h->attn_tiles, &h->x_tiles, &h->act_tiles};
    for (int i = 0; i < 3 && st == PLM_OK; ++i) {
      st = check_cuda(cudaMalloc(tiles[i], tile_elems[i] * 2), "row tiles");
      if (st == PLM_OK) st = check_cuda(cudaMemset(*tiles[i], 0, tile_elems[i] * 2), "memset");
    }
    if (st == PLM_OK) st = dev_alloc(&h->block_ctr, size_t(4) * L, "layer block counters");
    if (st == PLM_OK) st = check_cuda(cudaMemset(h->block_ctr, 0, size_t(4) * L * sizeof(int)), "memset");
    // the o, gate_up and down weights are read once here into their packed layout
    h->block_o_bytes = packed_tiles_bytes(hidden, q_size, 0);
    h->block_gate_up_bytes = packed_tiles_bytes(2 * I, hidden, I);
    h->block_layer_bytes = h->block_o_bytes + h->block_gate_up_bytes + packed_tiles_bytes(hidden, I, 0);
    if (st == PLM_OK)
      st = check_cuda(cudaMalloc(&h->block_tiles, size_t(L) * h->block_layer_bytes), "packed layer weights");
    for (int l = 0; l < L && st == PLM_OK; ++l) {
      uint8_t* dst = static_cast<uint8_t*>(h->block_tiles) + size_t(l) * h->block_layer_bytes;
      st = pack_weight_tiles(h->o[l], hidden, q_size, 0, dst, nullptr);
      if (st == PLM_OK) st = pack_weight_tiles(h->gate_up[l], 2 * I, hidden, I, dst + h->block_o_bytes, nullptr);
      if (st == PLM_OK)
        st = pack_weight_tiles(h->down[l], hidden, I, 0, dst + h->block_o_bytes + h->block_gate_up_bytes, nullptr);
    }
    if (st == PLM_OK) st = check_cuda(cudaDeviceSynchronize(), "packing the layer weights");
  }
  if (st != PLM_OK) return guard(st);
  // zero the activations once: rows past `rows` are read by TMA boxes but never stored
  {
    const std::pair<void*, size_t> zeroed[] = {{h->x_norm, R * hidden * 2}, {h->residual, R * hidden * 2},
                                               {h->y, R * hidden * 2},      {h->q, R * q_size * 2},
                                               {h->attn, R * q_size * 2},   {h->act, R * I * 2},
                                               {h->gathered, size_t(16) * hidden * 2}};
    for (const auto& z : zeroed)
      if (st == PLM_OK) st = check_cuda(cudaMemset(z.first, 0, z.second), "plm_create: zeroing the activations");
  }
  if (st != PLM_OK) return guard(st);

  // layouts: steady round [k] * k, round 0 [W - 1] (plm/decoder.py:145-146), causal chunk rows
  std::vector<int64_t> relpos, relaux;
  std::vector<int32_t> depth, own;
  round_layout(std::vector<int>(K, K), relpos, relaux, depth, own);
  st = dev_alloc(&h->st_relpos, h->W, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->st_relaux, h->W, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->st_depth, h->W, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->st_own, h->W, "layout");
  if (st == PLM_OK) st = upload_layout(relpos, h->st_relpos);
  if (st == PLM_OK) st = upload_layout(relaux, h->st_relaux);
  if (st == PLM_OK) st = upload_layout32(depth, h->st_depth);
  if (st == PLM_OK) st = upload_layout32(own, h->st_own);
  round_layout(std::vector<int>(1, h->W - 1), relpos, relaux, depth, own);
  if (st == PLM_OK) st = dev_alloc(&h->r0_relpos, h->W, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->r0_relaux, h->W, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->r0_depth, h->W, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->r0_own, h->W, "layout");
  if (st == PLM_OK) st = upload_layout(relpos, h->r0_relpos);
  if (st == PLM_OK) st = upload_layout(relaux, h->r0_relaux);
  if (st == PLM_OK) st = upload_layout32(depth, h->r0_depth);
  if (st == PLM_OK) st = upload_layout32(own, h->r0_own);
  std::vector<int32_t> causal(kMaxPrefillRows), unreachable(kMaxPrefillRows, kUnreachable);
  for (int i = 0; i < kMaxPrefillRows; ++i) causal[i] = i;
  if (st == PLM_OK) st = dev_alloc(&h->causal_depth, kMaxPrefillRows, "layout");
  if (st == PLM_OK) st = dev_alloc(&h->causal_own, kMaxPrefillRows, "layout");
  if (st == PLM_OK) st = upload_layout32(causal, h->causal_depth);
  if (st == PLM_OK) st = upload_layout32(unreachable, h->causal_own);
  if (st != PLM_OK) return guard(st);

  // paged KV pool [layer][K|V][num_pages][kv_heads][page_size][head_dim] and an identity block table
  h->plane_elems = size_t(rd->num_pages) * m->num_kv_heads * rd->page_size * hd;
  st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->kv), size_t(L) * 2 * h->plane_elems, "KV pool");
  if (st == PLM_OK) st = check_cuda(cudaMemset(h->kv, 0, size_t(L) * 2 * h->plane_elems * 2), "KV pool zero");
  const size_t round_elems = size_t(L) * 2 * h->W * m->num_kv_heads * hd;
  if (st == PLM_OK) st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->round_kv), round_elems, "round scratch");
  if (st == PLM_OK) st = check_cuda(cudaMemset(h->round_kv, 0, round_elems * 2), "round scratch zero");
  if (st == PLM_OK) st = dev_alloc(&h->commit, 2, "commit record");
  if (st == PLM_OK) st = check_cuda(cudaMemset(h->commit, 0, 2 * sizeof(int64_t)), "commit record zero");
  if (st == PLM_OK) st = dev_alloc(&h->block_table, rd->max_pages, "block table");
  if (st == PLM_OK) {
    std::vector<int32_t> ident(rd->max_pages);
    for (int i = 0; i < rd->max_pages; ++i) ident[i] = i < rd->num_pages ? i : -1;
    st = upload_layout32(ident, h->block_table);
  }
  // loop state
  if (st == PLM_OK) st = dev_alloc(&h->out, size_t(h->rd.out_capacity), "out");
  if (st == PLM_OK) st = dev_alloc(&h->base, 1, "state");
  if (st == PLM_OK) st = dev_alloc(&h->offset, 1, "state");
  if (st == PLM_OK) st = dev_alloc(&h->anchor, 1, "state");
  if (st == PLM_OK) st = dev_alloc(&h->pending, 32, "state");
  if (st == PLM_OK) st = dev_alloc(&h->round_sequence, size_t(h->rd.seq_capacity), "round sequence");
  if (st == PLM_OK) st = dev_alloc(&h->sequence_step, 1, "state");
  if (st == PLM_OK) st = dev_alloc(&h->aux_buf, size_t(h->rd.aux_len), "aux stream");
  if (st == PLM_OK) st = dev_alloc(&h->prompt, size_t(rd->max_pages) * rd->page_size, "prompt");
  if (st == PLM_OK) st = dev_alloc(&h->chunk_offsets, 4096, "chunk offsets");
  if (st == PLM_OK) st = dev_alloc(&h->stop, kStopWords, "stop block");
  if (st != PLM_OK) return guard(st);
  h->stop_host[kStopBudget] = INT64_MAX;  // no budget and no end-of-text until plm_set_stop
  h->stop_host[kStopEos] = -1;
  h->stop_host[kStopWindow] = 0;
  h->stop_host[kStopDone] = 0;
  st = check_cuda(cudaMemcpy(h->stop, h->stop_host, sizeof(h->stop_host), cudaMemcpyHostToDevice), "stop block");
  if (st != PLM_OK) return guard(st);
  {
    const struct {
      void* p;
      int value;
      size_t bytes;
    } init[] = {{h->out, 0xff, size_t(h->rd.out_capacity) * 8},
                {h->base, 0, 8},
                {h->offset, 0, 8},
                {h->anchor, 0, 8},
                {h->pending, 0, 32 * 8},
                {h->round_sequence, 0, size_t(h->rd.seq_capacity) * 8},
                {h->sequence_step, 0, 8},
                {h->aux_buf, 0, size_t(h->rd.aux_len) * 8},
                {h->prompt, 0, size_t(rd->max_pages) * rd->page_size * 8}};
    for (const auto& z : init)
      if (st == PLM_OK) st = check_cuda(cudaMemset(z.p, z.value, z.bytes), "plm_create: initialising the round state");
  }
  if (st != PLM_OK) return guard(st);
  h->attn_splits_round = attention_splits(m->num_heads, (h->W + 63) / 64, h->ctx->num_sms,
                                          int64_t(rd->max_pages) * rd->page_size, true);
  if (h->attn_splits_round > 8 &&
      !attention_two_clusters_fit(m->num_heads, (h->W + 63) / 64, hd, m->dtype))  // both clusters must be resident
    h->attn_splits_round = 8;
  if (h->attn_splits_round > 8) {
    const int q_tiles = (h->W + 63) / 64;
    const size_t n_arrive = attention_arrive_ints(m->num_heads, q_tiles);
    st = dev_alloc(&h->attn_part, attention_part_floats(m->num_heads, q_tiles, hd), "attention partials");
    if (st == PLM_OK) st = dev_alloc(&h->attn_arrive, n_arrive, "attention counters");
    if (st == PLM_OK) st = check_cuda(cudaMemset(h->attn_arrive, 0, n_arrive * sizeof(int)), "memset");
    if (st != PLM_OK) return guard(st);
  }

  // the Voronoi cost table -(aux_vocab . lm_head^T)^T, [vocab][A] (plm/auxiliary.py:56-65)
  if (w->table != nullptr || w->ptp != nullptr) {  // the PTP scheme decodes without a cost table
    h->table = const_cast<void*>(w->table);
  } else {
    st = dev_alloc(reinterpret_cast<__nv_bfloat16**>(&h->table), size_t(m->vocab) * m->aux_vocab, "Voronoi table");
    if (st != PLM_OK) return guard(st);
    h->own_table = true;
    for (int a0 = 0; a0 < m->aux_vocab && st == PLM_OK; a0 += 256) {
      plm_gemm_desc d = {};
      d.dtype = m->dtype;
      d.w = h->lm_head;
      d.n_out = m->vocab;
      d.k = hidden;
      d.x = static_cast<const __nv_bfloat16*>(h->aux_vocab) + size_t(a0) * hidden;
      d.rows = std::min(256, m->aux_vocab - a0);
      d.x_rows = d.rows;
      d.epi.kind = PLM_EPI_TABLE;
      d.epi.table = h->table;
      d.epi.aux = m->aux_vocab;
      d.epi.a0 = a0;
      CUtensorMap mx;
      st = gemm_row_map(&mx, d);
      if (st == PLM_OK) st = gemm_launch(h->ctx, d, &h->map_lm, &mx, nullptr, false);
    }
  }
  if (st == PLM_OK) st = check_cuda(cudaDeviceSynchronize(), "plm_create");
  if (st != PLM_OK) return guard(st);
  *out = h;
  return PLM_OK;
}

int plm_set_block_table(plm_handle* h, const int32_t* table, int32_t n) {
  if (!h || !table || n < 1 || n > h->rd.max_pages) return fail(PLM_ERR_INVALID, "plm_set_block_table: %d entries", n);
  for (int i = 0; i < n; ++i)
    if (table[i] < 0 || table[i] >= h->rd.num_pages)
      return fail(PLM_ERR_INVALID, "plm_set_block_table: entry %d = %d outside the pool", i, table[i]);
  return check_cuda(cudaMemcpy(h->block_table, table, size_t(n) * 4, cudaMemcpyHostToDevice), "block table");
}

int plm_set_aux_stream(plm_handle* h, const int64_t* cells, int64_t n, void* stream) {
  if (!h || !cells || n < 1 || n > h->rd.aux_len) return fail(PLM_ERR_INVALID, "plm_set_aux_stream: n=%lld", (long long)n);
  return check_cuda(cudaMemcpyAsync(h->aux_buf, cells, size_t(n) * 8, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                    "aux stream copy");
}

int plm_set_aux_uniforms(plm_handle* h, const float* u, int64_t n, void* stream) {
  if (!h || !u || n < 1 || n > h->rd.aux_len) return fail(PLM_ERR_INVALID, "plm_set_aux_uniforms: n=%lld", (long long)n);
  if (h->aux_u == nullptr) return fail(PLM_ERR_INVALID, "plm_set_aux_uniforms: the handle's scheme has no uniforms");
  return check_cuda(cudaMemcpyAsync(h->aux_u, u, size_t(n) * 4, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                    "uniform stream copy");
}

int plm_load_prompt(plm_handle* h, const int64_t* ids, int64_t n, void* stream) {
  const int64_t cap = int64_t(h ? h->rd.max_pages : 0) * (h ? h->rd.page_size : 0);
  if (!h || !ids || n < 1 || n > cap) return fail(PLM_ERR_INVALID, "plm_load_prompt: %lld tokens", (long long)n);
  h->prompt_len = n;
  return check_cuda(cudaMemcpyAsync(h->prompt, ids, size_t(n) * 8, cudaMemcpyDefault, static_cast<cudaStream_t>(stream)),
                    "prompt copy");
}

int plm_set_stop(plm_handle* h, int64_t max_tokens, int64_t eos_token, int64_t eos_window, void* stream) {
  if (!h || eos_token < -1 || eos_window < 0)
    return fail(PLM_ERR_INVALID, "plm_set_stop: eos %lld, window %lld", (long long)eos_token, (long long)eos_window);
  // The copy reads the handle's own host array: it must not change until the copy has run, so a stream that is
  // still behind the previous plm_set_stop is synchronised first.
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = check_cuda(cudaStreamSynchronize(s), "plm_set_stop: synchronize");
  if (st != PLM_OK) return st;
  h->stop_host[kStopBudget] = max_tokens;
  h->stop_host[kStopEos] = eos_token;
  h->stop_host[kStopWindow] = eos_window;
  h->stop_host[kStopDone] = 0;
  return check_cuda(cudaMemcpyAsync(h->stop, h->stop_host, sizeof(h->stop_host), cudaMemcpyHostToDevice, s),
                    "plm_set_stop: copy");
}

int plm_prefill(plm_handle* h, void* stream) {
  if (!h || h->prompt_len < 1) return fail(PLM_ERR_INVALID, "plm_prefill: no prompt loaded");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int width = h->rd.max_prefill;
  const int64_t n = h->prompt_len;
  const int chunks = int((n + width - 1) / width);
  if (chunks > 4096) return fail(PLM_ERR_INVALID, "plm_prefill: prompt too long");
  if (n + 2 * h->W > int64_t(h->rd.max_pages) * h->rd.page_size)
    return fail(PLM_ERR_INVALID, "plm_prefill: prompt of %lld leaves no room for a round", (long long)n);
  std::vector<int64_t> offs(chunks);
  for (int c = 0; c < chunks; ++c) offs[c] = int64_t(c) * width;
  int st = check_cuda(cudaMemcpyAsync(h->chunk_offsets, offs.data(), chunks * 8, cudaMemcpyHostToDevice, s),
                      "chunk offsets");
  if (st != PLM_OK) return st;
  for (int c = 0; c < chunks && st == PLM_OK; ++c) {
    const int rows = int(std::min<int64_t>(width, n - offs[c]));
    const bool last = c + 1 == chunks;
    const int splits = attention_splits(h->m.num_heads, (rows + 63) / 64, h->ctx->num_sms, offs[c] + rows);
    st = forward(h, kProloguePrefill, rows, h->chunk_offsets + c, nullptr, h->st_relaux, h->causal_depth,
                 h->causal_own, splits, last ? int(n - 1 - offs[c]) : -1, s);
  }
  if (st == PLM_OK) st = lm_head(h, h->gathered, 1, 1, s);
  if (st == PLM_OK) st = verify(h, 1, kBookFirstToken, nullptr, s);
  return st;
}

int plm_round0(plm_handle* h, void* stream) {
  if (!h) return fail(PLM_ERR_INVALID, "plm_round0: null handle");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = forward(h, kPrologueRound0, h->W, h->offset, h->r0_relpos, h->r0_relaux, h->r0_depth, h->r0_own,
                   h->attn_splits_round, -1, s);
  if (st == PLM_OK) st = lm_head(h, h->x_norm, h->W, 1, s);
  if (st == PLM_OK) st = verify(h, 1, kBookRound0, h->base, s);
  if (st == PLM_OK) st = commit_rows(h, s);
  return st;
}

int plm_layer_block(plm_handle* h, int32_t layer, int32_t rows, void* stream) {
  if (!h) return fail(PLM_ERR_INVALID, "plm_layer_block: null handle");
  if (h->mlp.sched == nullptr) return fail(PLM_ERR_UNSUPPORTED, "plm_layer_block: the handle runs separate launches");
  if (layer < 0 || layer >= h->m.num_layers || rows < 1 || rows > kMlpMaxRows)
    return fail(PLM_ERR_INVALID, "plm_layer_block: layer %d, rows %d", layer, rows);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the phase counters of this layer start at zero, as after a forward's prologue
  int st = check_cuda(cudaMemsetAsync(h->block_ctr + 4 * layer, 0, 4 * sizeof(int), s), "plm_layer_block counters");
  if (st == PLM_OK) st = layer_block_launch(h, layer, rows, s);
  return st;
}

int plm_round(plm_handle* h, void* stream) {
  if (!h) return fail(PLM_ERR_INVALID, "plm_round: null handle");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = forward(h, kPrologueSteady, h->W, h->offset, h->st_relpos, h->st_relaux, h->st_depth, h->st_own,
                   h->attn_splits_round, -1, s);
  if (st == PLM_OK) st = lm_head(h, h->x_norm, h->W, h->rd.k, s);
  if (st == PLM_OK) st = verify(h, h->rd.k, kBookSteady, h->base, s);
  if (st == PLM_OK) st = commit_rows(h, s);
  return st;
}

int plm_state(plm_handle* h, plm_state_ptrs* p) {
  if (!h || !p) return fail(PLM_ERR_INVALID, "plm_state: null argument");
  p->out = h->out;
  p->base = h->base;
  p->offset = h->offset;
  p->anchor = h->anchor;
  p->pending = h->pending;
  p->round_sequence = h->round_sequence;
  p->sequence_step = h->sequence_step;
  p->aux_buf = h->aux_buf;
  p->block_table = h->block_table;
  p->verify_logits = h->verify_logits;
  p->best_val = h->best_val;
  p->best_idx = h->best_idx;
  p->verify = h->verify;
  p->flags = h->flags;
  p->hidden_normed = h->x_norm;
  p->kv_cache = h->kv;
  p->table = h->table;
  p->out_capacity = h->rd.out_capacity;
  p->seq_capacity = h->rd.seq_capacity;
  p->aux_len = h->rd.aux_len;
  p->plane_elems = int64_t(h->plane_elems);
  p->width = h->W;
  p->lm_tiles = h->lm_tiles;
  p->row_capacity = h->R;
  p->stop = h->stop;
  p->round_kv = h->round_kv;
  p->commit = h->commit;
  return PLM_OK;
}

int plm_check(plm_handle* h, int32_t* device_error) {
  if (!h) return fail(PLM_ERR_INVALID, "plm_check: null handle");
  return plm_ctx_check(h->ctx, device_error);
}

}  // extern "C"

extern "C" int plm_borrowed_weights(plm_handle* h, int32_t* groups) {
  if (h == nullptr || groups == nullptr) return fail(PLM_ERR_INVALID, "plm_borrowed_weights: null argument");
  // qkv, lm_head, the norms and embeddings are always read in place; o, gate_up and down only without packed copies
  *groups = PLM_WEIGHTS_IN_PLACE | (h->block_tiles == nullptr ? PLM_WEIGHTS_BLOCK : 0);
  return PLM_OK;
}
