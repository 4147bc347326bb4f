/* C ABI of libplm_native.so: the B200 (sm_100a) kernels of the PLM decoding round.
 *
 * Conventions
 *   - Every function returns an int status: PLM_OK (0) or a negative PLM_ERR_* code; plm_last_error() gives the
 *     message of the calling thread's last failure.
 *   - All tensor arguments are plain device pointers (bf16/f16 storage, fp32 or int32/int64 as stated) and sizes;
 *     no framework types cross this boundary. `stream` is a cudaStream_t passed as void*.
 *   - Launch functions only enqueue work on `stream`; they never synchronise, so they can be captured into a
 *     CUDA graph. Device-side faults are not raised: a kernel that meets an index out of range or a wait that
 *     runs out of time records a code in the context's device error word (plm_ctx_check reads it).
 *   - A context (plm_ctx) owns the device error word and the kernels' arrival counters. It is bound to the device
 *     current at creation and must only be used from one host thread at a time.
 *
 * Reference interfaces replaced (paths inside justuswill/PLM-anon):
 *   plm_gemm        plm/fast_gemm.py:82-97 (triton_linear) installed at plm/fast_gemm.py:100-113, and the
 *                   vLLM unquantized linear it patches; epilogues fuse vLLM's SiluAndMul, rotary embedding and
 *                   reshape_and_cache_flash (called from plm/decoder.py:250-259 through the Llama forward) and
 *                   compute_logits + argmax (plm/decoder.py:318,362).
 *   plm_verify_decode  LogitVoronoiAuxiliary.decode_unmasked (plm/auxiliary.py:67-75) -> Voronoi.assign
 *                   (plm/iterate.py:322-342), nucleus_acceptance / floor_acceptance (plm/decoder.py:71-82) and
 *                   RoundDecoder._epilogue / _round0 bookkeeping (plm/decoder.py:351-365, 275-310, 384).
 *   plm_attention   FlexAttention under RoundMaskView (plm/mask.py:23-29, installed at plm/decoder.py:148-150,
 *                   165-169; vllm/v1/attention/backends/flex_attention.py:1070-1205).
 *   plm_kv_append   reshape_and_cache_flash (flex_attention.py:1047-1068) at the slots of plm/decoder.py:347.
 *   plm_add_rmsnorm vLLM RMSNorm with residual (fused_add_rms_norm) between the Llama sublayers.
 *   plm_commit      the KV commit of a round: the reference's implicit commit (offset += nc + 1 with the verify
 *                   rows already in place, plm/decoder.py:351-365) made explicit as a copy of the accepted verify
 *                   rows from round scratch into the permanent pages, the KV move of eagle3/tree.py:263-279.
 *   plm_create / plm_round / plm_round0 / plm_prefill / plm_state
 *                   RoundDecoder (plm/decoder.py:85-467): construction and state (88-146), the steady round
 *                   (312-324), round 0 (275-310), the prefill (369-403); RoundConfig.build (plm/rounds.py:71-81)
 *                   creates one. plm_set_aux_stream replaces _fill_aux (decoder.py:407-412).
 */
#ifndef PLM_NATIVE_H
#define PLM_NATIVE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define PLM_ABI_VERSION 8

enum plm_status {
  PLM_OK = 0,
  PLM_ERR_INVALID = -1,     /* bad argument (shape, pointer, dtype) */
  PLM_ERR_CUDA = -2,        /* a CUDA runtime call failed */
  PLM_ERR_DEVICE = -3,      /* a kernel recorded an error in the device error word */
  PLM_ERR_UNSUPPORTED = -4, /* a shape or option this build has no kernel for */
  PLM_ERR_NOMEM = -5        /* device allocation failed */
};

enum plm_dtype { PLM_BF16 = 0, PLM_F16 = 1 };

enum plm_epilogue {
  PLM_EPI_STORE = 0,    /* out[r][n] = Y[r][n] in the model dtype */
  PLM_EPI_SILU_MUL = 1, /* out[r][j] = silu(Y[r][j]) * Y[r][gate_offset + j], j < gate_offset */
  PLM_EPI_QKV_ROPE = 2, /* neox RoPE on q,k; q -> q_out, k,v -> paged cache at slots[r] */
  PLM_EPI_LOGITS = 3,   /* rows < n_verify: fp32 logits; other rows: per-tile (max, first index) */
  PLM_EPI_TABLE = 4,    /* table[n][a0 + r] = -Y[r][n] (the Voronoi cost table) */
  PLM_EPI_PARTIAL = 5   /* fp32 k-split partials: ((float*)out)[(s * rows + r) * ldo + n] for split s < splits
                           (splits must be given, <= 16); the consumer sums them in split order */
};

enum plm_accept_rule { PLM_RULE_NUCLEUS = 0, PLM_RULE_FLOOR = 1 };

enum plm_book_mode {
  PLM_BOOK_NONE = 0,        /* decode only */
  PLM_BOOK_STEADY = 1,      /* steady round: acceptance, outputs, next pending, base/offset commit */
  PLM_BOOK_ROUND0 = 2,      /* round 0: one verify row, nothing accepted */
  PLM_BOOK_FIRST_TOKEN = 3  /* after the prefill: first token, request state reset */
};

typedef struct plm_ctx plm_ctx;

/* Epilogue operands of plm_gemm (fields not used by the selected epilogue are ignored). */
typedef struct plm_gemm_epilogue {
  int32_t kind; /* enum plm_epilogue */
  int32_t gate_offset;
  /* PLM_EPI_QKV_ROPE */
  void* q_out;
  void* k_cache; /* [num_pages][num_kv_heads][page_size][head_dim] */
  void* v_cache;
  const int32_t* positions; /* [rows] */
  const int64_t* slots;     /* [rows] physical slot = page * page_size + index in page */
  const void* cos_sin;      /* [max_pos][head_dim] model dtype: cos | sin halves */
  int32_t num_heads, num_kv_heads, head_dim, page_size;
  int64_t num_slots;
  int32_t max_pos;
  /* PLM_EPI_LOGITS */
  float* verify_logits; /* [n_verify][vocab] */
  float* best_val;      /* [n_tiles][rows] */
  int32_t* best_idx;    /* [n_tiles][rows] */
  int32_t n_verify;
  int32_t vocab;
  /* PLM_EPI_TABLE */
  void* table;
  int32_t aux;
  int32_t a0;
  /* PLM_EPI_QKV_ROPE, PLM_EPI_SILU_MUL (nullable): fp32 corrections corr[(r - corr_from) * corr_ld + n] added to
   * output n of rows r >= corr_from before the epilogue's rotary embedding or SiLU, as y = round(round(y) + corr):
   * a gated-LoRA adapter's output on the gated rows (plm/gated_lora.py:45-57) */
  const float* corr;
  int32_t corr_from;
  int32_t corr_ld;
} plm_gemm_epilogue;

typedef struct plm_gemm_desc {
  int32_t dtype;  /* enum plm_dtype */
  const void* w;  /* [n_out][k] row-major weights */
  int32_t n_out;
  int32_t k;      /* multiple of 64 */
  const void* x;  /* [x_rows][k] row-major activations, 16-byte aligned */
  int32_t x_rows; /* allocated rows of x (>= rows) */
  int32_t rows;   /* rows to compute, 1..256 */
  void* out;      /* PLM_EPI_STORE / PLM_EPI_SILU_MUL / PLM_EPI_PARTIAL output */
  int32_t ldo;    /* output row stride in elements */
  int32_t splits; /* 0 = choose automatically */
  plm_gemm_epilogue epi;
} plm_gemm_desc;

/* Round state the verify kernel's last CTA updates (plm/decoder.py:351-365, 275-310, 384). */
typedef struct plm_bookkeeping {
  int32_t mode; /* enum plm_book_mode */
  int32_t k;
  const float* best_val;   /* [n_tiles][rows] lm_head per-tile row maxima (PLM_EPI_LOGITS) */
  const int32_t* best_idx; /* [n_tiles][rows] */
  int32_t n_tiles;
  int32_t rows;
  int64_t* out; /* [out_cap] */
  int64_t out_cap;
  int64_t* base;
  int64_t* offset;
  int64_t* anchor;
  int64_t* pending; /* [k - 1] */
  int64_t* round_sequence; /* [seq_cap] */
  int64_t seq_cap;
  int64_t* sequence_step;
  int64_t prompt_len;
  /* Nullable request stop block, int64[4]: token budget, end-of-text id (-1: none), end-of-text window, done flag.
   * A steady round whose bookkeeping finds the done flag set commits nothing; one that leaves base >= budget, or
   * confirms the end-of-text id at an output position below the window, sets it (the stop test of the reference's
   * host loop, plm/decoder.py:414-439). The first-token bookkeeping clears it. */
  int64_t* stop;
  /* Nullable commit record, int64[2], written by steady and round-0 bookkeeping: the first logical KV index and the
   * number of round rows to commit (nc + 1; 0 when the round committed nothing because the request had stopped).
   * plm_commit reads it. */
  int64_t* commit;
} plm_bookkeeping;

/* One verify decode per row: Voronoi assignment of the row's logits (plm/iterate.py:322-342 through
 * plm/auxiliary.py:67-75) and, for rows < n_accept, the relaxed acceptance rule (plm/decoder.py:71-82). */
typedef struct plm_verify_desc {
  int32_t dtype;
  const float* logits; /* [n_rows][logits_stride] */
  int32_t n_rows;
  int32_t vocab;
  int64_t logits_stride;
  const void* table; /* [vocab][aux] */
  int32_t aux;
  const int64_t* aux_buf;
  int64_t aux_len;
  const int64_t* aux_base; /* device scalar (nullable) */
  int32_t aux_row_offset;  /* row r reads aux_buf[*aux_base + aux_row_offset + r] */
  const int64_t* pending;  /* [n_accept] */
  int32_t n_accept;
  int32_t rule; /* enum plm_accept_rule */
  float threshold;
  int32_t top_m, shortlist, rounds, sweeps;
  double epsilon, refocus, endpoint;
  int64_t* verify; /* [n_rows] */
  int32_t* flags;  /* [n_rows] */
  int32_t* dbg_tokens;
  int32_t* dbg_counts;
  float* dbg_bias;
  float* dbg_stats;
  int32_t* dbg_sigma;
  int64_t* dbg_phase_ns; /* [n_rows][16] nanoseconds from kernel start to the end of each phase (diagnostic) */
  plm_bookkeeping book;
} plm_verify_desc;

/* Paged attention of `rows` query rows at logical KV indices [*offset, *offset + rows) under the round mask:
 * key kv is visible to row r iff kv < *offset + rows and (kv < *offset or kv - *offset <= depth[r] or
 * (kv - *offset >= own_start[r] and kv <= *offset + r)) (plm/mask.py:23-29). */
typedef struct plm_attention_desc {
  int32_t dtype;
  const void* q;               /* [rows][num_heads][head_dim] */
  const void* k_cache;         /* [num_pages][num_kv_heads][page_size][head_dim] */
  const void* v_cache;
  const int32_t* block_table;  /* [max_pages] */
  int32_t max_pages, num_pages, page_size;
  const int64_t* offset;       /* device scalar */
  int32_t rows;
  const int32_t* depth;        /* [rows] */
  const int32_t* own_start;    /* [rows] */
  int32_t num_heads, num_kv_heads, head_dim;
  void* out;                   /* [rows][num_heads * head_dim] */
  int32_t splits;              /* 0 = choose from max_keys; else 1 to 8 (one cluster), or 16: two clusters of
                                  8 merged through buffers the context owns (the second cluster works only when every
                                  split gets four key tiles); not under stream capture on its first use */
  int64_t max_keys;
} plm_attention_desc;

/* Scatter K/V rows [rows][num_kv_heads][head_dim] to logical KV indices *offset + r (reshape_and_cache_flash). */
typedef struct plm_kv_append_desc {
  int32_t dtype;
  const void* k;
  const void* v;
  void* k_cache;
  void* v_cache;
  const int32_t* block_table;
  int32_t max_pages, num_pages, page_size;
  const int64_t* offset;
  int32_t rows, num_kv_heads, head_dim;
} plm_kv_append_desc;

/* Copies round rows commit[0] .. commit[0] + commit[1] - 1 (logical KV indices) of every layer's K and V from the
 * round scratch into the paged cache through the block table: row j of the scratch goes to logical index
 * commit[0] + j. The commit record is read on the device (the verify bookkeeping writes it), so the call can follow
 * it in the same stream or graph. Rows past commit[1] and every other slot of the cache are left as they are. */
typedef struct plm_commit_desc {
  int32_t dtype;
  const void* scratch;        /* [layers][2][scratch_rows][num_kv_heads][head_dim] */
  int32_t scratch_rows;
  void* kv_cache;             /* [layers][2][num_pages][num_kv_heads][page_size][head_dim] */
  int64_t plane_elems;        /* num_pages * num_kv_heads * page_size * head_dim */
  int32_t layers, num_kv_heads, head_dim, page_size, num_pages, max_pages;
  const int32_t* block_table; /* [max_pages] */
  const int64_t* commit;      /* device int64[2]: first logical index, rows */
} plm_commit_desc;

/* residual <- x + residual; normed <- RMSNorm(residual_fp32) * weight (vLLM fused_add_rms_norm). */
typedef struct plm_add_rmsnorm_desc {
  int32_t dtype;
  const void* x;
  void* residual;
  void* normed;
  const void* weight;
  int32_t rows, hidden;
  float eps;
  int32_t gather_row; /* -1: none; else also copy that normed row to `gathered` */
  void* gathered;
  /* With partials != NULL, x is ignored and x[r] = bf16(sum over s < n_partials of partials[s * partial_stride +
   * r * hidden + i]) summed in split order (the PLM_EPI_PARTIAL output of the GEMM before this norm). */
  const float* partials;
  int32_t n_partials;
  int64_t partial_stride;
  /* Nullable: x[r] = round(x[r] + corr[(r - corr_from) * corr_ld + i]) for rows r >= corr_from before the residual
   * add (a gated-LoRA adapter's output on the gated rows, plm/gated_lora.py:45-57) */
  const float* corr;
  int32_t corr_from;
  int32_t corr_ld;
} plm_add_rmsnorm_desc;

/* ---- round engine (one handle = one request stream on one GPU, batch 1) ---- */
typedef struct plm_handle plm_handle;

/* Llama-architecture PLM (vLLM llama.py:81-314 with the auxiliary scheme of plm/auxiliary.py:17-75). */
typedef struct plm_model_desc {
  int32_t dtype;
  int32_t num_layers, hidden, num_heads, num_kv_heads, head_dim, intermediate;
  int32_t vocab;          /* text vocabulary: logits width */
  int32_t aux_vocab;      /* auxiliary vocabulary size A (power of two, 32..4096) */
  int32_t num_aux_tokens; /* ids in [vocab, vocab + num_aux_tokens) embed auxiliary vectors */
  float rms_eps;
  int32_t max_pos;        /* rows of the cos/sin table */
  int32_t top_m, shortlist, rounds, sweeps;
  double epsilon, refocus, endpoint;
} plm_model_desc;

/* The PTP scheme of the reference's gated-LoRA distilled model (plm/auxiliary.py:78-113, plm/gated_lora.py:35-90):
 * auxiliary rows blend rows of a float32 table at the request's uniforms, verify rows decode by inverse CDF over
 * the top_k probabilities, and each projection with adapters adds x A^T B^T on a round's gated rows (row 1 on in
 * round 0, row k on in a steady round, none in the prefill). Per layer and projection (nullable arrays, nullable
 * entries): A stacks the shards' down-projections [shards * rank][in]; B stacks their up-projections in output order
 * [out][rank], shard s of the output (q, k, v for qkv; gate, up for gate_up) reading rank slice s of x A^T. A handle
 * with adapters runs the MLP as separate launches. */
typedef struct plm_ptp_desc {
  const float* embedding; /* [num_embeddings][hidden] float32 */
  int32_t num_embeddings;
  int32_t top_k;          /* inverse-CDF bins, 1..256 */
  int32_t rank;           /* adapter rank (a multiple of 64; 0: no adapters) */
  const void* const* qkv_a;
  const void* const* qkv_b;
  const void* const* o_a;
  const void* const* o_b;
  const void* const* gate_up_a;
  const void* const* gate_up_b;
  const void* const* down_a;
  const void* const* down_b;
} plm_ptp_desc;

/* Borrowed device pointers; they must stay valid for the handle's lifetime. */
typedef struct plm_weight_ptrs {
  const void* embed;      /* [>= vocab][hidden] */
  const void* lm_head;    /* [>= vocab][hidden] */
  const void* final_norm; /* [hidden] */
  const void* aux_vocab;  /* [aux_vocab][hidden] */
  const void* mask_aux;   /* [hidden] */
  const void* cos_sin;    /* [max_pos][head_dim] */
  const void* const* qkv; /* per layer [(heads + 2 kv_heads) * head_dim][hidden] */
  const void* const* o;   /* per layer [hidden][heads * head_dim] */
  const void* const* gate_up; /* per layer [2 intermediate][hidden] */
  const void* const* down;    /* per layer [hidden][intermediate] */
  const void* const* input_norm;
  const void* const* post_norm;
  const void* table;      /* optional [vocab][aux_vocab] Voronoi table; NULL: built at creation */
  const plm_ptp_desc* ptp; /* NULL: the logit-Voronoi scheme of every PLM; else the PTP scheme (copied at creation) */
} plm_weight_ptrs;

typedef struct plm_round_desc {
  int32_t k;              /* verify rows; the round has k + k^2 rows */
  int32_t rule;           /* enum plm_accept_rule */
  float threshold;        /* nucleus mass (<= 0: exact match) or probability floor */
  int32_t page_size;
  int32_t num_pages;      /* physical pages in the KV pool */
  int32_t max_pages;      /* block-table entries (logical pages of one request) */
  int64_t out_capacity;   /* output token buffer */
  int64_t seq_capacity;   /* accepted-count record (0: 1 << 17) */
  int64_t aux_len;        /* auxiliary cell stream (0: 8192) */
  int32_t max_prefill;    /* rows per prefill chunk, 1..256 */
  int32_t separate_mlp;   /* 0: gate_up, SiLU and down of a forward of at most 128 rows run as one persistent
                             launch (default); 1: as two launches, like wider forwards */
} plm_round_desc;

/* Device addresses of a handle's state, for readers and for seeding synthetic workloads. */
typedef struct plm_state_ptrs {
  int64_t* out;
  int64_t* base;
  int64_t* offset;
  int64_t* anchor;
  int64_t* pending;
  int64_t* round_sequence;
  int64_t* sequence_step;
  int64_t* aux_buf;
  int32_t* block_table;
  float* verify_logits;  /* [k][vocab] */
  float* best_val;       /* [lm_tiles][width] */
  int32_t* best_idx;
  int64_t* verify;
  int32_t* flags;
  void* hidden_normed;   /* [row_capacity][hidden]: final-norm output of the last forward */
  void* kv_cache;        /* [layers][2][num_pages][kv_heads][page_size][head_dim] */
  void* table;
  int64_t out_capacity, seq_capacity, aux_len, plane_elems;
  int32_t width, lm_tiles, row_capacity;
  int64_t* stop;         /* [4] the request stop block (plm_bookkeeping.stop) */
  void* round_kv;        /* [layers][2][width][kv_heads][head_dim]: K and V of the last round's rows (scratch) */
  int64_t* commit;       /* [2] the last round's commit record (plm_bookkeeping.commit) */
} plm_state_ptrs;

/* ---- context ---- */
int plm_ctx_create(plm_ctx** out);
int plm_ctx_destroy(plm_ctx* ctx);
/* Synchronises the device, then returns the device error word in *device_error and clears it. */
int plm_ctx_check(plm_ctx* ctx, int32_t* device_error);
/* Number of output tiles plm_gemm uses for (epilogue kind, n_out): the leading size of best_val/best_idx. */
int plm_gemm_tiles(int32_t kind, int32_t n_out, int32_t gate_offset, int32_t* tiles);

/* ---- kernels ---- */
int plm_gemm(plm_ctx* ctx, const plm_gemm_desc* desc, void* stream);
/* Verify decode + acceptance + (optionally) the round bookkeeping, one CTA per row. */
int plm_verify_decode(plm_ctx* ctx, const plm_verify_desc* desc, void* stream);
/* plm_verify_decode without a context, allocating nothing. This entry point has no counterpart in the reference: it
 * serves callers that cannot allocate device memory, such as a host runtime bound over a foreign-function
 * interface whose device memory belongs to its own allocator, or a decode loop that must not stall (cudaMalloc and
 * cudaFree synchronise the device). Its scratch is a file-scope device array of 1024 bytes: the bookkeeping
 * arrival counter (zero at module load, reset to zero by every bookkeeping launch), the device error word used
 * when device_error is NULL, and 32 row slots for the decoded tokens and verdicts used when desc->verify or
 * desc->flags is NULL. More than 32 rows is rejected with PLM_ERR_INVALID. device_error, when given, is a device
 * int32 the caller has zeroed; the first device-side error code is written there. With device_error NULL, device-side
 * errors (an index out of range, a wait that ran out of time) go to the scratch's own error word, which the C ABI
 * cannot read back: callers that need to see them pass a zeroed device int32. The first call in a CUDA context
 * (with that device current) resolves the scratch's address with cudaGetSymbolAddress, so make it before any stream
 * capture. Calls on one device share the scratch: overlapping calls (other streams or threads) race. */
int plm_verify_decode_static(const plm_verify_desc* desc, int32_t* device_error, void* stream);

/* The PTP scheme's verify decode (plm/auxiliary.py:104-113, LinearInterpolationAuxiliary.decode_unmasked, which
 * the reference's RoundDecoder calls through _decode_verify at plm/decoder.py:260-262): per row, the softmax at
 * temperature 1, its top_k largest probabilities in token-id order renormalised, and the token of the first bin
 * whose right edge exceeds u[row] (the last edge is 1; ties at the top_k-th probability go to the lowest ids). */
typedef struct plm_icdf_desc {
  const float* logits; /* [n_rows][ld] float32 */
  int64_t ld;
  const float* u;      /* [n_rows] uniforms in [0, 1) */
  int32_t n_rows;
  int32_t vocab;       /* 1..53248 */
  int32_t top_k;       /* 1..256, at most vocab */
  int64_t* tokens;     /* [n_rows] out */
  int32_t* ids_out;    /* optional [n_rows][top_k] out: the chosen ids, ascending */
  float* edges_out;    /* optional [n_rows][top_k] out: the right bin edges */
} plm_icdf_desc;
int plm_icdf_decode(plm_ctx* ctx, const plm_icdf_desc* desc, void* stream);
int plm_attention(plm_ctx* ctx, const plm_attention_desc* desc, void* stream);
int plm_kv_append(plm_ctx* ctx, const plm_kv_append_desc* desc, void* stream);
int plm_add_rmsnorm(plm_ctx* ctx, const plm_add_rmsnorm_desc* desc, void* stream);
int plm_commit(plm_ctx* ctx, const plm_commit_desc* desc, void* stream);

/* ---- round engine ---- */
int plm_create(const plm_model_desc* model, const plm_weight_ptrs* weights, const plm_round_desc* round,
               plm_handle** out);
int plm_destroy(plm_handle* h);
int plm_set_block_table(plm_handle* h, const int32_t* table_host, int32_t n);
int plm_set_aux_stream(plm_handle* h, const int64_t* cells, int64_t n, void* stream);
/* The PTP scheme's auxiliary stream: n uniforms in [0, 1) (LinearInterpolationAuxiliary.sample_prior,
 * plm/auxiliary.py:92-94; the stream _fill_aux draws, plm/decoder.py:407-412). */
int plm_set_aux_uniforms(plm_handle* h, const float* u, int64_t n, void* stream);
int plm_load_prompt(plm_handle* h, const int64_t* ids, int64_t n, void* stream);
/* Sets the request's stop block on `stream` (done flag cleared): steady rounds stop committing once base reaches
 * max_tokens, or once a round confirms eos_token (>= 0; -1 disables the test) at an output position below
 * eos_window. Replaces the host-side stop test of plm/decoder.py:414-439, so a caller can keep rounds in flight:
 * rounds replayed after the stop leave the state as it was. A new handle stops at no budget and no end-of-text. */
int plm_set_stop(plm_handle* h, int64_t max_tokens, int64_t eos_token, int64_t eos_window, void* stream);
/* Causal prefill of the loaded prompt, then the first token and the request state of round 0. */
int plm_prefill(plm_handle* h, void* stream);
int plm_round0(plm_handle* h, void* stream);
/* One steady round: forward of k + k^2 rows (their K and V into the round scratch), lm_head, verify decode,
 * acceptance, and the KV commit of the accepted verify rows into the paged cache. Graph-capturable. */
int plm_round(plm_handle* h, void* stream);
/* One decoder layer's o_proj, post_attention_layernorm and mlp (vLLM llama.py:198-250 LlamaDecoderLayer.forward
 * after self_attn; plm/decoder.py:336 runs it inside the model forward) as the round runs it: the layer block over
 * the handle's first `rows` (1..128) activation rows, reading the attention output the last forward left and
 * updating the residual and the down partials. For measurement and tests; PLM_ERR_UNSUPPORTED when the handle was
 * created with separate_mlp. */
int plm_layer_block(plm_handle* h, int32_t layer, int32_t rows, void* stream);

/* Which of the caller's weight tensors the handle still reads after plm_create (a bit mask). PLM_WEIGHTS_IN_PLACE:
 * qkv, lm_head, the norms and the embeddings, always. PLM_WEIGHTS_BLOCK: the o, gate_up and down projections, read
 * only by a handle that runs them as separate launches (separate_mlp or gated-LoRA adapters); otherwise every launch
 * reads the handle's packed copies, and the caller may free those three tensors once plm_create has returned. */
#define PLM_WEIGHTS_IN_PLACE 1
#define PLM_WEIGHTS_BLOCK 2
int plm_borrowed_weights(plm_handle* h, int32_t* groups);
/* The layer block's unit schedule for num_sms CTAs (host only: no device is touched). No counterpart in the
 * reference: it exposes how plm_layer_block spreads o / norm / gate_up / down work over the SMs, for tests and
 * inspection. units gets *n_units codes, CTA after CTA; offsets[c] .. offsets[c + 1] are CTA c's (offsets has
 * num_sms + 1 entries). A code holds the kind in bits 28-29 (0 gate_up tile, 1 down unit, 2 o unit, 3 norm row),
 * the tile (the row of a norm unit) in bits 12-27 and the k-split in bits 0-11. PLM_ERR_INVALID with *n_units set
 * when capacity is too small; PLM_ERR_UNSUPPORTED for shapes the block does not take. */
int plm_block_schedule(int32_t num_sms, int32_t hidden, int32_t intermediate, int32_t q_size, int32_t* units,
                       int32_t capacity, int32_t* offsets, int32_t* n_units);
int plm_state(plm_handle* h, plm_state_ptrs* out);
int plm_check(plm_handle* h, int32_t* device_error);

/* ---- diagnostics ---- */
int plm_abi_version(void);
/* Copies the calling thread's last error message (NUL-terminated, truncated to n bytes). */
int plm_last_error(char* buf, size_t n);

#ifdef __cplusplus
}
#endif

#endif /* PLM_NATIVE_H */
