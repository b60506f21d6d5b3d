/*
 * longspark_b200 — C ABI of the B200 (sm_100a) drafting hot path of LongSpark.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (cudaStream_t passed as void*), launches asynchronously on that stream, and
 * returns an LS_* status.  Nothing here allocates device memory: scratch space
 * is a caller-provided workspace whose size the *_workspace_bytes queries
 * report, and whose counter region must be zeroed once after allocation (the
 * kernels leave it zeroed again).  Errors that can only be seen on the device
 * (bounded waits that gave up, out-of-range indices) are written to an
 * optional device status word (int, 0 = ok) the caller reads after a sync.
 *
 * Reference interfaces replaced (paths relative to the LongSpark project):
 *   SP = vendor/sglang/python/sglang/srt/speculative/
 *   SF = vendor/specforge/modeling/draft/
 *   LS = src/longspark/
 */
#ifndef LONGSPARK_B200_H
#define LONGSPARK_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LS_API __attribute__((visibility("default")))
#else
#define LS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LS_OK 0
#define LS_ERR_INVALID 1     /* bad shape / pointer / alignment argument      */
#define LS_ERR_CUDA 2        /* a CUDA runtime or driver call failed          */
#define LS_ERR_UNSUPPORTED 3 /* shape outside what the kernels implement      */
#define LS_ERR_WORKSPACE 4   /* workspace too small                           */

/* GEMM epilogues (what is written for out[token, feature]). */
#define LS_EPI_STORE 0      /* bf16(acc)                                            */
#define LS_EPI_SILU 1       /* bf16(silu(bf16(acc)))    (Linear -> SiLU)            */
#define LS_EPI_RESIDUAL 2   /* bf16(residual + bf16(acc))                           */
#define LS_EPI_QKV 3        /* per-head q/k RMSNorm + RoPE, v stored as is          */
#define LS_EPI_GATEUP 4     /* bf16(bf16(silu(gate)) * up), gate/up rows interleaved */
#define LS_EPI_LMHEAD 5     /* bf16 logits + per-128-row tile (max, argmax)         */
#define LS_EPI_MARKOV_ADD 6 /* bf16(base + bf16(acc))                               */

/* Weight layouts of ls_gemm. */
#define LS_W_ROWMAJOR 0
#define LS_W_TILED 1

/* Library version (major*10000 + minor*100 + patch). */
LS_API int ls_version(void);

/* Human-readable text of the last host-side error on this thread. */
LS_API const char* ls_last_error(void);

/* Number of SMs of the current device (grid sizing of the persistent kernels). */
LS_API int ls_device_sm_count(void);

/* ------------------------------------------------------------------------- */
/* Dense projections: out = epilogue(x[rows, k] . w[n_out, k]^T)             */
/* Replaces the cuBLAS GEMMs behind nn.Linear / SGLang QKVParallelLinear,     */
/* MergedColumnParallelLinear, RowParallelLinear of the drafter              */
/* (SP global16_native_draft_executor.py:141-165,435-457), the state-encoder  */
/* and shifted-input FeedForwards (SF draftfreekv.py:1498-1516), the bf16     */
/* vocabulary projection (SP global16_markov_precision.py:79-130) and the     */
/* Markov bias projection (SF draftfreekv.py:2346-2356).                      */
/* tcgen05/TMEM tensor cores, TMA loads, stream-K over (tile, k-block).       */
/* ------------------------------------------------------------------------- */
typedef struct ls_gemm_args {
  const void* x;        /* [rows, x_ld] bf16, K contiguous (activations)       */
  const void* w;        /* weights, layout per w_layout                        */
  int w_layout;         /* LS_W_ROWMAJOR: [n_out, k] bf16, K contiguous;
                           LS_W_TILED: ls_tile_weight() layout (16 KiB tiles streamed
                           as contiguous bulk copies)                           */
  int rows;             /* tokens                                              */
  int k;                /* reduction length, multiple of 64                    */
  int n_out;            /* output features, multiple of 128                    */
  int x_ld;             /* row pitch of x in elements (multiple of 8, >= k)    */
  int epilogue;         /* LS_EPI_*                                            */
  void* out;            /* bf16 output                                         */
  int out_ld;           /* row pitch of out in elements                        */
  const void* residual; /* LS_EPI_RESIDUAL: bf16 [rows, res_ld]; may alias out */
  int res_ld;
  int q_heads;          /* LS_EPI_QKV: tiles [0,q) are q heads, [q,q+kv) k heads */
  int kv_heads;
  const void* q_norm_w; /* [128] bf16                                          */
  const void* k_norm_w; /* [128] bf16                                          */
  float norm_eps;
  const int* positions; /* [rows] int32 RoPE positions                          */
  const float* inv_freq;/* [64] fp32 RoPE inverse frequencies                  */
  const float* rope_table; /* optional [rows, 128] fp32: bf16-rounded cos (0..63) and sin (64..127);
                              when NULL the epilogue evaluates them from positions and inv_freq */
  float* tile_max;      /* LS_EPI_LMHEAD: [rows, n_out/128] fp32                */
  int* tile_arg;        /* LS_EPI_LMHEAD: [rows, n_out/128] int32 (vocab index) */
  const void* base;     /* LS_EPI_MARKOV_ADD: bf16 [rows, base_ld]              */
  int base_ld;
  int* status;          /* optional device status word                          */
} ls_gemm_args;

/* Workspace layout: a 64 KiB region of per-tile arrival counters (zero it once
 * after allocation; every launch leaves it zeroed) followed by the fp32
 * partial tiles.  One workspace sized for the largest GEMM can be shared by
 * all GEMMs issued on the same stream. */
LS_API size_t ls_gemm_workspace_bytes(int rows, int k, int n_out);

/* The plan ls_gemm (fused_allreduce = 0) or ls_gemm_allreduce
 * (fused_allreduce = 1, `world` ranks, LS_TP_WIRE_* `wire` partials) picks
 * for a shape and epilogue on the current device (148 SMs assumed without
 * one), and what it needs: shared memory per CTA, TMEM columns, the GEMM
 * workspace, the exchange region.  kernel_weight_streaming: the instance with
 * the indexed producer runs (with tiled weights).  No counterpart in the
 * reference: it exists to inspect and test the planner without a GPU. */
typedef struct ls_gemm_plan {
  int bn;                      /* token tile                                    */
  int mw;                      /* 128-row feature tiles per work tile (1 or 2)  */
  int kg;                      /* k-blocks of 64 per pipeline stage             */
  int stages;
  int grid;                    /* CTAs                                          */
  int n_tiles, m_tiles;        /* token tiles, feature tiles                    */
  int kernel_weight_streaming;
  long long units;             /* stream-K units (work tiles x k-steps)         */
  size_t smem_bytes;           /* dynamic shared memory per CTA                 */
  size_t tmem_cols;
  size_t workspace_bytes;      /* counters + fp32 partials this plan uses       */
  size_t tp_sync_bytes;        /* fused: exchange region this plan uses, else 0 */
} ls_gemm_plan;
LS_API int ls_gemm_plan_info(int rows, int k, int n_out, int epilogue, int fused_allreduce, int world, int wire,
                             ls_gemm_plan* out);

/* Re-lay a row-major [n_out, k] bf16 weight matrix (n_out % 128 == 0,
 * k % 64 == 0) into the LS_W_TILED layout: 128 x 64 tiles stored
 * contiguously in (row tile, k tile) order, each already in the 128-byte
 * swizzled order the tensor cores read from shared memory (the 16-byte chunk
 * c of tile row r is stored at chunk c ^ (r % 8)).  out has n_out * k elements
 * and must not alias w. */
LS_API int ls_tile_weight(void* stream, const void* w, void* out, int n_out, int k);
LS_API int ls_gemm(void* stream, const ls_gemm_args* a, void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------------- */
/* (a) View refresh                                                          */
/* ------------------------------------------------------------------------- */

/* Scores of the S learned summary queries against new target K rows.
 * Replaces cache_position_scores / reference_position_scores
 * (SP global16_raw256_incremental.py:50-87, 400-456) and the GQA-5 variant
 * (LS patches/gqa5_attention.py:17-63); S, V and the GQA group are parameters.
 * query [batch, q_heads, slots, 128] bf16 (strides in elements, the batch
 * stride may be 0 for a shared query); new_keys [batch, rows, kv_heads, 128]
 * bf16 contiguous; out [batch, q_heads, slots, rows] fp32 contiguous. */
LS_API int ls_position_scores(void* stream, const void* query, long long q_stride_b, long long q_stride_h,
                       const void* new_keys, float* out, int batch, int q_heads, int kv_heads,
                       int slots, int rows, float softmax_scale);

/* Online-softmax merge of the first accept_lens[b] value rows into the fp32
 * (output, lse) state, in place on the slot pool.  Replaces
 * merge_accepted_positions_ / reference_merge_accepted_positions
 * (SP global16_raw256_incremental.py:90-166, 459-584).
 * state_out [capacity, q_heads, slots, 128] fp32 with row pitch state_stride
 * elements between pool entries; state_lse [capacity, q_heads, slots] fp32
 * with pitch lse_stride; scores [batch, q_heads, slots, rows] fp32;
 * values: value rows addressed as value_rows + (locs[b*rows + r] * kv_heads + h) * 128
 * (bf16); accept_lens [batch] int32 in [1, rows]; state_slots [batch] int32
 * (NULL = identity). */
LS_API int ls_merge_accepted(void* stream, float* state_out, long long state_stride, float* state_lse,
                      long long lse_stride, const float* scores, const void* value_rows,
                      const long long* locs, const int* accept_lens, const int* state_slots,
                      int batch, int q_heads, int kv_heads, int slots, int rows, int* status);

/* Fused view refresh over all tapped layers: for each request b it reads the
 * commit_lens[b] newly committed K/V rows at positions
 * [seq_lens[b]-commit_lens[b], seq_lens[b]) straight from the paged KV pool,
 * scores them against the learned summary queries and folds them into the
 * fp32 (output, lse) summary state of pool slot slots[b].  Replaces the
 * per-tapped-layer loop of LongSparkDraft._update_delta (LS engine/draft.py:215-260).
 * kv_k/kv_v: [tap_layers, pages, 16, kv_heads, 128] bf16; page_table
 * [batch, table_stride] int32 (logical page p of request b at
 * page_table[b*table_stride + (ring_pages ? p % ring_pages : p)]);
 * learned_query [tap_layers, q_heads, slots, 128] bf16;
 * state_out [capacity, tap_layers, q_heads, slots, 128] fp32;
 * state_lse [capacity, tap_layers, q_heads, slots] fp32. */
typedef struct ls_refresh_args {
  const void* kv_k;
  const void* kv_v;
  long long pool_pages;  /* pages per tapped layer in the pool */
  const int* page_table;
  int table_stride;
  int ring_pages;
  const int* seq_lens;    /* committed length after this commit */
  const int* commit_lens; /* rows committed this round, in [1, max_commit] */
  const int* slots;
  const void* learned_query;
  float* state_out;
  float* state_lse;
  void* state_bf16;       /* optional [capacity, bf16_layers, q_heads, slots, 128] bf16 copy of
                             state_out for the tapped layers the drafter attends to */
  int bf16_layers;        /* tapped layers [0, bf16_layers) get the bf16 copy */
  int capacity;           /* entries in the state pools (slots are checked against it) */
  int batch, tap_layers, q_heads, kv_heads, slots_per_head, max_commit;
  float softmax_scale;
  int* status;
} ls_refresh_args;

LS_API int ls_refresh_views(void* stream, const ls_refresh_args* a);

/* Copy packet K/V rows ([tap_layers, total_rows, kv_heads, 128] bf16, request b
 * owning rows [row_offsets[b], row_offsets[b] + counts[b])) into the paged pool
 * at positions [seq_lens[b]-counts[b], seq_lens[b]) through the page table, and
 * the boundary hidden state last_hidden [batch, tap_layers*hidden] into
 * hidden_pool[slots[b]].  Replaces the ring scatter of LongSparkDraft.update /
 * _update_delta (LS engine/draft.py:207-212, 257-260). */
LS_API int ls_window_scatter(void* stream, const void* keys, const void* values, long long total_rows,
                      const int* row_offsets, const int* counts, const int* seq_lens, void* kv_k,
                      void* kv_v, long long pool_pages, const int* page_table, int table_stride,
                      int ring_pages, const void* last_hidden, void* hidden_pool, int capacity, const int* slots,
                      int batch, int tap_layers, int kv_heads, int hidden, int* status);

/* ------------------------------------------------------------------------- */
/* Target-side export of the accepted rows, fused: launched on the target's   */
/* GPU after its verify pass, one kernel gathers each request's exported K/V  */
/* rows from the target's KV pool and stores them straight into the          */
/* drafter's paged pool through the drafter's page table — the drafter's own  */
/* GPU memory, or a peer GPU's reached over NVLink through an IPC mapping     */
/* (ls_ipc_open) or peer access — plus the boundary hidden states into its    */
/* hidden pool.  Replaces the target's gather (LS engine/target.py:213-228,   */
/* LS engine/state_export.py:14-47: index_select per layer, then a            */
/* dist.gather of the heads to rank 0 under target TP), the message transport */
/* (LS engine/transport.py) and the drafter's window scatter: under target TP */
/* every rank stores its own KV-head slice (head_offset), with no gather.    */
/* Plain 16-byte loads and stores only (no multicast, no TMA).  The index    */
/* arrays live in memory the launching GPU can read (its own, or a mapped     */
/* peer's).  The caller orders the export before the drafter's update of the  */
/* same requests (the update message, or an event, after this launch          */
/* completes).                                                                */
/* ------------------------------------------------------------------------- */
#define LS_EXPORT_MAX_LAYERS 8

typedef struct ls_export_args {
  const void* src_k[LS_EXPORT_MAX_LAYERS]; /* tapped layer l: the target's K pool [src_rows, src_heads, 128] bf16 */
  const void* src_v[LS_EXPORT_MAX_LAYERS]; /* same for V                                            */
  long long src_rows;
  int src_heads;            /* KV heads in a source row (this rank's slice under target TP)        */
  const long long* locations; /* [total_rows] source row of each exported row, request-major       */
  long long total_rows;
  const int* row_offsets;   /* [batch] first entry of request b in locations                       */
  const int* counts;        /* [batch] rows exported for request b                                 */
  const int* seq_lens;      /* [batch] drafter length after the commit: row i of request b lands at
                               position seq_lens[b] - counts[b] + i                                 */
  void* dst_k;              /* drafter pool [tap_layers, pool_pages, 16, dst_heads, 128] bf16       */
  void* dst_v;
  long long pool_pages;
  int dst_heads;
  int head_offset;          /* drafter head of source head 0 (head_offset + src_heads <= dst_heads) */
  const int* page_table;    /* [batch, table_stride] drafter page-table rows of the requests        */
  int table_stride;
  int ring_pages;           /* > 0: logical page p at column p % ring_pages                        */
  const void* last_hidden;  /* optional [batch, tap_layers * hidden] bf16 -> hidden_pool[slots[b]]  */
  void* hidden_pool;        /* [capacity, tap_layers * hidden] bf16                                 */
  const int* slots;         /* [batch] drafter pool slots (with last_hidden)                        */
  int capacity;
  int hidden;
  int batch;
  int tap_layers;
  int* status;              /* optional device status word: LS_DEV_BAD_INDEX for a location, page,
                               position or slot out of range (that row is skipped)                  */
} ls_export_args;

LS_API int ls_export_rows(void* stream, const ls_export_args* a);

/* Let kernels on the current device load and store peer_device's memory (the
 * export into a drafter on another GPU of the same process); a no-op when it
 * is already enabled or peer_device is the current device. */
LS_API int ls_enable_peer_access(int peer_device);

/* ------------------------------------------------------------------------- */
/* (b) Drafter attention over [summary | window | local rows]                */
/* Replaces Global16Raw256PagedDraftContext.attend (SP global16_raw256.py:   */
/* 1431-1647) and fused_global_local_raw_attention                           */
/* (SP global16_raw256_draft_all_attention.py:51-410).                       */
/* ------------------------------------------------------------------------- */
typedef struct ls_attention_args {
  const void* qkv;      /* [batch*block, (q_heads + 2*kv_heads)*128] bf16: rotated q | rotated k | v */
  int block;            /* P, drafter rows per request (<= 16)                    */
  const void* kv_k;     /* one tapped layer: [pages, 16, kv_heads, 128] bf16      */
  const void* kv_v;
  long long pool_pages; /* page ids are checked against it                        */
  const int* page_table;
  int table_stride;
  int ring_pages;
  const int* seq_lens;  /* committed length; the window is the last min(len, W) rows */
  int window;           /* W */
  const void* learned_query; /* one tapped layer: [q_heads, slots, 128] bf16       */
  const float* state_out;    /* [capacity, ...]: entry of request b at state_out + slots[b]*state_stride */
  long long state_stride;
  const void* state_bf16;    /* optional bf16 copy of the same entries (read instead of state_out) */
  long long state_bf16_stride;
  const int* slots;
  int capacity;         /* entries in the state pool                              */
  int slots_per_head;   /* S */
  int batch, q_heads, kv_heads;
  float softmax_scale;
  void* out;            /* [batch*block, q_heads*128] bf16 */
  int* status;
} ls_attention_args;

/* One launch: a cluster of 8 CTAs per (request, KV head) merges its partial
 * softmax states through distributed shared memory, so no workspace is needed
 * (ls_attention_workspace_bytes returns 0; workspace may be NULL).  Launched
 * with programmatic dependent launch: the window rows and the summary keys are
 * staged before the kernel waits for the preceding kernel of the stream, the
 * summary values (which a view refresh just before may write) after it. */
LS_API size_t ls_attention_workspace_bytes(int batch, int q_heads, int kv_heads, int window, int slots_per_head);
LS_API int ls_draft_attention(void* stream, const ls_attention_args* a, void* workspace, size_t workspace_bytes);

/* ------------------------------------------------------------------------- */
/* Elementwise pieces of the drafter pass                                     */
/* ------------------------------------------------------------------------- */

/* RMSNorm over rows of length n.  mode 0: SpecForge/HF rounding
 * bf16(w * bf16(x*rstd)) (SF draftfreekv.py:1518-1530); mode 1: F.rms_norm
 * rounding bf16(x*rstd*w) (target final norm, SF draftfreekv.py:3607-3647).
 * When w2 != NULL a second norm of the same mode follows in the same launch:
 * out2 = RMSNorm(out; w2) (two consecutive norms, e.g. the shifted-input norm
 * and the first decoder layer's input norm, SF draftfreekv.py:1737, 2299). */
LS_API int ls_rmsnorm(void* stream, const void* x, int x_ld, const void* w, void* out, int out_ld, int rows,
               int n, float eps, int mode, const void* w2, void* out2, int out2_ld);

/* ParallelShiftedInput input rows (SF draftfreekv.py:1692-1739):
 * out[b*block + i] = [bf16(embed[tok_i] + pos_emb[i]) | latest[b]],
 * where, when latest_norm_w != NULL, latest[b] is first normalised in the same
 * launch (mode-0 RMSNorm with latest_norm_w, norm_eps: the state encoder's
 * output norm, SF draftfreekv.py:1540), so `latest` is the encoder output;
 * tok_0 = anchors[b], tok_i = mask_token_id for i > 0.  out is [batch*block, 2*hidden].
 * When positions != NULL also writes the RoPE positions of the block rows,
 * positions[b*block + i] = seq_lens[b] + i (SF draftfreekv.py:3259-3263), and
 * when rope_table != NULL the table the QKV epilogue reads: per row,
 * bf16(cos(pos * inv_freq[j])) at j and bf16(sin(...)) at 64 + j, j < 64
 * (SF draftfreekv.py:1996-2007). */
LS_API int ls_shifted_input(void* stream, const long long* anchors, const int* seq_lens, int* positions,
                            const float* inv_freq, float* rope_table, const void* embed, const void* pos_emb,
                            const void* latest, const void* latest_norm_w, float norm_eps, void* out,
                            int batch, int block, int hidden, int vocab, int mask_token_id, int* status);

/* Gather rows: out[b] = src[idx[b]] (row_bytes each, 16-byte multiples);
 * indices outside [0, src_rows) are recorded in *status and the row is zeroed. */
LS_API int ls_gather_rows(void* stream, const void* src, long long src_rows, const int* idx, void* out, int rows,
                          long long row_bytes, int* status);

/* ------------------------------------------------------------------------- */
/* Greedy proposal tokens and the accept check                               */
/* ------------------------------------------------------------------------- */

/* Greedy Markov chain over bf16 base logits (DSparkVanillaMarkovHead.
 * sample_block_tokens at temperature 0, SF draftfreekv.py:2366-2407; without a
 * Markov head base_logits.argmax(-1), :3545-3578): for t in [0, block):
 * tok_t = argmax_v bf16(base[t, v] + bf16(w2[v] . w1[prev])), prev = tok_{t-1}
 * (anchors for t = 0), lowest index on ties.  Only tokens whose base logit lies
 * within a rigorous bound of the row maximum can win (Cauchy-Schwarz:
 * |bias| <= w1_row_bound * w2_row_bound); those candidates are listed per row
 * in parallel, every (previous candidate, candidate) bias is evaluated at once
 * and the serial chain is a table walk.  The tokens equal the full-vocabulary
 * scan's; a request whose band overflows the candidate buffers is evaluated
 * step by step over the band, and over the whole vocabulary if needed.
 * w1 == NULL: no Markov head.  base: [batch*block, vocab] bf16;
 * tile_max/tile_arg: [batch*block, vocab/128] from the LS_EPI_LMHEAD epilogue.
 * tokens [batch, block] int64.  When target != NULL ([batch, target_ld] int64)
 * also writes accept_out [batch] (greedy accepted-prefix length,
 * LS engine/target.py:472-477). */
typedef struct ls_markov_args {
  const void* base;
  const float* tile_max;
  const int* tile_arg;
  const void* w1;            /* [vocab, rank] bf16 or NULL */
  const void* w2;            /* [vocab, rank] bf16 */
  const float* w1_row_bound; /* device fp32, >= max_v ||w1[v]||_2 (ls_row_norm_bound) */
  const float* w2_row_bound; /* device fp32, >= max_v ||w2[v]||_2 */
  int rank;
  const long long* anchors;  /* [batch] */
  long long* tokens;         /* [batch, block] */
  const long long* target;   /* optional [batch, target_ld] */
  int target_ld;
  long long* accept_out;     /* optional [batch] */
  int batch, block, vocab;
  int* status;
} ls_markov_args;

LS_API size_t ls_markov_workspace_bytes(int batch, int block);
LS_API int ls_markov_argmax(void* stream, const ls_markov_args* a, void* workspace, size_t workspace_bytes);

/* ls_markov_argmax with its scratch in a fixed device array inside this
 * library (648.25 KiB per device) instead of a caller workspace.  No
 * counterpart in the reference, which allocates its step tensors through
 * PyTorch; this exists for callers that cannot allocate device memory when
 * they propose tokens: a serving process that handed all free HBM to its paged
 * KV-cache pool at start-up (a cudaMalloc in the middle of serving fails or
 * must evict cache pages), or a host binding over this C ABI that owns no
 * device allocator to carve a workspace from.  It calls no cudaMalloc,
 * cudaFree or allocating library routine.
 * Limit: batch x block <= LS_MARKOV_STATIC_MAX_ROWS; larger calls fail with
 * LS_ERR_WORKSPACE and launch nothing.
 * The first call on each device, made with that device current, looks up the
 * array's address (cudaGetSymbolAddress); make that first call before any
 * stream capture on the device.  Every call on a device shares the one array,
 * which keeps the last call's contents: each call clears the counters that must
 * start at zero with a memset on its own stream.  Calls that overlap on the
 * GPU (on different streams, or from threads without ordering between them)
 * race on the array and give undefined tokens; calls on one stream are
 * ordered and safe. */
#define LS_MARKOV_STATIC_MAX_ROWS 1024
LS_API int ls_markov_argmax_static(void* stream, const ls_markov_args* a);

/* Temperature > 0: step `step` of the sampled chain for every request.  Draws
 * token ~ softmax(logits[b] / T) (the reference's multinomial draw,
 * SF draftfreekv.py:2366-2407) as the Gumbel-max of logits / T + g with
 * g = -log(-log(u)), u = a 24-bit uniform from a counter-based hash of
 * (seed, b, step, token) (two lowbias32 rounds; restated by the oracle), and
 * writes tokens[b, step], q[b, step] = softmax(logits[b] / T)[token] (the
 * proposal probability of LS engine/draft.py:284-286) and prev[b] (int32 copy
 * of the token, the next step's Markov row index).  logits: the step's bf16
 * logits of request b at logits + b * logits_ld (base logits, or the
 * Markov-corrected step logits written by an LS_EPI_MARKOV_ADD GEMM). */
typedef struct ls_sample_step_args {
  const void* logits;
  long long logits_ld;
  int batch, vocab, block, step;
  float temperature;
  unsigned long long seed;
  long long* tokens;  /* [batch, block] */
  float* q;           /* optional [batch, block] */
  int* prev;          /* optional [batch] */
  int* status;
} ls_sample_step_args;

LS_API size_t ls_sample_step_workspace_bytes(int batch);
LS_API int ls_sample_step(void* stream, const ls_sample_step_args* a, void* workspace, size_t workspace_bytes);

/* Temperature > 0 verification: the reference's two-phase exact rejection
 * sampling (decide_acceptance + finish_sampling, LS engine/sampling.py:19-57,
 * as the target drives it at LS engine/target.py:478-491 with the drafter's q
 * rows of :613-614), both phases in one launch, one CTA per request.
 *   p = softmax(target / T) over the block + 1 verify rows of request b;
 *   lengths[b] = number of leading t with uniforms[b, t] * sampled_q[b, t]
 *                < p[t, candidates[b, t]];
 *   bonus[b] = count(final_uniforms[b] >= cumsum(probs)), at most vocab - 1,
 *   probs = max(p[L] - softmax(draft[L] / T), 0) / mass at a rejection
 *   (L = lengths[b] < block) when mass > 1e-8, else p[L].
 * target_logits: bf16, row t of request b at (b * (block + 1) + t) *
 * target_ld; draft_logits: the drafter's corrected bf16 logits, row t of
 * request b at (b * block + t) * draft_ld.  vocab and both strides multiples
 * of 8, logits 16-byte aligned.  A candidate outside [0, vocab) records
 * LS_DEV_BAD_TOKEN and is read as token 0. */
typedef struct ls_rejection_args {
  const void* target_logits;
  long long target_ld;
  const void* draft_logits;
  long long draft_ld;
  const long long* candidates;  /* [batch, block] */
  const float* sampled_q;       /* [batch, block]: q of each candidate */
  const float* uniforms;        /* [batch, block] */
  const float* final_uniforms;  /* [batch] */
  float temperature;            /* > 0 */
  int batch, block, vocab;
  long long* lengths;           /* out [batch] */
  long long* bonus;             /* out [batch] */
  int* status;                  /* optional device status word */
} ls_rejection_args;

LS_API int ls_rejection_sample(void* stream, const ls_rejection_args* a);

/* Greedy accept check: accept[b] = number of leading i < block with
 * target[b, i] == draft[b, i] (LS engine/target.py:472-477). */
LS_API int ls_accept(void* stream, const long long* target, int target_ld, const long long* draft, long long* accept,
              int batch, int block);

/* Row-norm bound of a [vocab, rank] bf16 matrix: writes max_v ||m[v]||_2 * (1 + 1e-6)
 * to *out (device fp32). */
LS_API int ls_row_norm_bound(void* stream, const void* m, int vocab, int rank, float* out);

/* ------------------------------------------------------------------------- */
/* Prefill summary: the fp32 (output, lse) summary state of every learned     */
/* query over a request's whole committed prefix [0, seq_lens[b]), read from  */
/* the paged K/V pool (which must hold the whole prefix: the target's cache,  */
/* not a window ring):                                                        */
/*   lse[s] = logsumexp_r(scale * q[s] . k[r]),                               */
/*   out[s] = sum_r exp(scale * q[s] . k[r] - lse[s]) * v[r].                  */
/* Replaces the target's FA3 pass over 16 qlen-1 sequences per tapped layer   */
/* (LS engine/target.py:230-253); definition: global_state_from_full_prefix   */
/* (SF global16_raw256.py:829-869).  Scores unrounded fp32; the softmax       */
/* weights enter the P.V tensor-core products as bf16 high part + bf16        */
/* residual, so the result follows the fp32 definition.  An empty prefix      */
/* writes output 0, lse -inf.  Writes state_out / state_lse (and the bf16     */
/* copy of the first bf16_layers layers) of slot slots[b].                    */
/* Needs q_heads % kv_heads == 0, slots % 16 == 0, (q_heads/kv_heads) * slots */
/* % 64 == 0, seq_lens[b] <= table_stride * 16.                               */
/* ------------------------------------------------------------------------- */
typedef struct ls_prefill_args {
  const void* kv_k;          /* [tap_layers, pool_pages, 16, kv_heads, 128] bf16 */
  const void* kv_v;
  long long pool_pages;
  const int* page_table;     /* [batch, table_stride] */
  int table_stride;
  const int* seq_lens;       /* [batch] prefix length */
  const int* slots;          /* [batch] state slot */
  const void* learned_query; /* [tap_layers, q_heads, slots_per_head, 128] bf16 */
  float* state_out;          /* [capacity, tap_layers, q_heads, slots_per_head, 128] */
  float* state_lse;          /* [capacity, tap_layers, q_heads, slots_per_head] */
  void* state_bf16;          /* optional [capacity, bf16_layers, q_heads, slots_per_head, 128] bf16 */
  int bf16_layers;
  int capacity, batch, tap_layers, q_heads, kv_heads, slots_per_head;
  float softmax_scale;
  int* status;
} ls_prefill_args;

LS_API int ls_prefill_summary(void* stream, const ls_prefill_args* a);

/* ------------------------------------------------------------------------- */
/* One whole greedy drafting round in one call                               */
/* ------------------------------------------------------------------------- */

/* The launch sequence of a round for hosts that are not Python: the calls the
 * Python engine (DraftEngine.draft) makes, in the same order and with the same
 * arguments, so a C, C++, Go or Java host binds one function instead of
 * replaying sixteen.  Replaces, on the reference side, the drafter forward of
 * one proposal (Global16NativeDraftExecutor, global16_native_draft_executor.py:
 * 548-645: state encoder, shifted input, decoder layers, LM head) plus the
 * summary update of LongSparkDraft._update_delta (src/longspark/engine/draft.py:
 * 215-260), the Markov chain (draftfreekv.py:2366-2407) and the accept check
 * (src/longspark/engine/target.py:472-477).  All pointers are device pointers;
 * "tiled" weights are in the ls_tile_weight layout. */
typedef struct ls_round_layer {
  const void* in_norm;   /* [hidden] bf16                                                  */
  const void* qkv;       /* tiled [(q_heads + 2 kv_heads) * 128, hidden]: q | k | v rows  */
  const void* q_norm;    /* [128] bf16                                                    */
  const void* k_norm;    /* [128] bf16                                                    */
  const void* o;         /* tiled [hidden, q_heads * 128]                                 */
  const void* post_norm; /* [hidden] bf16                                                  */
  const void* gate_up;   /* tiled [2 inter, hidden]: per 128-row tile 64 gate rows, then the
                            64 up rows of the same outputs                                 */
  const void* down;      /* tiled [hidden, inter]                                         */
  int view;              /* the tapped layer this layer attends to (its pool, learned
                            queries and summary entries); < bf16_layers when summary_bf16 */
} ls_round_layer;

typedef struct ls_round_args {
  /* shape */
  int hidden, q_heads, kv_heads, inter, vocab;
  int tap_layers, slots_per_head, window, block, max_commit;
  int markov_rank;       /* 0: no Markov head                                             */
  int mask_token_id;
  float rms_eps, final_eps;
  int n_layers;
  const ls_round_layer* layers;  /* host array of n_layers                                */
  /* weights */
  const void* enc_w1;    /* tiled [hidden, tap_layers * hidden]                           */
  const void* enc_w2;    /* tiled [hidden, hidden]                                        */
  const void* enc_norm;  /* [hidden] bf16                                                  */
  const void* embed;     /* [vocab, hidden] bf16                                          */
  const void* pos_emb;   /* [block, hidden] bf16                                          */
  const void* sh_w1;     /* tiled [hidden, 2 hidden]                                      */
  const void* sh_w2;     /* tiled [hidden, hidden]                                        */
  const void* sh_norm;   /* [hidden] bf16                                                  */
  const void* final_norm;/* [hidden] bf16                                                  */
  const void* lm_head;   /* tiled [vocab, hidden]                                         */
  const void* markov_w1; /* [vocab, markov_rank] bf16 or NULL                             */
  const void* markov_w2;
  const float* w1_bound; /* ls_row_norm_bound of markov_w1 / markov_w2                    */
  const float* w2_bound;
  const float* inv_freq; /* [64] fp32 RoPE inverse frequencies                            */
  /* views, by pool slot */
  const void* kv_k;      /* [tap_layers, pool_pages, 16, kv_heads, 128] bf16               */
  const void* kv_v;
  long long pool_pages;
  int ring_pages;
  const void* learned_query; /* [tap_layers, q_heads, slots, 128] bf16                    */
  float* summary_out;    /* [capacity, tap_layers, q_heads, slots, 128] fp32              */
  float* summary_lse;    /* [capacity, tap_layers, q_heads, slots] fp32                    */
  void* summary_bf16;    /* [capacity, bf16_layers, q_heads, slots, 128] bf16 or NULL      */
  int bf16_layers;
  const void* hidden_pool; /* [capacity, tap_layers * hidden] bf16 boundary hidden states  */
  int capacity;
  /* this round, batch order */
  int batch;
  const int* slots;      /* [batch] pool slots                                            */
  const int* seq_lens;   /* [batch] committed length                                      */
  const int* commit_lens;/* [batch] rows committed since the last round; NULL: no refresh */
  const int* page_table; /* [batch, table_stride]                                         */
  int table_stride;
  const long long* anchors;  /* [batch]                                                   */
  const long long* target;   /* [batch, target_ld] or NULL (no accept check)              */
  int target_ld;
  int slots_are_rows;    /* 1: slots[b] == b, the hidden states are read in place         */
  /* outputs */
  long long* tokens;     /* [batch, block]                                                */
  long long* accept;     /* [batch], with target                                          */
  void* logits;          /* [batch * block, vocab] bf16 base logits                       */
  int* status;           /* device status word                                            */
  /* scratch, ls_round_workspace_bytes(this) bytes, 256-byte aligned */
  void* workspace;
  size_t workspace_bytes;
} ls_round_args;

LS_API size_t ls_round_workspace_bytes(const ls_round_args* a);
LS_API int ls_draft_round(void* stream, const ls_round_args* a);

/* ------------------------------------------------------------------------- */
/* Tensor parallelism of the drafter over NVLink (one process per GPU).       */
/* No counterpart in the reference, which forces the drafter to one GPU       */
/* (SP global16_native_draft_executor.py:1101-1105); the design precedent is  */
/* the target's push/pull custom allreduce over IPC-mapped peer buffers       */
/* (vendor/sglang jit_kernel/csrc/distributed/custom_all_reduce_push.cuh).    */
/*                                                                            */
/* Every rank allocates one "symmetric heap" of the same size with           */
/* ls_ipc_alloc, exchanges the 64-byte handles (any host channel), opens the  */
/* peers' heaps with ls_ipc_open, and fills an ls_tp_group.  A buffer at      */
/* offset X of this rank's heap is reached on rank p at heap[p] + X, so a      */
/* kernel addresses the same buffer on every rank from one local pointer.     */
/* The heap holds, at sync_offset, a sync region of ls_tp_sync_bytes() bytes  */
/* (flags and exchange slots; zero it on every rank, then put a host barrier  */
/* between the ranks before the first TP launch).  Plain peer loads and       */
/* stores only: no multicast object, no TMA from peer memory.                 */
/* Every wait on a peer is bounded (2 s of %globaltimer); a wait that gives   */
/* up writes LS_DEV_TIMEOUT_PEER to the status word and the kernel returns;   */
/* the flags are then inconsistent: zero the sync region on every rank (after */
/* a host barrier) before the next TP launch.                                 */
/* ------------------------------------------------------------------------- */
#define LS_TP_MAX_RANKS 8
#define LS_TP_WIRE_F32 0  /* partial tiles cross NVLink as fp32                */
#define LS_TP_WIRE_BF16 1 /* partial tiles cross NVLink rounded to bf16 (as a  */
                          /* bf16 row-parallel linear + bf16 allreduce does)   */
#define LS_DEV_TIMEOUT_PEER 105

typedef struct ls_tp_group {
  int world;                      /* ranks, 1..LS_TP_MAX_RANKS                   */
  int rank;                       /* this process's rank                         */
  void* heap[LS_TP_MAX_RANKS];    /* every rank's heap, mapped in this process    */
  size_t heap_bytes;              /* size of each heap (the same on every rank)   */
  size_t sync_offset;             /* sync region offset (256-byte aligned)        */
} ls_tp_group;

/* cudaMalloc of `bytes` on the current device plus its IPC handle
 * (cudaIpcGetMemHandle, 64 bytes written to handle_out). */
LS_API int ls_ipc_alloc(size_t bytes, void** ptr_out, void* handle_out);
/* Map a peer's allocation from its 64-byte handle (cudaIpcOpenMemHandle with
 * lazy peer access). */
LS_API int ls_ipc_open(const void* handle, void** ptr_out);
LS_API int ls_ipc_close(void* ptr);
LS_API int ls_ipc_free(void* ptr);

/* Bytes of the sync region for row-parallel GEMMs with up to `rows` tokens and
 * `n_out` output features on `world` ranks with the given wire format (take
 * the maximum over the GEMMs that share the region). */
LS_API size_t ls_tp_sync_bytes(int world, int rows, int n_out, int wire);

/* Row-parallel GEMM fused with the allreduce of its output over the group:
 *   out = epilogue(sum over ranks of x_r . w_r^T)   on every rank,
 * where x_r / w_r are this rank's k-slice (a.x, a.w, a.k are local).
 * Epilogues LS_EPI_STORE and LS_EPI_RESIDUAL (residual: this rank's copy,
 * identical on every rank; may alias out).  `a.out` must lie inside this
 * rank's heap (16-byte aligned, out_ld a multiple of 8).  As soon as its
 * tensor cores finish an output tile, a rank peer-stores its fp32 (or bf16,
 * per `wire`) partial and raises a release flag:
 *  - two ranks (one-shot): to both ranks; each rank then sums the two
 *    partials of every tile in rank order and applies the epilogue itself;
 *  - four or more ranks (owner reduce + broadcast): to the tile's owner
 *    (rank t % world), which sums the partials in rank order, applies the
 *    epilogue once and stores the bf16 result into every rank's `out`, then
 *    flags each rank.
 * Either way every rank ends with the same bits, and the kernel returns when
 * this rank's `out` is complete.  Launch it on every rank with the same
 * shapes, in the same order relative to the other TP launches. */
LS_API int ls_gemm_allreduce(void* stream, const ls_gemm_args* a, const ls_tp_group* g, int wire, void* workspace,
                             size_t workspace_bytes);

/* Device-side barrier over the group (one small kernel): returns when every
 * rank has reached it; the writes of kernels before it on every rank are then
 * visible to kernels after it on every rank.  `slot` in [0, 16) selects an
 * epoch counter; each slot must be used by every rank the same number of
 * times. */
LS_API int ls_tp_barrier(void* stream, const ls_tp_group* g, int slot, int* status);

/* ls_markov_argmax over a vocabulary sharded by 128-token tiles: rank s holds
 * tiles [s * tiles_per_shard, min((s + 1) * tiles_per_shard, vocab / 128)) of
 * the LM head, i.e. its logits [batch*block, n_s * 128] and tile maxima
 * [batch*block, n_s] (LS_EPI_LMHEAD output of its weight shard; tile_arg
 * local to the shard).  a.base / a.tile_max / a.tile_arg are this rank's
 * shard, inside its heap, at the same offsets on every rank; a.vocab is the
 * full vocabulary; w1/w2 are full (replicated).  Every rank reads the band
 * tiles it needs from the owning rank's heap and computes the same tokens.
 * Put an ls_tp_barrier between the LM-head GEMMs and this call. */
LS_API int ls_markov_argmax_tp(void* stream, const ls_markov_args* a, const ls_tp_group* g, int tiles_per_shard,
                               void* workspace, size_t workspace_bytes);

#ifdef __cplusplus
}
#endif

#endif /* LONGSPARK_B200_H */
