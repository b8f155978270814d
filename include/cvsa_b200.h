/*
 * cvsa_b200.h -- C ABI of the B200-native CVSA decode step (libcvsa_b200.so).
 *
 * The CVSA decode step of DJ-Melvin/coverage-verified-sparse-attention is:
 * page scoring -> top-k page selection -> sparse paged decode emitting
 * (o, LSE) -> per-head coverage gate against tau -> complement recovery merged
 * by LSE. Every entry point below replaces one function of the reference's
 * Python/Triton call surface; the reference file:line is given beside each.
 *
 * Conventions (all entry points):
 *   - All tensor pointers are DEVICE pointers on the current CUDA device.
 *   - `stream` is a cudaStream_t passed as void* (NULL = legacy default
 *     stream). Every call only enqueues work on that stream; nothing blocks
 *     the host and nothing allocates memory (except the set-up call
 *     cvsa_peer_alloc): scratch comes from a
 *     caller-provided workspace whose size is queried with *_workspace_size.
 *     A workspace is 256-byte aligned and zeroed once before its first use
 *     (cvsa_workspace_reset). Its first 256 KiB hold counters the kernels
 *     return to zero, at a fixed offset, so one workspace can serve calls of
 *     any shapes in stream order; two calls that may run concurrently need
 *     separate workspaces. batch * num_kv_heads is limited to 65472.
 *   - Integer tensors are int32 unless stated; layouts are row-major and
 *     contiguous unless a stride is passed.
 *   - Return value: CVSA_OK (0) or a negative CVSA_ERR_* status; the message
 *     of the last failing call on this host thread is cvsa_last_error().
 *     Bad arguments return CVSA_ERR_INVALID (the reference raises ValueError);
 *     an exhausted page pool is CVSA_ERR_POOL (the reference asserts).
 *   - Device-side bounds checks (block ids, page indices) never trap: they
 *     record CVSA_DEV_ERR_* bits in a caller-visible error word and skip the
 *     access.
 */
#ifndef CVSA_B200_H_
#define CVSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CVSA_ABI_VERSION 2

/* element types */
enum {
  CVSA_DTYPE_F32 = 0,
  CVSA_DTYPE_F16 = 1,
  CVSA_DTYPE_BF16 = 2
};

/* status codes */
enum {
  CVSA_OK = 0,
  CVSA_ERR_INVALID = -1,     /* bad argument (reference: ValueError) */
  CVSA_ERR_UNSUPPORTED = -2, /* valid but not built (head_dim, block_size, GQA) */
  CVSA_ERR_WORKSPACE = -3,   /* workspace NULL, too small or misaligned */
  CVSA_ERR_CUDA = -4,        /* a CUDA runtime call or launch failed */
  CVSA_ERR_POOL = -5         /* page pool exhausted (reference: assert) */
};

/* bits of the device error word (cvsa_decode_step io.dev_error, append) */
enum {
  CVSA_DEV_ERR_BLOCK_RANGE = 1, /* a block table entry outside [0, num_blocks) */
  CVSA_DEV_ERR_PAGE_RANGE = 2,  /* a page index outside [0, max_pages) */
  CVSA_DEV_ERR_POOL = 4,        /* append: free list exhausted */
  CVSA_DEV_ERR_TABLE_FULL = 8,  /* append: sequence longer than the table */
  CVSA_DEV_ERR_TIMEOUT = 16     /* a bounded wait (async copy, peer rank) gave up */
};

/* Paged KV pool: [num_blocks, block_size, num_kv_heads, head_dim].
 * cvsa/runtime/kv_cache.py:24-50 (PagedKVCache.k_cache / v_cache). v_cache
 * shares k_cache's strides. head_dim is contiguous; rows must be 16-byte
 * aligned. */
typedef struct cvsa_kv_desc {
  const void* k_cache;
  const void* v_cache;
  int32_t dtype;
  int32_t num_blocks;
  int32_t block_size;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t reserved0;
  int64_t stride_block; /* elements */
  int64_t stride_token; /* elements */
  int64_t stride_head;  /* elements */
} cvsa_kv_desc_t;

/* Decode queries and per-sequence page tables.
 * q: [batch, num_q_heads, head_dim] contiguous (cvsa/backend.py:315).
 * block_tables: [batch, max_pages] (kv_cache.py:96-100); context_lens: [batch]. */
typedef struct cvsa_query_desc {
  const void* q;
  int32_t dtype;
  int32_t batch;
  int32_t num_q_heads;
  int32_t max_pages;
  const int32_t* block_tables;
  const int32_t* context_lens;
} cvsa_query_desc_t;

int cvsa_abi_version(void);
const char* cvsa_status_string(int status);
const char* cvsa_last_error(void);

/* Page scores, [batch, num_kv_heads, max_pages] float32:
 * max over valid tokens of (mean-pooled GQA q, rounded to q's dtype) . k,
 * times head_dim^-0.5; -inf at and beyond the context.
 * Replaces triton_score_pages, cvsa/kernels/page_scores.py:77-119
 * (kernel :13-74). */
int cvsa_score_pages(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                     float* page_scores, void* stream);

/* Quest page ranking scores, [batch, num_kv_heads, max_pages] float32: per
 * page and KV head, the channel-wise minimum and maximum of the keys of its
 * valid tokens, then sum_d max(q_d * kmin_d, q_d * kmax_d) * head_dim^-0.5 with
 * q the group mean of the query heads rounded to q's dtype; -inf for pages
 * without a valid token. A block id outside the pool sets
 * CVSA_DEV_ERR_BLOCK_RANGE in *dev_error (nullable) and scores -inf.
 * Replaces CVSABackend._quest_page_scores, cvsa/backend.py:572-620 (the
 * selector='quest' / light_normalizer ranking). */
int cvsa_quest_scores(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                      float* page_scores, int32_t* dev_error, void* stream);

/* Top-k page selection per (b, kv head): the first `sink_pages` and last
 * `local_pages` valid pages, plus the `budget` highest-scoring other valid
 * pages, ordered (score desc, page index asc); written in ascending page
 * order into page_indices [batch, num_kv_heads, max_sel] with the count in
 * n_per_head [batch, num_kv_heads]. max_sel >= budget + sink + local.
 * Replaces cvsa/backend.py:690,737-747 (torch.topk + n_per_head clamp). */
int cvsa_select_pages(const float* page_scores, int32_t batch, int32_t num_kv_heads,
                      int32_t max_pages, const int32_t* context_lens, int32_t block_size,
                      int32_t budget, int32_t sink_pages, int32_t local_pages,
                      int32_t* page_indices, int32_t max_sel, int32_t* n_per_head,
                      void* stream);

/* Coverage gate: cov = exp(lse(scores[sel[:n]]) - lse(scores[:max_pages])),
 * accept = cov >= tau (uint8 0/1), both [batch, num_kv_heads].
 * Replaces triton_check_coverage, cvsa/kernels/coverage.py:218-265
 * (kernel :160-215). */
int cvsa_check_coverage(const float* page_scores, int32_t batch, int32_t num_kv_heads,
                        int32_t max_pages, const int32_t* page_indices, int32_t max_sel,
                        const int32_t* n_per_head, float tau, uint8_t* accept,
                        float* coverage, void* stream);

/* Complement: valid pages not in the first n_per_head selected pages, in
 * ascending order, into complement [batch, num_kv_heads, max_comp];
 * n_complement = 0 for heads with accept != 0 (accept may be NULL).
 * Replaces triton_compute_complement, cvsa/kernels/coverage.py:99-150, and
 * compute_complement_pages, cvsa/complement.py:11-69. */
int cvsa_compute_complement(const int32_t* page_indices, int32_t max_sel,
                            const int32_t* n_per_head, const int32_t* context_lens,
                            int32_t batch, int32_t num_kv_heads, int32_t block_size,
                            const uint8_t* accept, int32_t* complement, int32_t max_comp,
                            int32_t* n_complement, void* stream);

/* Workspace bytes for cvsa_sparse_decode / cvsa_recover_merge with these
 * shapes (max_sel = width of page_indices). */
size_t cvsa_decode_workspace_size(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                                  int32_t max_sel);

/* Sparse paged decode over the first n_per_head[b,h] pages of page_indices
 * [batch, num_kv_heads, max_sel], all G query heads of a KV head at once.
 * Writes, for each non-NULL output:
 *   o_unnorm [batch, num_q_heads, head_dim] f32, m [batch, num_q_heads] f32
 *   (max scaled logit), l [batch, num_q_heads] f32 (sum exp(s - m));
 *   out [batch, num_q_heads, head_dim] in out_dtype = o / max(l, 1e-6).
 * A head with no valid token yields (0, -inf, 0) and out = 0.
 * Replaces triton_sparse_decode_unnorm (sparse_decode.py:537-573, kernels
 * :424-500, :609-661, :136-234, :577-606), triton_sparse_decode_reuse
 * (:681-721) and triton_sparse_decode (:286-350). */
int cvsa_sparse_decode(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                       const int32_t* page_indices, int32_t max_sel,
                       const int32_t* n_per_head, float* o_unnorm, float* m, float* l,
                       void* out, int32_t out_dtype, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Selective LSE merge of draft (o_d, m_d, l_d) and complement (o_c, m_c, l_c)
 * partials, [batch, G*num_kv_heads(, head_dim)] f32, with accept
 * [batch, num_kv_heads] (uint8): accepted heads o_d / max(l_d, 1e-6), others
 * the LSE merge divided by max(l, 1e-6). out in out_dtype.
 * Replaces triton_lse_merge, cvsa/kernels/coverage.py:329-367 (kernel
 * :274-326), and selective_lse_merge, cvsa/lse_merge.py:11-54. */
int cvsa_lse_merge(const float* o_d, const float* m_d, const float* l_d,
                   const float* o_c, const float* m_c, const float* l_c,
                   const uint8_t* accept, int32_t batch, int32_t num_kv_heads,
                   int32_t num_q_per_kv, int32_t head_dim, void* out, int32_t out_dtype,
                   void* stream);

/* Fixed-order merge of the attention partials of a page-split step (the
 * pages of every sequence split contiguously over `world` ranks; the
 * reference has no multi-GPU path, this combines its per-rank
 * triton_sparse_decode_unnorm partials, cvsa/kernels/sparse_decode.py:537-573,
 * as cvsa/lse_merge.py:11-54 combines two). parts: `world` rows of
 * row_stride floats in rank order (an all-gather's output); row r holds
 * o_unnorm [batch, Hq, head_dim], then m [batch, Hq], then l [batch, Hq]
 * (Hq = num_kv_heads * num_q_per_kv). With M = max_r m_r and
 * w_r = exp(m_r - M) (0 where m_r = -inf): out = sum_r w_r o_r /
 * max(sum_r w_r l_r, 1e-6), summed in rank order, in out_dtype. If need
 * ([batch, num_kv_heads] uint8) is given, only the query heads of KV heads
 * with need != 0 are written. */
int cvsa_rank_merge(const float* parts, int32_t world, int64_t row_stride, int32_t batch,
                    int32_t num_kv_heads, int32_t num_q_per_kv, int32_t head_dim,
                    const uint8_t* need, void* out, int32_t out_dtype, void* stream);

/* The two log-sum-exps of the coverage gate per (sequence, KV head) row of
 * page scores [rows, max_pages] f32: lse_all over every entry (-inf entries
 * carry no mass) and lse_sel over the first n_per_head entries of the row's
 * page_indices [rows, max_sel] (indices outside [0, max_pages) skipped);
 * -inf when empty. A page-split rank exchanges these instead of its scores:
 * coverage = exp(lse_sel - lse_all) of cvsa/kernels/coverage.py:179-215,
 * with the sums taken over the ranks (cvsa_rank_accept). */
int cvsa_page_lse(const float* page_scores, int32_t rows, int32_t max_pages,
                  const int32_t* page_indices, int32_t max_sel, const int32_t* n_per_head,
                  float* lse_all, float* lse_sel, void* stream);

/* The coverage gate of a page split: for each of `rows` rows, coverage =
 * exp(LSE_r sel_r - LSE_r all_r) over the `world` gathered rows of parts
 * (rank r's lse_all at parts[r * row_stride + off_all + i], lse_sel at
 * off_sel + i), accept[i] = coverage >= tau (uint8), the decision of
 * cvsa/kernels/coverage.py:205-215. */
int cvsa_rank_accept(const float* parts, int32_t world, int64_t row_stride, int64_t off_all,
                     int64_t off_sel, int32_t rows, float tau, uint8_t* accept, void* stream);

/* ---- page split: the scoring / lazy-check step over ranks ----------------
 * Each rank (one process per GPU) holds a contiguous range of every
 * sequence's pages. The scoring step of cvsa/backend.py:683-864 and the lazy
 * check of :392-465 take two all-gathers per layer:
 *   cvsa_score_pages -> cvsa_split_propose -> all-gather of the exchange rows
 *   -> cvsa_split_gate -> cvsa_split_attend -> all-gather of the partials
 *   -> cvsa_rank_merge.
 * A reuse step (backend.py:866-881) is cvsa_sparse_decode of the cached
 * selection into the partials, one all-gather, cvsa_rank_merge.
 * Rank r's exchange row holds, for the rows = batch * num_kv_heads heads:
 *   [0, rows)            lse_all_r    log-sum-exp of its pages' scores
 *   [rows, 2 rows)       lse_cached_r of the cached selection's pages (-inf: none)
 *   [2 rows, 3 rows)     lse_forced_r of its forced pages
 *   [3 rows, 3 rows + rows * max_sel)  its best `budget` non-forced pages'
 *                        scores per head, page order, -inf padded
 * (cvsa_split_row_floats floats). */
typedef struct cvsa_split_desc {
  int32_t world;        /* ranks */
  int32_t rank;         /* this rank (the all-gather's row order) */
  int32_t batch;
  int32_t num_kv_heads;
  int32_t max_pages;    /* this rank's block-table width */
  int32_t block_size;
  int32_t budget;       /* top-k budget of the whole sequence (backend.py:690) */
  int32_t max_sel;      /* >= budget + sink + local of the whole sequence */
  int32_t sink_pages;   /* this rank's forced leading pages (rank 0: the sink) */
  int32_t local_pages;  /* this rank's forced trailing pages (last rank: the window) */
  float tau;            /* coverage threshold */
} cvsa_split_desc_t;

/* page-split step counters (int64 each), accumulated by cvsa_split_gate */
enum {
  CVSA_SPLIT_CTR_SCORING = 0,     /* scoring steps (backend.py _total_scoring_steps) */
  CVSA_SPLIT_CTR_ACCEPT = 1,      /* lazy checks whose cached selection passed */
  CVSA_SPLIT_CTR_REJECT = 2,      /* lazy checks that rescored */
  CVSA_SPLIT_CTR_HEADS_ACC = 3,   /* heads accepted */
  CVSA_SPLIT_CTR_CHECKS = 4,      /* coverage checks */
  CVSA_SPLIT_CTR_HEADS_TOTAL = 5, /* heads gated */
  CVSA_SPLIT_NUM_COUNTERS = 6
};

/* Floats of one rank's exchange row (the layout above); 0 on bad input. */
int64_t cvsa_split_row_floats(const cvsa_split_desc_t* sd);

/* This rank's part of exchange A from its page scores [batch, num_kv_heads,
 * max_pages] (cvsa_score_pages) and local context lengths [batch]; the cached
 * selection (rows of max_sel local pages, counts) may be NULL. Writes the
 * exchange row and proposal_pages [rows, max_sel] (local page of each
 * candidate slot, -1 unused). Candidates are pages outside the rank's forced
 * pages with finite scores; the best are (score descending, page ascending). */
int cvsa_split_propose(const cvsa_split_desc_t* sd, const float* page_scores,
                       const int32_t* context_lens, const int32_t* cached_indices,
                       const int32_t* cached_n, float* exchange_row, int32_t* proposal_pages,
                       void* stream);

/* After the all-gather of exchange rows (exchange [world, row_stride]): the
 * global top-`budget` of the gathered candidates, the coverage gate of that
 * selection (its candidates plus every rank's forced pages against the sum
 * over all ranks' pages; coverage.py:160-215), the lazy gate of the cached
 * selection when has_cache, and this rank's share of the new selection (its
 * sink pages, its chosen pages, its local pages; ascending) in sel [rows,
 * max_sel] / n_sel [rows] with its bitmap [rows, ceil(max_pages / 32)]
 * (nullable); accept [rows] = the new selection's gate. Identical on every
 * rank. state [4] int32, zeroed once and left zeroed except state[3], the
 * decision word (bit0: every head accepted the cached selection, so the
 * cached one is decoded; backend.py:446). stats_mode bit0: this is a lazy
 * check step, bit1: lazy mode; counters [CVSA_SPLIT_NUM_COUNTERS] or NULL. */
int cvsa_split_gate(const cvsa_split_desc_t* sd, const float* exchange, int64_t row_stride,
                    const int32_t* proposal_pages, const int32_t* context_lens,
                    int32_t has_cache, int32_t stats_mode, int32_t* sel, int32_t* n_sel,
                    uint8_t* accept, uint32_t* bitmap, int32_t* state, int64_t* counters,
                    int32_t* dev_error, void* stream);

/* The attention of a page-split scoring / lazy-check step, into the partials
 * of exchange B (o_unnorm [B, Hq, D], m, l [B, Hq] float32): heads decode the
 * cached selection when decision (nullable) has bit0 set, else the new one
 * (sel / n_sel), and a head whose new gate rejected (accept == 0) attends
 * every valid page of the rank (exact recovery: draft and complement
 * together, backend.py:818-844). When the new selection is decoded it is
 * copied into cached_indices / cached_n (nullable: no copy). The workspace is
 * cvsa_decode_workspace_size(qd, kv, max_sel) bytes. */
int cvsa_split_attend(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                      int32_t* cached_indices, int32_t* cached_n, const int32_t* sel,
                      const int32_t* n_sel, int32_t max_sel, const int32_t* decision,
                      const uint8_t* accept, const uint32_t* bitmap, float* o_unnorm, float* m,
                      float* l, int32_t* dev_error, void* workspace, size_t workspace_bytes,
                      void* stream);

/* ---- exchanges over NVLink peer memory (one process per GPU) -------------
 * A replacement for the small all-gathers of the page split and the decision
 * all-reduce of the head-sharded step: every rank allocates one exchange
 * buffer (cvsa_peer_alloc), passes its 64-byte IPC handle to the other ranks
 * (any host channel), maps theirs (cvsa_peer_open) and puts the world base
 * pointers, in rank order, in a device array. A call stores this rank's row
 * into every rank's buffer over NVLink, each 4-byte word beside the call's
 * number in one 8-byte store, and reads the other ranks' words as they land
 * (bounded waits: cvsa_set_wait_limit; CVSA_DEV_ERR_TIMEOUT when a rank never
 * arrives). Every rank must make the same sequence of calls with the same
 * sizes. */
typedef struct cvsa_peer_desc {
  const uint64_t* bases; /* device [world]: each rank's exchange buffer, mapped here */
  int32_t world;         /* <= 8 */
  int32_t rank;
  int64_t row_cap;       /* floats per rank row the buffers were sized for */
  int32_t* dev_error;    /* [1] CVSA_DEV_ERR_* bits, or NULL */
} cvsa_peer_desc_t;

/* Bytes of one rank's exchange buffer for rows of up to row_cap floats. */
size_t cvsa_peer_buffer_bytes(int32_t world, int64_t row_cap);
/* Allocate and zero an exchange buffer (cudaMalloc, set-up time) and write
 * its CUDA IPC handle (64 bytes) to ipc_handle. */
int cvsa_peer_alloc(size_t bytes, void** ptr, void* ipc_handle);
/* Map another rank's exchange buffer from its IPC handle. */
int cvsa_peer_open(const void* ipc_handle, void** ptr);
/* Unmap a buffer opened with cvsa_peer_open / free one from cvsa_peer_alloc. */
int cvsa_peer_close(void* ptr);
int cvsa_peer_free(void* ptr);
/* out [world, n] = every rank's src [n] (floats, or any 32-bit words), rank order. */
int cvsa_peer_allgather(const cvsa_peer_desc_t* pd, const float* src, int64_t n, float* out,
                        void* stream);
/* out [n] = element-wise minimum over the ranks of src [n] int32 (in place allowed). */
int cvsa_peer_min_i32(const cvsa_peer_desc_t* pd, const int32_t* src, int64_t n, int32_t* out,
                      void* stream);
/* The page split's exchange of attention partials and their merge in one
 * call: part = this rank's [o_unnorm (B·Hq·D) | m (B·Hq) | l (B·Hq)] row; out
 * [B, Hq, D] (out_dtype) = the merge of every rank's row in rank order
 * (cvsa_rank_merge's arithmetic), only heads with need != 0 when need
 * ([B, H_kv] uint8) is given. */
int cvsa_peer_merge(const cvsa_peer_desc_t* pd, const float* part, int32_t batch,
                    int32_t num_kv_heads, int32_t num_q_per_kv, int32_t head_dim,
                    const uint8_t* need, void* out, int32_t out_dtype, void* stream);

/* Fused exact recovery: for heads with accept == 0, attend to the valid pages
 * NOT in the selection (skipped through a selection bitmap, never
 * materialised as an index list) and LSE-merge that complement partial with
 * the given draft partial; accepted heads get o_d / max(l_d, 1e-6).
 * Replaces cvsa/backend.py:819-842 (triton_compute_complement +
 * triton_sparse_decode_unnorm on the complement + triton_lse_merge). */
int cvsa_recover_merge(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                       const int32_t* page_indices, int32_t max_sel,
                       const int32_t* n_per_head, const uint8_t* accept,
                       const float* o_d, const float* m_d, const float* l_d, void* out,
                       int32_t out_dtype, void* workspace, size_t workspace_bytes,
                       void* stream);

/* ---- fused whole-layer step (cvsa/backend.py:313-366) ---------------- */

enum {
  CVSA_MODE_SCORE = 0, /* _scoring_step (backend.py:683-864): fresh selection */
  CVSA_MODE_LAZY = 1,  /* _lazy_step (backend.py:392-465): gate the cached
                          selection on fresh scores; reuse it if every
                          (b, h) accepts, else a full scoring step */
  CVSA_MODE_REUSE = 2, /* _reuse_step (backend.py:866-881): cached selection */
  CVSA_MODE_DENSE = 3  /* dense layer (cvsa/runtime/dense.py:70-111) */
};

enum {
  CVSA_RECOVERY_EXACT = 0, /* complement + LSE merge (backend.py:818-844) */
  CVSA_RECOVERY_NONE = 1,  /* rejected heads keep the draft */
  CVSA_RECOVERY_APPROX = 2 /* rejected heads decode an expanded selection of
                              approx_budget pages (backend.py:780-817) */
};

/* device counters accumulated by cvsa_decode_step (int64 each) */
enum {
  CVSA_CTR_PAGES_ATTENDED = 0, /* backend.py:368-390 _attn_work */
  CVSA_CTR_PAGES_MAX = 1,      /* _attn_work_max: sum n_valid * num_kv_heads */
  CVSA_CTR_HEAD_ACCEPT = 2,    /* _per_head_accept_sum */
  CVSA_CTR_HEAD_TOTAL = 3,     /* _per_head_total */
  CVSA_CTR_ACCEPT_STEPS = 4,   /* _accept_counts */
  CVSA_CTR_REJECT_STEPS = 5,   /* _reject_counts */
  CVSA_CTR_SCORING_STEPS = 6,  /* _total_scoring_steps */
  CVSA_CTR_COVERAGE_CHECKS = 7,/* _total_coverage_checks */
  CVSA_NUM_COUNTERS = 8
};

typedef struct cvsa_step_config {
  int32_t mode;          /* CVSA_MODE_* */
  int32_t budget;        /* top-k budget: max(3, int(max_pages * budget_pct)) */
  int32_t sink_pages;    /* forced leading pages (0 = reference behaviour) */
  int32_t local_pages;   /* forced trailing pages (0 = reference behaviour) */
  float tau;             /* coverage threshold */
  int32_t recovery;      /* CVSA_RECOVERY_* */
  int32_t has_cache;     /* LAZY: cached_* holds this layer's selection */
  int32_t lazy_stats;    /* 1: count stats the way lazy mode does
                            (backend.py:420-465), 0: the fixed-interval way
                            (backend.py:775-862) */
  int32_t approx_budget; /* CVSA_RECOVERY_APPROX: pages of the expanded selection,
                            min(max(budget + 1, int(max_pages * pct)), max_pages)
                            (backend.py:782-783); forced pages come on top as in
                            the draft selection. Needs a bf16/f16 pool. */
} cvsa_step_config_t;

typedef struct cvsa_step_io {
  int32_t* cached_indices; /* [batch, num_kv_heads, max_sel] in/out (_cached_selection) */
  int32_t* cached_n;       /* [batch, num_kv_heads] in/out */
  int32_t max_sel;         /* >= budget + sink_pages + local_pages */
  int32_t phase;           /* CVSA_PHASE_*: the whole step, or its two halves around
                              an exchange of the lazy decision between ranks */
  void* out;               /* [batch, num_q_heads, head_dim], q dtype */
  float* page_scores;      /* [batch, num_kv_heads, max_pages] out, or NULL */
  uint8_t* accept;         /* [batch, num_kv_heads] gate of the selection decoded, or NULL */
  float* coverage;         /* [batch, num_kv_heads] or NULL */
  int64_t* counters;       /* [CVSA_NUM_COUNTERS] accumulated, or NULL */
  int32_t* step_flags;     /* [1]: bit0 every head accepted, bit1 rescored; or NULL.
                              REUSE and DENSE steps leave it (and accept/coverage)
                              as the last gated step wrote them. */
  int32_t* dev_error;      /* [1]: CVSA_DEV_ERR_* bits OR-ed in, or NULL */
  /* Optional per-kernel timing (backend.py:225-250): NULL, or CVSA_NUM_EVENTS
   * cudaEvent_t handles recorded on `stream` around the scoring, selection/
   * gate and attention kernels (begin, end each). Kernels a mode does not run
   * leave their pair unrecorded. Timing disables launch overlap (PDL). */
  void* const* timing_events;
} cvsa_step_io_t;

/* Phases of cvsa_decode_step. A step whose KV heads are sharded over ranks
 * (one process per GPU, each holding some KV heads of every sequence) needs
 * the lazy decision of backend.py:446 (accept_mask.all()) over all heads:
 * run CVSA_PHASE_SELECT, all-reduce the word at cvsa_step_decision_word with
 * MIN over the ranks (bit0: every cached head accepted), then run
 * CVSA_PHASE_ATTEND with the same arguments and workspace. The step
 * statistics of the selection count the rank's own decision. */
enum {
  CVSA_PHASE_ALL = 0,     /* scoring, selection and attention */
  CVSA_PHASE_SELECT = 1,  /* scoring and selection (LAZY / SCORE modes) */
  CVSA_PHASE_ATTEND = 2   /* attention, after CVSA_PHASE_SELECT */
};

enum {
  CVSA_EV_SCORE_BEGIN = 0, CVSA_EV_SCORE_END = 1,
  CVSA_EV_SELECT_BEGIN = 2, CVSA_EV_SELECT_END = 3,
  CVSA_EV_ATTEND_BEGIN = 4, CVSA_EV_ATTEND_END = 5,
  CVSA_NUM_EVENTS = 6
};

size_t cvsa_step_workspace_size(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                                const cvsa_step_config_t* cfg, int32_t max_sel);

/* One CVSA attention step for one layer, entirely on the device: no host
 * synchronisation, so the call can be captured in a CUDA graph. The batch-
 * global lazy decision (backend.py:446, accept_mask.all()) is taken on the
 * device. The workspace must be zeroed once before its first use
 * (cvsa_workspace_reset); the kernels leave their counters zeroed. */
int cvsa_decode_step(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                     const cvsa_step_config_t* cfg, const cvsa_step_io_t* io,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Zero a workspace (cudaMemsetAsync). */
int cvsa_workspace_reset(void* workspace, size_t workspace_bytes, void* stream);

/* The device word (int32) of a step workspace that holds the lazy decision
 * between CVSA_PHASE_SELECT and CVSA_PHASE_ATTEND (backend.py:446). */
int cvsa_step_decision_word(void* workspace, int32_t** word);

/* Polls a kernel's bounded waits on other warps of its CTA make before it
 * gives up, records CVSA_DEV_ERR_TIMEOUT in the step's error word and returns
 * without writing its outputs; 0 (the default) restores each kernel's own
 * limit (about 4M polls). Applies to launches made after the call, by every
 * host thread (a captured launch keeps the value it was captured with). It
 * exists so a test can make the waits run out; after a timeout the
 * workspace's counters may be left non-zero, so reset the workspace
 * (cvsa_workspace_reset) before its next use. Not in the reference. */
int cvsa_set_wait_limit(uint32_t polls);

/* ---- paged KV runtime (cvsa/runtime/kv_cache.py) -------------------- */

/* Append one token's K/V [batch, num_kv_heads, head_dim] (kv dtype) for each
 * of `batch` sequences. For sequence b: position = context_lens[b]; when the
 * position starts a new page past pages_allocated[b], a block is popped from
 * free_list[*free_head] (atomically) and written to block_tables[b, page].
 * Then K/V are written and context_lens[b] is incremented. seq_ids (nullable)
 * maps row b of k_new/v_new to a sequence slot.
 * Replaces SequenceKVManager.append_token_kv, kv_cache.py:133-150, and
 * PagedKVCache.allocate_blocks/write_kv, kv_cache.py:53-71, as one launch.
 * Pool exhaustion sets CVSA_DEV_ERR_POOL in *dev_error. */
int cvsa_paged_append(const cvsa_kv_desc_t* kv, const void* k_new, const void* v_new,
                      int32_t batch, const int32_t* seq_ids, int32_t* block_tables,
                      int32_t max_pages, int32_t* context_lens, int32_t* pages_allocated,
                      const int32_t* free_list, int32_t free_list_len, int32_t* free_head,
                      int32_t* dev_error, void* stream);

/* Gather the K (and V) pages of `n_pages` logical pages of one sequence into
 * a dense [n_pages * block_size, num_kv_heads, head_dim] buffer (nullable
 * v_out). A block id outside the pool sets CVSA_DEV_ERR_BLOCK_RANGE.
 * The gather counterpart of PagedKVCache.write_kv_block, kv_cache.py:73-80. */
int cvsa_paged_gather(const cvsa_kv_desc_t* kv, const int32_t* block_table_row,
                      int32_t n_pages, void* k_out, void* v_out, int32_t* dev_error,
                      void* stream);

/* ---- allocation-free decode ------------------------------------------ */

/* Size of the library's built-in decode scratch (see below). */
#define CVSA_NOALLOC_SCRATCH_BYTES (8u << 20)

/* The same sparse decode as cvsa_sparse_decode (same arguments and outputs),
 * for callers that cannot allocate device memory where they decode -- e.g. a
 * server whose memory pool is fully reserved at start-up, or a host runtime
 * that owns every allocation -- and so cannot provide a workspace. Its
 * scratch is a fixed array inside the library image
 * (CVSA_NOALLOC_SCRATCH_BYTES on every GPU that loads the library, held until
 * the process exits); it allocates nothing. This entry point has no
 * counterpart in the reference.
 *   - The first call on a device looks up that array's device address with
 *     cudaGetSymbolAddress (the current device must be the one decoding);
 *     make that first call before any stream capture. The address is kept
 *     per device and CUDA context: after cudaDeviceReset (or any other end of
 *     the context) the next call looks it up again, so that call too must
 *     come before a capture.
 *   - Shapes whose scratch would exceed CVSA_NOALLOC_SCRATCH_BYTES are
 *     rejected with CVSA_ERR_UNSUPPORTED and a message naming both sizes.
 *   - Every call on a device shares the one array, and each call clears the
 *     part that must start at zero: two calls that can overlap on the GPU
 *     (different streams without ordering between them) race and must not
 *     be issued; calls ordered on one stream are safe. */
int cvsa_sparse_decode_noalloc(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kv,
                               const int32_t* page_indices, int32_t max_sel,
                               const int32_t* n_per_head, float* o_unnorm, float* m, float* l,
                               void* out, int32_t out_dtype, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CVSA_B200_H_ */
