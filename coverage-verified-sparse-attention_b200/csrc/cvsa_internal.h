// Internal (C++) launch interface between the C-ABI layer (abi.cu) and the
// kernel files. Nothing here is exported from the shared library.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/cvsa_b200.h"

namespace cvsa {

struct KvView {
  const void* k;
  const void* v;
  int dtype;
  int num_blocks;
  int bs;   // tokens per page
  int hkv;  // KV heads
  int d;    // head_dim
  int64_t sb, st, sh;  // strides (elements): block, token, head
};

struct QView {
  const void* q;
  int dtype;
  int B;
  int hq;
  int W;  // block-table width (max_pages)
  const int32_t* tables;
  const int32_t* lens;
};

int num_sms();
int dtype_bytes(int dtype);
// Polls a kernel's bounded waits on other warps make before giving up with
// CVSA_DEV_ERR_TIMEOUT (cvsa_set_wait_limit); 0 = each kernel's default.
uint32_t wait_limit();

// Every workspace starts with a fixed region of counters that must be zero
// when a kernel starts and that the kernels return to zero: per-(b, kv head)
// tickets of the attention kernel, then the selection kernel's batch-global
// words in its last 256 bytes. Its offset never depends on the call's
// shapes, so calls of different shapes can share one workspace.
constexpr size_t kSyncRegionBytes = 256 * 1024;
constexpr int kMaxHeadsPerCall = (int)((kSyncRegionBytes - 256) / 4);  // batch * num_kv_heads
inline int32_t* ws_head_done(void* ws) { return reinterpret_cast<int32_t*>(ws); }
inline int32_t* ws_select_sync(void* ws) {
  return reinterpret_cast<int32_t*>(reinterpret_cast<uint8_t*>(ws) + kSyncRegionBytes - 256);
}

// ---- score.cu ----
cudaError_t launch_score_pages(const QView& q, const KvView& kv, float* scores,
                               int32_t* dev_err, cudaStream_t s, bool pdl);
bool score_supported(const QView& q, const KvView& kv);

// ---- quest.cu ----
cudaError_t launch_quest_scores(const QView& q, const KvView& kv, float* scores,
                                int32_t* dev_err, cudaStream_t s, bool pdl);
bool quest_supported(const QView& q, const KvView& kv);

// ---- select.cu ----
struct SelectParams {
  const float* scores;        // [B, Hkv, W]
  int B, hkv, W, bs;
  const int32_t* lens;
  int budget, sink, local;
  float tau;
  // new selection (nullable when only the cached gate is wanted)
  int32_t* sel_idx;           // [B, Hkv, max_sel]
  int32_t* sel_n;             // [B, Hkv]
  int max_sel;
  uint32_t* sel_bitmap;       // [B, Hkv, bitmap_words] or null
  int bitmap_words;
  uint8_t* accept;            // [B, Hkv] gate of the new selection, or null
  float* cov;                 // [B, Hkv] or null
  // cached selection gate (lazy mode)
  const int32_t* cached_idx;  // [B, Hkv, cached_stride] or null
  const int32_t* cached_n;
  int cached_stride;
  uint8_t* cached_accept;     // [B, Hkv] or null
  float* cached_cov;
  // batch-global decision & statistics
  int32_t* sync_ctr;          // [2] zeroed, 8-byte aligned: one 64-bit counter
                              // (CTAs done | rejected heads << 32)
  int32_t* decision;          // [1] out: bit0 all cached heads accepted
  int64_t* counters;          // [CVSA_NUM_COUNTERS] or null
  int mode;                   // CVSA_MODE_SCORE / CVSA_MODE_LAZY / -1 (plain select)
  int has_cache;
  int lazy_stats;
  int32_t* step_flags;        // [1] or null
  // compact list of the attention kernel's complement items (recovery): per
  // head ceil(n_valid / comp_chunk) items when its new gate rejects and the
  // batch rescored, else 0; the last CTA writes the exclusive scan.
  int32_t* comp_cnt;          // [B*Hkv] or null
  int32_t* comp_off;          // [B*Hkv + 1]
  int comp_chunk;
  int decision_external;      // the decision may change before the attention kernel reads it
                              // (phased steps): complement counts ignore the local reuse
};
cudaError_t launch_select_gate(const SelectParams& p, cudaStream_t s, bool pdl);

cudaError_t launch_build_bitmap(const int32_t* idx, int max_sel, const int32_t* n, int BH, int W,
                                uint32_t* bitmap, int words, int32_t* dev_err, cudaStream_t s);
cudaError_t launch_check_coverage(const float* scores, int B, int hkv, int W,
                                  const int32_t* idx, int max_sel, const int32_t* n,
                                  float tau, uint8_t* accept, float* cov, cudaStream_t s);
cudaError_t launch_complement(const int32_t* idx, int max_sel, const int32_t* n,
                              const int32_t* lens, int B, int hkv, int bs,
                              const uint8_t* accept, int32_t* comp, int max_comp,
                              int32_t* n_comp, cudaStream_t s);

// ---- attend.cu ----
// Which page set each (b, h) attends to and what the finaliser writes.
struct AttendParams {
  // selection sources: src 0 = sel0/n0, src 1 = sel1/n1; `use_src1` (device
  // word, bit0) picks src 1 when `src_select` == 2, otherwise src_select
  // fixes the source.
  const int32_t* sel0; const int32_t* n0;
  const int32_t* sel1; const int32_t* n1;
  int sel_stride;
  int src_select;                 // 0, 1, or 2 = decided on device
  const int32_t* decision;        // device word read when src_select == 2 (bit0: reuse src0)
  bool dense;                     // attend all valid pages, no selection
  // recovery (exact): heads with accept == 0 also attend their complement,
  // read from `bitmap` of the source-1 selection.
  bool recover;
  const uint8_t* accept;          // [B, Hkv]
  const uint32_t* bitmap;         // [B, Hkv, bitmap_words]
  int bitmap_words;
  const int32_t* comp_off;        // [heads + 1] complement-item offsets (select kernel), or
                                  // null: every head's complement chunks are enumerated
  bool external_draft;            // recover_merge: draft partial given, not recomputed
  const float* ext_o; const float* ext_m; const float* ext_l;
  // approximate recovery: rejected heads decode their expanded selection
  // (exp_idx / exp_n, rows of exp_stride) instead of every valid page
  bool approx;
  const int32_t* exp_idx; const int32_t* exp_n;
  int exp_stride;
  // copy the source-1 selection into source 0 when source 1 was used
  bool commit_src1;
  int32_t* commit_idx; int32_t* commit_n;
  // outputs
  void* out; int out_dtype;       // normalised output or null
  float* o_unnorm; float* m_out; float* l_out;  // draft partial or null
  int64_t* counters;              // pages attended / max, or null (CTA 0 reduces them)
  int32_t* dev_err;
  // gate outputs of the selection actually decoded (nullable): source 0's
  // gate (acc0/cov0, nullable = accepted) or source 1's (acc1/cov1)
  uint8_t* accept_out; float* cov_out;
  const uint8_t* acc0; const float* cov0;
  const uint8_t* acc1; const float* cov1;
  // scratch: item partials (attend_workspace_bytes) and the zero-initialised
  // per-(b, h) tickets (ws_head_done of the call's workspace)
  void* partials; size_t partial_bytes;
  int32_t* head_done;
};
// Bytes of item-partial scratch (excluding the sync region).
size_t attend_workspace_bytes(const QView& q, const KvView& kv, int max_sel, bool recover,
                              bool dense);
cudaError_t launch_attend(const QView& q, const KvView& kv, const AttendParams& p,
                          int max_sel, cudaStream_t s, bool pdl);
bool attend_supported(const QView& q, const KvView& kv);
int attend_complement_chunk();  // logical pages per complement item

// ---- attend_stream.cu (bf16 / f16, 16-byte-aligned pools; launch_attend routes) ----
bool stream_attend_eligible(const QView& q, const KvView& kv);
size_t stream_attend_workspace_bytes(const QView& q, const KvView& kv, int max_sel);
cudaError_t launch_stream_attend(const QView& q, const KvView& kv, const AttendParams& p,
                                 int max_sel, cudaStream_t s, bool pdl);

// ---- split.cu (page-split step: selection over ranks) ----
struct SplitProposeParams {
  const float* scores;          // [rows, W] this rank's page scores
  int rows, W, H;               // rows = B * H
  const int32_t* lens;          // [B] this rank's context lengths (tokens in its range)
  int bs;
  const int32_t* cached_idx;    // [rows, cached_stride] or null
  const int32_t* cached_n;      // [rows]
  int cached_stride;
  int sink, local, budget, max_sel;
  float* ex;                    // this rank's exchange-A row
  int64_t off_all, off_cached, off_forced, off_cand;
  int32_t* prop_idx;            // [rows, max_sel] local pages of the candidates
};
struct SplitGateParams {
  const float* parts;           // [world, stride] gathered exchange-A rows
  int world, rank;
  int64_t stride, off_all, off_cached, off_forced, off_cand;
  int rows, H, max_sel, budget;
  float tau;
  const int32_t* prop_idx;      // [rows, max_sel] this rank's candidates' pages
  const int32_t* lens;          // [B] this rank's context lengths
  int bs, W;                    // W = this rank's table width
  int sink, local;              // this rank's forced pages
  int has_cache;                // gate the cached selection (lazy check step)
  int stats_mode;               // bit0: lazy check step, bit1: lazy mode
  int32_t* sel; int32_t* n;     // [rows, max_sel], [rows] this rank's new selection
  uint8_t* acc;                 // [rows] gate of the new selection
  uint32_t* bitmap;             // [rows, bitmap_words] of the new selection, or null
  int bitmap_words;             // >= ceil(W / 32)
  int32_t* state;               // [4] zeroed once: tickets, two accept counts, decision word
  int64_t* counters;            // [CVSA_SPLIT_NUM_COUNTERS] or null
  int32_t* dev_err;
};
size_t split_propose_smem(int W);
size_t split_gate_smem(int world, int max_sel, int bitmap_words);
cudaError_t launch_split_propose(const SplitProposeParams& p, cudaStream_t s, bool pdl);
cudaError_t launch_split_gate(const SplitGateParams& p, cudaStream_t s, bool pdl);

// ---- peer.cu (exchanges over NVLink peer memory) ----
struct PeerView {
  const uint64_t* bases;  // [world] device array: every rank's exchange buffer mapped here
  int world, rank;
  int64_t row_cap;        // floats per rank row
  int32_t* dev_err;
};
size_t peer_buffer_bytes(int world, int64_t row_cap);
bool peer_shape_ok(const PeerView& pv);
int peer_max_ctas();
cudaError_t launch_peer_gather(const PeerView& pv, const float* src, int64_t n, float* out,
                               bool min_i32, cudaStream_t s);
cudaError_t launch_peer_merge(const PeerView& pv, const float* part, int B, int hkv, int G, int D,
                              const uint8_t* need, void* out, int out_dtype, cudaStream_t s);

// ---- merge.cu ----
cudaError_t launch_lse_merge(const float* o_d, const float* m_d, const float* l_d,
                             const float* o_c, const float* m_c, const float* l_c,
                             const uint8_t* accept, int B, int hkv, int G, int D, void* out,
                             int out_dtype, cudaStream_t s);
cudaError_t launch_rank_merge(const float* parts, int world, int64_t stride, int B, int hkv,
                              int G, int D, const uint8_t* need, void* out, int out_dtype,
                              cudaStream_t s);
cudaError_t launch_page_lse(const float* scores, int rows, int W, const int32_t* idx,
                            int max_sel, const int32_t* n, float* lse_all, float* lse_sel,
                            cudaStream_t s);
cudaError_t launch_rank_accept(const float* parts, int world, int64_t stride, int64_t off_all,
                               int64_t off_sel, int rows, float tau, uint8_t* accept,
                               cudaStream_t s);

// ---- paged_kv.cu ----
cudaError_t launch_paged_append(const KvView& kv, const void* k_new, const void* v_new, int B,
                                const int32_t* seq_ids, int32_t* tables, int W, int32_t* lens,
                                int32_t* pages_alloc, const int32_t* free_list, int free_len,
                                int32_t* free_head, int32_t* dev_err, cudaStream_t s);
cudaError_t launch_paged_gather(const KvView& kv, const int32_t* row, int n_pages, void* k_out,
                                void* v_out, int32_t* dev_err, cudaStream_t s);

}  // namespace cvsa
