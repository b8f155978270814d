// extern "C" entry points of libcvsa_b200.so (declared in include/cvsa_b200.h).
//
// This layer validates arguments (returning the status codes the Python
// shims map to the reference's exceptions), carves caller-provided
// workspaces, and sequences the kernels of one CVSA layer step on the
// caller's stream. It never synchronises, and allocates device memory only in
// the set-up call cvsa_peer_alloc.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>

#include "cvsa_internal.h"

namespace cvsa {

int dtype_bytes(int dtype) {
  switch (dtype) {
    case CVSA_DTYPE_F32: return 4;
    case CVSA_DTYPE_F16: return 2;
    case CVSA_DTYPE_BF16: return 2;
    default: return 0;
  }
}

std::atomic<uint32_t> g_wait_limit{0};
uint32_t wait_limit() { return g_wait_limit.load(std::memory_order_relaxed); }

int num_sms() {
  static int cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
    n = 148;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

}  // namespace cvsa

using namespace cvsa;

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return CVSA_OK;
  return fail(CVSA_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

bool valid_dtype(int dt) { return dt == CVSA_DTYPE_F32 || dt == CVSA_DTYPE_F16 || dt == CVSA_DTYPE_BF16; }

int check_kv(const cvsa_kv_desc_t* kv, KvView* out) {
  if (!kv) return fail(CVSA_ERR_INVALID, "kv descriptor is NULL");
  if (!kv->k_cache || !kv->v_cache) return fail(CVSA_ERR_INVALID, "k_cache/v_cache is NULL");
  if (!valid_dtype(kv->dtype)) return fail(CVSA_ERR_INVALID, "kv dtype %d unknown", kv->dtype);
  if (kv->num_blocks <= 0 || kv->block_size <= 0 || kv->num_kv_heads <= 0 || kv->head_dim <= 0)
    return fail(CVSA_ERR_INVALID, "kv shape must be positive (blocks=%d bs=%d hkv=%d d=%d)",
                kv->num_blocks, kv->block_size, kv->num_kv_heads, kv->head_dim);
  const int eb = dtype_bytes(kv->dtype);
  if (kv->stride_head < kv->head_dim || kv->stride_token < 1 || kv->stride_block < 1)
    return fail(CVSA_ERR_INVALID, "kv strides inconsistent with head_dim");
  if ((reinterpret_cast<uintptr_t>(kv->k_cache) | reinterpret_cast<uintptr_t>(kv->v_cache)) % 16 ||
      (kv->stride_head * eb) % 16 || (kv->stride_token * eb) % 16 ||
      (kv->stride_block * eb) % 16 || (kv->head_dim * eb) % 16)
    return fail(CVSA_ERR_INVALID, "kv rows must be 16-byte aligned");
  out->k = kv->k_cache;
  out->v = kv->v_cache;
  out->dtype = kv->dtype;
  out->num_blocks = kv->num_blocks;
  out->bs = kv->block_size;
  out->hkv = kv->num_kv_heads;
  out->d = kv->head_dim;
  out->sb = kv->stride_block;
  out->st = kv->stride_token;
  out->sh = kv->stride_head;
  return CVSA_OK;
}

int check_q(const cvsa_query_desc_t* qd, const KvView& kv, bool need_q, QView* out) {
  if (!qd) return fail(CVSA_ERR_INVALID, "query descriptor is NULL");
  if (need_q && !qd->q) return fail(CVSA_ERR_INVALID, "q is NULL");
  if (!valid_dtype(qd->dtype)) return fail(CVSA_ERR_INVALID, "q dtype %d unknown", qd->dtype);
  if (qd->batch < 0) return fail(CVSA_ERR_INVALID, "batch < 0");
  if (qd->num_q_heads <= 0 || qd->num_q_heads % kv.hkv != 0)
    return fail(CVSA_ERR_INVALID, "num_q_heads=%d is not a positive multiple of num_kv_heads=%d",
                qd->num_q_heads, kv.hkv);
  if (qd->max_pages <= 0) return fail(CVSA_ERR_INVALID, "max_pages must be positive");
  if (qd->batch > 0 && (!qd->block_tables || !qd->context_lens))
    return fail(CVSA_ERR_INVALID, "block_tables/context_lens is NULL");
  if (need_q && (reinterpret_cast<uintptr_t>(qd->q) % 16))
    return fail(CVSA_ERR_INVALID, "q must be 16-byte aligned");
  if ((int64_t)qd->batch * kv.hkv > kMaxHeadsPerCall)
    return fail(CVSA_ERR_UNSUPPORTED, "batch * num_kv_heads above %d", kMaxHeadsPerCall);
  out->q = qd->q;
  out->dtype = qd->dtype;
  out->B = qd->batch;
  out->hq = qd->num_q_heads;
  out->W = qd->max_pages;
  out->tables = qd->block_tables;
  out->lens = qd->context_lens;
  return CVSA_OK;
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// Largest page count the select kernel can hold in shared memory.
constexpr int kMaxPagesSelect = 40000;

int bitmap_words(int W) { return (W + 31) / 32; }

// Decode / recovery workspace: [sync region][item partials][selection bitmap].
struct DecodeLayout {
  size_t partials, partial_bytes, bitmap, total;
};

DecodeLayout decode_layout(const QView& q, const KvView& kv, int max_sel) {
  DecodeLayout L;
  size_t a = attend_workspace_bytes(q, kv, max_sel, false, false);
  size_t b = attend_workspace_bytes(q, kv, max_sel, true, false);
  L.partials = kSyncRegionBytes;
  L.partial_bytes = a > b ? a : b;
  L.bitmap = L.partials + L.partial_bytes;
  L.total = L.bitmap + align256((size_t)q.B * kv.hkv * bitmap_words(q.W) * 4);
  return L;
}

size_t decode_ws(const QView& q, const KvView& kv, int max_sel) {
  return decode_layout(q, kv, max_sel).total;
}

// Step workspace: [sync region][scores][selection][n][bitmap][gates][partials].
struct StepLayout {
  size_t scores, sel, n, bitmap, acc_new, cov_new, acc_c, cov_c, comp_cnt, comp_off, exp_sel,
      exp_n, attend, total;
};

// exp_stride: row width of the expanded selection (approximate recovery), or 0
StepLayout step_layout(const QView& q, const KvView& kv, int max_sel, bool recover, bool dense,
                       int exp_stride = 0) {
  StepLayout L;
  const size_t bh = (size_t)q.B * kv.hkv;
  size_t off = kSyncRegionBytes;
  L.scores = off; off += align256(bh * q.W * 4);
  L.sel = off; off += align256(bh * max_sel * 4);
  L.n = off; off += align256(bh * 4);
  L.bitmap = off; off += align256(bh * bitmap_words(q.W) * 4);
  L.acc_new = off; off += align256(bh);
  L.cov_new = off; off += align256(bh * 4);
  L.acc_c = off; off += align256(bh);
  L.cov_c = off; off += align256(bh * 4);
  L.comp_cnt = off; off += align256(bh * 4);
  L.comp_off = off; off += align256((bh + 1) * 4);
  L.exp_sel = off; off += align256(bh * (size_t)exp_stride * 4);
  L.exp_n = off; off += align256(exp_stride > 0 ? bh * 4 : 0);
  L.attend = off; off += attend_workspace_bytes(q, kv, max_sel, recover, dense);
  L.total = off;
  return L;
}

}  // namespace

extern "C" {

int cvsa_abi_version(void) { return CVSA_ABI_VERSION; }

const char* cvsa_status_string(int status) {
  switch (status) {
    case CVSA_OK: return "ok";
    case CVSA_ERR_INVALID: return "invalid argument";
    case CVSA_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case CVSA_ERR_WORKSPACE: return "workspace too small or misaligned";
    case CVSA_ERR_CUDA: return "CUDA error";
    case CVSA_ERR_POOL: return "page pool exhausted";
    default: return "unknown status";
  }
}

const char* cvsa_last_error(void) { return g_last_error.c_str(); }

int cvsa_set_wait_limit(uint32_t polls) {
  g_wait_limit.store(polls, std::memory_order_relaxed);
  return CVSA_OK;
}

int cvsa_score_pages(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd, float* page_scores,
                     void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (!page_scores) return fail(CVSA_ERR_INVALID, "page_scores is NULL");
  if (!score_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "scoring built for block_size 16, head_dim 64/128/256");
  if (q.B == 0) return CVSA_OK;
  return cuda_status(launch_score_pages(q, kv, page_scores, nullptr, (cudaStream_t)stream, false),
                     "score_pages launch");
}

int cvsa_quest_scores(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd, float* page_scores,
                      int32_t* dev_error, void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (!page_scores) return fail(CVSA_ERR_INVALID, "page_scores is NULL");
  if (!quest_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED,
                "quest scoring built for block_size 16, head_dim 64/128/256 (fp32: 64/128), "
                "num_kv_heads * head_dim <= 12288");
  if (q.B == 0) return CVSA_OK;
  return cuda_status(launch_quest_scores(q, kv, page_scores, dev_error, (cudaStream_t)stream,
                                         false),
                     "quest_scores launch");
}

int cvsa_select_pages(const float* page_scores, int32_t batch, int32_t num_kv_heads,
                      int32_t max_pages, const int32_t* context_lens, int32_t block_size,
                      int32_t budget, int32_t sink_pages, int32_t local_pages,
                      int32_t* page_indices, int32_t max_sel, int32_t* n_per_head,
                      void* stream) {
  if (batch < 0 || num_kv_heads <= 0 || max_pages <= 0 || block_size <= 0)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if (budget < 0 || sink_pages < 0 || local_pages < 0)
    return fail(CVSA_ERR_INVALID, "budget/sink/local must be >= 0");
  if (max_sel < budget + sink_pages + local_pages || max_sel <= 0)
    return fail(CVSA_ERR_INVALID, "max_sel=%d < budget+sink+local=%d", max_sel,
                budget + sink_pages + local_pages);
  if (max_pages > kMaxPagesSelect)
    return fail(CVSA_ERR_UNSUPPORTED, "max_pages=%d above %d", max_pages, kMaxPagesSelect);
  if (batch == 0) return CVSA_OK;
  if (!page_scores || !context_lens || !page_indices || !n_per_head)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  SelectParams p;
  memset(&p, 0, sizeof(p));
  p.scores = page_scores;
  p.B = batch;
  p.hkv = num_kv_heads;
  p.W = max_pages;
  p.bs = block_size;
  p.lens = context_lens;
  p.budget = budget;
  p.sink = sink_pages;
  p.local = local_pages;
  p.tau = 0.f;
  p.sel_idx = page_indices;
  p.sel_n = n_per_head;
  p.max_sel = max_sel;
  p.mode = -1;
  return cuda_status(launch_select_gate(p, (cudaStream_t)stream, false), "select launch");
}

int cvsa_check_coverage(const float* page_scores, int32_t batch, int32_t num_kv_heads,
                        int32_t max_pages, const int32_t* page_indices, int32_t max_sel,
                        const int32_t* n_per_head, float tau, uint8_t* accept, float* coverage,
                        void* stream) {
  if (batch < 0 || num_kv_heads <= 0 || max_pages <= 0 || max_sel <= 0)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if (max_pages > kMaxPagesSelect)
    return fail(CVSA_ERR_UNSUPPORTED, "max_pages=%d above %d", max_pages, kMaxPagesSelect);
  if (batch == 0) return CVSA_OK;
  if (!page_scores || !page_indices || !n_per_head || !accept)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  return cuda_status(launch_check_coverage(page_scores, batch, num_kv_heads, max_pages,
                                           page_indices, max_sel, n_per_head, tau, accept,
                                           coverage, (cudaStream_t)stream),
                     "coverage launch");
}

int cvsa_compute_complement(const int32_t* page_indices, int32_t max_sel,
                            const int32_t* n_per_head, const int32_t* context_lens, int32_t batch,
                            int32_t num_kv_heads, int32_t block_size, const uint8_t* accept,
                            int32_t* complement, int32_t max_comp, int32_t* n_complement,
                            void* stream) {
  if (batch < 0 || num_kv_heads <= 0 || block_size <= 0 || max_sel <= 0 || max_comp <= 0)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if ((int64_t)max_comp + max_sel > 200000)
    return fail(CVSA_ERR_UNSUPPORTED, "max_comp + max_sel above 200000");
  if (batch == 0) return CVSA_OK;
  if (!page_indices || !n_per_head || !context_lens || !complement || !n_complement)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  return cuda_status(launch_complement(page_indices, max_sel, n_per_head, context_lens, batch,
                                       num_kv_heads, block_size, accept, complement, max_comp,
                                       n_complement, (cudaStream_t)stream),
                     "complement launch");
}

size_t cvsa_decode_workspace_size(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd,
                                  int32_t max_sel) {
  KvView kv;
  QView q;
  if (check_kv(kvd, &kv) || check_q(qd, kv, false, &q) || max_sel <= 0) return 0;
  return decode_ws(q, kv, max_sel);
}

int cvsa_sparse_decode(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd,
                       const int32_t* page_indices, int32_t max_sel, const int32_t* n_per_head,
                       float* o_unnorm, float* m, float* l, void* out, int32_t out_dtype,
                       void* workspace, size_t workspace_bytes, void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (max_sel <= 0) return fail(CVSA_ERR_INVALID, "max_sel must be positive");
  if (!attend_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "decode built for block_size 16, head_dim 64/128/256, G<=16");
  if (out && !valid_dtype(out_dtype)) return fail(CVSA_ERR_INVALID, "out dtype unknown");
  if (!out && !o_unnorm && !m && !l) return fail(CVSA_ERR_INVALID, "no output requested");
  if (q.B == 0) return CVSA_OK;
  if (!page_indices || !n_per_head) return fail(CVSA_ERR_INVALID, "NULL selection");
  const size_t need = decode_ws(q, kv, max_sel);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(CVSA_ERR_WORKSPACE, "workspace needs %zu bytes, 256-aligned", need);
  AttendParams p;
  memset(&p, 0, sizeof(p));
  p.sel0 = page_indices;
  p.n0 = n_per_head;
  p.sel_stride = max_sel;
  p.src_select = 0;
  p.out = out;
  p.out_dtype = out_dtype;
  p.o_unnorm = o_unnorm;
  p.m_out = m;
  p.l_out = l;
  const DecodeLayout L = decode_layout(q, kv, max_sel);
  p.partials = reinterpret_cast<uint8_t*>(workspace) + L.partials;
  p.partial_bytes = L.partial_bytes;
  p.head_done = ws_head_done(workspace);
  return cuda_status(launch_attend(q, kv, p, max_sel, (cudaStream_t)stream, false),
                     "decode launch");
}

int cvsa_lse_merge(const float* o_d, const float* m_d, const float* l_d, const float* o_c,
                   const float* m_c, const float* l_c, const uint8_t* accept, int32_t batch,
                   int32_t num_kv_heads, int32_t num_q_per_kv, int32_t head_dim, void* out,
                   int32_t out_dtype, void* stream) {
  if (batch < 0 || num_kv_heads <= 0 || num_q_per_kv <= 0 || head_dim <= 0)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if (!valid_dtype(out_dtype)) return fail(CVSA_ERR_INVALID, "out dtype unknown");
  if (batch == 0) return CVSA_OK;
  if (!o_d || !m_d || !l_d || !o_c || !m_c || !l_c || !accept || !out)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  return cuda_status(launch_lse_merge(o_d, m_d, l_d, o_c, m_c, l_c, accept, batch, num_kv_heads,
                                      num_q_per_kv, head_dim, out, out_dtype,
                                      (cudaStream_t)stream),
                     "lse_merge launch");
}

int cvsa_rank_merge(const float* parts, int32_t world, int64_t row_stride, int32_t batch,
                    int32_t num_kv_heads, int32_t num_q_per_kv, int32_t head_dim,
                    const uint8_t* need, void* out, int32_t out_dtype, void* stream) {
  if (world <= 0 || batch < 0 || num_kv_heads <= 0 || num_q_per_kv <= 0 || head_dim <= 0)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if (!valid_dtype(out_dtype)) return fail(CVSA_ERR_INVALID, "out dtype unknown");
  const int64_t rows = (int64_t)batch * num_kv_heads * num_q_per_kv;
  if (row_stride < rows * (head_dim + 2)) return fail(CVSA_ERR_INVALID, "row_stride too small");
  if (batch == 0) return CVSA_OK;
  if (!parts || !out) return fail(CVSA_ERR_INVALID, "NULL pointer");
  return cuda_status(launch_rank_merge(parts, world, row_stride, batch, num_kv_heads,
                                       num_q_per_kv, head_dim, need, out, out_dtype,
                                       (cudaStream_t)stream),
                     "rank_merge launch");
}

int cvsa_page_lse(const float* page_scores, int32_t rows, int32_t max_pages,
                  const int32_t* page_indices, int32_t max_sel, const int32_t* n_per_head,
                  float* lse_all, float* lse_sel, void* stream) {
  if (rows < 0 || max_pages <= 0 || max_sel <= 0) return fail(CVSA_ERR_INVALID, "bad shape");
  if (rows == 0) return CVSA_OK;
  if (!page_scores || !page_indices || !n_per_head || !lse_all || !lse_sel)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  return cuda_status(launch_page_lse(page_scores, rows, max_pages, page_indices, max_sel,
                                     n_per_head, lse_all, lse_sel, (cudaStream_t)stream),
                     "page_lse launch");
}

int cvsa_rank_accept(const float* parts, int32_t world, int64_t row_stride, int64_t off_all,
                     int64_t off_sel, int32_t rows, float tau, uint8_t* accept, void* stream) {
  if (world <= 0 || rows < 0 || off_all < 0 || off_sel < 0 || off_all + rows > row_stride ||
      off_sel + rows > row_stride)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if (rows == 0) return CVSA_OK;
  if (!parts || !accept) return fail(CVSA_ERR_INVALID, "NULL pointer");
  return cuda_status(launch_rank_accept(parts, world, row_stride, off_all, off_sel, rows, tau,
                                        accept, (cudaStream_t)stream),
                     "rank_accept launch");
}

namespace {
// Checks a split descriptor; rows = batch * num_kv_heads.
int check_split(const cvsa_split_desc_t* sd, int64_t* rows) {
  if (!sd) return fail(CVSA_ERR_INVALID, "NULL split descriptor");
  if (sd->world <= 0 || sd->rank < 0 || sd->rank >= sd->world || sd->batch < 0 ||
      sd->num_kv_heads <= 0 || sd->max_pages <= 0 || sd->block_size <= 0 || sd->budget < 0 ||
      sd->max_sel <= 0 || sd->sink_pages < 0 || sd->local_pages < 0)
    return fail(CVSA_ERR_INVALID, "bad split descriptor");
  if (sd->budget + sd->sink_pages + sd->local_pages > sd->max_sel)
    return fail(CVSA_ERR_INVALID, "max_sel < budget + sink_pages + local_pages");
  if ((int64_t)sd->batch * sd->num_kv_heads > INT32_MAX / 2)
    return fail(CVSA_ERR_INVALID, "too many heads");
  *rows = (int64_t)sd->batch * sd->num_kv_heads;
  return CVSA_OK;
}
}  // namespace

int64_t cvsa_split_row_floats(const cvsa_split_desc_t* sd) {
  int64_t rows;
  if (check_split(sd, &rows)) return 0;
  return rows * 3 + rows * sd->max_sel;
}

int cvsa_split_propose(const cvsa_split_desc_t* sd, const float* page_scores,
                       const int32_t* context_lens, const int32_t* cached_indices,
                       const int32_t* cached_n, float* exchange_row, int32_t* proposal_pages,
                       void* stream) {
  int64_t rows;
  int st = check_split(sd, &rows);
  if (st) return st;
  if (rows == 0) return CVSA_OK;
  if (!page_scores || !context_lens || !exchange_row || !proposal_pages)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  if ((cached_indices == nullptr) != (cached_n == nullptr))
    return fail(CVSA_ERR_INVALID, "cached_indices and cached_n go together");
  if (split_propose_smem(sd->max_pages) > 200 * 1024)
    return fail(CVSA_ERR_UNSUPPORTED, "split_propose supports up to 51200 pages per rank");
  SplitProposeParams p;
  memset(&p, 0, sizeof(p));
  p.scores = page_scores;
  p.rows = (int)rows;
  p.W = sd->max_pages;
  p.H = sd->num_kv_heads;
  p.lens = context_lens;
  p.bs = sd->block_size;
  p.cached_idx = cached_indices;
  p.cached_n = cached_n;
  p.cached_stride = sd->max_sel;
  p.sink = sd->sink_pages;
  p.local = sd->local_pages;
  p.budget = sd->budget;
  p.max_sel = sd->max_sel;
  p.ex = exchange_row;
  p.off_all = 0;
  p.off_cached = rows;
  p.off_forced = 2 * rows;
  p.off_cand = 3 * rows;
  p.prop_idx = proposal_pages;
  return cuda_status(launch_split_propose(p, (cudaStream_t)stream, false), "split_propose launch");
}

int cvsa_split_gate(const cvsa_split_desc_t* sd, const float* exchange, int64_t row_stride,
                    const int32_t* proposal_pages, const int32_t* context_lens,
                    int32_t has_cache, int32_t stats_mode, int32_t* sel, int32_t* n_sel,
                    uint8_t* accept, uint32_t* bitmap, int32_t* state, int64_t* counters,
                    int32_t* dev_error, void* stream) {
  int64_t rows;
  int st = check_split(sd, &rows);
  if (st) return st;
  if (row_stride < rows * 3 + rows * sd->max_sel) return fail(CVSA_ERR_INVALID, "row_stride too small");
  if (rows == 0) return CVSA_OK;
  if (!exchange || !proposal_pages || !context_lens || !sel || !n_sel || !accept || !state)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  const int words = bitmap_words(sd->max_pages);
  if (split_gate_smem(sd->world, sd->max_sel, words) > 200 * 1024)
    return fail(CVSA_ERR_UNSUPPORTED, "world * max_sel too large for split_gate");
  SplitGateParams p;
  memset(&p, 0, sizeof(p));
  p.parts = exchange;
  p.world = sd->world;
  p.rank = sd->rank;
  p.stride = row_stride;
  p.off_all = 0;
  p.off_cached = rows;
  p.off_forced = 2 * rows;
  p.off_cand = 3 * rows;
  p.rows = (int)rows;
  p.H = sd->num_kv_heads;
  p.max_sel = sd->max_sel;
  p.budget = sd->budget;
  p.tau = sd->tau;
  p.prop_idx = proposal_pages;
  p.lens = context_lens;
  p.bs = sd->block_size;
  p.W = sd->max_pages;
  p.sink = sd->sink_pages;
  p.local = sd->local_pages;
  p.has_cache = has_cache ? 1 : 0;
  p.stats_mode = stats_mode;
  p.sel = sel;
  p.n = n_sel;
  p.acc = accept;
  p.bitmap = bitmap;
  p.bitmap_words = words;
  p.state = state;
  p.counters = counters;
  p.dev_err = dev_error;
  return cuda_status(launch_split_gate(p, (cudaStream_t)stream, false), "split_gate launch");
}

int cvsa_split_attend(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd,
                      int32_t* cached_indices, int32_t* cached_n, const int32_t* sel,
                      const int32_t* n_sel, int32_t max_sel, const int32_t* decision,
                      const uint8_t* accept, const uint32_t* bitmap, float* o_unnorm, float* m,
                      float* l, int32_t* dev_error, void* workspace, size_t workspace_bytes,
                      void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (max_sel <= 0) return fail(CVSA_ERR_INVALID, "max_sel must be positive");
  if (!attend_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "decode built for block_size 16, head_dim 64/128/256, G<=16");
  if (!o_unnorm || !m || !l) return fail(CVSA_ERR_INVALID, "the partial outputs are required");
  if (q.B == 0) return CVSA_OK;
  if (!sel || !n_sel || !accept || !bitmap) return fail(CVSA_ERR_INVALID, "NULL selection");
  if (decision && (!cached_indices || !cached_n))
    return fail(CVSA_ERR_INVALID, "a decision needs the cached selection");
  if ((cached_indices == nullptr) != (cached_n == nullptr))
    return fail(CVSA_ERR_INVALID, "cached_indices and cached_n go together");
  const size_t need = decode_ws(q, kv, max_sel);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(CVSA_ERR_WORKSPACE, "workspace needs %zu bytes, 256-aligned", need);
  AttendParams p;
  memset(&p, 0, sizeof(p));
  p.sel0 = cached_indices;
  p.n0 = cached_n;
  p.sel1 = sel;
  p.n1 = n_sel;
  p.sel_stride = max_sel;
  p.src_select = decision ? 2 : 1;
  p.decision = decision;
  p.recover = true;
  p.accept = accept;
  p.bitmap = bitmap;
  p.bitmap_words = bitmap_words(q.W);
  p.commit_src1 = cached_indices != nullptr;
  p.commit_idx = cached_indices;
  p.commit_n = cached_n;
  p.o_unnorm = o_unnorm;
  p.m_out = m;
  p.l_out = l;
  p.dev_err = dev_error;
  const DecodeLayout L = decode_layout(q, kv, max_sel);
  p.partials = reinterpret_cast<uint8_t*>(workspace) + L.partials;
  p.partial_bytes = L.partial_bytes;
  p.head_done = ws_head_done(workspace);
  return cuda_status(launch_attend(q, kv, p, max_sel, (cudaStream_t)stream, false),
                     "split attend launch");
}

namespace {
int check_peer(const cvsa_peer_desc_t* pd, PeerView* pv) {
  if (!pd) return fail(CVSA_ERR_INVALID, "NULL peer descriptor");
  pv->bases = pd->bases;
  pv->world = pd->world;
  pv->rank = pd->rank;
  pv->row_cap = pd->row_cap;
  pv->dev_err = pd->dev_error;
  if (!peer_shape_ok(*pv)) return fail(CVSA_ERR_INVALID, "bad peer descriptor (world <= 8)");
  return CVSA_OK;
}
}  // namespace

size_t cvsa_peer_buffer_bytes(int32_t world, int64_t row_cap) {
  if (world < 1 || world > 8 || row_cap <= 0) return 0;
  return peer_buffer_bytes(world, row_cap);
}

int cvsa_peer_alloc(size_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes == 0) return fail(CVSA_ERR_INVALID, "bad peer_alloc arguments");
  void* p = nullptr;
  int st = cuda_status(cudaMalloc(&p, bytes), "cudaMalloc (peer buffer)");
  if (st) return st;
  st = cuda_status(cudaMemset(p, 0, bytes), "cudaMemset (peer buffer)");
  if (!st) {
    cudaIpcMemHandle_t h;
    st = cuda_status(cudaIpcGetMemHandle(&h, p), "cudaIpcGetMemHandle");
    if (!st) memcpy(ipc_handle, &h, sizeof(h));
  }
  if (st) {
    cudaFree(p);
    return st;
  }
  *ptr = p;
  return CVSA_OK;
}

int cvsa_peer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return fail(CVSA_ERR_INVALID, "NULL pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess),
                     "cudaIpcOpenMemHandle");
}

int cvsa_peer_close(void* ptr) {
  if (!ptr) return CVSA_OK;
  return cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

int cvsa_peer_free(void* ptr) {
  if (!ptr) return CVSA_OK;
  return cuda_status(cudaFree(ptr), "cudaFree (peer buffer)");
}

int cvsa_peer_allgather(const cvsa_peer_desc_t* pd, const float* src, int64_t n, float* out,
                        void* stream) {
  PeerView pv;
  int st = check_peer(pd, &pv);
  if (st) return st;
  if (n < 0 || n > pv.row_cap) return fail(CVSA_ERR_INVALID, "n outside [0, row_cap]");
  if (n == 0) return CVSA_OK;
  if (!src || !out) return fail(CVSA_ERR_INVALID, "NULL pointer");
  if (n > (int64_t)peer_max_ctas() * 256) return fail(CVSA_ERR_UNSUPPORTED, "row too long");
  return cuda_status(launch_peer_gather(pv, src, n, out, false, (cudaStream_t)stream),
                     "peer allgather launch");
}

int cvsa_peer_min_i32(const cvsa_peer_desc_t* pd, const int32_t* src, int64_t n, int32_t* out,
                      void* stream) {
  PeerView pv;
  int st = check_peer(pd, &pv);
  if (st) return st;
  if (n < 0 || n > pv.row_cap) return fail(CVSA_ERR_INVALID, "n outside [0, row_cap]");
  if (n == 0) return CVSA_OK;
  if (!src || !out) return fail(CVSA_ERR_INVALID, "NULL pointer");
  if (n > (int64_t)peer_max_ctas() * 256) return fail(CVSA_ERR_UNSUPPORTED, "row too long");
  return cuda_status(launch_peer_gather(pv, reinterpret_cast<const float*>(src), n,
                                        reinterpret_cast<float*>(out), true, (cudaStream_t)stream),
                     "peer min launch");
}

int cvsa_peer_merge(const cvsa_peer_desc_t* pd, const float* part, int32_t batch,
                    int32_t num_kv_heads, int32_t num_q_per_kv, int32_t head_dim,
                    const uint8_t* need, void* out, int32_t out_dtype, void* stream) {
  PeerView pv;
  int st = check_peer(pd, &pv);
  if (st) return st;
  if (batch < 0 || num_kv_heads <= 0 || num_q_per_kv <= 0 || head_dim <= 0)
    return fail(CVSA_ERR_INVALID, "bad shape");
  if (!valid_dtype(out_dtype)) return fail(CVSA_ERR_INVALID, "out dtype unknown");
  const int64_t rows = (int64_t)batch * num_kv_heads * num_q_per_kv;
  if (rows * (head_dim + 2) > pv.row_cap) return fail(CVSA_ERR_INVALID, "row_cap too small");
  if (rows == 0) return CVSA_OK;
  if (!part || !out) return fail(CVSA_ERR_INVALID, "NULL pointer");
  if (rows > peer_max_ctas()) return fail(CVSA_ERR_UNSUPPORTED, "too many query rows");
  if (head_dim > 256) return fail(CVSA_ERR_UNSUPPORTED, "head_dim above 256");
  return cuda_status(launch_peer_merge(pv, part, batch, num_kv_heads, num_q_per_kv, head_dim,
                                       need, out, out_dtype, (cudaStream_t)stream),
                     "peer merge launch");
}

int cvsa_recover_merge(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd,
                       const int32_t* page_indices, int32_t max_sel, const int32_t* n_per_head,
                       const uint8_t* accept, const float* o_d, const float* m_d, const float* l_d,
                       void* out, int32_t out_dtype, void* workspace, size_t workspace_bytes,
                       void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (max_sel <= 0) return fail(CVSA_ERR_INVALID, "max_sel must be positive");
  if (!attend_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "decode built for block_size 16, head_dim 64/128/256, G<=16");
  if (!valid_dtype(out_dtype)) return fail(CVSA_ERR_INVALID, "out dtype unknown");
  if (q.B == 0) return CVSA_OK;
  if (!page_indices || !n_per_head || !accept || !o_d || !m_d || !l_d || !out)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  const size_t need = decode_ws(q, kv, max_sel);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(CVSA_ERR_WORKSPACE, "workspace needs %zu bytes, 256-aligned", need);
  const DecodeLayout L = decode_layout(q, kv, max_sel);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(workspace) + L.bitmap);
  cudaStream_t s = (cudaStream_t)stream;
  st = cuda_status(launch_build_bitmap(page_indices, max_sel, n_per_head, q.B * kv.hkv, q.W, bitmap,
                                       bitmap_words(q.W), nullptr, s),
                   "bitmap launch");
  if (st) return st;
  AttendParams p;
  memset(&p, 0, sizeof(p));
  p.sel0 = page_indices;
  p.n0 = n_per_head;
  p.sel_stride = max_sel;
  p.src_select = 0;
  p.recover = true;
  p.accept = accept;
  p.bitmap = bitmap;
  p.bitmap_words = bitmap_words(q.W);
  p.external_draft = true;
  p.ext_o = o_d;
  p.ext_m = m_d;
  p.ext_l = l_d;
  p.out = out;
  p.out_dtype = out_dtype;
  p.partials = reinterpret_cast<uint8_t*>(workspace) + L.partials;
  p.partial_bytes = L.partial_bytes;
  p.head_done = ws_head_done(workspace);
  return cuda_status(launch_attend(q, kv, p, max_sel, s, false), "recover launch");
}

size_t cvsa_step_workspace_size(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd,
                                const cvsa_step_config_t* cfg, int32_t max_sel) {
  KvView kv;
  QView q;
  if (check_kv(kvd, &kv) || check_q(qd, kv, false, &q) || !cfg || max_sel <= 0) return 0;
  // size for the largest mode so one workspace serves every mode of a layer
  const int exp_stride = cfg->recovery == CVSA_RECOVERY_APPROX
                             ? cfg->approx_budget + cfg->sink_pages + cfg->local_pages : 0;
  StepLayout L = step_layout(q, kv, max_sel, true, false, exp_stride);
  StepLayout Ld = step_layout(q, kv, max_sel, false, true);
  return L.total > Ld.total ? L.total : Ld.total;
}

int cvsa_workspace_reset(void* workspace, size_t workspace_bytes, void* stream) {
  if (!workspace) return fail(CVSA_ERR_INVALID, "workspace is NULL");
  return cuda_status(cudaMemsetAsync(workspace, 0, workspace_bytes, (cudaStream_t)stream),
                     "workspace memset");
}

int cvsa_step_decision_word(void* workspace, int32_t** word) {
  if (!workspace || !word) return fail(CVSA_ERR_INVALID, "NULL pointer");
  *word = ws_select_sync(workspace) + 2;
  return CVSA_OK;
}

int cvsa_decode_step(const cvsa_query_desc_t* qd, const cvsa_kv_desc_t* kvd,
                     const cvsa_step_config_t* cfg, const cvsa_step_io_t* io, void* workspace,
                     size_t workspace_bytes, void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (!cfg || !io) return fail(CVSA_ERR_INVALID, "config/io is NULL");
  const int mode = cfg->mode;
  if (mode < CVSA_MODE_SCORE || mode > CVSA_MODE_DENSE)
    return fail(CVSA_ERR_INVALID, "unknown mode %d", mode);
  const int phase = io ? io->phase : CVSA_PHASE_ALL;
  if (phase < CVSA_PHASE_ALL || phase > CVSA_PHASE_ATTEND)
    return fail(CVSA_ERR_INVALID, "unknown phase %d", phase);
  if (phase != CVSA_PHASE_ALL && mode != CVSA_MODE_LAZY && mode != CVSA_MODE_SCORE)
    return fail(CVSA_ERR_INVALID, "phases split LAZY and SCORE steps only");
  if (cfg->recovery != CVSA_RECOVERY_EXACT && cfg->recovery != CVSA_RECOVERY_NONE &&
      cfg->recovery != CVSA_RECOVERY_APPROX)
    return fail(CVSA_ERR_INVALID, "unknown recovery %d", cfg->recovery);
  const bool approx = cfg->recovery == CVSA_RECOVERY_APPROX && mode != CVSA_MODE_DENSE;
  if (approx && cfg->approx_budget <= 0)
    return fail(CVSA_ERR_INVALID, "approx_budget must be > 0");
  if (cfg->budget < 0 || cfg->sink_pages < 0 || cfg->local_pages < 0)
    return fail(CVSA_ERR_INVALID, "budget/sink/local must be >= 0");
  if (!io->out) return fail(CVSA_ERR_INVALID, "out is NULL");
  const bool dense = mode == CVSA_MODE_DENSE;
  if (!dense) {
    if (!io->cached_indices || !io->cached_n) return fail(CVSA_ERR_INVALID, "cached selection is NULL");
    if (io->max_sel < cfg->budget + cfg->sink_pages + cfg->local_pages || io->max_sel <= 0)
      return fail(CVSA_ERR_INVALID, "max_sel=%d < budget+sink+local=%d", io->max_sel,
                  cfg->budget + cfg->sink_pages + cfg->local_pages);
  }
  if (!score_supported(q, kv) || !attend_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "built for block_size 16, head_dim 64/128/256, G<=16");
  if (q.W > kMaxPagesSelect)
    return fail(CVSA_ERR_UNSUPPORTED, "max_pages=%d above %d", q.W, kMaxPagesSelect);
  const int max_sel = dense ? 1 : io->max_sel;
  const size_t need = cvsa_step_workspace_size(qd, kvd, cfg, max_sel);
  if (!workspace || workspace_bytes < need || reinterpret_cast<uintptr_t>(workspace) % 256)
    return fail(CVSA_ERR_WORKSPACE, "workspace needs %zu bytes, 256-aligned", need);
  if (q.B == 0) return CVSA_OK;

  cudaStream_t s = (cudaStream_t)stream;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const bool recover = cfg->recovery == CVSA_RECOVERY_EXACT || approx;
  if (approx && !stream_attend_eligible(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "approximate recovery needs a bf16/f16 pool");
  const int exp_stride = approx ? cfg->approx_budget + cfg->sink_pages + cfg->local_pages : 0;
  StepLayout L = step_layout(q, kv, max_sel, true, dense, exp_stride);
  void* const* ev = io->timing_events;
  const bool pdl = ev == nullptr;
  auto rec = [&](int i) -> int {
    if (!ev || !ev[i]) return CVSA_OK;
    // External: under stream capture the record becomes an event node of the
    // graph (a plain record would only mark a dependency); outside capture it
    // is an ordinary record.
    return cuda_status(cudaEventRecordWithFlags((cudaEvent_t)ev[i], s, cudaEventRecordExternal),
                       "event record");
  };

  AttendParams ap;
  memset(&ap, 0, sizeof(ap));
  ap.out = io->out;
  ap.out_dtype = q.dtype;
  ap.counters = io->counters;
  ap.dev_err = io->dev_error;
  ap.partials = ws + L.attend;
  ap.partial_bytes = workspace_bytes - L.attend;
  ap.head_done = ws_head_done(workspace);

  if (dense || mode == CVSA_MODE_REUSE) {
    ap.dense = dense;
    ap.sel0 = io->cached_indices;
    ap.n0 = io->cached_n;
    ap.sel_stride = max_sel;
    ap.src_select = 0;
    // reuse and dense steps run no gate (backend.py:866-881): step_flags,
    // accept and coverage keep the values of the last gated step
    if ((st = rec(CVSA_EV_ATTEND_BEGIN))) return st;
    st = cuda_status(launch_attend(q, kv, ap, max_sel, s, pdl), "attend launch");
    if (st) return st;
    return rec(CVSA_EV_ATTEND_END);
  }

  // the two halves of a phased step share everything below; each launches its own
  const bool run_select = phase != CVSA_PHASE_ATTEND;
  const bool run_attend = phase != CVSA_PHASE_SELECT;
  float* scores = io->page_scores ? io->page_scores : reinterpret_cast<float*>(ws + L.scores);
  int32_t* sel_new = reinterpret_cast<int32_t*>(ws + L.sel);
  int32_t* n_new = reinterpret_cast<int32_t*>(ws + L.n);
  uint32_t* bitmap = reinterpret_cast<uint32_t*>(ws + L.bitmap);
  uint8_t* acc_new = ws + L.acc_new;
  float* cov_new = reinterpret_cast<float*>(ws + L.cov_new);
  uint8_t* acc_c = ws + L.acc_c;
  float* cov_c = reinterpret_cast<float*>(ws + L.cov_c);
  int32_t* sync = ws_select_sync(workspace);  // [0..1] select tickets, [2] decision

  if (run_select) {
    if ((st = rec(CVSA_EV_SCORE_BEGIN))) return st;
    st = cuda_status(launch_score_pages(q, kv, scores, io->dev_error, s, pdl), "score launch");
    if (st) return st;
    if ((st = rec(CVSA_EV_SCORE_END))) return st;
  }

  SelectParams sp;
  memset(&sp, 0, sizeof(sp));
  sp.scores = scores;
  sp.B = q.B;
  sp.hkv = kv.hkv;
  sp.W = q.W;
  sp.bs = kv.bs;
  sp.lens = q.lens;
  sp.budget = cfg->budget;
  sp.sink = cfg->sink_pages;
  sp.local = cfg->local_pages;
  sp.tau = cfg->tau;
  sp.sel_idx = sel_new;
  sp.sel_n = n_new;
  sp.max_sel = max_sel;
  sp.sel_bitmap = bitmap;
  sp.bitmap_words = bitmap_words(q.W);
  sp.accept = acc_new;
  sp.cov = cov_new;
  sp.cached_idx = io->cached_indices;
  sp.cached_n = io->cached_n;
  sp.cached_stride = max_sel;
  sp.cached_accept = acc_c;
  sp.cached_cov = cov_c;
  sp.sync_ctr = sync;
  sp.decision = sync + 2;
  sp.counters = io->counters;
  sp.mode = mode;
  sp.has_cache = cfg->has_cache;
  sp.lazy_stats = cfg->lazy_stats;
  sp.step_flags = io->step_flags;
  int32_t* comp_cnt = reinterpret_cast<int32_t*>(ws + L.comp_cnt);
  int32_t* comp_off = reinterpret_cast<int32_t*>(ws + L.comp_off);
  // the compact complement-item list only serves the general-layout kernel
  const bool comp_items = recover && !stream_attend_eligible(q, kv);
  if (comp_items) {
    sp.comp_cnt = comp_cnt;
    sp.comp_off = comp_off;
    sp.comp_chunk = attend_complement_chunk();
  }
  // a decision exchanged between the phases may turn a local reuse into a
  // rescore: keep the complement items either way
  sp.decision_external = phase != CVSA_PHASE_ALL;
  int32_t* exp_sel = reinterpret_cast<int32_t*>(ws + L.exp_sel);
  int32_t* exp_n = reinterpret_cast<int32_t*>(ws + L.exp_n);
  if (run_select) {
    if ((st = rec(CVSA_EV_SELECT_BEGIN))) return st;
    st = cuda_status(launch_select_gate(sp, s, pdl), "select launch");
    if (st) return st;
    if (approx) {
      // the expanded selection of backend.py:784-797 (same rule, larger budget)
      SelectParams xp;
      memset(&xp, 0, sizeof(xp));
      xp.scores = scores;
      xp.B = q.B;
      xp.hkv = kv.hkv;
      xp.W = q.W;
      xp.bs = kv.bs;
      xp.lens = q.lens;
      xp.budget = cfg->approx_budget;
      xp.sink = cfg->sink_pages;
      xp.local = cfg->local_pages;
      xp.sel_idx = exp_sel;
      xp.sel_n = exp_n;
      xp.max_sel = exp_stride;
      xp.mode = -1;
      st = cuda_status(launch_select_gate(xp, s, pdl), "expanded select launch");
      if (st) return st;
    }
    if ((st = rec(CVSA_EV_SELECT_END))) return st;
  }
  if (!run_attend) return CVSA_OK;

  ap.sel0 = io->cached_indices;
  ap.n0 = io->cached_n;
  ap.sel1 = sel_new;
  ap.n1 = n_new;
  ap.sel_stride = max_sel;
  ap.src_select = (mode == CVSA_MODE_LAZY) ? 2 : 1;
  ap.decision = sync + 2;
  ap.recover = recover;
  ap.approx = approx;
  ap.exp_idx = exp_sel;
  ap.exp_n = exp_n;
  ap.exp_stride = exp_stride;
  ap.comp_off = comp_items ? comp_off : nullptr;
  ap.accept = acc_new;
  ap.bitmap = bitmap;
  ap.bitmap_words = bitmap_words(q.W);
  ap.commit_src1 = true;
  ap.commit_idx = io->cached_indices;
  ap.commit_n = io->cached_n;
  ap.accept_out = io->accept;
  ap.cov_out = io->coverage;
  ap.acc0 = (mode == CVSA_MODE_LAZY) ? acc_c : nullptr;
  ap.cov0 = (mode == CVSA_MODE_LAZY) ? cov_c : nullptr;
  ap.acc1 = acc_new;
  ap.cov1 = cov_new;
  // the attend workspace must fit the recovery grid
  if (workspace_bytes - L.attend < attend_workspace_bytes(q, kv, max_sel, recover, false))
    return fail(CVSA_ERR_WORKSPACE, "workspace too small for recovery");
  if ((st = rec(CVSA_EV_ATTEND_BEGIN))) return st;
  st = cuda_status(launch_attend(q, kv, ap, max_sel, s, pdl), "attend launch");
  if (st) return st;
  return rec(CVSA_EV_ATTEND_END);
}

int cvsa_paged_append(const cvsa_kv_desc_t* kvd, const void* k_new, const void* v_new,
                      int32_t batch, const int32_t* seq_ids, int32_t* block_tables,
                      int32_t max_pages, int32_t* context_lens, int32_t* pages_allocated,
                      const int32_t* free_list, int32_t free_list_len, int32_t* free_head,
                      int32_t* dev_error, void* stream) {
  KvView kv;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  if (batch < 0 || max_pages <= 0 || free_list_len < 0) return fail(CVSA_ERR_INVALID, "bad shape");
  if (batch == 0) return CVSA_OK;
  if (!k_new || !v_new || !block_tables || !context_lens || !pages_allocated || !free_list ||
      !free_head)
    return fail(CVSA_ERR_INVALID, "NULL pointer");
  if ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new)) % 16)
    return fail(CVSA_ERR_INVALID, "k_new/v_new must be 16-byte aligned");
  return cuda_status(launch_paged_append(kv, k_new, v_new, batch, seq_ids, block_tables, max_pages,
                                         context_lens, pages_allocated, free_list, free_list_len,
                                         free_head, dev_error, (cudaStream_t)stream),
                     "append launch");
}

int cvsa_paged_gather(const cvsa_kv_desc_t* kvd, const int32_t* block_table_row, int32_t n_pages,
                      void* k_out, void* v_out, int32_t* dev_error, void* stream) {
  KvView kv;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  if (n_pages < 0) return fail(CVSA_ERR_INVALID, "n_pages < 0");
  if (n_pages == 0) return CVSA_OK;
  if (!block_table_row || !k_out) return fail(CVSA_ERR_INVALID, "NULL pointer");
  if ((reinterpret_cast<uintptr_t>(k_out) | reinterpret_cast<uintptr_t>(v_out)) % 16)
    return fail(CVSA_ERR_INVALID, "outputs must be 16-byte aligned");
  return cuda_status(launch_paged_gather(kv, block_table_row, n_pages, k_out, v_out, dev_error,
                                         (cudaStream_t)stream),
                     "gather launch");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free sparse decode.
//
// Some callers cannot allocate device memory at the point where they decode:
// an inference server whose memory pool is fully reserved up front, a plugin
// hosted by a runtime that owns every allocation, or a code path that must
// not call cudaMalloc because it would synchronise the device. For them,
// cvsa_sparse_decode_noalloc runs the same decode kernel as
// cvsa_sparse_decode but takes its scratch (item partials and the per-head
// tickets) from the array below, which is part of the library image: every
// GPU that loads the library holds CVSA_NOALLOC_SCRATCH_BYTES of it until the
// process exits.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_noalloc_scratch[CVSA_NOALLOC_SCRATCH_BYTES];

namespace {

// Identity of the calling thread's current CUDA context (the driver's context
// id, unique for the life of the process), or 0 if it cannot be read. The
// driver functions are looked up through the runtime, so the library needs no
// link against libcuda.
unsigned long long current_context_id() {
  using GetCurrent = CUresult (*)(CUcontext*);
  using GetId = CUresult (*)(CUcontext, unsigned long long*);
  static GetCurrent get_current = nullptr;
  static GetId get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<GetCurrent>(f);
    f = nullptr;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<GetId>(f);
  });
  CUcontext ctx = nullptr;
  unsigned long long id = 0;
  if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx ||
      get_id(ctx, &id) != CUDA_SUCCESS)
    return 0;
  return id;
}

// Device address of g_noalloc_scratch in the current context (the name is
// only a host-side stand-in for the symbol, not a device pointer). It is
// looked up once per device and context: after cudaDeviceReset, or when the
// primary context is destroyed and created again, the module is loaded anew
// and the array may sit at another address, so a new context id means a new
// lookup. Without a readable context id the lookup runs on every call.
void* noalloc_scratch_ptr(int* status) {
  static std::mutex mu;
  static void* ptrs[64] = {};
  static unsigned long long ctx_ids[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    *status = cuda_status(e, "cudaGetDevice");
    return nullptr;
  }
  if (dev < 0 || dev >= 64) {
    *status = fail(CVSA_ERR_UNSUPPORTED, "device ordinal %d above 63", dev);
    return nullptr;
  }
  // (0 before the runtime has made a context current on this thread: the
  // lookup below does, and the next call caches under the real id)
  const unsigned long long id = current_context_id();
  std::lock_guard<std::mutex> lock(mu);
  if (!ptrs[dev] || id == 0 || ctx_ids[dev] != id) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      *status = cuda_status(e == cudaSuccess ? cudaErrorInvalidSymbol : e,
                            "cudaGetSymbolAddress(no-alloc scratch)");
      return nullptr;
    }
    ptrs[dev] = p;
    ctx_ids[dev] = id;
  }
  *status = CVSA_OK;
  return ptrs[dev];
}

}  // namespace

extern "C" int cvsa_sparse_decode_noalloc(const cvsa_query_desc_t* qd,
                                          const cvsa_kv_desc_t* kvd,
                                          const int32_t* page_indices, int32_t max_sel,
                                          const int32_t* n_per_head, float* o_unnorm, float* m,
                                          float* l, void* out, int32_t out_dtype, void* stream) {
  KvView kv;
  QView q;
  int st = check_kv(kvd, &kv);
  if (st) return st;
  st = check_q(qd, kv, true, &q);
  if (st) return st;
  if (max_sel <= 0) return fail(CVSA_ERR_INVALID, "max_sel must be positive");
  if (!attend_supported(q, kv))
    return fail(CVSA_ERR_UNSUPPORTED, "decode built for block_size 16, head_dim 64/128/256, G<=16");
  if (out && !valid_dtype(out_dtype)) return fail(CVSA_ERR_INVALID, "out dtype unknown");
  if (!out && !o_unnorm && !m && !l) return fail(CVSA_ERR_INVALID, "no output requested");
  if (q.B == 0) return CVSA_OK;
  if (!page_indices || !n_per_head) return fail(CVSA_ERR_INVALID, "NULL selection");
  // scratch: [per-(b, h) tickets][item partials]
  const size_t heads = (size_t)q.B * kv.hkv;
  const size_t tickets = align256(heads * 4);
  const size_t need = tickets + attend_workspace_bytes(q, kv, max_sel, false, false);
  if (need > (size_t)CVSA_NOALLOC_SCRATCH_BYTES)
    return fail(CVSA_ERR_UNSUPPORTED,
                "decode needs %zu bytes of scratch; the no-alloc scratch holds %zu bytes "
                "(use cvsa_sparse_decode with a caller workspace)",
                need, (size_t)CVSA_NOALLOC_SCRATCH_BYTES);
  uint8_t* base = static_cast<uint8_t*>(noalloc_scratch_ptr(&st));
  if (!base) return st;
  cudaStream_t s = (cudaStream_t)stream;
  // The tickets must start at zero; a call that failed part-way could have left
  // them set, so clear them on the stream before every launch.
  st = cuda_status(cudaMemsetAsync(base, 0, heads * 4, s), "no-alloc scratch clear");
  if (st) return st;
  AttendParams p;
  memset(&p, 0, sizeof(p));
  p.sel0 = page_indices;
  p.n0 = n_per_head;
  p.sel_stride = max_sel;
  p.src_select = 0;
  p.out = out;
  p.out_dtype = out_dtype;
  p.o_unnorm = o_unnorm;
  p.m_out = m;
  p.l_out = l;
  p.head_done = reinterpret_cast<int32_t*>(base);
  p.partials = base + tickets;
  p.partial_bytes = (size_t)CVSA_NOALLOC_SCRATCH_BYTES - tickets;
  return cuda_status(launch_attend(q, kv, p, max_sel, s, false), "no-alloc decode launch");
}
