// Sparse paged decode, fused exact recovery and LSE merge.
//
// Restates, as one split-K kernel:
//   * the decode kernels of cvsa/kernels/sparse_decode.py (:424-500 unnorm,
//     :136-234 tiled, :577-606 tile reduce, :15-132 normalised): online
//     softmax over a page list with s = (q . k) * D^-0.5, producing
//     (o_unnorm, m, l) and o / max(l, 1e-6);
//   * cvsa/backend.py:819-842 exact recovery: for a rejected head, attention
//     over the valid pages NOT selected (cvsa/kernels/coverage.py:31-96 builds
//     that list; here selected pages are skipped through a bitmap), merged
//     with the draft by cvsa/kernels/coverage.py:274-326.
//
// Work decomposition. For every (b, kv head) there are `nd` draft items
// (chunks of the selection list) and `nc` complement items (chunks of the
// logical page range, minus selected pages) -- or, for dense layers, `nc`
// chunks of all valid pages. One CTA of 4 warps runs one item; inactive items
// (accepted heads' complement chunks, chunks past the end) exit at once. The
// 4 warps take the item's pages round robin; each warp streams its pages
// through its own 3-stage shared-memory ring filled by TMA (one box per
// 64-wide slice of head_dim for K and for V, 128-byte swizzle) and keeps its
// own online-softmax state. All G query heads of the KV head are packed into
// the M dimension of mma.sync m16n8k16 (bf16/f16 in, f32 accumulate):
// S = Q K^T (M = query heads, N = 16 tokens, K = head_dim) and O += P V
// (K = 16 tokens, N = head_dim); P goes from the S accumulators to the A
// operand in registers. The warps' states are merged in shared memory into an
// item partial (o, m, l) per query head; the last CTA of (b, h) to finish
// (atomic ticket, no spin) merges the item partials in a fixed order, so the
// result is deterministic, and writes the output. fp32 (and mixed-dtype)
// KV use a CUDA-core variant of the per-page step with the same framework.
#include <mutex>
#include <unordered_map>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kNW = 4;             // warps per CTA
constexpr int kStages = 3;         // per-warp TMA ring depth
constexpr int kMaxItemPages = 32;  // pages per item (list capacity)
constexpr int kBS = 16;            // tokens per page (kernels built for 16)

struct ItemCfg {
  int cd, nd;  // draft chunk pages, draft items per head
  int cc, nc;  // complement/dense chunk pages, items per head
  int iph;     // nd + nc
};

struct AttendArgs {
  CUtensorMap kmap;  // 64-byte aligned (type alignment)
  CUtensorMap vmap;
  const void* q;
  const void* k;
  const void* v;
  int64_t sb, st, sh;
  int B, hq, hkv, G, W, num_blocks;
  const int32_t* tables;
  const int32_t* lens;
  const int32_t* sel0;
  const int32_t* n0;
  const int32_t* sel1;
  const int32_t* n1;
  int sel_stride;
  int src_select;
  const int32_t* decision;
  int dense, recover;
  const uint8_t* accept;
  const uint32_t* bitmap;
  int bitmap_words;
  int external_draft;
  const float* ext_o;
  const float* ext_m;
  const float* ext_l;
  int commit;
  int32_t* commit_idx;
  int32_t* commit_n;
  void* out;
  int out_dtype;
  float* o_unnorm;
  float* m_out;
  float* l_out;
  int64_t* counters;
  int32_t* dev_err;
  uint8_t* accept_out;
  float* cov_out;
  const uint8_t* acc0;
  const float* cov0;
  const uint8_t* acc1;
  const float* cov1;
  float* part_o;   // [grid][G][D]
  float* part_ml;  // [grid][G][2]
  int32_t* head_done;
  ItemCfg ic;
  float scale;
};

// ---------------------------------------------------------------------------
// per-item bookkeeping shared by both per-page variants
// ---------------------------------------------------------------------------
struct ItemInfo {
  int bh, b, h, j;
  int ctx, nv;
  int src;  // 0/1 selection source, -1 dense
  int n_sel;
  const int32_t* sel;
  bool rec;
  int nd_act, nc_act, expected;
  int role;  // 0 draft/dense, 1 complement
  bool active;
};

__device__ __forceinline__ ItemInfo item_info(const AttendArgs& a) {
  ItemInfo it;
  const int item = blockIdx.x;
  it.bh = item / a.ic.iph;
  it.j = item % a.ic.iph;
  it.b = it.bh / a.hkv;
  it.h = it.bh % a.hkv;
  it.ctx = a.lens[it.b];
  it.nv = min(n_valid_pages(it.ctx, kBS), a.W);
  if (a.dense) {
    it.src = -1;
    it.n_sel = 0;
    it.sel = nullptr;
  } else {
    int s = a.src_select;
    if (s == 2) s = (a.decision[0] & 1) ? 0 : 1;
    it.src = s;
    it.sel = (s ? a.sel1 : a.sel0) + (int64_t)it.bh * a.sel_stride;
    it.n_sel = min(max((s ? a.n1 : a.n0)[it.bh], 0), a.sel_stride);
  }
  it.rec = a.recover && !a.dense && (a.external_draft || it.src == 1) && a.accept[it.bh] == 0;
  const int nvc = (it.nv + a.ic.cc - 1) / a.ic.cc;
  if (a.dense) {
    it.nd_act = 0;
    it.nc_act = max(1, nvc);
  } else if (a.external_draft) {
    it.nd_act = 0;
    it.nc_act = it.rec ? max(1, nvc) : 1;
  } else {
    it.nd_act = max(1, (it.n_sel + a.ic.cd - 1) / a.ic.cd);
    it.nc_act = it.rec ? max(1, nvc) : 0;
  }
  it.expected = it.nd_act + it.nc_act;
  if (it.j < a.ic.nd) {
    it.role = 0;
    it.active = it.j < it.nd_act;
  } else {
    it.role = a.dense ? 0 : 1;
    it.active = (it.j - a.ic.nd) < it.nc_act;
  }
  return it;
}

// Build this item's page list (ascending within the item) in shared memory.
__device__ __forceinline__ void build_page_list(const AttendArgs& a, const ItemInfo& it,
                                                int* list, int* cnt) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  int pg = -1;
  bool keep = false;
  if (it.j < a.ic.nd) {
    const int i0 = it.j * a.ic.cd;
    const int i = i0 + lane;
    if (lane < a.ic.cd && i < it.n_sel) {
      pg = it.sel[i];
      keep = pg >= 0 && pg < a.W;
      if (!keep) set_dev_error(a.dev_err, CVSA_DEV_ERR_PAGE_RANGE);
    }
  } else {
    const int c = it.j - a.ic.nd;
    const bool empty = a.external_draft && !it.rec;
    const int p = c * a.ic.cc + lane;
    if (!empty && lane < a.ic.cc && p < it.nv) {
      pg = p;
      keep = true;
      if (!a.dense) {
        const uint32_t word = a.bitmap[(int64_t)it.bh * a.bitmap_words + (p >> 5)];
        keep = ((word >> (p & 31)) & 1u) == 0;
      }
    }
  }
  const uint32_t m = __ballot_sync(0xffffffffu, keep);
  if (keep) list[__popc(m & ((1u << lane) - 1u))] = pg;
  if (lane == 0) *cnt = __popc(m);
}

// merge (m, l, o) partials: x = running, y = new; returns merged in x.
__device__ __forceinline__ void lse_combine(float& m, float& l, float& o, float m2, float l2,
                                            float o2) {
  if (m2 == neg_inf()) return;
  if (m == neg_inf()) {
    m = m2;
    l = l2;
    o = o2;
    return;
  }
  const float mx = fmaxf(m, m2);
  const float a1 = expf(m - mx), a2 = expf(m2 - mx);
  l = l * a1 + l2 * a2;
  o = o * a1 + o2 * a2;
  m = mx;
}

template <typename TO>
__device__ __forceinline__ void store_out(void* out, int64_t idx, float v) {
  reinterpret_cast<TO*>(out)[idx] = Elem<TO>::from_f(v);
}

__device__ __forceinline__ void store_out_dt(void* out, int dt, int64_t idx, float v) {
  if (dt == CVSA_DTYPE_BF16) store_out<__nv_bfloat16>(out, idx, v);
  else if (dt == CVSA_DTYPE_F16) store_out<__half>(out, idx, v);
  else store_out<float>(out, idx, v);
}

// Final merge for one (b, h): combine role-0 partials into the draft
// (o_d, m_d, l_d), role-1 partials into the complement, then write outputs.
// `ip_*` is this CTA's own item partial (used when it is the only item).
template <int D>
__device__ void finalize_head(const AttendArgs& a, const ItemInfo& it, const float* ip_o,
                              const float* ip_ml, bool single) {
  const int G = a.G;
  const int64_t item_base = (int64_t)it.bh * a.ic.iph;
  for (int e = threadIdx.x; e < G * D; e += kNW * 32) {
    const int g = e / D, d = e % D;
    float md = neg_inf(), ld = 0.f, od = 0.f;
    float mc = neg_inf(), lc = 0.f, oc = 0.f;
    if (single) {
      const float pm = ip_ml[g * 2], pl = ip_ml[g * 2 + 1], po = ip_o[g * D + d];
      if (it.role == 0) { md = pm; ld = pl; od = po; }
      else { mc = pm; lc = pl; oc = po; }
    } else {
      // role 0 items
      if (!a.external_draft) {
        const int n0 = a.dense ? it.nc_act : it.nd_act;
        const int off0 = a.dense ? a.ic.nd : 0;
        for (int i = 0; i < n0; ++i) {
          const int64_t itm = item_base + off0 + i;
          lse_combine(md, ld, od, a.part_ml[(itm * G + g) * 2], a.part_ml[(itm * G + g) * 2 + 1],
                      a.part_o[(itm * G + g) * D + d]);
        }
      }
      if (it.rec) {
        for (int i = 0; i < it.nc_act; ++i) {
          const int64_t itm = item_base + a.ic.nd + i;
          lse_combine(mc, lc, oc, a.part_ml[(itm * G + g) * 2], a.part_ml[(itm * G + g) * 2 + 1],
                      a.part_o[(itm * G + g) * D + d]);
        }
      }
    }
    const int64_t qrow = (int64_t)it.b * a.hq + (int64_t)it.h * G + g;
    if (a.external_draft) {
      md = a.ext_m[qrow];
      ld = a.ext_l[qrow];
      od = a.ext_o[qrow * D + d];
    }
    if (a.o_unnorm) a.o_unnorm[qrow * D + d] = od;
    if (d == 0) {
      if (a.m_out) a.m_out[qrow] = md;
      if (a.l_out) a.l_out[qrow] = ld;
    }
    if (a.out) {
      float r;
      if (it.rec) {
        // coverage.py:318-326 (rejected: merge, then divide by max(l, 1e-6))
        const float m_all = fmaxf(md, mc);
        const float sd = (md == neg_inf()) ? 0.f : expf(md - m_all);
        const float sc = (mc == neg_inf()) ? 0.f : expf(mc - m_all);
        const float lm = ld * sd + lc * sc;
        r = (od * sd + oc * sc) / fmaxf(lm, 1e-6f);
      } else {
        r = od / fmaxf(ld, 1e-6f);
      }
      store_out_dt(a.out, a.out_dtype, qrow * D + d, r);
    }
  }
  if (threadIdx.x == 0) {
    if (a.commit && it.src == 1) a.commit_n[it.bh] = it.n_sel;
    if (a.accept_out && !a.dense) {
      const uint8_t* ga = it.src == 1 ? a.acc1 : a.acc0;
      const float* gc = it.src == 1 ? a.cov1 : a.cov0;
      a.accept_out[it.bh] = ga ? ga[it.bh] : 1;
      if (a.cov_out) a.cov_out[it.bh] = gc ? gc[it.bh] : 1.f;
    }
    if (a.counters) {
      long long att = a.dense ? it.nv : it.n_sel;
      if (it.rec) att += max(it.nv - it.n_sel, 0);
      atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[CVSA_CTR_PAGES_ATTENDED]),
                (unsigned long long)att);
      atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[CVSA_CTR_PAGES_MAX]),
                (unsigned long long)it.nv);
    }
  }
  if (a.commit && it.src == 1) {
    for (int i = threadIdx.x; i < it.n_sel; i += kNW * 32)
      a.commit_idx[(int64_t)it.bh * a.sel_stride + i] = it.sel[i];
  }
}

// Merge the kNW warp states (wb_o [kNW][GP][D], wb_ml [kNW][GP][2]) into the
// item partial ip_o [G][D], ip_ml [G][2].
template <int D>
__device__ void merge_warps(int G, int GP, const float* wb_o, const float* wb_ml, float* ip_o,
                            float* ip_ml) {
  for (int e = threadIdx.x; e < G * D; e += kNW * 32) {
    const int g = e / D, d = e % D;
    float m = neg_inf(), l = 0.f, o = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w)
      lse_combine(m, l, o, wb_ml[(w * GP + g) * 2], wb_ml[(w * GP + g) * 2 + 1],
                  wb_o[(w * GP + g) * D + d]);
    ip_o[g * D + d] = o;
    if (d == 0) {
      ip_ml[g * 2] = m;
      ip_ml[g * 2 + 1] = l;
    }
  }
}

// ---------------------------------------------------------------------------
// tensor-core per-page step (bf16 / f16, q dtype == kv dtype)
// ---------------------------------------------------------------------------
template <typename T, int D, int GR>
struct MmaPath {
  static constexpr int kSub = D / 64;                 // 64-wide head_dim slices
  static constexpr int kTileBytes = kBS * 128;        // one swizzled slice
  static constexpr int kStageBytes = 2 * kSub * kTileBytes;  // K + V
  static constexpr int kGP = 8 * GR;                  // query rows per warp state
  static constexpr int kNT = D / 8;                   // n-tiles of O

  static constexpr size_t smem_bytes() {
    // stage ring (reused afterwards for the warp-state merge) + item partial
    // + barriers + page list + 1 KB alignment slack
    size_t ring = (size_t)kNW * kStages * kStageBytes;
    size_t wb = (size_t)kNW * kGP * D * 4 + (size_t)kNW * kGP * 2 * 4;
    size_t r = ring > wb ? ring : wb;
    return 1024 + r + (size_t)16 * D * 4 + 16 * 2 * 4 + kNW * kStages * 8 + (kMaxItemPages + 4) * 4;
  }

  __device__ static void run(const AttendArgs& a, const ItemInfo& it, uint8_t* ring, uint64_t* bars,
                             const int* list, int cnt, float* wb_o, float* wb_ml) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int gq = lane >> 2, tq = lane & 3;
    const int G = a.G;

    // Q as the A operand: rows g (and g+8 for GR == 2), 16 head_dim per k-step
    uint32_t qa[D / 16][2 * GR];
    {
      const T* qb = reinterpret_cast<const T*>(a.q) + ((int64_t)it.b * a.hq + (int64_t)it.h * G) * D;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
        for (int r = 0; r < GR; ++r) {
          const int g = gq + 8 * r;
          uint32_t lo = 0, hi = 0;
          if (g < G) {
            lo = *reinterpret_cast<const uint32_t*>(qb + (int64_t)g * D + ks * 16 + tq * 2);
            hi = *reinterpret_cast<const uint32_t*>(qb + (int64_t)g * D + ks * 16 + 8 + tq * 2);
          }
          qa[ks][r] = lo;       // a0 (row g) / a1 (row g+8)
          qa[ks][GR + r] = hi;  // a2 / a3
        }
      }
    }

    float o[kNT][2 * GR];
    float dummy[2] = {0.f, 0.f};
#pragma unroll
    for (int n = 0; n < kNT; ++n)
#pragma unroll
      for (int r = 0; r < 2 * GR; ++r) o[n][r] = 0.f;
    float m_run[GR], l_run[GR];
#pragma unroll
    for (int r = 0; r < GR; ++r) {
      m_run[r] = neg_inf();
      l_run[r] = 0.f;
    }

    const int nmine = cnt > w ? (cnt - w + kNW - 1) / kNW : 0;
    uint8_t* my_ring = ring + (size_t)w * kStages * kStageBytes;
    uint64_t* my_bar = bars + w * kStages;
    const int32_t* trow = a.tables + (int64_t)it.b * a.W;

    auto page_blk = [&](int jj) {
      const int pg = list[w + jj * kNW];
      const int blk = trow[pg];
      return (blk >= 0 && blk < a.num_blocks) ? blk : -1;
    };
    auto issue = [&](int jj) {
      if (lane == 0) {
        const int st = jj % kStages;
        const int blk = page_blk(jj);
        uint8_t* dst = my_ring + (size_t)st * kStageBytes;
        if (blk >= 0) {
          mbar_arrive_expect_tx(&my_bar[st], kStageBytes);
#pragma unroll
          for (int s = 0; s < kSub; ++s) {
            tma_load_4d(dst + s * kTileBytes, &a.kmap, &my_bar[st], s * 64, it.h, 0, blk);
            tma_load_4d(dst + (kSub + s) * kTileBytes, &a.vmap, &my_bar[st], s * 64, it.h, 0, blk);
          }
        } else {
          set_dev_error(a.dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
          mbar_arrive_expect_tx(&my_bar[st], 0);
        }
      }
    };

    const int npro = nmine < kStages ? nmine : kStages;
    for (int jj = 0; jj < npro; ++jj) issue(jj);

    bool failed = false;
    for (int jj = 0; jj < nmine; ++jj) {
      const int st = jj % kStages;
      const uint32_t ph = (jj / kStages) & 1;
      if (!mbar_wait_bounded(&my_bar[st], ph)) {
        failed = true;
        set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
        // drain the copies still in flight for this warp (bounded), then stop
        for (int k2 = jj + 1; k2 < nmine && k2 < jj + kStages; ++k2)
          mbar_wait_bounded(&my_bar[k2 % kStages], (k2 / kStages) & 1);
        break;
      }
      const int pg = list[w + jj * kNW];
      const bool ok = page_blk(jj) >= 0;
      const int ntok = ok ? min(kBS, it.ctx - pg * kBS) : 0;
      if (ntok > 0) {
        const uint32_t kbase = smem_u32(my_ring + (size_t)st * kStageBytes);
        const uint32_t vbase = kbase + kSub * kTileBytes;
        // ---- S = Q K^T over the 16 tokens of the page ----
        float s[2][4];
#pragma unroll
        for (int n = 0; n < 2; ++n)
#pragma unroll
          for (int r = 0; r < 4; ++r) s[n][r] = 0.f;
        {
          const int tok = (lane & 7) + ((lane >> 4) & 1) * 8;
          const int chsel = (lane >> 3) & 1;
#pragma unroll
          for (int ks = 0; ks < D / 16; ++ks) {
            const int sub = ks >> 2;
            const int ch = (ks & 3) * 2 + chsel;
            const uint32_t addr = kbase + sub * kTileBytes + tok * 128 + ((ch ^ (tok & 7)) << 4);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4(b0, b1, b2, b3, addr);
            uint32_t afr[4];
            afr[0] = qa[ks][0];
            afr[1] = GR == 2 ? qa[ks][1] : 0u;
            afr[2] = qa[ks][GR];
            afr[3] = GR == 2 ? qa[ks][GR + 1] : 0u;
            Mma<T>::m16n8k16(s[0], afr, b0, b1);
            Mma<T>::m16n8k16(s[1], afr, b2, b3);
          }
        }
        // ---- online softmax per query row ----
        float pv[2][4];
#pragma unroll
        for (int r = 0; r < GR; ++r) {
          float x[4];
          bool vld[4];
#pragma unroll
          for (int n = 0; n < 2; ++n)
#pragma unroll
            for (int i = 0; i < 2; ++i) {
              const int tok = n * 8 + tq * 2 + i;
              vld[n * 2 + i] = tok < ntok;
              x[n * 2 + i] = vld[n * 2 + i] ? s[n][2 * r + i] * a.scale : neg_inf();
            }
          float pm = fmaxf(fmaxf(x[0], x[1]), fmaxf(x[2], x[3]));
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 1));
          pm = fmaxf(pm, __shfl_xor_sync(0xffffffffu, pm, 2));
          const float mnew = fmaxf(m_run[r], pm);
          float alpha = 1.f;
          float p[4];
          if (mnew == neg_inf()) {
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = 0.f;
          } else {
            alpha = (m_run[r] == neg_inf()) ? 0.f : softmax_exp(m_run[r] - mnew);
#pragma unroll
            for (int i = 0; i < 4; ++i) p[i] = vld[i] ? softmax_exp(x[i] - mnew) : 0.f;
          }
          float rs = (p[0] + p[1]) + (p[2] + p[3]);
          rs += __shfl_xor_sync(0xffffffffu, rs, 1);
          rs += __shfl_xor_sync(0xffffffffu, rs, 2);
          l_run[r] = l_run[r] * alpha + rs;
          m_run[r] = mnew;
#pragma unroll
          for (int n = 0; n < kNT; ++n) {
            o[n][2 * r] *= alpha;
            o[n][2 * r + 1] *= alpha;
          }
          pv[0][2 * r] = p[0];
          pv[0][2 * r + 1] = p[1];
          pv[1][2 * r] = p[2];
          pv[1][2 * r + 1] = p[3];
        }
        uint32_t pa[4];
        pa[0] = Mma<T>::pack(pv[0][0], pv[0][1]);
        pa[1] = GR == 2 ? Mma<T>::pack(pv[0][2], pv[0][3]) : 0u;
        pa[2] = Mma<T>::pack(pv[1][0], pv[1][1]);
        pa[3] = GR == 2 ? Mma<T>::pack(pv[1][2], pv[1][3]) : 0u;
        // ---- O += P V ----
        {
          const int tok = (lane & 7) + ((lane >> 3) & 1) * 8;
          const int chsel = lane >> 4;
#pragma unroll
          for (int jp = 0; jp < D / 16; ++jp) {
            const int nt = jp * 2;
            const int sub = nt >> 3;
            const int ch = (nt & 7) + chsel;
            const uint32_t addr = vbase + sub * kTileBytes + tok * 128 + ((ch ^ (tok & 7)) << 4);
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(b0, b1, b2, b3, addr);
            if constexpr (GR == 2) {
              Mma<T>::m16n8k16(o[nt], pa, b0, b1);
              Mma<T>::m16n8k16(o[nt + 1], pa, b2, b3);
            } else {
              float c0[4] = {o[nt][0], o[nt][1], dummy[0], dummy[1]};
              Mma<T>::m16n8k16(c0, pa, b0, b1);
              o[nt][0] = c0[0];
              o[nt][1] = c0[1];
              float c1[4] = {o[nt + 1][0], o[nt + 1][1], dummy[0], dummy[1]};
              Mma<T>::m16n8k16(c1, pa, b2, b3);
              o[nt + 1][0] = c1[0];
              o[nt + 1][1] = c1[1];
            }
          }
        }
      }
      __syncwarp();
      if (jj + kStages < nmine) {
        fence_proxy_async_smem();
        issue(jj + kStages);
      }
    }
    if (failed) {
#pragma unroll
      for (int r = 0; r < GR; ++r) {
        m_run[r] = neg_inf();
        l_run[r] = 0.f;
      }
    }
    // The ring is reused as the warp-state buffer: wait for every warp.
    __syncthreads();
#pragma unroll
    for (int r = 0; r < GR; ++r) {
      const int g = gq + 8 * r;
#pragma unroll
      for (int n = 0; n < kNT; ++n) {
        wb_o[(w * kGP + g) * D + n * 8 + tq * 2] = failed ? 0.f : o[n][2 * r];
        wb_o[(w * kGP + g) * D + n * 8 + tq * 2 + 1] = failed ? 0.f : o[n][2 * r + 1];
      }
      if (tq == 0) {
        wb_ml[(w * kGP + g) * 2] = m_run[r];
        wb_ml[(w * kGP + g) * 2 + 1] = l_run[r];
      }
    }
  }
};

// ---------------------------------------------------------------------------
// CUDA-core per-page step (fp32 or mixed dtypes); lane owns head_dim columns
// d = lane + 32 i. Up to GM query heads per KV head.
// ---------------------------------------------------------------------------
template <typename T, typename TQ, int D, int GM>
struct SimtPath {
  static constexpr int kGP = GM;
  static constexpr int kPer = D / 32;
  static constexpr size_t smem_bytes() {
    size_t wb = (size_t)kNW * GM * D * 4 + (size_t)kNW * GM * 2 * 4;
    return 1024 + wb + (size_t)16 * D * 4 + 16 * 2 * 4 + kNW * kStages * 8 + (kMaxItemPages + 4) * 4;
  }
  __device__ static void run(const AttendArgs& a, const ItemInfo& it, uint8_t*, uint64_t*,
                             const int* list, int cnt, float* wb_o, float* wb_ml) {
    const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.G;
    float qv[GM][kPer];
    const TQ* qb = reinterpret_cast<const TQ*>(a.q) + ((int64_t)it.b * a.hq + (int64_t)it.h * G) * D;
#pragma unroll
    for (int g = 0; g < GM; ++g)
#pragma unroll
      for (int i = 0; i < kPer; ++i)
        qv[g][i] = g < G ? Elem<TQ>::to_f(qb[(int64_t)g * D + lane + 32 * i]) : 0.f;
    float o[GM][kPer];
    float m_run[GM], l_run[GM];
#pragma unroll
    for (int g = 0; g < GM; ++g) {
      m_run[g] = neg_inf();
      l_run[g] = 0.f;
#pragma unroll
      for (int i = 0; i < kPer; ++i) o[g][i] = 0.f;
    }
    const T* K = reinterpret_cast<const T*>(a.k);
    const T* V = reinterpret_cast<const T*>(a.v);
    const int32_t* trow = a.tables + (int64_t)it.b * a.W;
    for (int jj = w; jj < cnt; jj += kNW) {
      const int pg = list[jj];
      const int blk = trow[pg];
      if (blk < 0 || blk >= a.num_blocks) {
        if (lane == 0) set_dev_error(a.dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
        continue;
      }
      const int ntok = min(kBS, it.ctx - pg * kBS);
      for (int t = 0; t < ntok; ++t) {
        const int64_t base = (int64_t)blk * a.sb + (int64_t)t * a.st + (int64_t)it.h * a.sh;
        float kv[kPer], vv[kPer];
#pragma unroll
        for (int i = 0; i < kPer; ++i) {
          kv[i] = Elem<T>::to_f(K[base + lane + 32 * i]);
          vv[i] = Elem<T>::to_f(V[base + lane + 32 * i]);
        }
#pragma unroll
        for (int g = 0; g < GM; ++g) {
          if (g < G) {
            float dot = 0.f;
#pragma unroll
            for (int i = 0; i < kPer; ++i) dot = fmaf(qv[g][i], kv[i], dot);
            dot = warp_sum(dot);
            const float sc = dot * a.scale;
            const float mnew = fmaxf(m_run[g], sc);
            const float alpha = (m_run[g] == neg_inf()) ? 0.f : expf(m_run[g] - mnew);
            const float p = expf(sc - mnew);
            l_run[g] = l_run[g] * alpha + p;
#pragma unroll
            for (int i = 0; i < kPer; ++i) o[g][i] = o[g][i] * alpha + p * vv[i];
            m_run[g] = mnew;
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < GM; ++g) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) wb_o[(w * GM + g) * D + lane + 32 * i] = o[g][i];
      if (lane == 0) {
        wb_ml[(w * GM + g) * 2] = m_run[g];
        wb_ml[(w * GM + g) * 2 + 1] = l_run[g];
      }
    }
  }
};

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <class Path, int D>
__global__ void __launch_bounds__(kNW * 32)
attend_kernel(const __grid_constant__ AttendArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base_u32 & 1023)) & 1023);

  constexpr size_t kRing = Path::smem_bytes() - 1024 - (size_t)16 * D * 4 - 16 * 2 * 4 -
                           kNW * kStages * 8 - (kMaxItemPages + 4) * 4;
  uint8_t* ring = smem;
  float* wb_o = reinterpret_cast<float*>(smem);
  float* wb_ml = wb_o + (size_t)kNW * Path::kGP * D;
  float* ip_o = reinterpret_cast<float*>(smem + kRing);
  float* ip_ml = ip_o + 16 * D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ip_ml + 16 * 2);
  int* list = reinterpret_cast<int*>(bars + kNW * kStages);
  int* cnt = list + kMaxItemPages;
  int* flag_last = cnt + 1;

  pdl_wait();

  const ItemInfo it = item_info(a);
  if (!it.active) return;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNW * kStages; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
  }
  build_page_list(a, it, list, cnt);
  __syncthreads();
  const int n = *cnt;

  Path::run(a, it, ring, bars, list, n, wb_o, wb_ml);
  __syncthreads();
  merge_warps<D>(a.G, Path::kGP, wb_o, wb_ml, ip_o, ip_ml);
  __syncthreads();

  if (it.expected == 1) {
    finalize_head<D>(a, it, ip_o, ip_ml, true);
    return;
  }
  // publish this item's partial, then take a ticket for (b, h)
  const int64_t item = blockIdx.x;
  for (int e = threadIdx.x; e < a.G * D; e += kNW * 32) a.part_o[item * a.G * D + e] = ip_o[e];
  for (int e = threadIdx.x; e < a.G * 2; e += kNW * 32) a.part_ml[item * a.G * 2 + e] = ip_ml[e];
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(&a.head_done[it.bh], 1);
    *flag_last = (prev == it.expected - 1) ? 1 : 0;
  }
  __syncthreads();
  if (*flag_last) {
    __threadfence();
    finalize_head<D>(a, it, ip_o, ip_ml, false);
    if (threadIdx.x == 0) a.head_done[it.bh] = 0;
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// K or V pool as a 4-D tensor {D, Hkv, BS, NB}, box {64, 1, BS, 1}, 128 B swizzle.
bool make_pool_map(CUtensorMap* map, const void* base, const KvView& kv) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return false;
  const int eb = dtype_bytes(kv.dtype);
  cuuint64_t dims[4] = {(cuuint64_t)kv.d, (cuuint64_t)kv.hkv, (cuuint64_t)kv.bs,
                        (cuuint64_t)kv.num_blocks};
  cuuint64_t strides[3] = {(cuuint64_t)kv.sh * eb, (cuuint64_t)kv.st * eb, (cuuint64_t)kv.sb * eb};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)kv.bs, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMapDataType dt = kv.dtype == CVSA_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                       : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = enc(map, dt, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct MapKey {
  const void* p;
  int dtype, d, hkv, bs, nb;
  int64_t sb, st, sh;
  bool operator==(const MapKey& o) const {
    return p == o.p && dtype == o.dtype && d == o.d && hkv == o.hkv && bs == o.bs && nb == o.nb &&
           sb == o.sb && st == o.st && sh == o.sh;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<const void*>()(k.p) ^ (size_t)k.nb * 1315423911u ^ (size_t)k.sb;
  }
};

bool cached_pool_map(CUtensorMap* out, const void* base, const KvView& kv) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  MapKey key{base, kv.dtype, kv.d, kv.hkv, kv.bs, kv.num_blocks, kv.sb, kv.st, kv.sh};
  std::lock_guard<std::mutex> lock(mu);
  auto itr = cache.find(key);
  if (itr != cache.end()) {
    *out = itr->second;
    return true;
  }
  if (!make_pool_map(out, base, kv)) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, *out);
  return true;
}

ItemCfg item_cfg(const QView& q, const KvView& kv, int max_sel, bool recover, bool dense) {
  ItemCfg c;
  const int heads = q.B * kv.hkv;
  const int target = 8 * num_sms();  // aim for several waves of resident CTAs
  if (dense) {
    c.cd = 8;
    c.nd = 0;
  } else {
    int per_head = (target + heads - 1) / heads;
    int cd = (max_sel + per_head - 1) / max(per_head, 1);
    cd = ((cd + kNW - 1) / kNW) * kNW;
    c.cd = cd < 8 ? 8 : (cd > kMaxItemPages ? kMaxItemPages : cd);
    c.nd = (max_sel + c.cd - 1) / c.cd;
    if (c.nd < 1) c.nd = 1;
  }
  if (recover || dense) {
    c.cc = kMaxItemPages;
    c.nc = (q.W + c.cc - 1) / c.cc;
    if (c.nc < 1) c.nc = 1;
  } else {
    c.cc = kMaxItemPages;
    c.nc = 0;
  }
  c.iph = c.nd + c.nc;
  return c;
}

bool use_mma(const QView& q, const KvView& kv) {
  return (kv.dtype == CVSA_DTYPE_BF16 || kv.dtype == CVSA_DTYPE_F16) && q.dtype == kv.dtype &&
         (kv.d == 64 || kv.d == 128 || kv.d == 256) && (q.hq / kv.hkv) <= 16 &&
         ((kv.sh * 2) % 16 == 0) && ((kv.st * 2) % 16 == 0) && ((kv.sb * 2) % 16 == 0) &&
         (reinterpret_cast<uintptr_t>(kv.k) % 16 == 0) && (reinterpret_cast<uintptr_t>(kv.v) % 16 == 0);
}

template <class Path, int D>
cudaError_t launch_path(const AttendArgs& a, int grid, cudaStream_t s, bool pdl) {
  constexpr size_t smem = Path::smem_bytes();
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attend_kernel<Path, D>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  return launch_k(attend_kernel<Path, D>, dim3(grid), dim3(kNW * 32), smem, s, pdl, a);
}

template <typename T, int D>
cudaError_t dispatch_mma(const AttendArgs& a, int grid, cudaStream_t s, bool pdl) {
  if (a.G <= 8) return launch_path<MmaPath<T, D, 1>, D>(a, grid, s, pdl);
  return launch_path<MmaPath<T, D, 2>, D>(a, grid, s, pdl);
}

template <typename T, typename TQ, int D>
cudaError_t dispatch_simt_g(const AttendArgs& a, int grid, cudaStream_t s, bool pdl) {
  if (a.G <= 4) return launch_path<SimtPath<T, TQ, D, 4>, D>(a, grid, s, pdl);
  if (a.G <= 8) return launch_path<SimtPath<T, TQ, D, 8>, D>(a, grid, s, pdl);
  return launch_path<SimtPath<T, TQ, D, 16>, D>(a, grid, s, pdl);
}

template <typename T, typename TQ>
cudaError_t dispatch_simt_d(const AttendArgs& a, int d, int grid, cudaStream_t s, bool pdl) {
  switch (d) {
    case 64: return dispatch_simt_g<T, TQ, 64>(a, grid, s, pdl);
    case 128: return dispatch_simt_g<T, TQ, 128>(a, grid, s, pdl);
    case 256: return dispatch_simt_g<T, TQ, 256>(a, grid, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t dispatch_simt_q(const AttendArgs& a, int qdt, int d, int grid, cudaStream_t s,
                            bool pdl) {
  switch (qdt) {
    case CVSA_DTYPE_BF16: return dispatch_simt_d<T, __nv_bfloat16>(a, d, grid, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_simt_d<T, __half>(a, d, grid, s, pdl);
    case CVSA_DTYPE_F32: return dispatch_simt_d<T, float>(a, d, grid, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool attend_supported(const QView& q, const KvView& kv) {
  if (kv.bs != kBS) return false;
  if (kv.d != 64 && kv.d != 128 && kv.d != 256) return false;
  if (kv.hkv <= 0 || q.hq % kv.hkv != 0 || q.hq / kv.hkv > 16) return false;
  return true;
}

size_t attend_workspace_bytes(const QView& q, const KvView& kv, int max_sel, bool recover,
                              bool dense) {
  const ItemCfg ic = item_cfg(q, kv, max_sel, recover, dense);
  const size_t grid = (size_t)q.B * kv.hkv * ic.iph;
  const int G = q.hq / kv.hkv;
  size_t bytes = 0;
  bytes += grid * G * kv.d * 4;            // part_o
  bytes += grid * G * 2 * 4;               // part_ml
  bytes = (bytes + 255) & ~size_t(255);
  return bytes;
}

cudaError_t launch_attend(const QView& q, const KvView& kv, const AttendParams& p, int max_sel,
                          cudaStream_t s, bool pdl) {
  AttendArgs a;
  memset(&a, 0, sizeof(a));
  const bool mma = use_mma(q, kv);
  if (mma) {
    if (!cached_pool_map(&a.kmap, kv.k, kv) || !cached_pool_map(&a.vmap, kv.v, kv))
      return cudaErrorInvalidValue;
  }
  a.q = q.q;
  a.k = kv.k;
  a.v = kv.v;
  a.sb = kv.sb;
  a.st = kv.st;
  a.sh = kv.sh;
  a.B = q.B;
  a.hq = q.hq;
  a.hkv = kv.hkv;
  a.G = q.hq / kv.hkv;
  a.W = q.W;
  a.num_blocks = kv.num_blocks;
  a.tables = q.tables;
  a.lens = q.lens;
  a.sel0 = p.sel0;
  a.n0 = p.n0;
  a.sel1 = p.sel1;
  a.n1 = p.n1;
  a.sel_stride = p.sel_stride;
  a.src_select = p.src_select;
  a.decision = p.decision;
  a.dense = p.dense ? 1 : 0;
  a.recover = p.recover ? 1 : 0;
  a.accept = p.accept;
  a.bitmap = p.bitmap;
  a.bitmap_words = p.bitmap_words;
  a.external_draft = p.external_draft ? 1 : 0;
  a.ext_o = p.ext_o;
  a.ext_m = p.ext_m;
  a.ext_l = p.ext_l;
  a.commit = p.commit_src1 ? 1 : 0;
  a.commit_idx = p.commit_idx;
  a.commit_n = p.commit_n;
  a.out = p.out;
  a.out_dtype = p.out_dtype;
  a.o_unnorm = p.o_unnorm;
  a.m_out = p.m_out;
  a.l_out = p.l_out;
  a.counters = p.counters;
  a.dev_err = p.dev_err;
  a.accept_out = p.accept_out;
  a.cov_out = p.cov_out;
  a.acc0 = p.acc0;
  a.cov0 = p.cov0;
  a.acc1 = p.acc1;
  a.cov1 = p.cov1;
  a.ic = item_cfg(q, kv, max_sel, p.recover, p.dense);
  if (p.external_draft) {
    // recovery only: no draft items
    a.ic.nd = 0;
    a.ic.cc = kMaxItemPages;
    a.ic.nc = (q.W + a.ic.cc - 1) / a.ic.cc;
    if (a.ic.nc < 1) a.ic.nc = 1;
    a.ic.iph = a.ic.nc;
  }
  const size_t grid = (size_t)q.B * kv.hkv * a.ic.iph;
  const int G = a.G;
  a.part_o = reinterpret_cast<float*>(p.partials);
  a.part_ml = a.part_o + grid * G * kv.d;
  a.head_done = p.head_done;
  a.scale = 1.0f / sqrtf((float)kv.d);
  if (grid == 0) return cudaSuccess;
  if (grid > 0x7fffffff) return cudaErrorInvalidValue;
  if ((size_t)q.B * kv.hkv > (size_t)kMaxHeadsPerCall) return cudaErrorInvalidValue;
  if (p.partial_bytes < grid * G * (kv.d + 2) * 4) return cudaErrorInvalidValue;

  if (mma) {
    if (kv.dtype == CVSA_DTYPE_BF16) {
      switch (kv.d) {
        case 64: return dispatch_mma<__nv_bfloat16, 64>(a, (int)grid, s, pdl);
        case 128: return dispatch_mma<__nv_bfloat16, 128>(a, (int)grid, s, pdl);
        case 256: return dispatch_mma<__nv_bfloat16, 256>(a, (int)grid, s, pdl);
      }
    } else {
      switch (kv.d) {
        case 64: return dispatch_mma<__half, 64>(a, (int)grid, s, pdl);
        case 128: return dispatch_mma<__half, 128>(a, (int)grid, s, pdl);
        case 256: return dispatch_mma<__half, 256>(a, (int)grid, s, pdl);
      }
    }
    return cudaErrorInvalidValue;
  }
  switch (kv.dtype) {
    case CVSA_DTYPE_F32: return dispatch_simt_q<float>(a, q.dtype, kv.d, (int)grid, s, pdl);
    case CVSA_DTYPE_BF16: return dispatch_simt_q<__nv_bfloat16>(a, q.dtype, kv.d, (int)grid, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_simt_q<__half>(a, q.dtype, kv.d, (int)grid, s, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace cvsa
