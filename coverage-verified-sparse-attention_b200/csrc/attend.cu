// Sparse paged decode, fused exact recovery and LSE merge, for the layouts
// the TMA stream kernel (attend_stream.cu) does not take: fp32 KV, q and KV in
// different dtypes, or pools whose strides or base are not 16-byte aligned.
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
// Work decomposition. Each (b, kv head) has `nd` draft items (chunks of up to
// 32 pages of its selection) and, when it must recover, complement items
// (chunks of 32 logical pages minus the selected ones); a dense layer has
// chunks of all valid pages. Draft items are enumerated statically; the
// complement items of the rejected heads form a compact list whose per-head
// offsets the selection kernel's last CTA scanned. CTAs are persistent and walk
// this item space with a grid stride. A CTA of 4 warps runs one item at a
// time: the warps take its pages round robin and read K and V rows straight
// from global memory (lane = head_dim columns), each keeping an online-softmax
// state; warp states merge in shared memory into an item partial (o, m, l) per
// query head. A head with one item is finished by that CTA; otherwise the last
// CTA to finish an item of the head (atomic ticket, no spin) merges the
// partials in a fixed order -- draft chunks, then complement chunks -- so
// results are deterministic.
#include <mutex>
#include <unordered_map>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kNW = 4;             // warps per CTA
constexpr int kStages = 2;         // barrier words reserved per warp
constexpr int kMaxItemPages = 32;  // pages per item (list capacity)
constexpr int kBS = 16;            // tokens per page (kernels built for 16)

struct ItemCfg {
  int cd, nd;  // draft chunk pages, draft items per head
  int cc, nc;  // complement/dense chunk pages, items per head
  int iph;     // scratch slots per head (nd + nc)
};

struct AttendArgs {
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
  const int32_t* comp_off;  // [heads + 1] complement-item offsets, or null (static list)
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
  float* part_o;   // [heads * iph][G][D]
  float* part_ml;  // [heads * iph][G][2]
  int32_t* head_done;
  ItemCfg ic;
  int heads;       // B * hkv
  float scale;
};

// ---------------------------------------------------------------------------
// per-item bookkeeping shared by both per-page variants
// ---------------------------------------------------------------------------
struct ItemInfo {
  int bh, b, h;
  int ctx, nv;
  int src;  // 0/1 selection source, -1 dense
  int n_sel;
  const int32_t* sel;
  bool rec;
  int nd_act, nc_act, expected;
  int role;   // 0 draft/dense chunk, 1 complement chunk
  int chunk;  // chunk index within its role
  int slot;   // scratch slot of this item
  bool active;
};

__device__ __forceinline__ int item_source(const AttendArgs& a) {
  int s = a.src_select;
  if (s == 2) s = (a.decision[0] & 1) ? 0 : 1;
  return s;
}

__device__ __forceinline__ ItemInfo make_item(const AttendArgs& a, int bh, int role, int chunk) {
  ItemInfo it;
  it.bh = bh;
  it.b = bh / a.hkv;
  it.h = bh % a.hkv;
  it.role = role;
  it.chunk = chunk;
  it.ctx = a.lens[it.b];
  it.nv = min(n_valid_pages(it.ctx, kBS), a.W);
  if (a.dense) {
    it.src = -1;
    it.n_sel = 0;
    it.sel = nullptr;
  } else {
    const int s = item_source(a);
    it.src = s;
    it.sel = (s ? a.sel1 : a.sel0) + (int64_t)bh * a.sel_stride;
    it.n_sel = min(max((s ? a.n1 : a.n0)[bh], 0), a.sel_stride);
  }
  it.rec = a.recover && !a.dense && (a.external_draft || it.src == 1) && a.accept[bh] == 0;
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
  if (role == 0 && !a.dense) {
    it.active = chunk < it.nd_act;
    it.slot = bh * a.ic.iph + chunk;
  } else {
    it.active = chunk < it.nc_act;
    it.slot = bh * a.ic.iph + a.ic.nd + chunk;
  }
  return it;
}

// Virtual item space: [0, n_static) draft (or dense) chunks of every head,
// then complement chunks: a compact list when comp_off is given, else every
// head's chunks (inactive ones skipped).
__device__ __forceinline__ int n_static_items(const AttendArgs& a) {
  return a.heads * (a.dense ? a.ic.nc : a.ic.nd);
}

__device__ __forceinline__ int n_total_items(const AttendArgs& a) {
  const int ns = n_static_items(a);
  if (a.dense || !a.recover) return ns;
  if (a.comp_off) return ns + a.comp_off[a.heads];
  return ns + a.heads * a.ic.nc;
}

__device__ __forceinline__ ItemInfo decode_item(const AttendArgs& a, int v) {
  const int ns = n_static_items(a);
  if (v < ns) {
    const int per = a.dense ? a.ic.nc : a.ic.nd;
    return make_item(a, v / per, a.dense ? 0 : 0, v % per);
  }
  const int u = v - ns;
  if (a.comp_off) {
    // largest bh with comp_off[bh] <= u
    int lo = 0, hi = a.heads - 1;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (a.comp_off[mid] <= u) lo = mid;
      else hi = mid - 1;
    }
    return make_item(a, lo, 1, u - a.comp_off[lo]);
  }
  return make_item(a, u / a.ic.nc, 1, u % a.ic.nc);
}

// Build this item's page list (ascending within the item) in shared memory,
// with each page's physical block resolved once here (-1 when the block-table
// entry lies outside the pool), so the page loop never waits on the table.
__device__ __forceinline__ void build_page_list(const AttendArgs& a, const ItemInfo& it,
                                                int* list, int* blist, int* cnt) {
  if (threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  int pg = -1;
  bool keep = false;
  if (it.role == 0 && !a.dense) {
    const int i = it.chunk * a.ic.cd + lane;
    if (lane < a.ic.cd && i < it.n_sel) {
      pg = it.sel[i];
      keep = pg >= 0 && pg < a.W;
      if (!keep) set_dev_error(a.dev_err, CVSA_DEV_ERR_PAGE_RANGE);
    }
  } else {
    const bool empty = a.external_draft && !it.rec;
    const int p = it.chunk * a.ic.cc + lane;
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
  if (keep) {
    int blk = a.tables[(int64_t)it.b * a.W + pg];
    if (blk < 0 || blk >= a.num_blocks) {
      set_dev_error(a.dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
      blk = -1;
    }
    const int pos = __popc(m & ((1u << lane) - 1u));
    list[pos] = pg;
    blist[pos] = blk;
  }
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

// Final merge of one (b, h). `single`: the head has one item whose partial is
// ip_o/ip_ml (shared memory). Otherwise the partials of every item of the head
// are in part_o/part_ml; their (m, l) are staged in `stage` (shared, at least
// n_items * G * 2 floats when `fits`) and each output element sums its item
// partials with independent loads.
template <int D>
__device__ void finalize_head(const AttendArgs& a, const ItemInfo& it, const float* ip_o,
                              const float* ip_ml, bool single, float* stage, int stage_floats) {
  const int G = a.G;
  const int n0 = a.external_draft ? 0 : (a.dense ? it.nc_act : it.nd_act);
  const int off0 = a.dense ? a.ic.nd : 0;   // first slot of the role-0 items
  const int n1 = it.rec ? it.nc_act : 0;
  const int nitems = n0 + n1;
  const int64_t base = (int64_t)it.bh * a.ic.iph;
  // slot of item i of the combined list: role-0 items, then role-1 items
  auto slot_of = [&](int i) -> int64_t {
    return base + (i < n0 ? off0 + i : a.ic.nd + (i - n0));
  };
  const bool staged = !single && nitems * G * 2 + 4 * G <= stage_floats;
  if (staged) {
    // stage (m, l) of every item; then per (role, g): M, weights, L
    float* w = stage;                       // [nitems][G] weights (m replaced)
    float* lsum = stage + nitems * G;       // [nitems][G] l
    float* red = stage + 2 * nitems * G;    // [2][G][2]: M, L per role
    for (int e = threadIdx.x; e < nitems * G; e += kNW * 32) {
      const int i = e / G, g = e % G;
      const int64_t s = slot_of(i);
      w[e] = __ldcg(&a.part_ml[(s * G + g) * 2]);
      lsum[e] = __ldcg(&a.part_ml[(s * G + g) * 2 + 1]);
    }
    __syncthreads();
    if (threadIdx.x < 2 * G) {
      const int r = threadIdx.x / G, g = threadIdx.x % G;
      const int i0 = r == 0 ? 0 : n0, i1 = r == 0 ? n0 : nitems;
      float M = neg_inf();
      for (int i = i0; i < i1; ++i) M = fmaxf(M, w[i * G + g]);
      float L = 0.f;
      for (int i = i0; i < i1; ++i) {
        const float mi = w[i * G + g];
        const float wi = (mi == neg_inf()) ? 0.f : expf(mi - M);
        w[i * G + g] = wi;
        L += lsum[i * G + g] * wi;
      }
      red[(r * G + g) * 2] = M;
      red[(r * G + g) * 2 + 1] = L;
    }
    __syncthreads();
  }
  for (int e = threadIdx.x; e < G * D; e += kNW * 32) {
    const int g = e / D, d = e % D;
    float md = neg_inf(), ld = 0.f, od = 0.f;
    float mc = neg_inf(), lc = 0.f, oc = 0.f;
    if (single) {
      const float pm = ip_ml[g * 2], pl = ip_ml[g * 2 + 1], po = ip_o[g * D + d];
      if (it.role == 0) { md = pm; ld = pl; od = po; }
      else { mc = pm; lc = pl; oc = po; }
    } else if (staged) {
      const float* w = stage;
      const float* red = stage + 2 * nitems * G;
      md = red[g * 2];
      ld = red[g * 2 + 1];
      mc = red[(G + g) * 2];
      lc = red[(G + g) * 2 + 1];
      float acc0 = 0.f, acc1 = 0.f;
#pragma unroll 4
      for (int i = 0; i < n0; ++i)
        acc0 += w[i * G + g] * __ldcg(&a.part_o[(slot_of(i) * G + g) * D + d]);
#pragma unroll 4
      for (int i = n0; i < nitems; ++i)
        acc1 += w[i * G + g] * __ldcg(&a.part_o[(slot_of(i) * G + g) * D + d]);
      od = acc0;
      oc = acc1;
    } else {
      for (int i = 0; i < nitems; ++i) {
        const int64_t s = slot_of(i);
        const float pm = __ldcg(&a.part_ml[(s * G + g) * 2]);
        const float pl = __ldcg(&a.part_ml[(s * G + g) * 2 + 1]);
        const float po = __ldcg(&a.part_o[(s * G + g) * D + d]);
        if (i < n0) lse_combine(md, ld, od, pm, pl, po);
        else lse_combine(mc, lc, oc, pm, pl, po);
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

// Row stride (floats) of the warp-state buffer: D + 8 keeps the 8 query rows a
// warp writes at once in distinct shared-memory banks.
template <int D>
constexpr int wb_stride() { return D + 8; }

// Merge the kNW warp states (wb_o [kNW][GP][D + 8], wb_ml [kNW][GP][2]) into
// the item partial ip_o [G][D], ip_ml [G][2].
template <int D>
__device__ void merge_warps(int G, int GP, const float* wb_o, float* wb_ml, float* ip_o,
                            float* ip_ml) {
  constexpr int S = wb_stride<D>();
  // per query row: the merged (m, l) and each warp's weight exp(m_w - m),
  // computed once; the weights overwrite the warps' m in wb_ml
  if (threadIdx.x < G) {
    const int g = threadIdx.x;
    float m = neg_inf();
#pragma unroll
    for (int w = 0; w < kNW; ++w) m = fmaxf(m, wb_ml[(w * GP + g) * 2]);
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) {
      const float mw = wb_ml[(w * GP + g) * 2];
      const float sw = (mw == neg_inf()) ? 0.f : expf(mw - m);
      wb_ml[(w * GP + g) * 2] = sw;
      l += wb_ml[(w * GP + g) * 2 + 1] * sw;
    }
    ip_ml[g * 2] = m;
    ip_ml[g * 2 + 1] = l;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < G * D; e += kNW * 32) {
    const int g = e / D, d = e % D;
    float o = 0.f;
#pragma unroll
    for (int w = 0; w < kNW; ++w) o += wb_ml[(w * GP + g) * 2] * wb_o[(w * GP + g) * S + d];
    ip_o[g * D + d] = o;
  }
}

// ---------------------------------------------------------------------------
// CUDA-core per-page step (fp32 or mixed dtypes); lane owns head_dim columns
// d = lane + 32 i. Up to GM query heads per KV head.
// ---------------------------------------------------------------------------
template <typename T, typename TQ, int D, int GM>
struct SimtPath {
  static constexpr int kGP = GM;
  static constexpr int kPer = D / 32;
  static constexpr size_t ring_bytes() {
    // warp-state buffer; at least 64 KB so the finaliser can stage partials
    size_t wb = (size_t)kNW * GM * wb_stride<D>() * 4 + (size_t)kNW * GM * 2 * 4;
    return wb > 65536 ? wb : 65536;
  }
  __device__ static bool run(const AttendArgs& a, const ItemInfo& it, uint8_t*, uint64_t*,
                             const int* list, const int* blist, int cnt, float* wb_o,
                             float* wb_ml, uint32_t&) {
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
    for (int jj = w; jj < cnt; jj += kNW) {
      const int pg = list[jj];
      const int blk = blist[jj];
      if (blk < 0) continue;  // out-of-pool block (recorded when the list was built)
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
    __syncthreads();
#pragma unroll
    for (int g = 0; g < GM; ++g) {
#pragma unroll
      for (int i = 0; i < kPer; ++i) wb_o[(w * GM + g) * wb_stride<D>() + lane + 32 * i] = o[g][i];
      if (lane == 0) {
        wb_ml[(w * GM + g) * 2] = m_run[g];
        wb_ml[(w * GM + g) * 2 + 1] = l_run[g];
      }
    }
    return true;
  }
};

template <class Path, int D>
constexpr size_t kernel_smem_bytes() {
  // 1 KB alignment slack + ring/warp states + item partial (16 rows) +
  // barriers + page list, count and flags
  return 1024 + Path::ring_bytes() + (size_t)Path::kGP * D * 4 + Path::kGP * 2 * 4 + kNW * kStages * 8 +
         (2 * kMaxItemPages + 4) * 4;
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------
template <class Path, int D>
__global__ void __launch_bounds__(kNW * 32)
attend_kernel(const __grid_constant__ AttendArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t base_u32 = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (base_u32 & 1023)) & 1023);

  constexpr size_t kRing = Path::ring_bytes();
  uint8_t* ring = smem;
  float* wb_o = reinterpret_cast<float*>(smem);
  float* wb_ml = wb_o + (size_t)kNW * Path::kGP * wb_stride<D>();
  float* ip_o = reinterpret_cast<float*>(smem + kRing);
  float* ip_ml = ip_o + Path::kGP * D;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ip_ml + Path::kGP * 2);
  int* list = reinterpret_cast<int*>(bars + kNW * kStages);
  int* blist = list + kMaxItemPages;
  int* cnt = blist + kMaxItemPages;
  int* flag_last = cnt + 1;
  int* flag_fail = cnt + 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNW * kStages; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    *flag_fail = 0;
  }
  pdl_wait();
  const int n_total = n_total_items(a);
  __syncthreads();
  uint32_t gpage = 0;  // pages this warp has streamed through its ring so far

  for (int v = blockIdx.x; v < n_total; v += gridDim.x) {
    const ItemInfo it = decode_item(a, v);
    if (!it.active) continue;
    build_page_list(a, it, list, blist, cnt);
    __syncthreads();
    const int n = *cnt;
    if (!Path::run(a, it, ring, bars, list, blist, n, wb_o, wb_ml, gpage)) *flag_fail = 1;
    __syncthreads();
    if (*flag_fail) return;  // a copy never arrived: stop without touching outputs
    merge_warps<D>(a.G, Path::kGP, wb_o, wb_ml, ip_o, ip_ml);
    __syncthreads();
    if (it.expected == 1) {
      finalize_head<D>(a, it, ip_o, ip_ml, true, nullptr, 0);
    } else {
      // publish this item's partial, then take a ticket for (b, h)
      const int64_t slot = it.slot;
      for (int e = threadIdx.x; e < a.G * D; e += kNW * 32)
        a.part_o[slot * a.G * D + e] = ip_o[e];
      for (int e = threadIdx.x; e < a.G * 2; e += kNW * 32)
        a.part_ml[slot * a.G * 2 + e] = ip_ml[e];
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) {
        const int prev = atomicAdd(&a.head_done[it.bh], 1);
        *flag_last = (prev == it.expected - 1) ? 1 : 0;
      }
      __syncthreads();
      if (*flag_last) {
        __threadfence();
        finalize_head<D>(a, it, ip_o, ip_ml, false, reinterpret_cast<float*>(ring),
                         (int)(kRing / 4));
        if (threadIdx.x == 0) a.head_done[it.bh] = 0;
      }
    }
    __syncthreads();  // shared buffers are rewritten by the next item
  }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
ItemCfg item_cfg(const QView& q, const KvView& kv, int max_sel, bool recover, bool dense) {
  ItemCfg c;
  const int heads = q.B * kv.hkv;
  // aim for about two items per resident CTA slot (2 CTAs per SM)
  const int target = 4 * num_sms();
  if (dense) {
    c.cd = kMaxItemPages;
    c.nd = 0;
  } else {
    const int per_head = (target + heads - 1) / heads;
    int cd = (max_sel + per_head - 1) / per_head;
    cd = ((cd + kNW - 1) / kNW) * kNW;
    c.cd = cd < 8 ? 8 : (cd > kMaxItemPages ? kMaxItemPages : cd);
    c.nd = (max_sel + c.cd - 1) / c.cd;
    if (c.nd < 1) c.nd = 1;
  }
  c.cc = kMaxItemPages;
  c.nc = (recover || dense) ? (q.W + c.cc - 1) / c.cc : 0;
  if ((recover || dense) && c.nc < 1) c.nc = 1;
  c.iph = c.nd + c.nc;
  return c;
}

template <class Path, int D>
cudaError_t launch_path(const AttendArgs& a, int max_items, cudaStream_t s, bool pdl) {
  constexpr size_t smem = kernel_smem_bytes<Path, D>();
  // resident CTAs per SM, measured once per device (the attribute is per device)
  static int ctas_per_sm[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!ctas_per_sm[dev]) {
    e = cudaFuncSetAttribute(attend_kernel<Path, D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem);
    if (e != cudaSuccess) return e;
    int occ = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, attend_kernel<Path, D>, kNW * 32,
                                                      smem);
    if (e != cudaSuccess) return e;
    ctas_per_sm[dev] = occ < 1 ? 1 : occ;
  }
  int grid = num_sms() * ctas_per_sm[dev];
  if (grid > max_items) grid = max_items;
  if (grid < 1) grid = 1;
  return launch_k(attend_kernel<Path, D>, dim3(grid), dim3(kNW * 32), smem, s, pdl, a);
}

template <typename T, typename TQ, int D>
cudaError_t dispatch_simt_g(const AttendArgs& a, int max_items, cudaStream_t s, bool pdl) {
  if (a.G <= 4) return launch_path<SimtPath<T, TQ, D, 4>, D>(a, max_items, s, pdl);
  if (a.G <= 8) return launch_path<SimtPath<T, TQ, D, 8>, D>(a, max_items, s, pdl);
  return launch_path<SimtPath<T, TQ, D, 16>, D>(a, max_items, s, pdl);
}

template <typename T, typename TQ>
cudaError_t dispatch_simt_d(const AttendArgs& a, int d, int max_items, cudaStream_t s, bool pdl) {
  switch (d) {
    case 64: return dispatch_simt_g<T, TQ, 64>(a, max_items, s, pdl);
    case 128: return dispatch_simt_g<T, TQ, 128>(a, max_items, s, pdl);
    case 256: return dispatch_simt_g<T, TQ, 256>(a, max_items, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t dispatch_simt_q(const AttendArgs& a, int qdt, int d, int max_items, cudaStream_t s,
                            bool pdl) {
  switch (qdt) {
    case CVSA_DTYPE_BF16: return dispatch_simt_d<T, __nv_bfloat16>(a, d, max_items, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_simt_d<T, __half>(a, d, max_items, s, pdl);
    case CVSA_DTYPE_F32: return dispatch_simt_d<T, float>(a, d, max_items, s, pdl);
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

int attend_complement_chunk() { return kMaxItemPages; }

size_t attend_workspace_bytes(const QView& q, const KvView& kv, int max_sel, bool recover,
                              bool dense) {
  if (stream_attend_eligible(q, kv))
    return stream_attend_workspace_bytes(q, kv, dense ? 1 : max_sel);
  const ItemCfg ic = item_cfg(q, kv, max_sel, recover, dense);
  const size_t slots = (size_t)q.B * kv.hkv * ic.iph;
  const int G = q.hq / kv.hkv;
  size_t bytes = 0;
  bytes += slots * G * kv.d * 4;            // part_o
  bytes += slots * G * 2 * 4;               // part_ml
  bytes = (bytes + 255) & ~size_t(255);
  return bytes;
}

cudaError_t launch_attend(const QView& q, const KvView& kv, const AttendParams& p, int max_sel,
                          cudaStream_t s, bool pdl) {
  if (stream_attend_eligible(q, kv)) return launch_stream_attend(q, kv, p, max_sel, s, pdl);
  AttendArgs a;
  memset(&a, 0, sizeof(a));
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
  a.comp_off = p.comp_off;
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
  a.heads = q.B * kv.hkv;
  const size_t slots = (size_t)a.heads * a.ic.iph;
  const int G = a.G;
  a.part_o = reinterpret_cast<float*>(p.partials);
  a.part_ml = a.part_o + slots * G * kv.d;
  a.head_done = p.head_done;
  a.scale = 1.0f / sqrtf((float)kv.d);
  if (slots == 0) return cudaSuccess;
  if (slots > 0x7fffffff) return cudaErrorInvalidValue;
  if ((size_t)a.heads > (size_t)kMaxHeadsPerCall) return cudaErrorInvalidValue;
  if (p.partial_bytes < slots * G * (kv.d + 2) * 4) return cudaErrorInvalidValue;
  // upper bound of the virtual item space (the grid never exceeds it)
  const int max_items = (int)slots;

  switch (kv.dtype) {
    case CVSA_DTYPE_F32: return dispatch_simt_q<float>(a, q.dtype, kv.d, max_items, s, pdl);
    case CVSA_DTYPE_BF16: return dispatch_simt_q<__nv_bfloat16>(a, q.dtype, kv.d, max_items, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_simt_q<__half>(a, q.dtype, kv.d, max_items, s, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace cvsa
