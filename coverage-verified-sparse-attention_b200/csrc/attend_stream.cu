// Sparse paged decode over a balanced page stream: the decode-step attention
// for bf16 / f16 KV (q in the same dtype) in a 16-byte-aligned pool.
//
// Restates:
//   * cvsa/kernels/sparse_decode.py:424-500 (split decode over a page list:
//     s = (q . k) * D^-0.5, online softmax, unnormalised (o, m, l)) and
//     :15-132 (normalised output o / max(l, 1e-6));
//   * cvsa/backend.py:819-842, exact recovery of a rejected head. The
//     reference attends the selected pages (draft) and the remaining valid
//     pages (complement, cvsa/kernels/coverage.py:31-96) separately and merges
//     the two (coverage.py:274-326, o = (o_d s_d + o_c s_c) / max(l, 1e-6)).
//     Draft and complement partition the valid pages, so the merged result is
//     the softmax over all valid pages; a rejected head is attended over that
//     set directly, which is the same quantity with one merge fewer;
//   * recover_merge with an external draft: the complement only (selected
//     pages skipped through a bitmap), merged with the given draft.
//
// Work decomposition. Every head (b, kv head) of the launch contributes w_h
// pages to one flat stream: its selected pages (list heads), or all of its
// valid pages (range heads: dense steps and rejected heads). The stream of
// P = sum(w_h) pages is cut into gridDim.x equal contiguous ranges, one per
// persistent CTA (one CTA per SM), so the load is balanced to one page
// whatever the mix of lengths, selections and rejections.
//
// Inside a CTA, warp NC resolves the CTA's stream positions 32 at a time
// (head by binary search over the shared-memory prefix of w_h, then the
// selection entry and the block-table entry) into a shared-memory ring of
// page descriptors, running ahead of the consumers. Consumer warp k
// (0 <= k < NC) owns positions j with j % NC == k: it copies each page's K and
// V rows of its KV head (16 tokens x head_dim, 16-byte cp.async, 128-byte
// swizzled rows) into its own ring of S stages, S - 1 pages ahead of the one
// it computes, and runs S = Q K^T and O += P V on mma.sync m16n8k16 (all G
// query heads of the KV head packed into M) with the online softmax in
// registers. Pages are gathered at 256-byte granularity from pages scattered
// over the pool, which per-warp 16-byte copies serve at full rate where
// one small TMA box per 64 columns would bound each SM by its TMA issue rate.
// At the end of each head a consumer writes its state (o, m, l per query
// row, rescaled to the exact row max) to a global partial; consumer warps
// issue no memory fences while copies are in flight (a fence would wait for
// them). When its streaming is done, a CTA merges the partials of the heads
// that lie inside its range (one warp per query row); a head split over CTAs
// is merged by the last of them to finish (ticket per head, no spin).
// Partials merge in CTA then warp order, so results are deterministic for a
// given device.
#include <climits>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kBS = 16;                  // tokens per page
constexpr int kMaxChunkHeads = 2048;     // heads per launch (shared-memory head table)
constexpr int kMaxConsumers = 8;
constexpr int kMetaPerConsumer = 64;     // page descriptors in flight per consumer
constexpr int kMaxStages = 8;            // per-consumer ring depth (cp.async.wait_group)
constexpr int kSmemCap = 227 * 1024;     // dynamic shared memory per CTA on sm_100
constexpr uint32_t kSpinLimit = 1u << 22;
// the softmax reference max is refreshed when a score passes it by more than
// this (natural log units): probabilities stay below e^8 ~ 3e3
constexpr float kRescaleGap = 8.0f;
constexpr int kMaxQSlots = 8;  // heads whose query rows a CTA stages in shared memory

// a head's pages: none; its selection list; every valid page; every valid
// page outside its selection (bitmap); its expanded selection (approximate
// recovery)
enum : int { kKindEmpty = 0, kKindList = 1, kKindRange = 2, kKindRangeSkip = 3, kKindExp = 4 };

struct StreamArgs {
  const void* q;
  const void* k;
  const void* v;
  int64_t sb, st, sh;  // pool strides (elements): block, token, head
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
  int dense, recover, external_draft;
  const uint8_t* accept;
  const uint32_t* bitmap;
  int bitmap_words;
  const float* ext_o;
  const float* ext_m;
  const float* ext_l;
  int approx;              // rejected heads decode their expanded selection
  const int32_t* exp_idx;  // [heads][exp_stride]
  const int32_t* exp_n;
  int exp_stride;
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
  float* part_o;       // [slots][G][D] consumer partials of this launch
  float* part_ml;      // [slots][G][2]
  float* cpart_o;      // [heads + CTAs][G][D] per-CTA partials of split heads
  float* cpart_ml;     // [heads + CTAs][G][2]
  int32_t* head_done;  // per (b, kv head) of the whole call, zero at rest
  int h_base, n_heads; // heads [h_base, h_base + n_heads) of this launch
  int nc, stages, meta_cap;
  // shared-memory carve-up, byte offsets from the 1024-aligned base
  int off_meta, off_snt, off_pref, off_ctx, off_kind, off_span, off_misc, off_bnd;
  // the query rows of a CTA's first q_slots heads are copied into shared
  // memory at the start (one bulk copy per head on the mbarrier at off_qbar)
  int off_qbar, off_q, q_slots;
  // polls of a bounded wait on another warp (the producer's descriptors, a
  // free ring entry, the staged query rows) before it gives up; the waits
  // that drain the CTA's own copies before it exits keep the default
  uint32_t wait_polls;
  int grid;            // CTAs of the launch (<= the SM count)
  float scale;
};

// misc words
constexpr int kMiscFail = 4;       // a bounded wait gave up: stop
constexpr int kMiscProd = 5;       // page descriptors published (local positions)
constexpr int kMiscScan = 8;       // [33] block-scan scratch
constexpr int kMiscCons = 48;      // [kMaxConsumers] next position each consumer reads
constexpr int kMiscWon = 56;       // [2] this CTA merges its first / last head
constexpr int kMiscWmax = 58;      // the largest w_h of the launch
constexpr int kMiscWords = 64;
constexpr int kMaxBnd = 256;       // CTAs of a launch whose ranges may snap to head starts
constexpr int kMinPagesPerCta = 12;  // stream pages per CTA below which a launch uses fewer CTAs
// Longest head (pages) for which the ranges snap to head starts: a snapped cut
// moves by at most half a head, <= 16 page-heads (about 3 us of one SM's share
// of HBM), about the cross-CTA merge it saves; longer heads (ragged batches,
// long selections) keep equal cuts, where the shift would unbalance the CTAs
constexpr int kAlignMaxW = 32;

// Consumer warps a launch may use: 8, or 4 where the wider per-lane state
// (head_dim 256, or more than 8 query heads at head_dim 128) needs the larger
// register budget of a smaller CTA.
template <int D, int GR>
constexpr int max_consumers() { return (D == 256 || (D == 128 && GR == 2)) ? 4 : kMaxConsumers; }
constexpr int max_consumers_rt(int D, int G) {
  return (D == 256 || (D == 128 && G > 8)) ? 4 : kMaxConsumers;
}

__device__ __forceinline__ int block_excl_scan(int v, int* scratch, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  if (lane == 31) scratch[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int x = lane < nw ? scratch[lane] : 0;
    int xi = x;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, xi, o);
      if (lane >= o) xi += n;
    }
    if (lane < nw) scratch[lane] = xi - x;
    if (lane == 31) scratch[32] = xi;
  }
  __syncthreads();
  *total = scratch[32];
  const int r = scratch[warp] + incl - v;
  __syncthreads();
  return r;
}

// Bounded spin (lane-local) until *w >= target; false if it gave up.
__device__ __forceinline__ bool spin_until_ge(volatile int* w, int target, volatile int* fail,
                                              uint32_t limit) {
  uint32_t it = 0;
  while (*w < target) {
    if (*fail) return false;
    if (++it > limit) return false;
    __nanosleep(32);
  }
  return true;
}

template <int N>
__device__ __forceinline__ void store_vec(float* p, const float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      *reinterpret_cast<float4*>(p + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) *reinterpret_cast<float2*>(p + i) = make_float2(v[i], v[i + 1]);
  }
}

template <int N>
__device__ __forceinline__ void load_vec(const float* p, float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 t = *reinterpret_cast<const float4*>(p + i);
      v[i] = t.x; v[i + 1] = t.y; v[i + 2] = t.z; v[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 t = *reinterpret_cast<const float2*>(p + i);
      v[i] = t.x; v[i + 1] = t.y;
    }
  }
}

template <int N>
__device__ __forceinline__ void load_vec_cg(const float* p, float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4) {
      const float4 t = __ldcg(reinterpret_cast<const float4*>(p + i));
      v[i] = t.x; v[i + 1] = t.y; v[i + 2] = t.z; v[i + 3] = t.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2) {
      const float2 t = __ldcg(reinterpret_cast<const float2*>(p + i));
      v[i] = t.x; v[i + 1] = t.y;
    }
  }
}

// One partial row in global scratch (read with L1 bypassed: lines there may
// predate this launch's stores).
struct PartRow {
  const float* o;   // D values
  const float* ml;  // (m, l)
};

template <int N>
__device__ __forceinline__ void store_vec_cg(float* p, const float (&v)[N]) {
  if constexpr (N % 4 == 0) {
#pragma unroll
    for (int i = 0; i < N; i += 4)
      __stcg(reinterpret_cast<float4*>(p + i), make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]));
  } else {
#pragma unroll
    for (int i = 0; i < N; i += 2)
      __stcg(reinterpret_cast<float2*>(p + i), make_float2(v[i], v[i + 1]));
  }
}

template <typename TO>
__device__ __forceinline__ void store_o(void* out, int64_t idx, float v) {
  reinterpret_cast<TO*>(out)[idx] = Elem<TO>::from_f(v);
}

__device__ __forceinline__ void store_out(void* out, int dt, int64_t idx, float v) {
  if (dt == CVSA_DTYPE_BF16) store_o<__nv_bfloat16>(out, idx, v);
  else if (dt == CVSA_DTYPE_F16) store_o<__half>(out, idx, v);
  else store_o<float>(out, idx, v);
}

// Store PL consecutive outputs of one row in the output dtype, vectorised
// when the destination allows.
template <int PL>
__device__ __forceinline__ void store_row(void* out, int dt, int64_t idx, const float (&r)[PL]) {
  if (dt == CVSA_DTYPE_F32) {
    float* p = reinterpret_cast<float*>(out) + idx;
    if ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && PL % 4 == 0) {
#pragma unroll
      for (int i = 0; i < PL; i += 4)
        *reinterpret_cast<float4*>(p + i) = make_float4(r[i], r[i + 1], r[i + 2], r[i + 3]);
    } else {
#pragma unroll
      for (int i = 0; i < PL; ++i) p[i] = r[i];
    }
    return;
  }
  uint32_t w[PL / 2];
#pragma unroll
  for (int i = 0; i < PL / 2; ++i)
    w[i] = dt == CVSA_DTYPE_BF16 ? Mma<__nv_bfloat16>::pack(r[2 * i], r[2 * i + 1])
                                 : Mma<__half>::pack(r[2 * i], r[2 * i + 1]);
  uint32_t* p = reinterpret_cast<uint32_t*>(reinterpret_cast<uint16_t*>(out) + idx);
  if ((reinterpret_cast<uintptr_t>(p) & 7) == 0 && PL % 4 == 0) {
#pragma unroll
    for (int i = 0; i < PL / 2; i += 2) *reinterpret_cast<uint2*>(p + i) = make_uint2(w[i], w[i + 1]);
  } else if ((reinterpret_cast<uintptr_t>(p) & 3) == 0) {
#pragma unroll
    for (int i = 0; i < PL / 2; ++i) p[i] = w[i];
  } else {
#pragma unroll
    for (int i = 0; i < PL; ++i) store_out(out, dt, idx + i, r[i]);
  }
}

// Write the outputs of query row g of head bh from its merged state (M, L, o);
// lane holds o[d] for the D/32 consecutive columns d = lane * D/32 + i.
template <int D>
__device__ __forceinline__ void finish_row(const StreamArgs& a, int bh, int kind, int g, float M,
                                           float L, const float (&o)[D / 32]) {
  constexpr int PL = D / 32;
  const int lane = threadIdx.x & 31;
  const int b = bh / a.hkv, hh = bh % a.hkv;
  const int64_t qrow = (int64_t)b * a.hq + (int64_t)hh * a.G + g;
  const int64_t d0 = qrow * D + lane * PL;
  if (a.o_unnorm) {
#pragma unroll
    for (int i = 0; i < PL; ++i) a.o_unnorm[d0 + i] = o[i];
  }
  if (lane == 0) {
    if (a.m_out) a.m_out[qrow] = M;
    if (a.l_out) a.l_out[qrow] = L;
  }
  if (!a.out) return;
  float r[PL];
  if (a.external_draft) {
    const float md = a.ext_m[qrow], ld = a.ext_l[qrow];
    const bool merge = kind == kKindRangeSkip;
    // coverage.py:318-326: merge draft and complement, divide by max(l, 1e-6)
    const float m_all = merge ? fmaxf(md, M) : md;
    const float sd = (md == neg_inf()) ? 0.f : expf(md - m_all);
    const float sc = (!merge || M == neg_inf()) ? 0.f : expf(M - m_all);
    const float lm = fmaxf(merge ? ld * sd + L * sc : ld, 1e-6f);
#pragma unroll
    for (int i = 0; i < PL; ++i) {
      const float od = a.ext_o[d0 + i];
      r[i] = merge ? (od * sd + o[i] * sc) / lm : od / lm;
    }
  } else {
    const float lm = fmaxf(L, 1e-6f);
#pragma unroll
    for (int i = 0; i < PL; ++i) r[i] = o[i] / lm;
  }
  store_row<PL>(a.out, a.out_dtype, d0, r);
}

// Partial slot of consumer k of CTA c for head h. A CTA's heads are a
// contiguous range and CTA c's range never starts before CTA c - 1's ends, so
// (h + c) is distinct over the (head, CTA) pairs that meet: slots stay below
// (heads + CTAs) * NC.
__device__ __forceinline__ int64_t partial_slot(int h, int c, int k, int nc) {
  return (int64_t)(h + c) * nc + k;
}

// Merge np partial rows, the t-th at row_of(t) (a PartRow), in
// order t = 0..np-1 (deterministic), into (M, L, acc): the split-decode
// reduction of cvsa/kernels/sparse_decode.py:577-606 (maximum over the
// partials, weights exp(m_t - M), sums) at warp scale. Lane t holds partial
// t's (m, l) (one load round for up to 32 partials); the columns of kU
// partials are in flight together, the first kU issued with the (m, l) loads
// (they do not depend on M), so up to kU partials cost one round trip.
template <int D, class RowOf>
__device__ void merge_rows(int np, RowOf row_of, float& M, float& L, float (&acc)[D / 32]) {
  constexpr int PL = D / 32;
  constexpr int kU = PL >= 8 ? 4 : 32 / PL;
  const int lane = threadIdx.x & 31;
  float m0 = neg_inf(), l0 = 0.f;
  if (lane < np) {
    const PartRow r = row_of(lane);
    m0 = __ldcg(r.ml);
    l0 = __ldcg(r.ml + 1);
  }
  float ov0[kU][PL];
#pragma unroll
  for (int u = 0; u < kU; ++u) {
    if (u < np) {
      load_vec_cg<PL>(row_of(u).o + lane * PL, ov0[u]);
    } else {
#pragma unroll
      for (int i = 0; i < PL; ++i) ov0[u][i] = 0.f;
    }
  }
  M = m0;
  for (int t = lane + 32; t < np; t += 32) M = fmaxf(M, __ldcg(row_of(t).ml));
  M = warp_max(M);
  L = 0.f;
#pragma unroll
  for (int i = 0; i < PL; ++i) acc[i] = 0.f;
  if (M == neg_inf()) return;
  for (int t0 = 0; t0 < np; t0 += 32) {
    float w = 0.f;
    const int t = t0 + lane;
    if (t < np) {
      const float mt = t0 == 0 ? m0 : __ldcg(row_of(t).ml);
      const float lt = t0 == 0 ? l0 : __ldcg(row_of(t).ml + 1);
      w = (mt == neg_inf()) ? 0.f : expf(mt - M);
      L += lt * w;
    }
    const int cnt = min(32, np - t0);
    for (int v0 = 0; v0 < cnt; v0 += kU) {
      float ov[kU][PL];
      if (t0 == 0 && v0 == 0) {
#pragma unroll
        for (int u = 0; u < kU; ++u)
#pragma unroll
          for (int i = 0; i < PL; ++i) ov[u][i] = ov0[u][i];
      } else {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          if (v0 + u < cnt) {
            load_vec_cg<PL>(row_of(t0 + v0 + u).o + lane * PL, ov[u]);
          } else {
#pragma unroll
            for (int i = 0; i < PL; ++i) ov[u][i] = 0.f;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const float wv = __shfl_sync(0xffffffffu, w, (v0 + u) & 31);
#pragma unroll
        for (int i = 0; i < PL; ++i) acc[i] += wv * ov[u][i];
      }
    }
  }
  L = warp_sum(L);
}

// Where the partials of one merge live. Consumer partials of head h in CTA
// c: the t-th comes from consumer kk = kf + t (every slice non-empty) or the
// consumer of local position p0 + t (slices of at most one position), slot
// (h + c) NC + kk. CTA partials of head h: the t-th at row (h + fc + t) of
// the CTA-partial scratch.
struct MergeCtx {
  int c, NC, nloc, G;
  const float* part_o;
  const float* part_ml;
  float* cpart_o;
  float* cpart_ml;
};
struct RowSrc {
  int cpart, h, g, np;
  int kf, p0;  // consumer partials
  int fc;      // CTA partials
};
template <int D>
__device__ __forceinline__ PartRow part_row(const MergeCtx& x, const RowSrc& r, int t) {
  if (r.cpart) {
    const int64_t row = (int64_t)(r.h + r.fc + t) * x.G + r.g;
    return PartRow{x.cpart_o + row * D, x.cpart_ml + row * 2};
  }
  // (32-bit: nloc * NC stays far below 2^31)
  const int kk = x.nloc >= x.NC ? r.kf + t : ((r.p0 + t + 1) * x.NC - 1) / x.nloc;
  const int64_t row = ((int64_t)(r.h + x.c) * x.NC + kk) * x.G + r.g;
  return PartRow{x.part_o + row * D, x.part_ml + row * 2};
}

enum : int { kEmitFinish = 0, kEmitCtaPartial = 1 };

// One warp: merge the partials of r (none: the empty state) and either
// finish query row r.g of head r.h or store it as this CTA's partial of the
// head (inlined: an out-of-line copy measured slower).
template <int D>
__device__ __forceinline__ void merge_emit(const StreamArgs& a, MergeCtx x, RowSrc r, int emit,
                                        int kind) {
  constexpr int PL = D / 32;
  float M, L, acc[PL];
  merge_rows<D>(r.np, [&](int t) { return part_row<D>(x, r, t); }, M, L, acc);
  if (emit == kEmitFinish) {
    finish_row<D>(a, a.h_base + r.h, kind, r.g, M, L, acc);
  } else {
    const int lane = threadIdx.x & 31;
    const int64_t row = (int64_t)(r.h + x.c) * x.G + r.g;
    store_vec_cg<PL>(x.cpart_o + row * D + lane * PL, acc);
    if (lane == 0) {
      __stcg(&x.cpart_ml[row * 2], M);
      __stcg(&x.cpart_ml[row * 2 + 1], L);
    }
  }
}

template <typename T, int D, int GR>
__global__ void __launch_bounds__((max_consumers<D, GR>() + 1) * 32, 1)
stream_attend_kernel(const __grid_constant__ StreamArgs a) {
  constexpr int kSub = D / 64;                         // 64-column slices
  constexpr int kTile = kBS * 128;                     // one swizzled slice of a page
  constexpr uint32_t kStageBytes = 2 * kSub * kTile;   // K and V of one page
  constexpr int kRowChunks = D / 8;                    // 16-byte chunks per token row
  constexpr int kCopies = kBS * kRowChunks / 32;       // cp.async per lane per tensor and page

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ring = sm;
  int2* meta = reinterpret_cast<int2*>(sm + a.off_meta);
  int* stage_nt = reinterpret_cast<int*>(sm + a.off_snt);
  int* pref = reinterpret_cast<int*>(sm + a.off_pref);
  int* ctxv = reinterpret_cast<int*>(sm + a.off_ctx);
  uint8_t* kindv = sm + a.off_kind;
  uint32_t* span = reinterpret_cast<uint32_t*>(sm + a.off_span);  // first CTA << 16 | last CTA
  int* misc = reinterpret_cast<int*>(sm + a.off_misc);
  volatile int* vmisc = misc;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int NC = a.nc, S = a.stages, H = a.n_heads, G = a.G, MR = a.meta_cap;
  const int C = gridDim.x, c = blockIdx.x;
  const int nthreads = blockDim.x;

  uint64_t* qbar = reinterpret_cast<uint64_t*>(sm + a.off_qbar);
  T* qs = reinterpret_cast<T*>(sm + a.off_q);
  for (int i = tid; i < kMiscWords; i += nthreads) misc[i] = 0;
  if (tid == 0 && a.q_slots > 0) {
    mbar_init(qbar, 1);
    fence_mbar_init();
  }
  pdl_wait();

  // ---- head table: kind, context length and the exclusive prefix of w_h ----
  // (the decision word and both candidate counts are loaded together)
  const int dec = a.src_select == 2 ? a.decision[0] : 0;
  {
    const int per = (H + nthreads - 1) / nthreads;
    const int h0 = min(tid * per, H), h1 = min(h0 + per, H);
    int sum = 0, wmx = 0;
    long long att = 0, mx = 0;
    const int src = a.src_select == 2 ? ((dec & 1) ? 0 : 1) : a.src_select;
    for (int h = h0; h < h1; ++h) {
      const int bh = a.h_base + h;
      const int n0v = a.n0 ? a.n0[bh] : 0;
      const int n1v = a.n1 ? a.n1[bh] : 0;
      const int ctx = a.lens[bh / a.hkv];
      const int nv = min(n_valid_pages(ctx, kBS), a.W);
      int kind, w;
      if (a.dense) {
        kind = kKindRange;
        w = nv;
        att += nv;
      } else if (a.external_draft) {
        const bool rej = a.recover && a.accept[bh] == 0;
        kind = rej ? kKindRangeSkip : kKindEmpty;
        w = rej ? nv : 0;
      } else {
        const int ns = min(max(src ? n1v : n0v, 0), a.sel_stride);
        const bool rej = a.recover && src == 1 && a.accept[bh] == 0;
        if (rej && a.approx) {
          // backend.py:780-817: a rejected head's output is its expanded
          // selection alone (a superset of its draft)
          const int ne = min(max(a.exp_n[bh], 0), a.exp_stride);
          kind = kKindExp;
          w = ne;
          att += ne;
        } else {
          kind = rej ? kKindRange : kKindList;
          w = rej ? nv : ns;
          att += rej ? max(ns, nv) : ns;
        }
      }
      mx += nv;
      ctxv[h] = ctx;
      kindv[h] = (uint8_t)kind;
      pref[h] = w;
      sum += w;
      wmx = max(wmx, w);
    }
    if (c == 0 && a.counters) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        att += __shfl_xor_sync(0xffffffffu, att, o);
        mx += __shfl_xor_sync(0xffffffffu, mx, o);
      }
      if (lane == 0) {
        atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[CVSA_CTR_PAGES_ATTENDED]),
                  (unsigned long long)att);
        atomicAdd(reinterpret_cast<unsigned long long*>(&a.counters[CVSA_CTR_PAGES_MAX]),
                  (unsigned long long)mx);
      }
    }
    int total = 0;
    int base = block_excl_scan(sum, misc + kMiscScan, &total);
    if (wmx > 0) atomicMax(&misc[kMiscWmax], wmx);   // (misc is zeroed: the scan synced)
    for (int h = h0; h < h1; ++h) {
      const int w = pref[h];
      pref[h] = base;
      base += w;
    }
    if (tid == 0) pref[H] = total;
  }
  __syncthreads();
  const int src = a.src_select == 2 ? ((dec & 1) ? 0 : 1) : a.src_select;
  const int32_t* sel = src ? a.sel1 : a.sel0;
  // Committing the new selection and the gate of the decoded selection are
  // per-head copies with no readers in this launch: the producer warp does
  // them (spread over CTAs) once its descriptors are out.
  auto commit_heads = [&]() {
    if (!((a.commit && src == 1) || (a.accept_out && !a.dense))) return;
    for (int h = c; h < H; h += C) {
      const int bh = a.h_base + h;
      if (a.commit && src == 1) {
        const int ns = min(max(a.n1[bh], 0), a.sel_stride);
        const int64_t row = (int64_t)bh * a.sel_stride;
        for (int i = lane; i < ns; i += 32) a.commit_idx[row + i] = a.sel1[row + i];
        if (lane == 0) a.commit_n[bh] = ns;
      }
      if (lane == 0 && a.accept_out && !a.dense) {
        const uint8_t* ga = src == 1 ? a.acc1 : a.acc0;
        const float* gc = src == 1 ? a.cov1 : a.cov0;
        a.accept_out[bh] = ga ? ga[bh] : 1;
        if (a.cov_out) a.cov_out[bh] = gc ? gc[bh] : 1.f;
      }
    }
  };

  const int P = pref[H];
  // CTA c holds the stream positions [bnd[c], bnd[c + 1]): the equal cuts
  // P c / C or, when every head is short (at most kAlignMaxW pages and a CTA's
  // share: reuse steps with short selections), those cuts moved to the nearest
  // head start, so that no head is split over CTAs and the launch needs no
  // cross-CTA merge
  int* bnd = reinterpret_cast<int*>(sm + a.off_bnd);
  const int wmax = misc[kMiscWmax];
  const bool aligned = P > 0 && C <= kMaxBnd && wmax <= kAlignMaxW &&
                       (long long)wmax * C <= P;
  if (aligned) {
    for (int i = tid; i <= C; i += nthreads) {
      const int x = (int)((long long)P * i / C);
      int bi = x;
      if (i > 0 && i < C) {
        int lo = 0, hi = H - 1;  // largest h with pref[h] <= x
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (pref[mid] <= x) lo = mid;
          else hi = mid - 1;
        }
        const int s0 = pref[lo], s1 = pref[lo + 1];
        bi = (x - s0 <= s1 - x) ? s0 : s1;
      }
      bnd[i] = bi;
    }
    __syncthreads();
  }
  const int Xc = aligned ? bnd[c] : (int)((long long)P * c / C);
  const int Xe = aligned ? bnd[c + 1] : (int)((long long)P * (c + 1) / C);
  const int nloc = Xe - Xc;
  // first / last CTA that works on each head (an empty head belongs to the
  // CTA holding its position), computed once: position x lies in the last
  // CTA whose range starts at or before it (((x + 1) C - 1) / P for equal cuts)
  {
    auto cta_of = [&](int x) -> int {
      if (!aligned) return (int)(((long long)(x + 1) * C - 1) / P);
      int lo = 0, hi = C - 1;
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (bnd[mid] <= x) lo = mid;
        else hi = mid - 1;
      }
      return lo;
    };
    for (int h = tid; h < H; h += nthreads) {
      const int s0 = pref[h], w = pref[h + 1] - s0;
      const int f = s0 < P ? cta_of(s0) : C - 1;
      const int l = w > 0 ? cta_of(s0 + w - 1) : f;
      span[h] = ((uint32_t)f << 16) | (uint32_t)l;
    }
  }
  __syncthreads();
  auto first_cta = [&](int h) -> int { return (int)(span[h] >> 16); };
  auto last_cta = [&](int h) -> int { return (int)(span[h] & 0xffffu); };
  auto empty_head = [&](int h) -> bool { return pref[h + 1] == pref[h]; };
  // let the next kernel's CTAs be scheduled as this grid drains (it waits for
  // this grid's completion before reading anything it wrote)
  pdl_launch_dependents();

  const MergeCtx mctx{c, NC, nloc, G, a.part_o, a.part_ml, a.cpart_o, a.cpart_ml};
  // Empty heads (no pages) are finished from the empty state by CTA h % C,
  // one warp per query row.
  auto finish_empty_heads = [&]() {
    const int mine = c < H ? (H - 1 - c) / C + 1 : 0;
    for (int u = warp; u < mine * G; u += nthreads / 32) {
      const int h = c + (u / G) * C, g = u % G;
      if (empty_head(h))
        merge_emit<D>(a, mctx, RowSrc{0, h, g, 0, 0, 0, 0}, kEmitFinish, kindv[h]);
    }
  };
  if (P == 0) {
    finish_empty_heads();
    if (warp == NC) commit_heads();
    return;
  }
  // this CTA's heads: [hlo, hhi]
  int hlo, hhi;
  {
    int lo = 0, hi = H;  // first h with last_cta(h) >= c
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (last_cta(mid) >= c) hi = mid;
      else lo = mid + 1;
    }
    hlo = lo;
    lo = -1;
    hi = H - 1;  // last h with first_cta(h) <= c
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (first_cta(mid) <= c) lo = mid;
      else hi = mid - 1;
    }
    hhi = lo;
  }
  // stage the query rows of the first heads: a head switch then reads them
  // from shared memory instead of waiting behind the page stream in DRAM
  const int nq = hhi >= hlo ? min(hhi - hlo + 1, a.q_slots) : 0;
  const int q_elems = G * D;
  if (tid == 0 && nq > 0) {
    mbar_arrive_expect_tx(qbar, (uint32_t)(nq * q_elems * (int)sizeof(T)));
    const uint64_t qpol = make_evict_first_policy();
    for (int i = 0; i < nq; ++i) {
      const int bh = a.h_base + hlo + i;
      const T* src = reinterpret_cast<const T*>(a.q) +
                     ((int64_t)(bh / a.hkv) * a.hq + (int64_t)(bh % a.hkv) * G) * D;
      bulk_load(qs + (size_t)i * q_elems, src, (uint32_t)(q_elems * sizeof(T)), qbar, qpol);
    }
  }

  // Consumer k streams the contiguous local positions [slice(k), slice(k+1))
  // (sizes differ by at most one), so it meets few heads; they are handed out
  // in issue order j = k + q NC (its q-th position), which the producer
  // resolves in order.
  // (32-bit: P < 2^31, so nloc <= P / gridDim.x + 1 and nloc * NC < 2^31)
  auto slice_lo = [&](int kk) -> int { return nloc * kk / NC; };
  auto consumer_of = [&](int p) -> int { return ((p + 1) * NC - 1) / nloc; };
  const int qmax = (nloc + NC - 1) / NC;  // longest slice
  const int njobs = qmax * NC;

  if (warp == NC) {
    // ======================= page-descriptor producer =======================
    for (int xb = 0; xb < njobs; xb += 32) {
      const int j = xb + lane;  // issue index
      const int kk = j % NC, qq = j / NC;
      const int p = slice_lo(kk) + qq;  // local position
      int blk = -1, nt = 0;
      if (j < njobs && p < slice_lo(kk + 1)) {
        const int x = Xc + p;
        int lo = 0, hi = H - 1;  // largest h with pref[h] <= x (a non-empty head)
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (pref[mid] <= x) lo = mid;
          else hi = mid - 1;
        }
        const int h = lo;
        const int i = x - pref[h];
        const int bh = a.h_base + h;
        const int kind = kindv[h];
        int pg = i;
        bool ok = true;
        if (kind == kKindList || kind == kKindExp) {
          pg = kind == kKindList ? sel[(int64_t)bh * a.sel_stride + i]
                                 : a.exp_idx[(int64_t)bh * a.exp_stride + i];
          if (pg < 0 || pg >= a.W) {
            set_dev_error(a.dev_err, CVSA_DEV_ERR_PAGE_RANGE);
            ok = false;
          }
        } else if (kind == kKindRangeSkip) {
          const uint32_t word = a.bitmap[(int64_t)bh * a.bitmap_words + (pg >> 5)];
          ok = ((word >> (pg & 31)) & 1u) == 0;
        }
        if (ok) {
          const int ntok = min(kBS, ctxv[h] - pg * kBS);
          if (ntok > 0) {
            const int bk = a.tables[(int64_t)(bh / a.hkv) * a.W + pg];
            if (bk < 0 || bk >= a.num_blocks) {
              set_dev_error(a.dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
            } else {
              blk = bk;
              nt = ntok | ((bh % a.hkv) << 8);
            }
          }
        }
        // the ring entry is free once its previous index (same consumer) has
        // been read
        if (j >= MR && !spin_until_ge(vmisc + kMiscCons + kk, j - MR + 1, vmisc + kMiscFail, a.wait_polls)) {
          vmisc[kMiscFail] = 1;
          set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
        }
        meta[j % MR] = make_int2(blk, nt);
      }
      __threadfence_block();
      __syncwarp();
      if (lane == 0) vmisc[kMiscProd] = min(xb + 32, njobs);
      if (vmisc[kMiscFail]) break;
    }
    commit_heads();
  } else {

  // =============================== consumers ===============================
  const int k = warp;
  const int gq = lane >> 2, tq = lane & 3;
  const uint64_t policy = make_evict_first_policy();
  uint8_t* myring = ring + (size_t)k * S * kStageBytes;
  int* mynt = stage_nt + k * S;
  const T* Kp = reinterpret_cast<const T*>(a.k);
  const T* Vp = reinterpret_cast<const T*>(a.v);
  // lane's 16-byte chunk of copy r: token r * kTPI + lane / kRowChunks,
  // chunk lane % kRowChunks (global offset), swizzled into its stage row
  constexpr int kTPI = 32 / kRowChunks;  // tokens per copy instruction
  const int64_t lane_goff = (int64_t)(lane / kRowChunks) * a.st + (lane % kRowChunks) * 8;
  const int64_t step_goff = (int64_t)kTPI * a.st;
  uint32_t soffs[kCopies];
#pragma unroll
  for (int r = 0; r < kCopies; ++r) {
    const int t = r * kTPI + lane / kRowChunks, c16 = lane % kRowChunks;
    soffs[r] = (c16 >> 3) * kTile + t * 128 + (((c16 & 7) ^ (t & 7)) << 4);
  }

  // copy the page of my q-th position into stage q % S (a group is committed
  // even when nothing is copied, so group counting stays uniform); the
  // descriptor is {block, tokens | kv head << 8}
  const int my_lo = slice_lo(k), nmine = slice_lo(k + 1) - my_lo;
  auto issue = [&](int q) -> bool {
    const int j = k + q * NC;
    if (q < nmine) {
      if (lane == 0 && !spin_until_ge(vmisc + kMiscProd, j + 1, vmisc + kMiscFail, a.wait_polls)) {
        vmisc[kMiscFail] = 1;
        set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
      }
      __syncwarp();
      if (vmisc[kMiscFail]) return false;
      const int2 e = meta[j % MR];
      if (lane == 0) mynt[q % S] = e.y & 0xff;
      if ((e.y & 0xff) > 0) {
        const int hh = e.y >> 8;
        const int64_t gbase = (int64_t)e.x * a.sb + (int64_t)hh * a.sh + lane_goff;
        const T* kr = Kp + gbase;
        const T* vr = Vp + gbase;
        const uint32_t sbase = smem_u32(myring + (size_t)(q % S) * kStageBytes);
#pragma unroll
        for (int r = 0; r < kCopies; ++r) {
          cp_async16(sbase + soffs[r], kr + r * step_goff, policy);
          cp_async16(sbase + kSub * kTile + soffs[r], vr + r * step_goff, policy);
        }
      }
      // the descriptor has been consumed (the copies above used it): hand its
      // ring entry back to the producer
      __syncwarp();
      if (lane == 0) vmisc[kMiscCons + k] = j + NC;
    }
    cp_async_commit();
    return true;
  };

  // Running state of the current head in the transposed layout: O^T
  // (head_dim x query rows) as m16n8 accumulators, lane (gq, tq) holding
  // columns d = 16 mt + gq (+8) of query rows g = 8 n + 2 tq (+1); the
  // reference max m_use the state is scaled by (uniform over the 8 lanes of a
  // row), this lane's own max of the row's scores and its share of the row
  // sum (both combined over the lanes when the head is flushed).
  float o[D / 16][GR][4];
  float m_use[GR][2], m_loc[GR][2], l_part[GR][2];
  uint32_t qb[D / 16][GR][2];
  auto reset_state = [&]() {
#pragma unroll
    for (int mt = 0; mt < D / 16; ++mt)
#pragma unroll
      for (int n = 0; n < GR; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) o[mt][n][i] = 0.f;
#pragma unroll
    for (int n = 0; n < GR; ++n)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        m_use[n][i] = neg_inf();
        m_loc[n][i] = neg_inf();
        l_part[n][i] = 0.f;
      }
  };
  // Q^T as the B operand of S^T = K Q^T: b0 = Q[g][16 ks + 2 tq ..], b1 = +8,
  // from the staged copy where there is one
  bool q_staged = false;
  auto load_q = [&](int h) -> bool {
    const T* qp;
    if (h - hlo < nq) {
      if (!q_staged) {
        if (!mbar_wait_bounded(qbar, 0, a.wait_polls)) {
          vmisc[kMiscFail] = 1;
          set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
          return false;
        }
        q_staged = true;
      }
      qp = qs + (size_t)(h - hlo) * q_elems;
    } else {
      const int bh = a.h_base + h;
      const int b = bh / a.hkv, hh = bh % a.hkv;
      qp = reinterpret_cast<const T*>(a.q) + ((int64_t)b * a.hq + (int64_t)hh * G) * D;
    }
#pragma unroll
    for (int n = 0; n < GR; ++n) {
      const int g = n * 8 + gq;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t lo = 0, hi = 0;
        if (g < G) {
          lo = *reinterpret_cast<const uint32_t*>(qp + (int64_t)g * D + ks * 16 + tq * 2);
          hi = *reinterpret_cast<const uint32_t*>(qp + (int64_t)g * D + ks * 16 + 8 + tq * 2);
        }
        qb[ks][n][0] = lo;
        qb[ks][n][1] = hi;
      }
    }
    return true;
  };

  // Write the state of head h as this consumer's partial, rescaled from the
  // reference max m_use to the exact row max (f <= 1). Empty heads have no
  // partials.
  auto flush_head = [&](int h) {
    if (empty_head(h)) return;
    const int64_t slot = partial_slot(h, c, k, NC);
#pragma unroll
    for (int n = 0; n < GR; ++n)
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int g = n * 8 + tq * 2 + i;
        float mx = m_loc[n][i];
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        const float f = (m_use[n][i] == neg_inf()) ? 0.f : softmax_exp(m_use[n][i] - mx);
        float lsum = l_part[n][i];
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 4);
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 8);
        lsum += __shfl_xor_sync(0xffffffffu, lsum, 16);
        if (g < G) {
          float* po = a.part_o + (slot * G + g) * D;
#pragma unroll
          for (int mt = 0; mt < D / 16; ++mt) {
            __stcg(&po[mt * 16 + gq], o[mt][n][i] * f);
            __stcg(&po[mt * 16 + gq + 8], o[mt][n][2 + i] * f);
          }
          if (gq == 0) {
            __stcg(&a.part_ml[(slot * G + g) * 2], mx);
            __stcg(&a.part_ml[(slot * G + g) * 2 + 1], lsum * f);
          }
        }
      }
  };

  // ---- main loop over my positions ----
  bool ok = true;
  for (int q = 0; q < S - 1 && ok; ++q) ok = issue(q);
  int h = hlo;  // the head of my first position (a non-empty head)
  if (nmine > 0) {
    int lo = hlo, hi = hhi;
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (pref[mid] <= Xc + my_lo) lo = mid;
      else hi = mid - 1;
    }
    h = lo;
  }
  bool have_q = false;
  reset_state();
  for (int q = 0; q < nmine && ok; ++q) {
    ok = issue(q + S - 1);
    if (!ok) break;
    const int x = Xc + my_lo + q;
    while (x >= pref[h + 1]) {  // heads that end before x are done for me
      flush_head(h);
      ++h;
      have_q = false;
      reset_state();
    }
    if (!have_q) {
      if (!load_q(h)) break;
      have_q = true;
    }
    cp_async_wait_dyn(S - 1);
    __syncwarp();
    const int st = q % S;
    const int nt = mynt[st];
    if (nt > 0) {
      const uint32_t kbase = smem_u32(myring + (size_t)st * kStageBytes);
      const uint32_t vbase = kbase + kSub * kTile;
      // ---- S^T = K Q^T: M = the page's 16 tokens, N = query rows, two k-chains ----
      float sa[GR][4], sb[GR][4];
#pragma unroll
      for (int n = 0; n < GR; ++n)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          sa[n][i] = 0.f;
          sb[n][i] = 0.f;
        }
      {
        const int tok = (lane & 7) + ((lane >> 3) & 1) * 8;
        const int chsel = (lane >> 4) & 1;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const int sub = ks >> 2;
          const int ch = (ks & 3) * 2 + chsel;
          uint32_t af[4];
          ldmatrix_x4(af[0], af[1], af[2], af[3],
                      kbase + sub * kTile + tok * 128 + ((ch ^ (tok & 7)) << 4));
#pragma unroll
          for (int n = 0; n < GR; ++n) {
            if (ks & 1) Mma<T>::m16n8k16(sb[n], af, qb[ks][n][0], qb[ks][n][1]);
            else Mma<T>::m16n8k16(sa[n], af, qb[ks][n][0], qb[ks][n][1]);
          }
        }
      }
      // ---- online softmax: lane holds tokens gq, gq + 8 of rows 8n + 2tq (+1) ----
      // p = exp(s - m_use). The reference max m_use is raised, and the state
      // rescaled, only when a score passes it by more than kRescaleGap, so
      // p <= e^kRescaleGap and most pages need neither the row-max shuffles
      // nor the rescale; flush_head moves the state to the exact row max.
      const bool v0 = gq < nt, v1 = gq + 8 < nt;
      float xs[GR][4];
      bool grow = false;
#pragma unroll
      for (int n = 0; n < GR; ++n)
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float x0 = v0 ? (sa[n][i] + sb[n][i]) * a.scale : neg_inf();
          const float x1 = v1 ? (sa[n][2 + i] + sb[n][2 + i]) * a.scale : neg_inf();
          xs[n][i] = x0;
          xs[n][2 + i] = x1;
          const float lm = fmaxf(x0, x1);
          m_loc[n][i] = fmaxf(m_loc[n][i], lm);
          grow |= lm > m_use[n][i] + kRescaleGap;
        }
      if (__any_sync(0xffffffffu, grow)) {
#pragma unroll
        for (int n = 0; n < GR; ++n)
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            float mx = fmaxf(xs[n][i], xs[n][2 + i]);
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
            const float mnew = fmaxf(m_use[n][i], mx);
            if (mnew != m_use[n][i]) {
              const float alpha =
                  (m_use[n][i] == neg_inf()) ? 0.f : softmax_exp(m_use[n][i] - mnew);
              l_part[n][i] *= alpha;
#pragma unroll
              for (int mt = 0; mt < D / 16; ++mt) {
                o[mt][n][i] *= alpha;
                o[mt][n][2 + i] *= alpha;
              }
              m_use[n][i] = mnew;
            }
          }
      }
      uint32_t pb[GR][2];
#pragma unroll
      for (int n = 0; n < GR; ++n) {
        float p[4];
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float mu = m_use[n][i];
          const float p0 = (mu == neg_inf() || !v0) ? 0.f : softmax_exp(xs[n][i] - mu);
          const float p1 = (mu == neg_inf() || !v1) ? 0.f : softmax_exp(xs[n][2 + i] - mu);
          l_part[n][i] += p0 + p1;
          p[i] = p0;
          p[2 + i] = p1;
        }
        // P^T as the B operand: transpose the 8x8 token-by-row fragments
        pb[n][0] = movmatrix_trans(Mma<T>::pack(p[0], p[1]));
        pb[n][1] = movmatrix_trans(Mma<T>::pack(p[2], p[3]));
      }
      // ---- O^T += V^T P^T: M = 16 head_dim columns per tile, K = the 16 tokens ----
      {
        const int tok = (lane & 7) + ((lane >> 4) & 1) * 8;
        const int chsel = (lane >> 3) & 1;
#pragma unroll
        for (int mt = 0; mt < D / 16; ++mt) {
          const int sub = mt >> 2;
          const int ch = (mt & 3) * 2 + chsel;
          uint32_t af[4];
          ldmatrix_x4_trans(af[0], af[1], af[2], af[3],
                            vbase + sub * kTile + tok * 128 + ((ch ^ (tok & 7)) << 4));
#pragma unroll
          for (int n = 0; n < GR; ++n) Mma<T>::m16n8k16(o[mt][n], af, pb[n][0], pb[n][1]);
        }
      }
    }
    __syncwarp();  // the stage is refilled by the next issue
  }
  // the head of my last position is done for me
  if (ok && nmine > 0) flush_head(h);
  // no copy may still be landing in shared memory past this point (the
  // partials are read by this CTA only, after the barrier below)
  asm volatile("cp.async.wait_all;" ::: "memory");
  }  // consumers
  // the staged query rows have landed even if no consumer read them (no
  // bulk copy may outlive the CTA)
  if (tid == 0 && nq > 0 && !mbar_wait_bounded(qbar, 0)) {
    vmisc[kMiscFail] = 1;
    set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
  }

  // ============================ finish the heads ============================
  // Every warp is done streaming (no copies in flight): the partials written
  // by this CTA's consumers are visible to the whole CTA after the barrier.
  __syncthreads();
  if (vmisc[kMiscFail]) return;  // a copy never arrived: leave the outputs alone
  // Merges, one warp per query row. A head split over CTAs (only this CTA's
  // first and last head can be) is first merged over this CTA's consumers
  // into one CTA partial (slot head + CTA); the last of its CTAs to get here
  // (ticket per head, no spin) merges the CTA partials in CTA order. The
  // split heads' CTA partials are written first, so thread 0's tickets are in
  // flight while the other warps merge and finish the heads inside the range.
  auto split_head = [&](int i) -> int {  // this CTA's first (0) / last (1) head if split
    const int h = i == 0 ? hlo : hhi;
    if (hlo > hhi || (i == 1 && hhi == hlo) || empty_head(h) || first_cta(h) == last_cta(h))
      return -1;
    return h;
  };
  const int sh0 = split_head(0), sh1 = split_head(1);
  const int nwarps = nthreads / 32;
  // The consumers whose slices meet head h (a non-empty head of this CTA):
  // consumer_of(p0) .. consumer_of(p1 - 1) when every slice is non-empty
  // (nloc >= NC); otherwise each non-empty slice is one position, and the
  // t-th partial is that of position p0 + t.
  auto cons_src = [&](int h, int g) -> RowSrc {
    const int p0 = max(pref[h], Xc) - Xc, p1 = min(pref[h + 1], Xe) - Xc;
    const int kf = consumer_of(p0);
    const int np = nloc >= NC ? consumer_of(p1 - 1) - kf + 1 : p1 - p0;
    return RowSrc{0, h, g, np, kf, p0, 0};
  };
  for (int u = warp; u < 2 * G; u += nwarps) {
    const int h = u < G ? sh0 : sh1, g = u % G;
    if (h < 0) continue;
    merge_emit<D>(a, mctx, cons_src(h, g), kEmitCtaPartial, kindv[h]);
  }
  // Tickets: the barrier orders every warp's CTA-partial stores before
  // thread 0's fence, which publishes them before its ticket (both tickets in
  // flight together); the winner's fence orders the other CTAs' partials
  // before its reads.
  __syncthreads();
  int* won = misc + kMiscWon;
  if (warp == 0) {
    if (tid == 0) {
      won[0] = won[1] = 0;
      if (sh0 >= 0 || sh1 >= 0) {
        __threadfence();
        const int t0 = sh0 >= 0 ? atomicAdd(&a.head_done[a.h_base + sh0], 1) : -1;
        const int t1 = sh1 >= 0 ? atomicAdd(&a.head_done[a.h_base + sh1], 1) : -1;
        if (sh0 >= 0 && t0 == last_cta(sh0) - first_cta(sh0)) {
          won[0] = 1;
          a.head_done[a.h_base + sh0] = 0;
        }
        if (sh1 >= 0 && t1 == last_cta(sh1) - first_cta(sh1)) {
          won[1] = 1;
          a.head_done[a.h_base + sh1] = 0;
        }
        if (won[0] | won[1]) __threadfence();
      }
    }
  } else {
    // heads inside this CTA's range: merge over the consumers and finish
    const int nrow = (hhi - hlo + 1) * G;
    for (int u = warp - 1; u < nrow; u += nwarps - 1) {
      const int h = hlo + u / G, g = u % G;
      if (h == sh0 || h == sh1 || empty_head(h)) continue;
      merge_emit<D>(a, mctx, cons_src(h, g), kEmitFinish, kindv[h]);
    }
  }
  __syncthreads();
  for (int u = warp; u < 2 * G; u += nwarps) {
    const int i = u / G, g = u % G;
    if (!won[i]) continue;
    const int h = i == 0 ? hlo : hhi;
    const int fc = first_cta(h);
    merge_emit<D>(a, mctx, RowSrc{1, h, g, last_cta(h) - fc + 1, 0, 0, fc}, kEmitFinish,
                  kindv[h]);
  }
  finish_empty_heads();
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
struct Plan {
  int nc, stages, meta_cap, smem;
  int off_meta, off_snt, off_pref, off_ctx, off_kind, off_span, off_misc, off_bnd;
};

size_t up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Shared-memory plan for a launch of n_heads heads: the consumer count and
// per-consumer ring depth that keep the most pages in flight (ties go to more
// consumers).
bool make_plan(int D, int n_heads, int max_nc, Plan* best) {
  const size_t stage = (size_t)2 * (D / 64) * kBS * 128;
  bool found = false;
  int best_score = 0;
  for (int nc = max_nc; nc >= 2; --nc) {
    Plan p;
    const int meta_cap = kMetaPerConsumer * nc;
    const size_t tail = up((size_t)meta_cap * 8, 16) + up((size_t)nc * kMaxStages * 4, 16) +
                        up((size_t)(n_heads + 1) * 4, 16) + up((size_t)n_heads * 4, 16) +
                        up((size_t)n_heads, 16) + up((size_t)n_heads * 4, 16) + kMiscWords * 4 +
                        up((size_t)(kMaxBnd + 1) * 4, 16);
    const size_t avail = (size_t)kSmemCap - 1024;  // alignment slack of the dynamic base
    if (avail <= tail) continue;
    int stages = (int)((avail - tail) / (stage * nc));
    if (stages > kMaxStages) stages = kMaxStages;
    if (stages < 2) continue;
    size_t off = (size_t)nc * stages * stage;
    p.off_meta = (int)off; off += up((size_t)meta_cap * 8, 16);
    p.off_snt = (int)off; off += up((size_t)nc * stages * 4, 16);
    p.off_pref = (int)off; off += up((size_t)(n_heads + 1) * 4, 16);
    p.off_ctx = (int)off; off += up((size_t)n_heads * 4, 16);
    p.off_kind = (int)off; off += up((size_t)n_heads, 16);
    p.off_span = (int)off; off += up((size_t)n_heads * 4, 16);
    p.off_misc = (int)off; off += kMiscWords * 4;
    p.off_bnd = (int)off; off += up((size_t)(kMaxBnd + 1) * 4, 16);
    if (off + 1024 > (size_t)kSmemCap) continue;
    p.nc = nc;
    p.stages = stages;
    p.meta_cap = meta_cap;
    p.smem = (int)(off + 1024);
    // three stages keep two pages in flight per consumer while it computes
    // one; past that, more consumers beat deeper rings
    const int score = nc * (stages < 3 ? stages : 3) * 16 + nc * stages;
    if (!found || score > best_score) {
      *best = p;
      best_score = score;
      found = true;
    }
  }
  return found;
}

template <typename T, int D, int GR>
cudaError_t launch_typed(StreamArgs& a, cudaStream_t s, bool pdl) {
  Plan pl;
  if (!make_plan(D, a.n_heads, max_consumers<D, GR>(), &pl)) return cudaErrorInvalidValue;
  a.nc = pl.nc;
  a.stages = pl.stages;
  a.meta_cap = pl.meta_cap;
  a.off_meta = pl.off_meta;
  a.off_snt = pl.off_snt;
  a.off_pref = pl.off_pref;
  a.off_ctx = pl.off_ctx;
  a.off_kind = pl.off_kind;
  a.off_span = pl.off_span;
  a.off_misc = pl.off_misc;
  a.off_bnd = pl.off_bnd;
  // query-row staging in the shared memory the plan leaves over
  {
    const size_t qbytes = (size_t)a.G * D * sizeof(T);
    size_t off = up((size_t)pl.smem - 1024, 16);
    a.off_qbar = (int)off;
    off += 16;
    a.off_q = (int)off;
    int slots = 0;
    const bool q_aligned = (reinterpret_cast<uintptr_t>(a.q) & 15) == 0 && qbytes % 16 == 0;
    if (q_aligned && off + qbytes + 1024 <= (size_t)kSmemCap)
      slots = (int)(((size_t)kSmemCap - 1024 - off) / qbytes);
    a.q_slots = slots < kMaxQSlots ? slots : kMaxQSlots;
    pl.smem = (int)(off + (size_t)a.q_slots * qbytes + 1024);
  }
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(stream_attend_kernel<T, D, GR>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemCap);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  return launch_k(stream_attend_kernel<T, D, GR>, dim3(a.grid), dim3((pl.nc + 1) * 32),
                  (size_t)pl.smem, s, pdl, a);
}

template <typename T>
cudaError_t dispatch(StreamArgs& a, int d, cudaStream_t s, bool pdl) {
  const bool g2 = a.G > 8;
  switch (d) {
    case 64: return g2 ? launch_typed<T, 64, 2>(a, s, pdl) : launch_typed<T, 64, 1>(a, s, pdl);
    case 128: return g2 ? launch_typed<T, 128, 2>(a, s, pdl) : launch_typed<T, 128, 1>(a, s, pdl);
    case 256: return g2 ? launch_typed<T, 256, 2>(a, s, pdl) : launch_typed<T, 256, 1>(a, s, pdl);
  }
  return cudaErrorInvalidValue;
}

// Heads per launch: the shared-memory head table holds up to kMaxChunkHeads,
// the stream length of one launch stays within int32, and the partial scratch
// of one launch stays within kMaxPartialBytes.
constexpr size_t kMaxPartialBytes = (size_t)64 << 20;

size_t partial_bytes_per_slot(int G, int D) { return (size_t)G * (D + 2) * 4; }

int chunk_heads(const QView& q, const KvView& kv, int max_sel) {
  const long long per = (long long)(q.W > max_sel ? q.W : max_sel) + 1;
  long long ch = (long long)INT_MAX / per;
  if (ch > kMaxChunkHeads) ch = kMaxChunkHeads;
  const int G = q.hq / kv.hkv;
  const long long slots_cap =
      (long long)(kMaxPartialBytes / partial_bytes_per_slot(G, kv.d)) /
          max_consumers_rt(kv.d, G) - num_sms();
  if (ch > slots_cap) ch = slots_cap;
  return ch < 1 ? 1 : (int)ch;
}

// Partial scratch for launches of `chunk` heads: every (head, CTA) pair of a
// launch is at most chunk + gridDim.x - 1, times the consumer count.
struct PartialLayout {
  size_t o, ml, co, cml, total;
};
PartialLayout partial_layout(const QView& q, const KvView& kv, int chunk) {
  const int G = q.hq / kv.hkv;
  const size_t slots = (size_t)(chunk + num_sms()) * max_consumers_rt(kv.d, G);
  PartialLayout L;
  size_t off = 0;
  L.o = off; off += up(slots * G * kv.d * 4, 256);
  L.ml = off; off += up(slots * G * 2 * 4, 256);
  const size_t cslots = (size_t)chunk + num_sms();
  L.co = off; off += up(cslots * G * kv.d * 4, 256);
  L.cml = off; off += up(cslots * G * 2 * 4, 256);
  L.total = off;
  return L;
}

}  // namespace

bool stream_attend_eligible(const QView& q, const KvView& kv) {
  return (kv.dtype == CVSA_DTYPE_BF16 || kv.dtype == CVSA_DTYPE_F16) && q.dtype == kv.dtype &&
         kv.bs == kBS && (kv.d == 64 || kv.d == 128 || kv.d == 256) && kv.hkv > 0 &&
         q.hq % kv.hkv == 0 && (q.hq / kv.hkv) <= 16 && ((kv.sh * 2) % 16 == 0) &&
         ((kv.st * 2) % 16 == 0) && ((kv.sb * 2) % 16 == 0) &&
         (reinterpret_cast<uintptr_t>(kv.k) % 16 == 0) &&
         (reinterpret_cast<uintptr_t>(kv.v) % 16 == 0);
}

size_t stream_attend_workspace_bytes(const QView& q, const KvView& kv, int max_sel) {
  const int heads = q.B * kv.hkv;
  int chunk = chunk_heads(q, kv, max_sel);
  if (chunk > heads) chunk = heads < 1 ? 1 : heads;
  return partial_layout(q, kv, chunk).total;
}

cudaError_t launch_stream_attend(const QView& q, const KvView& kv, const AttendParams& p,
                                 int max_sel, cudaStream_t s, bool pdl) {
  StreamArgs a;
  memset(&a, 0, sizeof(a));
  const int heads = q.B * kv.hkv;
  if (heads <= 0) return cudaSuccess;
  if (heads > kMaxHeadsPerCall) return cudaErrorInvalidValue;
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
  a.external_draft = p.external_draft ? 1 : 0;
  a.accept = p.accept;
  a.bitmap = p.bitmap;
  a.bitmap_words = p.bitmap_words;
  a.ext_o = p.ext_o;
  a.ext_m = p.ext_m;
  a.ext_l = p.ext_l;
  a.approx = p.approx ? 1 : 0;
  a.exp_idx = p.exp_idx;
  a.exp_n = p.exp_n;
  a.exp_stride = p.exp_stride;
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
  a.scale = 1.0f / sqrtf((float)kv.d);
  a.wait_polls = wait_limit() ? wait_limit() : kSpinLimit;
  int chunk = chunk_heads(q, kv, p.dense ? 1 : max_sel);
  if (chunk > heads) chunk = heads;
  const PartialLayout L = partial_layout(q, kv, chunk);
  if (p.partial_bytes < L.total) return cudaErrorInvalidValue;
  uint8_t* base = reinterpret_cast<uint8_t*>(p.partials);
  a.part_o = reinterpret_cast<float*>(base + L.o);
  a.part_ml = reinterpret_cast<float*>(base + L.ml);
  a.cpart_o = reinterpret_cast<float*>(base + L.co);
  a.cpart_ml = reinterpret_cast<float*>(base + L.cml);
  a.head_done = p.head_done;
  // A launch whose stream is short (a bound known on the host: every head's
  // list width, or its table width when it may read every valid page) runs
  // on fewer CTAs, each with at least kMinPagesPerCta pages: the per-CTA
  // start-up and the cross-CTA merges cost more than the SMs left idle
  // (measured: 840 page-heads, 17.5 us on 148 CTAs, 14.2 us on 64).
  const int width = (p.dense || p.recover) ? q.W
                    : (p.approx && p.exp_stride > max_sel ? p.exp_stride : max_sel);
  for (int h0 = 0; h0 < heads; h0 += chunk) {
    a.h_base = h0;
    a.n_heads = heads - h0 < chunk ? heads - h0 : chunk;
    const long long bound = (long long)a.n_heads * width;
    const int sms = num_sms();
    a.grid = bound < (long long)sms * kMinPagesPerCta
                 ? (int)((bound + kMinPagesPerCta - 1) / kMinPagesPerCta)
                 : sms;
    if (a.grid < 1) a.grid = 1;
    cudaError_t e = kv.dtype == CVSA_DTYPE_BF16 ? dispatch<__nv_bfloat16>(a, kv.d, s, pdl)
                                                : dispatch<__half>(a, kv.d, s, pdl);
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace cvsa
