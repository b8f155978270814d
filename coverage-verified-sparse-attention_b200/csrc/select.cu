// Top-k page selection + coverage gate per (sequence b, kv head h).
//
// Restates, for one (b, h) row of page scores:
//   * cvsa/backend.py:690,737-747 -- the top `budget` pages by score, with
//     n_per_head = min(budget, n_valid); here the order is (score desc, page
//     index asc) and the first `sink` / last `local` valid pages are forced in
//     (both off by default);
//   * cvsa/kernels/coverage.py:160-215 -- cov = exp(lse(scores[sel]) -
//     lse(scores[all W pages])), max seeded with -1e20, log(sum + 1e-30),
//     accept = cov >= tau; the selected scores are summed over the list
//     entries, as the reference gathers them;
//   * cvsa/backend.py:424-446 -- in lazy mode, the same gate on the CACHED
//     selection, reduced over the whole batch on the device (the reference's
//     host-side accept_mask.all()) by the last CTA to finish.
// The k-th largest score is found exactly on order-preserving 32-bit keys;
// ties at that key go to the lowest page indices through a prefix count, and
// the selection is written in ascending page order with a bitmap of it (read
// by the fused recovery kernel to skip selected pages). Two variants:
//   * tables of up to 1024 pages: one WARP per (b, h), scores in registers
//     (lane l owns a contiguous run of pages), the threshold by a 32-step
//     bisection on the key (one warp reduction per step), no block barriers;
//   * longer tables: one CTA per (b, h), scores in shared memory, a 4-pass
//     8-bit radix select with warp-aggregated shared histograms.
// Both finish with the batch-global decision and, for the attention kernel,
// the exclusive scan of each head's complement-item count (rejected heads
// only), taken by the last CTA to finish: no host synchronisation.
#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

template <int NT>
struct BlockScan {
  static constexpr int NWARP = NT / 32;
  // exclusive prefix sum of `v` across the block (thread order), plus total.
  __device__ static int exclusive(int v, int* wsum, int& total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) wsum[w] = x;
    __syncthreads();
    if (w == 0) {
      int t = lane < NWARP ? wsum[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t += y;
      }
      if (lane < NWARP) wsum[lane] = t;  // inclusive warp prefix
    }
    __syncthreads();
    const int before = (w == 0 ? 0 : wsum[w - 1]);
    total = wsum[NWARP - 1];
    const int excl = before + x - v;
    __syncthreads();
    return excl;
  }
};

__device__ __forceinline__ int warp_excl_scan(int v, int& total) {
  const int lane = threadIdx.x & 31;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  total = __shfl_sync(0xffffffffu, x, 31);
  return x - v;
}

template <int NT>
__device__ float block_reduce_max(float v, float* red) {
  v = warp_max(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) red[w] = v;
  __syncthreads();
  float r = -3.402823466e38f;
  if (threadIdx.x < 32) {
    r = (lane < NT / 32) ? red[lane] : neg_inf();
    r = warp_max(r);
    if (lane == 0) red[32] = r;
  }
  __syncthreads();
  r = red[32];
  __syncthreads();
  return r;
}

template <int NT>
__device__ float block_reduce_sum(float v, float* red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  if (lane == 0) red[w] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float r = (lane < NT / 32) ? red[lane] : 0.f;
    r = warp_sum(r);
    if (lane == 0) red[32] = r;
  }
  __syncthreads();
  float r = red[32];
  __syncthreads();
  return r;
}

// log-sum-exp over the selected entries of s[] (flagged), reference form.
template <int NT>
__device__ float lse_flagged(const float* s, const uint8_t* flag, int W, float* red) {
  float m = -1e20f;
  for (int i = threadIdx.x; i < W; i += NT)
    if (flag[i]) m = fmaxf(m, s[i]);
  m = block_reduce_max<NT>(m, red);
  m = fmaxf(m, -1e20f);
  float sum = 0.f;
  for (int i = threadIdx.x; i < W; i += NT)
    if (flag[i]) sum += expf(s[i] - m);
  sum = block_reduce_sum<NT>(sum, red);
  return m + logf(sum + 1e-30f);
}

// log-sum-exp over the entries of an index list (duplicates count, like the
// reference's gather at coverage.py:196-204); warp-cooperative.
__device__ __forceinline__ float lse_list_warp(const float* row, int W, const int32_t* idx,
                                               int n) {
  const int lane = threadIdx.x & 31;
  float m = -1e20f;
  for (int i = lane; i < n; i += 32) {
    const int pg = idx[i];
    if (pg >= 0 && pg < W) m = fmaxf(m, row[pg]);
  }
  m = fmaxf(warp_max(m), -1e20f);
  float sum = 0.f;
  for (int i = lane; i < n; i += 32) {
    const int pg = idx[i];
    if (pg >= 0 && pg < W) sum += expf(row[pg] - m);
  }
  sum = warp_sum(sum);
  return m + logf(sum + 1e-30f);
}

// lse_list_warp over a shared-memory copy of the row; the first 256 list
// entries are loaded in one round (8 per lane), longer lists in further rounds.
__device__ __forceinline__ float lse_list_smem(const float* srow, int W, const int32_t* idx, int n) {
  constexpr int kPer = 8;
  const int lane = threadIdx.x & 31;
  auto val = [&](int pg) -> float { return (pg >= 0 && pg < W) ? srow[pg] : neg_inf(); };
  float v[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = lane + 32 * j;
    v[j] = i < n ? val(idx[i]) : neg_inf();
  }
  float m = neg_inf();
#pragma unroll
  for (int j = 0; j < kPer; ++j) m = fmaxf(m, v[j]);
  for (int i = lane + 32 * kPer; i < n; i += 32) m = fmaxf(m, val(idx[i]));
  m = fmaxf(warp_max(m), -1e20f);
  float sum = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j)
    if (v[j] != neg_inf()) sum += expf(v[j] - m);
  for (int i = lane + 32 * kPer; i < n; i += 32) {
    const float x = val(idx[i]);
    if (x != neg_inf()) sum += expf(x - m);
  }
  sum = warp_sum(sum);
  return m + logf(sum + 1e-30f);
}

__device__ __forceinline__ void count_head(const SelectParams& p, bool acc) {
  if (!p.counters) return;
  atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_ACCEPT]),
            (unsigned long long)(acc ? 1 : 0));
  atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_TOTAL]), 1ull);
}

// Last-CTA epilogue shared by both variants: batch-global decision, step
// statistics, flags, and the exclusive scan of the complement-item counts.
// Every thread of every CTA calls it; `cta_rejects` is read in thread 0.
// The two sync words form one 64-bit counter (CTAs done in the low half,
// rejected heads in the high half), so one atomic both reports this CTA and
// tells the last one the batch's reject count.
template <int NT>
__device__ void finish_select(const SelectParams& p, int cta_rejects, int* s_flag, int* wsum) {
  if (!p.sync_ctr) return;
  unsigned long long* ctr = reinterpret_cast<unsigned long long*>(p.sync_ctr);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();  // this thread's comp_cnt before the count
    const unsigned long long old =
        atomicAdd(ctr, 1ull | ((unsigned long long)(unsigned)cta_rejects << 32));
    const bool last = (int)(uint32_t)old == (int)gridDim.x - 1;
    s_flag[0] = last ? 1 : 0;
    if (last) {
      const int rejects = (int)(old >> 32) + cta_rejects;
      int all_accept;
      if (p.mode == CVSA_MODE_LAZY) {
        all_accept = (p.has_cache && rejects == 0) ? 1 : 0;
      } else {
        all_accept = (rejects == 0) ? 1 : 0;
      }
      if (p.decision) p.decision[0] = all_accept;
      if (p.counters) {
        unsigned long long* c = reinterpret_cast<unsigned long long*>(p.counters);
        if (p.mode == CVSA_MODE_LAZY) {
          atomicAdd(&c[CVSA_CTR_COVERAGE_CHECKS], 1ull);
          if (all_accept) {
            atomicAdd(&c[CVSA_CTR_ACCEPT_STEPS], 1ull);
          } else {
            atomicAdd(&c[CVSA_CTR_REJECT_STEPS], 1ull);
            atomicAdd(&c[CVSA_CTR_SCORING_STEPS], 1ull);
          }
        } else {
          atomicAdd(&c[CVSA_CTR_SCORING_STEPS], 1ull);
          if (!p.lazy_stats)
            atomicAdd(&c[all_accept ? CVSA_CTR_ACCEPT_STEPS : CVSA_CTR_REJECT_STEPS], 1ull);
        }
      }
      if (p.step_flags) {
        int fl = 0;
        if (p.mode == CVSA_MODE_LAZY) fl = all_accept ? 1 : 2;
        else fl = (all_accept ? 1 : 0) | 2;
        p.step_flags[0] = fl;
      }
      s_flag[1] = all_accept;
      *ctr = 0ull;  // ready for the next launch (no other CTA touches it now)
    }
  }
  __syncthreads();
  if (!s_flag[0] || !p.comp_off) return;
  __threadfence();  // the other CTAs' comp_cnt
  const int heads = p.B * p.hkv;
  const bool reuse = (p.mode == CVSA_MODE_LAZY) && s_flag[1] && !p.decision_external;
  int carry = 0;
  for (int base = 0; base < heads; base += NT) {
    const int i = base + threadIdx.x;
    const int v = (i < heads && !reuse) ? __ldcg(&p.comp_cnt[i]) : 0;
    int tot = 0;
    const int ex = BlockScan<NT>::exclusive(v, wsum, tot);
    if (i < heads) p.comp_off[i] = carry + ex;
    carry += tot;
  }
  if (threadIdx.x == 0) p.comp_off[heads] = carry;
}

// ---------------------------------------------------------------------------
// warp per (b, h): tables of up to 32 * EPL pages
// ---------------------------------------------------------------------------
// k at or below which the threshold is found by k max-extraction rounds over
// per-lane sorted keys rather than by the 32-step bisection
constexpr int kExtractMax = 64;

// Ascending bitonic sort of N (power of two) values held in registers.
template <int N>
__device__ __forceinline__ void sort_asc(uint32_t (&a)[N]) {
#pragma unroll
  for (int size = 2; size <= N; size <<= 1)
#pragma unroll
    for (int stride = size / 2; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < N; ++i) {
        const int j = i ^ stride;
        if (j > i) {
          const uint32_t x = a[i], y = a[j];
          const bool up = (i & size) == 0;
          a[i] = up ? min(x, y) : max(x, y);
          a[j] = up ? max(x, y) : min(x, y);
        }
      }
}

// Two heads per CTA: the per-head search is instruction-bound, so heads are
// spread over as many SMs as possible.
constexpr int kWarpSelWarps = 2;

template <int EPL>
__global__ void __launch_bounds__(kWarpSelWarps * 32) select_gate_warp_kernel(SelectParams p) {
  constexpr int NT = kWarpSelWarps * 32;
  __shared__ int wsum[NT / 32];
  __shared__ int s_flag[2];
  __shared__ int s_rej;
  __shared__ int s_heads[2];  // heads counted / accepted by this CTA
  __shared__ float s_row_all[kWarpSelWarps][32 * EPL];
  if (threadIdx.x < 2) s_heads[threadIdx.x] = 0;
  if (threadIdx.x == 0) s_rej = 0;
  __syncthreads();
  pdl_wait();
  // head counters: one atomic per CTA instead of one per head
  auto count = [&](bool acc) {
    if (!p.counters) return;
    atomicAdd(&s_heads[0], 1);
    if (acc) atomicAdd(&s_heads[1], 1);
  };

  const int lane = threadIdx.x & 31;
  const int heads = p.B * p.hkv;
  const int bh = blockIdx.x * kWarpSelWarps + (threadIdx.x >> 5);
  if (bh < heads) {
    const int b = bh / p.hkv;
    const int W = p.W;
    const float* row = p.scores + (int64_t)bh * W;
    const int p0 = lane * EPL;
    // every load of the head is issued before any is used
    float s[EPL];
    if ((W % 4) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
#pragma unroll
      for (int i = 0; i < EPL; i += 4) {
        if (p0 + i < W) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(row + p0 + i));
          s[i] = v.x; s[i + 1] = v.y; s[i + 2] = v.z; s[i + 3] = v.w;
        } else {
          s[i] = s[i + 1] = s[i + 2] = s[i + 3] = neg_inf();
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) s[i] = (p0 + i < W) ? __ldcg(row + p0 + i) : neg_inf();
    }
    const int nv = min(n_valid_pages(p.lens[b], p.bs), W);
    float* srow = s_row_all[threadIdx.x >> 5];
#pragma unroll
    for (int i = 0; i < EPL; ++i) srow[p0 + i] = s[i];
    __syncwarp();

    // lse over all W pages (coverage.py:179-195): -inf entries contribute 0
    float m = -1e20f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) m = fmaxf(m, s[i]);
    m = fmaxf(warp_max(m), -1e20f);
    float sum = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) sum += expf(s[i] - m);
    const float lse_all = m + logf(warp_sum(sum) + 1e-30f);

    // ---- cached-selection gate (lazy) ----
    if (p.mode == CVSA_MODE_LAZY && p.has_cache && p.cached_idx) {
      const int nc = min(max(p.cached_n[bh], 0), p.cached_stride);
      const float lse_c =
          lse_list_smem(srow, W, p.cached_idx + (int64_t)bh * p.cached_stride, nc);
      const float cov = expf(lse_c - lse_all);
      const bool acc = cov >= p.tau;
      if (lane == 0) {
        if (p.cached_accept) p.cached_accept[bh] = acc ? 1 : 0;
        if (p.cached_cov) p.cached_cov[bh] = cov;
        if (!acc) atomicAdd(&s_rej, 1);
        count(acc);
      }
    }

    // ---- new selection ----
    if (p.sel_idx) {
      const int sink = p.sink, local = p.local;
      bool cand[EPL], forced[EPL];
      int nf = 0;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        const int pg = p0 + i;
        forced[i] = pg < nv && (pg < sink || pg >= nv - local);
        cand[i] = pg < nv && !forced[i];
        nf += forced[i] ? 1 : 0;
      }
      const int n_cand = nv - (int)__reduce_add_sync(0xffffffffu, (unsigned)nf);
      const int k = min(p.budget, n_cand);
      const bool all_cand = k >= n_cand;
      uint32_t key[EPL];
#pragma unroll
      for (int i = 0; i < EPL; ++i) key[i] = float_key(s[i]);
      uint32_t thr = 0;
      int take_eq = 0;
      if (k > 0 && !all_cand && k <= kExtractMax) {
        // T = the k-th largest candidate key: each lane sorts its keys in
        // registers (non-candidates as 0, below every candidate key but NaN's,
        // which leaves the k-th value unchanged), then k rounds take the warp
        // maximum of the lanes' largest remaining keys; the lowest lane
        // holding it drops that key
        uint32_t kk[EPL];
#pragma unroll
        for (int i = 0; i < EPL; ++i) kk[i] = cand[i] ? key[i] : 0u;
        sort_asc<EPL>(kk);
#pragma unroll 1
        for (int r = 0; r < k; ++r) {
          thr = __reduce_max_sync(0xffffffffu, kk[EPL - 1]);
          const unsigned who = __ballot_sync(0xffffffffu, kk[EPL - 1] == thr);
          if (lane == __ffs(who) - 1) {
#pragma unroll
            for (int i = EPL - 1; i > 0; --i) kk[i] = kk[i - 1];
            kk[0] = 0u;
          }
        }
      } else if (k > 0 && !all_cand) {
        // largest T with #{candidates with key >= T} >= k, bit by bit; the
        // warp-wide count is a sum of independent ballots. T lies between the
        // smallest and largest candidate key, so the bits above their highest
        // differing bit are fixed from the start.
        uint32_t kmin = 0xffffffffu, kmax = 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i)
          if (cand[i]) {
            kmin = min(kmin, key[i]);
            kmax = max(kmax, key[i]);
          }
        kmin = __reduce_min_sync(0xffffffffu, kmin);
        kmax = __reduce_max_sync(0xffffffffu, kmax);
        const int top = 31 - __clz(kmin ^ kmax);  // -1 when all keys are equal
        thr = top >= 0 ? (kmax & ~((2u << top) - 1u)) : kmax;
        if (top == 31) thr = 0;
#pragma unroll 1
        for (int bit = top; bit >= 0; --bit) {
          const uint32_t c = thr | (1u << bit);
          int cnt = 0;
#pragma unroll
          for (int i = 0; i < EPL; ++i)
            cnt += __popc(__ballot_sync(0xffffffffu, cand[i] && key[i] >= c));
          if (cnt >= k) thr = c;
        }
      }
      if (k > 0 && !all_cand) {
        unsigned gt = 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) gt += (cand[i] && key[i] > thr) ? 1u : 0u;
        take_eq = k - (int)__reduce_add_sync(0xffffffffu, gt);
      }
      int my_eq = 0;
      if (k > 0 && !all_cand) {
#pragma unroll
        for (int i = 0; i < EPL; ++i) my_eq += (cand[i] && key[i] == thr) ? 1 : 0;
      }
      int tot_eq = 0;
      int rank = warp_excl_scan(my_eq, tot_eq);
      bool sel[EPL];
      int my_sel = 0;
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        bool t = forced[i];
        if (cand[i] && k > 0) {
          if (all_cand) {
            t = true;
          } else if (key[i] > thr) {
            t = true;
          } else if (key[i] == thr) {
            t = rank < take_eq;
            ++rank;
          }
        }
        sel[i] = t;
        my_sel += t ? 1 : 0;
      }
      int n_sel = 0;
      int pos = warp_excl_scan(my_sel, n_sel);
      int32_t* out = p.sel_idx + (int64_t)bh * p.max_sel;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (sel[i]) {
          if (pos < p.max_sel) out[pos] = p0 + i;
          ++pos;
        }
      if (p.sel_bitmap) {
        constexpr int LPW = (EPL >= 32) ? 1 : 32 / EPL;  // lanes per 32-bit word
        uint32_t bits = 0;
#pragma unroll
        for (int i = 0; i < EPL; ++i) bits |= sel[i] ? (1u << i) : 0u;
        uint32_t word = (EPL >= 32) ? bits : (bits << ((lane % LPW) * EPL));
#pragma unroll
        for (int o = LPW / 2; o >= 1; o >>= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
        const int wi = lane / LPW;
        if (lane % LPW == 0 && wi < p.bitmap_words)
          p.sel_bitmap[(int64_t)bh * p.bitmap_words + wi] = word;
      }
      // coverage of the new selection
      float ms = -1e20f;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (sel[i]) ms = fmaxf(ms, s[i]);
      ms = fmaxf(warp_max(ms), -1e20f);
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i)
        if (sel[i]) ss += expf(s[i] - ms);
      const float lse_s = ms + logf(warp_sum(ss) + 1e-30f);
      const float cov = expf(lse_s - lse_all);
      const bool acc = cov >= p.tau;
      if (lane == 0) {
        p.sel_n[bh] = min(n_sel, p.max_sel);
        if (p.accept) p.accept[bh] = acc ? 1 : 0;
        if (p.cov) p.cov[bh] = cov;
        if (p.comp_cnt) p.comp_cnt[bh] = acc ? 0 : (nv + p.comp_chunk - 1) / p.comp_chunk;
        if (p.mode == CVSA_MODE_SCORE) {
          if (!acc) atomicAdd(&s_rej, 1);
          if (!p.lazy_stats) count(acc);
        }
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && p.counters && s_heads[0]) {
    atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_ACCEPT]),
              (unsigned long long)s_heads[1]);
    atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_TOTAL]),
              (unsigned long long)s_heads[0]);
  }
  finish_select<NT>(p, s_rej, s_flag, wsum);
  // (triggered at the end: an early trigger, which places the next kernel's
  // CTAs beside these small ones while they run, measured slower)
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// CTA per (b, h): long tables
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(NT) select_gate_kernel(SelectParams p) {
  extern __shared__ float s_scores[];  // [W] then uint8 flags [W]
  __shared__ float red[33];
  __shared__ int wsum[NT / 32];
  __shared__ uint32_t hist[256];
  __shared__ int bcast[4];
  __shared__ int s_flag[2];

  pdl_wait();

  const int bh = blockIdx.x;
  const int b = bh / p.hkv;
  const int W = p.W;
  const int tid = threadIdx.x;
  uint8_t* flag = reinterpret_cast<uint8_t*>(s_scores + W);

  const int ctx = p.lens[b];
  const int nv = min(n_valid_pages(ctx, p.bs), W);
  const float* row = p.scores + (int64_t)bh * W;
  for (int i = tid; i < W; i += NT) s_scores[i] = row[i];
  __syncthreads();

  // lse over all W pages (coverage.py:179-195): -inf entries contribute 0.
  float m = -1e20f;
  for (int i = tid; i < W; i += NT) m = fmaxf(m, s_scores[i]);
  const float m_all = fmaxf(block_reduce_max<NT>(m, red), -1e20f);
  float sum = 0.f;
  for (int i = tid; i < W; i += NT) sum += expf(s_scores[i] - m_all);
  const float lse_all = m_all + logf(block_reduce_sum<NT>(sum, red) + 1e-30f);

  const float tau = p.tau;
  int rejects = 0;  // of the deciding gate, thread 0

  // ---- cached-selection gate (lazy) ----
  if ((p.mode == CVSA_MODE_LAZY) && p.has_cache && p.cached_idx) {
    if (tid < 32) {
      const int nc = min(max(p.cached_n[bh], 0), p.cached_stride);
      const float lse_c = lse_list_warp(s_scores, W, p.cached_idx + (int64_t)bh * p.cached_stride,
                                        nc);
      const float cov = expf(lse_c - lse_all);
      const bool acc = cov >= tau;
      if (tid == 0) {
        if (p.cached_accept) p.cached_accept[bh] = acc ? 1 : 0;
        if (p.cached_cov) p.cached_cov[bh] = cov;
        rejects = acc ? 0 : 1;
        count_head(p, acc);
      }
    }
    __syncthreads();
  }

  // ---- new selection ----
  if (p.sel_idx) {
    const int sink = p.sink, local = p.local;
    // candidate = valid and not forced
    auto is_forced = [&](int pg) { return pg < nv && (pg < sink || pg >= nv - local); };
    int n_forced = 0;
    {
      int f = 0;
      for (int i = tid; i < nv; i += NT) f += is_forced(i) ? 1 : 0;
      n_forced = (int)block_reduce_sum<NT>((float)f, red);
    }
    const int n_cand = nv - n_forced;
    const int k = min(p.budget, n_cand);

    // contiguous chunk per thread for order-preserving scans
    const int ept = (W + NT - 1) / NT;
    const int c0 = tid * ept;
    const int c1 = min(c0 + ept, W);

    uint32_t thr = 0;     // threshold key (k-th largest among candidates)
    int take_eq = 0;      // number of == thr candidates to take (lowest index first)
    const bool all_cand = (k >= n_cand);
    if (k > 0 && !all_cand) {
      uint32_t prefix = 0, pmask = 0;
      int krem = k;
      const int lane = tid & 31;
      for (int shift = 24; shift >= 0; shift -= 8) {
        for (int i = tid; i < 256; i += NT) hist[i] = 0;
        __syncthreads();
        for (int base = 0; base < ept; ++base) {
          const int pg = c0 + base;
          bool act = false;
          uint32_t digit = 0;
          if (pg < c1 && pg < nv && !is_forced(pg)) {
            const uint32_t key = float_key(s_scores[pg]);
            if ((key & pmask) == prefix) {
              act = true;
              digit = (key >> shift) & 255u;
            }
          }
          const uint32_t tag = act ? digit : (256u + lane);
          const uint32_t peers = __match_any_sync(0xffffffffu, tag);
          if (act && (__ffs(peers) - 1) == lane) atomicAdd(&hist[digit], (uint32_t)__popc(peers));
        }
        __syncthreads();
        if (tid < 32) {
          uint32_t c[8];
          uint32_t tot = 0;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            c[j] = hist[lane * 8 + j];
            tot += c[j];
          }
          // count of keys in bins strictly above this lane's bins
          uint32_t incl = tot;
#pragma unroll
          for (int o = 1; o < 32; o <<= 1) {
            uint32_t y = __shfl_down_sync(0xffffffffu, incl, o);
            if (lane + o < 32) incl += y;
          }
          uint32_t running = incl - tot;
#pragma unroll
          for (int j = 7; j >= 0; --j) {
            if (running < (uint32_t)krem && running + c[j] >= (uint32_t)krem) {
              bcast[0] = lane * 8 + j;
              bcast[1] = krem - (int)running;
            }
            running += c[j];
          }
        }
        __syncthreads();
        prefix |= ((uint32_t)bcast[0]) << shift;
        pmask |= 255u << shift;
        krem = bcast[1];
        __syncthreads();
      }
      thr = prefix;
      take_eq = krem;
    }

    // rank among == thr candidates (index order) to apply the tie rule
    int my_eq = 0;
    if (k > 0 && !all_cand) {
      for (int pg = c0; pg < c1; ++pg)
        if (pg < nv && !is_forced(pg) && float_key(s_scores[pg]) == thr) ++my_eq;
    }
    int tot_eq = 0;
    int eq_before = BlockScan<NT>::exclusive(my_eq, wsum, tot_eq);

    int my_sel = 0;
    for (int pg = c0; pg < c1; ++pg) {
      bool sel = false;
      if (pg < nv) {
        if (is_forced(pg)) {
          sel = true;
        } else if (k > 0) {
          if (all_cand) {
            sel = true;
          } else {
            const uint32_t key = float_key(s_scores[pg]);
            if (key > thr) {
              sel = true;
            } else if (key == thr) {
              sel = eq_before < take_eq;
              ++eq_before;
            }
          }
        }
      }
      flag[pg] = sel ? 1 : 0;
      my_sel += sel ? 1 : 0;
    }
    int n_sel = 0;
    const int pos0 = BlockScan<NT>::exclusive(my_sel, wsum, n_sel);
    {
      int32_t* out = p.sel_idx + (int64_t)bh * p.max_sel;
      int pos = pos0;
      for (int pg = c0; pg < c1; ++pg)
        if (flag[pg]) {
          if (pos < p.max_sel) out[pos] = pg;
          ++pos;
        }
    }
    __syncthreads();
    if (p.sel_bitmap) {
      uint32_t* bm = p.sel_bitmap + (int64_t)bh * p.bitmap_words;
      for (int wd = tid; wd < p.bitmap_words; wd += NT) {
        uint32_t bits = 0;
        const int base = wd * 32;
#pragma unroll 4
        for (int j = 0; j < 32; ++j)
          if (base + j < W && flag[base + j]) bits |= 1u << j;
        bm[wd] = bits;
      }
    }
    const float lse_s = lse_flagged<NT>(s_scores, flag, W, red);
    const float cov = expf(lse_s - lse_all);
    const bool acc = cov >= tau;
    if (tid == 0) {
      p.sel_n[bh] = min(n_sel, p.max_sel);
      if (p.accept) p.accept[bh] = acc ? 1 : 0;
      if (p.cov) p.cov[bh] = cov;
      if (p.comp_cnt) p.comp_cnt[bh] = acc ? 0 : (nv + p.comp_chunk - 1) / p.comp_chunk;
      if (p.mode == CVSA_MODE_SCORE) {
        rejects = acc ? 0 : 1;
        if (!p.lazy_stats) count_head(p, acc);
      }
    }
  }
  finish_select<NT>(p, rejects, s_flag, wsum);
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// CTA of NT threads per (b, h): tables of 257 to 16384 pages (NT = 128 up to
// 1024 pages, 1024 above)
// ---------------------------------------------------------------------------
// Thread t holds the EPT contiguous pages [t * EPT, (t + 1) * EPT) in
// registers, so every block scan is in page order. The kernel is built from
// few block-wide steps, since each costs a barrier round on one SM:
//  1. one max-type reduction (order-preserving keys, REDUX) of the row max,
//     the valid-page max, the candidate range and the cached list's max;
//  2. one sum reduction of both log-sum-exp sums, while the candidates are
//     counted into kBigBins equal-width bins of their score range (the bin
//     index is monotone in the score, so every candidate of a higher bin
//     ranks above every candidate of a lower one);
//  3. one scan over the bins finds the bin that holds the k-th candidate;
//  4. that bin's entries are gathered and ranked directly (key descending,
//     page ascending), which gives the cut (key, page) of the last one taken;
//  5. one scan compacts the selection and sums its lse terms.
// A bin too crowded to rank directly (heavy ties), or a candidate range that
// is not finite, falls back to a radix select of the k-th key (4 bits per
// pass over a packed 16-bin digit histogram) and a scan of the equal keys.
constexpr int kBigNT = 1024;    // threads of the long-table variant (bins: 2 per thread;
                                // bin entries ranked directly: min(threads, 256))

__device__ __forceinline__ float key_float(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}

template <int EPT, int NT>
__global__ void __launch_bounds__(NT) select_gate_big_kernel(SelectParams p) {
  constexpr int NW = NT / 32;
  constexpr int kBigBins = 2 * NT;                      // two bins per thread
  constexpr int kBigBinCap = NT < 256 ? NT : 256;       // one thread ranks one entry
  __shared__ uint32_t s_kred[NW][6];
  __shared__ float s_fred[NW][2];
  __shared__ int s_hist[kBigBins];
  __shared__ unsigned long long s_gent[kBigBinCap];  // key << 32 | ~page
  __shared__ uint32_t wcnt[NW][8];
  __shared__ int s_iscan[NW];
  __shared__ float red[33];
  __shared__ int wsum[NW];
  __shared__ int s_flag[2];
  __shared__ int s_pick, s_above, s_bin, s_nbin, s_tidx;
  __shared__ uint32_t s_tkey;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int i = tid; i < kBigBins; i += NT) s_hist[i] = 0;
  if (tid == 0) s_nbin = 0;
  pdl_wait();
  // all of this grid is resident (one CTA per head): the next kernel's CTAs
  // may take the free SMs now; they wait for this grid before reading
  pdl_launch_dependents();

  const int bh = blockIdx.x;
  const int b = bh / p.hkv;
  const int W = p.W;
  const float* row = p.scores + (int64_t)bh * W;
  const int p0 = tid * EPT;
  const bool gate_cached = p.mode == CVSA_MODE_LAZY && p.has_cache && p.cached_idx;
  // the cached list, one entry per thread per round (duplicates count, like
  // the reference's gather at coverage.py:196-204)
  const int32_t* ci = gate_cached ? p.cached_idx + (int64_t)bh * p.cached_stride : nullptr;
  int ci0 = -1;
  if (gate_cached && tid < p.cached_stride) ci0 = __ldcg(ci + tid);
  float s[EPT];
  if ((W % 4) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
#pragma unroll
    for (int i = 0; i < EPT; i += 4) {
      if (p0 + i < W) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(row + p0 + i));
        s[i] = v.x; s[i + 1] = v.y; s[i + 2] = v.z; s[i + 3] = v.w;
      } else {
        s[i] = s[i + 1] = s[i + 2] = s[i + 3] = neg_inf();
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < EPT; ++i) s[i] = (p0 + i < W) ? __ldcg(row + p0 + i) : neg_inf();
  }
  const int nv = min(n_valid_pages(p.lens[b], p.bs), W);
  const int nc = gate_cached ? min(max(p.cached_n[bh], 0), p.cached_stride) : 0;
  auto cval = [&](int pg) -> float { return (pg >= 0 && pg < W) ? __ldcg(row + pg) : neg_inf(); };
  const float c0 = tid < nc ? cval(ci0) : neg_inf();

  const int sink = p.sink, local = p.local;
  bool cand[EPT], forced[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const int pg = p0 + i;
    forced[i] = pg < nv && (pg < sink || pg >= nv - local);
    cand[i] = pg < nv && !forced[i];
  }
  // forced pages: [0, sink) and [nv - local, nv) inside [0, nv)
  const int f_lo = min(max(sink, 0), nv);
  const int f_hi = max(nv - max(local, 0), 0);
  const int tot_forced = nv <= 0 ? 0 : f_lo + (nv - f_hi) - max(0, f_lo - f_hi);
  const int n_cand = nv - tot_forced;
  const int k = p.sel_idx ? min(p.budget, n_cand) : 0;
  const bool all_cand = k >= n_cand;

  // ---- 1. max-type reduction over keys ----
  const uint32_t kfloor = float_key(-1e20f);
  uint32_t r[6] = {kfloor, kfloor, 0u, 0xffffffffu, kfloor, 0u};
  // r: row max, valid max, candidate max, candidate min, cached max, non-finite candidate
  uint32_t key[EPT];
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const uint32_t ky = float_key(s[i]);
    key[i] = ky;
    r[0] = max(r[0], ky);
    if (p0 + i < nv) r[1] = max(r[1], ky);
    if (cand[i]) {
      r[2] = max(r[2], ky);
      r[3] = min(r[3], ky);
      if (!isfinite(s[i])) r[5] = 1u;
    }
  }
  r[4] = max(r[4], float_key(c0));
  for (int i = tid + NT; i < nc; i += NT) r[4] = max(r[4], float_key(cval(__ldcg(ci + i))));
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    const uint32_t v = (j == 3) ? __reduce_min_sync(0xffffffffu, r[j])
                                : __reduce_max_sync(0xffffffffu, r[j]);
    if (lane == 0) s_kred[warp][j] = v;
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < 6; ++j) {
    const uint32_t v = lane < NW ? s_kred[lane][j] : (j == 3 ? 0xffffffffu : 0u);
    r[j] = (j == 3) ? __reduce_min_sync(0xffffffffu, v) : __reduce_max_sync(0xffffffffu, v);
  }
  const float m_all = key_float(r[0]);    // = max(-1e20, row max) (coverage.py:179-195)
  const float m_valid = key_float(r[1]);
  const float mc = key_float(r[4]);
  const bool nonfinite = r[5] != 0u;

  // ---- 2. sum reduction; candidate bins ----
  // exp(s - m_all), kept for the selection's sum where registers allow
  constexpr bool kKeepE = EPT <= 8;
  float e[kKeepE ? EPT : 1];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < EPT; ++i) {
    const float x = expf(s[i] - m_all);
    if constexpr (kKeepE) e[i] = x;
    sum += x;
  }
  float sc = (c0 != neg_inf()) ? expf(c0 - mc) : 0.f;
  for (int i = tid + NT; i < nc; i += NT) {
    const float x = cval(__ldcg(ci + i));
    if (x != neg_inf()) sc += expf(x - mc);
  }
  bool use_bins = false;
  float lo_s = 0.f, scale = 0.f;
  if (k > 0 && !all_cand && !nonfinite) {
    lo_s = key_float(r[3]);
    scale = (float)kBigBins / (key_float(r[2]) - lo_s);
    use_bins = scale > 0.f && scale < 3.0e38f;
  }
  // candidate bins, two 16-bit indices per word (0xffff: not a candidate)
  uint32_t binw[(EPT + 1) / 2];
#pragma unroll
  for (int i = 0; i < (EPT + 1) / 2; ++i) binw[i] = 0xffffffffu;
  if (use_bins) {
#pragma unroll
    for (int i = 0; i < EPT; ++i)
      if (cand[i]) {
        const int bn = min(kBigBins - 1, (int)((s[i] - lo_s) * scale));
        atomicAdd(&s_hist[bn], 1);
        binw[i >> 1] = (i & 1) ? ((binw[i >> 1] & 0xffffu) | ((uint32_t)bn << 16))
                               : ((binw[i >> 1] & 0xffff0000u) | (uint32_t)bn);
      }
  }
  auto bin_at = [&](int i) -> uint32_t { return (binw[i >> 1] >> ((i & 1) * 16)) & 0xffffu; };
  sum = warp_sum(sum);
  sc = warp_sum(sc);
  if (lane == 0) { s_fred[warp][0] = sum; s_fred[warp][1] = sc; }
  __syncthreads();
  sum = warp_sum(lane < NW ? s_fred[lane][0] : 0.f);
  sc = warp_sum(lane < NW ? s_fred[lane][1] : 0.f);
  const float lse_all = m_all + logf(sum + 1e-30f);

  const float tau = p.tau;
  int rejects = 0;  // of the deciding gate, thread 0

  // ---- cached-selection gate (lazy) ----
  if (gate_cached) {
    const float cov = expf(mc + logf(sc + 1e-30f) - lse_all);
    const bool acc = cov >= tau;
    if (tid == 0) {
      if (p.cached_accept) p.cached_accept[bh] = acc ? 1 : 0;
      if (p.cached_cov) p.cached_cov[bh] = cov;
      rejects = acc ? 0 : 1;
      count_head(p, acc);
    }
  }

  // ---- new selection ----
  if (p.sel_idx) {
    // the last candidate taken, in (key descending, page ascending) order
    uint32_t tkey = 0;
    int tidx = -1;
    if (use_bins) {
      // ---- 3. the bin holding the k-th candidate (bins in descending order) ----
      const int b_hi = kBigBins - 1 - 2 * tid;
      const int h1 = s_hist[b_hi], h0 = s_hist[b_hi - 1];
      const int c = h1 + h0;
      int x = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) s_iscan[warp] = x;
      __syncthreads();
      const int wv = lane < NW ? s_iscan[lane] : 0;
      const int excl = (int)__reduce_add_sync(0xffffffffu, lane < warp ? wv : 0) + x - c;
      if (excl < k && k <= excl + h1) { s_bin = b_hi; s_above = excl; }
      else if (excl + h1 < k && k <= excl + c) { s_bin = b_hi - 1; s_above = excl + h1; }
      __syncthreads();
      // ---- 4. gather and rank the bin ----
      const uint32_t tb = (uint32_t)s_bin;
      const int take = k - s_above;
#pragma unroll
      for (int i = 0; i < EPT; ++i)
        if (bin_at(i) == tb) {
          const int slot = atomicAdd(&s_nbin, 1);
          if (slot < kBigBinCap)
            s_gent[slot] = ((unsigned long long)key[i] << 32) | (uint32_t)~(uint32_t)(p0 + i);
        }
      __syncthreads();
      const int nb = s_nbin;
      if (nb <= kBigBinCap) {
        // rank = entries ahead in (key descending, page ascending) order
        if (tid < nb) {
          const unsigned long long me = s_gent[tid];
          int rank = 0;
          int j = 0;
          for (; j + 4 <= nb; j += 4) {
            rank += (s_gent[j] > me ? 1 : 0) + (s_gent[j + 1] > me ? 1 : 0) +
                    (s_gent[j + 2] > me ? 1 : 0) + (s_gent[j + 3] > me ? 1 : 0);
          }
          for (; j < nb; ++j) rank += s_gent[j] > me ? 1 : 0;
          if (rank == take - 1) { s_tkey = (uint32_t)(me >> 32); s_tidx = (int)~(uint32_t)me; }
        }
        __syncthreads();
        tkey = s_tkey;
        tidx = s_tidx;
      } else {
        use_bins = false;
      }
    }
    if (k > 0 && !all_cand && !use_bins) {
      // radix select of the k-th largest candidate key, 4 bits per pass: each
      // thread histograms the digit of its candidates that share the prefix
      // found so far (16 bins of 8 bits in two 64-bit words), the bins are
      // widened to 16-bit pairs and summed by REDUX per warp, then across
      // warps by warp 0, which picks the largest digit d with
      // above + #{prefix digit >= d} >= k ("above" = candidates whose key is
      // already known to exceed the prefix).
      uint32_t thr = 0;
      int above = 0;  // warp 0's copy
#pragma unroll 1
      for (int shift = 28; shift >= 0; shift -= 4) {
        const uint32_t pmask = (shift == 28) ? 0u : (0xffffffffu << (shift + 4));
        const uint32_t pref = thr & pmask;
        unsigned long long lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < EPT; ++i) {
          const uint32_t ky = key[i];
          if (cand[i] && (ky & pmask) == pref) {
            const uint32_t d = (ky >> shift) & 15u;
            const unsigned long long inc = 1ull << ((d & 7u) * 8u);
            if (d < 8) lo += inc; else hi += inc;
          }
        }
        const uint32_t w32[4] = {(uint32_t)lo, (uint32_t)(lo >> 32), (uint32_t)hi,
                                 (uint32_t)(hi >> 32)};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // bins 4j..4j+3 -> two words of 16-bit fields
          const unsigned a = __reduce_add_sync(0xffffffffu, __byte_perm(w32[j], 0u, 0x4140));
          const unsigned c = __reduce_add_sync(0xffffffffu, __byte_perm(w32[j], 0u, 0x4342));
          if (lane == 0) { wcnt[warp][2 * j] = a; wcnt[warp][2 * j + 1] = c; }
        }
        __syncthreads();
        if (warp == 0) {
          uint32_t tot[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tot[j] = __reduce_add_sync(0xffffffffu, lane < NW ? wcnt[lane][j] : 0u);
          int pick = 0, suffix = 0, pick_above = above;
#pragma unroll
          for (int dd = 15; dd >= 1; --dd) {
            const int c = (int)((tot[dd >> 1] >> ((dd & 1) * 16)) & 0xffffu);
            // keep the first (largest) digit that reaches k
            if (pick == 0 && above + suffix + c >= k) { pick = dd; pick_above = above + suffix; }
            suffix += c;
          }
          if (pick == 0) pick_above = above + suffix;
          above = pick_above;
          if (lane == 0) { s_pick = pick; s_above = above; }
        }
        __syncthreads();
        thr |= (uint32_t)s_pick << shift;
      }
      // equal keys are taken lowest page first: the take_eq-th one in page order
      const int take_eq = k - s_above;
      int my_eq = 0;
#pragma unroll
      for (int i = 0; i < EPT; ++i) my_eq += (cand[i] && key[i] == thr) ? 1 : 0;
      int tot_eq = 0;
      const int rank = BlockScan<NT>::exclusive(my_eq, wsum, tot_eq);
      if (rank < take_eq && take_eq <= rank + my_eq) {
        int e = rank;
#pragma unroll
        for (int i = 0; i < EPT; ++i)
          if (cand[i] && key[i] == thr) {
            if (e == take_eq - 1) s_tidx = p0 + i;
            ++e;
          }
      }
      __syncthreads();
      tkey = thr;
      tidx = s_tidx;
    }

    // ---- 5. compaction and the selection's lse ----
    // every valid page's score is at most m_valid, and the selection holds
    // the best candidate and all forced pages unless k == 0 with candidates
    // left out, so max over the selection == m_valid (coverage.py:196-204)
    float ms = m_valid;
    if (k == 0 && n_cand > 0) {
      float mf = -1e20f;
#pragma unroll
      for (int i = 0; i < EPT; ++i)
        if (forced[i]) mf = fmaxf(mf, key_float(key[i]));
      ms = fmaxf(block_reduce_max<NT>(mf, red), -1e20f);
    }
    // the step-2 terms exp(s - m_all) are the selection's terms when
    // ms == m_all (no finite score past the valid pages); the scores are
    // otherwise rebuilt from their keys (exact but for -0 -> +0)
    const bool reuse_e = kKeepE && ms == m_all;
    bool sel[EPT];
    int my_sel = 0;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < EPT; ++i) {
      bool t = forced[i];
      if (cand[i] && k > 0)
        t = all_cand || key[i] > tkey || (key[i] == tkey && p0 + i <= tidx);
      sel[i] = t;
      my_sel += t ? 1 : 0;
      if (t) {
        if constexpr (kKeepE) ss += reuse_e ? e[i] : expf(key_float(key[i]) - ms);
        else ss += expf(key_float(key[i]) - ms);
      }
    }
    int x = my_sel;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    ss = warp_sum(ss);
    if (lane == 31) s_iscan[warp] = x;
    if (lane == 0) s_fred[warp][0] = ss;
    __syncthreads();
    const int wv = lane < NW ? s_iscan[lane] : 0;
    int pos = (int)__reduce_add_sync(0xffffffffu, lane < warp ? wv : 0) + x - my_sel;
    const int n_sel = (int)__reduce_add_sync(0xffffffffu, wv);
    ss = warp_sum(lane < NW ? s_fred[lane][0] : 0.f);
    int32_t* out = p.sel_idx + (int64_t)bh * p.max_sel;
#pragma unroll
    for (int i = 0; i < EPT; ++i)
      if (sel[i]) {
        if (pos < p.max_sel) out[pos] = p0 + i;
        ++pos;
      }
    if (p.sel_bitmap) {
      // EPT pages per thread: 32 / EPT threads per 32-bit word (EPT <= 32)
      constexpr int TPW = (EPT >= 32) ? 1 : 32 / EPT;
      uint32_t bits = 0;
#pragma unroll
      for (int i = 0; i < EPT; ++i) bits |= sel[i] ? (1u << i) : 0u;
      uint32_t word = (EPT >= 32) ? bits : (bits << ((lane % TPW) * EPT));
#pragma unroll
      for (int o = TPW / 2; o >= 1; o >>= 1) word |= __shfl_xor_sync(0xffffffffu, word, o);
      const int wi = tid / TPW;
      if (lane % TPW == 0 && wi < p.bitmap_words) p.sel_bitmap[(int64_t)bh * p.bitmap_words + wi] = word;
    }
    const float lse_s = ms + logf(ss + 1e-30f);
    const float cov = expf(lse_s - lse_all);
    const bool acc = cov >= tau;
    if (tid == 0) {
      p.sel_n[bh] = min(n_sel, p.max_sel);
      if (p.accept) p.accept[bh] = acc ? 1 : 0;
      if (p.cov) p.cov[bh] = cov;
      if (p.comp_cnt) p.comp_cnt[bh] = acc ? 0 : (nv + p.comp_chunk - 1) / p.comp_chunk;
      if (p.mode == CVSA_MODE_SCORE) {
        rejects = acc ? 0 : 1;
        if (!p.lazy_stats) count_head(p, acc);
      }
    }
  }
  // the decision counts this CTA's head once (thread 0 holds it)
  finish_select<NT>(p, tid == 0 ? rejects : 0, s_flag, wsum);
}

template <int EPT, int NT = kBigNT>
cudaError_t launch_sel_big(const SelectParams& p, cudaStream_t s, bool pdl) {
  return launch_k(select_gate_big_kernel<EPT, NT>, dim3(p.B * p.hkv), dim3(NT), 0, s, pdl, p);
}

template <int NT>
cudaError_t launch_sel(const SelectParams& p, cudaStream_t s, bool pdl) {
  const size_t smem = (size_t)p.W * sizeof(float) + (size_t)p.W + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(select_gate_kernel<NT>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(select_gate_kernel<NT>, dim3(p.B * p.hkv), dim3(NT), smem, s, pdl, p);
}

template <int EPL>
cudaError_t launch_sel_warp(const SelectParams& p, cudaStream_t s, bool pdl) {
  const int heads = p.B * p.hkv;
  const int grid = (heads + kWarpSelWarps - 1) / kWarpSelWarps;
  return launch_k(select_gate_warp_kernel<EPL>, dim3(grid), dim3(kWarpSelWarps * 32), 0, s, pdl,
                  p);
}

// ---- standalone coverage gate (coverage.py:160-215) ----
template <int NT>
__global__ void __launch_bounds__(NT)
coverage_kernel(const float* scores, int W, const int32_t* idx, int max_sel, const int32_t* n,
                float tau, uint8_t* accept, float* cov_out) {
  extern __shared__ float s_sc[];
  __shared__ float red[33];
  __shared__ float s_lse;
  const int bh = blockIdx.x;
  const float* row = scores + (int64_t)bh * W;
  for (int i = threadIdx.x; i < W; i += NT) s_sc[i] = row[i];
  __syncthreads();
  float m = -1e20f;
  for (int i = threadIdx.x; i < W; i += NT) m = fmaxf(m, s_sc[i]);
  const float m_all = fmaxf(block_reduce_max<NT>(m, red), -1e20f);
  float sum = 0.f;
  for (int i = threadIdx.x; i < W; i += NT) sum += expf(s_sc[i] - m_all);
  const float lse_all = m_all + logf(block_reduce_sum<NT>(sum, red) + 1e-30f);
  if (threadIdx.x < 32) {
    const int ns = min(max(n[bh], 0), max_sel);
    const float l = lse_list_warp(s_sc, W, idx + (int64_t)bh * max_sel, ns);
    if (threadIdx.x == 0) s_lse = l;
  }
  __syncthreads();
  const float c = expf(s_lse - lse_all);
  if (threadIdx.x == 0) {
    accept[bh] = c >= tau ? 1 : 0;
    if (cov_out) cov_out[bh] = c;
  }
}

// ---- standalone complement list (coverage.py:31-96 / complement.py) ----
template <int NT>
__global__ void __launch_bounds__(NT)
complement_kernel(const int32_t* idx, int max_sel, const int32_t* n, const int32_t* lens,
                  int hkv, int bs, const uint8_t* accept, int32_t* comp, int max_comp,
                  int32_t* n_comp, int Wflag) {
  extern __shared__ uint8_t flag[];
  __shared__ int wsum[NT / 32];
  const int bh = blockIdx.x;
  const int b = bh / hkv;
  const int nv = n_valid_pages(lens[b], bs);
  if (accept && accept[bh]) {
    if (threadIdx.x == 0) n_comp[bh] = 0;
    return;
  }
  for (int i = threadIdx.x; i < Wflag; i += NT) flag[i] = 0;
  __syncthreads();
  const int ns = n[bh];
  for (int i = threadIdx.x; i < min(ns, max_sel); i += NT) {
    const int pg = idx[(int64_t)bh * max_sel + i];
    if (pg >= 0 && pg < Wflag) flag[pg] = 1;
  }
  __syncthreads();
  const int ept = (nv + NT - 1) / NT;
  const int c0 = threadIdx.x * ept, c1 = min(c0 + ept, nv);
  // pages at or past Wflag cannot be selected (indices are checked above)
  auto selected = [&](int pg) { return pg < Wflag && flag[pg]; };
  int mine = 0;
  for (int pg = c0; pg < c1; ++pg) mine += selected(pg) ? 0 : 1;
  int total = 0;
  int pos = BlockScan<NT>::exclusive(mine, wsum, total);
  for (int pg = c0; pg < c1; ++pg)
    if (!selected(pg)) {
      if (pos < max_comp) comp[(int64_t)bh * max_comp + pos] = pg;
      ++pos;
    }
  if (threadIdx.x == 0) n_comp[bh] = total;
}

// selection bitmap from an index list (for externally supplied selections)
__global__ void bitmap_kernel(const int32_t* idx, int max_sel, const int32_t* n, int W,
                              uint32_t* bitmap, int words, int32_t* dev_err) {
  const int bh = blockIdx.x;
  uint32_t* bm = bitmap + (int64_t)bh * words;
  for (int w = threadIdx.x; w < words; w += blockDim.x) bm[w] = 0u;
  __syncthreads();
  const int ns = min(n[bh], max_sel);
  for (int i = threadIdx.x; i < ns; i += blockDim.x) {
    const int pg = idx[(int64_t)bh * max_sel + i];
    if (pg >= 0 && pg < W) atomicOr(&bm[pg >> 5], 1u << (pg & 31));
    else set_dev_error(dev_err, CVSA_DEV_ERR_PAGE_RANGE);
  }
}

}  // namespace

cudaError_t launch_build_bitmap(const int32_t* idx, int max_sel, const int32_t* n, int BH, int W,
                                uint32_t* bitmap, int words, int32_t* dev_err, cudaStream_t s) {
  if (BH == 0) return cudaSuccess;
  bitmap_kernel<<<BH, 256, 0, s>>>(idx, max_sel, n, W, bitmap, words, dev_err);
  return cudaGetLastError();
}

cudaError_t launch_select_gate(const SelectParams& p, cudaStream_t s, bool pdl) {
  if (p.W <= 128) return launch_sel_warp<4>(p, s, pdl);
  if (p.W <= 256) return launch_sel_warp<8>(p, s, pdl);
  // 257..1024 pages: a CTA of 128 threads per head (4 times the warps of one
  // warp per head, so the block steps' latency is shared among more warps)
  if (p.W <= 512) return launch_sel_big<4, 128>(p, s, pdl);
  if (p.W <= 1024) return launch_sel_big<8, 128>(p, s, pdl);
  if (p.W <= 4096) return launch_sel_big<4>(p, s, pdl);
  if (p.W <= 8192) return launch_sel_big<8>(p, s, pdl);
  if (p.W <= 16384) return launch_sel_big<16>(p, s, pdl);
  return launch_sel<1024>(p, s, pdl);
}

cudaError_t launch_check_coverage(const float* scores, int B, int hkv, int W, const int32_t* idx,
                                  int max_sel, const int32_t* n, float tau, uint8_t* accept,
                                  float* cov, cudaStream_t s) {
  const size_t smem = (size_t)W * 4 + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(coverage_kernel<256>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  coverage_kernel<256><<<B * hkv, 256, smem, s>>>(scores, W, idx, max_sel, n, tau, accept, cov);
  return cudaGetLastError();
}

cudaError_t launch_complement(const int32_t* idx, int max_sel, const int32_t* n,
                              const int32_t* lens, int B, int hkv, int bs, const uint8_t* accept,
                              int32_t* comp, int max_comp, int32_t* n_comp, cudaStream_t s) {
  // flags cover every page index the complement can name (< max_comp + max_sel)
  const int wflag = max_comp + max_sel;
  const size_t smem = (size_t)wflag + 16;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(complement_kernel<256>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  complement_kernel<256><<<B * hkv, 256, smem, s>>>(idx, max_sel, n, lens, hkv, bs, accept, comp,
                                                     max_comp, n_comp, wflag);
  return cudaGetLastError();
}

}  // namespace cvsa
