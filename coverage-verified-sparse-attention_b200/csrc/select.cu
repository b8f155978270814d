// Top-k page selection + coverage gate, one CTA per (sequence b, kv head h).
//
// Restates, for one (b, h) row of page scores:
//   * cvsa/backend.py:690,737-747 -- the top `budget` pages by score, with
//     n_per_head = min(budget, n_valid); here the order is (score desc, page
//     index asc) and the first `sink` / last `local` valid pages are forced in
//     (both off by default);
//   * cvsa/kernels/coverage.py:160-215 -- cov = exp(lse(scores[sel]) -
//     lse(scores[all W pages])), max seeded with -1e20, log(sum + 1e-30),
//     accept = cov >= tau;
//   * cvsa/backend.py:424-446 -- in lazy mode, the same gate on the CACHED
//     selection, reduced over the whole batch on the device (the reference's
//     host-side accept_mask.all()) by the last CTA to finish.
// Top-k is an exact radix select on order-preserving 32-bit keys (4 passes
// of 8 bits, warp-aggregated shared-memory histograms), then ties at the
// threshold key go to the lowest page indices via a block prefix scan. The
// selection is emitted in ascending page order together with a bitmap of it
// (consumed by the fused recovery kernel to skip selected pages).
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

template <int NT>
__global__ void __launch_bounds__(NT) select_gate_kernel(SelectParams p) {
  extern __shared__ float s_scores[];  // [W] then uint8 flags [W]
  __shared__ float red[33];
  __shared__ int wsum[NT / 32];
  __shared__ uint32_t hist[256];
  __shared__ int bcast[4];

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
  bool deciding_reject = false;

  // ---- cached-selection gate (lazy) ----
  const bool do_cached = (p.mode == CVSA_MODE_LAZY) && p.has_cache && p.cached_idx;
  if (do_cached) {
    for (int i = tid; i < W; i += NT) flag[i] = 0;
    __syncthreads();
    const int nc = p.cached_n[bh];
    const int32_t* ci = p.cached_idx + (int64_t)bh * p.cached_stride;
    for (int i = tid; i < nc; i += NT) {
      const int pg = ci[i];
      if (pg >= 0 && pg < W) flag[pg] = 1;
    }
    __syncthreads();
    const float lse_c = lse_flagged<NT>(s_scores, flag, W, red);
    const float cov = expf(lse_c - lse_all);
    const bool acc = cov >= tau;
    if (tid == 0) {
      if (p.cached_accept) p.cached_accept[bh] = acc ? 1 : 0;
      if (p.cached_cov) p.cached_cov[bh] = cov;
      deciding_reject = !acc;
      if (p.counters) {
        atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_ACCEPT]),
                  (unsigned long long)(acc ? 1 : 0));
        atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_TOTAL]), 1ull);
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
      if (p.mode == CVSA_MODE_SCORE) {
        deciding_reject = !acc;
        if (p.counters && !p.lazy_stats) {
          atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_ACCEPT]),
                    (unsigned long long)(acc ? 1 : 0));
          atomicAdd(reinterpret_cast<unsigned long long*>(&p.counters[CVSA_CTR_HEAD_TOTAL]),
                    1ull);
        }
      }
    }
  }

  // ---- batch-global decision by the last CTA (no host sync) ----
  if (p.sync_ctr && tid == 0) {
    if (deciding_reject) atomicAdd(&p.sync_ctr[1], 1);
    __threadfence();
    const int done = atomicAdd(&p.sync_ctr[0], 1);
    if (done == (int)gridDim.x - 1) {
      __threadfence();
      const int rejects = atomicAdd(&p.sync_ctr[1], 0);
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
          if (!p.lazy_stats) atomicAdd(&c[all_accept ? CVSA_CTR_ACCEPT_STEPS
                                                     : CVSA_CTR_REJECT_STEPS], 1ull);
        }
      }
      if (p.step_flags) {
        int fl = 0;
        if (p.mode == CVSA_MODE_LAZY) fl = all_accept ? 1 : 2;
        else fl = (all_accept ? 1 : 0) | 2;
        p.step_flags[0] = fl;
      }
      p.sync_ctr[1] = 0;
      __threadfence();
      p.sync_ctr[0] = 0;
    }
  }
  pdl_launch_dependents();
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

// ---- standalone coverage gate (coverage.py:160-215) ----
template <int NT>
__global__ void __launch_bounds__(NT)
coverage_kernel(const float* scores, int W, const int32_t* idx, int max_sel, const int32_t* n,
                float tau, uint8_t* accept, float* cov_out) {
  extern __shared__ float s_sc[];
  __shared__ float red[33];
  uint8_t* flag = reinterpret_cast<uint8_t*>(s_sc + W);
  const int bh = blockIdx.x;
  const float* row = scores + (int64_t)bh * W;
  for (int i = threadIdx.x; i < W; i += NT) {
    s_sc[i] = row[i];
    flag[i] = 0;
  }
  __syncthreads();
  float m = -1e20f;
  for (int i = threadIdx.x; i < W; i += NT) m = fmaxf(m, s_sc[i]);
  const float m_all = fmaxf(block_reduce_max<NT>(m, red), -1e20f);
  float sum = 0.f;
  for (int i = threadIdx.x; i < W; i += NT) sum += expf(s_sc[i] - m_all);
  const float lse_all = m_all + logf(block_reduce_sum<NT>(sum, red) + 1e-30f);
  const int ns = n[bh];
  for (int i = threadIdx.x; i < min(ns, max_sel); i += NT) {
    const int pg = idx[(int64_t)bh * max_sel + i];
    if (pg >= 0 && pg < W) flag[pg] = 1;
  }
  __syncthreads();
  const float lse_s = lse_flagged<NT>(s_sc, flag, W, red);
  const float c = expf(lse_s - lse_all);
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
  if (p.W <= 1024) return launch_sel<256>(p, s, pdl);
  if (p.W <= 8192) return launch_sel<512>(p, s, pdl);
  return launch_sel<1024>(p, s, pdl);
}

cudaError_t launch_check_coverage(const float* scores, int B, int hkv, int W, const int32_t* idx,
                                  int max_sel, const int32_t* n, float tau, uint8_t* accept,
                                  float* cov, cudaStream_t s) {
  const size_t smem = (size_t)W * 5 + 16;
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
