// Page-split step kernels: every rank (one process per GPU) holds a
// contiguous range of every sequence's pages, and the single-GPU step of
// cvsa/backend.py:683-864 (scoring step) and :392-465 (lazy check) runs as
//   score (this rank's pages) -> split_propose -> all-gather A ->
//   split_gate -> attention partials -> all-gather B -> rank merge,
// two exchanges per scoring or lazy-check step, one per reuse step.
//
// split_propose, per (b, h) row of this rank's page scores, writes into the
// rank's exchange-A row:
//   * lse_all_r: log-sum-exp over the row's pages (coverage.py:179-195);
//   * lse_cached_r: over the cached selection's entries (the lazy gate of
//     backend.py:424-446), -inf without a cache;
//   * lse_forced_r: over this rank's forced pages (the sink pages live on
//     rank 0, the local pages on the last rank);
//   * the scores of this rank's best `budget` non-forced pages with finite
//     scores (score descending, page ascending), in page order, -inf padded
//     to max_sel; their local page indices stay on the rank (prop_idx).
// A rank's best `budget` candidates hold every one of its pages that is in
// the global top-`budget`, so the global selection is the top-`budget` of
// the gathered candidates. Concatenated in rank order they are in global
// page order, so (score descending, position ascending) is the reference's
// tie rule (lowest page first).
//
// split_gate, per row, takes the same decisions on every rank from the same
// gathered rows: lse_all over the ranks; the lazy gate of the cached
// selection; the global top-`budget`; the new selection's log-sum-exp (its
// chosen candidates and every rank's forced pages) and gate cov >= tau;
// this rank's share of the new selection (its sink pages, its chosen
// candidates, its local pages) in ascending page order with its bitmap. The
// last CTA takes the batch decision (every head accepted the cached
// selection: backend.py:446) and counts the step, so nothing reaches the
// host and the step can be captured in a CUDA graph.
//
// Both kernels find the k-th largest candidate exactly on order-preserving
// keys: a 2048-bin histogram of the top key bits, then a direct rank of the
// keys in the bin holding it (radix passes over the low bits when that bin is
// crowded); ties at the k-th key go to the lowest positions through a block
// prefix count. Non-finite scores are never candidates.
#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

template <int NT>
__device__ __forceinline__ int block_excl(int v, int* wsum, int& total) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) wsum[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = lane < NW ? wsum[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    if (lane < NW) wsum[lane] = t;
  }
  __syncthreads();
  const int before = w == 0 ? 0 : wsum[w - 1];
  total = wsum[NW - 1];
  __syncthreads();
  return before + x - v;
}

template <int NT>
__device__ __forceinline__ int block_sum(int v, int* wsum) {
  int total;
  block_excl<NT>(v, wsum, total);
  return total;
}

// (m, s) pairs of the block combined; every thread gets the block's pair.
template <int NT>
__device__ __forceinline__ void block_lse(float& m, float& s, float* pm, float* ps) {
  constexpr int NW = NT / 32;
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  lse_warp_pair(m, s);
  if (lane == 0) {
    pm[w] = m;
    ps[w] = s;
  }
  __syncthreads();
  if (w == 0) {
    m = lane < NW ? pm[lane] : neg_inf();
    s = lane < NW ? ps[lane] : 0.f;
    lse_warp_pair(m, s);
    if (lane == 0) {
      pm[0] = m;
      ps[0] = s;
    }
  }
  __syncthreads();
  m = pm[0];
  s = ps[0];
  __syncthreads();
}

// The k-th largest nonzero key of keys[0, n) (1 <= k <= number of nonzero
// keys). One pass histograms the top 11 key bits (2048 bins) and a block scan
// finds the bin holding the k-th key; that bin's keys (usually a few dozen)
// are gathered and each ranks itself against the others. A bin too full for
// that (more than NT keys: heavy ties or a narrow score range) is resolved by
// radix passes over the remaining 21 bits (8, 8 and 5). `above` returns the
// number of keys strictly greater than the result. Scratch: hist[2048],
// bin_keys[NT], sh[6], wsum (block_excl).
constexpr int kTopBins = 2048;
constexpr int kTopShift = 21;

template <int NT>
__device__ uint32_t block_kth_key(const uint32_t* keys, int n, int k, int* hist,
                                  uint32_t* bin_keys, int* sh, int* wsum, int& above) {
  constexpr int BPT = kTopBins / NT;  // bins per thread, highest first
  const int tid = threadIdx.x, lane = tid & 31;
  for (int i = tid; i < kTopBins; i += NT) hist[i] = 0;
  __syncthreads();
  for (int i = tid; i < n; i += NT) {
    const uint32_t key = keys[i];
    if (key != 0u) atomicAdd(&hist[key >> kTopShift], 1);
  }
  __syncthreads();
  int c_sum = 0;
#pragma unroll
  for (int e = 0; e < BPT; ++e) c_sum += hist[kTopBins - 1 - (tid * BPT + e)];
  int tot;
  const int excl = block_excl<NT>(c_sum, wsum, tot);
  if (excl < k && k <= excl + c_sum) {
    int run = excl;
#pragma unroll
    for (int e = 0; e < BPT; ++e) {
      const int bin = kTopBins - 1 - (tid * BPT + e);
      const int c = hist[bin];
      if (run < k && k <= run + c) {
        sh[0] = bin;
        sh[1] = run;
        sh[2] = c;
      }
      run += c;
    }
  }
  if (tid == 0) sh[3] = 0;
  __syncthreads();
  const uint32_t top = (uint32_t)sh[0];
  int abv = sh[1];
  const int cnt = sh[2];
  if (cnt <= NT) {
    for (int i = tid; i < n; i += NT) {
      const uint32_t key = keys[i];
      if (key != 0u && (key >> kTopShift) == top) bin_keys[atomicAdd(&sh[3], 1)] = key;
    }
    __syncthreads();
    const int kk = k - abv;  // rank of the wanted key inside the bin, from 1
    if (tid < cnt) {
      const uint32_t my = bin_keys[tid];
      int g = 0, eq = 0;
      for (int j = 0; j < cnt; ++j) {
        const uint32_t v = bin_keys[j];
        g += v > my;
        eq += v == my;
      }
      if (g < kk && kk <= g + eq) {  // every key equal to the answer agrees
        sh[4] = (int)my;
        sh[5] = abv + g;
      }
    }
    __syncthreads();
    above = sh[5];
    const uint32_t T = (uint32_t)sh[4];
    __syncthreads();
    return T;
  }
  // radix passes over the low 21 bits of the keys in the bin
  uint32_t prefix = top << kTopShift, mask = ~0u << kTopShift;
#pragma unroll
  for (int pass = 0; pass < 3; ++pass) {
    const int shift = pass == 0 ? 13 : pass == 1 ? 5 : 0;
    const int nb = pass == 2 ? 32 : 256, bpl = nb / 32;
    const uint32_t dmask = (uint32_t)nb - 1u;
    for (int i = tid; i < nb; i += NT) hist[i] = 0;
    __syncthreads();
    for (int i0 = 0; i0 < n; i0 += NT) {
      const int i = i0 + tid;
      const uint32_t key = i < n ? keys[i] : 0u;
      const bool in = key != 0u && (key & mask) == prefix;
      const unsigned act = __ballot_sync(0xffffffffu, in);
      if (in) {
        const uint32_t d = (key >> shift) & dmask;
        const unsigned peers = __match_any_sync(act, d);
        if (lane == __ffs(peers) - 1) atomicAdd(&hist[d], __popc(peers));
      }
    }
    __syncthreads();
    if (tid < 32) {
      // lane holds bins nb - 1 - bpl lane - e (e < bpl), highest digits first
      int c[8], sum = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        c[e] = e < bpl ? hist[nb - 1 - bpl * lane - e] : 0;
        sum += c[e];
      }
      int incl = sum;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int ex = incl - sum, need = k - abv;
      if (ex < need && need <= incl) {
        int run = ex;
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (e < bpl && run < need && need <= run + c[e]) {
            sh[0] = nb - 1 - bpl * lane - e;
            sh[1] = run;
          }
          run += c[e];
        }
      }
    }
    __syncthreads();
    prefix |= (uint32_t)sh[0] << shift;
    mask |= dmask << shift;
    abv += sh[1];
    __syncthreads();
  }
  above = abv;
  return prefix;
}

__device__ __forceinline__ uint32_t cand_key(float s) {
  return isfinite(s) ? float_key(s) : 0u;
}

constexpr int kSplitNT = 256;
constexpr int kSplitSmemCap = 200 * 1024;  // dynamic shared memory of one CTA

// ---------------------------------------------------------------------------
// split_propose: one CTA per (b, h) row; keys of the row in shared memory
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(NT) split_propose_kernel(const __grid_constant__ SplitProposeParams p) {
  extern __shared__ uint32_t keys[];  // [W]
  __shared__ int hist[kTopBins];
  __shared__ uint32_t bin_keys[NT];
  __shared__ int sh[6];
  __shared__ int wsum[NT / 32];
  __shared__ float pm[NT / 32], ps[NT / 32];
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x;
  const int b = row / p.H, W = p.W;
  const int nv = min(n_valid_pages(p.lens[b], p.bs), W);
  const int f_hi = min(p.sink, nv);              // forced sink pages [0, f_hi)
  const int t_lo = max(nv - p.local, f_hi);      // forced local pages [t_lo, nv)
  const float* sr = p.scores + (int64_t)row * W;
  float ma = neg_inf(), sa = 0.f, mf = neg_inf(), sf = 0.f, mc = neg_inf(), sc = 0.f;
  int cnt = 0;
  for (int pg = tid; pg < W; pg += NT) {
    const float s = sr[pg];
    lse_push(ma, sa, s);
    const bool forced = pg < f_hi || (pg >= t_lo && pg < nv);
    if (forced) lse_push(mf, sf, s);
    const uint32_t key = (!forced && pg < nv) ? cand_key(s) : 0u;
    keys[pg] = key;
    cnt += key != 0u;
  }
  if (p.cached_idx) {
    const int nc = min(max(p.cached_n[row], 0), p.cached_stride);
    for (int j = tid; j < nc; j += NT) {
      const int pg = p.cached_idx[(int64_t)row * p.cached_stride + j];
      if (pg >= 0 && pg < W) lse_push(mc, sc, sr[pg]);
    }
  }
  block_lse<NT>(ma, sa, pm, ps);
  block_lse<NT>(mf, sf, pm, ps);
  block_lse<NT>(mc, sc, pm, ps);
  cnt = block_sum<NT>(cnt, wsum);
  const int k = min(p.budget, cnt);
  uint32_t T = 0xffffffffu;
  int above = 0;
  if (k > 0) T = block_kth_key<NT>(keys, W, k, hist, bin_keys, sh, wsum, above);
  const int take = k - above;  // ties at T, lowest pages first
  // contiguous pages per thread, so the compaction keeps page order
  const int per = (W + NT - 1) / NT;
  const int p0 = min(tid * per, W), p1 = min(p0 + per, W);
  int my_eq = 0;
  if (k > 0)
    for (int pg = p0; pg < p1; ++pg) my_eq += keys[pg] == T;
  int tot;
  const int eq_before = block_excl<NT>(my_eq, wsum, tot);
  int my_n = 0;
  if (k > 0) {
    int e = eq_before;
    for (int pg = p0; pg < p1; ++pg) {
      const uint32_t key = keys[pg];
      if (key > T) ++my_n;
      else if (key == T && key != 0u) my_n += (e++ < take);
    }
  }
  const int slot0 = block_excl<NT>(my_n, wsum, tot);
  float* cand = p.ex + p.off_cand + (int64_t)row * p.max_sel;
  int32_t* pidx = p.prop_idx + (int64_t)row * p.max_sel;
  if (k > 0) {
    int e = eq_before, slot = slot0;
    for (int pg = p0; pg < p1; ++pg) {
      const uint32_t key = keys[pg];
      bool take_it = key > T;
      if (key == T && key != 0u) take_it = e++ < take;
      if (take_it) {
        cand[slot] = sr[pg];
        pidx[slot] = pg;
        ++slot;
      }
    }
  }
  for (int j = k + tid; j < p.max_sel; j += NT) {
    cand[j] = neg_inf();
    pidx[j] = -1;
  }
  if (tid == 0) {
    p.ex[p.off_all + row] = lse_value(ma, sa);
    p.ex[p.off_cached + row] = lse_value(mc, sc);
    p.ex[p.off_forced + row] = lse_value(mf, sf);
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------
// split_gate: one CTA per (b, h) row over the world * max_sel gathered
// candidates
// ---------------------------------------------------------------------------
template <int NT>
__global__ void __launch_bounds__(NT) split_gate_kernel(const __grid_constant__ SplitGateParams p) {
  extern __shared__ uint32_t smem[];  // keys [K] then the bitmap [bitmap_words]
  __shared__ int hist[kTopBins];
  __shared__ uint32_t bin_keys[NT];
  __shared__ int sh[6];
  __shared__ int wsum[NT / 32];
  __shared__ float pm[NT / 32], ps[NT / 32];
  __shared__ float s_lse_all;
  pdl_wait();
  const int row = blockIdx.x, tid = threadIdx.x;
  const int N = p.world, MS = p.max_sel, K = N * MS;
  uint32_t* keys = smem;
  uint32_t* sbm = smem + K;
  const int b = row / p.H;
  const int nv = min(n_valid_pages(p.lens[b], p.bs), p.W);
  const int f_hi = min(p.sink, nv);
  const int t_lo = max(nv - p.local, f_hi);
  auto cand_at = [&](int j) -> float {
    const int r = j / MS, sl = j - r * MS;
    return p.parts[(int64_t)r * p.stride + p.off_cand + (int64_t)row * MS + sl];
  };
  int cnt = 0;
  for (int j = tid; j < K; j += NT) {
    const uint32_t key = cand_key(cand_at(j));
    keys[j] = key;
    cnt += key != 0u;
  }
  for (int w = tid; w < p.bitmap_words; w += NT) sbm[w] = 0u;
  cnt = block_sum<NT>(cnt, wsum);
  const int k = min(p.budget, cnt);
  uint32_t T = 0xffffffffu;
  int above = 0;
  if (k > 0) T = block_kth_key<NT>(keys, K, k, hist, bin_keys, sh, wsum, above);
  const int take = k - above;
  const int per = (K + NT - 1) / NT;
  const int j0 = min(tid * per, K), j1 = min(j0 + per, K);
  int my_eq = 0;
  if (k > 0)
    for (int j = j0; j < j1; ++j) my_eq += keys[j] == T;
  int tot;
  const int eq_before = block_excl<NT>(my_eq, wsum, tot);
  // chosen candidates: their log-sum-exp, and the ones in this rank's block
  const int mlo = p.rank * MS, mhi = mlo + MS;
  float ms = neg_inf(), ss = 0.f;
  int my_mine = 0;
  if (k > 0) {
    int e = eq_before;
    for (int j = j0; j < j1; ++j) {
      const uint32_t key = keys[j];
      bool ch = key > T;
      if (key == T && key != 0u) ch = e++ < take;
      if (ch) {
        lse_push(ms, ss, cand_at(j));
        my_mine += (j >= mlo && j < mhi);
      }
    }
  }
  int n_mine;
  const int mine_before = block_excl<NT>(my_mine, wsum, n_mine);
  block_lse<NT>(ms, ss, pm, ps);
  int32_t* sel = p.sel + (int64_t)row * MS;
  const int32_t* pidx = p.prop_idx + (int64_t)row * MS;
  if (k > 0 && my_mine > 0) {
    int e = eq_before, slot = f_hi + mine_before;
    for (int j = j0; j < j1; ++j) {
      const uint32_t key = keys[j];
      bool ch = key > T;
      if (key == T && key != 0u) ch = e++ < take;
      if (ch && j >= mlo && j < mhi) {
        const int pg = pidx[j - mlo];
        if (pg < 0 || pg >= p.W) {
          set_dev_error(p.dev_err, CVSA_DEV_ERR_PAGE_RANGE);
        } else {
          sel[slot] = pg;
          atomicOr(&sbm[pg >> 5], 1u << (pg & 31));
        }
        ++slot;
      }
    }
  }
  const int n_tail = nv - t_lo;
  const int n_sel = f_hi + n_mine + n_tail;  // <= sink + budget + local <= max_sel
  for (int i = tid; i < f_hi; i += NT) {
    sel[i] = i;
    atomicOr(&sbm[i >> 5], 1u << (i & 31));
  }
  for (int i = tid; i < n_tail; i += NT) {
    const int pg = t_lo + i;
    sel[f_hi + n_mine + i] = pg;
    atomicOr(&sbm[pg >> 5], 1u << (pg & 31));
  }
  for (int i = n_sel + tid; i < MS; i += NT) sel[i] = 0;
  __syncthreads();
  if (p.bitmap)
    for (int w = tid; w < p.bitmap_words; w += NT)
      p.bitmap[(int64_t)row * p.bitmap_words + w] = sbm[w];
  if (tid == 0) {
    // the gate of coverage.py:160-215 over the ranks' sums, in rank order
    float ma = neg_inf(), sa = 0.f, mc = neg_inf(), sc = 0.f;
    for (int r = 0; r < N; ++r) {
      const float* pr = p.parts + (int64_t)r * p.stride;
      lse_push(ma, sa, pr[p.off_all + row]);
      lse_push(mc, sc, pr[p.off_cached + row]);
      lse_push(ms, ss, pr[p.off_forced + row]);
    }
    const float lse_all = lse_value(ma, sa);
    s_lse_all = lse_all;
    const bool acc1 = expf(lse_value(ms, ss) - lse_all) >= p.tau;
    p.n[row] = n_sel;
    p.acc[row] = acc1 ? 1 : 0;
    const bool acc0 = p.has_cache && expf(lse_value(mc, sc) - lse_all) >= p.tau;
    if (acc0) atomicAdd(&p.state[1], 1);
    if (acc1) atomicAdd(&p.state[2], 1);
    __threadfence();
    const int ticket = atomicAdd(&p.state[0], 1);
    if (ticket == (int)gridDim.x - 1) {
      __threadfence();
      const int n0 = atomicAdd(&p.state[1], 0), n1 = atomicAdd(&p.state[2], 0);
      const int rows = (int)gridDim.x;
      const bool reuse = p.has_cache && n0 == rows;
      p.state[3] = reuse ? 1 : 0;  // bit0: the cached selection is decoded
      int64_t* c = p.counters;
      if (c) {
        const bool check = (p.stats_mode & 1) != 0, lazy = (p.stats_mode & 2) != 0;
        if (check) c[CVSA_SPLIT_CTR_CHECKS] += 1;
        if (check && !p.has_cache) c[CVSA_SPLIT_CTR_REJECT] += 1;
        if (check && p.has_cache) {
          c[CVSA_SPLIT_CTR_HEADS_TOTAL] += rows;
          c[CVSA_SPLIT_CTR_HEADS_ACC] += n0;
          c[reuse ? CVSA_SPLIT_CTR_ACCEPT : CVSA_SPLIT_CTR_REJECT] += 1;
          if (!reuse) c[CVSA_SPLIT_CTR_SCORING] += 1;
        } else {
          c[CVSA_SPLIT_CTR_SCORING] += 1;
        }
        if (!lazy) {
          c[CVSA_SPLIT_CTR_HEADS_ACC] += n1;
          c[CVSA_SPLIT_CTR_HEADS_TOTAL] += rows;
        }
      }
      p.state[0] = 0;
      p.state[1] = 0;
      p.state[2] = 0;
    }
  }
  pdl_launch_dependents();
}

}  // namespace

size_t split_propose_smem(int W) { return (size_t)W * 4; }

size_t split_gate_smem(int world, int max_sel, int bitmap_words) {
  return (size_t)world * max_sel * 4 + (size_t)bitmap_words * 4;
}

cudaError_t launch_split_propose(const SplitProposeParams& p, cudaStream_t s, bool pdl) {
  if (p.rows <= 0) return cudaSuccess;
  const size_t smem = split_propose_smem(p.W);
  if (smem > (size_t)kSplitSmemCap) return cudaErrorInvalidValue;
  if (p.W > 2048) {
    auto k = split_propose_kernel<1024>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(p.rows), dim3(1024), smem, s, pdl, p);
  }
  auto k = split_propose_kernel<kSplitNT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(p.rows), dim3(kSplitNT), smem, s, pdl, p);
}

cudaError_t launch_split_gate(const SplitGateParams& p, cudaStream_t s, bool pdl) {
  if (p.rows <= 0) return cudaSuccess;
  if (p.bitmap_words < (p.W + 31) / 32) return cudaErrorInvalidValue;
  const size_t smem = split_gate_smem(p.world, p.max_sel, p.bitmap_words);
  if (smem > (size_t)kSplitSmemCap) return cudaErrorInvalidValue;
  if ((long long)p.world * p.max_sel > 2048) {
    auto k = split_gate_kernel<1024>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem);
    if (e != cudaSuccess) return e;
    return launch_k(k, dim3(p.rows), dim3(1024), smem, s, pdl, p);
  }
  auto k = split_gate_kernel<kSplitNT>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  return launch_k(k, dim3(p.rows), dim3(kSplitNT), smem, s, pdl, p);
}

}  // namespace cvsa
