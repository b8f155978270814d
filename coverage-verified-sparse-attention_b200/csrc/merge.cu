// Selective LSE merge of draft and complement partials.
//
// Restates cvsa/kernels/coverage.py:274-326 (and cvsa/lse_merge.py:11-54):
// accepted heads o_d / max(l_d, 1e-6); rejected heads
// (o_d e^{m_d-M} + o_c e^{m_c-M}) / max(l_d e^{m_d-M} + l_c e^{m_c-M}, 1e-6)
// with M = max(m_d, m_c). The accept mask is per KV head, expanded over its G
// query heads (q head index // G). One warp per query head, 16-byte stores.
// A side whose m is -inf carries no mass (the reference would form NaN from
// exp(-inf - -inf) there; its merge kernel never sees that case because
// accepted heads skip this branch).
#include "cvsa_common.cuh"
#include "cvsa_internal.h"

namespace cvsa {
namespace {

template <typename TO>
__global__ void lse_merge_kernel(const float* __restrict__ o_d, const float* __restrict__ m_d,
                                 const float* __restrict__ l_d, const float* __restrict__ o_c,
                                 const float* __restrict__ m_c, const float* __restrict__ l_c,
                                 const uint8_t* __restrict__ accept, int rows, int hq, int G,
                                 int D, TO* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int b = row / hq;
  const int qh = row % hq;
  const int kvh = qh / G;
  const int hkv = hq / G;
  const bool acc = accept[b * hkv + kvh] != 0;
  const float md = m_d[row], ld = l_d[row];
  float sd = 1.f, sc = 0.f, denom;
  if (acc) {
    denom = fmaxf(ld, 1e-6f);
  } else {
    const float mc = m_c[row], lc = l_c[row];
    const float M = fmaxf(md, mc);
    sd = (md == neg_inf()) ? 0.f : expf(md - M);
    sc = (mc == neg_inf()) ? 0.f : expf(mc - M);
    denom = fmaxf(ld * sd + lc * sc, 1e-6f);
  }
  for (int d = lane; d < D; d += 32) {
    const int64_t i = (int64_t)row * D + d;
    float v = o_d[i] * sd;
    if (!acc) v += o_c[i] * sc;
    out[i] = Elem<TO>::from_f(v / denom);
  }
}

// Fixed-order merge over the ranks of a page split: `world` exchanged rows of
// `stride` floats, row r = [o_unnorm rows*D | m rows | l rows] of rank r.
// M = max_r m_r, w_r = exp(m_r - M) (0 where m_r = -inf, M taken as 0 when
// every m_r is -inf), out = sum_r w_r o_r / max(sum_r w_r l_r, 1e-6), summed
// in rank order. One warp per query-head row; rows whose KV head has
// need == 0 are left untouched when `need` is given.
template <typename TO>
__global__ void rank_merge_kernel(const float* __restrict__ parts, int world, int64_t stride,
                                  int rows, int hq, int G, int D,
                                  const uint8_t* __restrict__ need, TO* __restrict__ out) {
  const int row = blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  if (need != nullptr) {
    const int b = row / hq;
    if (need[b * (hq / G) + (row % hq) / G] == 0) return;
  }
  const int64_t m_off = (int64_t)rows * D;
  const int64_t l_off = m_off + rows;
  float M = neg_inf();
  for (int r = 0; r < world; ++r) M = fmaxf(M, parts[r * stride + m_off + row]);
  const float base = (M == neg_inf()) ? 0.f : M;
  float L = 0.f;
  for (int r = 0; r < world; ++r) {
    const float mr = parts[r * stride + m_off + row];
    if (mr != neg_inf()) L += parts[r * stride + l_off + row] * expf(mr - base);
  }
  const float denom = fmaxf(L, 1e-6f);
  for (int d = lane; d < D; d += 32) {
    float v = 0.f;
    for (int r = 0; r < world; ++r) {
      const float mr = parts[r * stride + m_off + row];
      if (mr != neg_inf()) v += parts[r * stride + (int64_t)row * D + d] * expf(mr - base);
    }
    out[(int64_t)row * D + d] = Elem<TO>::from_f(v / denom);
  }
}

// Per (sequence, KV head) row of page scores: log-sum-exp over the W entries
// (-inf entries carry no mass) and over the first n entries of the row's
// selection (entries outside [0, W) are skipped); -inf when empty. One CTA
// of kLseThreads per row (a row can hold thousands of pages): an online
// (max, sum) per thread, combined across each warp and then across warps.
constexpr int kLseThreads = 256;

__global__ void __launch_bounds__(kLseThreads)
page_lse_kernel(const float* __restrict__ scores, int W, const int32_t* __restrict__ idx,
                int max_sel, const int32_t* __restrict__ n, float* __restrict__ lse_all,
                float* __restrict__ lse_sel) {
  constexpr int kWarps = kLseThreads / 32;
  __shared__ float part_m[2][kWarps], part_s[2][kWarps];
  const int row = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const float* sr = scores + (int64_t)row * W;
  float ma = neg_inf(), sa = 0.f, msel = neg_inf(), ssel = 0.f;
  for (int p = threadIdx.x; p < W; p += kLseThreads) lse_push(ma, sa, sr[p]);
  const int cnt = min(n[row], max_sel);
  for (int j = threadIdx.x; j < cnt; j += kLseThreads) {
    const int p = idx[(int64_t)row * max_sel + j];
    if (p >= 0 && p < W) lse_push(msel, ssel, sr[p]);
  }
  lse_warp_pair(ma, sa);
  lse_warp_pair(msel, ssel);
  if (lane == 0) {
    part_m[0][warp] = ma;
    part_s[0][warp] = sa;
    part_m[1][warp] = msel;
    part_s[1][warp] = ssel;
  }
  __syncthreads();
  if (warp == 0) {
    ma = lane < kWarps ? part_m[0][lane] : neg_inf();
    sa = lane < kWarps ? part_s[0][lane] : 0.f;
    msel = lane < kWarps ? part_m[1][lane] : neg_inf();
    ssel = lane < kWarps ? part_s[1][lane] : 0.f;
    lse_warp_pair(ma, sa);
    lse_warp_pair(msel, ssel);
    if (lane == 0) {
      lse_all[row] = lse_value(ma, sa);
      lse_sel[row] = lse_value(msel, ssel);
    }
  }
}

// The coverage gate over the ranks of a page split: row i's coverage is
// exp(LSE_r sel_r - LSE_r all_r) over the gathered per-rank log-sum-exps
// (rank r's values at parts[r * stride + off_all + i] and off_sel + i);
// accept[i] = coverage >= tau.
__global__ void rank_accept_kernel(const float* __restrict__ parts, int world, int64_t stride,
                                   int64_t off_all, int64_t off_sel, int rows, float tau,
                                   uint8_t* __restrict__ accept) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows) return;
  float ma = neg_inf(), sa = 0.f, ms = neg_inf(), ss = 0.f;
  for (int r = 0; r < world; ++r) {
    lse_push(ma, sa, parts[r * stride + off_all + i]);
    lse_push(ms, ss, parts[r * stride + off_sel + i]);
  }
  accept[i] = expf(lse_value(ms, ss) - lse_value(ma, sa)) >= tau ? 1 : 0;
}

}  // namespace

cudaError_t launch_lse_merge(const float* o_d, const float* m_d, const float* l_d,
                             const float* o_c, const float* m_c, const float* l_c,
                             const uint8_t* accept, int B, int hkv, int G, int D, void* out,
                             int out_dtype, cudaStream_t s) {
  const int rows = B * hkv * G;
  if (rows == 0) return cudaSuccess;
  const int wpb = 8;
  const int grid = (rows + wpb - 1) / wpb;
  const int hq = hkv * G;
  switch (out_dtype) {
    case CVSA_DTYPE_BF16:
      lse_merge_kernel<<<grid, wpb * 32, 0, s>>>(o_d, m_d, l_d, o_c, m_c, l_c, accept, rows, hq,
                                                 G, D, (__nv_bfloat16*)out);
      break;
    case CVSA_DTYPE_F16:
      lse_merge_kernel<<<grid, wpb * 32, 0, s>>>(o_d, m_d, l_d, o_c, m_c, l_c, accept, rows, hq,
                                                 G, D, (__half*)out);
      break;
    case CVSA_DTYPE_F32:
      lse_merge_kernel<<<grid, wpb * 32, 0, s>>>(o_d, m_d, l_d, o_c, m_c, l_c, accept, rows, hq,
                                                 G, D, (float*)out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_rank_merge(const float* parts, int world, int64_t stride, int B, int hkv,
                              int G, int D, const uint8_t* need, void* out, int out_dtype,
                              cudaStream_t s) {
  const int rows = B * hkv * G;
  if (rows == 0) return cudaSuccess;
  const int wpb = 8;
  const int grid = (rows + wpb - 1) / wpb;
  const int hq = hkv * G;
  switch (out_dtype) {
    case CVSA_DTYPE_BF16:
      rank_merge_kernel<<<grid, wpb * 32, 0, s>>>(parts, world, stride, rows, hq, G, D, need,
                                                  (__nv_bfloat16*)out);
      break;
    case CVSA_DTYPE_F16:
      rank_merge_kernel<<<grid, wpb * 32, 0, s>>>(parts, world, stride, rows, hq, G, D, need,
                                                  (__half*)out);
      break;
    case CVSA_DTYPE_F32:
      rank_merge_kernel<<<grid, wpb * 32, 0, s>>>(parts, world, stride, rows, hq, G, D, need,
                                                  (float*)out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t launch_page_lse(const float* scores, int rows, int W, const int32_t* idx,
                            int max_sel, const int32_t* n, float* lse_all, float* lse_sel,
                            cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  page_lse_kernel<<<rows, kLseThreads, 0, s>>>(scores, W, idx, max_sel, n, lse_all, lse_sel);
  return cudaGetLastError();
}

cudaError_t launch_rank_accept(const float* parts, int world, int64_t stride, int64_t off_all,
                               int64_t off_sel, int rows, float tau, uint8_t* accept,
                               cudaStream_t s) {
  if (rows == 0) return cudaSuccess;
  rank_accept_kernel<<<(rows + 127) / 128, 128, 0, s>>>(parts, world, stride, off_all, off_sel,
                                                         rows, tau, accept);
  return cudaGetLastError();
}

}  // namespace cvsa
