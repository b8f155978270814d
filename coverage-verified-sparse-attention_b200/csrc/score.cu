// Page scoring: score[b,h,p] = max_t (q_rep[b,h] . K[blk(b,p), t, h, :]) * D^-0.5
//
// Restates cvsa/kernels/page_scores.py:13-74 (one Triton program per page) as
// an HBM-streaming kernel. The whole cost is reading every valid page's K
// once, so the kernel is shaped for bandwidth:
//   * a warp owns (sequence b, group of HPW kv heads, chunk of pages); lanes
//     are split into HPW groups of LPR lanes, one group per head, each lane
//     covering 16 bytes of head_dim;
//   * for a page, each lane issues BS independent 16-byte loads (one per
//     token row; a warp instruction reads HPW adjacent rows = 512 contiguous
//     bytes for Llama geometry), so BS*16 B per lane are in flight;
//   * the BS partial dot products of a lane are reduced across the LPR lanes
//     of its head with a butterfly that halves the value count at every
//     shuffle step (BS-1 shuffles for BS tokens instead of BS*log2(LPR)),
//     leaving one full dot product per lane; then the max over tokens.
// q_rep is the mean of the G query heads of the group computed in fp32 and
// rounded to q's dtype, as torch does for q.view(B,Hkv,G,D).mean(2) on CUDA
// (page_scores.py:94-95). The dot is fp32; the scale is applied after the max
// (fp32 rounding is monotone, so this equals max of scaled dots).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kScoreWarps = 8;
constexpr int kPagesPerUnit = 8;

template <typename TQ, int VN>
__device__ __forceinline__ void load_q_slice(const TQ* p, float* f) {
  // VN consecutive elements of TQ (16 B for 16-bit types with VN = 8).
#pragma unroll
  for (int i = 0; i < VN; ++i) f[i] = Elem<TQ>::to_f(p[i]);
}

// Butterfly multi-reduction: v[0..N) are partial sums (one per token) of this
// lane's slice; the L lanes of an aligned group hold slices of the same
// tokens. After the call, lane holds max(N/L,1) complete sums in v[0..),
// for the tokens given by butterfly_token().
template <int N, int L>
__device__ __forceinline__ void butterfly(float (&v)[N], int lane) {
  int n = N;
#pragma unroll
  for (int off = L / 2; off >= 1; off >>= 1) {
    if (n > 1) {
      const bool upper = (lane & off) != 0;
      const int h = n / 2;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        if (i < h) {
          float send = upper ? v[i] : v[i + h];
          float keep = upper ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
      }
      n = h;
    } else {
      v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
    }
  }
}

template <int N, int L>
__device__ __forceinline__ int butterfly_token(int lane, int i) {
  constexpr int S = (L >= 32) ? 5 : (L >= 16) ? 4 : (L >= 8) ? 3 : (L >= 4) ? 2 : (L >= 2) ? 1 : 0;
  constexpr int LN = (N >= 32) ? 5 : (N >= 16) ? 4 : (N >= 8) ? 3 : (N >= 4) ? 2 : (N >= 2) ? 1 : 0;
  constexpr int H = S < LN ? S : LN;
  constexpr int MB = LN - H;  // log2 of values left per lane
  return (((lane >> (S - H)) & ((1 << H) - 1)) << MB) | i;
}

template <typename T, typename TQ, int D, int BS>
__global__ void __launch_bounds__(kScoreWarps * 32)
score_pages_kernel(const TQ* __restrict__ q, const T* __restrict__ kc,
                   const int32_t* __restrict__ tables, const int32_t* __restrict__ lens,
                   float* __restrict__ scores, int32_t* dev_err, int B, int hq, int hkv,
                   int W, int num_blocks, int64_t sb, int64_t st, int64_t sh, float scale,
                   int n_chunks, int n_hgroups) {
  constexpr int VN = 16 / sizeof(T);          // elements per 16-byte vector
  constexpr int LPR = D / VN;                 // lanes per head row
  constexpr int HPW = 32 / LPR;               // heads per warp
  constexpr int M = (BS / LPR) > 0 ? (BS / LPR) : 1;  // sums left per lane
  static_assert(LPR >= 1 && LPR <= 32 && (32 % LPR) == 0, "head_dim not supported");

  pdl_wait();

  const int lane = threadIdx.x & 31;
  const int sub = lane % LPR;         // lane within head group
  const int hl = lane / LPR;          // head within warp
  const int G = hq / hkv;
  const int warp_global = blockIdx.x * kScoreWarps + (threadIdx.x >> 5);
  const int total_warps = gridDim.x * kScoreWarps;
  const int total_units = B * n_chunks * n_hgroups;

  for (int u = warp_global; u < total_units; u += total_warps) {
    const int hg = u % n_hgroups;
    const int rest = u / n_hgroups;
    const int chunk = rest % n_chunks;
    const int b = rest / n_chunks;
    const int h = hg * HPW + hl;
    const bool head_ok = h < hkv;
    const int ctx = lens[b];
    const int nv = n_valid_pages(ctx, BS);
    const int p0 = chunk * kPagesPerUnit;
    const int p1 = min(p0 + kPagesPerUnit, W);
    float* srow = scores + ((int64_t)b * hkv + (head_ok ? h : 0)) * W;

    // q_rep slice for (b, h): sum over the group in order, * (1/G), rounded.
    float qf[VN];
    if (head_ok && p0 < nv) {
      float acc[VN];
#pragma unroll
      for (int i = 0; i < VN; ++i) acc[i] = 0.f;
      const TQ* qb = q + ((int64_t)b * hq + (int64_t)h * G) * D + sub * VN;
      for (int g = 0; g < G; ++g) {
        float t[VN];
        load_q_slice<TQ, VN>(qb + (int64_t)g * D, t);
#pragma unroll
        for (int i = 0; i < VN; ++i) acc[i] = (g == 0) ? t[i] : acc[i] + t[i];
      }
      const float inv = 1.0f / (float)G;
#pragma unroll
      for (int i = 0; i < VN; ++i) qf[i] = Elem<TQ>::to_f(Elem<TQ>::from_f(acc[i] * inv));
    }

    // the unit's block-table entries, one per lane, fetched together up front
    const int my_blk = (p0 + lane < min(p1, nv)) ? tables[(int64_t)b * W + p0 + lane] : -1;
    for (int p = p0; p < p1; ++p) {
      const int blk = __shfl_sync(0xffffffffu, my_blk, p - p0);
      if (p >= nv) {
        if (head_ok && sub == 0) srow[p] = neg_inf();
        continue;
      }
      const bool blk_ok = blk >= 0 && blk < num_blocks;
      if (!blk_ok) {
        if (lane == 0) set_dev_error(dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
        if (head_ok && sub == 0) srow[p] = neg_inf();
        continue;
      }
      const int ntok = min(BS, ctx - p * BS);
      float v[BS];
      if (head_ok) {
        const T* base = kc + (int64_t)blk * sb + (int64_t)h * sh + sub * VN;
        uint4 raw[BS];
#pragma unroll
        for (int t = 0; t < BS; ++t) raw[t] = ldg_stream16(base + (int64_t)t * st);
#pragma unroll
        for (int t = 0; t < BS; ++t) {
          float kf[VN];
          Vec16<T>::unpack(raw[t], kf);
          float a = 0.f;
#pragma unroll
          for (int i = 0; i < VN; ++i) a = fmaf(qf[i], kf[i], a);
          v[t] = a;
        }
      } else {
#pragma unroll
        for (int t = 0; t < BS; ++t) v[t] = 0.f;
      }
      butterfly<BS, LPR>(v, lane);
      float mx = neg_inf();
#pragma unroll
      for (int i = 0; i < M; ++i) {
        const int tok = butterfly_token<BS, LPR>(lane, i);
        if (tok < ntok) mx = fmaxf(mx, v[i]);
      }
#pragma unroll
      for (int off = LPR / 2; off >= 1; off >>= 1)
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (head_ok && sub == 0) srow[p] = mx * scale;
    }
  }
  pdl_launch_dependents();
}

template <typename T, typename TQ, int D, int BS>
cudaError_t launch_typed(const QView& q, const KvView& kv, float* scores, int32_t* dev_err,
                         cudaStream_t s, bool pdl) {
  constexpr int VN = 16 / sizeof(T);
  constexpr int LPR = D / VN;
  constexpr int HPW = 32 / LPR;
  const int n_chunks = (q.W + kPagesPerUnit - 1) / kPagesPerUnit;
  const int n_hgroups = (kv.hkv + HPW - 1) / HPW;
  const long long units = (long long)q.B * n_chunks * n_hgroups;
  if (units == 0) return cudaSuccess;
  const int warps_needed = (int)((units + 0) );
  int blocks = (warps_needed + kScoreWarps - 1) / kScoreWarps;
  const int cap = num_sms() * 8;
  if (blocks > cap) blocks = cap;
  const float scale = 1.0f / sqrtf((float)D);
  return launch_k(score_pages_kernel<T, TQ, D, BS>, dim3(blocks), dim3(kScoreWarps * 32), 0, s,
                  pdl, (const TQ*)q.q, (const T*)kv.k, q.tables, q.lens, scores, dev_err, q.B,
                  q.hq, kv.hkv, q.W, kv.num_blocks, kv.sb, kv.st, kv.sh, scale, n_chunks,
                  n_hgroups);
}

template <typename T, typename TQ>
cudaError_t dispatch_d(const QView& q, const KvView& kv, float* scores, int32_t* dev_err,
                       cudaStream_t s, bool pdl) {
  if (kv.bs != 16) return cudaErrorInvalidValue;
  switch (kv.d) {
    case 64: return launch_typed<T, TQ, 64, 16>(q, kv, scores, dev_err, s, pdl);
    case 128: return launch_typed<T, TQ, 128, 16>(q, kv, scores, dev_err, s, pdl);
    case 256:
      if (sizeof(T) == 4) return cudaErrorInvalidValue;
      return launch_typed<T, TQ, (sizeof(T) == 4 ? 128 : 256), 16>(q, kv, scores, dev_err, s,
                                                                     pdl);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t dispatch_q(const QView& q, const KvView& kv, float* scores, int32_t* dev_err,
                       cudaStream_t s, bool pdl) {
  switch (q.dtype) {
    case CVSA_DTYPE_BF16: return dispatch_d<T, __nv_bfloat16>(q, kv, scores, dev_err, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_d<T, __half>(q, kv, scores, dev_err, s, pdl);
    case CVSA_DTYPE_F32: return dispatch_d<T, float>(q, kv, scores, dev_err, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

bool score_supported(const QView& q, const KvView& kv) {
  if (kv.bs != 16) return false;
  if (kv.d != 64 && kv.d != 128 && kv.d != 256) return false;
  if (kv.dtype == CVSA_DTYPE_F32 && kv.d == 256) return false;
  return true;
}

cudaError_t launch_score_pages(const QView& q, const KvView& kv, float* scores,
                               int32_t* dev_err, cudaStream_t s, bool pdl) {
  switch (kv.dtype) {
    case CVSA_DTYPE_BF16: return dispatch_q<__nv_bfloat16>(q, kv, scores, dev_err, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_q<__half>(q, kv, scores, dev_err, s, pdl);
    case CVSA_DTYPE_F32: return dispatch_q<float>(q, kv, scores, dev_err, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cvsa
