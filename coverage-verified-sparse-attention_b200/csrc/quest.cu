// Quest page ranking: score[b,h,p] = sum_d max(q_d kmin_d, q_d kmax_d) * D^-0.5
//
// Restates cvsa/backend.py:572-620 (_quest_page_scores, the Quest upper bound
// of Tang et al., ICML 2024): for each page and KV head, the channel-wise
// minimum and maximum of the keys of its valid tokens (tokens at or past the
// context length are left out), then the upper bound of q . k over the box
// they span, with q the group mean of the query heads rounded to q's dtype
// (the pooling of page scoring, page_scores.py:94-95). Pages without a valid
// token score -inf. The products and the sum are fp32 (the reference casts
// the bounds and q_rep to fp32 before multiplying).
//
// The cost is one read of every valid page's keys, so the kernel is laid out
// like the general scoring kernel: a CTA owns one sequence and a chunk of
// kChunk consecutive pages; its q_rep rows (every KV head) are computed once
// into shared memory; each warp takes pages of the chunk in turn and, for
// every KV head, issues the 16-byte loads of all 16 token rows at once (lanes
// split into token-row groups of D / VN lanes), folds min / max over its rows,
// combines the row groups with shuffles, and reduces the bound over the lanes
// of a row.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kQuestWarps = 4;
constexpr int kChunk = 32;   // pages per CTA
constexpr int kBS = 16;      // tokens per page

struct QuestArgs {
  const void* q;
  const void* k;
  const int32_t* tables;
  const int32_t* lens;
  float* scores;
  int32_t* dev_err;
  int B, hq, hkv, W, num_blocks;
  int64_t sb, st, sh;  // pool strides (elements)
  float scale;
};

template <typename T, typename TQ, int D>
__global__ void __launch_bounds__(kQuestWarps * 32) quest_scores_kernel(QuestArgs a) {
  constexpr int VN = 16 / (int)sizeof(T);   // channels per 16-byte chunk
  constexpr int LPR = D / VN;               // lanes per token row
  constexpr int TPI = 32 / LPR;             // token rows per load instruction
  constexpr int NI = kBS / TPI;             // load instructions per (page, head)
  static_assert(LPR >= 1 && LPR <= 32 && 32 % LPR == 0, "head_dim not supported");

  extern __shared__ float qrep[];           // [hkv][D]
  const int b = blockIdx.y;
  const int p0 = blockIdx.x * kChunk;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = a.hq / a.hkv;
  pdl_wait();
  const int ctx = a.lens[b];
  const int nv = min(n_valid_pages(ctx, kBS), a.W);

  // q_rep rows: the group's query heads summed in order, times 1/G, rounded
  // to q's dtype (torch's fp32 mean on the device, page_scores.py:94-95)
  const float inv = 1.0f / (float)G;
  const TQ* q = reinterpret_cast<const TQ*>(a.q) + (int64_t)b * a.hq * D;
  for (int i = threadIdx.x; i < a.hkv * D; i += blockDim.x) {
    const int h = i / D, d = i % D;
    float acc = 0.f;
    for (int g = 0; g < G; ++g) {
      const float t = Elem<TQ>::to_f(q[(int64_t)(h * G + g) * D + d]);
      acc = g == 0 ? t : acc + t;
    }
    qrep[i] = Elem<TQ>::to_f(Elem<TQ>::from_f(acc * inv));
  }
  __syncthreads();
  pdl_launch_dependents();

  const int row = lane / LPR;        // token row within a load instruction
  const int c0 = (lane % LPR) * VN;  // first channel of the lane
  const T* K = reinterpret_cast<const T*>(a.k);
  for (int p = p0 + warp; p < min(p0 + kChunk, a.W); p += kQuestWarps) {
    float* srow = a.scores + (int64_t)b * a.hkv * a.W + p;
    int blk = -1;
    if (p < nv) {
      blk = a.tables[(int64_t)b * a.W + p];
      if (blk < 0 || blk >= a.num_blocks) {
        if (lane == 0) set_dev_error(a.dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
        blk = -1;
      }
    }
    if (blk < 0) {
      // no valid token (past the context, or a block outside the pool)
      for (int h = lane; h < a.hkv; h += 32) srow[(int64_t)h * a.W] = neg_inf();
      continue;
    }
    const int ntok = min(kBS, ctx - p * kBS);
    for (int h = 0; h < a.hkv; ++h) {
      const T* base = K + (int64_t)blk * a.sb + (int64_t)h * a.sh + c0;
      uint4 raw[NI];
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        const int t = i * TPI + row;
        raw[i] = t < ntok ? ldg_stream16(base + (int64_t)t * a.st) : make_uint4(0, 0, 0, 0);
      }
      float mn[VN], mx[VN];
#pragma unroll
      for (int j = 0; j < VN; ++j) {
        mn[j] = __int_as_float(0x7f800000);
        mx[j] = neg_inf();
      }
#pragma unroll
      for (int i = 0; i < NI; ++i) {
        if (i * TPI + row < ntok) {
          float f[VN];
          Vec16<T>::unpack(raw[i], f);
#pragma unroll
          for (int j = 0; j < VN; ++j) {
            mn[j] = fminf(mn[j], f[j]);
            mx[j] = fmaxf(mx[j], f[j]);
          }
        }
      }
      // combine the row groups (lanes lane ^ LPR, ^ 2 LPR, ... hold the same
      // channels of other token rows)
#pragma unroll
      for (int off = LPR; off < 32; off <<= 1) {
#pragma unroll
        for (int j = 0; j < VN; ++j) {
          mn[j] = fminf(mn[j], __shfl_xor_sync(0xffffffffu, mn[j], off));
          mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], off));
        }
      }
      float s = 0.f;
      const float* qr = qrep + h * D + c0;
#pragma unroll
      for (int j = 0; j < VN; ++j) s += fmaxf(qr[j] * mn[j], qr[j] * mx[j]);
#pragma unroll
      for (int off = LPR / 2; off >= 1; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0) srow[(int64_t)h * a.W] = s * a.scale;
    }
  }
}

template <typename T, typename TQ>
cudaError_t launch_d(const QuestArgs& a, int d, cudaStream_t s, bool pdl) {
  const dim3 grid((a.W + kChunk - 1) / kChunk, a.B);
  const size_t smem = (size_t)a.hkv * d * sizeof(float);
  switch (d) {
    case 64:
      return launch_k(quest_scores_kernel<T, TQ, 64>, grid, dim3(kQuestWarps * 32), smem, s, pdl, a);
    case 128:
      return launch_k(quest_scores_kernel<T, TQ, 128>, grid, dim3(kQuestWarps * 32), smem, s, pdl,
                      a);
    case 256:
      if constexpr (sizeof(T) == 4) return cudaErrorInvalidValue;
      else
        return launch_k(quest_scores_kernel<T, TQ, 256>, grid, dim3(kQuestWarps * 32), smem, s,
                        pdl, a);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
cudaError_t launch_q(const QuestArgs& a, int qdt, int d, cudaStream_t s, bool pdl) {
  switch (qdt) {
    case CVSA_DTYPE_BF16: return launch_d<T, __nv_bfloat16>(a, d, s, pdl);
    case CVSA_DTYPE_F16: return launch_d<T, __half>(a, d, s, pdl);
    case CVSA_DTYPE_F32: return launch_d<T, float>(a, d, s, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

bool quest_supported(const QView& q, const KvView& kv) {
  if (kv.bs != kBS) return false;
  if (kv.d != 64 && kv.d != 128 && kv.d != 256) return false;
  if (kv.dtype == CVSA_DTYPE_F32 && kv.d == 256) return false;
  // q_rep rows of every KV head in shared memory
  return (size_t)kv.hkv * kv.d * sizeof(float) <= 48 * 1024 && q.hq % kv.hkv == 0;
}

cudaError_t launch_quest_scores(const QView& q, const KvView& kv, float* scores,
                                int32_t* dev_err, cudaStream_t s, bool pdl) {
  if (q.B == 0 || q.W == 0) return cudaSuccess;
  QuestArgs a;
  a.q = q.q;
  a.k = kv.k;
  a.tables = q.tables;
  a.lens = q.lens;
  a.scores = scores;
  a.dev_err = dev_err;
  a.B = q.B;
  a.hq = q.hq;
  a.hkv = kv.hkv;
  a.W = q.W;
  a.num_blocks = kv.num_blocks;
  a.sb = kv.sb;
  a.st = kv.st;
  a.sh = kv.sh;
  a.scale = 1.0f / sqrtf((float)kv.d);
  switch (kv.dtype) {
    case CVSA_DTYPE_BF16: return launch_q<__nv_bfloat16>(a, q.dtype, kv.d, s, pdl);
    case CVSA_DTYPE_F16: return launch_q<__half>(a, q.dtype, kv.d, s, pdl);
    case CVSA_DTYPE_F32: return launch_q<float>(a, q.dtype, kv.d, s, pdl);
  }
  return cudaErrorInvalidValue;
}

}  // namespace cvsa
