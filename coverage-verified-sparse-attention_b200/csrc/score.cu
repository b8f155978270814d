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

#include <type_traits>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kScoreWarps = 8;
constexpr int kPagesPerUnit = 8;
constexpr int kBlk = 16;  // tokens per page

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

// ---------------------------------------------------------------------------
// Whole-page streaming variant (bf16 / f16 pools whose pages are contiguous
// blocks of 16 tokens x all KV heads): the valid pages of all sequences form
// one flat stream, cut into equal contiguous ranges, one per persistent CTA.
// A producer warp copies each page (16 * Hkv * D elements, e.g. 32 KB) into a
// shared-memory ring with one bulk copy; consumer warp w computes the page
// max of heads w, w + 8, ... from shared memory (lanes of a token row take 16
// bytes each; two rows per load instruction) with the same butterfly
// reduction as above. Large contiguous copies keep HBM at its streaming rate
// with one instruction per page.
// ---------------------------------------------------------------------------
constexpr int kSSNC = 8;          // consumer warps
constexpr int kSSMaxB = 4096;     // sequences per launch (shared-memory prefix)
constexpr int kSSMaxStages = 8;
constexpr int kSSSmemCap = 227 * 1024;

struct ScoreStreamArgs {
  const void* q;
  const void* k;
  const int32_t* tables;
  const int32_t* lens;
  float* scores;
  int32_t* dev_err;
  int B, hq, hkv, W, num_blocks;
  int64_t sb;           // block stride (elements)
  uint32_t page_bytes;  // 16 * hkv * D * sizeof(T)
  int stages;
  float scale;
};

template <typename T, typename TQ, int D>
__global__ void __launch_bounds__((kSSNC + 1) * 32, 1)
score_stream_kernel(const __grid_constant__ ScoreStreamArgs a) {
  constexpr int VN = 16 / sizeof(T);   // elements per 16-byte chunk
  constexpr int LPR = D / VN;          // lanes per token row of one head
  constexpr int TPI = 32 / LPR;        // token rows per load instruction
  constexpr int NI = 16 / TPI;         // load instructions per (head, page)
  constexpr int HPW = 2;               // heads per consumer warp (hkv <= 16)
  static_assert(LPR >= 2 && LPR <= 32 && 32 % LPR == 0, "head_dim not supported");

  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int S = a.stages;
  const uint32_t PB = a.page_bytes;
  uint8_t* ring = sm;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + (size_t)S * PB);
  uint64_t* empty = full + S;
  int2* meta = reinterpret_cast<int2*>(empty + S);  // (b, page) of a stage; page < 0: skipped
  int* bpref = reinterpret_cast<int*>(meta + S);    // [B + 1] prefix of valid pages
  int* scan = bpref + a.B + 1;                       // [33]

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nthreads = blockDim.x;
  const int C = gridDim.x, c = blockIdx.x;
  const int B = a.B, W = a.W, hkv = a.hkv;

  if (tid == 0) {
    for (int i = 0; i < S; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], kSSNC);
    }
    fence_mbar_init();
  }
  pdl_wait();
  {
    const int per = (B + nthreads - 1) / nthreads;
    const int b0 = min(tid * per, B), b1 = min(b0 + per, B);
    int sum = 0;
    for (int b = b0; b < b1; ++b) {
      const int nv = min(n_valid_pages(a.lens[b], kBlk), W);
      bpref[b] = nv;
      sum += nv;
    }
    // block exclusive scan of the per-thread sums
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) scan[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int nw = nthreads >> 5;
      const int x = lane < nw ? scan[lane] : 0;
      int xi = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, xi, o);
        if (lane >= o) xi += n;
      }
      if (lane < nw) scan[lane] = xi - x;
      if (lane == 31) scan[32] = xi;
    }
    __syncthreads();
    int base = scan[warp] + incl - sum;
    for (int b = b0; b < b1; ++b) {
      const int nv = bpref[b];
      bpref[b] = base;
      base += nv;
    }
    if (tid == 0) bpref[B] = scan[32];
  }
  __syncthreads();
  // pages past each sequence's end score -inf (rows spread over CTAs)
  for (int r = c; r < B * hkv; r += C) {
    const int b = r / hkv;
    for (int p = (bpref[b + 1] - bpref[b]) + tid; p < W; p += nthreads)
      a.scores[(int64_t)r * W + p] = neg_inf();
  }
  const int P = bpref[B];
  const int Xc = (int)((long long)P * c / C);
  const int Xe = (int)((long long)P * (c + 1) / C);
  const int n = Xe - Xc;

  if (warp == kSSNC) {
    // ================================ producer ================================
    const uint64_t policy = make_evict_first_policy();
    const T* K = reinterpret_cast<const T*>(a.k);
    int issued = 0;
    bool failed = false;
    for (int xb = 0; xb < n && !failed; xb += 32) {
      const int j = xb + lane;
      int b = 0, p = -1, blk = -1;
      if (j < n) {
        const int x = Xc + j;
        int lo = 0, hi = B - 1;  // largest b with bpref[b] <= x
        while (lo < hi) {
          const int mid = (lo + hi + 1) >> 1;
          if (bpref[mid] <= x) lo = mid;
          else hi = mid - 1;
        }
        b = lo;
        p = x - bpref[b];
        blk = a.tables[(int64_t)b * W + p];
        if (blk < 0 || blk >= a.num_blocks) {
          set_dev_error(a.dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
          blk = -1;
        }
      }
      const int cnt = min(32, n - xb);
      for (int t = 0; t < cnt; ++t) {
        const int tb = __shfl_sync(0xffffffffu, b, t);
        const int tp = __shfl_sync(0xffffffffu, p, t);
        const int tk = __shfl_sync(0xffffffffu, blk, t);
        if (lane == 0 && !failed) {
          const int jj = xb + t, st = jj % S, u = jj / S;
          if (u > 0 && !mbar_wait_bounded(&empty[st], (u - 1) & 1)) {
            failed = true;
            set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
          } else {
            meta[st] = make_int2(tb, tk >= 0 ? tp : -1 - tp);
            if (tk >= 0) {
              mbar_arrive_expect_tx(&full[st], PB);
              bulk_load(ring + (size_t)st * PB, K + (int64_t)tk * a.sb, PB, &full[st], policy);
            } else {
              mbar_arrive(&full[st]);
            }
            ++issued;
          }
        }
      }
      failed = __shfl_sync(0xffffffffu, failed ? 1 : 0, 0) != 0;
    }
    // no copy may still be landing in shared memory when the CTA exits
    if (lane == 0)
      for (int jj = max(0, issued - S); jj < issued; ++jj)
        mbar_wait_bounded(&full[jj % S], (jj / S) & 1);
    return;
  }

  // ================================ consumers ================================
  const int sub = lane % LPR, half = lane / LPR;
  const int G = a.hq / hkv;
  // KV heads to consumer warps: with hkv >= 8, warp w takes heads w and w + 8
  // of every page; with fewer heads (a rank of a head-sharded model holds one
  // or two) the warps of head h take turns over the pages, so all of them work
  const int wph = hkv >= kSSNC ? 1 : kSSNC / hkv;          // warps per head
  const int h0 = hkv >= kSSNC ? warp : warp % hkv;
  const int pslot = hkv >= kSSNC ? 0 : warp / hkv;         // my pages: j % wph == pslot
  const bool has_head = hkv >= kSSNC || warp < hkv * wph;
  int cur_b = -1, ctx = 0;
  float qf[HPW][VN];
  // q_rep slices of my heads for sequence b: mean of the group in fp32,
  // rounded to q's dtype (page_scores.py:94-95)
  auto load_qrep = [&](int b) {
    cur_b = b;
    ctx = a.lens[b];
#pragma unroll
    for (int e = 0; e < HPW; ++e) {
      const int h = h0 + e * kSSNC;
      if (h < hkv) {
        float acc[VN];
        const TQ* qb = reinterpret_cast<const TQ*>(a.q) + ((int64_t)b * a.hq + (int64_t)h * G) * D +
                       sub * VN;
        for (int g = 0; g < G; ++g) {
          float t[VN];
          load_q_slice<TQ, VN>(qb + (int64_t)g * D, t);
#pragma unroll
          for (int i = 0; i < VN; ++i) acc[i] = (g == 0) ? t[i] : acc[i] + t[i];
        }
        const float inv = 1.0f / (float)G;
#pragma unroll
        for (int i = 0; i < VN; ++i) qf[e][i] = Elem<TQ>::to_f(Elem<TQ>::from_f(acc[i] * inv));
      }
    }
  };
  if (n > 0) {
    // the first sequence's q_rep is computed while the first pages are in
    // flight (after they land its loads would queue behind the page stream);
    // the q rows of the next two sequences are prefetched into L2
    auto seq_of = [&](int x) -> int {
      int lo = 0, hi = B - 1;  // largest b with bpref[b] <= x
      while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (bpref[mid] <= x) lo = mid;
        else hi = mid - 1;
      }
      return lo;
    };
    const int b_first = seq_of(Xc), b_last = min(seq_of(Xe - 1), b_first + 2);
    const int row_bytes = a.hq * D * (int)sizeof(TQ);
    for (int b = b_first + 1; b <= b_last; ++b) {
      const char* qrow = reinterpret_cast<const char*>(a.q) + (int64_t)b * row_bytes;
      for (int off = (warp * 32 + lane) * 128; off < row_bytes; off += kSSNC * 32 * 128)
        asm volatile("prefetch.global.L2 [%0];" ::"l"(qrow + off));
    }
    load_qrep(b_first);
  }
  // the loop is compiled twice: with one warp per head (kTurns false, the
  // common case) it carries no page-ownership test at all (a runtime test
  // there measured 9 us slower per launch at config 2)
  auto consume = [&](auto turns) {
    constexpr bool kTurns = decltype(turns)::value;
    for (int j = 0; j < n; ++j) {
      const int st = j % S;
      if (!mbar_wait_bounded(&full[st], (j / S) & 1)) {
        if (lane == 0) set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
        break;
      }
      const int2 m = meta[st];
      const int b = m.x;
      const bool ok = m.y >= 0;
      const int p = ok ? m.y : -1 - m.y;
      if (b != cur_b) load_qrep(b);
      const int ntok = min(kBlk, ctx - p * kBlk);
      const bool mine = !kTurns || (has_head && (j % wph) == pslot);
  #pragma unroll
      for (int e = 0; e < HPW; ++e) {
        const int h = h0 + e * kSSNC;
        if (!mine || h >= hkv) continue;
        float mx = neg_inf();
        if (ok) {
          const uint8_t* base = ring + (size_t)st * PB + ((size_t)h * D + sub * VN) * sizeof(T);
          float v[NI];
  #pragma unroll
          for (int i = 0; i < NI; ++i) {
            const int t = i * TPI + half;
            const uint4 raw =
                *reinterpret_cast<const uint4*>(base + (size_t)t * hkv * D * sizeof(T));
            float kf[VN];
            Vec16<T>::unpack(raw, kf);
            float acc = 0.f;
  #pragma unroll
            for (int x = 0; x < VN; ++x) acc = fmaf(qf[e][x], kf[x], acc);
            v[i] = acc;
          }
          butterfly<NI, LPR>(v, lane);
          const int tok = butterfly_token<NI, LPR>(lane, 0) * TPI + half;
          mx = tok < ntok ? v[0] : neg_inf();
        }
        mx = warp_max(mx);
        if (lane == 0)
          a.scores[((int64_t)b * hkv + h) * W + p] = ok ? mx * a.scale : neg_inf();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
  };
  if (wph > 1) consume(std::true_type{});
  else consume(std::false_type{});
}

template <typename T, typename TQ, int D>
cudaError_t launch_stream_typed(const QView& q, const KvView& kv, float* scores, int32_t* dev_err,
                                cudaStream_t s, bool pdl, int stages, int smem) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(score_stream_kernel<T, TQ, D>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kSSSmemCap);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  ScoreStreamArgs a;
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
  a.page_bytes = (uint32_t)(kBlk * kv.hkv * D * sizeof(T));
  a.stages = stages;
  a.scale = 1.0f / sqrtf((float)D);
  return launch_k(score_stream_kernel<T, TQ, D>, dim3(num_sms()), dim3((kSSNC + 1) * 32),
                  (size_t)smem, s, pdl, a);
}

// Ring stages and shared memory for the streaming variant, or 0 when the
// layout does not fit it.
int stream_plan(const QView& q, const KvView& kv, int* smem) {
  const size_t pb = (size_t)kBlk * kv.hkv * kv.d * dtype_bytes(kv.dtype);
  const size_t fixed = 1024 + (size_t)(q.B + 1 + 33) * 4 + 256;
  int stages = 0;
  while (stages < kSSMaxStages &&
         fixed + (size_t)(stages + 1) * (pb + 16 + 8) <= (size_t)kSSSmemCap)
    ++stages;
  if (stages < 3) return 0;
  *smem = (int)(fixed + (size_t)stages * (pb + 24));
  return stages;
}

bool stream_eligible(const QView& q, const KvView& kv) {
  if (kv.dtype != CVSA_DTYPE_BF16 && kv.dtype != CVSA_DTYPE_F16) return false;
  if (kv.bs != kBlk || kv.hkv > kSSNC * 2 || q.B > kSSMaxB || q.B < 1) return false;
  if (kv.d != 64 && kv.d != 128 && kv.d != 256) return false;
  // a page must be one contiguous, 16-byte-aligned block
  if (kv.sh != kv.d || kv.st != (int64_t)kv.hkv * kv.d) return false;
  if ((kv.sb * 2) % 16 != 0 || (reinterpret_cast<uintptr_t>(kv.k) % 16) != 0) return false;
  int smem = 0;
  return stream_plan(q, kv, &smem) > 0;
}

template <typename T>
cudaError_t stream_dispatch_q(const QView& q, const KvView& kv, float* scores, int32_t* dev_err,
                              cudaStream_t s, bool pdl, int stages, int smem) {
  switch (q.dtype) {
#define CVSA_SS_D(TQ)                                                                         \
  switch (kv.d) {                                                                             \
    case 64: return launch_stream_typed<T, TQ, 64>(q, kv, scores, dev_err, s, pdl, stages, smem); \
    case 128: return launch_stream_typed<T, TQ, 128>(q, kv, scores, dev_err, s, pdl, stages, smem); \
    case 256: return launch_stream_typed<T, TQ, 256>(q, kv, scores, dev_err, s, pdl, stages, smem); \
  }                                                                                           \
  return cudaErrorInvalidValue;
    case CVSA_DTYPE_BF16: { CVSA_SS_D(__nv_bfloat16) }
    case CVSA_DTYPE_F16: { CVSA_SS_D(__half) }
    case CVSA_DTYPE_F32: { CVSA_SS_D(float) }
#undef CVSA_SS_D
  }
  return cudaErrorInvalidValue;
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
  if (stream_eligible(q, kv)) {
    int smem = 0;
    const int stages = stream_plan(q, kv, &smem);
    return kv.dtype == CVSA_DTYPE_BF16
               ? stream_dispatch_q<__nv_bfloat16>(q, kv, scores, dev_err, s, pdl, stages, smem)
               : stream_dispatch_q<__half>(q, kv, scores, dev_err, s, pdl, stages, smem);
  }
  switch (kv.dtype) {
    case CVSA_DTYPE_BF16: return dispatch_q<__nv_bfloat16>(q, kv, scores, dev_err, s, pdl);
    case CVSA_DTYPE_F16: return dispatch_q<__half>(q, kv, scores, dev_err, s, pdl);
    case CVSA_DTYPE_F32: return dispatch_q<float>(q, kv, scores, dev_err, s, pdl);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace cvsa
