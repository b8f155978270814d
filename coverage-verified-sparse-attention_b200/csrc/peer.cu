// Exchanges between the ranks of one node over NVLink peer memory (one
// process per GPU), for the page split's two all-gathers and merge and the
// head-sharded step's decision word: each rank stores its row into every
// rank's exchange buffer through the peer mapping (CUDA IPC), and reads the
// other ranks' rows from its own buffer once they have landed. No library
// collective and no multicast object is involved.
//
// Every 4-byte word travels as one 8-byte store of (word, call number), so a
// reader knows a word has landed when it sees its call number beside it: no
// fence, flag or second round trip is needed (an aligned 8-byte store is
// seen whole or not at all).
//
// Exchange buffer of a rank (the same layout on every rank, mapped by every
// peer):
//   [0, 8 KB)       the call counter (u32) and the CTAs-done ticket (local)
//   [8 KB, ...)     u32x2 [2][world][row_cap]: slot = call & 1
// Every call of every rank uses the next call number e; a rank's call e
// starts after its call e - 1 finished, which read every peer's words of call
// e - 1, so every peer has finished its call e - 2 -- the last reader of slot
// e & 1 -- before the slot is written again. Every wait is bounded
// (cvsa_set_wait_limit, default about a second): a rank that never arrives
// makes the call record CVSA_DEV_ERR_TIMEOUT and return instead of hanging.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cvsa_common.cuh"
#include "cvsa_internal.h"
#include "cvsa_launch.cuh"

namespace cvsa {
namespace {

constexpr int kPeerMaxCta = 65535;
constexpr int kPeerMaxWorld = 8;
constexpr size_t kPeerCallOff = 0;
constexpr size_t kPeerDataOff = 8192;
constexpr uint32_t kPeerSpinDefault = 0xffffffffu;  // no poll cap: the time cap applies
constexpr int kGatherThreads = 256;
constexpr int kGatherChunk = 256;                 // words per CTA
constexpr int kMergeThreads = 128;                // one query row per CTA
constexpr int kPeerMaxD = 256;                    // head_dim of the merge

struct PeerArgs {
  const uint64_t* bases;  // [world] every rank's exchange buffer, as mapped here
  int world, rank;
  int64_t row_cap;        // words per rank row of a slot
  uint32_t polls;
  int32_t* dev_err;
};

__device__ __forceinline__ uint2* peer_row(const PeerArgs& a, int q, uint32_t slot, int r) {
  return reinterpret_cast<uint2*>(a.bases[q] + kPeerDataOff) +
         ((int64_t)slot * a.world + r) * a.row_cap;
}

__device__ __forceinline__ void st_word_pair(uint2* p, uint32_t w0, uint32_t w1, uint32_t e) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %2};" ::"l"(p), "r"(w0), "r"(e),
               "r"(w1)
               : "memory");
}
__device__ __forceinline__ void st_word(uint2* p, uint32_t w, uint32_t e) {
  asm volatile("st.volatile.global.v2.u32 [%0], {%1, %2};" ::"l"(p), "r"(w), "r"(e) : "memory");
}
__device__ __forceinline__ uint2 ld_word(const uint2* p) {
  uint2 v;
  asm volatile("ld.volatile.global.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p)
               : "memory");
  return v;
}

// Push words [lo, hi) of src, tagged with call e, into row `rank` of slot
// `slot` at every rank.
__device__ __forceinline__ void push_range(const PeerArgs& a, uint32_t slot, uint32_t e,
                                           const uint32_t* src, int64_t lo, int64_t hi) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const bool vec = ((lo | hi) & 1) == 0 && (reinterpret_cast<uintptr_t>(src) & 7) == 0 &&
                   (a.row_cap & 1) == 0;
  // rank r starts with rank r + 1, so the ranks do not all write to the
  // same GPU at once
  for (int k = 1; k <= a.world; ++k) {
    const int q = (a.rank + k) % a.world;
    uint2* dst = peer_row(a, q, slot, a.rank);
    if (vec) {
      for (int64_t i = lo + 2 * tid; i < hi; i += 2 * nt) {
        const uint2 w = *reinterpret_cast<const uint2*>(src + i);
        st_word_pair(dst + i, w.x, w.y, e);
      }
    } else {
      for (int64_t i = lo + tid; i < hi; i += nt) st_word(dst + i, src[i], e);
    }
  }
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Fetch `count` words of call e from this rank's own buffer: word j is
// map(j) = (rank q, word i) of slot `slot`; sink(j, value) takes it once it
// has landed. Loads go out kFetchBatch at a time before any is checked, so
// their round trips overlap; a word not there yet is polled until it is, or
// until the wait runs out (a.polls polls or kPeerWaitNs), which marks the CTA
// failed (s_fail: no thread waits again), records the timeout and sinks 0.
constexpr int kFetchBatch = 8;
constexpr uint64_t kPeerWaitNs = 2000000000ull;

template <class Map, class Sink>
__device__ __forceinline__ void fetch_words(const PeerArgs& a, uint32_t slot, uint32_t e,
                                            int count, Map map, Sink sink, volatile int* s_fail) {
  const int nt = blockDim.x;
  for (int j0 = threadIdx.x; j0 < count; j0 += kFetchBatch * nt) {
    const uint2* p[kFetchBatch];
    uint2 v[kFetchBatch];
#pragma unroll
    for (int b = 0; b < kFetchBatch; ++b) {
      const int j = j0 + b * nt;
      int q = 0;
      int64_t i = 0;
      if (j < count) map(j, q, i);
      p[b] = peer_row(a, a.rank, slot, q) + i;
    }
#pragma unroll
    for (int b = 0; b < kFetchBatch; ++b)
      v[b] = (j0 + b * nt < count) ? ld_word(p[b]) : make_uint2(0u, e);
#pragma unroll
    for (int b = 0; b < kFetchBatch; ++b) {
      const int j = j0 + b * nt;
      if (j >= count) continue;
      if (v[b].y != e) {
        uint32_t n = 0;
        const uint64_t t0 = global_ns();
        while (v[b].y != e && !*s_fail) {
          if (++n >= a.polls || global_ns() - t0 > kPeerWaitNs) {
            *s_fail = 1;
            set_dev_error(a.dev_err, CVSA_DEV_ERR_TIMEOUT);
            break;
          }
          __nanosleep(32);
          v[b] = ld_word(p[b]);
        }
      }
      sink(j, v[b].y == e ? v[b].x : 0u);
    }
  }
}

// The call number of this launch (read by every CTA before any CTA of the
// launch can finish), and its advance by the last CTA to finish.
__device__ __forceinline__ uint32_t call_number(const PeerArgs& a) {
  return *reinterpret_cast<volatile uint32_t*>(a.bases[a.rank] + kPeerCallOff) + 1u;
}
__device__ __forceinline__ void finish_call(const PeerArgs& a, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* call = reinterpret_cast<uint32_t*>(a.bases[a.rank] + kPeerCallOff);
    uint32_t* done = call + 1;
    __threadfence();
    if (atomicAdd(done, 1u) == gridDim.x - 1) {
      *done = 0;
      *reinterpret_cast<volatile uint32_t*>(call) = e;
      __threadfence();
    }
  }
}

// All-gather of n words per rank: out[q * n + i] = rank q's src[i]; with
// min_i32, out[i] = min over ranks of the int32 words instead (src may be out).
__global__ void __launch_bounds__(kGatherThreads)
peer_gather_kernel(const __grid_constant__ PeerArgs a, const uint32_t* __restrict__ src,
                   int64_t n, uint32_t* __restrict__ out, int min_i32) {
  __shared__ int s_fail;
  __shared__ uint32_t s_w[kPeerMaxWorld][kGatherChunk];
  if (threadIdx.x == 0) s_fail = 0;
  const uint32_t e = call_number(a);
  const uint32_t slot = e & 1u;
  const int64_t lo = (int64_t)blockIdx.x * kGatherChunk;
  const int len = (int)(min(n, lo + kGatherChunk) - lo);
  __syncthreads();
  push_range(a, slot, e, src, lo, lo + len);
  __syncthreads();  // every read of src (out, in place) is done
  auto map = [&](int j, int& q, int64_t& i) {
    q = j / len;
    i = lo + (j - q * len);
  };
  if (min_i32) {
    fetch_words(a, slot, e, a.world * len, map,
                [&](int j, uint32_t w) { s_w[j / len][j % len] = w; }, &s_fail);
    __syncthreads();
    for (int i = threadIdx.x; i < len; i += blockDim.x) {
      int32_t v = (int32_t)s_w[0][i];
      for (int q = 1; q < a.world; ++q) v = min(v, (int32_t)s_w[q][i]);
      out[lo + i] = (uint32_t)v;
    }
  } else {
    fetch_words(a, slot, e, a.world * len, map,
                [&](int j, uint32_t w) {
                  const int q = j / len;
                  out[(int64_t)q * n + lo + (j - q * len)] = w;
                },
                &s_fail);
  }
  finish_call(a, e);
}

// Exchange of attention partials and their merge: rank r's row is
// [o (rows x D) | m (rows) | l (rows)] (rows = B * Hq). CTA `row` pushes and
// merges that query row in rank order, as cvsa_rank_merge does, and writes
// the normalised output (out dtype TO); with `need`, only the rows of heads
// where need != 0 are written.
template <typename TO>
__global__ void __launch_bounds__(kMergeThreads)
peer_merge_kernel(const __grid_constant__ PeerArgs a, const float* __restrict__ part, int rows,
                  int hq, int G, int D, const uint8_t* __restrict__ need, TO* __restrict__ out) {
  __shared__ int s_fail;
  __shared__ float s_o[kPeerMaxWorld][kPeerMaxD];
  __shared__ float s_ml[kPeerMaxWorld][2];
  if (threadIdx.x == 0) s_fail = 0;
  const uint32_t e = call_number(a);
  const uint32_t slot = e & 1u;
  const int row = blockIdx.x;
  const int64_t m_off = (int64_t)rows * D, l_off = m_off + rows;
  const uint32_t* pw = reinterpret_cast<const uint32_t*>(part);
  __syncthreads();
  push_range(a, slot, e, pw, (int64_t)row * D, (int64_t)(row + 1) * D);
  if (threadIdx.x < a.world) {
    // m and l of the row: two single words per rank
    const int q = (a.rank + 1 + threadIdx.x) % a.world;
    st_word(peer_row(a, q, slot, a.rank) + m_off + row, pw[m_off + row], e);
    st_word(peer_row(a, q, slot, a.rank) + l_off + row, pw[l_off + row], e);
  }
  const int per = D + 2;
  fetch_words(
      a, slot, e, a.world * per,
      [&](int j, int& q, int64_t& i) {
        q = j / per;
        const int r = j - q * per;
        i = r < D ? (int64_t)row * D + r : (r == D ? m_off : l_off) + row;
      },
      [&](int j, uint32_t w) {
        const int q = j / per, r = j - q * per;
        if (r < D) s_o[q][r] = __uint_as_float(w);
        else s_ml[q][r - D] = __uint_as_float(w);
      },
      &s_fail);
  __syncthreads();
  bool want = true;
  if (need != nullptr) {
    const int b = row / hq;
    want = need[b * (hq / G) + (row % hq) / G] != 0;
  }
  if (want) {
    float M = neg_inf();
    for (int q = 0; q < a.world; ++q) M = fmaxf(M, s_ml[q][0]);
    const float base = (M == neg_inf()) ? 0.f : M;
    float L = 0.f;
    for (int q = 0; q < a.world; ++q) {
      const float mr = s_ml[q][0];
      if (mr != neg_inf()) L += s_ml[q][1] * expf(mr - base);
    }
    const float denom = fmaxf(L, 1e-6f);
    for (int d = threadIdx.x; d < D; d += blockDim.x) {
      float v = 0.f;
      for (int q = 0; q < a.world; ++q) {
        const float mr = s_ml[q][0];
        if (mr != neg_inf()) v += s_o[q][d] * expf(mr - base);
      }
      out[(int64_t)row * D + d] = Elem<TO>::from_f(v / denom);
    }
  }
  finish_call(a, e);
}

PeerArgs make_args(const PeerView& pv) {
  PeerArgs a;
  a.bases = pv.bases;
  a.world = pv.world;
  a.rank = pv.rank;
  a.row_cap = pv.row_cap;
  const uint32_t lim = wait_limit();
  a.polls = lim ? lim : kPeerSpinDefault;
  a.dev_err = pv.dev_err;
  return a;
}

}  // namespace

size_t peer_buffer_bytes(int world, int64_t row_cap) {
  return kPeerDataOff + (size_t)2 * world * row_cap * sizeof(uint2);
}

bool peer_shape_ok(const PeerView& pv) {
  return pv.world >= 1 && pv.world <= kPeerMaxWorld && pv.rank >= 0 && pv.rank < pv.world &&
         pv.row_cap > 0 && pv.bases != nullptr;
}

cudaError_t launch_peer_gather(const PeerView& pv, const float* src, int64_t n, float* out,
                               bool min_i32, cudaStream_t s) {
  if (n <= 0) return cudaSuccess;
  if (!peer_shape_ok(pv) || n > pv.row_cap) return cudaErrorInvalidValue;
  const int64_t ctas = (n + kGatherChunk - 1) / kGatherChunk;
  if (ctas > kPeerMaxCta) return cudaErrorInvalidValue;
  peer_gather_kernel<<<(int)ctas, kGatherThreads, 0, s>>>(
      make_args(pv), reinterpret_cast<const uint32_t*>(src), n, reinterpret_cast<uint32_t*>(out),
      min_i32 ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_peer_merge(const PeerView& pv, const float* part, int B, int hkv, int G, int D,
                              const uint8_t* need, void* out, int out_dtype, cudaStream_t s) {
  const int rows = B * hkv * G;
  if (rows <= 0) return cudaSuccess;
  if (!peer_shape_ok(pv) || (int64_t)rows * (D + 2) > pv.row_cap || D > kPeerMaxD)
    return cudaErrorInvalidValue;
  const int ctas = rows;
  if (ctas > kPeerMaxCta) return cudaErrorInvalidValue;
  const PeerArgs a = make_args(pv);
  const int hq = hkv * G;
  switch (out_dtype) {
    case CVSA_DTYPE_BF16:
      peer_merge_kernel<<<ctas, kMergeThreads, 0, s>>>(a, part, rows, hq, G, D, need,
                                                          (__nv_bfloat16*)out);
      break;
    case CVSA_DTYPE_F16:
      peer_merge_kernel<<<ctas, kMergeThreads, 0, s>>>(a, part, rows, hq, G, D, need,
                                                          (__half*)out);
      break;
    case CVSA_DTYPE_F32:
      peer_merge_kernel<<<ctas, kMergeThreads, 0, s>>>(a, part, rows, hq, G, D, need,
                                                          (float*)out);
      break;
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

int peer_max_ctas() { return kPeerMaxCta; }

}  // namespace cvsa
