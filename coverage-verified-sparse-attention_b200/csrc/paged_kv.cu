// Paged KV runtime kernels.
//
// append: one decode token per sequence, for the whole batch in one launch.
// Restates SequenceKVManager.append_token_kv (cvsa/runtime/kv_cache.py:
// 133-150) -- position = context_len; a page that starts at the position and
// lies past the pages already allocated takes a fresh block (the reference's
// bump allocator, kv_cache.py:53-62, generalised to a device free list whose
// head is advanced atomically, so pages may come from a shuffled pool); the
// token's K/V rows go to block_tables[b, page] at offset position % bs; the
// context length is incremented. One warp per (sequence, kv head) row copy,
// 16-byte vectors; lane 0 of the sequence's first warp does the bookkeeping.
//
// gather: the K/V rows of a sequence's pages into a dense buffer (inverse of
// PagedKVCache.write_kv_block, kv_cache.py:73-80).
#include "cvsa_common.cuh"
#include "cvsa_internal.h"

namespace cvsa {
namespace {

__global__ void append_kernel(uint8_t* k, uint8_t* v, int64_t sb_b, int64_t st_b, int64_t sh_b,
                              int num_blocks, int bs, int hkv, int row_bytes,
                              const uint8_t* k_new, const uint8_t* v_new, int B,
                              const int32_t* seq_ids, int32_t* tables, int W, int32_t* lens,
                              int32_t* pages_alloc, const int32_t* free_list, int free_len,
                              int32_t* free_head, int32_t* dev_err) {
  // block = one sequence; warps = kv heads (looped)
  const int r = blockIdx.x;
  if (r >= B) return;
  const int seq = seq_ids ? seq_ids[r] : r;
  __shared__ int s_blk, s_off;
  if (threadIdx.x == 0) {
    const int pos = lens[seq];
    const int page = pos / bs;
    const int off = pos % bs;
    int blk = -1;
    if (page >= W) {
      set_dev_error(dev_err, CVSA_DEV_ERR_TABLE_FULL);
    } else {
      if (off == 0 && page >= pages_alloc[seq]) {
        const int slot = atomicAdd(free_head, 1);
        if (slot < free_len) {
          blk = free_list[slot];
          tables[(int64_t)seq * W + page] = blk;
          pages_alloc[seq] = page + 1;
        } else {
          set_dev_error(dev_err, CVSA_DEV_ERR_POOL);
        }
      } else {
        blk = tables[(int64_t)seq * W + page];
      }
      if (blk >= 0 && blk >= num_blocks) {
        set_dev_error(dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
        blk = -1;
      }
      if (blk >= 0) lens[seq] = pos + 1;
    }
    s_blk = blk;
    s_off = off;
  }
  __syncthreads();
  const int blk = s_blk;
  if (blk < 0) return;
  const int nvec = row_bytes / 16;
  for (int e = threadIdx.x; e < hkv * nvec; e += blockDim.x) {
    const int h = e / nvec, c = e % nvec;
    const int64_t dst = (int64_t)blk * sb_b + (int64_t)s_off * st_b + (int64_t)h * sh_b + c * 16;
    const int64_t src = ((int64_t)r * hkv + h) * row_bytes + c * 16;
    *reinterpret_cast<uint4*>(k + dst) = *reinterpret_cast<const uint4*>(k_new + src);
    *reinterpret_cast<uint4*>(v + dst) = *reinterpret_cast<const uint4*>(v_new + src);
  }
}

__global__ void gather_kernel(const uint8_t* k, const uint8_t* v, int64_t sb_b, int64_t st_b,
                              int64_t sh_b, int num_blocks, int bs, int hkv, int row_bytes,
                              const int32_t* row, int n_pages, uint8_t* k_out, uint8_t* v_out,
                              int32_t* dev_err) {
  const int p = blockIdx.x;
  if (p >= n_pages) return;
  const int blk = row[p];
  if (blk < 0 || blk >= num_blocks) {
    if (threadIdx.x == 0) set_dev_error(dev_err, CVSA_DEV_ERR_BLOCK_RANGE);
    return;
  }
  const int nvec = row_bytes / 16;
  const int per_tok = hkv * nvec;
  for (int e = threadIdx.x; e < bs * per_tok; e += blockDim.x) {
    const int t = e / per_tok, rem = e % per_tok, h = rem / nvec, c = rem % nvec;
    const int64_t src = (int64_t)blk * sb_b + (int64_t)t * st_b + (int64_t)h * sh_b + c * 16;
    const int64_t dst = (((int64_t)p * bs + t) * hkv + h) * row_bytes + c * 16;
    *reinterpret_cast<uint4*>(k_out + dst) = *reinterpret_cast<const uint4*>(k + src);
    if (v_out) *reinterpret_cast<uint4*>(v_out + dst) = *reinterpret_cast<const uint4*>(v + src);
  }
}

}  // namespace

cudaError_t launch_paged_append(const KvView& kv, const void* k_new, const void* v_new, int B,
                                const int32_t* seq_ids, int32_t* tables, int W, int32_t* lens,
                                int32_t* pages_alloc, const int32_t* free_list, int free_len,
                                int32_t* free_head, int32_t* dev_err, cudaStream_t s) {
  if (B == 0) return cudaSuccess;
  const int eb = dtype_bytes(kv.dtype);
  const int row_bytes = kv.d * eb;
  append_kernel<<<B, 128, 0, s>>>((uint8_t*)kv.k, (uint8_t*)kv.v, kv.sb * eb, kv.st * eb,
                                  kv.sh * eb, kv.num_blocks, kv.bs, kv.hkv, row_bytes,
                                  (const uint8_t*)k_new, (const uint8_t*)v_new, B, seq_ids,
                                  tables, W, lens, pages_alloc, free_list, free_len, free_head,
                                  dev_err);
  return cudaGetLastError();
}

cudaError_t launch_paged_gather(const KvView& kv, const int32_t* row, int n_pages, void* k_out,
                                void* v_out, int32_t* dev_err, cudaStream_t s) {
  if (n_pages == 0) return cudaSuccess;
  const int eb = dtype_bytes(kv.dtype);
  gather_kernel<<<n_pages, 256, 0, s>>>((const uint8_t*)kv.k, (const uint8_t*)kv.v, kv.sb * eb,
                                        kv.st * eb, kv.sh * eb, kv.num_blocks, kv.bs, kv.hkv,
                                        kv.d * eb, row, n_pages, (uint8_t*)k_out,
                                        (uint8_t*)v_out, dev_err);
  return cudaGetLastError();
}

}  // namespace cvsa
