// Block-level operations on the paged Q4 pool, sm_100a:
//  * blocks_copy_kernel: whole blocks between the pool and a packed byte buffer laid out as
//    the reference's persisted tensors (L{l}_B{b}_{K,V}_{weights,scales,biases}, each
//    [1, Hkv, tokens, cols], safetensors_cache_adapter.py:141-199 / :284-327), so a save is
//    one gather + one device->host copy and a load one host->device copy + one scatter.
//  * block_reserve_kernel / block_release_kernel: the pool's free list on the device
//    (BlockPool.allocate / free, domain/services.py:111-223: LIFO, all-or-nothing per
//    call), so sequences can grow, shrink and be dropped inside a captured step.
// One CTA per call for the free-list kernels: rows are scanned in order and block ids are
// taken from / returned to the top of the stack in row-major order, so the device result
// is the one the host BlockPool gives for the same sequence of calls.  No waits; errors
// are status bits.
#include "am_common.cuh"
#include "am_internal.h"

namespace am {

// ------------------------------------------------------------------ pack / unpack
__device__ __forceinline__ void copy_bytes(uint8_t* dst, const uint8_t* src, int64_t n) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) |
                      static_cast<uintptr_t>(n);
  if ((a & 15) == 0) {
    uint4* d = reinterpret_cast<uint4*>(dst);
    const uint4* s = reinterpret_cast<const uint4*>(src);
    for (int64_t i = threadIdx.x; i < n / 16; i += blockDim.x) d[i] = s[i];
  } else if ((a & 3) == 0) {
    uint32_t* d = reinterpret_cast<uint32_t*>(dst);
    const uint32_t* s = reinterpret_cast<const uint32_t*>(src);
    for (int64_t i = threadIdx.x; i < n / 4; i += blockDim.x) d[i] = s[i];
  } else if ((a & 1) == 0) {
    uint16_t* d = reinterpret_cast<uint16_t*>(dst);
    const uint16_t* s = reinterpret_cast<const uint16_t*>(src);
    for (int64_t i = threadIdx.x; i < n / 2; i += blockDim.x) d[i] = s[i];
  } else {
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  }
}

// grid (n_blocks, 6 sections): section s of block i is Hkv contiguous runs of
// tokens[i] rows, one per head, at offsets[i * 6 + s] in the buffer.
__global__ void __launch_bounds__(256) blocks_copy_kernel(BlockCopyParams p) {
  const int i = blockIdx.x, s = blockIdx.y;
  const int32_t blk = p.block_ids[i];
  const int32_t T = p.tokens[i];
  if (blk < 0 || blk >= p.num_blocks || T < 0 || T > p.block_tokens) {
    if (threadIdx.x == 0 && s == 0) flag_status(p.status, AM_STATUS_BAD_BLOCK);
    return;
  }
  const int64_t rb = p.row_bytes[s];
  uint8_t* pool = static_cast<uint8_t*>(p.pool[s]);
  const int64_t off = p.offsets[(int64_t)i * 6 + s];
  for (int h = 0; h < p.hkv; ++h) {
    uint8_t* slab = pool + ((int64_t)blk * p.hkv + h) * p.block_tokens * rb;
    uint8_t* buf = p.buf + off + (int64_t)h * T * rb;
    if (p.to_buffer) {
      copy_bytes(buf, slab, (int64_t)T * rb);
    } else {
      copy_bytes(slab, buf, (int64_t)T * rb);
    }
  }
}

// ------------------------------------------------------------------ device free list
// Exclusive prefix sum of one value per thread over the CTA (blockDim.x <= 1024, a
// multiple of 32); returns this thread's prefix and writes the CTA total.
__device__ int cta_exclusive_scan(int v, int* total) {
  __shared__ int warp_sums[32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  int x = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, off);
    if (lane >= off) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nw ? warp_sums[lane] : 0;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    if (lane < nw) warp_sums[lane] = w;
  }
  __syncthreads();
  const int before = (warp > 0 ? warp_sums[warp - 1] : 0) + x - v;
  *total = warp_sums[nw - 1];
  __syncthreads();
  return before;
}

// Make table[r][0, ceil((lengths[r] + add[r]) / block_tokens)) valid: every missing entry
// (< 0) takes the next id from the top of the free stack, rows in order, entries in order.
// All-or-nothing: if the pool cannot cover every missing entry, nothing is taken and
// AM_STATUS_POOL_EXHAUSTED is set.
__global__ void __launch_bounds__(1024) block_reserve_kernel(BlockListParams p) {
  __shared__ int s_need;
  const int top = *p.free_top;
  if (top < 0 || top > p.capacity) {  // not a free list of this pool: touch nothing
    if (threadIdx.x == 0) flag_status(p.status, AM_STATUS_BAD_BLOCK);
    return;
  }
  // pass 1: total missing entries
  int need_total = 0;
  for (int r0 = 0; r0 < p.rows; r0 += blockDim.x) {
    const int r = r0 + threadIdx.x;
    int m = 0;
    if (r < p.rows) {
      const int64_t want = ((int64_t)p.lengths[r] + p.counts[r] + p.block_tokens - 1) / p.block_tokens;
      const int hi = static_cast<int>(want < p.table_stride ? want : (int64_t)p.table_stride);
      if (want > p.table_stride) flag_status(p.status, AM_STATUS_BAD_POSITION);
      for (int j = 0; j < hi; ++j) m += p.table[(int64_t)r * p.table_stride + j] < 0;
    }
    int tot;
    cta_exclusive_scan(m, &tot);
    need_total += tot;
  }
  if (threadIdx.x == 0) s_need = need_total;
  __syncthreads();
  if (s_need > top) {
    if (threadIdx.x == 0) flag_status(p.status, AM_STATUS_POOL_EXHAUSTED);
    return;
  }
  // pass 2: assign
  int base = 0;
  for (int r0 = 0; r0 < p.rows; r0 += blockDim.x) {
    const int r = r0 + threadIdx.x;
    int m = 0, hi = 0;
    if (r < p.rows) {
      const int64_t want = ((int64_t)p.lengths[r] + p.counts[r] + p.block_tokens - 1) / p.block_tokens;
      hi = static_cast<int>(want < p.table_stride ? want : (int64_t)p.table_stride);
      for (int j = 0; j < hi; ++j) m += p.table[(int64_t)r * p.table_stride + j] < 0;
    }
    int tot;
    int k = base + cta_exclusive_scan(m, &tot);
    if (r < p.rows) {
      for (int j = 0; j < hi; ++j) {
        int32_t* e = p.table + (int64_t)r * p.table_stride + j;
        if (*e < 0) *e = p.free_ids[top - 1 - k++];
      }
    }
    base += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) *p.free_top = top - s_need;
}

// Return table[r][keep[r], table_stride) (entries >= 0) to the free stack, rows in order,
// entries in order, and clear them to -1.  A release that would overflow the stack (a
// double free) changes nothing and sets AM_STATUS_BAD_BLOCK.
__global__ void __launch_bounds__(1024) block_release_kernel(BlockListParams p) {
  __shared__ int s_total;
  const int top = *p.free_top;
  if (top < 0 || top > p.capacity) {
    if (threadIdx.x == 0) flag_status(p.status, AM_STATUS_BAD_BLOCK);
    return;
  }
  int total = 0;
  for (int r0 = 0; r0 < p.rows; r0 += blockDim.x) {
    const int r = r0 + threadIdx.x;
    int m = 0;
    if (r < p.rows) {
      for (int j = max(0, p.counts[r]); j < p.table_stride; ++j) {
        const int32_t v = p.table[(int64_t)r * p.table_stride + j];
        m += v >= 0 && v < p.capacity;
      }
    }
    int tot;
    cta_exclusive_scan(m, &tot);
    total += tot;
  }
  if (threadIdx.x == 0) s_total = total;
  __syncthreads();
  if (top + s_total > p.capacity) {
    if (threadIdx.x == 0) flag_status(p.status, AM_STATUS_BAD_BLOCK);
    return;
  }
  int base = 0;
  for (int r0 = 0; r0 < p.rows; r0 += blockDim.x) {
    const int r = r0 + threadIdx.x;
    int m = 0;
    if (r < p.rows) {
      for (int j = max(0, p.counts[r]); j < p.table_stride; ++j) {
        const int32_t v = p.table[(int64_t)r * p.table_stride + j];
        m += v >= 0 && v < p.capacity;
      }
    }
    int tot;
    int k = base + cta_exclusive_scan(m, &tot);
    if (r < p.rows) {
      for (int j = max(0, p.counts[r]); j < p.table_stride; ++j) {
        int32_t* e = p.table + (int64_t)r * p.table_stride + j;
        if (*e >= 0 && *e < p.capacity) p.free_ids[top + k++] = *e;
        if (*e >= 0) *e = -1;
      }
    }
    base += tot;
  }
  __syncthreads();
  if (threadIdx.x == 0) *p.free_top = top + s_total;
}

cudaError_t launch_blocks_copy(const BlockCopyParams& p, int n_blocks, cudaStream_t stream) {
  if (n_blocks <= 0) return cudaSuccess;
  blocks_copy_kernel<<<dim3(n_blocks, 6), 256, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_block_reserve(const BlockListParams& p, cudaStream_t stream) {
  block_reserve_kernel<<<1, 1024, 0, stream>>>(p);
  return cudaGetLastError();
}

cudaError_t launch_block_release(const BlockListParams& p, cudaStream_t stream) {
  block_release_kernel<<<1, 1024, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace am
