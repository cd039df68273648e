// K7: segment metadata of a packed stream, one pass over sequence_ids.
//
// Replaces the position-id computation of flex_packed_forward
// (src/mouse_core/models/backbone/flex_train.py:84-92; same formula as
// models/base.py:1226-1236): a new run starts wherever
// sequence_ids[i] != sequence_ids[i-1], and position[i] = i - start of
// i's run. Also emits what the varlen attention kernels need instead of the
// reference's BlockMask (flex_train.py:116-125):
//   run_start[i]  first index of i's run (the smallest kv index token i may
//                 attend when runs carry distinct ids),
//   run_end[i]    one past the last index of i's run (optional; the end of
//                 the query range that may attend key i),
//   tile_lo[t]    run_start of the first token of query tile t (TILE tokens),
//   flags[0]      1 if some id is smaller than its predecessor (ids are not
//                 sorted, so one id may own several runs and the caller must
//                 first make each id contiguous).
// One CTA of 1024 threads scans the stream in chunks of 4096 with a carried
// prefix (and, for run_end, backwards with a carried suffix); integer work,
// bit-exact.
#include "common.cuh"
#include "kernels.h"

namespace mb {

constexpr int kMetaThreads = 1024;
constexpr int kMetaItems = 4;

__global__ void __launch_bounds__(kMetaThreads) segment_meta_kernel(const int64_t* __restrict__ seq, int L, int tile,
                                                                  int64_t* __restrict__ pos,
                                                                  int32_t* __restrict__ run_start,
                                                                  int32_t* __restrict__ run_end,
                                                                  int32_t* __restrict__ tile_lo, int32_t* flags) {
  __shared__ int warp_max[32];
  __shared__ int carry_s;
  __shared__ int unsorted_s;
  const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
  if (tid == 0) {
    carry_s = 0;
    unsorted_s = 0;
  }
  __syncthreads();
  for (int base = 0; base < L; base += kMetaThreads * kMetaItems) {
    const int i0 = base + tid * kMetaItems;
    // Latest run start among this thread's items (-1 if none starts here).
    int last = -1;
    bool unsorted = false;
#pragma unroll
    for (int k = 0; k < kMetaItems; ++k) {
      const int i = i0 + k;
      if (i < L) {
        const bool boundary = (i == 0) || (seq[i] != seq[i - 1]);
        if (boundary) last = i;
        if (i > 0 && seq[i] < seq[i - 1]) unsorted = true;
      }
    }
    if (unsorted) unsorted_s = 1;
    // Inclusive max-scan of `last` over the block.
    int x = last;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x = max(x, y);
    }
    if (lane == 31) warp_max[w] = x;
    __syncthreads();
    if (w == 0) {
      int t = warp_max[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, t, o);
        if (lane >= o) t = max(t, y);
      }
      warp_max[lane] = t;
    }
    __syncthreads();
    // Exclusive prefix: run start in force before this thread's first item.
    int before = __shfl_up_sync(0xffffffffu, x, 1);
    if (lane == 0) before = -1;
    if (w > 0) before = max(before, warp_max[w - 1]);
    int cur = max(before, carry_s);
#pragma unroll
    for (int k = 0; k < kMetaItems; ++k) {
      const int i = i0 + k;
      if (i < L) {
        if (i == 0 || seq[i] != seq[i - 1]) cur = i;
        run_start[i] = cur;
        pos[i] = (int64_t)(i - cur);
      }
    }
    __syncthreads();
    if (tid == kMetaThreads - 1) carry_s = max(carry_s, warp_max[31]);
    __syncthreads();
  }
  // Reverse pass: run_end[i] = first index after i's run (next boundary, or L).
  if (run_end) {
    __syncthreads();
    if (tid == 0) carry_s = L;
    __syncthreads();
    const int nchunks = (L + kMetaThreads * kMetaItems - 1) / (kMetaThreads * kMetaItems);
    for (int ci = nchunks - 1; ci >= 0; --ci) {
      const int base = ci * kMetaThreads * kMetaItems;
      const int i0 = base + tid * kMetaItems;
      // Earliest boundary strictly after each item, among this thread's items.
      int first = 0x7fffffff;
#pragma unroll
      for (int k = kMetaItems - 1; k >= 0; --k) {
        const int i = i0 + k;
        if (i + 1 < L && seq[i + 1] != seq[i]) first = i + 1;
      }
      // Inclusive suffix-min over threads (higher tid = later items).
      int x = first;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_down_sync(0xffffffffu, x, o);
        if (lane + o < 32) x = min(x, y);
      }
      if (lane == 0) warp_max[w] = x;
      __syncthreads();
      if (w == 0) {
        int t = warp_max[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const int y = __shfl_down_sync(0xffffffffu, t, o);
          if (lane + o < 32) t = min(t, y);
        }
        warp_max[lane] = t;
      }
      __syncthreads();
      // Exclusive suffix: earliest boundary after this thread's last item.
      int after = __shfl_down_sync(0xffffffffu, x, 1);
      if (lane == 31) after = 0x7fffffff;
      if (w < 31) after = min(after, warp_max[w + 1]);
      int nxt = min(after, carry_s);
#pragma unroll
      for (int k = kMetaItems - 1; k >= 0; --k) {
        const int i = i0 + k;
        if (i < L) {
          if (i + 1 < L && seq[i + 1] != seq[i]) nxt = i + 1;
          run_end[i] = nxt;
        }
      }
      __syncthreads();
      if (tid == 0) carry_s = min(carry_s, warp_max[0]);
      __syncthreads();
    }
  }
  __syncthreads();
  const int ntiles = (L + tile - 1) / tile;
  for (int t = tid; t < ntiles; t += kMetaThreads) tile_lo[t] = run_start[t * tile];
  if (tid == 0) flags[0] = unsorted_s;
}

cudaError_t launch_segment_meta(const int64_t* seq, int L, int tile, int64_t* pos_out, int32_t* run_start,
                                int32_t* run_end, int32_t* tile_lo, int32_t* flags, cudaStream_t stream) {
  if (L <= 0) return cudaSuccess;
  segment_meta_kernel<<<1, kMetaThreads, 0, stream>>>(seq, L, tile, pos_out, run_start, run_end, tile_lo, flags);
  return cudaGetLastError();
}

}  // namespace mb
