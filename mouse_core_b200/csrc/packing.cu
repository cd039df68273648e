// K9: the decode step's layout glue on the device.
//  * flat_rank_kernel: the stable rank of every token among the tokens of its
//    sequence id, the per-id token counts and their maximum, and the [B, S]
//    local prediction indices with real steps in the trailing columns
//    (models/base.py:1163-1201, _flat_to_batched_left_pad), in one CTA.
//  * flat_scatter_kernel: the flat [L, D] rows into the right-padded
//    [B, Lmax, D] layout at (id, rank).
//  * left_align_kernel: right-padded rows shifted so their content ends at the
//    last column, prediction indices shifted with them
//    (models/embedding/packing.py:8-28, left_align_content).
// All three move bytes only: rows are copied in 16-byte vectors when the row
// size allows, and every index equals the reference's bit for bit.
#include "common.cuh"
#include "kernels.h"

namespace mb {

// stats[0 .. B-1] = tokens per id, stats[B] = their maximum, stats[B + 1] = 1
// when a prediction index lies outside [-L, L) or past the N given (those
// local indices are written as -1); negative indices count from the end.
__global__ void __launch_bounds__(1024)
    flat_rank_kernel(const int64_t* __restrict__ seq, int L, int B, const int64_t* __restrict__ pred, int N,
                     const int32_t* __restrict__ steps, const int32_t* __restrict__ step_off, int S,
                     int32_t* __restrict__ rank, int32_t* __restrict__ stats, int64_t* __restrict__ local) {
  extern __shared__ int cnt[];  // [B]
  __shared__ int s_max, s_bad;
  for (int b = threadIdx.x; b < B; b += blockDim.x) cnt[b] = 0;
  if (threadIdx.x == 0) {
    s_max = 0;
    s_bad = 0;
  }
  __syncthreads();
  // Warp 0 walks the tokens in order, 32 at a time. Tokens of one id within a
  // step rank by lane after every earlier token of that id; the lowest lane of
  // the group then advances the id's counter. Ids outside [0, B) rank -1.
  if (threadIdx.x < 32) {
    const int lane = threadIdx.x;
    const unsigned lower = (1u << lane) - 1u;
    for (int base = 0; base < L; base += 32) {
      const int i = base + lane;
      const unsigned active = __ballot_sync(0xffffffffu, i < L);
      if (i < L) {
        const long long id = seq[i];
        const bool in = id >= 0 && id < B;
        const unsigned long long key = in ? (unsigned long long)id : ~0ull;
        const unsigned peers = __match_any_sync(active, key);
        const int before = __popc(peers & lower);
        const int r = in ? cnt[id] + before : -1;
        __syncwarp(active);
        if (in && before == 0) cnt[id] += __popc(peers);
        rank[i] = r;
      }
      __syncwarp();
    }
  }
  __syncthreads();
  int m = 0;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    stats[b] = cnt[b];
    m = max(m, cnt[b]);
  }
  atomicMax(&s_max, m);
  // Row b's n = steps[b] prediction tokens fill columns S - n .. S - 1; their
  // absolute indices start at pred[step_off[b]].
  const long long cells = (long long)B * S;
  for (long long e = threadIdx.x; e < cells; e += blockDim.x) {
    const int b = (int)(e / S), c = (int)(e % S);
    const int n = steps[b];
    long long v = 0;
    if (c >= S - n) {
      const long long k = (long long)step_off[b] + (c - (S - n));
      long long a = (k >= 0 && k < N) ? pred[k] : -1 - (long long)L;
      if (a < 0) a += L;  // Python indexing: -1 is the last token
      if (a < 0 || a >= L) {
        s_bad = 1;
        v = -1;
      } else {
        v = rank[a];
      }
    }
    local[e] = v;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    stats[B] = s_max;
    stats[B + 1] = s_bad;
  }
}

// Copy `chunks` units of T per row.
template <typename T>
__device__ __forceinline__ void copy_row(T* __restrict__ dst, const T* __restrict__ src, int chunks, int lane) {
  for (int c = lane; c < chunks; c += 32) dst[c] = src[c];
}

template <typename T>
__device__ __forceinline__ void zero_row(T* __restrict__ dst, int chunks, int lane) {
  const T z{};
  for (int c = lane; c < chunks; c += 32) dst[c] = z;
}

// One warp per flat token: row i goes to out[seq[i], rank[i]] (rank -1: dropped).
template <typename T>
__global__ void __launch_bounds__(256) flat_scatter_kernel(const T* __restrict__ emb, int L, int chunks,
                                                           const int64_t* __restrict__ seq,
                                                           const int32_t* __restrict__ rank, int Lmax,
                                                           T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  for (long long i = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; i < L; i += warps) {
    const int r = rank[i];
    if (r < 0) continue;
    const long long b = seq[i];
    copy_row(out + (b * Lmax + r) * chunks, emb + i * chunks, chunks, lane);
  }
}

// One warp per output row (b, col): content of row b is its first rl =
// pi[b, S-1] + 1 columns; with rl > 0 it moves to columns L - rl .. L - 1 and
// every other column is zero; with rl <= 0 the whole row is zero and the
// indices stay. Indices: pi[b, s] + (rl > 0 ? L - rl : 0).
template <typename T>
__global__ void __launch_bounds__(256) left_align_kernel(const T* __restrict__ emb, int B, int L, int chunks,
                                                         const int64_t* __restrict__ pi, int S,
                                                         T* __restrict__ out, int64_t* __restrict__ out_idx) {
  const int lane = threadIdx.x & 31;
  const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
  const long long rows = (long long)B * L;
  for (long long w = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < rows; w += warps) {
    const int b = (int)(w / L), col = (int)(w % L);
    const long long rl = pi[(long long)b * S + S - 1] + 1;
    const long long off = rl > 0 ? L - rl : 0;
    const long long src = col - off;
    T* dst = out + w * chunks;
    if (rl > 0 && src >= 0 && src < L)
      copy_row(dst, emb + ((long long)b * L + src) * chunks, chunks, lane);
    else
      zero_row(dst, chunks, lane);
  }
  const long long cells = (long long)B * S;
  for (long long e = (long long)blockIdx.x * blockDim.x + threadIdx.x; e < cells;
       e += (long long)gridDim.x * blockDim.x) {
    const long long b = e / S;
    const long long rl = pi[b * S + S - 1] + 1;
    out_idx[e] = pi[e] + (rl > 0 ? L - rl : 0);
  }
}

// Widest copy unit (16, 4 or 1 bytes) that divides the row and both bases.
static int copy_unit(int row_bytes, const void* a, const void* b) {
  const uintptr_t x = reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b);
  if (row_bytes % 16 == 0 && x % 16 == 0) return 16;
  if (row_bytes % 4 == 0 && x % 4 == 0) return 4;
  return 1;
}

static int glue_blocks(long long warps_needed) {
  return (int)std::max<long long>(1, std::min<long long>((warps_needed + 7) / 8, 148 * 16));
}

cudaError_t launch_flat_rank(const int64_t* seq, int L, int B, const int64_t* pred, int N, const int32_t* steps,
                             const int32_t* step_off, int S, int32_t* rank, int32_t* stats, int64_t* local,
                             cudaStream_t stream) {
  const int smem = B * (int)sizeof(int);
  cudaError_t e = cudaFuncSetAttribute(flat_rank_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  flat_rank_kernel<<<1, 1024, smem, stream>>>(seq, L, B, pred, N, steps, step_off, S, rank, stats, local);
  return cudaGetLastError();
}

cudaError_t launch_flat_scatter(const void* emb, int L, int row_bytes, const int64_t* seq, const int32_t* rank,
                                int Lmax, void* out, cudaStream_t stream) {
  const int blocks = glue_blocks(L);
  const int unit = copy_unit(row_bytes, emb, out);
  if (unit == 16)
    flat_scatter_kernel<uint4><<<blocks, 256, 0, stream>>>(static_cast<const uint4*>(emb), L, row_bytes / 16, seq,
                                                           rank, Lmax, static_cast<uint4*>(out));
  else if (unit == 4)
    flat_scatter_kernel<uint32_t><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t*>(emb), L, row_bytes / 4,
                                                              seq, rank, Lmax, static_cast<uint32_t*>(out));
  else
    flat_scatter_kernel<uint8_t><<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(emb), L, row_bytes, seq,
                                                             rank, Lmax, static_cast<uint8_t*>(out));
  return cudaGetLastError();
}

cudaError_t launch_left_align(const void* emb, int B, int L, int row_bytes, const int64_t* pi, int S, void* out,
                              int64_t* out_idx, cudaStream_t stream) {
  const int blocks = glue_blocks(std::max<long long>((long long)B * L, ((long long)B * S + 31) / 32));
  const int unit = copy_unit(row_bytes, emb, out);
  if (unit == 16)
    left_align_kernel<uint4><<<blocks, 256, 0, stream>>>(static_cast<const uint4*>(emb), B, L, row_bytes / 16, pi,
                                                         S, static_cast<uint4*>(out), out_idx);
  else if (unit == 4)
    left_align_kernel<uint32_t><<<blocks, 256, 0, stream>>>(static_cast<const uint32_t*>(emb), B, L,
                                                            row_bytes / 4, pi, S, static_cast<uint32_t*>(out),
                                                            out_idx);
  else
    left_align_kernel<uint8_t><<<blocks, 256, 0, stream>>>(static_cast<const uint8_t*>(emb), B, L, row_bytes, pi, S,
                                                           static_cast<uint8_t*>(out), out_idx);
  return cudaGetLastError();
}

}  // namespace mb
