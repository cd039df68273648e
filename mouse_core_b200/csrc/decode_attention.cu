// K1: paged split-KV GQA attention for cached decode (and in-call prefill).
//
// Replaces the FlexAttention call of FlexDecodeSession.forward
// (src/mouse_core/models/backbone/flex_decode.py:226-229) and its BlockMask
// (flex_decode.py:129-134, 198-202): query (b, s) of q-head hq attends the
// cached slots 0..q_pos[b, s] of row b through kv-head hq / G, with slots
// beyond the row's written length reading as zero (outputs 0 when the row has
// no slot at all), exactly like the reference's zero-initialised buffer.
//
// HBM layout: one layer's pool is [num_pages, Hkv, page, HD] bf16, so the
// page of one kv-head is a contiguous [page, HD] slab. A block table
// [B, max_pages] int32 maps logical page i of row b to a pool page.
//
// Two schedules share one TMA producer:
//  * split mode (G*S <= 16 query rows per (row, kv-head)): persistent CTAs
//    walk a device-built work list of (row, chunk) entries x kv-heads. A
//    producer warp stages each item's metadata and Q rows in a 2-slot
//    shared-memory ring and streams its K/V tiles through a 3-stage TMA ring,
//    so the consumers never wait on dependent global loads; four consumer
//    warps split each tile's tokens, run QK^T and PV on the tensor pipe
//    (m16n8k16) with an online softmax, then merge across warps in shared
//    memory. Rows with several chunks write (O, lse) partials and the last
//    CTA of a (row, kv-head) — found with an atomic ticket — merges them.
//  * block mode (more rows): one CTA per (64-row query block, kv-head, row);
//    the four warps split the query rows and walk the causal KV range.
//
// Every wait is bounded (common.cuh); TMA loads never use multicast.
#include <atomic>
#include "common.cuh"
#include "kernels.h"

namespace mb {

template <int HD>
struct AttnTile {
  static constexpr int T = 8192 / HD;             // tokens per tile (64 | 128)
  static constexpr int STAGES = 3;
  static constexpr int TILE_BYTES = T * HD * 2;    // 16 KB for K (and for V)
  static constexpr int NBOX = TILE_BYTES / 8192;   // 64x64 boxes per tile
  static constexpr int KS = HD / 16;               // k-steps of QK^T
  static constexpr int ND = HD / 8;                // n-tiles of PV
};

// Shared-memory byte offset of (token row `rr` of the tile, 16-byte chunk
// `ch` of HD) inside one K or V tile made of 64x64 swizzled boxes.
template <int HD>
__device__ __forceinline__ uint32_t tile_off(uint32_t rr, uint32_t ch) {
  if constexpr (HD == 128) {
    return (ch >> 3) * 8192u + swz128(rr, ch & 7u);
  } else {
    return (rr >> 6) * 8192u + swz128(rr & 63u, ch);
  }
}

// Issue the K and V loads of tile [t0, t0 + T) of (row b, kv-head h).
template <int HD>
__device__ __forceinline__ void issue_tile(const CUtensorMap* kmap, const CUtensorMap* vmap, uint8_t* kdst,
                                           uint8_t* vdst, uint64_t* bar, const AttnParams& p, int b, int h,
                                           int t0, int len) {
  using C = AttnTile<HD>;
  mbar_arrive_expect_tx(bar, 2 * C::TILE_BYTES);
#pragma unroll
  for (int box = 0; box < C::NBOX; ++box) {
    const int g = (HD == 128) ? 0 : box;   // 64-token row group
    const int cb = (HD == 128) ? box : 0;  // 64-element column block
    const int tok = t0 + 64 * g;
    int y = -64;  // wholly out of bounds: the TMA unit fills zeros
    if (tok < len) {
      const int pidx = tok / p.page_size;
      const int pg = (pidx < p.max_pages) ? p.block_table[(size_t)b * p.max_pages + pidx] : -1;
      if (pg >= 0 && pg < p.num_pages) {
        y = (pg * p.Hkv + h) * p.page_size + (tok % p.page_size);
      } else {
        report(kDevBadPage);
      }
    }
    tma_load_2d(kdst + box * 8192, kmap, bar, cb * 64, y);
    tma_load_2d(vdst + box * 8192, vmap, bar, cb * 64, y);
  }
}

// Load the A fragments of 16 query rows (row r -> (s, g) = (r / G, r % G)).
// Rows >= nrows are zero.
template <int HD>
__device__ __forceinline__ void load_q_frags(uint32_t (&qa)[HD / 16][4], const AttnParams& p, int b, int h,
                                             int row0, int nrows, int lane) {
  const int gid = lane >> 2, tig = lane & 3;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = row0 + gid + 8 * half;
    const __nv_bfloat16* src = nullptr;
    if (r < nrows) {
      const int s = r / p.G, g = r % p.G;
      src = p.q + (((size_t)b * p.S + s) * p.Hq + (size_t)h * p.G + g) * HD;
    }
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      uint32_t lo = 0, hi = 0;
      if (src) {
        lo = *reinterpret_cast<const uint32_t*>(src + kk * 16 + tig * 2);
        hi = *reinterpret_cast<const uint32_t*>(src + kk * 16 + 8 + tig * 2);
      }
      qa[kk][half] = lo;       // a0a1 (row gid) / a2a3 (row gid+8)
      qa[kk][2 + half] = hi;   // a4a5 / a6a7
    }
  }
}

// S[j] (j < NJ n-tiles of 8 tokens starting at tile row `rbase`) = Q K^T.
template <int HD, int NJ>
__device__ __forceinline__ void qk_tile(float (&s)[NJ][4], const uint32_t (&qa)[HD / 16][4], uint32_t kbase,
                                        int rbase, int lane) {
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
    s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    const uint32_t rr = rbase + j * 8 + (lane & 7);
#pragma unroll
    for (int kp = 0; kp < HD / 32; ++kp) {
      uint32_t r0, r1, r2, r3;
      ldmatrix_x4(r0, r1, r2, r3, kbase + tile_off<HD>(rr, kp * 4 + (lane >> 3)));
      mma_bf16_16816(s[j], qa[2 * kp], r0, r1);
      mma_bf16_16816(s[j], qa[2 * kp + 1], r2, r3);
    }
  }
}

// O += P V for the NJ*8 tokens starting at tile row `rbase`.
template <int HD, int NJ>
__device__ __forceinline__ void pv_tile(float (&o)[HD / 8][4], const float (&s)[NJ][4], uint32_t vbase, int rbase,
                                        int lane) {
#pragma unroll
  for (int kt = 0; kt < NJ / 2; ++kt) {
    uint32_t pa[4];
    pa[0] = pack_bf16x2(s[2 * kt][0], s[2 * kt][1]);
    pa[1] = pack_bf16x2(s[2 * kt][2], s[2 * kt][3]);
    pa[2] = pack_bf16x2(s[2 * kt + 1][0], s[2 * kt + 1][1]);
    pa[3] = pack_bf16x2(s[2 * kt + 1][2], s[2 * kt + 1][3]);
    const uint32_t rr = rbase + kt * 16 + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
    for (int d = 0; d < HD / 8; d += 2) {
      uint32_t r0, r1, r2, r3;
      ldmatrix_x4_trans(r0, r1, r2, r3, vbase + tile_off<HD>(rr, d + (lane >> 4)));
      mma_bf16_16816(o[d], pa, r0, r1);
      mma_bf16_16816(o[d + 1], pa, r2, r3);
    }
  }
}

// Mask (token >= kv_end of the row -> -inf), scale to log2 units and fold the
// tile into the running (m, l, o) of this thread's two rows.
template <int HD, int NJ>
__device__ __forceinline__ void online_softmax(float (&s)[NJ][4], float (&o)[HD / 8][4], float (&m)[2],
                                               float (&l)[2], int tok0, const int (&kv_end)[2], float scale_log2,
                                               int lane) {
  const int tig = lane & 3;
  float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
  for (int j = 0; j < NJ; ++j) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int t = tok0 + j * 8 + tig * 2 + (e & 1);
      const int half = e >> 1;
      const float v = (t < kv_end[half]) ? s[j][e] * scale_log2 : -INFINITY;
      s[j][e] = v;
      mx[half] = fmaxf(mx[half], v);
    }
  }
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    mx[half] = fmaxf(mx[half], __shfl_xor_sync(0xffffffffu, mx[half], 1));
    mx[half] = fmaxf(mx[half], __shfl_xor_sync(0xffffffffu, mx[half], 2));
    const float m_new = fmaxf(m[half], mx[half]);
    const float m_use = (m_new == -INFINITY) ? 0.f : m_new;
    const float alpha = exp2f(m[half] - m_use);
    m[half] = m_new;
    l[half] *= alpha;
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) {
      o[d][2 * half] *= alpha;
      o[d][2 * half + 1] *= alpha;
    }
    float rs = 0.f;
#pragma unroll
    for (int j = 0; j < NJ; ++j) {
      const float p0 = exp2f(s[j][2 * half] - m_use);
      const float p1 = exp2f(s[j][2 * half + 1] - m_use);
      s[j][2 * half] = p0;
      s[j][2 * half + 1] = p1;
      rs += p0 + p1;
    }
    l[half] += rs;
  }
}

template <int HD>
struct SplitSmem {
  static constexpr int RING = 2 * AttnTile<HD>::STAGES * AttnTile<HD>::TILE_BYTES;
  // Item slots staged by the producer: 16 Q rows (padded against bank
  // conflicts) + metadata ints.
  static constexpr int QROW = HD * 2 + 16;
  static constexpr int META = 32;  // ints
  static constexpr int SLOT = 16 * QROW + META * 4;
  static constexpr int NSLOT = 2;
  // after the ring and slots: comb_o [4][R][HD] f32, comb_m [4][R], comb_l [4][R], bars, flag
  static size_t bytes(int R) {
    return 1024 + RING + NSLOT * SLOT + (size_t)4 * R * HD * 4 + (size_t)8 * R * 4 +
           (2 * AttnTile<HD>::STAGES + 2 * NSLOT) * 8 + 16;
  }
};

// Position of the n-th (0-based) set bit of `mask`.
__device__ __forceinline__ int nth_bit(int mask, int n) {
  for (int i = 0; i < n; ++i) mask &= mask - 1;
  return __ffs(mask) - 1;
}

// Item metadata slot layout (ints after the Q rows).
// kMetaB < 0 marks the end of the CTA's work; kMetaItem is the item's index
// in the row-ordered work list (entry * Hkv + kv-head), where its partial
// result goes.
// kMetaWidth is the item's member mask (bit k: batch row b + k; more than one
// bit for a chunk several rows share, whose queries are R rows per member)
// and kMetaChunk the chunk's index in each row.
enum : int { kMetaB = 0, kMetaH, kMetaBegin, kMetaEnd, kMetaChunks, kMetaItem, kMetaWidth, kMetaChunk, kMetaKvEnd = 8 };

template <int HD>
__global__ void __launch_bounds__(160, 2) split_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                           const __grid_constant__ CUtensorMap vmap,
                                                           const AttnParams p) {
  using C = AttnTile<HD>;
  using SM = SplitSmem<HD>;
  constexpr int TW = C::T / 4;   // tokens per warp per tile
  constexpr int NJ = TW / 8;     // n-tiles per warp
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kring = smem;
  uint8_t* vring = smem + C::STAGES * C::TILE_BYTES;
  uint8_t* slots = smem + SM::RING;
  const int R = p.R;
  float* comb_o = reinterpret_cast<float*>(slots + SM::NSLOT * SM::SLOT);
  float* comb_m = comb_o + 4 * R * HD;
  float* comb_l = comb_m + 4 * R;
  uint64_t* full = reinterpret_cast<uint64_t*>(comb_l + 4 * R);
  uint64_t* empty = full + C::STAGES;
  uint64_t* item_full = empty + C::STAGES;
  uint64_t* item_empty = item_full + SM::NSLOT;
  int* flag = reinterpret_cast<int*>(item_empty + SM::NSLOT);
  // Set by the first wait of this CTA that runs out: every role then stops
  // (consumers together, at a barrier), the producer lets its issued copies
  // land, and no output of an incomplete item is written.
  int* abort = flag + 1;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    for (int s = 0; s < SM::NSLOT; ++s) {
      mbar_init(&item_full[s], 1);
      mbar_init(&item_empty[s], 1);
    }
    *abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  const int n_items = *p.n_order * p.Hkv;

  if (warp == 4) {
    // ---------------------------------------------------------- producer warp
    // Per item: stage its metadata and Q rows in a slot (all lanes), then
    // lane 0 streams the item's K/V tiles into the TMA ring.
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    // Items are taken one at a time from a counter over the longest-first
    // order, so CTAs that drew short items simply take more of them.
    uint32_t it = 0;  // tiles issued (lane 0)
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      bool ok = true;
      int next = -1;
      if (lane == 0) {
        ok = mbar_wait_abortable(&item_empty[slot], ((k >> 1) & 1) ^ 1, kDevTimeoutEmpty, abort) &&
             !*reinterpret_cast<volatile int*>(abort);
        if (ok) next = atomicAdd(&p.work[0], 1);
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
      next = __shfl_sync(0xffffffffu, next, 0);
      uint8_t* sq = slots + slot * SM::SLOT;
      int* meta = reinterpret_cast<int*>(sq + 16 * SM::QROW);
      if (next >= n_items) {  // no work left: tell the consumers
        if (lane == 0) {
          meta[kMetaB] = -1;
          mbar_arrive(&item_full[slot]);
        }
        break;
      }
      const int e = p.order[next / p.Hkv];
      const int item = e * p.Hkv + next % p.Hkv;
      const int2 ent = p.entries[e];
      const int h = item % p.Hkv, b = ent.x;
      const int len = p.kv_len[b];
      const int tf = p.t_from[e];  // a row's tail item starts inside the chunk
      const int t_begin = tf >= 0 ? tf : ent.y * p.chunk_tokens;
      const int t_end = min(ent.y * p.chunk_tokens + p.chunk_tokens, len);
      const int members = p.width[e];  // nonzero for an entry in the order
      const int width = __popc(members);
      if (lane < 16) {
        int ke = len;
        if (width > 1) {
          // A shared chunk lies wholly below every query of its rows; a
          // member holding only its head sees keys up to its own pages.
          ke = t_end;
          if (lane < width * R) {
            const int kb = p.kv_bound[p.row_start[b + nth_bit(members, lane / R)] + ent.y];
            if (kb > 0) ke = kb;
          }
        } else if (lane < R) {
          ke = min(p.q_pos[(size_t)b * p.S + lane / p.G] + 1, len);
        }
        meta[kMetaKvEnd + lane] = ke;
      }
      if (lane == 0) {
        meta[kMetaB] = b;
        meta[kMetaH] = h;
        meta[kMetaBegin] = t_begin;
        meta[kMetaEnd] = t_end;
        meta[kMetaChunks] = p.row_chunks[b];
        meta[kMetaItem] = item;
        meta[kMetaWidth] = members;
        meta[kMetaChunk] = ent.y;
      }
      // Query row r of the item: query row r % R (= s * G + g) of the item's
      // (r / R)-th member row.
      for (int c = lane; c < 16 * (HD / 8); c += 32) {
        const int r = c / (HD / 8), ch = c % (HD / 8);
        uint4 val = make_uint4(0, 0, 0, 0);
        if (r < width * R) {
          const int bb = b + nth_bit(members, r / R), rr = r % R;
          const int s_ = rr / p.G, g = rr % p.G;
          val = *reinterpret_cast<const uint4*>(p.q + (((size_t)bb * p.S + s_) * p.Hq + (size_t)h * p.G + g) * HD +
                                                ch * 8);
        }
        *reinterpret_cast<uint4*>(sq + r * SM::QROW + ch * 16) = val;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&item_full[slot]);
        for (int t0 = t_begin; t0 < t_end; t0 += C::T, ++it) {
          const int st = it % C::STAGES;
          // A consumer that gave up sets `abort` before releasing its stage,
          // so a stage whose load may still be in flight is never reused.
          if (!mbar_wait_abortable(&empty[st], ((it / C::STAGES) & 1) ^ 1, kDevTimeoutEmpty, abort) ||
              *reinterpret_cast<volatile int*>(abort)) {
            ok = false;
            break;
          }
          issue_tile<HD>(&kmap, &vmap, kring + st * C::TILE_BYTES, vring + st * C::TILE_BYTES, &full[st], p, b,
                         h, t0, len);
        }
      }
      if (!__shfl_sync(0xffffffffu, ok, 0)) break;
    }
    // Every load this CTA issued lands before the CTA may exit (only the last
    // STAGES can still be in flight).
    if (lane == 0) {
      for (uint32_t j = it > (uint32_t)C::STAGES ? it - C::STAGES : 0u; j < it; ++j)
        mbar_drain(&full[j % C::STAGES], (j / C::STAGES) & 1);
      // The last CTA to finish taking work resets the counter for the next
      // launch (the next layer replays this kernel without a new plan).
      __threadfence();
      if (atomicAdd(&p.work[1], 1) == (int)gridDim.x - 1) {
        p.work[0] = 0;
        p.work[1] = 0;
      }
    }
    return;
  }

  // ------------------------------------------------------------ consumers
  const int tid = threadIdx.x;  // 0..127
  const int gid = lane >> 2, tig = lane & 3;
  uint32_t it = 0;
  for (int k = 0;; ++k) {
    const int slot = k & 1;
    bool alive = mbar_wait_abortable(&item_full[slot], (k >> 1) & 1, kDevTimeoutFull, abort);
    // All four consumer warps leave together (the barrier's OR) when any of
    // them found no staged item: its metadata would be garbage.
    if (named_barrier_or(1, 128, !alive)) break;
    const uint8_t* sq = slots + slot * SM::SLOT;
    const int* meta = reinterpret_cast<const int*>(sq + 16 * SM::QROW);
    const int b = meta[kMetaB], h = meta[kMetaH];
    if (b < 0) break;  // the producer found no work left (the same value for every consumer)
    const int t_begin = meta[kMetaBegin], t_end = meta[kMetaEnd];
    const int nchunks = meta[kMetaChunks];  // of row b (a shared chunk's rows all have more than one)
    const int members = meta[kMetaWidth], chunk = meta[kMetaChunk];
    const int width = __popc(members);
    const int item = meta[kMetaItem];
    const int kv_end[2] = {meta[kMetaKvEnd + gid], meta[kMetaKvEnd + gid + 8]};
    uint32_t qa[HD / 16][4];
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const uint8_t* row = sq + (gid + 8 * half) * SM::QROW;
        qa[kk][half] = *reinterpret_cast<const uint32_t*>(row + (kk * 16 + tig * 2) * 2);
        qa[kk][2 + half] = *reinterpret_cast<const uint32_t*>(row + (kk * 16 + 8 + tig * 2) * 2);
      }
    }

    float o[HD / 8][4];
#pragma unroll
    for (int d = 0; d < HD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
    float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

    for (int t0 = t_begin; t0 < t_end; t0 += C::T, ++it) {
      const int st = it % C::STAGES;
      if (alive && !mbar_wait_abortable(&full[st], (it / C::STAGES) & 1, kDevTimeoutFull, abort)) alive = false;
      if (alive) {
        const uint32_t kb = smem_u32(kring + st * C::TILE_BYTES);
        const uint32_t vb = smem_u32(vring + st * C::TILE_BYTES);
        const int rbase = warp * TW;
        if (t0 + rbase < t_end) {  // skip the empty tail of a partial tile
          float s[NJ][4];
          qk_tile<HD, NJ>(s, qa, kb, rbase, lane);
          online_softmax<HD, NJ>(s, o, m, l, t0 + rbase, kv_end, p.scale_log2, lane);
          pv_tile<HD, NJ>(o, s, vb, rbase, lane);
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[st]);
    }
    // An item with a tile that never arrived is not written (the CTA stops).
    if (named_barrier_or(1, 128, !alive)) break;

    // ---- merge the four warps' (m, l, o), R query rows at a time (one member
    // row of the item per round; a shared chunk has `width` of them)
    for (int bi = 0; bi < width; ++bi) {
      const int r0 = bi * R;
      if (bi > 0) named_barrier(1, 128);  // the previous round has read comb_*
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float lh = l[half];
        lh += __shfl_xor_sync(0xffffffffu, lh, 1);
        lh += __shfl_xor_sync(0xffffffffu, lh, 2);
        const int r = gid + 8 * half - r0;
        if (r >= 0 && r < R) {
          if (tig == 0) {
            comb_m[warp * R + r] = m[half];
            comb_l[warp * R + r] = lh;
          }
#pragma unroll
          for (int d = 0; d < HD / 8; ++d) {
            float2 v = make_float2(o[d][2 * half], o[d][2 * half + 1]);
            *reinterpret_cast<float2*>(&comb_o[((size_t)warp * R + r) * HD + d * 8 + tig * 2]) = v;
          }
        }
      }
      named_barrier(1, 128);
      const int bb = b + nth_bit(members, bi);
      // A lone item's partial goes to its own entry (a row's chunk or its
      // tail); a shared item's to each member's entry for the chunk.
      const size_t pit = width == 1 ? (size_t)item : ((size_t)p.row_start[bb] + chunk) * p.Hkv + h;
      for (int idx = tid; idx < R * HD; idx += 128) {
        const int r = idx / HD, col = idx % HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < 4; ++w) M = fmaxf(M, comb_m[w * R + r]);
        const float Mu = (M == -INFINITY) ? 0.f : M;
        float L = 0.f, O = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          const float f = exp2f(comb_m[w * R + r] - Mu);
          L += comb_l[w * R + r] * f;
          O += comb_o[((size_t)w * R + r) * HD + col] * f;
        }
        const float val = (L > 0.f) ? O / L : 0.f;
        if (nchunks == 1) {  // (width 1 only: a shared chunk's rows have later chunks)
          const int s_ = r / p.G, g = r % p.G;
          p.out[(((size_t)b * p.S + s_) * p.Hq + (size_t)h * p.G + g) * HD + col] = __float2bfloat16_rn(val);
        } else {
          p.part_o[(pit * R + r) * HD + col] = val;
          if (col == 0) p.part_lse[pit * R + r] = (L > 0.f) ? M + log2f(L) : -INFINITY;
        }
      }
    }
    if (nchunks > 1) {
      // Release this CTA's partials, take a ticket per covered row; the last
      // CTA of a (row, kv-head) acquires every partial and merges them.
      for (int bi = 0; bi < width; ++bi) {
        const int bb = b + nth_bit(members, bi);
        const int nch = p.row_chunks[bb];
        named_barrier(1, 128);
        if (tid == 0) {
          __threadfence();
          const int ticket = atomicAdd(&p.counters[bb * p.Hkv + h], 1);
          *flag = (ticket == nch - 1);
          if (*flag) __threadfence();
        }
        named_barrier(1, 128);
        if (*flag) {
          const int first = p.row_start[bb];
          for (int idx = tid; idx < R * HD; idx += 128) {
            const int r = idx / HD, col = idx % HD;
            float M = -INFINITY;
            for (int c = 0; c < nch; ++c)
              M = fmaxf(M, __ldcg(&p.part_lse[((size_t)(first + c) * p.Hkv + h) * R + r]));
            const float Mu = (M == -INFINITY) ? 0.f : M;
            float den = 0.f, num = 0.f;
            for (int c = 0; c < nch; ++c) {
              const size_t pc = (size_t)(first + c) * p.Hkv + h;
              const float f = exp2f(__ldcg(&p.part_lse[pc * R + r]) - Mu);
              den += f;
              num += f * __ldcg(&p.part_o[(pc * R + r) * HD + col]);
            }
            const int s_ = r / p.G, g = r % p.G;
            p.out[(((size_t)bb * p.S + s_) * p.Hq + (size_t)h * p.G + g) * HD + col] =
                __float2bfloat16_rn(den > 0.f ? num / den : 0.f);
          }
          if (tid == 0) p.counters[bb * p.Hkv + h] = 0;
        }
      }
    }
    named_barrier(1, 128);
    if (tid == 0) mbar_arrive(&item_empty[slot]);
  }
}

// Work list of (row, chunk) entries: max(1, ceil(kv_len / chunk)) per row,
// in row order, plus each row's first entry and chunk count, and the order
// the split kernel's CTAs take the entries in: longest chunk first (a
// counting sort on the chunk length in 64-token units), so the short chunks
// of short rows fill in at the end instead of leaving a tail of long ones.
// Also clears the per-(row, kv-head) tickets and the work counters. One CTA
// of 1024 threads.
//
// Shared chunks (block_table given): rows are taken in aligned blocks of
// NG = 16 / q_rows. In each block, the first row whose chunk j qualifies
// leads, and every row of the block whose chunk j lies on the very same pages
// (forked prefixes) joins its item: the K/V tiles are read once for all of
// their queries (at most 16 MMA rows). The item's entry holds the member
// rows as a bit mask (bit k: leader + k); the members' own entries get 0 and
// no item, their partials are written by the shared item. A chunk qualifies
// when it is whole and wholly below every query (end <= kv_len - q_rows).
constexpr int kPlanBuckets = 33;  // chunk lengths 0 .. 2048 in 64-token units

__global__ void __launch_bounds__(1024) decode_plan_kernel(const int32_t* kv_len, const int32_t* block_table,
                                                           int max_pages, int page_size, int B, int Hkv,
                                                           int q_rows, int chunk, int max_entries, int2* entries,
                                                           int* n_entries, int* row_start, int* row_chunks,
                                                           int* counters, int* order, int* n_order, int* width,
                                                           int* kv_bound, int* t_from, int* work) {
  __shared__ int warp_tot[32];
  __shared__ int total_s, n_order_s;
  __shared__ int hist[kPlanBuckets];
  __shared__ int cursor[kPlanBuckets];
  const int tid = threadIdx.x;
  if (tid < kPlanBuckets) hist[tid] = 0;
  if (tid == 0) n_order_s = 0;
  const int per = (B + 1023) / 1024;
  const int r0 = min(tid * per, B), r1 = min(r0 + per, B);
  const int unit = max(chunk / (kPlanBuckets - 1), 1);
  auto bucket_of = [&](int sz) {  // descending rank of an item of `sz` tokens
    return (kPlanBuckets - 1) - min((max(sz, 0) + unit - 1) / unit, kPlanBuckets - 1);
  };
  auto len_of = [&](int r) { return max(kv_len[r], 0); };
  auto chunks_of = [&](int r) { return max(1, (len_of(r) + chunk - 1) / chunk); };
  const bool share = block_table != nullptr && page_size > 0 && chunk % page_size == 0 && q_rows > 0 &&
                     q_rows <= 8;
  const int NG = share ? 16 / q_rows : 1;
  const int ppc = share ? chunk / page_size : 0;  // pages per chunk
  auto eligible = [&](int r, int j) {
    return (j + 1) * chunk <= len_of(r) - q_rows && (j + 1) * ppc <= max_pages;
  };
  // Leading pages of chunk j that rows ra and rb hold on the same page ids.
  auto common_pages = [&](int ra, int rb, int j) {
    const int lim = min(ppc, max_pages - j * ppc);
    const int32_t* ta = block_table + (size_t)ra * max_pages + (size_t)j * ppc;
    const int32_t* tb = block_table + (size_t)rb * max_pages + (size_t)j * ppc;
    int q = 0;
    while (q < lim && ta[q] >= 0 && ta[q] == tb[q]) ++q;
    return q;
  };
  // The row that leads chunk j in r's block: its first row whose chunk j is
  // whole and below every query; -1 when there is none.
  auto leader = [&](int r, int j) {
    const int blk0 = r - r % NG, blk1 = min(blk0 + NG, B);
    for (int x = blk0; x < blk1; ++x)
      if (eligible(x, j)) return x;
    return -1;
  };
  // Where row r's own pages start inside chunk j when it shares only the
  // chunk's head with the leader (a branch forked inside the chunk): that
  // token, or 0.
  auto head_bound = [&](int r, int j, int lead) {
    if (lead < 0 || lead == r) return 0;
    const int sp = common_pages(lead, r, j);
    if (sp == 0 || sp == ppc) return 0;
    const int bnd = j * chunk + sp * page_size;
    return bnd <= len_of(r) - q_rows ? bnd : 0;
  };
  auto joins = [&](int lead, int x, int j) {  // row x's chunk j (or its head) rides on lead's item
    return (eligible(x, j) && common_pages(lead, x, j) == ppc) || head_bound(x, j, lead) > 0;
  };
  // Rows whose item is entry (r, j)'s, as a mask over rows r .. r + NG - 1
  // (bit 0: r itself); 0 when the block leader's item covers the entry.
  auto members_of = [&](int r, int j) {
    if (NG == 1) return 1;
    const int lead = leader(r, j);
    if (lead < 0) return 1;
    if (lead != r) return joins(lead, r, j) ? 0 : 1;
    int mask = 1;
    const int blk1 = min(r - r % NG + NG, B);
    for (int x = r + 1; x < blk1; ++x)
      if (joins(r, x, j)) mask |= 1 << (x - r);
    return mask;
  };
  // The chunk whose head row r shares with its leader, so that the chunk's
  // rest is an extra item of the row (its "tail"), and where the tail
  // starts; -1 when the row has none.
  auto tail_of = [&](int r, int& bnd) {
    bnd = 0;
    if (NG == 1) return -1;
    const int c = chunks_of(r);
    for (int j = 0; j < c; ++j) {
      const int b_ = head_bound(r, j, leader(r, j));
      if (b_ > 0) {
        bnd = b_;
        return j;
      }
    }
    return -1;
  };
  int cnt = 0;
  for (int r = r0; r < r1; ++r) {
    int bnd;
    cnt += chunks_of(r) + (tail_of(r, bnd) >= 0 ? 1 : 0);
  }
  __syncthreads();
  // block exclusive scan of cnt
  const int lane = tid & 31, w = tid >> 5;
  int x = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[w] = x;
  __syncthreads();
  if (w == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += y;
    }
    warp_tot[lane] = t;  // inclusive
    if (lane == 31) total_s = t;
  }
  __syncthreads();
  int base = x - cnt + (w > 0 ? warp_tot[w - 1] : 0);
  const int total = total_s;
  if (total > max_entries) {
    if (tid == 0) {
      *n_entries = 0;
      *n_order = 0;
      work[0] = 0;
      work[1] = 0;
      report(kDevBadPage);
    }
    return;
  }
  int mine = 0;  // entries of this thread's rows that get an item
  for (int r = r0; r < r1; ++r) {
    const int len = len_of(r);
    const int c = chunks_of(r);
    int bnd;
    const int jt = tail_of(r, bnd);
    row_start[r] = base;
    row_chunks[r] = c + (jt >= 0 ? 1 : 0);
    for (int j = 0; j < c; ++j) {
      entries[base + j] = make_int2(r, j);
      const int wd = members_of(r, j);
      width[base + j] = wd;
      kv_bound[base + j] = j == jt ? bnd : 0;  // read by the leader's item for this row's queries
      t_from[base + j] = -1;
      if (wd > 0) {
        atomicAdd(&hist[bucket_of(min(chunk, len - j * chunk))], 1);
        ++mine;
      }
    }
    if (jt >= 0) {  // the tail: tokens bnd .. of chunk jt, an item of this row alone
      entries[base + c] = make_int2(r, jt);
      width[base + c] = 1;
      kv_bound[base + c] = 0;
      t_from[base + c] = bnd;
      atomicAdd(&hist[bucket_of(min(len, (jt + 1) * chunk) - bnd)], 1);
      ++mine;
    }
    base += c + (jt >= 0 ? 1 : 0);
  }
  atomicAdd(&n_order_s, mine);
  for (int i = tid; i < B * Hkv; i += 1024) counters[i] = 0;
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int k = 0; k < kPlanBuckets; ++k) {
      cursor[k] = acc;
      acc += hist[k];
    }
    *n_entries = total;
    *n_order = n_order_s;
    work[0] = 0;
    work[1] = 0;
  }
  __syncthreads();
  base = x - cnt + (w > 0 ? warp_tot[w - 1] : 0);
  for (int r = r0; r < r1; ++r) {
    const int len = len_of(r);
    const int c = chunks_of(r);
    for (int j = 0; j < c; ++j)
      if (width[base + j] > 0) order[atomicAdd(&cursor[bucket_of(min(chunk, len - j * chunk))], 1)] = base + j;
    if (row_chunks[r] > c) {
      const int jt = entries[base + c].y;
      order[atomicAdd(&cursor[bucket_of(min(len, (jt + 1) * chunk) - t_from[base + c])], 1)] = base + c;
    }
    base += row_chunks[r];
  }
}

// Block mode: one CTA per (64-row query block, kv-head, row).
template <int HD>
__global__ void __launch_bounds__(160) block_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                                                           const __grid_constant__ CUtensorMap vmap,
                                                           const AttnParams p) {
  using C = AttnTile<HD>;
  constexpr int NJ = C::T / 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* kring = smem;
  uint8_t* vring = smem + C::STAGES * C::TILE_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * C::STAGES * C::TILE_BYTES);
  uint64_t* empty = full + C::STAGES;
  __shared__ int kv_hi_s;
  __shared__ int abort_s;  // as in the split kernel: the first wait that runs out stops the CTA

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int R = p.R;
  const int len = p.kv_len[b];
  if (threadIdx.x == 0) {
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    abort_s = 0;
    fence_barrier_init();
    // KV range this block needs: up to the largest q_pos of its rows.
    const int r_lo = qb * 64, r_hi = min(r_lo + 64, R);
    int mx = -1;
    for (int s = r_lo / p.G; s <= (r_hi - 1) / p.G; ++s) mx = max(mx, p.q_pos[(size_t)b * p.S + s]);
    kv_hi_s = min(mx + 1, len);
  }
  __syncthreads();
  const int kv_hi = kv_hi_s;

  if (warp == 4) {
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      uint32_t it = 0;  // tiles issued
      for (int t0 = 0; t0 < kv_hi; t0 += C::T, ++it) {
        const int st = it % C::STAGES;
        if (!mbar_wait_abortable(&empty[st], ((it / C::STAGES) & 1) ^ 1, kDevTimeoutEmpty, &abort_s) ||
            *reinterpret_cast<volatile int*>(&abort_s))
          break;
        issue_tile<HD>(&kmap, &vmap, kring + st * C::TILE_BYTES, vring + st * C::TILE_BYTES, &full[st], p, b, h,
                       t0, len);
      }
      // The issued loads land before the CTA may exit.
      for (uint32_t j = it > (uint32_t)C::STAGES ? it - C::STAGES : 0u; j < it; ++j)
        mbar_drain(&full[j % C::STAGES], (j / C::STAGES) & 1);
    }
    return;
  }

  const int gid = lane >> 2, tig = lane & 3;
  const int row0 = qb * 64 + warp * 16;
  int kv_end[2];
  int warp_hi = 0;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = row0 + gid + 8 * half;
    kv_end[half] = (r < R) ? min(p.q_pos[(size_t)b * p.S + r / p.G] + 1, len) : 0;
    warp_hi = max(warp_hi, kv_end[half]);
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) warp_hi = max(warp_hi, __shfl_xor_sync(0xffffffffu, warp_hi, o));

  uint32_t qa[HD / 16][4];
  load_q_frags<HD>(qa, p, b, h, row0, R, lane);
  float o[HD / 8][4];
#pragma unroll
  for (int d = 0; d < HD / 8; ++d) o[d][0] = o[d][1] = o[d][2] = o[d][3] = 0.f;
  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};

  bool alive = true;
  uint32_t it = 0;
  for (int t0 = 0; t0 < kv_hi; t0 += C::T, ++it) {
    const int st = it % C::STAGES;
    if (alive && !mbar_wait_abortable(&full[st], (it / C::STAGES) & 1, kDevTimeoutFull, &abort_s)) alive = false;
    if (alive && t0 < warp_hi) {
      const uint32_t kb = smem_u32(kring + st * C::TILE_BYTES);
      const uint32_t vb = smem_u32(vring + st * C::TILE_BYTES);
      float s[NJ][4];
      qk_tile<HD, NJ>(s, qa, kb, 0, lane);
      online_softmax<HD, NJ>(s, o, m, l, t0, kv_end, p.scale_log2, lane);
      pv_tile<HD, NJ>(o, s, vb, 0, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);
  }
  // Rows whose keys did not all arrive are not written.
  if (named_barrier_or(1, 128, !alive)) return;

#pragma unroll
  for (int half = 0; half < 2; ++half) {
    l[half] += __shfl_xor_sync(0xffffffffu, l[half], 1);
    l[half] += __shfl_xor_sync(0xffffffffu, l[half], 2);
    const int r = row0 + gid + 8 * half;
    if (r < R) {
      const int s = r / p.G, g = r % p.G;
      __nv_bfloat16* dst = p.out + (((size_t)b * p.S + s) * p.Hq + (size_t)h * p.G + g) * HD;
      const float inv = (l[half] > 0.f) ? 1.f / l[half] : 0.f;
#pragma unroll
      for (int d = 0; d < HD / 8; ++d) {
        *reinterpret_cast<uint32_t*>(dst + d * 8 + tig * 2) =
            pack_bf16x2(o[d][2 * half] * inv, o[d][2 * half + 1] * inv);
      }
    }
  }
}

// ------------------------------------------------------------------ host side

// Tokens per split-mode work item. Measured on B200 (K1 share of the copy
// bandwidth): hd 128 decode of 256 rows with U[64,4096] contexts 0.82 at 1024,
// 0.87 at 2048, 0.86 at 4096; hd 64 with 512 rows log-uniform in [128,16384]
// 0.76 at 2048, 0.73 at 4096, 0.65 at 8192.
size_t decode_chunk_tokens(int) { return 2048; }

size_t decode_workspace_layout(int B, int Hkv, int R, int head_dim, int max_kv_len, WorkspaceLayout* lay) {
  const size_t chunk = decode_chunk_tokens(head_dim);
  const size_t per_row = std::max<size_t>(1, ((size_t)std::max(max_kv_len, 0) + chunk - 1) / chunk);
  const size_t max_entries = (size_t)B * (per_row + 1);  // + one tail entry per row (shared plans)
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t off = 0;
  lay->max_entries = max_entries;
  lay->entries = off;    off = up(off + max_entries * sizeof(int2));
  lay->n_entries = off;  off = up(off + sizeof(int));
  lay->row_start = off;  off = up(off + (size_t)B * sizeof(int));
  lay->row_chunks = off; off = up(off + (size_t)B * sizeof(int));
  lay->counters = off;   off = up(off + (size_t)B * Hkv * sizeof(int));
  lay->order = off;      off = up(off + max_entries * sizeof(int));
  lay->n_order = off;    off = up(off + sizeof(int));
  lay->width = off;      off = up(off + max_entries * sizeof(int));
  lay->kv_bound = off;   off = up(off + max_entries * sizeof(int));
  lay->t_from = off;     off = up(off + max_entries * sizeof(int));
  lay->work = off;       off = up(off + 2 * sizeof(int));
  lay->part_lse = off;   off = up(off + max_entries * Hkv * R * sizeof(float));
  lay->part_o = off;     off = up(off + max_entries * Hkv * R * head_dim * sizeof(float));
  lay->total = off;
  return off;
}

// SM count of the current device, cached per device ordinal (several host
// threads may launch at once: the cache entries are atomics).
static int num_sms() {
  static std::atomic<int> cache[kMaxDevices];
  const int dev = device_slot();
  if (dev < 0) return 148;
  int n = cache[dev].load(std::memory_order_relaxed);
  if (n <= 0) {
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev].store(n, std::memory_order_relaxed);
  }
  return n;
}

template <int HD>
static cudaError_t launch_split(const CUtensorMap& km, const CUtensorMap& vm, const AttnParams& p,
                                size_t max_items, cudaStream_t stream) {
  const size_t smem = SplitSmem<HD>::bytes(p.R);
  cudaError_t e = cudaFuncSetAttribute(split_decode_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, split_decode_kernel<HD>, 160, smem);
  if (e != cudaSuccess) return e;
  occ = std::max(occ, 1);
  const size_t grid = std::min<size_t>((size_t)num_sms() * occ, std::max<size_t>(max_items, 1));
  split_decode_kernel<HD><<<(unsigned)grid, 160, smem, stream>>>(km, vm, p);
  return cudaGetLastError();
}

template <int HD>
static cudaError_t launch_block(const CUtensorMap& km, const CUtensorMap& vm, const AttnParams& p,
                                cudaStream_t stream) {
  const size_t smem = 1024 + 2 * AttnTile<HD>::STAGES * AttnTile<HD>::TILE_BYTES + 2 * AttnTile<HD>::STAGES * 8;
  cudaError_t e = cudaFuncSetAttribute(block_decode_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((p.R + 63) / 64, p.Hkv, p.B);
  block_decode_kernel<HD><<<grid, 160, smem, stream>>>(km, vm, p);
  return cudaGetLastError();
}

cudaError_t launch_decode_plan(const int32_t* kv_len, const int32_t* block_table, int max_pages, int page_size,
                               int B, int Hkv, int q_rows, int head_dim, const WorkspaceLayout& lay, uint8_t* ws,
                               cudaStream_t stream) {
  decode_plan_kernel<<<1, 1024, 0, stream>>>(
      kv_len, block_table, max_pages, page_size, B, Hkv, q_rows, (int)decode_chunk_tokens(head_dim),
      (int)lay.max_entries, reinterpret_cast<int2*>(ws + lay.entries), reinterpret_cast<int*>(ws + lay.n_entries),
      reinterpret_cast<int*>(ws + lay.row_start), reinterpret_cast<int*>(ws + lay.row_chunks),
      reinterpret_cast<int*>(ws + lay.counters), reinterpret_cast<int*>(ws + lay.order),
      reinterpret_cast<int*>(ws + lay.n_order), reinterpret_cast<int*>(ws + lay.width),
      reinterpret_cast<int*>(ws + lay.kv_bound), reinterpret_cast<int*>(ws + lay.t_from),
      reinterpret_cast<int*>(ws + lay.work));
  return cudaGetLastError();
}

cudaError_t launch_decode_attention(const CUtensorMap& km, const CUtensorMap& vm, AttnParams p,
                                    const WorkspaceLayout& lay, uint8_t* ws, bool split, cudaStream_t stream) {
  if (split) {
    p.chunk_tokens = (int)decode_chunk_tokens(p.head_dim);
    p.entries = reinterpret_cast<const int2*>(ws + lay.entries);
    p.n_entries = reinterpret_cast<const int*>(ws + lay.n_entries);
    p.row_start = reinterpret_cast<const int*>(ws + lay.row_start);
    p.row_chunks = reinterpret_cast<const int*>(ws + lay.row_chunks);
    p.counters = reinterpret_cast<int*>(ws + lay.counters);
    p.order = reinterpret_cast<const int*>(ws + lay.order);
    p.n_order = reinterpret_cast<const int*>(ws + lay.n_order);
    p.width = reinterpret_cast<const int*>(ws + lay.width);
    p.kv_bound = reinterpret_cast<const int*>(ws + lay.kv_bound);
    p.t_from = reinterpret_cast<const int*>(ws + lay.t_from);
    p.work = reinterpret_cast<int*>(ws + lay.work);
    p.part_lse = reinterpret_cast<float*>(ws + lay.part_lse);
    p.part_o = reinterpret_cast<float*>(ws + lay.part_o);
    const size_t max_items = lay.max_entries * p.Hkv;
    return p.head_dim == 128 ? launch_split<128>(km, vm, p, max_items, stream)
                             : launch_split<64>(km, vm, p, max_items, stream);
  }
  return p.head_dim == 128 ? launch_block<128>(km, vm, p, stream) : launch_block<64>(km, vm, p, stream);
}

}  // namespace mb
