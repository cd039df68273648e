// K5: packed varlen segment-causal GQA attention forward on tcgen05.
//
// Replaces the FlexAttention call of flex_packed_forward
// (src/mouse_core/models/backbone/flex_train.py:147) with its mask
// (flex_train.py:98-102): query i attends key j iff j <= i and both lie in the
// same segment. Segments are runs of sequence_ids; K7 turns them into
// run_start[i] (the smallest j token i may see) and tile_lo[t] (run_start of
// query tile t's first token), so the mask is run_start[i] <= j <= i and no
// BlockMask is needed: a query tile only visits key tiles from
// tile_lo[t] / 128 to its diagonal.
//
// Work tile = one 128-token query tile x one pair of q-heads sharing a
// kv-head (a single q-head when the GQA group is odd). The kernel is
// persistent: one CTA per SM takes tiles from a counter, longest-history
// query tiles first; the producer hands each tile id to the other warps
// through a two-slot ring, and barrier phases follow a running key-tile count
// across tiles. Q is released after a tile's last Q K^T MMA, so the next
// tile's Q loads during the last softmax, P V and epilogue; O is released
// once the epilogue has read it. Warp roles of the training forward (320
// threads):
//   warp 0      TMA producer: Q once per tile, K/V tiles through a 2-3 stage ring
//   warp 1      TMEM allocator; the whole warp issues every tcgen05.mma
//   warps 2-5   softmax of head 0 (thread = query row = TMEM lane), then
//               the tile's epilogue for it
//   warps 6-9   softmax of head 1, then its epilogue
// The paged prefill (512 threads, four warpgroups) moves the epilogue to its
// own warps: warps 0-1 as above, 2-3 idle (they complete the control
// warpgroup), 4-7 and 8-11 softmax, 12-15 the epilogue of both heads, which
// drains a tile's O while the softmax warps already work on the next tile;
// it is launched with 128 registers a thread and setmaxnreg moves them from
// the control and epilogue warpgroups to the softmax ones (FwdRegs).
// Tensor memory (512 columns): S_h = Q_h K^T at columns 128h, O_h at 256 + HD h.
// Softmax reads S, writes P (bf16 pairs) back over the first 64 columns of
// S_h, and the MMA O_h += P V takes P straight from TMEM. The two heads
// ping-pong: while one head's softmax runs, the tensor core works on the
// other head. O is rescaled only when a row maximum grows by more than 2^8
// (exact: the final normalisation uses the same stale maximum).
// Outputs: out [L, Hq, HD] bf16 and lse [Hq, L] f32 in log2 units of the
// scaled scores (log2 sum 2^(s * scale * log2 e)).
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

#include <atomic>

namespace mb {

// Block: 16 warps in four warpgroups (see the role table above). The block is
// launched with 128 registers a thread; setmaxnreg then moves them from the
// control and epilogue warpgroups to the two softmax warpgroups.
// The paged prefill's work tiles are short (1-8 key tiles for a rebuild
// window), so a dedicated epilogue warpgroup drains O there while the softmax
// warps start the next tile (512 threads, setmaxnreg split below). The
// training forward's tiles are longer and ran ~4% slower that way (the extra
// warps share the sub-partitions), so it keeps the softmax warps draining O
// themselves (320 threads, 168 registers each).
template <bool PAGED>
constexpr int fwd_threads() {
  return PAGED ? 512 : 320;
}
constexpr int kFwdLaunchRegs = 128;  // 65536 / 512: the paged prefill's launch allocation
struct FwdRegs {  // paged prefill: control, epilogue and softmax warpgroups
  static constexpr int ctrl = 56, epi = 80, softmax = 184;
  static_assert(128 * ctrl + 128 * epi + 256 * softmax <= 512 * kFwdLaunchRegs,
                "the register split must fit the launch allocation");
};

template <int HD>
struct FwdTile {
  static constexpr int BM = 128, BN = 128;
  static constexpr int NCB = HD / 64;                 // 64-element column blocks
  static constexpr int BOX = 128 * 128;               // bytes of a 64 x 128-row box
  static constexpr int QTILE = NCB * BOX;             // one head's Q tile
  static constexpr int KVTILE = NCB * BOX;            // one K (or V) tile
  static constexpr int STAGES = HD == 128 ? 2 : 3;
  static constexpr int RING = 2 * STAGES * KVTILE;
  static constexpr int SMEM = 1024 + 2 * QTILE + RING + 4352;
  static constexpr uint32_t TMEM_COLS = 512;
};

struct FwdBarriers {
  uint64_t tile_full[2], tile_empty[2];  // tile-id ring (producer -> MMA + softmax warps)
  uint64_t q_full, q_empty;
  uint64_t k_full[3], v_full[3], kv_empty[3];
  uint64_t s_full[2], p_full[2];
  uint64_t o_full, o_empty;
  uint64_t stats_full[2];  // a tile's row max / row sum handed from the softmax to the epilogue warps
  uint64_t mma_drain;      // every MMA of the CTA complete, before TMEM is freed
  uint32_t tmem_base;
  int tile[2];
  int q_armed;  // Q tiles whose loads the producer issued (kept here: its registers are few)
  float stats[2][2][2][128];  // [tile parity][head][max, sum][row]
};
static_assert(sizeof(FwdBarriers) <= 4352, "barrier / stats block outgrew its shared memory share");

// One work tile: 128 query rows starting at flat row q0 (rows up to row_end
// belong to it), q-heads h0 .. h0 + heads_per_cta - 1 over kv-head kvh, and
// its key tiles t_lo .. t_lo + n - 1. Paged prefill: row b of the batch,
// key tiles of that row's cache.
struct FwdWork {
  int q0, row_end, h0, kvh, qt, t_lo, n, b;
};

constexpr int kPrefillRowBlock = 4;
// Score of a masked key (-2^90): its exponential is 0 (or, on the FMA-pipe
// path, 2^-126), and a row max equal to it means no visible key.
constexpr float kMaskedScore = -1.2379401e27f;

template <bool PAGED>
__device__ __forceinline__ FwdWork fwd_work(int tile, const VarlenParams& p) {
  const int groups = p.Hq / p.heads_per_cta;
  FwdWork w;
  w.h0 = (tile % groups) * p.heads_per_cta;
  w.kvh = w.h0 / p.G;
  if constexpr (PAGED) {
    // Rows in blocks of kPrefillRowBlock; inside a block, later query tiles
    // (more keys) first, then row, then head group. The query tiles that read
    // the same row's K/V run close together, so the re-reads hit L2.
    const int n_qt = (p.S + 127) / 128;
    const int rest = tile / groups;
    const int blk = rest / (kPrefillRowBlock * n_qt);
    const int r_in = rest - blk * kPrefillRowBlock * n_qt;
    const int nb = min(kPrefillRowBlock, p.B - blk * kPrefillRowBlock);  // rows in this block
    w.qt = n_qt - 1 - r_in / nb;
    w.b = blk * kPrefillRowBlock + r_in % nb;
    w.q0 = w.b * p.S + w.qt * 128;
    w.row_end = w.b * p.S + p.S;
    // q_pos grows along a row (left pads sit at 0), so the tile's last row
    // bounds the keys it needs; a tile with no key still runs one masked one.
    const int last = min(w.qt * 128 + 127, p.S - 1);
    const int hi = min(p.q_pos[(size_t)w.b * p.S + last] + 1, p.kv_len[w.b]);
    w.t_lo = 0;
    w.n = max(1, (hi + 127) / 128);
  } else {
    const int n_qt = (p.L + 127) / 128;
    w.qt = n_qt - 1 - tile / groups;  // longest-history tiles of a stream first
    w.b = 0;
    w.q0 = w.qt * 128;
    w.row_end = p.L;
    w.t_lo = p.tile_lo[w.qt] / 128;
    w.n = min(w.q0 + 127, p.L - 1) / 128 - w.t_lo + 1;
  }
  return w;
}

// K or V key tile [kv0, kv0 + 128) of row b, kv-head kvh from the page pool:
// two 64-row boxes per 64-column block (a 64- or 128-token page holds whole
// boxes), written where the contiguous kernel's 128-row box would put them.
// Boxes past the row's keys or the block table read zeros (y = -64).
template <int HD>
__device__ __forceinline__ void load_paged_kv(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                              const VarlenParams& p, int b, int kvh, int kv0) {
  using C = FwdTile<HD>;
  const int len = p.kv_len[b];
#pragma unroll
  for (int g = 0; g < 2; ++g) {
    const int tok = kv0 + 64 * g;
    int y = -64;
    if (tok < len) {
      const int pidx = tok / p.page_size;
      const int pg = pidx < p.max_pages ? p.block_table[(size_t)b * p.max_pages + pidx] : -1;
      if (pg >= 0 && pg < p.num_pages)
        y = (pg * p.Hkv + kvh) * p.page_size + tok % p.page_size;
      else
        report(kDevBadPage);
    }
#pragma unroll
    for (int cb = 0; cb < C::NCB; ++cb) tma_load_2d(dst + cb * C::BOX + g * (C::BOX / 2), map, bar, cb * 64, y);
  }
}

template <int HD, bool PAGED>
__global__ void __launch_bounds__(fwd_threads<PAGED>(), 1) varlen_fwd_kernel(const __grid_constant__ CUtensorMap qmap,
                                                           const __grid_constant__ CUtensorMap kmap,
                                                           const __grid_constant__ CUtensorMap vmap,
                                                           const VarlenParams p) {
  using C = FwdTile<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;                         // [2][QTILE]
  uint8_t* ks = smem + 2 * C::QTILE;          // [STAGES][KVTILE]
  uint8_t* vs = ks + C::STAGES * C::KVTILE;   // [STAGES][KVTILE]
  FwdBarriers* bars = reinterpret_cast<FwdBarriers*>(vs + C::STAGES * C::KVTILE);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int hpc = p.heads_per_cta;
  const int n_work = PAGED ? p.B * ((p.S + C::BM - 1) / C::BM) * (p.Hq / hpc)
                           : ((p.L + C::BM - 1) / C::BM) * (p.Hq / hpc);

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->tile_full[s], 1);
      mbar_init(&bars->tile_empty[s], PAGED ? 13 : 9);  // MMA warp + 8 softmax warps (+ 4 epilogue warps)
      mbar_init(&bars->stats_full[s], 8);
    }
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_empty, 1);
    for (int s = 0; s < C::STAGES; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int h = 0; h < 2; ++h) {
      mbar_init(&bars->s_full[h], 1);
      mbar_init(&bars->p_full[h], 4);
    }
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, PAGED ? 4 : 8);  // whoever drains O
    mbar_init(&bars->mma_drain, 1);
    bars->q_armed = 0;
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  // Tile k of this CTA from the ring (each consumer warp reads every slot once).
  auto take_tile = [&](int k, bool& ok) {
    ok = mbar_wait_warp(&bars->tile_full[k & 1], (k >> 1) & 1, kDevTimeoutFull);
    const int tile = ok ? *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) : -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->tile_empty[k & 1]);
    return tile;
  };

  constexpr int kSoftmaxWarp0 = PAGED ? 4 : 2;
  if (warp < kSoftmaxWarp0) {
  if constexpr (PAGED) regs_dec<FwdRegs::ctrl>();
  if (warp == 0) {
    // ------------------------------------------------------------ producer
    bool ok = true;
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    int J = 0;  // K/V tile pairs issued so far (lane 0): ring slots and phases continue
    for (int k = 0; ok; ++k) {
      int tile = -1;
      if (lane == 0) {
        if (PAGED && p.tile_counter == nullptr)  // one tile per CTA
          tile = k == 0 ? (int)blockIdx.x : -1;
        else
          tile = k == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(p.tile_counter, 1);
        if (tile >= n_work) tile = -1;
        ok = mbar_wait(&bars->tile_empty[k & 1], ((k >> 1) & 1) ^ 1, kDevTimeoutEmpty);
        if (ok) {
          *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) = tile;
          mbar_arrive(&bars->tile_full[k & 1]);
        }
      }
      tile = __shfl_sync(0xffffffffu, tile, 0);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || tile < 0) break;
      const FwdWork w = fwd_work<PAGED>(tile, p);
      if (lane == 0) {
        // The Q slots are free once the previous tile's last Q K^T completed.
        if (k > 0) ok = mbar_wait(&bars->q_empty, (k - 1) & 1, kDevTimeoutEmpty);
        if (ok) {
          mbar_arrive_expect_tx(&bars->q_full, hpc * C::QTILE);
          for (int hh = 0; hh < hpc; ++hh)
            for (int cb = 0; cb < C::NCB; ++cb)
              tma_load_3d(qs + hh * C::QTILE + cb * C::BOX, &qmap, &bars->q_full, cb * 64, w.h0 + hh, w.q0);
          *reinterpret_cast<volatile int*>(&bars->q_armed) = k + 1;
        }
        int j = 0;
        for (; ok && j < w.n; ++j) {
          const int jj = J + j;
          const int st = jj % C::STAGES;
          if (!(ok = mbar_wait(&bars->kv_empty[st], ((jj / C::STAGES) & 1) ^ 1, kDevTimeoutEmpty))) break;
          const int kv0 = (w.t_lo + j) * C::BN;
          mbar_arrive_expect_tx(&bars->k_full[st], C::KVTILE);
          if constexpr (PAGED) {
            load_paged_kv<HD>(ks + st * C::KVTILE, &kmap, &bars->k_full[st], p, w.b, w.kvh, kv0);
          } else {
            for (int cb = 0; cb < C::NCB; ++cb)
              tma_load_3d(ks + st * C::KVTILE + cb * C::BOX, &kmap, &bars->k_full[st], cb * 64, w.kvh, kv0);
          }
          mbar_arrive_expect_tx(&bars->v_full[st], C::KVTILE);
          if constexpr (PAGED) {
            load_paged_kv<HD>(vs + st * C::KVTILE, &vmap, &bars->v_full[st], p, w.b, w.kvh, kv0);
          } else {
            for (int cb = 0; cb < C::NCB; ++cb)
              tma_load_3d(vs + st * C::KVTILE + cb * C::BOX, &vmap, &bars->v_full[st], cb * 64, w.kvh, kv0);
          }
        }
        J += j;  // w.n, or the pairs issued before a wait ran out
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    // Every load issued lands before the CTA exits, also when a wait ran out.
    if (lane == 0) {
      drain_ring(&bars->q_full, 1, *reinterpret_cast<volatile int*>(&bars->q_armed));
      drain_ring(bars->k_full, C::STAGES, J);
      drain_ring(bars->v_full, C::STAGES, J);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    // The whole warp runs this loop; each group of MMAs is one straight-line
    // asm block issued by an elected lane.
    constexpr uint32_t ID_QK = umma_idesc_bf16(128, 128, 0, 0);
    constexpr uint32_t ID_PV = umma_idesc_bf16(128, HD, 0, 1);
    auto issue_qk = [&](int hh, int st) {
      const uint64_t dq = umma_desc_sw128(smem_u32(qs + hh * C::QTILE), 16, 1024);
      const uint64_t dk = umma_desc_sw128(smem_u32(ks + st * C::KVTILE), 16, 1024);
      if constexpr (HD == 128)
        umma_ss_k128_warp(tbase + 128 * hh, dq, dk, ID_QK);
      else
        umma_ss_k64_warp(tbase + 128 * hh, dq, dk, ID_QK);
      umma_commit_warp(&bars->s_full[hh]);
    };
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const int n = fwd_work<PAGED>(tile, p).n;
      if (!(ok = mbar_wait_warp(&bars->q_full, k & 1, kDevTimeoutFull))) break;
      if (!(ok = mbar_wait_warp(&bars->k_full[J % C::STAGES], (J / C::STAGES) & 1, kDevTimeoutFull))) break;
      for (int hh = 0; hh < hpc; ++hh) issue_qk(hh, J % C::STAGES);
      if (n == 1) umma_commit_warp(&bars->q_empty);  // that was the tile's last Q K^T
      for (int j = 0; ok && j < n; ++j) {
        const int jj = J + j;
        const int st = jj % C::STAGES;
        if (!(ok = mbar_wait_warp(&bars->v_full[st], (jj / C::STAGES) & 1, kDevTimeoutFull))) break;
        const bool more = j + 1 < n;
        const int st1 = (jj + 1) % C::STAGES;
        bool k_next = false;
        const uint64_t dv = umma_desc_sw128(smem_u32(vs + st * C::KVTILE), C::BOX, 1024);
        for (int hh = 0; hh < hpc; ++hh) {
          if (!(ok = mbar_wait_warp(&bars->p_full[hh], jj & 1, kDevTimeoutFull))) break;
          // The tile's first P V overwrites O: the previous epilogue must hold it.
          if (j == 0 && hh == 0 && k > 0 && !(ok = mbar_wait_warp(&bars->o_empty, (k - 1) & 1, kDevTimeoutFull)))
            break;
          // O_h += P_h V (P bf16 in the first 64 columns of S_h)
          umma_ts_t128_linear_warp(tbase + 256 + HD * hh, tbase + 128 * hh, dv, ID_PV, j > 0 ? 1u : 0u);
          if (more) {
            if (!k_next) {
              if (!(ok = mbar_wait_warp(&bars->k_full[st1], ((jj + 1) / C::STAGES) & 1, kDevTimeoutFull))) break;
              k_next = true;
            }
            issue_qk(hh, st1);
          }
        }
        if (!ok) break;
        if (more && j + 2 == n) umma_commit_warp(&bars->q_empty);  // the tile's last Q K^T is queued
        umma_commit_warp(&bars->kv_empty[st]);
      }
      if (!ok) break;
      umma_commit_warp(&bars->o_full);
      J += n;
    }
    umma_drain_warp(&bars->mma_drain);  // before TMEM is freed, also when a wait ran out
  }
  } else if (warp < kSoftmaxWarp0 + 8) {
    if constexpr (PAGED) regs_inc<FwdRegs::softmax>();
    // ------------------------------------------------------------ softmax
    const int hh = (warp - kSoftmaxWarp0) >> 2;
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    const int r = sub * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    const uint32_t t_s = tbase + 128 * hh + lane_bits;
    const uint32_t t_o = tbase + 256 + HD * hh + lane_bits;
    const bool active = hh < hpc;
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const FwdWork w = fwd_work<PAGED>(tile, p);
      const int q_tok = w.q0 + r;  // flat query row
      const bool row_ok = q_tok < w.row_end;
      int lo, hi;
      if constexpr (PAGED) {  // cached keys 0 .. q_pos of the row (none past its length)
        lo = 0;
        hi = row_ok ? min(p.q_pos[q_tok], p.kv_len[w.b] - 1) : -1;
      } else {  // same segment, causal
        lo = row_ok ? p.run_start[q_tok] : 0x7fffffff;
        hi = q_tok;
      }
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; active && j < w.n; ++j) {
        const int jj = J + j;
        const int kv0 = (w.t_lo + j) * C::BN;
        if (ok) ok = mbar_wait_warp(&bars->s_full[hh], jj & 1, kDevTimeoutFull);
        tc_fence_after();
        float alpha = 1.f;
        bool rescale = false;
        if (ok) {
          const bool full = row_ok && kv0 >= lo && kv0 + C::BN - 1 <= hi;
          // One TMEM read of the whole 128-column score row into registers.
          uint32_t v[128];
#pragma unroll
          for (int c = 0; c < 4; ++c) tmem_ld32(t_s + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
          tmem_wait_ld();
          if (!full) {
            // Keys outside [lo, hi] go to kMaskedScore by arithmetic alone:
            // the minimum with two linear bounds, huge inside the row's key
            // range and hugely negative past either end of it, then the
            // maximum with kMaskedScore (a score no real one comes near).
            const float big = 1.2676506e30f;  // 2^100
            const float lo_e = row_ok ? (float)max(lo - kv0, 0) - 0.5f : 1000.f;
            const float hi_e = row_ok ? (float)min(hi - kv0, C::BN - 1) + 0.5f : -1000.f;
            const float hb = hi_e * big, lb = -lo_e * big;
#pragma unroll
            for (int e = 0; e < 128; ++e) {
              const float m = fmin3(__uint_as_float(v[e]), fmaf(-(float)e, big, hb), fmaf((float)e, big, lb));
              v[e] = __float_as_uint(fmaxf(m, kMaskedScore));
            }
          }
          // Row max and (below) row sum as 8 independent chains: one long
          // dependent chain per thread would serialise the softmax warp.
          // Three-input maxima halve the max instructions.
          float mp[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) mp[q] = fmaxf(__uint_as_float(v[q]), __uint_as_float(v[8 + q]));
#pragma unroll
          for (int e = 16; e < 128; e += 16)
#pragma unroll
            for (int q = 0; q < 8; ++q) mp[q] = fmax3(mp[q], __uint_as_float(v[e + q]), __uint_as_float(v[e + 8 + q]));
          float mx = fmax3(fmax3(mp[0], mp[1], mp[2]), fmax3(mp[3], mp[4], mp[5]), fmaxf(mp[6], mp[7]));
          if (mx <= kMaskedScore) mx = -INFINITY;  // no key of this tile is visible to the row
          // The scale is positive, so the max of raw scores gives the max of scaled ones.
          const float m_tile = mx * p.scale_log2;
          const float m_new = fmaxf(m_used, m_tile);
          if (m_new > m_used + 8.f) {
            rescale = true;
            alpha = exp2f(m_used - m_new);
            m_used = m_new;
          }
          const float neg_mu = (m_used == -INFINITY) ? 0.f : -m_used;
          float ls[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) ls[q] = 0.f;
          // Scale and shift, exponentials and row sums on packed fp32 pairs.
          // In the training forward one pair in four takes its 2^x on the FMA
          // pipe (exp2_fma2, relative error 1e-4), which unloads the SFU, the
          // bound of this loop; the paged prefill, whose outputs feed the
          // decode cache, keeps every exponential on the SFU.
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[16];
#pragma unroll
            for (int e = 0; e < 32; e += 2) {
              float x0, x1, p0, p1;
              ffma2(x0, x1, __uint_as_float(v[32 * c + e]), __uint_as_float(v[32 * c + e + 1]), p.scale_log2,
                    p.scale_log2, neg_mu, neg_mu);
              if (!PAGED && ((e >> 1) & 7) >= 6) {
                exp2_fma2(p0, p1, x0, x1);
              } else {
                p0 = fast_exp2(x0);
                p1 = fast_exp2(x1);
              }
              const int q = 2 * ((e >> 1) & 3);
              fadd2(ls[q], ls[q + 1], ls[q], ls[q + 1], p0, p1);
              pk[e >> 1] = pack_bf16x2(p0, p1);
            }
            tmem_st16(t_s + 16 * c, pk);
          }
          const float lt = ((ls[0] + ls[1]) + (ls[2] + ls[3])) + ((ls[4] + ls[5]) + (ls[6] + ls[7]));
          l = l * alpha + lt;
          if (__any_sync(0xffffffffu, rescale && j > 0)) {
            const float a = (rescale && j > 0) ? alpha : 1.f;
#pragma unroll
            for (int c = 0; c < HD / 32; ++c) {
              uint32_t o[32];
              tmem_ld32(t_o + 32 * c, o);
              tmem_wait_ld();
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * a);
              tmem_st32(t_o + 32 * c, o);
            }
          }
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->p_full[hh]);
      }
      if constexpr (PAGED) {
        // Hand the rows' max and sum to the epilogue warps and go straight
        // on to the next tile: its first S is usually waiting already.
        // (Every softmax warp arrives, a warp without a head included.)
        bars->stats[k & 1][hh][0][r] = m_used;
        bars->stats[k & 1][hh][1][r] = l;
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->stats_full[k & 1]);
      } else {
        // Epilogue: O out of TMEM in 32-column chunks, normalised and
        // stored with lse; the accumulator is released after its last
        // chunk. A warp without a head (odd GQA group) only keeps the
        // o_empty count.
        if (!(ok = ok && mbar_wait_warp(&bars->o_full, k & 1, kDevTimeoutFull))) break;
        tc_fence_after();
        if (active) {
          const int h = w.h0 + hh;
          const float inv = (l > 0.f) ? 1.f / l : 0.f;
          uint4* d4 = reinterpret_cast<uint4*>(p.out + ((size_t)q_tok * p.Hq + h) * HD);
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + 32 * c, o);
            tmem_wait_ld();
            if (c == HD / 32 - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive(&bars->o_empty);
            }
            if (row_ok) {
#pragma unroll
              for (int q4 = 0; q4 < 4; ++q4) {
                uint4 u;
                u.x = pack_bf16x2(__uint_as_float(o[8 * q4 + 0]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv);
                u.y = pack_bf16x2(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv);
                u.z = pack_bf16x2(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv);
                u.w = pack_bf16x2(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv);
                d4[4 * c + q4] = u;
              }
            }
          }
          if (row_ok) p.lse[(size_t)h * p.L + q_tok] = (l > 0.f) ? m_used + log2f(l) : -INFINITY;
        } else {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->o_empty);
        }
      }
      J += w.n;
    }
  } else if constexpr (PAGED) {
    regs_dec<FwdRegs::epi>();
    // ------------------------------------------------------------ epilogue
    // O of both heads out of TMEM in 32-column chunks, normalised with the
    // softmax warps' row sums and stored with lse; the accumulator is
    // released after the last chunk, so the next tile's first P V may
    // overwrite it. Runs under the next tile's first softmax phase.
    const int sub = warp & 3;  // TMEM lane quarter this warp may access
    const int r = sub * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    // Its waits sleep between polls: a tile's O is ready only at the tile's
    // end, and polling all along would take issue slots and barrier-unit
    // cycles from the softmax warps on the same sub-partitions.
    auto wait = [&](uint64_t* bar, uint32_t parity) {
      return __all_sync(0xffffffffu, mbar_wait_sleepy(bar, parity, kDevTimeoutFull));
    };
    bool ok = true;
    for (int k = 0; ok; ++k) {
      ok = wait(&bars->tile_full[k & 1], (k >> 1) & 1);
      const int tile = ok ? *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) : -1;
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->tile_empty[k & 1]);
      if (!ok || tile < 0) break;
      const FwdWork w = fwd_work<PAGED>(tile, p);
      const int q_tok = w.q0 + r;
      const bool row_ok = q_tok < w.row_end;
      if (!(ok = wait(&bars->o_full, k & 1))) break;
      if (!(ok = wait(&bars->stats_full[k & 1], (k >> 1) & 1))) break;
      tc_fence_after();
      for (int hh = 0; hh < hpc; ++hh) {
        const int h = w.h0 + hh;
        const float m_used = bars->stats[k & 1][hh][0][r];
        const float l = bars->stats[k & 1][hh][1][r];
        const float inv = (l > 0.f) ? 1.f / l : 0.f;
        const uint32_t t_o = tbase + 256 + HD * hh + lane_bits;
        uint4* d4 = reinterpret_cast<uint4*>(p.out + ((size_t)q_tok * p.Hq + h) * HD);
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(t_o + 32 * c, o);
          tmem_wait_ld();
          if (row_ok) {
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              uint4 u;
              u.x = pack_bf16x2(__uint_as_float(o[8 * q4 + 0]) * inv, __uint_as_float(o[8 * q4 + 1]) * inv);
              u.y = pack_bf16x2(__uint_as_float(o[8 * q4 + 2]) * inv, __uint_as_float(o[8 * q4 + 3]) * inv);
              u.z = pack_bf16x2(__uint_as_float(o[8 * q4 + 4]) * inv, __uint_as_float(o[8 * q4 + 5]) * inv);
              u.w = pack_bf16x2(__uint_as_float(o[8 * q4 + 6]) * inv, __uint_as_float(o[8 * q4 + 7]) * inv);
              d4[4 * c + q4] = u;
            }
          }
        }
        if (row_ok && !PAGED) p.lse[(size_t)h * p.L + q_tok] = (l > 0.f) ? m_used + log2f(l) : -INFINITY;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->o_empty);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tbase, C::TMEM_COLS);
  }
}

// Prepare one instantiation for launch on the current device (once per
// device): its dynamic shared memory, and for the paged prefill a check that
// the kernel is launched with the registers the setmaxnreg split draws on
// (an increase beyond the launch allocation would never complete).
template <int HD, bool PAGED>
cudaError_t fwd_prepare(int smem) {
  static std::atomic<int> ready[kMaxDevices];
  const int dev = device_slot();
  if (dev >= 0 && ready[dev].load(std::memory_order_acquire)) return cudaSuccess;
  cudaFuncAttributes a{};
  cudaError_t e = cudaFuncGetAttributes(&a, varlen_fwd_kernel<HD, PAGED>);
  if (e != cudaSuccess) return e;
  if (PAGED && a.numRegs < kFwdLaunchRegs) return cudaErrorInvalidConfiguration;
  e = cudaFuncSetAttribute(varlen_fwd_kernel<HD, PAGED>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e == cudaSuccess && dev >= 0) ready[dev].store(1, std::memory_order_release);
  return e;
}

cudaError_t launch_varlen_fwd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                              const VarlenParams& p, cudaStream_t stream) {
  const int n_work = ((p.L + 127) / 128) * (p.Hq / p.heads_per_cta);
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = std::max(1, std::min(n_work, sms));  // persistent: one CTA per SM
  cudaError_t e = cudaMemsetAsync(p.tile_counter, 0, sizeof(int), stream);
  if (e != cudaSuccess) return e;
  if (p.head_dim == 128) {
    const int smem = FwdTile<128>::SMEM;
    e = fwd_prepare<128, false>(smem);
    if (e != cudaSuccess) return e;
    varlen_fwd_kernel<128, false><<<grid, fwd_threads<false>(), smem, stream>>>(qm, km, vm, p);
  } else {
    const int smem = FwdTile<64>::SMEM;
    e = fwd_prepare<64, false>(smem);
    if (e != cudaSuccess) return e;
    varlen_fwd_kernel<64, false><<<grid, fwd_threads<false>(), smem, stream>>>(qm, km, vm, p);
  }
  return cudaGetLastError();
}

// Paged prefill: persistent CTAs (one per SM) taking (row, 128-query tile,
// q-head pair) tiles from p.tile_counter when the caller gave scratch for it,
// else one CTA per tile.
cudaError_t launch_paged_prefill(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                                 const VarlenParams& p, cudaStream_t stream) {
  long long n_work = (long long)p.B * ((p.S + 127) / 128) * (p.Hq / p.heads_per_cta);
  if (n_work <= 0) return cudaSuccess;
  if (n_work >= (1ll << 31)) return cudaErrorInvalidValue;
  cudaError_t e;
  if (p.tile_counter) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    n_work = std::min<long long>(n_work, sms);
    e = cudaMemsetAsync(p.tile_counter, 0, sizeof(int), stream);
    if (e != cudaSuccess) return e;
  }
  if (p.head_dim == 128) {
    const int smem = FwdTile<128>::SMEM;
    e = fwd_prepare<128, true>(smem);
    if (e != cudaSuccess) return e;
    varlen_fwd_kernel<128, true><<<(unsigned)n_work, fwd_threads<true>(), smem, stream>>>(qm, km, vm, p);
  } else {
    const int smem = FwdTile<64>::SMEM;
    e = fwd_prepare<64, true>(smem);
    if (e != cudaSuccess) return e;
    varlen_fwd_kernel<64, true><<<(unsigned)n_work, fwd_threads<true>(), smem, stream>>>(qm, km, vm, p);
  }
  return cudaGetLastError();
}

}  // namespace mb
