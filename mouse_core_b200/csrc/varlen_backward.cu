// K6: packed varlen segment-causal GQA attention backward on tcgen05.
//
// Gradient of K5 (the attention of flex_train.py:147 under the mask of
// flex_train.py:98-102); the reference gets it from autograd through compiled
// flex_attention. With z = scale * q k^T masked to run_start[i] <= j <= i,
// P = softmax(z) = 2^(z log2 e - lse2), D_i = sum_d dO[i,d] O[i,d]:
//   dV = P^T dO,  dS = P o (dO V^T - D),  dQ = scale dS K,  dK = scale dS^T Q,
// with dK/dV summed over the q-heads sharing a kv-head.
//
// Three kernels, deterministic (every output element is computed by one CTA;
// the only atomics are the persistent kernels' tile counters):
//  * delta:  D[h, i] (fp32) from dO and O.
//  * dkdv:   per (128-key tile, kv-head) tile (persistent, like dq), walking every (q-head of the
//            group, 128-query tile) item whose queries may see its keys. Keys
//            sit on the TMEM lanes: S^T = K Q^T and dP^T = V dO^T land in two
//            128-column regions; the element-wise warps write P^T (bf16) over
//            the S^T columns they read and dS^T over the dP^T columns, and
//            dV += P^T dO, dK += dS^T Q accumulate in TMEM over the walk. The
//            MMA order per item is dV(t) (by halves: queries 0-63 as soon as
//            the P warps have written them, 64-127 after), S^T(t+1), dK(t),
//            dP^T(t+1). Separate P warps and dS warps run the two
//            element-wise phases, so one item's dS phase runs beside the
//            next item's P phase; the dS warps read P^T back from TMEM
//            before S^T(t+1) may overwrite it.
//  * dq:     per (128-query tile, q-head) tile, walking the key tiles the
//            forward visits: S = Q K^T (double-buffered in TMEM), dP = dO V^T,
//            dS (bf16, over the S columns it came from), dQ += dS K. The
//            kernel is persistent (one CTA per SM, tiles from a counter) so a
//            tile's epilogue overlaps the next tile's loads and first MMAs.
//  * stored-dS path (when the caller gives a dS scratch): the dkdv kernel
//            also writes every bf16 dS^T block to global memory (coalesced:
//            query chunks of 8, 128 key rows x 16 bytes each), and dq_stored
//            computes dQ = scale dS K as one GEMM per query tile over those
//            blocks. 5 GEMM-equivalents per tile pair instead of 7, for
//            32 KB written and read back per pair and q-head.
//
// Pipelining (one item stream per CTA, every MMA 128 x 128 or 128 x HD wide):
//  * The element-wise warps signal once per phase (one mbarrier arrive per
//    warp); in dq they also signal once dP is in registers so the next item's
//    dP MMA can start.
//  * The MMA warp runs its loop with all 32 lanes and issues through
//    elect.sync, and it waits on a barrier only after queuing a full group of
//    8 MMAs: each wait costs the issuing warp a few hundred cycles, which the
//    queued MMAs cover.
//  * The operand needed first (Q in dkdv, K in dq) has a 3-slot TMA ring, the
//    other (dO, V) a 2-slot ring, so loads run an item or more ahead.
//  * tcgen05.mma operations of one CTA execute in issue order, so an MMA may
//    overwrite TMEM columns that an earlier MMA reads as its A operand.
// Warp roles (576 threads): warp 0 TMA producer, warp 1 TMEM allocator and
// MMA issuer, warps 2-17 element-wise; warp w owns TMEM lanes 32*(w%4). In dq
// warp w takes column quarter (w-2)/4 of each 128-column tile (four warps
// per lane quarter hide the TMEM and MUFU latencies); in dkdv warps 2-9 are
// P warps and 10-17 dS warps, each taking a 64-column half.
#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mb {

template <int HD>
struct BwdTile {
  static constexpr int NCB = HD / 64;
  static constexpr int BOX = 128 * 128;   // one 64-element x 128-row box
  static constexpr int TILE = NCB * BOX;  // one 128-row x HD tile
};

// ---------------------------------------------------------------- delta
// D[h, i] = sum_d dO[i, h, d] O[i, h, d]: HBM-bound (2 * hd * 2 bytes read per
// row). hd / 8 threads share a row, each loading 16 bytes of both tensors, and
// each thread keeps two rows in flight.
__device__ __forceinline__ float dot8_bf16(uint4 a, uint4 b) {
  const uint32_t* x = reinterpret_cast<const uint32_t*>(&a);
  const uint32_t* y = reinterpret_cast<const uint32_t*>(&b);
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 u = unpack_bf16x2(x[i]), v = unpack_bf16x2(y[i]);
    acc = fmaf(u.x, v.x, fmaf(u.y, v.y, acc));
  }
  return acc;
}

__global__ void __launch_bounds__(256) bwd_delta_kernel(const __nv_bfloat16* __restrict__ out,
                                                        const __nv_bfloat16* __restrict__ dout, int L, int Hq,
                                                        int hd, float* __restrict__ delta,
                                                        int* __restrict__ tile_counter) {
  // The persistent kernels launched after this one on the same stream take
  // their tiles from these counters.
  if (blockIdx.x == 0 && threadIdx.x < 2) tile_counter[threadIdx.x] = 0;
  const int tpr = hd >> 3;  // threads per row (16 or 8), a power of two dividing 32
  const long long rows = (long long)L * Hq;
  const long long tid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long stride = ((long long)gridDim.x * blockDim.x) / tpr;
  const int part = (int)(tid % tpr);
  // The row groups of one warp advance together (the stride is a multiple of
  // the groups per warp), so the loop test on the warp's first row keeps the
  // shuffles below convergent; rows past the end are masked per group.
  // Four rows per thread per pass: eight 16-byte loads in flight.
  constexpr int R = 4;
  const long long gw = (tid & 31) / tpr;
  for (long long r0 = tid / tpr; r0 - gw < rows; r0 += R * stride) {
    uint4 a[R], b[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const long long r = r0 + i * stride;
      a[i] = b[i] = make_uint4(0, 0, 0, 0);
      if (r < rows) {
        a[i] = __ldg(reinterpret_cast<const uint4*>(out + r * hd) + part);
        b[i] = __ldg(reinterpret_cast<const uint4*>(dout + r * hd) + part);
      }
    }
    float s[R];
#pragma unroll
    for (int i = 0; i < R; ++i) s[i] = dot8_bf16(a[i], b[i]);
    for (int o = tpr >> 1; o > 0; o >>= 1)
#pragma unroll
      for (int i = 0; i < R; ++i) s[i] += __shfl_xor_sync(0xffffffffu, s[i], o);
    if (part == 0) {
#pragma unroll
      for (int i = 0; i < R; ++i) {
        const long long r = r0 + i * stride;
        if (r < rows) delta[(r % Hq) * (long long)L + r / Hq] = s[i];
      }
    }
  }
}

// ---------------------------------------------------------------- shared pieces
// D = A B^T over HD; A and B K-major in smem (128 rows x HD); issued by the
// whole MMA warp as one straight-line group.
template <int HD>
__device__ __forceinline__ void mma_kmajor_ss(uint32_t d, uint32_t a_base, uint32_t b_base, uint32_t idesc) {
  const uint64_t da = umma_desc_sw128(a_base, 16, 1024), db = umma_desc_sw128(b_base, 16, 1024);
  if constexpr (HD == 128)
    umma_ss_k128_warp(d, da, db, idesc);
  else
    umma_ss_k64_warp(d, da, db, idesc);
}

// D (+)= A_tmem[128 x 128 tokens (bf16)] * B[128 tokens x HD], B MN-major in
// smem; whole MMA warp. A is written by the element-wise warps: column quarter
// q packs its 32 tokens into columns [32q, 32q + 16) of the 128-column region
// it read them from.
template <int HD>
__device__ __forceinline__ void mma_tmem_a(uint32_t d, uint32_t a_tmem, uint32_t b_base, uint32_t idesc,
                                           bool accumulate) {
  umma_ts_t128_quarters_warp(d, a_tmem, umma_desc_sw128(b_base, BwdTile<HD>::BOX, 1024), idesc,
                             accumulate ? 1u : 0u);
}

// One half (K rows 64 * half .. + 63) of mma_tmem_a.
template <int HD>
__device__ __forceinline__ void mma_tmem_a_half(uint32_t d, uint32_t a_tmem, uint32_t b_base, uint32_t idesc,
                                                bool accumulate, int half) {
  umma_ts_t64_quarters_warp(d, a_tmem + 64 * half,
                            umma_desc_sw128(b_base, BwdTile<HD>::BOX, 1024) + 512 * (uint64_t)half, idesc,
                            (accumulate || half) ? 1u : 0u);
}

constexpr int kBwdThreads = 576;  // producer + MMA warp + 16 element-wise warps
constexpr int kEwWarps = 16;
// The dK/dV kernel splits its element-wise warps by phase: warps 2-9 turn
// S^T into P^T, warps 10-17 turn dP^T into dS^T, so one item's dS phase runs
// beside the next item's P phase instead of after it.
constexpr int kPWarps = 8, kDsWarps = 8;
// Of each warp's 32 exponentials per item, this many run on the FMA pipe
// (exp2_fma) instead of the SFU, whose throughput bounds the P phase.
constexpr int kFmaExp = 4;

// ---------------------------------------------------------------- dq kernel
// Persistent: one CTA per SM takes (query tile, q-head) tiles from a global
// counter, heaviest query tiles first. The producer hands each tile id to
// the MMA and element-wise warps through a two-slot ring; barrier phases and
// ring slots follow a running item count across tiles, so the next tile's
// Q / dO loads and first S / dP MMAs overlap the previous tile's epilogue.
struct DqBars {
  uint64_t tile_full[2], tile_empty[2];  // tile-id ring (producer -> MMA + element-wise warps)
  uint64_t fixed_full, fixed_empty;      // Q, dO of the current tile; free again
  uint64_t k_full[3], k_empty[3], v_full[2], v_empty[2];
  uint64_t s_full[2];   // S(j) in TMEM region j & 1
  uint64_t dp_full;     // dP(j)
  uint64_t dp_loaded;   // element-wise warps hold dP(j) in registers
  uint64_t ds_done[2];  // bf16 dS of item j in TMEM (set j & 1)
  uint64_t acc_full;    // dQ of the tile complete in TMEM
  uint64_t acc_empty;   // the element-wise warps have read it out
  uint64_t mma_drain;   // every MMA of the CTA complete, before TMEM is freed
  uint32_t tmem_base;
  int tile[2];
};

struct DqTile {
  int q0, h, kvh, t_lo, n;
};

__device__ __forceinline__ DqTile dq_tile(int tile, const VarlenBwdParams& p) {
  const int n_qt = (p.L + 127) / 128;
  DqTile d;
  const int qt = n_qt - 1 - tile / p.Hq;
  d.h = tile % p.Hq;
  d.kvh = d.h / p.G;
  d.q0 = qt * 128;
  d.t_lo = p.run_start[d.q0] / 128;
  d.n = min(d.q0 + 127, p.L - 1) / 128 - d.t_lo + 1;
  return d;
}

template <int HD>
__global__ void __launch_bounds__(kBwdThreads, 1) varlen_bwd_dq_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              const __grid_constant__ CUtensorMap dom,
                                                              const VarlenBwdParams p) {
  using C = BwdTile<HD>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (!smem_base_aligned(smem)) {
    if (threadIdx.x == 0) report(kDevBadSmem);
    return;
  }
  uint8_t* qs = smem;
  uint8_t* dos = smem + C::TILE;
  uint8_t* kring = smem + 2 * C::TILE;  // [3][TILE]
  uint8_t* vring = smem + 5 * C::TILE;  // [2][TILE]
  DqBars* bars = reinterpret_cast<DqBars*>(smem + 7 * C::TILE);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = ((p.L + 127) / 128) * p.Hq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->tile_full[s], 1);
      mbar_init(&bars->tile_empty[s], 1 + kEwWarps);
    }
    mbar_init(&bars->fixed_full, 1);
    mbar_init(&bars->fixed_empty, 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->ds_done[s], kEwWarps);
    }
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->dp_loaded, kEwWarps);
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, kEwWarps);
    mbar_init(&bars->mma_drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t t_p = tbase + 256, t_dq = tbase + 384;

  // Tile k of this CTA from the ring (every consumer warp reads each slot once).
  auto take_tile = [&](int k, bool& ok) {
    ok = mbar_wait_warp(&bars->tile_full[k & 1], (k >> 1) & 1, kDevTimeoutFull);
    const int tile = ok ? *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) : -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->tile_empty[k & 1]);
    return tile;
  };

  if (warp == 0) {
    bool ok = true;
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      prefetch_tensormap(&dom);
    }
    int J = 0;  // items of earlier tiles: ring slots and phases continue across tiles
    int n_fixed = 0, n_k = 0, n_v = 0;  // loads issued into each ring (lane 0)
    for (int k = 0; ok; ++k) {
      int tile = -1;
      if (lane == 0) {
        tile = k == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(p.tile_counter, 1);
        if (tile >= n_tiles) tile = -1;
        ok = mbar_wait(&bars->tile_empty[k & 1], ((k >> 1) & 1) ^ 1, kDevTimeoutEmpty);
        if (ok) {
          *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) = tile;
          mbar_arrive(&bars->tile_full[k & 1]);
        }
      }
      tile = __shfl_sync(0xffffffffu, tile, 0);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || tile < 0) break;
      const DqTile d = dq_tile(tile, p);
      if (lane == 0) {
        // Q / dO slots are free once the previous tile's MMAs have completed.
        if (k > 0) ok = mbar_wait(&bars->fixed_empty, (k - 1) & 1, kDevTimeoutEmpty);
        if (ok) {
          mbar_arrive_expect_tx(&bars->fixed_full, 2 * C::TILE);
          for (int cb = 0; cb < C::NCB; ++cb) {
            tma_load_3d(qs + cb * C::BOX, &qmap, &bars->fixed_full, cb * 64, d.h, d.q0);
            tma_load_3d(dos + cb * C::BOX, &dom, &bars->fixed_full, cb * 64, d.h, d.q0);
          }
          ++n_fixed;
        }
        for (int j = 0; ok && j < d.n; ++j) {
          const int jj = J + j;
          const int ks = jj % 3, vsl = jj & 1;
          const int kv0 = (d.t_lo + j) * 128;
          if (!(ok = mbar_wait(&bars->k_empty[ks], ((jj / 3) & 1) ^ 1, kDevTimeoutEmpty))) break;
          mbar_arrive_expect_tx(&bars->k_full[ks], C::TILE);
          for (int cb = 0; cb < C::NCB; ++cb)
            tma_load_3d(kring + ks * C::TILE + cb * C::BOX, &kmap, &bars->k_full[ks], cb * 64, d.kvh, kv0);
          ++n_k;
          if (!(ok = mbar_wait(&bars->v_empty[vsl], ((jj >> 1) & 1) ^ 1, kDevTimeoutEmpty))) break;
          mbar_arrive_expect_tx(&bars->v_full[vsl], C::TILE);
          for (int cb = 0; cb < C::NCB; ++cb)
            tma_load_3d(vring + vsl * C::TILE + cb * C::BOX, &vmap, &bars->v_full[vsl], cb * 64, d.kvh, kv0);
          ++n_v;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      J += d.n;
    }
    // Every load issued lands before the CTA exits, also when a wait ran out.
    if (lane == 0) {
      drain_ring(&bars->fixed_full, 1, n_fixed);
      drain_ring(bars->k_full, 3, n_k);
      drain_ring(bars->v_full, 2, n_v);
    }
  } else if (warp == 1) {
    constexpr uint32_t ID_S = umma_idesc_bf16(128, 128, 0, 0);
    constexpr uint32_t ID_DQ = umma_idesc_bf16(128, HD, 0, 1);
    const uint32_t qa = smem_u32(qs), da = smem_u32(dos);
    auto issue_s = [&](int jj) {  // S = Q K^T of running item jj into region jj & 1
      const int ks = jj % 3;
      if (!mbar_wait_warp(&bars->k_full[ks], (jj / 3) & 1, kDevTimeoutFull)) return false;
      mma_kmajor_ss<HD>(tbase + 128 * (jj & 1), qa, smem_u32(kring + ks * C::TILE), ID_S);
      umma_commit_warp(&bars->s_full[jj & 1]);
      return true;
    };
    auto issue_dp = [&](int jj) {  // dP = dO V^T; V's slot is free once it completes
      const int vsl = jj & 1;
      if (!mbar_wait_warp(&bars->v_full[vsl], (jj >> 1) & 1, kDevTimeoutFull)) return false;
      mma_kmajor_ss<HD>(t_p, da, smem_u32(vring + vsl * C::TILE), ID_S);
      umma_commit_warp(&bars->dp_full);
      umma_commit_warp(&bars->v_empty[vsl]);
      return true;
    };
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const int n = dq_tile(tile, p).n;
      if (!(ok = mbar_wait_warp(&bars->fixed_full, k & 1, kDevTimeoutFull))) break;
      if (!(ok = issue_s(J))) break;
      if (n > 1 && !(ok = issue_s(J + 1))) break;
      if (!(ok = issue_dp(J))) break;
      for (int j = 0; ok && j < n; ++j) {
        const int jj = J + j;
        if (!(ok = mbar_wait_warp(&bars->dp_loaded, jj & 1, kDevTimeoutFull))) break;
        if (j + 1 < n && !(ok = issue_dp(jj + 1))) break;
        if (!(ok = mbar_wait_warp(&bars->ds_done[jj & 1], (jj >> 1) & 1, kDevTimeoutFull))) break;
        // The first dQ MMA of a tile overwrites the accumulator: the previous
        // tile's epilogue must have read it out.
        if (j == 0 && k > 0 && !(ok = mbar_wait_warp(&bars->acc_empty, (k - 1) & 1, kDevTimeoutFull))) break;
        // dQ += dS K over the 128 keys of item jj.
        mma_tmem_a<HD>(t_dq, tbase + 128 * (jj & 1), smem_u32(kring + (jj % 3) * C::TILE), ID_DQ, j > 0);
        umma_commit_warp(&bars->k_empty[jj % 3]);
        if (j + 2 < n) ok = issue_s(jj + 2);
      }
      if (!ok) break;
      umma_commit_warp(&bars->acc_full);
      umma_commit_warp(&bars->fixed_empty);
      J += n;
    }
    umma_drain_warp(&bars->mma_drain);  // before TMEM is freed, also when a wait ran out
  } else {
    const int cq = (warp - 2) >> 2;  // column quarter of every 128-column tile
    const int sub = warp & 3;         // TMEM lane quarter
    const int r = sub * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const DqTile d = dq_tile(tile, p);
      const int q_tok = d.q0 + r;
      const bool row_ok = q_tok < p.L;
      const int lo = row_ok ? p.run_start[q_tok] : 0x7fffffff;
      const float neg_lse = row_ok ? -p.lse[(size_t)d.h * p.L + q_tok] : 0.f;
      const float dlt = row_ok ? p.delta[(size_t)d.h * p.L + q_tok] : 0.f;
      for (int j = 0; j < d.n; ++j) {
        const int jj = J + j;
        const int kc0 = (d.t_lo + j) * 128 + 32 * cq;  // first key of this warp's 32 columns
        const uint32_t ts = tbase + 128 * (jj & 1) + lane_bits + 32 * cq;
        uint32_t pk[16];  // P as bf16 pairs, the precision dS is formed from in both kernels
        if (ok) ok = mbar_wait_warp(&bars->s_full[jj & 1], (jj >> 1) & 1, kDevTimeoutFull);
        tc_fence_after();
        if (ok) {
          uint32_t sv[32];
          tmem_ld32(ts, sv);
          tmem_wait_ld();
          float pf[32];
#pragma unroll
          for (int c = 0; c < 32; ++c) {
            const float xc = fmaf(__uint_as_float(sv[c]), p.scale_log2, neg_lse);
            pf[c] = c < 32 - kFmaExp ? fast_exp2(xc) : exp2_fma(xc);
          }
          if (!(row_ok && kc0 >= lo && kc0 + 31 <= q_tok)) {
#pragma unroll
            for (int c = 0; c < 32; ++c)
              if (!row_ok || kc0 + c < lo || kc0 + c > q_tok) pf[c] = 0.f;
          }
#pragma unroll
          for (int e = 0; e < 16; ++e) pk[e] = pack_bf16x2(pf[2 * e], pf[2 * e + 1]);
        }
        if (ok) ok = mbar_wait_warp(&bars->dp_full, jj & 1, kDevTimeoutFull);
        tc_fence_after();
        uint32_t dv[32];
        if (ok) {
          tmem_ld32(t_p + lane_bits + 32 * cq, dv);
          tmem_wait_ld();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->dp_loaded);
        if (ok) {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            const float2 pp = unpack_bf16x2(pk[e]);
            pk[e] = pack_bf16x2(pp.x * (__uint_as_float(dv[2 * e]) - dlt), pp.y * (__uint_as_float(dv[2 * e + 1]) - dlt));
          }
          tmem_st16(ts, pk);  // dS over S columns this warp already read
          tmem_wait_st();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&bars->ds_done[jj & 1]);
      }
      if (!ok) break;
      // Epilogue: column quarter cq writes dQ columns [cq HD/4, (cq + 1) HD/4),
      // 16 at a time; the accumulator is released as soon as it is in registers.
      constexpr int W = HD / 4;  // 32 or 16 columns
      const int col = cq * W;
      uint32_t v[W / 16][16];
      if (!(ok = mbar_wait_warp(&bars->acc_full, k & 1, kDevTimeoutFull))) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < W / 16; ++c) tmem_ld16(t_dq + lane_bits + col + 16 * c, v[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty);
      if (row_ok) {
        uint4* d4 = reinterpret_cast<uint4*>(p.dq + ((size_t)q_tok * p.Hq + d.h) * HD + col);
#pragma unroll
        for (int c = 0; c < W / 16; ++c)
#pragma unroll
          for (int q4 = 0; q4 < 2; ++q4) {
            const uint32_t* u = v[c] + 8 * q4;
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(u[0]) * p.scale, __uint_as_float(u[1]) * p.scale);
            w.y = pack_bf16x2(__uint_as_float(u[2]) * p.scale, __uint_as_float(u[3]) * p.scale);
            w.z = pack_bf16x2(__uint_as_float(u[4]) * p.scale, __uint_as_float(u[5]) * p.scale);
            w.w = pack_bf16x2(__uint_as_float(u[6]) * p.scale, __uint_as_float(u[7]) * p.scale);
            d4[2 * c + q4] = w;
          }
      }
      J += d.n;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------- dkdv kernel
// Persistent like the dq kernel: one CTA per SM takes (key tile, kv-head)
// tiles from the second counter; K and V are released after a tile's last
// S^T / dP^T MMAs, so the next tile's K / V load during its last item and
// epilogue, and dV / dK are released once the epilogue has read them.
struct DkdvBars {
  uint64_t tile_full[2], tile_empty[2];  // tile-id ring (producer -> MMA + element-wise warps)
  uint64_t fixed_full, fixed_empty;      // K, V of the current tile; free again
  uint64_t q_full[3], q_empty[3], d_full[2], d_empty[2];
  uint64_t s_full, dp_full;  // S^T(t), dP^T(t)
  uint64_t p_half;           // bf16 P^T of query quarters 0-1 in TMEM
  uint64_t p_done;           // bf16 P^T of the current item in TMEM
  uint64_t p_read;           // the dS warps hold that P^T in registers
  uint64_t ds_done;          // bf16 dS^T of the current item in TMEM
  uint64_t acc_full;         // dV, dK of the tile complete in TMEM
  uint64_t acc_empty;        // the element-wise warps have read them out
  uint64_t mma_drain;        // every MMA of the CTA complete, before TMEM is freed
  uint32_t tmem_base;
  int tile[2];
};

struct DkdvTile {
  int kv0, kvh, i_lo, nqi, n;
};

__device__ __forceinline__ DkdvTile dkdv_tile(int tile, const VarlenBwdParams& p) {
  DkdvTile d;
  const int kt = tile / p.Hkv;
  d.kvh = tile % p.Hkv;
  d.kv0 = kt * 128;
  const int last = min(d.kv0 + 127, p.L - 1);
  d.i_lo = kt;
  d.nqi = (p.run_end[last] - 1) / 128 - d.i_lo + 1;
  d.n = p.G * d.nqi;  // (q-head, query tile) items
  return d;
}

template <int HD>
__global__ void __launch_bounds__(kBwdThreads, 1) varlen_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                const __grid_constant__ CUtensorMap kmap,
                                                                const __grid_constant__ CUtensorMap vmap,
                                                                const __grid_constant__ CUtensorMap dom,
                                                                const VarlenBwdParams p) {
  using C = BwdTile<HD>;
  extern __shared__ __align__(1024) uint8_t smem[];
  if (!smem_base_aligned(smem)) {
    if (threadIdx.x == 0) report(kDevBadSmem);
    return;
  }
  uint8_t* ks = smem;
  uint8_t* vs = smem + C::TILE;
  uint8_t* qring = smem + 2 * C::TILE;  // [3][TILE]
  uint8_t* dring = smem + 5 * C::TILE;  // [2][TILE]
  float* lse_ring = reinterpret_cast<float*>(smem + 7 * C::TILE);  // [3][128], with the Q slot
  float* dlt_ring = lse_ring + 3 * 128;                             // [2][128], with the dO slot
  DkdvBars* bars = reinterpret_cast<DkdvBars*>(dlt_ring + 2 * 128);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = ((p.L + 127) / 128) * p.Hkv;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->tile_full[s], 1);
      mbar_init(&bars->tile_empty[s], 1 + kPWarps + kDsWarps);
    }
    mbar_init(&bars->fixed_full, 1);
    mbar_init(&bars->fixed_empty, 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&bars->q_full[s], 2);  // TMA bytes + the lse staging arrive
      mbar_init(&bars->q_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->d_full[s], 2);  // TMA bytes + the delta staging arrive
      mbar_init(&bars->d_empty[s], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->dp_full, 1);
    mbar_init(&bars->p_half, kPWarps);
    mbar_init(&bars->p_done, kPWarps);
    mbar_init(&bars->p_read, kDsWarps);
    mbar_init(&bars->ds_done, kDsWarps);
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->acc_empty, kPWarps + kDsWarps);
    mbar_init(&bars->mma_drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t t_s = tbase, t_x = tbase + 128, t_dv = tbase + 256, t_dk = tbase + 256 + HD;

  // Tile k of this CTA from the ring (each consumer warp reads every slot once).
  auto take_tile = [&](int k, bool& ok) {
    ok = mbar_wait_warp(&bars->tile_full[k & 1], (k >> 1) & 1, kDevTimeoutFull);
    const int tile = ok ? *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) : -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->tile_empty[k & 1]);
    return tile;
  };

  if (warp == 0) {
    // Producer warp: lane 0 issues TMA; all lanes stage lse / delta.
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      prefetch_tensormap(&dom);
    }
    bool ok = true;
    int J = 0;  // items of earlier tiles: ring slots and phases continue across tiles
    int n_fixed = 0, n_q = 0, n_d = 0;  // loads issued into each ring (lane 0)
    for (int k = 0; ok; ++k) {
      int tile = -1;
      if (lane == 0) {
        tile = k == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(p.tile_counter + 1, 1);
        if (tile >= n_tiles) tile = -1;
        ok = mbar_wait(&bars->tile_empty[k & 1], ((k >> 1) & 1) ^ 1, kDevTimeoutEmpty);
        if (ok) {
          *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) = tile;
          mbar_arrive(&bars->tile_full[k & 1]);
        }
      }
      tile = __shfl_sync(0xffffffffu, tile, 0);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || tile < 0) break;
      const DkdvTile d = dkdv_tile(tile, p);
      if (lane == 0) {
        // K / V slots are free once the previous tile's last S^T and dP^T completed.
        if (k > 0) ok = mbar_wait(&bars->fixed_empty, (k - 1) & 1, kDevTimeoutEmpty);
        if (ok) {
          mbar_arrive_expect_tx(&bars->fixed_full, 2 * C::TILE);
          for (int cb = 0; cb < C::NCB; ++cb) {
            tma_load_3d(ks + cb * C::BOX, &kmap, &bars->fixed_full, cb * 64, d.kvh, d.kv0);
            tma_load_3d(vs + cb * C::BOX, &vmap, &bars->fixed_full, cb * 64, d.kvh, d.kv0);
          }
          ++n_fixed;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      // lse / delta of the next item are loaded into registers one item ahead,
      // so their global-memory latency never delays a TMA issue.
      float lpre[4], dpre[4];
      auto prefetch = [&](int t) {
        const int hq = d.kvh * p.G + t / d.nqi;
        const int q0 = (d.i_lo + t % d.nqi) * 128;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int q = q0 + lane + 32 * i;
          lpre[i] = (q < p.L) ? p.lse[(size_t)hq * p.L + q] : INFINITY;
          dpre[i] = (q < p.L) ? p.delta[(size_t)hq * p.L + q] : 0.f;
        }
      };
      prefetch(0);
      for (int t = 0; ok && t < d.n; ++t) {
        const int tt = J + t;
        const int qs = tt % 3, dsl = tt & 1;
        const int hq = d.kvh * p.G + t / d.nqi;
        const int q0 = (d.i_lo + t % d.nqi) * 128;
        if (lane == 0) ok = mbar_wait(&bars->q_empty[qs], ((tt / 3) & 1) ^ 1, kDevTimeoutEmpty);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&bars->q_full[qs], C::TILE);
          for (int cb = 0; cb < C::NCB; ++cb)
            tma_load_3d(qring + qs * C::TILE + cb * C::BOX, &qmap, &bars->q_full[qs], cb * 64, hq, q0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) lse_ring[qs * 128 + lane + 32 * i] = lpre[i];
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars->q_full[qs]);
          ++n_q;
        }
        if (lane == 0) ok = mbar_wait(&bars->d_empty[dsl], ((tt >> 1) & 1) ^ 1, kDevTimeoutEmpty);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) break;
        if (lane == 0) {
          mbar_arrive_expect_tx(&bars->d_full[dsl], C::TILE);
          for (int cb = 0; cb < C::NCB; ++cb)
            tma_load_3d(dring + dsl * C::TILE + cb * C::BOX, &dom, &bars->d_full[dsl], cb * 64, hq, q0);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) dlt_ring[dsl * 128 + lane + 32 * i] = dpre[i];
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&bars->d_full[dsl]);
          ++n_d;
        }
        if (t + 1 < d.n) prefetch(t + 1);
      }
      J += d.n;
    }
    // Every load issued lands before the CTA exits, also when a wait ran out
    // (a Q or dO slot's phase also takes its staging arrive, made just above).
    if (lane == 0) {
      drain_ring(&bars->fixed_full, 1, n_fixed);
      drain_ring(bars->q_full, 3, n_q);
      drain_ring(bars->d_full, 2, n_d);
    }
  } else if (warp == 1) {
    constexpr uint32_t ID_S = umma_idesc_bf16(128, 128, 0, 0);
    constexpr uint32_t ID_G = umma_idesc_bf16(128, HD, 0, 1);
    const uint32_t ka = smem_u32(ks), va = smem_u32(vs);
    auto issue_s = [&](int tt) {  // S^T = K Q^T of running item tt
      const int qs = tt % 3;
      if (!mbar_wait_warp(&bars->q_full[qs], (tt / 3) & 1, kDevTimeoutFull)) return false;
      mma_kmajor_ss<HD>(t_s, ka, smem_u32(qring + qs * C::TILE), ID_S);
      umma_commit_warp(&bars->s_full);
      return true;
    };
    auto issue_dp = [&](int tt) {  // dP^T = V dO^T of running item tt
      const int dsl = tt & 1;
      if (!mbar_wait_warp(&bars->d_full[dsl], (tt >> 1) & 1, kDevTimeoutFull)) return false;
      mma_kmajor_ss<HD>(t_x, va, smem_u32(dring + dsl * C::TILE), ID_S);
      umma_commit_warp(&bars->dp_full);
      return true;
    };
    // One item: dV(t) once P^T is in TMEM, then S^T(t+1) over the P^T columns
    // dV has read, dK(t) once dS^T is in TMEM, then dP^T(t+1) over the dS^T
    // columns dK has read.
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const int n = dkdv_tile(tile, p).n;
      if (!(ok = mbar_wait_warp(&bars->fixed_full, k & 1, kDevTimeoutFull))) break;
      if (!(ok = issue_s(J))) break;
      if (!(ok = issue_dp(J))) break;
      if (n == 1) umma_commit_warp(&bars->fixed_empty);  // K and V have no further reader
      for (int t = 0; ok && t < n; ++t) {
        const int tt = J + t;
        // dV += P^T dO, by halves as the P warps finish query quarters 0-1 and 2-3
        if (!(ok = mbar_wait_warp(&bars->p_half, tt & 1, kDevTimeoutFull))) break;
        // The tile's first dV / dK overwrite the accumulators: the previous
        // tile's epilogue must have read them.
        if (t == 0 && k > 0 && !(ok = mbar_wait_warp(&bars->acc_empty, (k - 1) & 1, kDevTimeoutFull))) break;
        mma_tmem_a_half<HD>(t_dv, t_s, smem_u32(dring + (tt & 1) * C::TILE), ID_G, t > 0, 0);
        if (!(ok = mbar_wait_warp(&bars->p_done, tt & 1, kDevTimeoutFull))) break;
        mma_tmem_a_half<HD>(t_dv, t_s, smem_u32(dring + (tt & 1) * C::TILE), ID_G, t > 0, 1);
        // S^T(t+1) overwrites P^T(t): the dS warps must hold it first.
        if (!(ok = mbar_wait_warp(&bars->p_read, tt & 1, kDevTimeoutFull))) break;
        if (t + 1 < n && !(ok = issue_s(tt + 1))) break;
        if (!(ok = mbar_wait_warp(&bars->ds_done, tt & 1, kDevTimeoutFull))) break;
        mma_tmem_a<HD>(t_dk, t_x, smem_u32(qring + (tt % 3) * C::TILE), ID_G, t > 0);  // dK += dS^T Q
        // Both slots (and their staged lse / delta, read until the dS^T phase
        // ends) are free once dK(t) completes.
        umma_commit_warp(&bars->q_empty[tt % 3]);
        umma_commit_warp(&bars->d_empty[tt & 1]);
        if (t + 1 < n) {
          if (!(ok = issue_dp(tt + 1))) break;
          if (t + 2 == n) umma_commit_warp(&bars->fixed_empty);  // the tile's last S^T and dP^T are queued
        }
      }
      if (!ok) break;
      umma_commit_warp(&bars->acc_full);
      J += n;
    }
    umma_drain_warp(&bars->mma_drain);  // before TMEM is freed, also when a wait ran out
  } else {
    const bool p_warp = warp < 2 + kPWarps;
    const int ch = (warp - (p_warp ? 2 : 2 + kPWarps)) >> 2;  // column half of every 128-column tile
    const int sub = warp & 3;                                   // TMEM lane quarter
    const int r = sub * 32 + lane;
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const DkdvTile d = dkdv_tile(tile, p);
      const int k_tok = d.kv0 + r;
      const bool k_ok = k_tok < p.L;
      const int q_end = k_ok ? p.run_end[k_tok] : 0;  // queries k_tok <= q < q_end see this key
      if (p_warp) {
        // P phase, per item: S^T -> P^T for query quarters ch and ch + 2, each
        // packed to bf16 over the first 16 of its columns; quarters 0-1 are
        // signalled first so the dV MMAs on them start while 2-3 are computed.
        for (int t = 0; t < d.n; ++t) {
          const int tt = J + t;
          if (ok) ok = mbar_wait_warp(&bars->q_full[tt % 3], (tt / 3) & 1, kDevTimeoutFull);
          if (ok) ok = mbar_wait_warp(&bars->s_full, tt & 1, kDevTimeoutFull);
          tc_fence_after();
          if (ok) {
#pragma unroll 1
            for (int h = 0; h < 2; ++h) {
              const int cq = ch + 2 * h;
              const uint32_t ts = t_s + lane_bits + 32 * cq;
              const int qc0 = (d.i_lo + t % d.nqi) * 128 + 32 * cq;  // first query of these 32 columns
              uint32_t sv[32];
              tmem_ld32(ts, sv);
              tmem_wait_ld();
              const float4* l4 = reinterpret_cast<const float4*>(lse_ring + (tt % 3) * 128 + 32 * cq);
              float x[32];
#pragma unroll
              for (int c4 = 0; c4 < 8; ++c4) {
                const float4 l = l4[c4];
                x[4 * c4 + 0] = fmaf(__uint_as_float(sv[4 * c4 + 0]), p.scale_log2, -l.x);
                x[4 * c4 + 1] = fmaf(__uint_as_float(sv[4 * c4 + 1]), p.scale_log2, -l.y);
                x[4 * c4 + 2] = fmaf(__uint_as_float(sv[4 * c4 + 2]), p.scale_log2, -l.z);
                x[4 * c4 + 3] = fmaf(__uint_as_float(sv[4 * c4 + 3]), p.scale_log2, -l.w);
              }
#pragma unroll
              for (int e = 0; e < 32; ++e) x[e] = e < 32 - kFmaExp ? fast_exp2(x[e]) : exp2_fma(x[e]);
              if (!(k_ok && qc0 >= k_tok && qc0 + 31 < q_end)) {
#pragma unroll
                for (int e = 0; e < 32; ++e) {
                  const int q = qc0 + e;
                  if (q < k_tok || q >= q_end) x[e] = 0.f;
                }
              }
              uint32_t pk[16];
#pragma unroll
              for (int e = 0; e < 16; ++e) pk[e] = pack_bf16x2(x[2 * e], x[2 * e + 1]);
              tmem_st16(ts, pk);
              if (h == 0) {
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&bars->p_half);
              }
            }
            tmem_wait_st();
          } else if (lane == 0) {
            mbar_arrive(&bars->p_half);  // keep the phase count when a wait gave up
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->p_done);
        }
      } else {
        // dS phase, per item: read P^T back (then S^T(t+1) may overwrite it),
        // dS^T = P^T o (dP^T - D), packed over the dP^T columns.
        for (int t = 0; t < d.n; ++t) {
          const int tt = J + t;
          // Stored-dS path: this thread's key row of the item's dS^T block, laid
          // out as 16 chunks of 8 queries, each chunk 128 key rows x 16 bytes,
          // so a warp's store of one chunk is 512 contiguous bytes.
          __nv_bfloat16* ds_row = nullptr;
          if (p.ds != nullptr) {
            const int qi = d.i_lo + t % d.nqi;
            const int lo = p.pair_off[qi], hi = p.pair_off[qi + 1];
            const int pair = lo + d.kv0 / 128 - p.tile_lo[qi] / 128;
            if (pair >= lo && pair < hi && hi <= p.n_pairs) {
              const int hq = d.kvh * p.G + t / d.nqi;
              ds_row = p.ds + ((size_t)hq * p.n_pairs + pair) * (128 * 128) + 8 * r + 64 * 128 * ch;
            } else if (lane == 0) {
              report(kDevBadPair);
            }
          }
          uint32_t pk[2][16];
          if (ok) ok = mbar_wait_warp(&bars->p_done, tt & 1, kDevTimeoutFull);
          tc_fence_after();
          if (ok) {
            tmem_ld16(t_s + lane_bits + 64 * ch, pk[0]);
            tmem_ld16(t_s + lane_bits + 64 * ch + 32, pk[1]);
            tmem_wait_ld();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->p_read);
          if (ok) ok = mbar_wait_warp(&bars->d_full[tt & 1], (tt >> 1) & 1, kDevTimeoutFull);
          if (ok) ok = mbar_wait_warp(&bars->dp_full, tt & 1, kDevTimeoutFull);
          tc_fence_after();
          if (ok) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int cq = 2 * ch + h;
              const uint32_t tx = t_x + lane_bits + 32 * cq;
              uint32_t dv[32];
              tmem_ld32(tx, dv);
              tmem_wait_ld();
              const float4* d4 = reinterpret_cast<const float4*>(dlt_ring + (tt & 1) * 128 + 32 * cq);
#pragma unroll
              for (int e4 = 0; e4 < 8; ++e4) {
                const float4 dd = d4[e4];
                const float2 p01 = unpack_bf16x2(pk[h][2 * e4]), p23 = unpack_bf16x2(pk[h][2 * e4 + 1]);
                pk[h][2 * e4] = pack_bf16x2(p01.x * (__uint_as_float(dv[4 * e4]) - dd.x),
                                            p01.y * (__uint_as_float(dv[4 * e4 + 1]) - dd.y));
                pk[h][2 * e4 + 1] = pack_bf16x2(p23.x * (__uint_as_float(dv[4 * e4 + 2]) - dd.z),
                                                p23.y * (__uint_as_float(dv[4 * e4 + 3]) - dd.w));
              }
              tmem_st16(tx, pk[h]);
              if (ds_row != nullptr) {
#pragma unroll
                for (int m = 0; m < 4; ++m)  // query chunk 8 ch + 4 h + m
                  *reinterpret_cast<uint4*>(ds_row + (4 * h + m) * (8 * 128)) =
                      make_uint4(pk[h][4 * m], pk[h][4 * m + 1], pk[h][4 * m + 2], pk[h][4 * m + 3]);
              }
            }
            tmem_wait_st();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->ds_done);
        }
      }
      // Epilogue: the P warps write dV, the dS warps dK (scaled); each warp
      // covers half of the HD columns of its 32 keys; the accumulators are
      // released after the last chunk is read.
      if (!(ok = ok && mbar_wait_warp(&bars->acc_full, k & 1, kDevTimeoutFull))) break;
      tc_fence_after();
      const bool is_v = p_warp;
      const int col0 = ch * (HD / 2);
      const uint32_t src = (is_v ? t_dv : t_dk) + lane_bits + col0;
      const float mul = is_v ? 1.f : p.scale;
      __nv_bfloat16* dst = (is_v ? p.dv : p.dk) + ((size_t)k_tok * p.Hkv + d.kvh) * HD + col0;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        uint32_t v[32];
        tmem_ld32(src + 32 * c, v);
        tmem_wait_ld();
        if (c == HD / 64 - 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->acc_empty);
        }
        if (k_ok) {
          uint4* o4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * q4 + 0]) * mul, __uint_as_float(v[8 * q4 + 1]) * mul);
            w.y = pack_bf16x2(__uint_as_float(v[8 * q4 + 2]) * mul, __uint_as_float(v[8 * q4 + 3]) * mul);
            w.z = pack_bf16x2(__uint_as_float(v[8 * q4 + 4]) * mul, __uint_as_float(v[8 * q4 + 5]) * mul);
            w.w = pack_bf16x2(__uint_as_float(v[8 * q4 + 6]) * mul, __uint_as_float(v[8 * q4 + 7]) * mul);
            o4[q4] = w;
          }
        }
      }
      J += d.n;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tbase, 512);
  }
}

// ---------------------------------------------------------------- dq kernel, stored dS
// dQ = scale * dS K as one GEMM per (query tile, q-head) tile over the dS^T
// blocks the dK/dV kernel stored: A = dS (M = queries, K = keys), whose
// stored layout (query chunks of 8, each 128 key rows x 16 bytes) is the
// non-swizzled MN-major canonical layout, so one 32 KB bulk copy per block
// lands it ready for the MMA; B = K MN-major by TMA; fp32 accumulators in
// TMEM. Two accumulators, so a tile's epilogue overlaps the next tile's MMAs.
// Persistent, heaviest query tiles first (first counter).
// Warp 0 issues TMA, warp 1 the MMAs, warps 2-9 the epilogue (warp w reads
// TMEM lane quarter w % 4 and half of the HD columns).
constexpr int kDqsStages = 3;
constexpr int kDqsEpiWarps = 8;
constexpr int kDqsThreads = 32 * (2 + kDqsEpiWarps);

struct DqsBars {
  uint64_t tile_full[2], tile_empty[2];              // tile-id ring
  uint64_t full[kDqsStages], empty[kDqsStages];      // dS block + K tile per stage
  uint64_t acc_full[2], acc_empty[2];                // the two dQ accumulators
  uint64_t mma_drain;                                // every MMA of the CTA complete, before TMEM is freed
  uint32_t tmem_base;
  int tile[2];
};

struct DqsTile {
  int q0, h, kvh, t_lo, n, pair0;
};

__device__ __forceinline__ DqsTile dqs_tile(int tile, const VarlenBwdParams& p) {
  const int n_qt = (p.L + 127) / 128;
  DqsTile d;
  const int qt = n_qt - 1 - tile / p.Hq;
  d.h = tile % p.Hq;
  d.kvh = d.h / p.G;
  d.q0 = qt * 128;
  d.t_lo = p.tile_lo[qt] / 128;
  d.n = qt - d.t_lo + 1;  // key tiles t_lo .. qt, the pairs pair_off[qt] ..
  d.pair0 = p.pair_off[qt];
  return d;
}

template <int HD>
__global__ void __launch_bounds__(kDqsThreads, 1)
    varlen_bwd_dq_stored_kernel(const __grid_constant__ CUtensorMap kmap, const VarlenBwdParams p) {
  using C = BwdTile<HD>;
  constexpr int A_BYTES = 128 * 128 * 2;    // one dS block
  constexpr int STAGE = A_BYTES + C::TILE;  // and the K tile
  extern __shared__ __align__(1024) uint8_t smem[];
  if (!smem_base_aligned(smem)) {
    if (threadIdx.x == 0) report(kDevBadSmem);
    return;
  }
  DqsBars* bars = reinterpret_cast<DqsBars*>(smem + kDqsStages * STAGE);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tiles = ((p.L + 127) / 128) * p.Hq;

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->tile_full[s], 1);
      mbar_init(&bars->tile_empty[s], 1 + kDqsEpiWarps);
      mbar_init(&bars->acc_full[s], 1);
      mbar_init(&bars->acc_empty[s], kDqsEpiWarps);
    }
    for (int s = 0; s < kDqsStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->mma_drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, 2 * HD);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  auto take_tile = [&](int k, bool& ok) {
    ok = mbar_wait_warp(&bars->tile_full[k & 1], (k >> 1) & 1, kDevTimeoutFull);
    const int tile = ok ? *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) : -1;
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->tile_empty[k & 1]);
    return tile;
  };

  if (warp == 0) {
    if (lane == 0) prefetch_tensormap(&kmap);
    bool ok = true;
    int J = 0;  // items of earlier tiles: stage slots and phases continue across tiles
    int n_full = 0;  // stages loaded (lane 0)
    for (int k = 0; ok; ++k) {
      int tile = -1;
      if (lane == 0) {
        tile = k == 0 ? (int)blockIdx.x : (int)gridDim.x + atomicAdd(p.tile_counter, 1);
        if (tile >= n_tiles) tile = -1;
        ok = mbar_wait(&bars->tile_empty[k & 1], ((k >> 1) & 1) ^ 1, kDevTimeoutEmpty);
        if (ok) {
          *reinterpret_cast<volatile int*>(&bars->tile[k & 1]) = tile;
          mbar_arrive(&bars->tile_full[k & 1]);
        }
      }
      tile = __shfl_sync(0xffffffffu, tile, 0);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok || tile < 0) break;
      const DqsTile d = dqs_tile(tile, p);
      if (lane == 0) {
        const bool pairs_ok = d.pair0 >= 0 && d.pair0 + d.n <= p.n_pairs;
        if (!pairs_ok) report(kDevBadPair);  // the blocks are then not read (dQ of the tile is garbage)
        for (int t = 0; ok && t < d.n; ++t) {
          const int it = J + t, s = it % kDqsStages;
          ok = mbar_wait(&bars->empty[s], ((it / kDqsStages) & 1) ^ 1, kDevTimeoutEmpty);
          if (!ok) break;
          uint8_t* st = smem + s * STAGE;
          mbar_arrive_expect_tx(&bars->full[s], pairs_ok ? STAGE : C::TILE);
          if (pairs_ok)
            bulk_load(st, p.ds + ((size_t)d.h * p.n_pairs + d.pair0 + t) * (128 * 128), A_BYTES, &bars->full[s]);
          for (int cb = 0; cb < C::NCB; ++cb)
            tma_load_3d(st + A_BYTES + cb * C::BOX, &kmap, &bars->full[s], cb * 64, d.kvh, (d.t_lo + t) * 128);
          ++n_full;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      J += d.n;
    }
    // Every load issued lands before the CTA exits, also when a wait ran out.
    if (lane == 0) drain_ring(bars->full, kDqsStages, n_full);
  } else if (warp == 1) {
    constexpr uint32_t ID = umma_idesc_bf16(128, HD, 1, 1);
    bool ok = true;
    int J = 0;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const int n = dqs_tile(tile, p).n;
      const uint32_t acc = tbase + (k & 1) * HD;
      // Accumulator k & 1 last held tile k - 2: its epilogue must have read it.
      if (k >= 2 && !(ok = mbar_wait_warp(&bars->acc_empty[k & 1], ((k >> 1) - 1) & 1, kDevTimeoutFull))) break;
      tc_fence_after();
      for (int t = 0; t < n; ++t) {
        const int it = J + t, s = it % kDqsStages;
        if (!(ok = mbar_wait_warp(&bars->full[s], (it / kDqsStages) & 1, kDevTimeoutFull))) break;
        tc_fence_after();
        const uint32_t st = smem_u32(smem + s * STAGE);
        umma_ss_mn_t128_warp(acc, umma_desc_noswz(st, 128, 2048), umma_desc_sw128(st + A_BYTES, C::BOX, 1024), ID,
                             t > 0);
        umma_commit_warp(&bars->empty[s]);
      }
      if (!ok) break;
      umma_commit_warp(&bars->acc_full[k & 1]);
      J += n;
    }
    umma_drain_warp(&bars->mma_drain);  // before TMEM is freed, also when a wait ran out
  } else {
    const int sub = warp & 3, half = (warp - 2) >> 2;
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    constexpr int W = HD / 2;  // columns per warp
    bool ok = true;
    for (int k = 0; ok; ++k) {
      const int tile = take_tile(k, ok);
      if (!ok || tile < 0) break;
      const DqsTile d = dqs_tile(tile, p);
      if (!(ok = mbar_wait_warp(&bars->acc_full[k & 1], (k >> 1) & 1, kDevTimeoutFull))) break;
      tc_fence_after();
      const uint32_t src = tbase + (k & 1) * HD + lane_bits + half * W;
      uint32_t v[W / 32][32];
#pragma unroll
      for (int c = 0; c < W / 32; ++c) tmem_ld32(src + 32 * c, v[c]);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->acc_empty[k & 1]);
      const int q_tok = d.q0 + sub * 32 + lane;
      if (q_tok < p.L) {
        uint4* d4 = reinterpret_cast<uint4*>(p.dq + ((size_t)q_tok * p.Hq + d.h) * HD + half * W);
#pragma unroll
        for (int c = 0; c < W / 32; ++c)
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            const uint32_t* u = v[c] + 8 * q4;
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(u[0]) * p.scale, __uint_as_float(u[1]) * p.scale);
            w.y = pack_bf16x2(__uint_as_float(u[2]) * p.scale, __uint_as_float(u[3]) * p.scale);
            w.z = pack_bf16x2(__uint_as_float(u[4]) * p.scale, __uint_as_float(u[5]) * p.scale);
            w.w = pack_bf16x2(__uint_as_float(u[6]) * p.scale, __uint_as_float(u[7]) * p.scale);
            d4[4 * c + q4] = w;
          }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tbase, 2 * HD);
  }
}

// Stored-dS pair offsets: pair_off[i] = number of (query tile, key tile)
// pairs of query tiles before i, query tile i visiting key tiles
// tile_lo[i] / 128 .. i; pair_off[T] = all pairs. One block of 1024 threads
// scans the T = ceil(L / 128) entries in chunks with a carried total.
__global__ void __launch_bounds__(1024) pair_offsets_kernel(const int32_t* __restrict__ tile_lo, int T,
                                                            int32_t* __restrict__ pair_off) {
  __shared__ int warp_sum[32];
  __shared__ int carry;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < T; base += 1024) {
    const int i = base + threadIdx.x;
    const int v = i < T ? i - tile_lo[i] / 128 + 1 : 0;
    int x = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += y;
    }
    if (lane == 31) warp_sum[warp] = x;
    __syncthreads();
    if (warp == 0) {
      int w = warp_sum[lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += y;
      }
      warp_sum[lane] = w;
    }
    __syncthreads();
    const int excl = carry + (warp > 0 ? warp_sum[warp - 1] : 0) + x - v;
    if (i < T) pair_off[i] = excl;
    __syncthreads();
    if (threadIdx.x == 1023) carry = excl + v;
    __syncthreads();
  }
  if (threadIdx.x == 0) pair_off[T] = carry;
}

cudaError_t launch_varlen_pair_offsets(const int32_t* tile_lo, int L, int32_t* pair_off, cudaStream_t stream) {
  pair_offsets_kernel<<<1, 1024, 0, stream>>>(tile_lo, (L + 127) / 128, pair_off);
  return cudaGetLastError();
}

template <int HD>
static cudaError_t launch_bwd_hd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                                 const CUtensorMap& dom, const VarlenBwdParams& p, cudaStream_t stream) {
  using C = BwdTile<HD>;
  const int n_t = (p.L + 127) / 128;
  const int smem_dq = 7 * C::TILE + (int)sizeof(DqBars);
  const int smem_kv = 7 * C::TILE + 5 * 128 * 4 + (int)sizeof(DkdvBars);
  cudaError_t e = cudaFuncSetAttribute(varlen_bwd_dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_kv);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(varlen_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dq);
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int kv_grid = std::max(1, std::min(n_t * p.Hkv, sms));  // persistent: one CTA per SM
  varlen_bwd_dkdv_kernel<HD><<<kv_grid, kBwdThreads, smem_kv, stream>>>(qm, km, vm, dom, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  const int dq_grid = std::max(1, std::min(n_t * p.Hq, sms));  // persistent: one CTA per SM
  if (p.ds != nullptr) {
    constexpr int smem_dqs = kDqsStages * (128 * 128 * 2 + C::TILE) + (int)sizeof(DqsBars);
    e = cudaFuncSetAttribute(varlen_bwd_dq_stored_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dqs);
    if (e != cudaSuccess) return e;
    varlen_bwd_dq_stored_kernel<HD><<<dq_grid, kDqsThreads, smem_dqs, stream>>>(km, p);
    return cudaGetLastError();
  }
  varlen_bwd_dq_kernel<HD><<<dq_grid, kBwdThreads, smem_dq, stream>>>(qm, km, vm, dom, p);
  return cudaGetLastError();
}

cudaError_t launch_varlen_bwd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                              const CUtensorMap& dom, const __nv_bfloat16* out, const __nv_bfloat16* dout,
                              VarlenBwdParams p, cudaStream_t stream) {
  // Whole rows per thread group; a grid of 8 blocks per SM keeps enough loads
  // in flight to saturate HBM.
  const long long threads_needed = (long long)p.L * p.Hq * (p.head_dim / 8);
  const int blocks = (int)std::max<long long>(1, std::min<long long>((threads_needed + 255) / 256, 148 * 8));
  bwd_delta_kernel<<<blocks, 256, 0, stream>>>(out, dout, p.L, p.Hq, p.head_dim, p.delta, p.tile_counter);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return p.head_dim == 128 ? launch_bwd_hd<128>(qm, km, vm, dom, p, stream)
                           : launch_bwd_hd<64>(qm, km, vm, dom, p, stream);
}

}  // namespace mb
