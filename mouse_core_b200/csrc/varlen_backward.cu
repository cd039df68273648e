// K6: packed varlen segment-causal GQA attention backward on tcgen05.
//
// Gradient of K5 (the attention of flex_train.py:147 under the mask of
// flex_train.py:98-102); the reference gets it from autograd through compiled
// flex_attention. With z = scale * q k^T masked to run_start[i] <= j <= i,
// P = softmax(z) = 2^(z log2 e - lse2), D_i = sum_d dO[i,d] O[i,d]:
//   dV = P^T dO,  dS = P o (dO V^T - D),  dQ = scale dS K,  dK = scale dS^T Q,
// with dK/dV summed over the q-heads sharing a kv-head.
//
// Three kernels, no atomics (deterministic):
//  * delta:  D[h, i] (fp32) from dO and O.
//  * dkdv:   one CTA per (128-key tile, kv-head). It walks every (q-head of the
//            group, 128-query tile) pair whose queries may see its keys (from
//            its own tile to the end of its last key's run). Per pair, with
//            keys on the TMEM lanes: S^T = K Q^T, P^T, dP^T = V dO^T,
//            dS^T = P^T o (dP^T - D), then dV += P^T dO and dK += dS^T Q with
//            P^T / dS^T taken from TMEM. dV, dK accumulate in TMEM across the
//            whole walk.
//  * dq:     one CTA per (128-query tile, q-head), walking the same key tiles
//            as the forward: S = Q K^T, P, dP = dO V^T, dS, dQ += dS K.
// Warp roles (320 threads): warp 0 TMA producer, warp 1 TMEM allocator and
// MMA issuer, warps 2-5 and 6-9 the element-wise work of the two streams
// (thread = TMEM lane = one key / query row). Both walks alternate
// two streams (even / odd pairs) so one stream's element-wise work overlaps
// the other's MMAs. Each stream has one 128-column
// TMEM scratch that holds S, then dP, then the bf16 dS (and P) operands;
// P stays in registers (as bf16 pairs, the precision the MMAs take it in)
// across the dP MMA.
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
__global__ void bwd_delta_kernel(const __nv_bfloat16* __restrict__ out, const __nv_bfloat16* __restrict__ dout,
                                 int L, int Hq, int hd, float* __restrict__ delta) {
  const int warps = (gridDim.x * blockDim.x) >> 5;
  const int lane = threadIdx.x & 31;
  for (long long w = (long long)(blockIdx.x * blockDim.x + threadIdx.x) >> 5; w < (long long)L * Hq; w += warps) {
    const long long i = w / Hq;
    const int h = (int)(w % Hq);
    const __nv_bfloat16* o = out + (i * Hq + h) * hd;
    const __nv_bfloat16* g = dout + (i * Hq + h) * hd;
    float acc = 0.f;
    for (int d = lane * 2; d < hd; d += 64) {
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(o + d));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(g + d));
      acc += a.x * b.x + a.y * b.y;
    }
    acc = warp_sum(acc);
    if (lane == 0) delta[(long long)h * L + i] = acc;
  }
}

// ---------------------------------------------------------------- shared pieces
struct BwdBars {
  uint64_t fixed_full;          // K,V (dkdv) or Q,dO (dq)
  uint64_t ring_full[2], ring_empty[2];
  uint64_t ring_v_full[2];      // dq only: V half of a ring slot
  uint64_t s_full[2], ew1[2], dp_full[2], ew2[2];
  uint64_t acc_full;
  uint32_t tmem_base;
};

__device__ __forceinline__ void init_bwd_bars(BwdBars* b, int ring_full_count) {
  mbar_init(&b->fixed_full, 1);
  for (int s = 0; s < 2; ++s) {
    mbar_init(&b->ring_full[s], ring_full_count);
    mbar_init(&b->ring_empty[s], 1);
    mbar_init(&b->ring_v_full[s], 1);
    mbar_init(&b->s_full[s], 1);
    mbar_init(&b->ew1[s], 4);
    mbar_init(&b->dp_full[s], 1);
    mbar_init(&b->ew2[s], 4);
  }
  mbar_init(&b->acc_full, 1);
  fence_barrier_init();
}

// D = A B^T over HD; A and B K-major in smem (128 rows x HD). The start
// address is the descriptor's low field, so K-steps add (offset >> 4) to the
// 64-bit descriptor (shared-memory addresses stay below 2^18, no carry).
// Issue loops stay rolled to keep the issuing warp's registers few.
template <int HD>
__device__ __forceinline__ void mma_kmajor_ss(uint32_t d, uint32_t a_base, uint32_t b_base, uint32_t idesc) {
  const uint64_t da = umma_desc_sw128(a_base, 16, 1024), db = umma_desc_sw128(b_base, 16, 1024);
#pragma unroll 1
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint32_t off = ((kk >> 2) * BwdTile<HD>::BOX + (kk & 3) * 32) >> 4;
    umma_ss(d, da + off, db + off, idesc, kk > 0);
  }
}

// D (+)= A_tmem[128 x 128 (bf16, 64 cols)] * B[128 x HD] with B MN-major in smem.
template <int HD>
__device__ __forceinline__ void mma_tmem_a(uint32_t d, uint32_t a_tmem, uint32_t b_base, uint32_t idesc,
                                           bool accumulate) {
  const uint64_t db = umma_desc_sw128(b_base, BwdTile<HD>::BOX, 1024);
#pragma unroll 1
  for (int kk = 0; kk < 8; ++kk)
    umma_ts(d, a_tmem + 8 * kk, db + (uint64_t)((kk * 2048) >> 4), idesc, (accumulate || kk > 0) ? 1u : 0u);
}

// ---------------------------------------------------------------- dq kernel
template <int HD>
__global__ void __launch_bounds__(320, 1) varlen_bwd_dq_kernel(const __grid_constant__ CUtensorMap qmap,
                                                              const __grid_constant__ CUtensorMap kmap,
                                                              const __grid_constant__ CUtensorMap vmap,
                                                              const __grid_constant__ CUtensorMap dom,
                                                              const VarlenBwdParams p) {
  using C = BwdTile<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* qs = smem;
  uint8_t* dos = smem + C::TILE;
  uint8_t* ks = smem + 2 * C::TILE;   // [2][TILE]
  uint8_t* vs = smem + 4 * C::TILE;   // [2][TILE]
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + 6 * C::TILE);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (p.L + 127) / 128;
  const int qt = n_qt - 1 - (int)blockIdx.x;
  const int q0 = qt * 128;
  const int h = blockIdx.y;
  const int kvh = h / p.G;
  const int t_lo = p.run_start[q0] / 128;
  const int t_hi = min(q0 + 127, p.L - 1) / 128;
  const int n = t_hi - t_lo + 1;

  if (threadIdx.x == 0) init_bwd_bars(bars, 1);
  if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t t_dq = tbase + 256;

  if (warp == 0) {
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      prefetch_tensormap(&dom);
      mbar_arrive_expect_tx(&bars->fixed_full, 2 * C::TILE);
      for (int cb = 0; cb < C::NCB; ++cb) {
        tma_load_3d(qs + cb * C::BOX, &qmap, &bars->fixed_full, cb * 64, h, q0);
        tma_load_3d(dos + cb * C::BOX, &dom, &bars->fixed_full, cb * 64, h, q0);
      }
      for (int j = 0; j < n; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bars->ring_empty[s], ((j >> 1) & 1) ^ 1, kDevTimeoutEmpty)) break;
        const int kv0 = (t_lo + j) * 128;
        mbar_arrive_expect_tx(&bars->ring_full[s], C::TILE);
        for (int cb = 0; cb < C::NCB; ++cb)
          tma_load_3d(ks + s * C::TILE + cb * C::BOX, &kmap, &bars->ring_full[s], cb * 64, kvh, kv0);
        mbar_arrive_expect_tx(&bars->ring_v_full[s], C::TILE);
        for (int cb = 0; cb < C::NCB; ++cb)
          tma_load_3d(vs + s * C::TILE + cb * C::BOX, &vmap, &bars->ring_v_full[s], cb * 64, kvh, kv0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t ID_DQ = umma_idesc_bf16(128, HD, 0, 1);
      bool ok = mbar_wait(&bars->fixed_full, 0, kDevTimeoutFull);
      const uint32_t qa = smem_u32(qs), da = smem_u32(dos);
      auto issue_s = [&](int j) {
        const int s = j & 1;
        if (!mbar_wait(&bars->ring_full[s], (j >> 1) & 1, kDevTimeoutFull)) return false;
        tc_fence_after();
        mma_kmajor_ss<HD>(tbase + 128 * s, qa, smem_u32(ks + s * C::TILE), ID_S);
        umma_commit(&bars->s_full[s]);
        return true;
      };
      tc_fence_after();
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int j0 = 0; ok && j0 < n; j0 += 2) {
        for (int j = j0; ok && j < min(j0 + 2, n); ++j) {
          const int s = j & 1;
          ok = mbar_wait(&bars->ew1[s], (j >> 1) & 1, kDevTimeoutFull) &&
               mbar_wait(&bars->ring_v_full[s], (j >> 1) & 1, kDevTimeoutFull);
          if (!ok) break;
          tc_fence_after();
          mma_kmajor_ss<HD>(tbase + 128 * s, da, smem_u32(vs + s * C::TILE), ID_S);  // dP = dO V^T
          umma_commit(&bars->dp_full[s]);
        }
        for (int j = j0; ok && j < min(j0 + 2, n); ++j) {
          const int s = j & 1;
          if (!(ok = mbar_wait(&bars->ew2[s], (j >> 1) & 1, kDevTimeoutFull))) break;
          tc_fence_after();
          mma_tmem_a<HD>(t_dq, tbase + 128 * s, smem_u32(ks + s * C::TILE), ID_DQ, j > 0);  // dQ += dS K
          umma_commit(&bars->ring_empty[s]);
          if (j + 2 < n) ok = issue_s(j + 2);
        }
      }
      umma_commit(&bars->acc_full);
    }
  } else {
    const int grp = (warp - 2) >> 2;  // stream: even / odd key tiles
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const int q_tok = q0 + r;
    const bool row_ok = q_tok < p.L;
    const int lo = row_ok ? p.run_start[q_tok] : 0x7fffffff;
    const float neg_lse = row_ok ? -p.lse[(size_t)h * p.L + q_tok] : 0.f;
    const float dlt = row_ok ? p.delta[(size_t)h * p.L + q_tok] : 0.f;
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    const uint32_t t_x = tbase + 128 * grp + lane_bits;
    const uint32_t t_p = tbase + 384 + 64 * grp + lane_bits;
    bool ok = true;
    for (int j = grp; j < n; j += 2) {
      const int kv0 = (t_lo + j) * 128;
      const uint32_t par = (j >> 1) & 1;
      if (ok) ok = mbar_wait_warp(&bars->s_full[grp], par, kDevTimeoutFull);
      tc_fence_after();
      if (ok) {
        const bool full = row_ok && kv0 >= lo && kv0 + 127 <= q_tok;
        uint32_t v[128];
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_x + 32 * c, *reinterpret_cast<uint32_t(*)[32]>(v + 32 * c));
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const int col = 16 * c + e;
            float x0 = fast_exp2(fmaf(__uint_as_float(v[col]), p.scale_log2, neg_lse));
            float x1 = fast_exp2(fmaf(__uint_as_float(v[col + 1]), p.scale_log2, neg_lse));
            if (!full) {
              const int kv = kv0 + col;
              if (!row_ok || kv < lo || kv > q_tok) x0 = 0.f;
              if (!row_ok || kv + 1 < lo || kv + 1 > q_tok) x1 = 0.f;
            }
            pk[e >> 1] = pack_bf16x2(x0, x1);
          }
          tmem_st8(t_p + 8 * c, pk);  // P parked in spare TMEM across the dP MMA
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ew1[grp]);
      if (ok) ok = mbar_wait_warp(&bars->dp_full[grp], par, kDevTimeoutFull);
      tc_fence_after();
      if (ok) {
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          uint32_t v[64], pp[32];
          tmem_ld32(t_x + 64 * hf, *reinterpret_cast<uint32_t(*)[32]>(v));
          tmem_ld32(t_x + 64 * hf + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
          tmem_ld32(t_p + 32 * hf, pp);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint32_t pk[8];
#pragma unroll
            for (int e = 0; e < 16; e += 2) {
              const int col = 16 * c + e;
              const float2 pf = unpack_bf16x2(pp[col >> 1]);
              pk[e >> 1] = pack_bf16x2(pf.x * (__uint_as_float(v[col]) - dlt),
                                       pf.y * (__uint_as_float(v[col + 1]) - dlt));
            }
            tmem_st8(t_x + 32 * hf + 8 * c, pk);  // dS over dP columns already read
          }
        }
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ew2[grp]);
    }
    // Epilogue: stream 0 writes dQ columns [0, HD/2), stream 1 [HD/2, HD).
    if (ok) ok = mbar_wait_warp(&bars->acc_full, 0, kDevTimeoutFull);
    tc_fence_after();
    if (ok) {
      __nv_bfloat16* dst = p.dq + ((size_t)q_tok * p.Hq + h) * HD;
#pragma unroll
      for (int c = 0; c < HD / 64; ++c) {
        const int col = grp * (HD / 2) + 32 * c;
        uint32_t v[32];
        tmem_ld32(t_dq + lane_bits + col, v);
        tmem_wait_ld();
        if (row_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + col);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * q4 + 0]) * p.scale, __uint_as_float(v[8 * q4 + 1]) * p.scale);
            w.y = pack_bf16x2(__uint_as_float(v[8 * q4 + 2]) * p.scale, __uint_as_float(v[8 * q4 + 3]) * p.scale);
            w.z = pack_bf16x2(__uint_as_float(v[8 * q4 + 4]) * p.scale, __uint_as_float(v[8 * q4 + 5]) * p.scale);
            w.w = pack_bf16x2(__uint_as_float(v[8 * q4 + 6]) * p.scale, __uint_as_float(v[8 * q4 + 7]) * p.scale);
            d4[q4] = w;
          }
        }
      }
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
template <int HD>
__global__ void __launch_bounds__(320, 1) varlen_bwd_dkdv_kernel(const __grid_constant__ CUtensorMap qmap,
                                                                const __grid_constant__ CUtensorMap kmap,
                                                                const __grid_constant__ CUtensorMap vmap,
                                                                const __grid_constant__ CUtensorMap dom,
                                                                const VarlenBwdParams p) {
  using C = BwdTile<HD>;
  constexpr int VEC = 2 * 128 * 4;  // lse + delta of one query tile (f32)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* ks = smem;
  uint8_t* vs = smem + C::TILE;
  uint8_t* qring = smem + 2 * C::TILE;     // [2][TILE]
  uint8_t* dring = smem + 4 * C::TILE;     // [2][TILE]
  float* vecs = reinterpret_cast<float*>(smem + 6 * C::TILE);  // [2][2][128]
  BwdBars* bars = reinterpret_cast<BwdBars*>(smem + 6 * C::TILE + 2 * VEC);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_kt = (p.L + 127) / 128;
  const int kt = (int)blockIdx.x;
  const int kv0 = kt * 128;
  const int kvh = blockIdx.y;
  const int last = min(kv0 + 127, p.L - 1);
  const int i_lo = kt;
  const int i_hi = (p.run_end[last] - 1) / 128;
  const int nqi = i_hi - i_lo + 1;
  const int n = p.G * nqi;  // (q-head, query tile) pairs
  (void)n_kt;

  if (threadIdx.x == 0) init_bwd_bars(bars, 2);
  if (warp == 1) tmem_alloc(&bars->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;
  const uint32_t t_dv = tbase + 256, t_dk = tbase + 256 + HD;

  if (warp == 0) {
    // Producer warp: lane 0 issues TMA; all lanes stage lse / delta.
    if (lane == 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      prefetch_tensormap(&dom);
      mbar_arrive_expect_tx(&bars->fixed_full, 2 * C::TILE);
      for (int cb = 0; cb < C::NCB; ++cb) {
        tma_load_3d(ks + cb * C::BOX, &kmap, &bars->fixed_full, cb * 64, kvh, kv0);
        tma_load_3d(vs + cb * C::BOX, &vmap, &bars->fixed_full, cb * 64, kvh, kv0);
      }
    }
    bool ok = true;
    for (int t = 0; t < n; ++t) {
      const int s = t & 1;
      const int hq = kvh * p.G + t / nqi;
      const int q0 = (i_lo + t % nqi) * 128;
      if (lane == 0) ok = ok && mbar_wait(&bars->ring_empty[s], ((t >> 1) & 1) ^ 1, kDevTimeoutEmpty);
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars->ring_full[s], 2 * C::TILE);
        for (int cb = 0; cb < C::NCB; ++cb) {
          tma_load_3d(qring + s * C::TILE + cb * C::BOX, &qmap, &bars->ring_full[s], cb * 64, hq, q0);
          tma_load_3d(dring + s * C::TILE + cb * C::BOX, &dom, &bars->ring_full[s], cb * 64, hq, q0);
        }
      }
      float* lse_s = vecs + s * 256;
      for (int c = lane; c < 128; c += 32) {
        const int q = q0 + c;
        lse_s[c] = (q < p.L) ? p.lse[(size_t)hq * p.L + q] : INFINITY;
        lse_s[128 + c] = (q < p.L) ? p.delta[(size_t)hq * p.L + q] : 0.f;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ring_full[s]);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t ID_S = umma_idesc_bf16(128, 128, 0, 0);
      constexpr uint32_t ID_G = umma_idesc_bf16(128, HD, 0, 1);
      bool ok = mbar_wait(&bars->fixed_full, 0, kDevTimeoutFull);
      const uint32_t ka = smem_u32(ks), va = smem_u32(vs);
      auto issue_s = [&](int t) {
        const int s = t & 1;
        if (!mbar_wait(&bars->ring_full[s], (t >> 1) & 1, kDevTimeoutFull)) return false;
        tc_fence_after();
        mma_kmajor_ss<HD>(tbase + 128 * s, ka, smem_u32(qring + s * C::TILE), ID_S);  // S^T = K Q^T
        umma_commit(&bars->s_full[s]);
        return true;
      };
      tc_fence_after();
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int t0 = 0; ok && t0 < n; t0 += 2) {
        for (int t = t0; ok && t < min(t0 + 2, n); ++t) {
          const int s = t & 1;
          if (!(ok = mbar_wait(&bars->ew1[s], (t >> 1) & 1, kDevTimeoutFull))) break;
          tc_fence_after();
          mma_kmajor_ss<HD>(tbase + 128 * s, va, smem_u32(dring + s * C::TILE), ID_S);  // dP^T = V dO^T
          umma_commit(&bars->dp_full[s]);
        }
        for (int t = t0; ok && t < min(t0 + 2, n); ++t) {
          const int s = t & 1;
          if (!(ok = mbar_wait(&bars->ew2[s], (t >> 1) & 1, kDevTimeoutFull))) break;
          tc_fence_after();
          mma_tmem_a<HD>(t_dv, tbase + 128 * s + 64, smem_u32(dring + s * C::TILE), ID_G, t > 0);  // dV += P^T dO
          mma_tmem_a<HD>(t_dk, tbase + 128 * s, smem_u32(qring + s * C::TILE), ID_G, t > 0);       // dK += dS^T Q
          umma_commit(&bars->ring_empty[s]);
          if (t + 2 < n) ok = issue_s(t + 2);
        }
      }
      umma_commit(&bars->acc_full);
    }
  } else {
    const int grp = (warp - 2) >> 2;
    const int sub = warp & 3;
    const int r = sub * 32 + lane;
    const int k_tok = kv0 + r;
    const bool k_ok = k_tok < p.L;
    const int q_end = k_ok ? p.run_end[k_tok] : 0;  // queries k_tok <= q < q_end see this key
    const uint32_t lane_bits = (uint32_t)(sub * 32) << 16;
    const uint32_t t_x = tbase + 128 * grp + lane_bits;
    bool ok = true;
    for (int t = grp; t < n; t += 2) {
      const int s = t & 1;
      const int q0 = (i_lo + t % nqi) * 128;
      const uint32_t par = (t >> 1) & 1;
      if (ok) ok = mbar_wait_warp(&bars->ring_full[s], par, kDevTimeoutFull);
      if (ok) ok = mbar_wait_warp(&bars->s_full[s], par, kDevTimeoutFull);
      tc_fence_after();
      const float* lse_s = vecs + s * 256;
      uint32_t pr[64];  // P^T as bf16 pairs, kept across the dP^T MMA
      if (ok) {
        const bool full = k_ok && q0 >= k_tok && q0 + 127 < q_end;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t v[16];
          tmem_ld16(t_x + 16 * c, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const int col = 16 * c + e;
            float x0 = fast_exp2(fmaf(__uint_as_float(v[e]), p.scale_log2, -lse_s[col]));
            float x1 = fast_exp2(fmaf(__uint_as_float(v[e + 1]), p.scale_log2, -lse_s[col + 1]));
            if (!full) {
              const int q = q0 + col;
              if (q < k_tok || q >= q_end) x0 = 0.f;
              if (q + 1 < k_tok || q + 1 >= q_end) x1 = 0.f;
            }
            pr[col >> 1] = pack_bf16x2(x0, x1);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ew1[s]);
      if (ok) ok = mbar_wait_warp(&bars->dp_full[s], par, kDevTimeoutFull);
      tc_fence_after();
      if (ok) {
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t v[16];
          tmem_ld16(t_x + 16 * c, v);
          tmem_wait_ld();
          uint32_t pk[8];
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const int col = 16 * c + e;
            const float2 pf = unpack_bf16x2(pr[col >> 1]);
            pk[e >> 1] = pack_bf16x2(pf.x * (__uint_as_float(v[e]) - lse_s[128 + col]),
                                     pf.y * (__uint_as_float(v[e + 1]) - lse_s[128 + col + 1]));
          }
          tmem_st8(t_x + 8 * c, pk);  // dS^T over dP^T columns already read
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_st16(t_x + 64 + 16 * c, *reinterpret_cast<uint32_t(*)[16]>(pr + 16 * c));
        tmem_wait_st();
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->ew2[s]);
    }
    // Epilogue: stream 0 writes dV, stream 1 writes dK (scaled).
    if (ok) ok = mbar_wait_warp(&bars->acc_full, 0, kDevTimeoutFull);
    tc_fence_after();
    if (ok) {
      const uint32_t src = (grp == 0 ? t_dv : t_dk) + lane_bits;
      const float mul = (grp == 0) ? 1.f : p.scale;
      __nv_bfloat16* dst = (grp == 0 ? p.dv : p.dk) + ((size_t)k_tok * p.Hkv + kvh) * HD;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(src + 32 * c, v);
        tmem_wait_ld();
        if (k_ok) {
          uint4* d4 = reinterpret_cast<uint4*>(dst + 32 * c);
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 w;
            w.x = pack_bf16x2(__uint_as_float(v[8 * q4 + 0]) * mul, __uint_as_float(v[8 * q4 + 1]) * mul);
            w.y = pack_bf16x2(__uint_as_float(v[8 * q4 + 2]) * mul, __uint_as_float(v[8 * q4 + 3]) * mul);
            w.z = pack_bf16x2(__uint_as_float(v[8 * q4 + 4]) * mul, __uint_as_float(v[8 * q4 + 5]) * mul);
            w.w = pack_bf16x2(__uint_as_float(v[8 * q4 + 6]) * mul, __uint_as_float(v[8 * q4 + 7]) * mul);
            d4[q4] = w;
          }
        }
      }
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

template <int HD>
static cudaError_t launch_bwd_hd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                                 const CUtensorMap& dom, const VarlenBwdParams& p, cudaStream_t stream) {
  using C = BwdTile<HD>;
  const int n_t = (p.L + 127) / 128;
  const int smem_dq = 1024 + 6 * C::TILE + (int)sizeof(BwdBars) + 64;
  const int smem_kv = 1024 + 6 * C::TILE + 2 * 2 * 128 * 4 + (int)sizeof(BwdBars) + 64;
  cudaError_t e = cudaFuncSetAttribute(varlen_bwd_dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_kv);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(varlen_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_dq);
  if (e != cudaSuccess) return e;
  varlen_bwd_dkdv_kernel<HD><<<dim3(n_t, p.Hkv), 320, smem_kv, stream>>>(qm, km, vm, dom, p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  varlen_bwd_dq_kernel<HD><<<dim3(n_t, p.Hq), 320, smem_dq, stream>>>(qm, km, vm, dom, p);
  return cudaGetLastError();
}

cudaError_t launch_varlen_bwd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                              const CUtensorMap& dom, const __nv_bfloat16* out, const __nv_bfloat16* dout,
                              VarlenBwdParams p, cudaStream_t stream) {
  const long long warps_needed = (long long)p.L * p.Hq;
  const int blocks = (int)std::min<long long>((warps_needed + 7) / 8, 148 * 32);
  bwd_delta_kernel<<<blocks, 256, 0, stream>>>(out, dout, p.L, p.Hq, p.head_dim, p.delta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return p.head_dim == 128 ? launch_bwd_hd<128>(qm, km, vm, dom, p, stream)
                           : launch_bwd_hd<64>(qm, km, vm, dom, p, stream);
}

}  // namespace mb
