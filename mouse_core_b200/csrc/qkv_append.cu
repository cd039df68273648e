// K13: the decode layer's QKV projection with K2 as its epilogue.
//
// One tcgen05 GEMM y = x W^T (x [T, K] bf16: the normalised hidden states of
// the step's tokens; W [N, K] bf16: q_proj | k_proj | v_proj stacked,
// N = (Hq + 2 Hkv) * HD) whose fp32 accumulator tile — 128 tokens x 128
// columns, one head at hd 128 and two at hd 64 — goes from TMEM straight into
// the K2 arithmetic: bias, q/k RMSNorm, RoPE, one rounding to bf16, q to its
// output and k/v to their page slots. Replaces the fp32 QKV GEMM and
// mb_kv_append_f32 of the fp32-residual decode layer (the q/k/v projections,
// q_norm/k_norm, rotary embedding and cache scatter of
// models/backbone/flex_decode.py:204-224): the [T, N] fp32 projection never
// leaves the SM.
//
// The RoPE cos/sin of each token and frequency come from a table built once
// per step (rope_table_kernel: the same sincosf of pos * inv_freq as K2, so
// the rotation factors are K2's), shared by every layer.
//
// CTA (192 threads): warp 0 TMA producer (64-element K-boxes of x and W, 128
// rows each, 128-byte swizzle, a 4-stage ring), warp 1 TMEM owner and MMA
// issuer (M = N = 128, K = 16 per instruction, fp32 in 128 TMEM columns),
// warps 2-5 the epilogue: warp w reads TMEM lane quarter w % 4, so each
// thread holds one token's 128 columns and normalises and rotates its
// head(s) without any exchange between threads. Every wait is bounded; the
// producer lets its loads land and the MMA warp its MMAs complete before
// TMEM is freed.
#include <atomic>

#include "common.cuh"
#include "kernels.h"
#include "tcgen05.cuh"

namespace mb {

constexpr int kQaStages = 4;
constexpr int kQaThreads = 192;
constexpr int kQaBox = 128 * 64 * 2;  // 128 rows x 64 bf16 elements

struct QaBars {
  uint64_t full[kQaStages], empty[kQaStages];
  uint64_t acc_full;   // the tile's last MMA complete
  uint64_t mma_drain;  // every MMA complete, before TMEM is freed
  uint32_t tmem_base;
};

// D (+)= A B^T over 64 elements of K (four K-steps of 16, 32 bytes apart in
// the 128-byte swizzled rows); `accumulate` applies to the first K-step.
__device__ __forceinline__ void umma_ss_k64_acc_warp(uint32_t d, uint64_t da, uint64_t db, uint32_t idesc,
                                                     uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred e, t, p;\n\t.reg .b64 a, b;\n\t"
      "elect.sync _|e, 0xffffffff;\n\tsetp.eq.b32 t, %3, %3;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t"
      "add.s64 a, %1, 2;\n\tadd.s64 b, %2, 2;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 4;\n\tadd.s64 b, %2, 4;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t"
      "add.s64 a, %1, 6;\n\tadd.s64 b, %2, 6;\n\t@e tcgen05.mma.cta_group::1.kind::f16 [%0], a, b, %3, t;\n\t}"
      ::"r"(d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate));
}

// table[t][j] = (cos, sin)(pos[t] * inv_freq[j]) * attn_scaling, j < HD / 2:
// the rotation factors K2 computes per element.
__global__ void __launch_bounds__(256) rope_table_kernel(const int32_t* __restrict__ pos, int T,
                                                         const float* __restrict__ inv_freq, int half,
                                                         float attn_scaling, float2* __restrict__ table) {
  const long long n = (long long)T * half;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const int t = (int)(i / half), j = (int)(i % half);
    float s, c;
    sincosf((float)pos[t] * inv_freq[j], &s, &c);
    table[i] = make_float2(c * attn_scaling, s * attn_scaling);
  }
}

template <int HD>
__global__ void __launch_bounds__(kQaThreads, 1) qkv_append_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ CUtensorMap wmap,
                                                                   const QkvAppendParams p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  if (!smem_base_aligned(smem)) {
    if (threadIdx.x == 0) report(kDevBadSmem);
    return;
  }
  uint8_t* xs = smem;                      // [STAGES][128 tokens x 64]
  uint8_t* ws = smem + kQaStages * kQaBox;  // [STAGES][128 columns x 64]
  QaBars* bars = reinterpret_cast<QaBars*>(smem + 2 * kQaStages * kQaBox);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * 128, n0 = blockIdx.y * 128;
  const int nk = (p.K + 63) / 64;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kQaStages; ++s) {
      mbar_init(&bars->full[s], 1);
      mbar_init(&bars->empty[s], 1);
    }
    mbar_init(&bars->acc_full, 1);
    mbar_init(&bars->mma_drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) tmem_alloc(&bars->tmem_base, 128);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = bars->tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      prefetch_tensormap(&xmap);
      prefetch_tensormap(&wmap);
      int issued = 0;
      for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kQaStages;
        if (!mbar_wait(&bars->empty[s], ((kb / kQaStages) & 1) ^ 1, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&bars->full[s], 2 * kQaBox);
        tma_load_2d(xs + s * kQaBox, &xmap, &bars->full[s], kb * 64, m0);  // rows past T read as zero
        tma_load_2d(ws + s * kQaBox, &wmap, &bars->full[s], kb * 64, n0);
        ++issued;
      }
      drain_ring(bars->full, kQaStages, issued);  // every load lands before the CTA exits
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issue
    constexpr uint32_t ID = umma_idesc_bf16(128, 128, 0, 0);
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kQaStages;
      if (!(ok = mbar_wait_warp(&bars->full[s], (kb / kQaStages) & 1, kDevTimeoutFull))) break;
      tc_fence_after();
      const uint64_t da = umma_desc_sw128(smem_u32(xs + s * kQaBox), 16, 1024);
      const uint64_t db = umma_desc_sw128(smem_u32(ws + s * kQaBox), 16, 1024);
      umma_ss_k64_acc_warp(tbase, da, db, ID, kb > 0 ? 1u : 0u);
      umma_commit_warp(&bars->empty[s]);
    }
    if (ok) umma_commit_warp(&bars->acc_full);
    umma_drain_warp(&bars->mma_drain);  // before TMEM is freed, also when a wait ran out
  } else {
    // ------------------------------------------------------------ epilogue
    const int sub = warp & 3;
    const int t = m0 + sub * 32 + lane;  // this thread's token
    const uint32_t trow = tbase + ((uint32_t)(sub * 32) << 16);
    const bool ok = mbar_wait_warp(&bars->acc_full, 0, kDevTimeoutFull);
    tc_fence_after();
    const long long slot = (t < p.T && p.slot != nullptr) ? (long long)p.slot[t] : -1;
    const bool cached = slot >= 0 && slot < p.num_slots && p.k_pool != nullptr && p.v_pool != nullptr;
    const long long page = cached ? slot / p.page_size : 0;
    const int off = cached ? (int)(slot % p.page_size) : 0;
#pragma unroll 1
    for (int hh = 0; ok && hh < 128 / HD; ++hh) {
      const int head = n0 / HD + hh;  // in q | k | v order
      const int col0 = n0 + hh * HD;
      float x[HD];
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(trow + hh * HD + 32 * c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) x[32 * c + e] = __uint_as_float(v[e]);
      }
      if (t >= p.T) continue;
      if (p.bias != nullptr) {
#pragma unroll
        for (int e = 0; e < HD; ++e) x[e] += __bfloat162float(p.bias[col0 + e]);
      }
      const bool is_q = head < p.Hq;
      const bool is_k = !is_q && head < p.Hq + p.Hkv;
      if (is_q || is_k) {
        const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
        if (nw != nullptr) {
          float ss = 0.f;
#pragma unroll
          for (int e = 0; e < HD; ++e) ss = fmaf(x[e], x[e], ss);
          const float r = rsqrtf(ss / (float)HD + p.eps);
#pragma unroll
          for (int e = 0; e < HD; ++e) x[e] = x[e] * r * __bfloat162float(nw[e]);
        }
        // rotate_half: dim j pairs with j + HD / 2, both turned by frequency j.
        const float4* cs4 = reinterpret_cast<const float4*>(p.rope + (size_t)t * (HD / 2));
#pragma unroll
        for (int j2 = 0; j2 < HD / 4; ++j2) {
          const float4 f = cs4[j2];  // (cos, sin) of frequencies 2 j2 and 2 j2 + 1
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int j = 2 * j2 + u;
            const float c = u ? f.z : f.x, s = u ? f.w : f.y;
            const float a = x[j], b = x[j + HD / 2];
            x[j] = a * c - b * s;
            x[j + HD / 2] = b * c + a * s;
          }
        }
      }
      __nv_bfloat16* dst = nullptr;
      if (is_q) {
        dst = p.q_out + ((size_t)t * p.Hq + head) * HD;
      } else if (cached) {
        const int kvh = is_k ? head - p.Hq : head - p.Hq - p.Hkv;
        dst = (is_k ? p.k_pool : p.v_pool) + ((page * p.Hkv + kvh) * p.page_size + off) * (size_t)HD;
      }
      if (dst != nullptr) {
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int q = 0; q < HD / 8; ++q)
          d4[q] = make_uint4(pack_bf16x2(x[8 * q], x[8 * q + 1]), pack_bf16x2(x[8 * q + 2], x[8 * q + 3]),
                             pack_bf16x2(x[8 * q + 4], x[8 * q + 5]), pack_bf16x2(x[8 * q + 6], x[8 * q + 7]));
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tbase, 128);
  }
}

cudaError_t launch_rope_table(const int32_t* pos, int T, const float* inv_freq, int head_dim, float attn_scaling,
                              float* table, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  const long long n = (long long)T * (head_dim / 2);
  const int blocks = (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, 148 * 8));
  rope_table_kernel<<<blocks, 256, 0, stream>>>(pos, T, inv_freq, head_dim / 2, attn_scaling,
                                                reinterpret_cast<float2*>(table));
  return cudaGetLastError();
}

template <int HD>
static cudaError_t launch_qkv_append_hd(const CUtensorMap& xm, const CUtensorMap& wm, const QkvAppendParams& p,
                                        cudaStream_t stream) {
  constexpr int smem = 2 * kQaStages * kQaBox + (int)sizeof(QaBars);
  static std::atomic<int> ready[kMaxDevices];  // the attribute is set once per device
  const int dev = device_slot();
  if (dev < 0 || !ready[dev].load(std::memory_order_acquire)) {
    cudaError_t e = cudaFuncSetAttribute(qkv_append_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0) ready[dev].store(1, std::memory_order_release);
  }
  const dim3 grid((unsigned)((p.T + 127) / 128), (unsigned)(p.N / 128));
  qkv_append_kernel<HD><<<grid, kQaThreads, smem, stream>>>(xm, wm, p);
  return cudaGetLastError();
}

cudaError_t launch_qkv_append(const CUtensorMap& xm, const CUtensorMap& wm, const QkvAppendParams& p,
                              cudaStream_t stream) {
  if (p.T <= 0) return cudaSuccess;
  return p.head_dim == 128 ? launch_qkv_append_hd<128>(xm, wm, p, stream)
                           : launch_qkv_append_hd<64>(xm, wm, p, stream);
}

}  // namespace mb
