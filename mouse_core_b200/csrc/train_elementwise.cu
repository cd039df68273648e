// Element-wise pieces of the packed training layer, forward and backward
// (K4): the decoder layer of flex_packed_forward (flex_train.py:128-150)
// calls transformers modules whose eager bf16 ops each make a pass over HBM;
// these kernels fuse each group into one pass per direction.
//
//  * RMSNorm (Qwen3RMSNorm / LlamaRMSNorm: fp32 variance, x * rsqrt(var + eps)
//    rounded to bf16, then multiplied by the bf16 weight): forward saves the
//    per-row rstd; backward computes dx in fp32 and per-block partial sums of
//    the weight gradient.
//  * the heads of the fused QKV projection: q/k per-head RMSNorm + rotate-half
//    RoPE (Qwen3Attention: q_norm / k_norm on each head, then q * cos +
//    rotate_half(q) * sin with bf16 rounding after each op; Llama applies RoPE
//    without the norm) and v, read straight out of the projection in one
//    pass, with their gradients written back into the fused QKV gradient.
//  * the backward of the SiLU-gated product (Qwen3MLP / LlamaMLP: silu(gate)
//    rounded to bf16, times up) over the [rows, 2I] gate|up projection.
// The forwards repeat the modules' rounding steps; the backwards compute in
// fp32 and round once.
#include "common.cuh"
#include "kernels.h"

namespace mb {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Rounds a pair to bf16 with one packed conversion (the conversion pipe, not
// the memory system, bounds the forwards that round after every op).
__device__ __forceinline__ void bf16r2(float& a, float& b) {
  const float2 r = __bfloat1622float2(__floats2bfloat162_rn(a, b));
  a = r.x;
  b = r.y;
}

// Blocks of `kernel` that fit on the device at once (one full wave).
template <typename K>
static int resident_blocks(K kernel, int threads, int smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, threads, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return per_sm * sms;
}

// ---------------------------------------------------------------- RMSNorm
// One warp per row, rows grid-strided; each lane owns NCH = D / 256 chunks of
// 8 contiguous elements (D a multiple of 256, at most 2048).
template <int NCH>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ res,
                                                          const __nv_bfloat16* __restrict__ w, float eps, int rows,
                                                          __nv_bfloat16* __restrict__ sum,
                                                          __nv_bfloat16* __restrict__ y, float* __restrict__ rstd) {
  constexpr int D = NCH * 256;
  const int lane = threadIdx.x & 31;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    const __nv_bfloat16* xr = x + (size_t)row * D;
    uint4 xv[NCH];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      xv[c] = *reinterpret_cast<const uint4*>(xr + c * 256 + lane * 8);
      if (res != nullptr) {  // the residual add, rounded to bf16 as the module's add is
        const uint4 rv = *reinterpret_cast<const uint4*>(res + off);
        uint32_t* a = reinterpret_cast<uint32_t*>(&xv[c]);
        const uint32_t* b = reinterpret_cast<const uint32_t*>(&rv);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 fa = unpack_bf16x2(a[i]), fb = unpack_bf16x2(b[i]);
          a[i] = pack_bf16x2(fa.x + fb.x, fa.y + fb.y);
        }
        *reinterpret_cast<uint4*>(sum + off) = xv[c];
      }
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&xv[c]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(u[i]);
        ss = fmaf(f.x, f.x, fmaf(f.y, f.y, ss));
      }
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + eps);
    if (lane == 0) rstd[row] = r;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 256 + lane * 8);
      const uint32_t* u = reinterpret_cast<const uint32_t*>(&xv[c]);
      const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = unpack_bf16x2(u[i]), g = unpack_bf16x2(wu[i]);
        ou[i] = pack_bf16x2(g.x * bf16r(f.x * r), g.y * bf16r(f.y * r));
      }
      *reinterpret_cast<uint4*>(y + (size_t)row * D + c * 256 + lane * 8) = o;
    }
  }
}

// dx = rstd * (g - n * mean(g * n)) with g = dy * w and n = x * rstd (fp32);
// the weight gradient sums dy * bf16(n) over rows: each block writes its
// partial sum (one row of `partial`, D floats). A row's dy and x stay in
// registers between the reduction and the dx pass; the weight lives in
// registers for the whole kernel.
constexpr int kNormBwdWarps = 4;

template <int NCH>
__global__ void __launch_bounds__(kNormBwdWarps * 32) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const float* __restrict__ rstd,
                                                          const __nv_bfloat16* __restrict__ dsum, int rows,
                                                          __nv_bfloat16* __restrict__ dx,
                                                          float* __restrict__ partial) {
  constexpr int D = NCH * 256;
  extern __shared__ float red[];  // [warps][D] weight-gradient rows, then the weight [D]
  float* wsm = red + kNormBwdWarps * D;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  // this warp's running weight-gradient sum lives in its row of `red`: lane l
  // owns the 8-float chunks at c * 256 + 8 l
  float* acc = red + warp * D;
#pragma unroll
  for (int c = 0; c < NCH; ++c) {
    float4* a4 = reinterpret_cast<float4*>(acc + c * 256 + lane * 8);
    a4[0] = a4[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int i = threadIdx.x; i < D; i += blockDim.x) wsm[i] = __bfloat162float(w[i]);
  __syncthreads();
#pragma unroll 1
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    const float r = rstd[row];
    uint4 dv[NCH], xv[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      dv[c] = *reinterpret_cast<const uint4*>(dy + off);
      xv[c] = *reinterpret_cast<const uint4*>(x + off);
    }
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t* du = reinterpret_cast<const uint32_t*>(&dv[c]);
      const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv[c]);
      const float2* wf = reinterpret_cast<const float2*>(wsm + c * 256 + lane * 8);
      float4* a4 = reinterpret_cast<float4*>(acc + c * 256 + lane * 8);
      float dw[8];
      *reinterpret_cast<float4*>(dw) = a4[0];
      *reinterpret_cast<float4*>(dw + 4) = a4[1];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 d2 = unpack_bf16x2(du[i]), x2 = unpack_bf16x2(xu[i]), w2 = wf[i];
        float n0 = x2.x * r, n1 = x2.y * r;
        dot = fmaf(d2.x * w2.x, n0, fmaf(d2.y * w2.y, n1, dot));
        bf16r2(n0, n1);
        dw[2 * i] = fmaf(d2.x, n0, dw[2 * i]);
        dw[2 * i + 1] = fmaf(d2.y, n1, dw[2 * i + 1]);
      }
      a4[0] = *reinterpret_cast<const float4*>(dw);
      a4[1] = *reinterpret_cast<const float4*>(dw + 4);
    }
    dot = warp_sum(dot) / (float)D;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const uint32_t* du = reinterpret_cast<const uint32_t*>(&dv[c]);
      const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv[c]);
      const float2* wf = reinterpret_cast<const float2*>(wsm + c * 256 + lane * 8);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
      uint4 sv = make_uint4(0, 0, 0, 0);  // gradient reaching the normalised input directly (residual path)
      if (dsum != nullptr) sv = *reinterpret_cast<const uint4*>(dsum + (size_t)row * D + c * 256 + lane * 8);
      const uint32_t* su = reinterpret_cast<const uint32_t*>(&sv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 d2 = unpack_bf16x2(du[i]), x2 = unpack_bf16x2(xu[i]), w2 = wf[i], s2 = unpack_bf16x2(su[i]);
        ou[i] = pack_bf16x2(r * (d2.x * w2.x - x2.x * r * dot) + s2.x, r * (d2.y * w2.y - x2.y * r * dot) + s2.y);
      }
      *reinterpret_cast<uint4*>(dx + (size_t)row * D + c * 256 + lane * 8) = o;
    }
  }
  // Block-level reduction of the weight gradient.
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) s += red[k * D + j];
    partial[(size_t)blockIdx.x * D + j] = s;
  }
}

// out[j] = sum over p of partial[p][j] for j < split, out2[j - split] for the
// rest: a block owns 32 columns, its 16 warps stride the P partial rows
// (coalesced 128-byte row segments).
__global__ void __launch_bounds__(512) colsum_kernel(const float* __restrict__ partial, int P, int D, int split,
                                                     float* __restrict__ out, float* __restrict__ out2) {
  __shared__ float red[16][33];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int j = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (j < D) {
#pragma unroll 8
    for (int p = warp; p < P; p += 16) s += partial[(size_t)p * D + j];
  }
  red[warp][lane] = s;
  __syncthreads();
  if (warp == 0) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) t += red[k][lane];
    if (j < split) out[j] = t;
    else if (j < D) out2[j - split] = t;
  }
}

static void launch_colsum(const float* partial, int P, int D, int split, float* out, float* out2,
                          cudaStream_t stream) {
  colsum_kernel<<<(D + 31) / 32, 512, 0, stream>>>(partial, P, D, split, out, out2);
}

static int norm_blocks(int rows) { return std::max(1, std::min((rows + 7) / 8, 148 * 4)); }

// One full wave of the backward kernel for dim D (its shared memory holds
// the per-warp weight-gradient rows and the weight), cached per device.
static int norm_bwd_blocks(int rows, int D) {
  static std::atomic<int> cache[kMaxDevices][9];
  const int nch = D / 256;
  if (nch < 1 || nch > 8) return 1;
  const int dev = device_slot();
  int cap[9] = {0};
  if (dev >= 0) cap[nch] = cache[dev][nch].load(std::memory_order_relaxed);
  if (!cap[nch]) {
    const int smem = (kNormBwdWarps + 1) * D * (int)sizeof(float);
    switch (nch) {
#define MB_CAP(N)                                                                                          \
  case N:                                                                                                  \
    cudaFuncSetAttribute(rmsnorm_bwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);       \
    cap[N] = resident_blocks(rmsnorm_bwd_kernel<N>, kNormBwdWarps * 32, smem);                                            \
    break;
      MB_CAP(1) MB_CAP(2) MB_CAP(3) MB_CAP(4) MB_CAP(5) MB_CAP(6) MB_CAP(7) MB_CAP(8)
#undef MB_CAP
    }
    if (dev >= 0) cache[dev][nch].store(cap[nch], std::memory_order_relaxed);
  }
  return std::max(1, std::min((rows + kNormBwdWarps - 1) / kNormBwdWarps, cap[nch]));
}

#define MB_NORM_DISPATCH(NCH_RT, CALL) \
  switch (NCH_RT) {                    \
    case 1: CALL(1); break;            \
    case 2: CALL(2); break;            \
    case 3: CALL(3); break;            \
    case 4: CALL(4); break;            \
    case 5: CALL(5); break;            \
    case 6: CALL(6); break;            \
    case 7: CALL(7); break;            \
    case 8: CALL(8); break;            \
    default: return cudaErrorInvalidValue; \
  }

cudaError_t launch_rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* res, const __nv_bfloat16* w, float eps,
                               int rows, int D, __nv_bfloat16* sum, __nv_bfloat16* y, float* rstd,
                               cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int blocks = norm_blocks(rows);
#define MB_FWD(N) rmsnorm_fwd_kernel<N><<<blocks, 256, 0, stream>>>(x, res, w, eps, rows, sum, y, rstd)
  MB_NORM_DISPATCH(D / 256, MB_FWD)
#undef MB_FWD
  return cudaGetLastError();
}

int rmsnorm_bwd_partials(int rows, int D) { return norm_bwd_blocks(rows, D); }

cudaError_t launch_rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w,
                               const float* rstd, const __nv_bfloat16* dsum, int rows, int D, __nv_bfloat16* dx,
                               float* partial, float* dw, cudaStream_t stream) {
  if (rows <= 0) {
    cudaMemsetAsync(dw, 0, sizeof(float) * D, stream);
    return cudaGetLastError();
  }
  const int blocks = norm_bwd_blocks(rows, D);
  const int smem = (kNormBwdWarps + 1) * D * (int)sizeof(float);
  cudaError_t e = cudaSuccess;
#define MB_BWD(N)                                                                                          \
  do {                                                                                                     \
    e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);  \
    if (e == cudaSuccess) rmsnorm_bwd_kernel<N><<<blocks, kNormBwdWarps * 32, smem, stream>>>(dy, x, w, rstd, dsum, rows, dx, partial); \
  } while (0)
  MB_NORM_DISPATCH(D / 256, MB_BWD)
#undef MB_BWD
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  launch_colsum(partial, blocks, D, D, dw, nullptr, stream);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- fused QKV heads
// One warp per token over the token's Hq + 2 Hkv heads of the fused QKV
// projection (row stride xs): q heads and k heads through the optional
// per-head RMSNorm and rotate-half RoPE, v heads copied. Each lane owns 8
// contiguous elements (one 16-byte access) of one head: LPH = HD / 8 lanes
// per head, HPW = 32 / LPH heads per warp access. A lane's rotate-half
// partner is lane ^ (LPH / 2) and a head's norm reduction stays inside its
// LPH-lane group, so every lane runs the same shuffles whatever the role of
// its head (roles only select what is stored). Heads are taken kChunk
// accesses at a time with all loads issued before the arithmetic.
template <int HD>
struct QkvGeom {
  static constexpr int LPH = HD / 8;
  static constexpr int HPW = 32 / LPH;
};

__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  const uint32_t* u = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 a = unpack_bf16x2(u[i]);
    f[2 * i] = a.x;
    f[2 * i + 1] = a.y;
  }
}

__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  return make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]), pack_bf16x2(f[4], f[5]),
                    pack_bf16x2(f[6], f[7]));
}

template <int LPH>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
  for (int o = LPH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct QkvFwdArgs {
  const __nv_bfloat16* qkv;
  long long xs;
  const __nv_bfloat16* qw;  // [HD] or null (no per-head norm)
  const __nv_bfloat16* kw;
  float q_eps, k_eps;
  const __nv_bfloat16* cosv;  // [L, HD]
  const __nv_bfloat16* sinv;
  int L, Hq, Hkv;
  __nv_bfloat16* q;  // [L, Hq, HD]
  __nv_bfloat16* k;  // [L, Hkv, HD]
  __nv_bfloat16* v;  // [L, Hkv, HD]
  float* q_rstd;     // [L * Hq] (with the norm)
  float* k_rstd;     // [L * Hkv]
};

template <int HD>
__global__ void __launch_bounds__(256) qkv_heads_fwd_kernel(QkvFwdArgs a) {
  constexpr int LPH = QkvGeom<HD>::LPH, HPW = QkvGeom<HD>::HPW, kChunk = 8;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPH, j = (lane % LPH) * 8;
  const bool lo = (lane % LPH) < LPH / 2;  // holds elements of the first half
  const int T = a.Hq + 2 * a.Hkv;
  const int accesses = (T + HPW - 1) / HPW;
  const bool norm = a.qw != nullptr;
  float qw[8], kw[8];
  if (norm) {
    unpack8(*reinterpret_cast<const uint4*>(a.qw + j), qw);
    unpack8(*reinterpret_cast<const uint4*>(a.kw + j), kw);
  }
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < a.L; t += warps) {
    float c[8], sn[8];
    unpack8(*reinterpret_cast<const uint4*>(a.cosv + (size_t)t * HD + j), c);
    unpack8(*reinterpret_cast<const uint4*>(a.sinv + (size_t)t * HD + j), sn);
    const __nv_bfloat16* row = a.qkv + (long long)t * a.xs;
    for (int a0 = 0; a0 < accesses; a0 += kChunk) {
      uint4 xv[kChunk];
#pragma unroll
      for (int u = 0; u < kChunk; ++u) {
        const int h = (a0 + u) * HPW + sub;
        if (a0 + u < accesses && h < T) xv[u] = *reinterpret_cast<const uint4*>(row + h * HD + j);
      }
#pragma unroll
      for (int u = 0; u < kChunk; ++u) {
        if (a0 + u >= accesses) break;  // warp-uniform
        const int h = (a0 + u) * HPW + sub;
        const bool live = h < T;
        const bool is_q = h < a.Hq, is_k = !is_q && h < a.Hq + a.Hkv;
        float x[8];
        if (live) unpack8(xv[u], x);
        else
#pragma unroll
          for (int i = 0; i < 8; ++i) x[i] = 0.f;
        if (norm) {
          float ss = 0.f;
#pragma unroll
          for (int i = 0; i < 8; ++i) ss = fmaf(x[i], x[i], ss);
          ss = group_sum<LPH>(ss);
          const float eps = is_q ? a.q_eps : a.k_eps;
          const float r = rsqrtf(ss / (float)HD + eps);
          if (live && (lane % LPH) == 0 && (is_q || is_k)) {
            if (is_q) a.q_rstd[(size_t)t * a.Hq + h] = r;
            else a.k_rstd[(size_t)t * a.Hkv + (h - a.Hq)] = r;
          }
          if (is_q || is_k) {
#pragma unroll
            for (int i = 0; i < 8; i += 2) {
              float n0 = x[i] * r, n1 = x[i + 1] * r;
              bf16r2(n0, n1);
              n0 *= is_q ? qw[i] : kw[i];
              n1 *= is_q ? qw[i + 1] : kw[i + 1];
              bf16r2(n0, n1);
              x[i] = n0;
              x[i + 1] = n1;
            }
          }
        }
        float o[8];
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          const float p0 = __shfl_xor_sync(0xffffffffu, x[i], LPH / 2);
          const float p1 = __shfl_xor_sync(0xffffffffu, x[i + 1], LPH / 2);
          float a0 = x[i] * c[i], a1 = x[i + 1] * c[i + 1];
          float b0 = (lo ? -p0 : p0) * sn[i], b1 = (lo ? -p1 : p1) * sn[i + 1];
          bf16r2(a0, a1);
          bf16r2(b0, b1);
          o[i] = a0 + b0;  // rounded once more by the store's pack
          o[i + 1] = a1 + b1;
        }
        if (!live) continue;
        if (is_q) {
          *reinterpret_cast<uint4*>(a.q + ((size_t)t * a.Hq + h) * HD + j) = pack8(o);
        } else if (is_k) {
          *reinterpret_cast<uint4*>(a.k + ((size_t)t * a.Hkv + (h - a.Hq)) * HD + j) = pack8(o);
        } else {
          *reinterpret_cast<uint4*>(a.v + ((size_t)t * a.Hkv + (h - a.Hq - a.Hkv)) * HD + j) = xv[u];
        }
      }
    }
  }
}

struct QkvBwdArgs {
  const __nv_bfloat16* dq;  // [L, Hq, HD]
  const __nv_bfloat16* dk;  // [L, Hkv, HD]
  const __nv_bfloat16* dv;  // [L, Hkv, HD]
  const __nv_bfloat16* qkv;
  long long xs;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  const __nv_bfloat16* cosv;
  const __nv_bfloat16* sinv;
  const float* q_rstd;
  const float* k_rstd;
  int L, Hq, Hkv;
  __nv_bfloat16* dqkv;
  long long dxs;
  float* partial;  // [gridDim.x][2 * HD] (q_norm | k_norm weight-gradient partials)
};

// dn = dy * cos + rotate_half^T(dy * sin); with the norm, dx = rstd * (g - n *
// mean(g * n)) with g = dn * w, n = x * rstd, and the weight gradient sums
// dn * bf16(n). v heads pass their gradient through.
template <int HD>
__global__ void __launch_bounds__(256, 2) qkv_heads_bwd_kernel(QkvBwdArgs a) {
  constexpr int LPH = QkvGeom<HD>::LPH, HPW = QkvGeom<HD>::HPW, kChunk = 4;
  __shared__ float red[8][2][HD];
  __shared__ __align__(16) float wsm[2][HD];  // q_norm | k_norm weights
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int sub = lane / LPH, j = (lane % LPH) * 8;
  const bool lo = (lane % LPH) < LPH / 2;
  const int T = a.Hq + 2 * a.Hkv;
  const int accesses = (T + HPW - 1) / HPW;
  const bool norm = a.qw != nullptr;
  float dwq[8], dwk[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) dwq[i] = dwk[i] = 0.f;
  if (norm) {
    for (int i = threadIdx.x; i < 2 * HD; i += blockDim.x)
      wsm[i / HD][i % HD] = __bfloat162float((i < HD ? a.qw : a.kw)[i % HD]);
  }
  __syncthreads();
  const int warps = (gridDim.x * blockDim.x) >> 5;
  for (int t = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; t < a.L; t += warps) {
    float c[8], sn[8];
    unpack8(*reinterpret_cast<const uint4*>(a.cosv + (size_t)t * HD + j), c);
    unpack8(*reinterpret_cast<const uint4*>(a.sinv + (size_t)t * HD + j), sn);
    const __nv_bfloat16* row = a.qkv + (long long)t * a.xs;
    __nv_bfloat16* drow = a.dqkv + (long long)t * a.dxs;
    for (int a0 = 0; a0 < accesses; a0 += kChunk) {
      uint4 dv[kChunk], xv[kChunk];
      float r[kChunk];
#pragma unroll
      for (int u = 0; u < kChunk; ++u) {
        const int h = (a0 + u) * HPW + sub;
        if (a0 + u < accesses && h < T) {
          if (h < a.Hq) {
            dv[u] = *reinterpret_cast<const uint4*>(a.dq + ((size_t)t * a.Hq + h) * HD + j);
            if (norm) r[u] = a.q_rstd[(size_t)t * a.Hq + h];
          } else if (h < a.Hq + a.Hkv) {
            dv[u] = *reinterpret_cast<const uint4*>(a.dk + ((size_t)t * a.Hkv + (h - a.Hq)) * HD + j);
            if (norm) r[u] = a.k_rstd[(size_t)t * a.Hkv + (h - a.Hq)];
          } else {
            dv[u] = *reinterpret_cast<const uint4*>(a.dv + ((size_t)t * a.Hkv + (h - a.Hq - a.Hkv)) * HD + j);
          }
          if (norm && h < a.Hq + a.Hkv) xv[u] = *reinterpret_cast<const uint4*>(row + h * HD + j);
        }
      }
#pragma unroll
      for (int u = 0; u < kChunk; ++u) {
        if (a0 + u >= accesses) break;  // warp-uniform
        const int h = (a0 + u) * HPW + sub;
        const bool live = h < T;
        const bool is_q = h < a.Hq, is_k = !is_q && h < a.Hq + a.Hkv;
        const bool rope = live && (is_q || is_k);
        float d[8];
        if (live) unpack8(dv[u], d);
        else
#pragma unroll
          for (int i = 0; i < 8; ++i) d[i] = 0.f;
        float out[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float p = __shfl_xor_sync(0xffffffffu, d[i] * sn[i], LPH / 2);
          out[i] = d[i] * c[i] + (lo ? p : -p);
        }
        if (norm) {
          float n[8], g[8], dot = 0.f;
          float x[8];
          if (rope) unpack8(xv[u], x);
          else
#pragma unroll
            for (int i = 0; i < 8; ++i) x[i] = 0.f;
          const float rr = rope ? r[u] : 0.f;
          const float4* wr = reinterpret_cast<const float4*>(&wsm[is_q ? 0 : 1][j]);
          const float4 w0 = wr[0], w1 = wr[1];
          const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            n[i] = x[i] * rr;
            g[i] = out[i] * wv[i];
            dot = fmaf(g[i], n[i], dot);
          }
          dot = group_sum<LPH>(dot) / (float)HD;
          if (rope) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              if (is_q) dwq[i] = fmaf(out[i], bf16r(n[i]), dwq[i]);
              else dwk[i] = fmaf(out[i], bf16r(n[i]), dwk[i]);
              out[i] = rr * (g[i] - n[i] * dot);
            }
          }
        }
        if (!live) continue;
        *reinterpret_cast<uint4*>(drow + h * HD + j) = rope ? pack8(out) : dv[u];
      }
    }
  }
  if (a.partial) {
    // lanes with the same element offset j (one per head slot) and all warps
    // of the block sum into one partial row of 2 * HD floats
#pragma unroll
    for (int s2 = 0; s2 < HPW; ++s2) {
      if (sub == s2) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          red[warp][0][j + i] = (s2 == 0 ? 0.f : red[warp][0][j + i]) + dwq[i];
          red[warp][1][j + i] = (s2 == 0 ? 0.f : red[warp][1][j + i]) + dwk[i];
        }
      }
      __syncwarp();
    }
    __syncthreads();
    for (int col = threadIdx.x; col < 2 * HD; col += blockDim.x) {
      float s = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w][col / HD][col % HD];
      a.partial[(size_t)blockIdx.x * 2 * HD + col] = s;
    }
  }
}

static int qkv_blocks(int L, int HD, bool bwd) {
  static int cap[2][2] = {{0, 0}, {0, 0}};
  const int hi = HD == 128, b = bwd;
  if (!cap[b][hi]) {
    if (bwd) cap[b][hi] = hi ? resident_blocks(qkv_heads_bwd_kernel<128>, 256, 0)
                             : resident_blocks(qkv_heads_bwd_kernel<64>, 256, 0);
    else cap[b][hi] = hi ? resident_blocks(qkv_heads_fwd_kernel<128>, 256, 0)
                         : resident_blocks(qkv_heads_fwd_kernel<64>, 256, 0);
  }
  return std::max(1, std::min((L + 7) / 8, cap[b][hi]));
}

int qkv_heads_bwd_partials(int L, int HD) { return qkv_blocks(L, HD, true); }

cudaError_t launch_qkv_heads_fwd(const __nv_bfloat16* qkv, long long xs, int L, int Hq, int Hkv, int HD,
                                 const __nv_bfloat16* qw, const __nv_bfloat16* kw, float q_eps, float k_eps,
                                 const __nv_bfloat16* cosv, const __nv_bfloat16* sinv, __nv_bfloat16* q,
                                 __nv_bfloat16* k, __nv_bfloat16* v, float* q_rstd, float* k_rstd,
                                 cudaStream_t stream) {
  if (L <= 0) return cudaSuccess;
  const QkvFwdArgs a{qkv, xs, qw, kw, q_eps, k_eps, cosv, sinv, L, Hq, Hkv, q, k, v, q_rstd, k_rstd};
  if (HD == 128) qkv_heads_fwd_kernel<128><<<qkv_blocks(L, 128, false), 256, 0, stream>>>(a);
  else qkv_heads_fwd_kernel<64><<<qkv_blocks(L, 64, false), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_qkv_heads_bwd(const __nv_bfloat16* dq, const __nv_bfloat16* dk, const __nv_bfloat16* dv,
                                 const __nv_bfloat16* qkv, long long xs, int L, int Hq, int Hkv, int HD,
                                 const __nv_bfloat16* qw, const __nv_bfloat16* kw, const __nv_bfloat16* cosv,
                                 const __nv_bfloat16* sinv, const float* q_rstd, const float* k_rstd,
                                 __nv_bfloat16* dqkv, long long dxs, float* dqw, float* dkw, float* partial,
                                 cudaStream_t stream) {
  const bool norm = qw != nullptr;
  if (L <= 0) {
    if (norm) {
      cudaMemsetAsync(dqw, 0, sizeof(float) * HD, stream);
      cudaMemsetAsync(dkw, 0, sizeof(float) * HD, stream);
    }
    return cudaGetLastError();
  }
  const int blocks = qkv_blocks(L, HD, true);
  const QkvBwdArgs a{dq, dk, dv, qkv, xs, qw, kw, cosv, sinv, q_rstd, k_rstd, L, Hq, Hkv, dqkv, dxs,
                     norm ? partial : nullptr};
  if (HD == 128) qkv_heads_bwd_kernel<128><<<blocks, 256, 0, stream>>>(a);
  else qkv_heads_bwd_kernel<64><<<blocks, 256, 0, stream>>>(a);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !norm) return e;
  launch_colsum(partial, blocks, 2 * HD, HD, dqw, dkw, stream);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- SiLU-gated product
// gu = [rows, 2I] (gate | up). The forward h = bf16(bf16(silu(g)) * u) is
// launch_silu_mul (elementwise.cu); backward dg = dh * u * silu'(g),
// du = dh * bf16(silu(g)). Vector path: 8 elements (16 bytes) per thread,
// blockIdx.y strides rows; otherwise pairs of elements.
__device__ __forceinline__ void silu_bwd2(float g, float u, float d, float& dg, float& du) {
  const float s = 1.f / (1.f + expf(-g));
  dg = d * u * s * (1.f + g * (1.f - s));
  du = d * bf16r(g * s);
}

__global__ void __launch_bounds__(128) silu_mul_bwd_vec_kernel(const __nv_bfloat16* __restrict__ gu,
                                                               const __nv_bfloat16* __restrict__ dh, int rows, int I,
                                                               __nv_bfloat16* __restrict__ dgu) {
  const int vpr = I >> 3;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= vpr) return;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const size_t gbase = (size_t)row * 2 * I + (size_t)c * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + gbase);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + gbase + I);
    const uint4 dv = *reinterpret_cast<const uint4*>(dh + (size_t)row * I + (size_t)c * 8);
    const uint32_t* g2 = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* u2 = reinterpret_cast<const uint32_t*>(&uv);
    const uint32_t* d2 = reinterpret_cast<const uint32_t*>(&dv);
    uint4 og, ou;
    uint32_t* og2 = reinterpret_cast<uint32_t*>(&og);
    uint32_t* ou2 = reinterpret_cast<uint32_t*>(&ou);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 g = unpack_bf16x2(g2[i]), u = unpack_bf16x2(u2[i]), d = unpack_bf16x2(d2[i]);
      float dg0, du0, dg1, du1;
      silu_bwd2(g.x, u.x, d.x, dg0, du0);
      silu_bwd2(g.y, u.y, d.y, dg1, du1);
      og2[i] = pack_bf16x2(dg0, dg1);
      ou2[i] = pack_bf16x2(du0, du1);
    }
    *reinterpret_cast<uint4*>(dgu + gbase) = og;
    *reinterpret_cast<uint4*>(dgu + gbase + I) = ou;
  }
}

__global__ void silu_mul_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                    int rows, int I, __nv_bfloat16* __restrict__ dgu) {
  const int ppr = I >> 1;
  for (int row = blockIdx.y; row < rows; row += gridDim.y)
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < ppr; c += gridDim.x * blockDim.x) {
      const size_t gbase = (size_t)row * 2 * I + (size_t)c * 2;
      const float2 g = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + gbase));
      const float2 u = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + gbase + I));
      const float2 d = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dh + (size_t)row * I + (size_t)c * 2));
      float dg0, du0, dg1, du1;
      silu_bwd2(g.x, u.x, d.x, dg0, du0);
      silu_bwd2(g.y, u.y, d.y, dg1, du1);
      *reinterpret_cast<uint32_t*>(dgu + gbase) = pack_bf16x2(dg0, dg1);
      *reinterpret_cast<uint32_t*>(dgu + gbase + I) = pack_bf16x2(du0, du1);
    }
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

cudaError_t launch_silu_mul_bwd(const __nv_bfloat16* gu, const __nv_bfloat16* dh, int rows, int I,
                                __nv_bfloat16* dgu, cudaStream_t stream) {
  if (rows <= 0 || I <= 0) return cudaSuccess;
  const int by = std::min(rows, 65535);
  if (I % 8 == 0 && aligned16(gu) && aligned16(dh) && aligned16(dgu)) {
    const dim3 grid((unsigned)((I / 8 + 127) / 128), (unsigned)by);
    silu_mul_bwd_vec_kernel<<<grid, 128, 0, stream>>>(gu, dh, rows, I, dgu);
  } else {
    const dim3 grid((unsigned)std::min((I / 2 + 127) / 128, 64), (unsigned)by);
    silu_mul_bwd_kernel<<<grid, 128, 0, stream>>>(gu, dh, rows, I, dgu);
  }
  return cudaGetLastError();
}

}  // namespace mb
