// Element-wise pieces of the packed training layer, forward and backward
// (K4): the decoder layer of flex_packed_forward (flex_train.py:128-150)
// calls transformers modules whose eager bf16 ops each make a pass over HBM;
// these kernels fuse each group into one pass per direction.
//
//  * RMSNorm (Qwen3RMSNorm / LlamaRMSNorm: fp32 variance, x * rsqrt(var + eps)
//    rounded to bf16, then multiplied by the bf16 weight): forward saves the
//    per-row rstd; backward computes dx in fp32 and per-block partial sums of
//    the weight gradient.
//  * q/k per-head RMSNorm + rotate-half RoPE (Qwen3Attention: q_norm / k_norm
//    on each head, then q * cos + rotate_half(q) * sin with bf16 rounding after
//    each op; Llama applies RoPE without the norm), reading q or k straight
//    out of the fused QKV projection and writing their gradients back into it.
//  * the backward of the SiLU-gated product (Qwen3MLP / LlamaMLP: silu(gate)
//    rounded to bf16, times up) over the [rows, 2I] gate|up projection.
// The forwards repeat the modules' rounding steps; the backwards compute in
// fp32 and round once.
#include "common.cuh"
#include "kernels.h"

namespace mb {

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// ---------------------------------------------------------------- RMSNorm
// One warp per row, rows grid-strided; each lane owns NCH = D / 256 chunks of
// 8 contiguous elements (D a multiple of 256, at most 2048).
template <int NCH>
__global__ void __launch_bounds__(256) rmsnorm_fwd_kernel(const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w, float eps, int rows,
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
      xv[c] = *reinterpret_cast<const uint4*>(xr + c * 256 + lane * 8);
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
// partial sum (one row of `partial`, D floats). Two passes over the row: the
// first forms mean(g * n) and the weight gradient, the second (from L1) dx.
template <int NCH>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                          const __nv_bfloat16* __restrict__ x,
                                                          const __nv_bfloat16* __restrict__ w,
                                                          const float* __restrict__ rstd, int rows,
                                                          __nv_bfloat16* __restrict__ dx,
                                                          float* __restrict__ partial) {
  constexpr int D = NCH * 256;
  extern __shared__ float red[];  // [8 warps][D]
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int warps = (gridDim.x * blockDim.x) >> 5;
  float dw[NCH][8];
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) dw[c][i] = 0.f;
  for (int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; row < rows; row += warps) {
    const float r = rstd[row];
    float dot = 0.f;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      const uint4 dv = *reinterpret_cast<const uint4*>(dy + off);
      const uint4 xv = *reinterpret_cast<const uint4*>(x + off);
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 256 + lane * 8);
      const uint32_t* du = reinterpret_cast<const uint32_t*>(&dv);
      const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv);
      const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 d2 = unpack_bf16x2(du[i]), x2 = unpack_bf16x2(xu[i]), w2 = unpack_bf16x2(wu[i]);
        const float n0 = x2.x * r, n1 = x2.y * r;
        dot = fmaf(d2.x * w2.x, n0, fmaf(d2.y * w2.y, n1, dot));
        dw[c][2 * i] = fmaf(d2.x, bf16r(n0), dw[c][2 * i]);
        dw[c][2 * i + 1] = fmaf(d2.y, bf16r(n1), dw[c][2 * i + 1]);
      }
    }
    dot = warp_sum(dot) / (float)D;
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const size_t off = (size_t)row * D + c * 256 + lane * 8;
      const uint4 dv = *reinterpret_cast<const uint4*>(dy + off);
      const uint4 xv = *reinterpret_cast<const uint4*>(x + off);
      const uint4 wv = *reinterpret_cast<const uint4*>(w + c * 256 + lane * 8);
      const uint32_t* du = reinterpret_cast<const uint32_t*>(&dv);
      const uint32_t* xu = reinterpret_cast<const uint32_t*>(&xv);
      const uint32_t* wu = reinterpret_cast<const uint32_t*>(&wv);
      uint4 o;
      uint32_t* ou = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 d2 = unpack_bf16x2(du[i]), x2 = unpack_bf16x2(xu[i]), w2 = unpack_bf16x2(wu[i]);
        ou[i] = pack_bf16x2(r * (d2.x * w2.x - x2.x * r * dot), r * (d2.y * w2.y - x2.y * r * dot));
      }
      *reinterpret_cast<uint4*>(dx + off) = o;
    }
  }
  // Block-level reduction of the weight gradient.
#pragma unroll
  for (int c = 0; c < NCH; ++c)
#pragma unroll
    for (int i = 0; i < 8; ++i) red[warp * D + c * 256 + lane * 8 + i] = dw[c][i];
  __syncthreads();
  for (int j = threadIdx.x; j < D; j += blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < (int)(blockDim.x >> 5); ++k) s += red[k * D + j];
    partial[(size_t)blockIdx.x * D + j] = s;
  }
}

// out[j] = sum over p of partial[p][j].
__global__ void colsum_kernel(const float* __restrict__ partial, int P, int D, float* __restrict__ out) {
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < D; j += gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < P; ++k) s += partial[(size_t)k * D + j];
    out[j] = s;
  }
}

static int norm_blocks(int rows) { return std::max(1, std::min((rows + 7) / 8, 148 * 4)); }

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

cudaError_t launch_rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* w, float eps, int rows, int D,
                               __nv_bfloat16* y, float* rstd, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int blocks = norm_blocks(rows);
#define MB_FWD(N) rmsnorm_fwd_kernel<N><<<blocks, 256, 0, stream>>>(x, w, eps, rows, y, rstd)
  MB_NORM_DISPATCH(D / 256, MB_FWD)
#undef MB_FWD
  return cudaGetLastError();
}

int rmsnorm_bwd_partials(int rows) { return norm_blocks(rows); }

cudaError_t launch_rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w,
                               const float* rstd, int rows, int D, __nv_bfloat16* dx, float* partial, float* dw,
                               cudaStream_t stream) {
  if (rows <= 0) {
    cudaMemsetAsync(dw, 0, sizeof(float) * D, stream);
    return cudaGetLastError();
  }
  const int blocks = norm_blocks(rows);
  const int smem = 8 * D * (int)sizeof(float);
  cudaError_t e = cudaSuccess;
#define MB_BWD(N)                                                                                          \
  do {                                                                                                     \
    e = cudaFuncSetAttribute(rmsnorm_bwd_kernel<N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);  \
    if (e == cudaSuccess) rmsnorm_bwd_kernel<N><<<blocks, 256, smem, stream>>>(dy, x, w, rstd, rows, dx, partial); \
  } while (0)
  MB_NORM_DISPATCH(D / 256, MB_BWD)
#undef MB_BWD
  if (e != cudaSuccess) return e;
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  colsum_kernel<<<(D + 255) / 256, 256, 0, stream>>>(partial, blocks, D, dw);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- q/k norm + RoPE
// One warp per (token, head); lane l holds elements [EPL*l, EPL*l + EPL) of
// the HD-element head (EPL = HD / 32) and rotate-half partners sit in lane
// l ^ 16. x rows are `xs` elements apart (a slice of the fused QKV output).
template <int HD>
__global__ void __launch_bounds__(256) qk_norm_rope_fwd_kernel(const __nv_bfloat16* __restrict__ x, long long xs,
                                                               const __nv_bfloat16* __restrict__ w, float eps,
                                                               const __nv_bfloat16* __restrict__ cosv,
                                                               const __nv_bfloat16* __restrict__ sinv, int L, int H,
                                                               __nv_bfloat16* __restrict__ y,
                                                               float* __restrict__ rstd) {
  constexpr int EPL = HD / 32;
  const int lane = threadIdx.x & 31;
  const long long items = (long long)L * H;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long it = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < items; it += warps) {
    const long long tok = it / H;
    const int h = (int)(it % H);
    const __nv_bfloat16* xr = x + tok * xs + (long long)h * HD + lane * EPL;
    float v[EPL];
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      const float2 f = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(xr + i));
      v[i] = f.x;
      v[i + 1] = f.y;
    }
    if (w) {
      float ss = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; ++i) ss = fmaf(v[i], v[i], ss);
      ss = warp_sum(ss);
      const float r = rsqrtf(ss / (float)HD + eps);
      if (lane == 0) rstd[it] = r;
#pragma unroll
      for (int i = 0; i < EPL; ++i) v[i] = bf16r(__bfloat162float(w[lane * EPL + i]) * bf16r(v[i] * r));
    }
    float o[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[i], 16);
      const float rh = lane < 16 ? -partner : partner;
      const int d = lane * EPL + i;
      const float c = __bfloat162float(cosv[tok * HD + d]), s = __bfloat162float(sinv[tok * HD + d]);
      o[i] = bf16r(bf16r(v[i] * c) + bf16r(rh * s));
    }
    __nv_bfloat16* yr = y + it * HD + lane * EPL;
#pragma unroll
    for (int i = 0; i < EPL; i += 2) *reinterpret_cast<uint32_t*>(yr + i) = pack_bf16x2(o[i], o[i + 1]);
  }
}

// Gradient of the above: dn = dy * cos + rotate_half^T(dy * sin); with the
// norm, dx = rstd * (g - n * mean(g * n)) with g = dn * w, n = x * rstd, and
// the weight gradient sums dn * bf16(n) (per-block partials of HD floats).
template <int HD>
__global__ void __launch_bounds__(256) qk_norm_rope_bwd_kernel(const __nv_bfloat16* __restrict__ dy,
                                                               const __nv_bfloat16* __restrict__ x, long long xs,
                                                               const __nv_bfloat16* __restrict__ w,
                                                               const __nv_bfloat16* __restrict__ cosv,
                                                               const __nv_bfloat16* __restrict__ sinv,
                                                               const float* __restrict__ rstd, int L, int H,
                                                               __nv_bfloat16* __restrict__ dx, long long dxs,
                                                               float* __restrict__ partial) {
  constexpr int EPL = HD / 32;
  __shared__ float red[8][HD];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const long long items = (long long)L * H;
  const long long warps = ((long long)gridDim.x * blockDim.x) >> 5;
  float dw[EPL];
#pragma unroll
  for (int i = 0; i < EPL; ++i) dw[i] = 0.f;
  for (long long it = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5; it < items; it += warps) {
    const long long tok = it / H;
    const int h = (int)(it % H);
    const __nv_bfloat16* dyr = dy + it * HD + lane * EPL;
    float dn[EPL];
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      const float2 d2 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dyr + i));
      const int d = lane * EPL + i;
      const float2 c2 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(cosv + tok * HD + d));
      const float2 s2 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(sinv + tok * HD + d));
      // dn_j = dy_j cos_j + (j < HD/2 ? (dy sin)_{j+HD/2} : -(dy sin)_{j-HD/2})
      const float ds0 = d2.x * s2.x, ds1 = d2.y * s2.y;
      const float p0 = __shfl_xor_sync(0xffffffffu, ds0, 16), p1 = __shfl_xor_sync(0xffffffffu, ds1, 16);
      dn[i] = d2.x * c2.x + (lane < 16 ? p0 : -p0);
      dn[i + 1] = d2.y * c2.y + (lane < 16 ? p1 : -p1);
    }
    float out[EPL];
    if (w) {
      const float r = rstd[it];
      const __nv_bfloat16* xr = x + tok * xs + (long long)h * HD + lane * EPL;
      float n[EPL], g[EPL];
      float dot = 0.f;
#pragma unroll
      for (int i = 0; i < EPL; i += 2) {
        const float2 x2 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(xr + i));
        n[i] = x2.x * r;
        n[i + 1] = x2.y * r;
      }
#pragma unroll
      for (int i = 0; i < EPL; ++i) {
        g[i] = dn[i] * __bfloat162float(w[lane * EPL + i]);
        dot = fmaf(g[i], n[i], dot);
        dw[i] = fmaf(dn[i], bf16r(n[i]), dw[i]);
      }
      dot = warp_sum(dot) / (float)HD;
#pragma unroll
      for (int i = 0; i < EPL; ++i) out[i] = r * (g[i] - n[i] * dot);
    } else {
#pragma unroll
      for (int i = 0; i < EPL; ++i) out[i] = dn[i];
    }
    __nv_bfloat16* dxr = dx + tok * dxs + (long long)h * HD + lane * EPL;
#pragma unroll
    for (int i = 0; i < EPL; i += 2) *reinterpret_cast<uint32_t*>(dxr + i) = pack_bf16x2(out[i], out[i + 1]);
  }
  if (partial) {
#pragma unroll
    for (int i = 0; i < EPL; ++i) red[warp][lane * EPL + i] = dw[i];
    __syncthreads();
    for (int j = threadIdx.x; j < HD; j += blockDim.x) {
      float s = 0.f;
      for (int k = 0; k < (int)(blockDim.x >> 5); ++k) s += red[k][j];
      partial[(size_t)blockIdx.x * HD + j] = s;
    }
  }
}

static int head_blocks(long long items) { return (int)std::max<long long>(1, std::min<long long>((items + 7) / 8, 148 * 8)); }

int qk_norm_rope_bwd_partials(int L, int H) { return head_blocks((long long)L * H); }

cudaError_t launch_qk_norm_rope_fwd(const __nv_bfloat16* x, long long xs, const __nv_bfloat16* w, float eps,
                                    const __nv_bfloat16* cosv, const __nv_bfloat16* sinv, int L, int H, int HD,
                                    __nv_bfloat16* y, float* rstd, cudaStream_t stream) {
  const long long items = (long long)L * H;
  if (items <= 0) return cudaSuccess;
  if (HD == 128)
    qk_norm_rope_fwd_kernel<128><<<head_blocks(items), 256, 0, stream>>>(x, xs, w, eps, cosv, sinv, L, H, y, rstd);
  else
    qk_norm_rope_fwd_kernel<64><<<head_blocks(items), 256, 0, stream>>>(x, xs, w, eps, cosv, sinv, L, H, y, rstd);
  return cudaGetLastError();
}

cudaError_t launch_qk_norm_rope_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, long long xs,
                                    const __nv_bfloat16* w, const __nv_bfloat16* cosv, const __nv_bfloat16* sinv,
                                    const float* rstd, int L, int H, int HD, __nv_bfloat16* dx, long long dxs,
                                    float* partial, float* dw, cudaStream_t stream) {
  const long long items = (long long)L * H;
  if (items <= 0) {
    if (dw) cudaMemsetAsync(dw, 0, sizeof(float) * HD, stream);
    return cudaGetLastError();
  }
  const int blocks = head_blocks(items);
  float* part = w ? partial : nullptr;
  if (HD == 128)
    qk_norm_rope_bwd_kernel<128><<<blocks, 256, 0, stream>>>(dy, x, xs, w, cosv, sinv, rstd, L, H, dx, dxs, part);
  else
    qk_norm_rope_bwd_kernel<64><<<blocks, 256, 0, stream>>>(dy, x, xs, w, cosv, sinv, rstd, L, H, dx, dxs, part);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess || !w) return e;
  colsum_kernel<<<1, 128, 0, stream>>>(partial, blocks, HD, dw);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- SiLU-gated product
// gu = [rows, 2I] (gate | up). The forward h = bf16(bf16(silu(g)) * u) is
// launch_silu_mul (elementwise.cu); backward dg = dh * u * silu'(g),
// du = dh * bf16(silu(g)).
__global__ void silu_mul_bwd_kernel(const __nv_bfloat16* __restrict__ gu, const __nv_bfloat16* __restrict__ dh,
                                    int I, long long pairs, __nv_bfloat16* __restrict__ dgu) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < pairs;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = (i * 2) / I, col = (i * 2) % I;
    const float2 g = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + row * 2 * I + col));
    const float2 u = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + row * 2 * I + I + col));
    const float2 d = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(dh + row * I + col));
    const float s0 = 1.f / (1.f + expf(-g.x)), s1 = 1.f / (1.f + expf(-g.y));
    const float a0 = bf16r(g.x * s0), a1 = bf16r(g.y * s1);
    const float dg0 = d.x * u.x * s0 * (1.f + g.x * (1.f - s0));
    const float dg1 = d.y * u.y * s1 * (1.f + g.y * (1.f - s1));
    *reinterpret_cast<uint32_t*>(dgu + row * 2 * I + col) = pack_bf16x2(dg0, dg1);
    *reinterpret_cast<uint32_t*>(dgu + row * 2 * I + I + col) = pack_bf16x2(d.x * a0, d.y * a1);
  }
}

static int pair_blocks(long long pairs) { return (int)std::max<long long>(1, std::min<long long>((pairs + 255) / 256, 148 * 16)); }

cudaError_t launch_silu_mul_bwd(const __nv_bfloat16* gu, const __nv_bfloat16* dh, int rows, int I,
                                __nv_bfloat16* dgu, cudaStream_t stream) {
  const long long pairs = (long long)rows * I / 2;
  if (pairs <= 0) return cudaSuccess;
  silu_mul_bwd_kernel<<<pair_blocks(pairs), 256, 0, stream>>>(gu, dh, I, pairs, dgu);
  return cudaGetLastError();
}

}  // namespace mb
