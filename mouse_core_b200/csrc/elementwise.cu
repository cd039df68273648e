// Row-wise glue kernels of the decoder layer around the attention kernels:
// residual add + RMSNorm (transformers Qwen3RMSNorm / LlamaRMSNorm, variance
// in fp32, as called at flex_decode.py:210, 232 and flex_train.py:135, 150)
// and the SiLU-gated product of the MLP (Qwen3MLP / LlamaMLP forward:
// down(silu(gate(x)) * up(x)); the gate and up projections run as one GEMM
// whose output is [rows, 2I] = gate | up).
#include "common.cuh"
#include "kernels.h"

namespace mb {

// One CTA per row. sum = x (+ residual), rounded to bf16 like the reference's
// bf16 residual stream; norm = sum * rsqrt(mean(sum^2) + eps) * w.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* x, const __nv_bfloat16* residual,
                                                      const __nv_bfloat16* w, float eps, int D,
                                                      __nv_bfloat16* sum_out, __nv_bfloat16* norm_out) {
  const size_t row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * D;
  const __nv_bfloat16* rr = residual ? residual + row * D : nullptr;
  __shared__ float red[8];
  float ss = 0.f;
  for (int i = threadIdx.x * 2; i < D; i += blockDim.x * 2) {
    float2 v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + i));
    if (rr) {
      const float2 r2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(rr + i));
      const __nv_bfloat162 s2 = __floats2bfloat162_rn(v.x + r2.x, v.y + r2.y);
      if (sum_out) *reinterpret_cast<__nv_bfloat162*>(sum_out + row * D + i) = s2;
      v = __bfloat1622float2(s2);
    }
    ss += v.x * v.x + v.y * v.y;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)D + eps);
  for (int i = threadIdx.x * 2; i < D; i += blockDim.x * 2) {
    float2 v;
    if (rr)  // re-read this thread's own rounded sum (the caller passes sum_out with residual)
      v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(sum_out + row * D + i));
    else
      v = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(xr + i));
    const float2 w2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + i));
    *reinterpret_cast<__nv_bfloat162*>(norm_out + row * D + i) = __floats2bfloat162_rn(v.x * r * w2.x, v.y * r * w2.y);
  }
}

cudaError_t launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* residual, const __nv_bfloat16* w,
                           float eps, int rows, int D, __nv_bfloat16* sum_out, __nv_bfloat16* norm_out,
                           cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int threads = std::min(256, std::max(32, ((D / 2 + 31) / 32) * 32));
  rmsnorm_kernel<<<rows, threads, 0, stream>>>(x, residual, w, eps, D, sum_out, norm_out);
  return cudaGetLastError();
}

// silu(gate) is rounded to bf16 before the product, as the module's bf16
// activation output is. Vector path: 8 elements (16 bytes) per thread,
// blockIdx.y strides rows; otherwise pairs of elements.
__device__ __forceinline__ float silu_bf16(float g) {
  return __bfloat162float(__float2bfloat16_rn(g / (1.f + expf(-g))));
}

__global__ void __launch_bounds__(128) silu_mul_vec_kernel(const __nv_bfloat16* __restrict__ gu, int rows, int I,
                                                           __nv_bfloat16* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (I >> 3)) return;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const size_t gbase = (size_t)row * 2 * I + (size_t)c * 8;
    const uint4 gv = *reinterpret_cast<const uint4*>(gu + gbase);
    const uint4 uv = *reinterpret_cast<const uint4*>(gu + gbase + I);
    const uint32_t* g2 = reinterpret_cast<const uint32_t*>(&gv);
    const uint32_t* u2 = reinterpret_cast<const uint32_t*>(&uv);
    uint4 o;
    uint32_t* o2 = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 g = unpack_bf16x2(g2[i]), u = unpack_bf16x2(u2[i]);
      o2[i] = pack_bf16x2(silu_bf16(g.x) * u.x, silu_bf16(g.y) * u.y);
    }
    *reinterpret_cast<uint4*>(out + (size_t)row * I + (size_t)c * 8) = o;
  }
}

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ gu, int rows, int I,
                                __nv_bfloat16* __restrict__ out) {
  for (int row = blockIdx.y; row < rows; row += gridDim.y)
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < (I >> 1); c += gridDim.x * blockDim.x) {
      const size_t gbase = (size_t)row * 2 * I + (size_t)c * 2;
      const float2 g = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + gbase));
      const float2 u = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(gu + gbase + I));
      *reinterpret_cast<uint32_t*>(out + (size_t)row * I + (size_t)c * 2) =
          pack_bf16x2(silu_bf16(g.x) * u.x, silu_bf16(g.y) * u.y);
    }
}

cudaError_t launch_silu_mul(const __nv_bfloat16* gate_up, int rows, int I, __nv_bfloat16* out, cudaStream_t stream) {
  if (rows <= 0 || I <= 0) return cudaSuccess;
  const int by = std::min(rows, 65535);
  const bool vec = I % 8 == 0 && (reinterpret_cast<uintptr_t>(gate_up) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0;
  if (vec) {
    silu_mul_vec_kernel<<<dim3((unsigned)((I / 8 + 127) / 128), (unsigned)by), 128, 0, stream>>>(gate_up, rows, I, out);
  } else {
    silu_mul_kernel<<<dim3((unsigned)std::min((I / 2 + 127) / 128, 64), (unsigned)by), 128, 0, stream>>>(gate_up, rows,
                                                                                                      I, out);
  }
  return cudaGetLastError();
}

// ---------------------------------------------------------------- fp32 residual stream
// The same layer glue for decoding with an fp32 residual stream: the sum of
// the residual and the sublayer output stays fp32 (no bf16 rounding at the
// adds), and only the GEMM inputs are rounded to bf16, once each. One CTA per
// row; `x` is the fp32 stream (or `x_bf16`, the bf16 embeddings entering the
// first layer), `delta` the fp32 sublayer output or null; `sum_out` may alias
// `x` (every element is read and written by the same thread).
__global__ void __launch_bounds__(256) rmsnorm_f32_kernel(const float* x, const __nv_bfloat16* x_bf16,
                                                          const float* delta, const __nv_bfloat16* w, float eps,
                                                          int D, float* sum_out, __nv_bfloat16* norm_out) {
  const size_t row = blockIdx.x;
  __shared__ float red[8];
  float ss = 0.f;
  for (int i = threadIdx.x * 2; i < D; i += blockDim.x * 2) {
    float2 v = x ? *reinterpret_cast<const float2*>(x + row * D + i)
                 : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x_bf16 + row * D + i));
    if (delta) {
      const float2 d = *reinterpret_cast<const float2*>(delta + row * D + i);
      v.x += d.x;
      v.y += d.y;
    }
    if (sum_out) *reinterpret_cast<float2*>(sum_out + row * D + i) = v;
    ss += v.x * v.x + v.y * v.y;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = (threadIdx.x < blockDim.x / 32) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float r = rsqrtf(red[0] / (float)D + eps);
  for (int i = threadIdx.x * 2; i < D; i += blockDim.x * 2) {
    float2 v;
    if (sum_out) {
      v = *reinterpret_cast<const float2*>(sum_out + row * D + i);
    } else {
      v = x ? *reinterpret_cast<const float2*>(x + row * D + i)
            : __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(x_bf16 + row * D + i));
      if (delta) {
        const float2 d = *reinterpret_cast<const float2*>(delta + row * D + i);
        v.x += d.x;
        v.y += d.y;
      }
    }
    const float2 w2 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(w + i));
    *reinterpret_cast<__nv_bfloat162*>(norm_out + row * D + i) = __floats2bfloat162_rn(v.x * r * w2.x, v.y * r * w2.y);
  }
}

cudaError_t launch_rmsnorm_f32(const float* x, const __nv_bfloat16* x_bf16, const float* delta,
                               const __nv_bfloat16* w, float eps, int rows, int D, float* sum_out,
                               __nv_bfloat16* norm_out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int threads = std::min(256, std::max(32, ((D / 2 + 31) / 32) * 32));
  rmsnorm_f32_kernel<<<rows, threads, 0, stream>>>(x, x_bf16, delta, w, eps, D, sum_out, norm_out);
  return cudaGetLastError();
}

// out = bf16(silu(g) * u) for an fp32 [rows, 2I] = gate | up, 4 elements per thread.
__global__ void __launch_bounds__(128) silu_mul_f32_kernel(const float* __restrict__ gu, int rows, int I,
                                                           __nv_bfloat16* __restrict__ out) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= (I >> 2)) return;
  for (int row = blockIdx.y; row < rows; row += gridDim.y) {
    const size_t gbase = (size_t)row * 2 * I + (size_t)c * 4;
    const float4 g = *reinterpret_cast<const float4*>(gu + gbase);
    const float4 u = *reinterpret_cast<const float4*>(gu + gbase + I);
    uint2 o;
    o.x = pack_bf16x2(g.x / (1.f + expf(-g.x)) * u.x, g.y / (1.f + expf(-g.y)) * u.y);
    o.y = pack_bf16x2(g.z / (1.f + expf(-g.z)) * u.z, g.w / (1.f + expf(-g.w)) * u.w);
    *reinterpret_cast<uint2*>(out + (size_t)row * I + (size_t)c * 4) = o;
  }
}

cudaError_t launch_silu_mul_f32(const float* gate_up, int rows, int I, __nv_bfloat16* out, cudaStream_t stream) {
  if (rows <= 0 || I <= 0) return cudaSuccess;
  const int by = std::min(rows, 65535);
  silu_mul_f32_kernel<<<dim3((unsigned)((I / 4 + 127) / 128), (unsigned)by), 128, 0, stream>>>(gate_up, rows, I, out);
  return cudaGetLastError();
}

}  // namespace mb
