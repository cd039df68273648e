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

__global__ void silu_mul_kernel(const __nv_bfloat16* gu, int I, long long total_pairs, __nv_bfloat16* out) {
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < total_pairs;
       i += (long long)gridDim.x * blockDim.x) {
    const long long row = (i * 2) / I, col = (i * 2) % I;
    const float2 g = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * I + col));
    const float2 u = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(gu + row * 2 * I + I + col));
    // silu(gate) is rounded to bf16 before the product, as the module's bf16
    // activation output is.
    const float a = __bfloat162float(__float2bfloat16_rn(g.x / (1.f + expf(-g.x))));
    const float b = __bfloat162float(__float2bfloat16_rn(g.y / (1.f + expf(-g.y))));
    *reinterpret_cast<__nv_bfloat162*>(out + row * I + col) = __floats2bfloat162_rn(a * u.x, b * u.y);
  }
}

cudaError_t launch_silu_mul(const __nv_bfloat16* gate_up, int rows, int I, __nv_bfloat16* out, cudaStream_t stream) {
  const long long pairs = (long long)rows * I / 2;
  if (pairs <= 0) return cudaSuccess;
  const int blocks = (int)std::min<long long>((pairs + 255) / 256, 148 * 16);
  silu_mul_kernel<<<blocks, 256, 0, stream>>>(gate_up, I, pairs, out);
  return cudaGetLastError();
}

}  // namespace mb
