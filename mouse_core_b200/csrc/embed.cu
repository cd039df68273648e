// K11: token embedding of a flat TokenBatch in one pass.
//
// Replaces NumericEmbedder.forward (src/mouse_core/models/embedding/
// embedding.py:293-326): there, one masked gather per embedding table
// (embeds[types == tid] = table(ids[mask])) and one masked static-Fourier
// evaluation per Fourier modality (embeds[mask] = fourier(scalars, ids),
// models/embedding/encoding.py:67-86: scale * cos(x * freqs[id] + phases[id]))
// each make a pass over the token stream and allocate mask/index tensors.
// Here one warp writes each token's row: a 16-byte-vector copy of its table
// row, or its Fourier features computed in fp32 and rounded once; a token
// whose type has neither stays zero, as in the reference's zero-initialised
// output. HBM-bound: L * D * elem bytes written, table rows read.
#include "common.cuh"
#include "kernels.h"

namespace mb {

template <typename T>
__device__ __forceinline__ void store_pair(T* dst, float a, float b);

template <>
__device__ __forceinline__ void store_pair<__nv_bfloat16>(__nv_bfloat16* dst, float a, float b) {
  *reinterpret_cast<__nv_bfloat162*>(dst) = __floats2bfloat162_rn(a, b);
}

template <>
__device__ __forceinline__ void store_pair<float>(float* dst, float a, float b) {
  *reinterpret_cast<float2*>(dst) = make_float2(a, b);
}

template <typename T>
__global__ void __launch_bounds__(256) embed_tokens_kernel(EmbedParams p) {
  const int warps = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  T* out = static_cast<T*>(p.out);
  constexpr int VEC = 16 / sizeof(T);  // elements per 16-byte vector
  for (long long t = (long long)blockIdx.x * warps + (threadIdx.x >> 5); t < p.L; t += (long long)gridDim.x * warps) {
    T* row = out + t * p.D;
    const int type = p.types[t];
    const int kind = (type >= 0 && type < p.n_types) ? p.kinds[type] : 0;
    const int id = p.ids[t];
    if (kind == 1) {  // table row
      const T* src = static_cast<const T*>(p.tables[type]);
      if (id < 0 || id >= p.vocab[type]) {
        report(kDevBadIndex);
        src = nullptr;
      }
      if (src) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src + (size_t)id * p.D);
        uint4* d4 = reinterpret_cast<uint4*>(row);
        for (int c = lane; c < p.D / VEC; c += 32) d4[c] = s4[c];
        continue;
      }
    } else if (kind == 2) {  // static Fourier features of the scalar, bank `id`
      if (id >= 0 && id < p.freq_sets) {
        const float x = p.scalars[t];
        const float* w = p.freqs + (size_t)id * p.D;
        const float* b = p.phases + (size_t)id * p.D;
        for (int c = lane * 2; c < p.D; c += 64)
          store_pair<T>(row + c, p.fourier_scale * cosf(fmaf(x, w[c], b[c])),
                        p.fourier_scale * cosf(fmaf(x, w[c + 1], b[c + 1])));
        continue;
      }
      report(kDevBadIndex);
    }
    for (int c = lane * 2; c < p.D; c += 64) store_pair<T>(row + c, 0.f, 0.f);
  }
}

cudaError_t launch_embed_tokens(const EmbedParams& p, bool out_f32, cudaStream_t stream) {
  if (p.L <= 0) return cudaSuccess;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long blocks = std::min<long long>((p.L + 7) / 8, (long long)sms * 8);
  if (out_f32)
    embed_tokens_kernel<float><<<(unsigned)blocks, 256, 0, stream>>>(p);
  else
    embed_tokens_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace mb
