// K2: fused q/k RMSNorm + RoPE + paged K/V append, and K3: page copy.
//
// K2 replaces, per layer of FlexDecodeSession.forward, the q/k norm calls
// (src/mouse_core/models/backbone/flex_decode.py:214-217), the rotary embedding
// (flex_decode.py:204, 221 via transformers' apply_rotary_pos_emb) and the
// cache scatter (flex_decode.py:223-224): one pass over the fused QKV
// projection output writes the rotated queries and stores the rotated keys and
// the values of real tokens at their page slots. Arithmetic is fp32 with one
// rounding to bf16 per output element (the reference rounds after each bf16
// op; both agree within the bf16 tolerance of the tests).
//
// K3 copies whole pages (all kv-heads of one layer) from a list of source
// pages to destination pages: the copy-on-write step when branches fork a
// shared partial page, and the rebuild-from-cache copy.
#include "common.cuh"
#include "kernels.h"

namespace mb {

template <int HD>
__global__ void __launch_bounds__(256) append_kernel(const AppendParams p) {
  constexpr int E = HD / 32;  // elements per lane
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nheads = p.Hq + 2 * p.Hkv;
  const int pos = p.pos[t];
  const long long slot = p.slot ? (long long)p.slot[t] : -1;
  const bool cached = slot >= 0 && slot < p.num_slots && p.k_pool != nullptr;
  const long long page = cached ? slot / p.page_size : 0;
  const int off = cached ? (int)(slot % p.page_size) : 0;

  // cos/sin of this lane's E rotary frequencies (shared by every q/k head).
  float cs[E], sn[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int j = (lane & 15) * E + e;
    float s_, c_;
    sincosf((float)pos * p.inv_freq[j], &s_, &c_);
    cs[e] = c_ * p.attn_scaling;
    sn[e] = s_ * p.attn_scaling;
  }

  for (int hh = warp; hh < nheads; hh += blockDim.x / 32) {
    const size_t src_off = (size_t)t * p.qkv_stride + (size_t)hh * HD + lane * E;
    float x[E];
    if (p.qkv_f32) {  // fp32 projection output (fp32 residual-stream decoding)
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const float2 v2 = *reinterpret_cast<const float2*>(p.qkv_f32 + src_off + e);
        x[e] = v2.x;
        x[e + 1] = v2.y;
      }
    } else {
#pragma unroll
      for (int e = 0; e < E; e += 2) {
        const __nv_bfloat162 v2 = *reinterpret_cast<const __nv_bfloat162*>(p.qkv + src_off + e);
        x[e] = __low2float(v2);
        x[e + 1] = __high2float(v2);
      }
    }
    const bool is_q = hh < p.Hq;
    const bool is_k = !is_q && hh < p.Hq + p.Hkv;
    __nv_bfloat16* dst_pool = nullptr;
    __nv_bfloat16* dst_flat = nullptr;
    if (is_q) {
      dst_flat = p.q_out + ((size_t)t * p.Hq + hh) * HD + lane * E;
    } else {
      const int kvh = is_k ? hh - p.Hq : hh - p.Hq - p.Hkv;
      if (cached)
        dst_pool = (is_k ? p.k_pool : p.v_pool) + ((page * p.Hkv + kvh) * p.page_size + off) * (size_t)HD + lane * E;
      __nv_bfloat16* flat = is_k ? p.k_out : p.v_out;
      if (flat) dst_flat = flat + ((size_t)t * p.Hkv + kvh) * HD + lane * E;
    }
    if (is_q || is_k) {
      const __nv_bfloat16* nw = is_q ? p.q_norm_w : p.k_norm_w;
      if (nw) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) ss += x[e] * x[e];
        ss = warp_sum(ss);
        const float r = rsqrtf(ss / (float)HD + p.eps);
#pragma unroll
        for (int e = 0; e < E; ++e) x[e] = x[e] * r * __bfloat162float(nw[lane * E + e]);
      }
      // rotate_half: dims [0, HD/2) pair with [HD/2, HD); lane l <-> l ^ 16.
      float y[E];
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
        y[e] = (lane < 16) ? x[e] * cs[e] - partner * sn[e] : x[e] * cs[e] + partner * sn[e];
      }
#pragma unroll
      for (int e = 0; e < E; ++e) x[e] = y[e];
    }
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const __nv_bfloat162 v2 = __floats2bfloat162_rn(x[e], x[e + 1]);
      if (dst_flat) *reinterpret_cast<__nv_bfloat162*>(dst_flat + e) = v2;
      if (dst_pool) *reinterpret_cast<__nv_bfloat162*>(dst_pool + e) = v2;
    }
  }
}

cudaError_t launch_append(const AppendParams& p, cudaStream_t stream) {
  if (p.T <= 0) return cudaSuccess;
  const int nheads = p.Hq + 2 * p.Hkv;
  const int threads = nheads >= 8 ? 256 : 32 * nheads;
  if (p.head_dim == 128)
    append_kernel<128><<<p.T, threads, 0, stream>>>(p);
  else
    append_kernel<64><<<p.T, threads, 0, stream>>>(p);
  return cudaGetLastError();
}

__global__ void page_copy_kernel(const uint4* src, uint4* dst, const int32_t* src_pages, const int32_t* dst_pages,
                                 long long page_vecs) {
  const int i = blockIdx.y;
  const long long s = (long long)src_pages[i] * page_vecs;
  const long long d = (long long)dst_pages[i] * page_vecs;
  for (long long v = (long long)blockIdx.x * blockDim.x + threadIdx.x; v < page_vecs;
       v += (long long)gridDim.x * blockDim.x)
    dst[d + v] = src[s + v];
}

cudaError_t launch_page_copy(const __nv_bfloat16* src_pool, __nv_bfloat16* dst_pool, const int32_t* src_pages,
                             const int32_t* dst_pages, int n, long long page_elems, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const long long vecs = page_elems / 8;
  const int gx = (int)std::min<long long>((vecs + 255) / 256, 64);
  page_copy_kernel<<<dim3(gx, n), 256, 0, stream>>>(reinterpret_cast<const uint4*>(src_pool),
                                                    reinterpret_cast<uint4*>(dst_pool), src_pages, dst_pages, vecs);
  return cudaGetLastError();
}

constexpr int kStepRestart = 1 << 30;  // decode_step_meta code flag: the row restarts at length 0

// One decode step's metadata on the device (each row appends at most one
// token): the current length L = kv_len[b] (left there by the previous step),
// the new token's position L, its cache slot from the block table, and the
// new length L + 1. code[b] (or -1 for every row when code is NULL):
//   -1  append; the token's page is already in the table;
//   >=0 append; the token opens page code[b], written into the table first;
//       with bit 30 set the row was emptied: it restarts at length 0 and the
//       page (the low bits) goes to column 0;
//   -2  append nothing (position max(L - 1, 0), no slot, length kept);
//   -3  the row was emptied and appends nothing (position 0, length 0).
// A column past the table's width is reported (kDevBadPage) and the token is
// not cached (slot -1).
__global__ void decode_step_meta_kernel(int B, int width, int page_size, const int32_t* __restrict__ code,
                                        int32_t* __restrict__ block_table, int32_t* __restrict__ q_pos,
                                        int32_t* __restrict__ kv_len, int32_t* __restrict__ slot) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int c = code ? code[b] : -1;
  int L = kv_len[b];
  if (c == -2 || c == -3) {
    if (c == -3) L = 0;
    q_pos[b] = max(L - 1, 0);
    slot[b] = -1;
    kv_len[b] = L;
    return;
  }
  if (c >= 0 && (c & kStepRestart)) L = 0;
  const int np = c >= 0 ? (c & ~kStepRestart) : -1;
  const int col = L / page_size;
  int s = -1;
  if (L < 0 || col >= width) {
    report(kDevBadPage);
  } else {
    int32_t* entry = block_table + (size_t)b * width + col;
    if (np >= 0) *entry = np;
    s = (np >= 0 ? np : *entry) * page_size + L % page_size;
  }
  q_pos[b] = L;
  slot[b] = s;
  kv_len[b] = L + 1;
}

cudaError_t launch_decode_step_meta(int B, int width, int page_size, const int32_t* new_page, int32_t* block_table,
                                    int32_t* q_pos, int32_t* kv_len, int32_t* slot, cudaStream_t stream) {
  if (B <= 0) return cudaSuccess;
  decode_step_meta_kernel<<<(B + 127) / 128, 128, 0, stream>>>(B, width, page_size, new_page, block_table, q_pos,
                                                               kv_len, slot);
  return cudaGetLastError();
}

}  // namespace mb
