// extern "C" entry points declared in include/mouse_b200.h: argument
// validation, TMA descriptor encoding and kernel launches. No exceptions cross
// the ABI; every failure returns a status and records a message.
#include <string>

#include "../../include/mouse_b200.h"
#include "common.cuh"
#include "kernels.h"

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(MB_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  }
  return fn;
}

// 2-D view [rows, head_dim] of one layer's pool, 64x64 boxes, 128B swizzle.
int encode_pool_map(CUtensorMap* map, const void* pool, long long rows, int head_dim) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)head_dim, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)head_dim * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(pool), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MB_OK;
}

// 3-D view {head_dim, heads, tokens} of a token-major [L, heads, head_dim]
// tensor: 64-element x 1-head x 128-token boxes, 128B swizzle.
int encode_token_map(CUtensorMap* map, const void* base, int L, int heads, int head_dim) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[3] = {(cuuint64_t)head_dim, (cuuint64_t)heads, (cuuint64_t)L};
  cuuint64_t strides[2] = {(cuuint64_t)head_dim * 2, (cuuint64_t)heads * head_dim * 2};
  cuuint32_t box[3] = {64, 1, 128};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MB_OK;
}

// A row-major bf16 matrix [rows, cols] read in boxes of 64 columns x 128
// rows with the 128-byte swizzle (the K-major operand layout of tcgen05).
int encode_matrix_map(CUtensorMap* map, const void* base, long long rows, int cols) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(MB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MB_ERR_CUDA, "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) + ")");
  return MB_OK;
}

int check_decode_shape(int batch, int q_len, int q_heads, int kv_heads, int head_dim, int page_size) {
  if (batch < 0 || q_len < 0 || q_heads <= 0 || kv_heads <= 0)
    return fail(MB_ERR_INVALID_ARG, "batch/q_len must be >= 0 and head counts > 0");
  if (q_heads % kv_heads != 0) return fail(MB_ERR_INVALID_ARG, "q_heads must be a multiple of kv_heads");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (page_size <= 0 || page_size % 64 != 0) return fail(MB_ERR_UNSUPPORTED, "page_size must be a multiple of 64");
  return MB_OK;
}

}  // namespace

extern "C" {

const char* mb_last_error(void) { return g_err.c_str(); }

int mb_version(void) { return 100; }

int mb_device_status(int* status_out, int clear) {
  if (!status_out) return fail(MB_ERR_INVALID_ARG, "status_out is NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  e = cudaMemcpyFromSymbol(status_out, mb::g_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_fail(e, "read device status");
  if (clear) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(mb::g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_fail(e, "clear device status");
  }
  return MB_OK;
}

int mb_set_wait_limit(long long cycles) {
  const long long v = cycles < 0 ? mb::kWaitCycles : cycles;
  cudaError_t e = cudaMemcpyToSymbol(mb::g_wait_limit, &v, sizeof(v));
  if (e != cudaSuccess) return cuda_fail(e, "set wait limit");
  e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  return MB_OK;
}

size_t mb_decode_workspace_bytes(int batch, int kv_heads, int q_rows, int head_dim, int max_kv_len) {
  if (batch <= 0 || kv_heads <= 0 || q_rows <= 0 || q_rows > 16) return 0;
  if (head_dim != 64 && head_dim != 128) return 0;
  mb::WorkspaceLayout lay;
  return mb::decode_workspace_layout(batch, kv_heads, q_rows, head_dim, max_kv_len, &lay);
}

int mb_decode_plan(const int32_t* kv_len, int batch, int kv_heads, int q_rows, int head_dim, int max_kv_len,
                   void* workspace, size_t workspace_bytes, mb_stream_t stream) {
  if (batch <= 0) return MB_OK;
  if (!kv_len) return fail(MB_ERR_INVALID_ARG, "kv_len is NULL");
  if (q_rows <= 0 || q_rows > 16) return fail(MB_ERR_INVALID_ARG, "a plan exists only for 1..16 query rows");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  mb::WorkspaceLayout lay;
  const size_t need = mb::decode_workspace_layout(batch, kv_heads, q_rows, head_dim, max_kv_len, &lay);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(MB_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes, 256-byte aligned");
  cudaError_t e = mb::launch_decode_plan(kv_len, nullptr, 0, 0, batch, kv_heads, q_rows, head_dim, lay,
                                         static_cast<uint8_t*>(workspace), (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "decode plan launch");
}

int mb_decode_plan_shared(const int32_t* kv_len, const int32_t* block_table, int max_pages, int page_size,
                          int batch, int kv_heads, int q_rows, int head_dim, int max_kv_len, void* workspace,
                          size_t workspace_bytes, mb_stream_t stream) {
  if (batch <= 0) return MB_OK;
  if (!kv_len || !block_table) return fail(MB_ERR_INVALID_ARG, "kv_len or block_table is NULL");
  if (q_rows <= 0 || q_rows > 16) return fail(MB_ERR_INVALID_ARG, "a plan exists only for 1..16 query rows");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (max_pages <= 0 || page_size <= 0) return fail(MB_ERR_INVALID_ARG, "max_pages and page_size must be positive");
  mb::WorkspaceLayout lay;
  const size_t need = mb::decode_workspace_layout(batch, kv_heads, q_rows, head_dim, max_kv_len, &lay);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(MB_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes, 256-byte aligned");
  cudaError_t e = mb::launch_decode_plan(kv_len, block_table, max_pages, page_size, batch, kv_heads, q_rows,
                                         head_dim, lay, static_cast<uint8_t*>(workspace), (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "decode plan launch");
}

int mb_decode_attention(const void* q, const void* k_pool, const void* v_pool, int num_pages,
                        const int32_t* block_table, int max_pages, const int32_t* q_pos, const int32_t* kv_len,
                        int batch, int q_len, int q_heads, int kv_heads, int head_dim, int page_size, float scale,
                        int max_kv_len, int plan_ready, void* out, void* workspace, size_t workspace_bytes,
                        mb_stream_t stream) {
  int rc = check_decode_shape(batch, q_len, q_heads, kv_heads, head_dim, page_size);
  if (rc) return rc;
  if (batch == 0 || q_len == 0) return MB_OK;
  if (!q || !k_pool || !v_pool || !block_table || !q_pos || !kv_len || !out)
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (num_pages <= 0 || max_pages <= 0) return fail(MB_ERR_INVALID_ARG, "num_pages and max_pages must be > 0");
  if (!aligned(k_pool, 16) || !aligned(v_pool, 16) || !aligned(q, 4) || !aligned(out, 4))
    return fail(MB_ERR_INVALID_ARG, "pools must be 16-byte aligned, q/out 4-byte aligned");
  if (max_kv_len < 0 || (long long)max_kv_len > (long long)max_pages * page_size)
    return fail(MB_ERR_INVALID_ARG, "max_kv_len exceeds max_pages * page_size");
  const long long rows = (long long)num_pages * kv_heads * page_size;
  if (rows >= (1ll << 31)) return fail(MB_ERR_UNSUPPORTED, "pool too large for one layer (>= 2^31 rows)");

  const int G = q_heads / kv_heads;
  const int R = G * q_len;
  const bool split = R <= 16;

  CUtensorMap km, vm;
  if ((rc = encode_pool_map(&km, k_pool, rows, head_dim))) return rc;
  if ((rc = encode_pool_map(&vm, v_pool, rows, head_dim))) return rc;

  mb::AttnParams p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.block_table = block_table;
  p.q_pos = q_pos;
  p.kv_len = kv_len;
  p.B = batch;
  p.S = q_len;
  p.Hq = q_heads;
  p.Hkv = kv_heads;
  p.G = G;
  p.R = R;
  p.head_dim = head_dim;
  p.max_pages = max_pages;
  p.page_size = page_size;
  p.num_pages = num_pages;
  p.scale_log2 = scale * 1.4426950408889634f;

  // Prefill chunks of at least kPrefillMinRows queries per row run on the
  // tcgen05 kernel (128-query tiles, TMEM accumulators, page-gathering TMA);
  // shorter multi-row chunks keep the warp-MMA block mode.
  constexpr int kPrefillMinRows = 64;
  if (!split && q_len >= kPrefillMinRows && aligned(q, 16) && aligned(out, 16) &&
      (long long)batch * q_len < (1ll << 31)) {
    CUtensorMap qm;
    if ((rc = encode_token_map(&qm, q, batch * q_len, q_heads, head_dim))) return rc;
    mb::VarlenParams vp{};
    vp.L = batch * q_len;
    vp.Hq = q_heads;
    vp.Hkv = kv_heads;
    vp.G = G;
    vp.heads_per_cta = (G % 2 == 0) ? 2 : 1;
    vp.head_dim = head_dim;
    vp.scale_log2 = p.scale_log2;
    vp.out = static_cast<__nv_bfloat16*>(out);
    vp.block_table = block_table;
    vp.q_pos = q_pos;
    vp.kv_len = kv_len;
    vp.B = batch;
    vp.S = q_len;
    vp.max_pages = max_pages;
    vp.page_size = page_size;
    vp.num_pages = num_pages;
    // With any workspace the kernel runs persistent CTAs over a tile counter
    // kept in its first 4 bytes.
    if (workspace && workspace_bytes >= sizeof(int) && aligned(workspace, 4))
      vp.tile_counter = static_cast<int*>(workspace);
    cudaError_t e = mb::launch_paged_prefill(qm, km, vm, vp, (cudaStream_t)stream);
    return e == cudaSuccess ? MB_OK : cuda_fail(e, "paged prefill launch");
  }

  mb::WorkspaceLayout lay{};
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  if (split) {
    const size_t need = mb::decode_workspace_layout(batch, kv_heads, R, head_dim, max_kv_len, &lay);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
      return fail(MB_ERR_WORKSPACE, "workspace needs " + std::to_string(need) + " bytes, 256-byte aligned");
    if (!plan_ready) {
      cudaError_t e =
          mb::launch_decode_plan(kv_len, nullptr, 0, 0, batch, kv_heads, R, head_dim, lay, ws, (cudaStream_t)stream);
      if (e != cudaSuccess) return cuda_fail(e, "decode plan launch");
    }
  }
  cudaError_t e = mb::launch_decode_attention(km, vm, p, lay, ws, split, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "decode attention launch");
}

}  // extern "C"

namespace {
int kv_append_impl(const void* qkv, bool qkv_f32, int tokens, int qkv_stride, const int32_t* pos,
                   const int32_t* slot, const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                   float attention_scaling, int q_heads, int kv_heads, int head_dim, int page_size,
                   long long num_pages, void* q_out, void* k_out, void* v_out, void* k_pool, void* v_pool,
                   mb_stream_t stream) {
  if (tokens < 0) return fail(MB_ERR_INVALID_ARG, "tokens must be >= 0");
  if (tokens == 0) return MB_OK;
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (q_heads <= 0 || kv_heads <= 0) return fail(MB_ERR_INVALID_ARG, "head counts must be > 0");
  if (!qkv || !pos || !inv_freq || !q_out) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (qkv_stride < (q_heads + 2 * kv_heads) * head_dim)
    return fail(MB_ERR_INVALID_ARG, "qkv_stride smaller than (q_heads + 2 * kv_heads) * head_dim");
  if (qkv_stride % 2 || !aligned(qkv, qkv_f32 ? 8 : 4) || !aligned(q_out, 4))
    return fail(MB_ERR_INVALID_ARG, "qkv (4-byte, 8 for fp32) / q_out (4-byte) must be aligned with an even stride");
  if ((k_pool == nullptr) != (v_pool == nullptr)) return fail(MB_ERR_INVALID_ARG, "pass both pools or neither");
  if (k_pool && (!slot || page_size <= 0 || num_pages <= 0))
    return fail(MB_ERR_INVALID_ARG, "paged append needs slot, page_size and num_pages");
  mb::AppendParams p{};
  if (qkv_f32)
    p.qkv_f32 = static_cast<const float*>(qkv);
  else
    p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.T = tokens;
  p.qkv_stride = qkv_stride;
  p.pos = pos;
  p.slot = slot;
  p.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  p.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  p.eps = eps;
  p.inv_freq = inv_freq;
  p.attn_scaling = attention_scaling;
  p.Hq = q_heads;
  p.Hkv = kv_heads;
  p.head_dim = head_dim;
  p.page_size = page_size > 0 ? page_size : 1;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_out = static_cast<__nv_bfloat16*>(k_out);
  p.v_out = static_cast<__nv_bfloat16*>(v_out);
  p.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  p.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  p.num_slots = k_pool ? num_pages * (long long)page_size : 0;
  cudaError_t e = mb::launch_append(p, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "kv append launch");
}
}  // namespace

extern "C" {

int mb_kv_append(const void* qkv, int tokens, int qkv_stride, const int32_t* pos, const int32_t* slot,
                 const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                 float attention_scaling, int q_heads, int kv_heads, int head_dim, int page_size,
                 long long num_pages, void* q_out, void* k_out, void* v_out, void* k_pool, void* v_pool,
                 mb_stream_t stream) {
  return kv_append_impl(qkv, false, tokens, qkv_stride, pos, slot, q_norm_w, k_norm_w, eps, inv_freq,
                        attention_scaling, q_heads, kv_heads, head_dim, page_size, num_pages, q_out, k_out, v_out,
                        k_pool, v_pool, stream);
}

int mb_kv_append_f32(const float* qkv, int tokens, int qkv_stride, const int32_t* pos, const int32_t* slot,
                     const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                     float attention_scaling, int q_heads, int kv_heads, int head_dim, int page_size,
                     long long num_pages, void* q_out, void* k_out, void* v_out, void* k_pool, void* v_pool,
                     mb_stream_t stream) {
  return kv_append_impl(qkv, true, tokens, qkv_stride, pos, slot, q_norm_w, k_norm_w, eps, inv_freq,
                        attention_scaling, q_heads, kv_heads, head_dim, page_size, num_pages, q_out, k_out, v_out,
                        k_pool, v_pool, stream);
}

int mb_rope_table(const int32_t* pos, int tokens, const float* inv_freq, int head_dim, float attention_scaling,
                  float* table, mb_stream_t stream) {
  if (tokens < 0) return fail(MB_ERR_INVALID_ARG, "tokens must be >= 0");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (tokens == 0) return MB_OK;
  if (!pos || !inv_freq || !table) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(table, 16)) return fail(MB_ERR_INVALID_ARG, "table must be 16-byte aligned");
  cudaError_t e = mb::launch_rope_table(pos, tokens, inv_freq, head_dim, attention_scaling, table,
                                        (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "rope table launch");
}

int mb_qkv_append(const void* x, int tokens, int hidden, const void* w_qkv, const void* bias, const float* rope_table,
                  const void* q_norm_w, const void* k_norm_w, float eps, const int32_t* slot, int q_heads,
                  int kv_heads, int head_dim, int page_size, long long num_pages, void* q_out, void* k_pool,
                  void* v_pool, mb_stream_t stream) {
  if (tokens < 0 || hidden <= 0 || q_heads <= 0 || kv_heads <= 0)
    return fail(MB_ERR_INVALID_ARG, "tokens >= 0, hidden > 0 and head counts > 0 required");
  if (q_heads % kv_heads) return fail(MB_ERR_INVALID_ARG, "q_heads must be a multiple of kv_heads");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  const long long n = (long long)(q_heads + 2 * kv_heads) * head_dim;
  if (n % 128) return fail(MB_ERR_UNSUPPORTED, "(q_heads + 2 kv_heads) * head_dim must be a multiple of 128");
  if (hidden % 8) return fail(MB_ERR_UNSUPPORTED, "hidden must be a multiple of 8");
  if (tokens == 0) return MB_OK;
  if (!x || !w_qkv || !rope_table || !q_out) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(x, 16) || !aligned(w_qkv, 16) || !aligned(rope_table, 16) || !aligned(q_out, 16))
    return fail(MB_ERR_INVALID_ARG, "x, w_qkv, rope_table and q_out must be 16-byte aligned");
  if (k_pool || v_pool) {
    if (!k_pool || !v_pool || !slot) return fail(MB_ERR_INVALID_ARG, "k_pool, v_pool and slot go together");
    if (page_size <= 0 || num_pages <= 0) return fail(MB_ERR_INVALID_ARG, "page_size and num_pages must be > 0");
    if (!aligned(k_pool, 16) || !aligned(v_pool, 16)) return fail(MB_ERR_INVALID_ARG, "pools must be 16-byte aligned");
  }
  CUtensorMap xm, wm;
  int rc;
  if ((rc = encode_matrix_map(&xm, x, tokens, hidden))) return rc;
  if ((rc = encode_matrix_map(&wm, w_qkv, n, hidden))) return rc;
  mb::QkvAppendParams p{};
  p.T = tokens;
  p.K = hidden;
  p.N = (int)n;
  p.Hq = q_heads;
  p.Hkv = kv_heads;
  p.head_dim = head_dim;
  p.page_size = page_size;
  p.bias = static_cast<const __nv_bfloat16*>(bias);
  p.rope = reinterpret_cast<const float2*>(rope_table);
  p.q_norm_w = static_cast<const __nv_bfloat16*>(q_norm_w);
  p.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_w);
  p.eps = eps;
  p.slot = k_pool ? slot : nullptr;
  p.num_slots = k_pool ? num_pages * page_size : 0;
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.k_pool = static_cast<__nv_bfloat16*>(k_pool);
  p.v_pool = static_cast<__nv_bfloat16*>(v_pool);
  cudaError_t e = mb::launch_qkv_append(xm, wm, p, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "qkv append launch");
}

int mb_page_copy(const void* src_pool, void* dst_pool, const int32_t* src_pages, const int32_t* dst_pages, int n,
                 long long page_elems, mb_stream_t stream) {
  if (n < 0) return fail(MB_ERR_INVALID_ARG, "n must be >= 0");
  if (n == 0) return MB_OK;
  if (!src_pool || !dst_pool || !src_pages || !dst_pages) return fail(MB_ERR_INVALID_ARG, "NULL pointer");
  if (page_elems <= 0 || page_elems % 8 || !aligned(src_pool, 16) || !aligned(dst_pool, 16))
    return fail(MB_ERR_INVALID_ARG, "page_elems must be a positive multiple of 8 and pools 16-byte aligned");
  cudaError_t e = mb::launch_page_copy(static_cast<const __nv_bfloat16*>(src_pool),
                                       static_cast<__nv_bfloat16*>(dst_pool), src_pages, dst_pages, n, page_elems,
                                       (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "page copy launch");
}

int mb_decode_step_meta(int batch, int max_pages, int page_size, const int32_t* new_page, int32_t* block_table,
                        int32_t* q_pos, int32_t* kv_len, int32_t* slot, mb_stream_t stream) {
  if (batch < 0 || max_pages <= 0 || page_size <= 0)
    return fail(MB_ERR_INVALID_ARG, "batch >= 0, max_pages > 0 and page_size > 0 required");
  if (batch == 0) return MB_OK;
  if (!block_table || !q_pos || !kv_len || !slot) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = mb::launch_decode_step_meta(batch, max_pages, page_size, new_page, block_table, q_pos, kv_len, slot,
                                              (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "decode step meta launch");
}

int mb_rmsnorm(const void* x, const void* residual, const void* weight, float eps, int rows, int dim, void* sum_out,
               void* norm_out, mb_stream_t stream) {
  if (rows < 0 || dim <= 0 || dim % 2) return fail(MB_ERR_INVALID_ARG, "rows >= 0 and an even dim > 0 required");
  if (rows == 0) return MB_OK;
  if (!x || !weight || !norm_out) return fail(MB_ERR_INVALID_ARG, "NULL pointer");
  if (residual && !sum_out) return fail(MB_ERR_INVALID_ARG, "residual needs sum_out");
  if (!aligned(x, 4) || !aligned(norm_out, 4) || (residual && (!aligned(residual, 4) || !aligned(sum_out, 4))))
    return fail(MB_ERR_INVALID_ARG, "buffers must be 4-byte aligned");
  cudaError_t e = mb::launch_rmsnorm(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
                                     static_cast<const __nv_bfloat16*>(weight), eps, rows, dim,
                                     static_cast<__nv_bfloat16*>(sum_out), static_cast<__nv_bfloat16*>(norm_out),
                                     (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "rmsnorm launch");
}

int mb_rmsnorm_f32(const float* x, const void* x_bf16, const float* delta, const void* weight, float eps, int rows,
                   int dim, float* sum_out, void* norm_out, mb_stream_t stream) {
  if (rows < 0 || dim <= 0 || dim % 2) return fail(MB_ERR_INVALID_ARG, "rows >= 0 and an even dim > 0 required");
  if (rows == 0) return MB_OK;
  if ((x == nullptr) == (x_bf16 == nullptr)) return fail(MB_ERR_INVALID_ARG, "pass exactly one of x and x_bf16");
  if (!weight || !norm_out) return fail(MB_ERR_INVALID_ARG, "NULL pointer");
  if ((x && !aligned(x, 8)) || (x_bf16 && !aligned(x_bf16, 4)) || (delta && !aligned(delta, 8)) ||
      (sum_out && !aligned(sum_out, 8)) || !aligned(norm_out, 4) || !aligned(weight, 4))
    return fail(MB_ERR_INVALID_ARG, "misaligned buffer (fp32 buffers 8-byte, bf16 4-byte)");
  cudaError_t e = mb::launch_rmsnorm_f32(x, static_cast<const __nv_bfloat16*>(x_bf16), delta,
                                         static_cast<const __nv_bfloat16*>(weight), eps, rows, dim, sum_out,
                                         static_cast<__nv_bfloat16*>(norm_out), (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "rmsnorm_f32 launch");
}

int mb_silu_mul_f32(const float* gate_up, int rows, int inter, void* out, mb_stream_t stream) {
  if (rows < 0 || inter <= 0 || inter % 4) return fail(MB_ERR_INVALID_ARG, "rows >= 0 and inter % 4 == 0 required");
  if (rows == 0) return MB_OK;
  if (!gate_up || !out || !aligned(gate_up, 16) || !aligned(out, 8))
    return fail(MB_ERR_INVALID_ARG, "NULL or misaligned pointer (gate_up 16-byte, out 8-byte)");
  cudaError_t e = mb::launch_silu_mul_f32(gate_up, rows, inter, static_cast<__nv_bfloat16*>(out),
                                          (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "silu_mul_f32 launch");
}

int mb_embed_tokens(const int32_t* types, const int32_t* ids, const float* scalars, long long tokens, int dim,
                    const int32_t* kinds, const void* const* tables, const int32_t* vocab, int n_types,
                    const float* fourier_freqs, const float* fourier_phases, int freq_sets, float fourier_scale,
                    void* out, int out_f32, mb_stream_t stream) {
  if (tokens < 0 || dim <= 0 || n_types < 0 || freq_sets < 0)
    return fail(MB_ERR_INVALID_ARG, "tokens >= 0, dim > 0, n_types >= 0 and freq_sets >= 0 required");
  if (tokens == 0) return MB_OK;
  if (dim % (out_f32 ? 4 : 8)) return fail(MB_ERR_UNSUPPORTED, "dim must be a multiple of 16 bytes of elements");
  if (!types || !ids || !scalars || !out || (n_types > 0 && (!kinds || !tables || !vocab)))
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (freq_sets > 0 && (!fourier_freqs || !fourier_phases))
    return fail(MB_ERR_INVALID_ARG, "Fourier banks need freqs and phases");
  if (!aligned(out, 16)) return fail(MB_ERR_INVALID_ARG, "out must be 16-byte aligned");
  mb::EmbedParams p{};
  p.types = types;
  p.ids = ids;
  p.scalars = scalars;
  p.L = tokens;
  p.D = dim;
  p.n_types = n_types;
  p.kinds = kinds;
  p.tables = tables;
  p.vocab = vocab;
  p.freqs = fourier_freqs;
  p.phases = fourier_phases;
  p.freq_sets = freq_sets;
  p.fourier_scale = fourier_scale;
  p.out = out;
  cudaError_t e = mb::launch_embed_tokens(p, out_f32 != 0, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "embed tokens launch");
}

size_t mb_td_loss_scratch_bytes(int n) {
  if (n <= 0) return 0;
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  return up((size_t)n * 4) * 2 + up((size_t)mb::td_blocks(n) * 6 * 4) + 256 + up((size_t)n);
}

namespace {
int td_params(const float* q, const float* q_target, const int64_t* action, const float* reward, const int64_t* done,
              const int64_t* seq, int n, int actions, const float* gammas, float cql_weight, float cql_eps,
              void* scratch, size_t scratch_bytes, float* out, mb::TdParams* p) {
  if (n < 2) return fail(MB_ERR_INVALID_ARG, "Not enough valid q values in data.");
  if (actions <= 0) return fail(MB_ERR_INVALID_ARG, "actions must be > 0");
  if (!q || !action || !out || !scratch) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  const size_t need = mb_td_loss_scratch_bytes(n);
  if (scratch_bytes < need || !aligned(scratch, 256))
    return fail(MB_ERR_WORKSPACE, "TD loss scratch needs " + std::to_string(need) + " bytes, 256-byte aligned");
  auto up = [](size_t x) { return (x + 255) & ~size_t(255); };
  uint8_t* base = static_cast<uint8_t*>(scratch);
  size_t o = 0;
  p->err = reinterpret_cast<float*>(base + o);       o += up((size_t)n * 4);
  p->cql_scale = reinterpret_cast<float*>(base + o); o += up((size_t)n * 4);
  p->partials = reinterpret_cast<float*>(base + o);  o += up((size_t)mb::td_blocks(n) * 6 * 4);
  p->ticket = reinterpret_cast<int*>(base + o);      o += 256;
  p->valid = base + o;
  p->q = q;
  p->q_target = q_target;
  p->action = action;
  p->reward = reward;
  p->done = done;
  p->seq = seq;
  p->N = n;
  p->A = actions;
  for (int k = 0; k < 5; ++k) p->gamma[k] = gammas ? gammas[k] : 0.f;
  p->cql_weight = cql_weight;
  p->cql_eps = cql_eps;
  p->out = out;
  return MB_OK;
}
}  // namespace

int mb_td_loss_fwd(const float* q, const float* q_target, const int64_t* action, const float* reward,
                   const int64_t* done, const int64_t* sequence_id, int n, int actions, const float* gammas,
                   float cql_weight, float cql_eps, void* scratch, size_t scratch_bytes, float* out,
                   mb_stream_t stream) {
  mb::TdParams p{};
  int rc = td_params(q, q_target, action, reward, done, sequence_id, n, actions, gammas, cql_weight, cql_eps,
                     scratch, scratch_bytes, out, &p);
  if (rc) return rc;
  if (!q_target || !reward || !done || !gammas) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = mb::launch_td_loss_fwd(p, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "td loss forward launch");
}

int mb_td_loss_bwd(const float* q, const int64_t* action, int n, int actions, float cql_weight, void* scratch,
                   size_t scratch_bytes, const float* out, const float* grad_out, float* dq, mb_stream_t stream) {
  mb::TdParams p{};
  int rc = td_params(q, nullptr, action, nullptr, nullptr, nullptr, n, actions, nullptr, cql_weight, 0.f, scratch,
                     scratch_bytes, const_cast<float*>(out), &p);
  if (rc) return rc;
  if (!dq) return fail(MB_ERR_INVALID_ARG, "dq is NULL");
  p.dq = dq;
  cudaError_t e = mb::launch_td_loss_bwd(p, grad_out, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "td loss backward launch");
}

int mb_silu_mul(const void* gate_up, int rows, int inter, void* out, mb_stream_t stream) {
  if (rows < 0 || inter <= 0 || inter % 2) return fail(MB_ERR_INVALID_ARG, "rows >= 0 and an even inter required");
  if (rows == 0) return MB_OK;
  if (!gate_up || !out || !aligned(gate_up, 4) || !aligned(out, 4))
    return fail(MB_ERR_INVALID_ARG, "NULL or misaligned pointer");
  cudaError_t e = mb::launch_silu_mul(static_cast<const __nv_bfloat16*>(gate_up), rows, inter,
                                      static_cast<__nv_bfloat16*>(out), (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "silu_mul launch");
}

int mb_varlen_attention_fwd(const void* q, const void* k, const void* v, int L, int q_heads, int kv_heads,
                            int head_dim, const int32_t* run_start, const int32_t* tile_lo, float scale, void* out,
                            float* lse, mb_stream_t stream) {
  if (L < 0 || q_heads <= 0 || kv_heads <= 0) return fail(MB_ERR_INVALID_ARG, "L >= 0 and head counts > 0 required");
  if (q_heads % kv_heads) return fail(MB_ERR_INVALID_ARG, "q_heads must be a multiple of kv_heads");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (L == 0) return MB_OK;
  if (!q || !k || !v || !run_start || !tile_lo || !out || !lse)
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
    return fail(MB_ERR_INVALID_ARG, "q, k, v and out must be 16-byte aligned");
  CUtensorMap qm, km, vm;
  int rc;
  if ((rc = encode_token_map(&qm, q, L, q_heads, head_dim))) return rc;
  if ((rc = encode_token_map(&km, k, L, kv_heads, head_dim))) return rc;
  if ((rc = encode_token_map(&vm, v, L, kv_heads, head_dim))) return rc;
  mb::VarlenParams p{};
  p.L = L;
  p.Hq = q_heads;
  p.Hkv = kv_heads;
  p.G = q_heads / kv_heads;
  p.heads_per_cta = (p.G % 2 == 0) ? 2 : 1;
  p.head_dim = head_dim;
  p.run_start = run_start;
  p.tile_lo = tile_lo;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.out = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.tile_counter = reinterpret_cast<int*>(lse + (size_t)q_heads * L);
  cudaError_t e = mb::launch_varlen_fwd(qm, km, vm, p, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "varlen attention forward launch");
}

namespace {

// Shared body of the two backward entry points; ds == nullptr selects the
// recompute path.
int varlen_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout, const float* lse,
               int L, int q_heads, int kv_heads, int head_dim, const int32_t* run_start, const int32_t* run_end,
               const int32_t* tile_lo, const int32_t* pair_off, int n_pairs, float scale, void* dq, void* dk,
               void* dv, float* delta, void* ds, size_t ds_bytes, mb_stream_t stream) {
  if (L < 0 || q_heads <= 0 || kv_heads <= 0) return fail(MB_ERR_INVALID_ARG, "L >= 0 and head counts > 0 required");
  if (q_heads % kv_heads) return fail(MB_ERR_INVALID_ARG, "q_heads must be a multiple of kv_heads");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if (L == 0) return MB_OK;
  if (!q || !k || !v || !out || !dout || !lse || !run_start || !run_end || !dq || !dk || !dv || !delta)
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(dout, 16) || !aligned(dq, 16) ||
      !aligned(dk, 16) || !aligned(dv, 16) || !aligned(out, 4))
    return fail(MB_ERR_INVALID_ARG, "q, k, v, dout, dq, dk, dv must be 16-byte aligned");
  CUtensorMap qm, km, vm, dm;
  int rc;
  if (ds) {
    const long long tiles = (L + 127) / 128;
    if (!tile_lo || !pair_off) return fail(MB_ERR_INVALID_ARG, "the stored-dS path needs tile_lo and pair_off");
    if (n_pairs < tiles) return fail(MB_ERR_INVALID_ARG, "n_pairs must be at least ceil(L / 128)");
    if (ds_bytes < MB_VARLEN_BWD_DS_BYTES(q_heads, n_pairs))
      return fail(MB_ERR_WORKSPACE, "ds scratch smaller than MB_VARLEN_BWD_DS_BYTES(q_heads, n_pairs)");
    if (!aligned(ds, 16)) return fail(MB_ERR_INVALID_ARG, "ds scratch must be 16-byte aligned");
  }
  if ((rc = encode_token_map(&qm, q, L, q_heads, head_dim))) return rc;
  if ((rc = encode_token_map(&km, k, L, kv_heads, head_dim))) return rc;
  if ((rc = encode_token_map(&vm, v, L, kv_heads, head_dim))) return rc;
  if ((rc = encode_token_map(&dm, dout, L, q_heads, head_dim))) return rc;
  mb::VarlenBwdParams p{};
  p.L = L;
  p.Hq = q_heads;
  p.Hkv = kv_heads;
  p.G = q_heads / kv_heads;
  p.head_dim = head_dim;
  p.run_start = run_start;
  p.run_end = run_end;
  p.lse = lse;
  p.delta = delta;
  p.tile_counter = reinterpret_cast<int*>(delta + (size_t)q_heads * L);
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.dq = static_cast<__nv_bfloat16*>(dq);
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  p.tile_lo = tile_lo;
  p.pair_off = pair_off;
  p.n_pairs = ds ? n_pairs : 0;
  p.ds = static_cast<__nv_bfloat16*>(ds);
  cudaError_t e = mb::launch_varlen_bwd(qm, km, vm, dm, static_cast<const __nv_bfloat16*>(out),
                                        static_cast<const __nv_bfloat16*>(dout), p, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "varlen attention backward launch");
}

}  // namespace

int mb_varlen_attention_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout,
                            const float* lse, int L, int q_heads, int kv_heads, int head_dim,
                            const int32_t* run_start, const int32_t* run_end, float scale, void* dq, void* dk,
                            void* dv, float* delta, mb_stream_t stream) {
  return varlen_bwd(q, k, v, out, dout, lse, L, q_heads, kv_heads, head_dim, run_start, run_end, nullptr, nullptr, 0,
                    scale, dq, dk, dv, delta, nullptr, 0, stream);
}

int mb_varlen_bwd_pair_offsets(const int32_t* tile_lo, int L, int32_t* pair_off, mb_stream_t stream) {
  if (L < 0) return fail(MB_ERR_INVALID_ARG, "L must be >= 0");
  if (!pair_off || (L > 0 && !tile_lo)) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = mb::launch_varlen_pair_offsets(tile_lo, L, pair_off, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "pair offsets launch");
}

int mb_varlen_attention_bwd_stored(const void* q, const void* k, const void* v, const void* out, const void* dout,
                                   const float* lse, int L, int q_heads, int kv_heads, int head_dim,
                                   const int32_t* run_start, const int32_t* run_end, const int32_t* tile_lo,
                                   const int32_t* pair_off, int n_pairs, float scale, void* dq, void* dk, void* dv,
                                   float* delta, void* ds_scratch, size_t ds_bytes, mb_stream_t stream) {
  if (L > 0 && !ds_scratch) return fail(MB_ERR_INVALID_ARG, "ds_scratch is NULL");
  return varlen_bwd(q, k, v, out, dout, lse, L, q_heads, kv_heads, head_dim, run_start, run_end, tile_lo, pair_off,
                    n_pairs, scale, dq, dk, dv, delta, ds_scratch, ds_bytes, stream);
}

// ---------------------------------------------------------------- decode-step layout glue (K9)

int mb_flat_rank(const int64_t* sequence_ids, int L, int batch, const int64_t* prediction_indices, int n_pred,
                 const int32_t* step_counts, const int32_t* step_offsets, int steps, int32_t* rank, int32_t* stats,
                 int64_t* local_indices, mb_stream_t stream) {
  if (L < 0 || batch < 0 || n_pred < 0 || steps < 0) return fail(MB_ERR_INVALID_ARG, "sizes must be >= 0");
  if (batch > MB_FLAT_RANK_MAX_BATCH) return fail(MB_ERR_UNSUPPORTED, "batch above MB_FLAT_RANK_MAX_BATCH");
  if (!stats || (L > 0 && (!sequence_ids || !rank)) || (batch > 0 && steps > 0 && (!step_counts || !step_offsets ||
                                                                                    !local_indices)) ||
      (n_pred > 0 && !prediction_indices))
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = mb::launch_flat_rank(sequence_ids, L, batch, prediction_indices, n_pred, step_counts, step_offsets,
                                       steps, rank, stats, local_indices, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "flat rank launch");
}

int mb_flat_scatter(const void* embeds, int L, int row_bytes, const int64_t* sequence_ids, const int32_t* rank,
                    int batch, int max_len, void* out, mb_stream_t stream) {
  if (L < 0 || row_bytes <= 0 || batch < 0 || max_len < 0) return fail(MB_ERR_INVALID_ARG, "bad sizes");
  const size_t out_bytes = (size_t)batch * (size_t)max_len * (size_t)row_bytes;
  if (out_bytes == 0) return MB_OK;
  if (!out || (L > 0 && (!embeds || !sequence_ids || !rank))) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = cudaMemsetAsync(out, 0, out_bytes, (cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "flat scatter zero fill");
  if (L == 0) return MB_OK;
  e = mb::launch_flat_scatter(embeds, L, row_bytes, sequence_ids, rank, max_len, out, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "flat scatter launch");
}

int mb_left_align(const void* embeds, int batch, int L, int row_bytes, const int64_t* prediction_indices, int steps,
                  void* aligned, int64_t* aligned_indices, mb_stream_t stream) {
  if (batch < 0 || L < 0 || row_bytes <= 0 || steps <= 0)
    return fail(MB_ERR_INVALID_ARG, "batch, L >= 0, row_bytes > 0 and steps >= 1 required");
  if (batch == 0) return MB_OK;
  if (!prediction_indices || !aligned_indices || (L > 0 && (!embeds || !aligned)))
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = mb::launch_left_align(embeds, batch, L, row_bytes, prediction_indices, steps, aligned,
                                        aligned_indices, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "left align launch");
}

int mb_segment_meta(const int64_t* sequence_ids, int L, int tile, int64_t* position, int32_t* run_start,
                    int32_t* run_end, int32_t* tile_lo, int32_t* flags, mb_stream_t stream) {
  if (L < 0 || tile <= 0) return fail(MB_ERR_INVALID_ARG, "L must be >= 0 and tile > 0");
  if (L == 0) return MB_OK;
  if (!sequence_ids || !position || !run_start || !tile_lo || !flags)
    return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  cudaError_t e = mb::launch_segment_meta(sequence_ids, L, tile, position, run_start, run_end, tile_lo, flags,
                                          (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "segment meta launch");
}

// ---------------------------------------------------------------- training element-wise (K4)

namespace {
int check_norm_dim(int rows, int dim) {
  if (rows < 0) return fail(MB_ERR_INVALID_ARG, "rows must be >= 0");
  if (dim <= 0 || dim % 256 || dim > 2048) return fail(MB_ERR_UNSUPPORTED, "dim must be a multiple of 256, <= 2048");
  return MB_OK;
}

int check_head_shape(int L, int heads, int head_dim) {
  if (L < 0 || heads <= 0) return fail(MB_ERR_INVALID_ARG, "L >= 0 and heads > 0 required");
  if (head_dim != 64 && head_dim != 128) return fail(MB_ERR_UNSUPPORTED, "head_dim must be 64 or 128");
  if ((long long)L * heads > 0x7fffffffLL) return fail(MB_ERR_UNSUPPORTED, "L * heads must be below 2^31");
  return MB_OK;
}
}  // namespace

int mb_rmsnorm_fwd(const void* x, const void* weight, float eps, int rows, int dim, void* y, float* rstd,
                   mb_stream_t stream) {
  if (int rc = check_norm_dim(rows, dim)) return rc;
  if (rows == 0) return MB_OK;
  if (!x || !weight || !y || !rstd) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(x, 16) || !aligned(weight, 16) || !aligned(y, 16))
    return fail(MB_ERR_INVALID_ARG, "x, weight and y must be 16-byte aligned");
  cudaError_t e = mb::launch_rmsnorm_fwd(static_cast<const __nv_bfloat16*>(x), nullptr,
                                         static_cast<const __nv_bfloat16*>(weight), eps, rows, dim, nullptr,
                                         static_cast<__nv_bfloat16*>(y), rstd, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "rmsnorm fwd launch");
}

int mb_add_rmsnorm_fwd(const void* x, const void* residual, const void* weight, float eps, int rows, int dim,
                       void* sum_out, void* y, float* rstd, mb_stream_t stream) {
  if (int rc = check_norm_dim(rows, dim)) return rc;
  if (rows == 0) return MB_OK;
  if (!x || !residual || !weight || !sum_out || !y || !rstd) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(x, 16) || !aligned(residual, 16) || !aligned(weight, 16) || !aligned(sum_out, 16) || !aligned(y, 16))
    return fail(MB_ERR_INVALID_ARG, "x, residual, weight, sum_out and y must be 16-byte aligned");
  cudaError_t e = mb::launch_rmsnorm_fwd(static_cast<const __nv_bfloat16*>(x), static_cast<const __nv_bfloat16*>(residual),
                                         static_cast<const __nv_bfloat16*>(weight), eps, rows, dim,
                                         static_cast<__nv_bfloat16*>(sum_out), static_cast<__nv_bfloat16*>(y), rstd,
                                         (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "add rmsnorm fwd launch");
}

size_t mb_rmsnorm_bwd_scratch_floats(int rows, int dim) {
  if (rows <= 0 || dim <= 0) return 0;
  if (dim % 256 || dim > 2048) return 0;
  return (size_t)mb::rmsnorm_bwd_partials(rows, dim) * (size_t)dim;
}

namespace {

int rmsnorm_bwd_common(const void* dy, const void* x, const void* weight, const float* rstd, const void* dsum,
                       int rows, int dim, void* dx, float* dweight, float* scratch, size_t scratch_floats,
                       mb_stream_t stream) {
  if (int rc = check_norm_dim(rows, dim)) return rc;
  if (!dweight) return fail(MB_ERR_INVALID_ARG, "dweight is NULL");
  if (rows > 0) {
    if (!dy || !x || !weight || !rstd || !dx || !scratch) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
    if (scratch_floats < mb_rmsnorm_bwd_scratch_floats(rows, dim))
      return fail(MB_ERR_INVALID_ARG, "scratch is smaller than mb_rmsnorm_bwd_scratch_floats");
    if (!aligned(dy, 16) || !aligned(x, 16) || !aligned(weight, 16) || !aligned(dx, 16))
      return fail(MB_ERR_INVALID_ARG, "dy, x, weight and dx must be 16-byte aligned");
  }
  if (dsum && !aligned(dsum, 16)) return fail(MB_ERR_INVALID_ARG, "dsum must be 16-byte aligned");
  cudaError_t e = mb::launch_rmsnorm_bwd(static_cast<const __nv_bfloat16*>(dy), static_cast<const __nv_bfloat16*>(x),
                                         static_cast<const __nv_bfloat16*>(weight), rstd,
                                         static_cast<const __nv_bfloat16*>(dsum), rows, dim,
                                         static_cast<__nv_bfloat16*>(dx), scratch, dweight, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "rmsnorm bwd launch");
}

}  // namespace

int mb_rmsnorm_bwd(const void* dy, const void* x, const void* weight, const float* rstd, int rows, int dim, void* dx,
                   float* dweight, float* scratch, size_t scratch_floats, mb_stream_t stream) {
  return rmsnorm_bwd_common(dy, x, weight, rstd, nullptr, rows, dim, dx, dweight, scratch, scratch_floats, stream);
}

int mb_rmsnorm_bwd_add(const void* dy, const void* x, const void* weight, const float* rstd, const void* dsum,
                       int rows, int dim, void* dx, float* dweight, float* scratch, size_t scratch_floats,
                       mb_stream_t stream) {
  if (rows > 0 && !dsum) return fail(MB_ERR_INVALID_ARG, "dsum is NULL");
  return rmsnorm_bwd_common(dy, x, weight, rstd, dsum, rows, dim, dx, dweight, scratch, scratch_floats, stream);
}

int mb_qkv_heads_fwd(const void* qkv, long long qkv_row_stride, int L, int q_heads, int kv_heads, int head_dim,
                     const void* q_norm_weight, const void* k_norm_weight, float q_eps, float k_eps, const void* cos,
                     const void* sin, void* q, void* k, void* v, float* q_rstd, float* k_rstd, mb_stream_t stream) {
  if (int rc = check_head_shape(L, q_heads + 2 * kv_heads, head_dim)) return rc;
  if (kv_heads <= 0 || q_heads <= 0) return fail(MB_ERR_INVALID_ARG, "head counts must be > 0");
  if (!q_norm_weight != !k_norm_weight) return fail(MB_ERR_INVALID_ARG, "pass both norm weights or neither");
  if (L == 0) return MB_OK;
  if (!qkv || !cos || !sin || !q || !k || !v) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (q_norm_weight && (!q_rstd || !k_rstd)) return fail(MB_ERR_INVALID_ARG, "the norm needs q_rstd and k_rstd");
  if (qkv_row_stride < (long long)(q_heads + 2 * kv_heads) * head_dim || qkv_row_stride % 8)
    return fail(MB_ERR_INVALID_ARG, "qkv_row_stride must be a multiple of 8 and >= (q_heads + 2 kv_heads) * head_dim");
  const void* ptrs[] = {qkv, cos, sin, q, k, v, q_norm_weight, k_norm_weight};
  for (const void* p : ptrs)
    if (p && !aligned(p, 16)) return fail(MB_ERR_INVALID_ARG, "tensors must be 16-byte aligned");
  cudaError_t e = mb::launch_qkv_heads_fwd(
      static_cast<const __nv_bfloat16*>(qkv), qkv_row_stride, L, q_heads, kv_heads, head_dim,
      static_cast<const __nv_bfloat16*>(q_norm_weight), static_cast<const __nv_bfloat16*>(k_norm_weight), q_eps,
      k_eps, static_cast<const __nv_bfloat16*>(cos), static_cast<const __nv_bfloat16*>(sin),
      static_cast<__nv_bfloat16*>(q), static_cast<__nv_bfloat16*>(k), static_cast<__nv_bfloat16*>(v), q_rstd, k_rstd,
      (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "qkv heads fwd launch");
}

size_t mb_qkv_heads_bwd_scratch_floats(int L, int head_dim) {
  if (L <= 0 || (head_dim != 64 && head_dim != 128)) return 0;
  return (size_t)mb::qkv_heads_bwd_partials(L, head_dim) * 2 * (size_t)head_dim;
}

int mb_qkv_heads_bwd(const void* dq, const void* dk, const void* dv, const void* qkv, long long qkv_row_stride,
                     int L, int q_heads, int kv_heads, int head_dim, const void* q_norm_weight,
                     const void* k_norm_weight, const void* cos, const void* sin, const float* q_rstd,
                     const float* k_rstd, void* dqkv, long long dqkv_row_stride, float* dq_norm_weight,
                     float* dk_norm_weight, float* scratch, size_t scratch_floats, mb_stream_t stream) {
  if (int rc = check_head_shape(L, q_heads + 2 * kv_heads, head_dim)) return rc;
  if (kv_heads <= 0 || q_heads <= 0) return fail(MB_ERR_INVALID_ARG, "head counts must be > 0");
  const bool norm = q_norm_weight != nullptr;
  if (norm != (k_norm_weight != nullptr)) return fail(MB_ERR_INVALID_ARG, "pass both norm weights or neither");
  if (norm && (!dq_norm_weight || !dk_norm_weight)) return fail(MB_ERR_INVALID_ARG, "norm weights need dweights");
  if (L > 0) {
    if (!dq || !dk || !dv || !cos || !sin || !dqkv) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
    if (norm && (!qkv || !q_rstd || !k_rstd || !scratch))
      return fail(MB_ERR_INVALID_ARG, "the norm needs qkv, q_rstd, k_rstd and scratch");
    if (norm && scratch_floats < mb_qkv_heads_bwd_scratch_floats(L, head_dim))
      return fail(MB_ERR_INVALID_ARG, "scratch is smaller than mb_qkv_heads_bwd_scratch_floats");
    const long long need = (long long)(q_heads + 2 * kv_heads) * head_dim;
    if (dqkv_row_stride < need || dqkv_row_stride % 8 || (norm && (qkv_row_stride < need || qkv_row_stride % 8)))
      return fail(MB_ERR_INVALID_ARG, "row strides must be multiples of 8 and >= (q_heads + 2 kv_heads) * head_dim");
    const void* ptrs[] = {dq, dk, dv, qkv, cos, sin, dqkv, q_norm_weight, k_norm_weight};
    for (const void* p : ptrs)
      if (p && !aligned(p, 16)) return fail(MB_ERR_INVALID_ARG, "tensors must be 16-byte aligned");
  }
  cudaError_t e = mb::launch_qkv_heads_bwd(
      static_cast<const __nv_bfloat16*>(dq), static_cast<const __nv_bfloat16*>(dk),
      static_cast<const __nv_bfloat16*>(dv), static_cast<const __nv_bfloat16*>(qkv), qkv_row_stride, L, q_heads,
      kv_heads, head_dim, static_cast<const __nv_bfloat16*>(q_norm_weight),
      static_cast<const __nv_bfloat16*>(k_norm_weight), static_cast<const __nv_bfloat16*>(cos),
      static_cast<const __nv_bfloat16*>(sin), q_rstd, k_rstd, static_cast<__nv_bfloat16*>(dqkv), dqkv_row_stride,
      dq_norm_weight, dk_norm_weight, scratch, (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "qkv heads bwd launch");
}

int mb_silu_mul_bwd(const void* gate_up, const void* dh, int rows, int inter, void* dgate_up, mb_stream_t stream) {
  if (rows < 0 || inter <= 0 || inter % 2) return fail(MB_ERR_INVALID_ARG, "rows >= 0 and an even inter required");
  if (rows == 0) return MB_OK;
  if (!gate_up || !dh || !dgate_up) return fail(MB_ERR_INVALID_ARG, "a required pointer is NULL");
  if (!aligned(gate_up, 4) || !aligned(dh, 4) || !aligned(dgate_up, 4))
    return fail(MB_ERR_INVALID_ARG, "buffers must be 4-byte aligned");
  cudaError_t e = mb::launch_silu_mul_bwd(static_cast<const __nv_bfloat16*>(gate_up),
                                          static_cast<const __nv_bfloat16*>(dh), rows, inter,
                                          static_cast<__nv_bfloat16*>(dgate_up), (cudaStream_t)stream);
  return e == cudaSuccess ? MB_OK : cuda_fail(e, "silu_mul bwd launch");
}

}  // extern "C"
