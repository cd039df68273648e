// Internal declarations shared by the kernel files and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <algorithm>

namespace mb {

struct AttnParams {
  const __nv_bfloat16* q;      // [B, S, Hq, HD]
  __nv_bfloat16* out;          // [B, S, Hq, HD]
  const int32_t* block_table;  // [B, max_pages]
  const int32_t* q_pos;        // [B, S]
  const int32_t* kv_len;       // [B]
  int B, S, Hq, Hkv, G, R, head_dim;
  int max_pages, page_size, num_pages;
  int chunk_tokens;
  float scale_log2;
  // split-mode work list (inside the caller's workspace)
  const int2* entries;
  const int* n_entries;
  const int* row_start;
  const int* row_chunks;
  int* counters;
  const int* order;            // entries, longest chunk first (the order CTAs take work in)
  const int* n_order;          // entries in `order`
  const int* width;            // per entry: member mask of its item (bit k: row + k; 1 alone; 0 covered)
  const int* kv_bound;         // per entry: a member's key end inside a shared chunk (0: the whole chunk)
  const int* t_from;           // per entry: a tail item's first token (-1: the chunk's start)
  int* work;                   // [2]: next work item, CTAs finished (zeroed by the plan and the last CTA)
  float* part_lse;
  float* part_o;
};

struct WorkspaceLayout {
  size_t max_entries;
  size_t entries, n_entries, row_start, row_chunks, counters, order, n_order, width, kv_bound, t_from, work,
      part_lse, part_o;
  size_t total;
};

size_t decode_chunk_tokens(int head_dim);
size_t decode_workspace_layout(int B, int Hkv, int R, int head_dim, int max_kv_len, WorkspaceLayout* lay);
// block_table == nullptr: every (row, chunk) is its own item. Otherwise the
// plan also finds chunks whose pages consecutive rows share (see the plan
// kernel) and gives each run one item; the caller's queries must see every
// cached slot (q_pos[b, s] >= kv_len[b] - q_rows).
cudaError_t launch_decode_plan(const int32_t* kv_len, const int32_t* block_table, int max_pages, int page_size,
                               int B, int Hkv, int q_rows, int head_dim, const WorkspaceLayout& lay, uint8_t* ws,
                               cudaStream_t stream);
cudaError_t launch_decode_attention(const CUtensorMap& km, const CUtensorMap& vm, AttnParams p,
                                    const WorkspaceLayout& lay, uint8_t* ws, bool split, cudaStream_t stream);

struct AppendParams {
  const __nv_bfloat16* qkv;  // [T, qkv_stride]: q | k | v (bf16), or
  const float* qkv_f32;      // the same in fp32 (exactly one of the two is set)
  int T, qkv_stride;
  const int32_t* pos;        // [T] RoPE position
  const int32_t* slot;       // [T] page * page_size + offset, or -1 (not cached)
  const __nv_bfloat16* q_norm_w;  // [HD] or null
  const __nv_bfloat16* k_norm_w;  // [HD] or null
  float eps;
  const float* inv_freq;     // [HD/2]
  float attn_scaling;
  int Hq, Hkv, head_dim, page_size;
  __nv_bfloat16* q_out;      // [T, Hq, HD]
  __nv_bfloat16* k_out;      // [T, Hkv, HD] or null (contiguous copy of the new keys)
  __nv_bfloat16* v_out;      // [T, Hkv, HD] or null
  __nv_bfloat16* k_pool;     // [P, Hkv, page, HD] or null
  __nv_bfloat16* v_pool;
  long long num_slots;       // P * page_size (slot bound check)
};
cudaError_t launch_append(const AppendParams& p, cudaStream_t stream);

// K13 (qkv_append.cu): the QKV GEMM of the decode layer with K2 as its
// epilogue. x [T, K] and W [N, K] bf16 come through the tensor maps.
struct QkvAppendParams {
  int T, K, N;                    // tokens, hidden size, (Hq + 2 Hkv) * HD (a multiple of 128)
  int Hq, Hkv, head_dim, page_size;
  const __nv_bfloat16* bias;      // [N] or null
  const float2* rope;             // [T, HD/2] (cos, sin) * attention scaling, from launch_rope_table
  const __nv_bfloat16* q_norm_w;  // [HD] or null
  const __nv_bfloat16* k_norm_w;  // [HD] or null
  float eps;
  const int32_t* slot;            // [T] page * page_size + offset, or -1 (not cached); null: none cached
  long long num_slots;            // P * page_size (slot bound check), 0 without pools
  __nv_bfloat16* q_out;           // [T, Hq, HD]
  __nv_bfloat16* k_pool;          // [P, Hkv, page, HD] or null
  __nv_bfloat16* v_pool;
};
cudaError_t launch_qkv_append(const CUtensorMap& xm, const CUtensorMap& wm, const QkvAppendParams& p,
                              cudaStream_t stream);
cudaError_t launch_rope_table(const int32_t* pos, int T, const float* inv_freq, int head_dim, float attn_scaling,
                              float* table, cudaStream_t stream);

cudaError_t launch_page_copy(const __nv_bfloat16* src_pool, __nv_bfloat16* dst_pool, const int32_t* src_pages,
                             const int32_t* dst_pages, int n, long long page_elems, cudaStream_t stream);

cudaError_t launch_rmsnorm(const __nv_bfloat16* x, const __nv_bfloat16* residual, const __nv_bfloat16* w,
                           float eps, int rows, int D, __nv_bfloat16* sum_out, __nv_bfloat16* norm_out,
                           cudaStream_t stream);
cudaError_t launch_silu_mul(const __nv_bfloat16* gate_up, int rows, int I, __nv_bfloat16* out, cudaStream_t stream);
// fp32 residual stream variants: sum = x (+ delta) kept in fp32, norm rounded
// once to bf16; SiLU product of an fp32 gate|up rounded once to bf16.
cudaError_t launch_rmsnorm_f32(const float* x, const __nv_bfloat16* x_bf16, const float* delta,
                               const __nv_bfloat16* w, float eps, int rows, int D, float* sum_out,
                               __nv_bfloat16* norm_out, cudaStream_t stream);
cudaError_t launch_silu_mul_f32(const float* gate_up, int rows, int I, __nv_bfloat16* out, cudaStream_t stream);

struct VarlenParams {
  int L, Hq, Hkv, G, heads_per_cta, head_dim;
  const int32_t* run_start;  // [L]
  const int32_t* tile_lo;    // [ceil(L / 128)]
  float scale_log2;
  __nv_bfloat16* out;        // [L, Hq, HD]
  float* lse;                // [Hq, L], log2 units
  int* tile_counter;         // [1] scratch: the persistent kernel's tile counter
  // Paged prefill (the same kernel over a decode session's page pool):
  // queries [B * S, Hq, HD] (row b * S + s), query (b, s) sees the cached
  // keys 0 .. q_pos[b, s] of row b through block_table; out [B * S, Hq, HD];
  // no lse. One CTA per work tile (tile_counter unused).
  const int32_t* block_table;  // [B, max_pages]
  const int32_t* q_pos;        // [B, S]
  const int32_t* kv_len;       // [B]
  int B, S, max_pages, page_size, num_pages;
};
cudaError_t launch_varlen_fwd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                              const VarlenParams& p, cudaStream_t stream);
// qm: 3-D token map over the B * S query rows; km / vm: 2-D 64 x 64-box maps
// of one layer's K / V pool (the decode kernel's maps).
cudaError_t launch_paged_prefill(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                                 const VarlenParams& p, cudaStream_t stream);

struct VarlenBwdParams {
  int L, Hq, Hkv, G, head_dim;
  const int32_t* run_start;  // [L]
  const int32_t* run_end;    // [L]
  const float* lse;          // [Hq, L] log2 units (from the forward)
  float* delta;              // [Hq, L] scratch: rowsum(dO * O)
  int* tile_counter;         // [2] scratch: tile counters of the persistent kernels
  float scale, scale_log2;
  __nv_bfloat16* dq;         // [L, Hq, HD]
  __nv_bfloat16* dk;         // [L, Hkv, HD]
  __nv_bfloat16* dv;         // [L, Hkv, HD]
  // Stored-dS path (ds != nullptr): the dK/dV kernel writes each (q-head,
  // query tile i, key tile j) block of dS^T to
  // ds + ((h * n_pairs + pair_off[i] + j - tile_lo[i] / 128) * 128 * 128),
  // element (key r, query c) at (c / 8) * 1024 + r * 8 + c % 8, and dQ is one
  // GEMM over those blocks.
  const int32_t* tile_lo;    // [ceil(L/128)] run_start of each query tile's first token
  const int32_t* pair_off;   // [ceil(L/128) + 1]
  int n_pairs;
  __nv_bfloat16* ds;
};
cudaError_t launch_varlen_bwd(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm,
                              const CUtensorMap& dom, const __nv_bfloat16* out, const __nv_bfloat16* dout,
                              VarlenBwdParams p, cudaStream_t stream);
cudaError_t launch_varlen_pair_offsets(const int32_t* tile_lo, int L, int32_t* pair_off, cudaStream_t stream);

// Decode-step layout glue (packing.cu).
cudaError_t launch_flat_rank(const int64_t* seq, int L, int B, const int64_t* pred, int N, const int32_t* steps,
                             const int32_t* step_off, int S, int32_t* rank, int32_t* stats, int64_t* local,
                             cudaStream_t stream);
cudaError_t launch_flat_scatter(const void* emb, int L, int row_bytes, const int64_t* seq, const int32_t* rank,
                                int Lmax, void* out, cudaStream_t stream);
cudaError_t launch_left_align(const void* emb, int B, int L, int row_bytes, const int64_t* pi, int S, void* out,
                              int64_t* out_idx, cudaStream_t stream);

// Training element-wise kernels (train_elementwise.cu).
cudaError_t launch_rmsnorm_fwd(const __nv_bfloat16* x, const __nv_bfloat16* res, const __nv_bfloat16* w, float eps,
                               int rows, int D, __nv_bfloat16* sum, __nv_bfloat16* y, float* rstd,
                               cudaStream_t stream);
int rmsnorm_bwd_partials(int rows, int D);
cudaError_t launch_rmsnorm_bwd(const __nv_bfloat16* dy, const __nv_bfloat16* x, const __nv_bfloat16* w,
                               const float* rstd, const __nv_bfloat16* dsum, int rows, int D, __nv_bfloat16* dx,
                               float* partial, float* dw, cudaStream_t stream);
int qkv_heads_bwd_partials(int L, int HD);
cudaError_t launch_qkv_heads_fwd(const __nv_bfloat16* qkv, long long xs, int L, int Hq, int Hkv, int HD,
                                 const __nv_bfloat16* qw, const __nv_bfloat16* kw, float q_eps, float k_eps,
                                 const __nv_bfloat16* cosv, const __nv_bfloat16* sinv, __nv_bfloat16* q,
                                 __nv_bfloat16* k, __nv_bfloat16* v, float* q_rstd, float* k_rstd,
                                 cudaStream_t stream);
cudaError_t launch_qkv_heads_bwd(const __nv_bfloat16* dq, const __nv_bfloat16* dk, const __nv_bfloat16* dv,
                                 const __nv_bfloat16* qkv, long long xs, int L, int Hq, int Hkv, int HD,
                                 const __nv_bfloat16* qw, const __nv_bfloat16* kw, const __nv_bfloat16* cosv,
                                 const __nv_bfloat16* sinv, const float* q_rstd, const float* k_rstd,
                                 __nv_bfloat16* dqkv, long long dxs, float* dqw, float* dkw, float* partial,
                                 cudaStream_t stream);
cudaError_t launch_silu_mul_bwd(const __nv_bfloat16* gu, const __nv_bfloat16* dh, int rows, int I,
                                __nv_bfloat16* dgu, cudaStream_t stream);

cudaError_t launch_decode_step_meta(int B, int width, int page_size, const int32_t* new_page, int32_t* block_table,
                                    int32_t* q_pos, int32_t* kv_len, int32_t* slot, cudaStream_t stream);

cudaError_t launch_segment_meta(const int64_t* seq, int L, int tile, int64_t* pos_out, int32_t* run_start,
                                int32_t* run_end, int32_t* tile_lo, int32_t* flags, cudaStream_t stream);

// Token embedding (embed.cu).
struct EmbedParams {
  const int32_t* types;        // [L] token type (modality) id
  const int32_t* ids;          // [L] table row, or Fourier bank for Fourier types
  const float* scalars;        // [L] Fourier input
  long long L;
  int D, n_types;
  const int32_t* kinds;        // [n_types]: 0 none, 1 table, 2 Fourier
  const void* const* tables;   // [n_types] device pointers to [vocab, D] rows (table kinds)
  const int32_t* vocab;        // [n_types]
  const float* freqs;          // [freq_sets, D]
  const float* phases;         // [freq_sets, D]
  int freq_sets;
  float fourier_scale;
  void* out;                   // [L, D], the tables' dtype (bf16 or fp32)
};
cudaError_t launch_embed_tokens(const EmbedParams& p, bool out_f32, cudaStream_t stream);

// TD loss (td_loss.cu).
struct TdParams {
  const float* q;         // [N, A] online action values (fp32)
  const float* q_target;  // [N, A] target action values
  const int64_t* action;  // [N]
  const float* reward;    // [N]
  const int64_t* done;    // [N] done codes 0..4
  const int64_t* seq;     // [N] sequence ids, or null (every pair valid)
  int N, A;
  float gamma[5];
  float cql_weight, cql_eps;
  float* err;             // [N] scratch: per-pair TD error
  uint8_t* valid;         // [N] scratch
  float* cql_scale;       // [N] scratch (CQL only)
  float* partials;        // [blocks * 6] scratch
  int* ticket;            // [1] scratch, zero before the first call (left zero)
  float* out;             // [6]: loss, valid pairs, q mean, std, min, max
  float* dq;              // [N, A] gradient (backward)
};
int td_blocks(int N);
cudaError_t launch_td_loss_fwd(const TdParams& p, cudaStream_t stream);
cudaError_t launch_td_loss_bwd(const TdParams& p, const float* grad_out, cudaStream_t stream);

}  // namespace mb
