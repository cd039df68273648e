/*
 * mouse_b200.h — C ABI of the B200 (sm_100a) attention hot path of mouse-core.
 *
 * Plain pointers, sizes and a CUDA stream; no framework types. Every entry
 * point returns an mb_status (0 = MB_OK) and never throws; the text of the
 * last error on the calling thread is available from mb_last_error(). Device
 * buffers are owned by the caller; the library allocates nothing, frees
 * nothing and starts no host threads. All kernels are enqueued on `stream`.
 *
 * The reference (micahr234/mouse-core v0.4.0) is pure Python; each entry
 * point below names the reference call site it replaces (file:line, paths
 * relative to the reference's src/mouse_core/).
 *
 * Layouts (bf16 unless stated):
 *   q / out        [batch, q_len, q_heads, head_dim]   (== the reference's
 *                  q.transpose(1, 2) of flex_decode.py:218 before the kernel)
 *   k_pool/v_pool  [num_pages, kv_heads, page_size, head_dim], one layer
 *   block_table    int32 [batch, max_pages]: logical page i of row b
 *   q_pos          int32 [batch, q_len]: query (b, s) attends slots 0..q_pos
 *   kv_len         int32 [batch]: slots written for row b (after this call's
 *                  append)
 */
#ifndef MOUSE_B200_H
#define MOUSE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* mb_stream_t; /* a cudaStream_t; NULL = default stream */

enum mb_status {
  MB_OK = 0,
  MB_ERR_INVALID_ARG = 1, /* bad shape, pointer, alignment or size */
  MB_ERR_UNSUPPORTED = 2, /* a shape the kernels are not built for */
  MB_ERR_WORKSPACE = 3,   /* workspace missing or too small */
  MB_ERR_CUDA = 4         /* a CUDA runtime/driver call failed */
};

/* Text of the last error raised on this thread ("" if none). */
const char* mb_last_error(void);

/* ABI version of this library (major * 100 + minor). */
int mb_version(void);

/* Read (and optionally clear) the device status word the kernels report
 * bounded-wait timeouts and out-of-pool page ids through. Synchronizes the
 * device. 0 = healthy; 1 / 2 = a consumer / producer wait ran out; 3 = a page
 * id outside the pool (or a token past the block table); 4 = misaligned
 * dynamic shared memory; 5 = a stored-dS pair index outside the scratch;
 * 6 = a CTA's own copies or MMAs did not complete before it exited; 7 = an embedding id
 * outside its table, or a TD action / done code out of range. */
int mb_device_status(int* status_out, int clear);

/* Diagnostics, no counterpart in the reference (whose kernels come from
 * Inductor and never wait on one another): set how many clock cycles every
 * bounded wait of the kernels on the current device spins after its first
 * failed test before it gives up, records 1 or 2 in the status word and lets
 * its CTA stop cleanly; < 0 restores the default (4e9 cycles, about two
 * seconds). A small value makes a healthy pipeline's waits run out, which is
 * how the timeout path is tested; it applies to kernels launched after the
 * call returns (the call synchronizes the device). */
int mb_set_wait_limit(long long cycles);

/* ---------------------------------------------------------------------
 * Cached decode attention (K1).
 * Replaces models/backbone/flex_decode.py:226-229
 *   self._flex(q, k_cache[li], v_cache[li], block_mask=..., scale=..., enable_gqa=True)
 * with the mask of flex_decode.py:129-134 (kv_idx <= q_pos[b, q]) and the
 * per-call BlockMask build of flex_decode.py:198-202. Slots of row b at or
 * beyond kv_len[b] read as zero, as the reference's zero-filled cache does.
 * ------------------------------------------------------------------- */

/* Bytes of workspace mb_decode_attention needs when q_rows = (q_heads /
 * kv_heads) * q_len <= 16 (split mode); 0 otherwise. max_kv_len bounds
 * kv_len[b] over the batch. */
size_t mb_decode_workspace_bytes(int batch, int kv_heads, int q_rows, int head_dim, int max_kv_len);

/* Build the split-mode work list (row, chunk) from kv_len into `workspace`.
 * It depends only on kv_len, so one plan serves every layer of a step. */
int mb_decode_plan(const int32_t* kv_len, int batch, int kv_heads, int q_rows, int head_dim, int max_kv_len,
                   void* workspace, size_t workspace_bytes, mb_stream_t stream);

/* mb_decode_plan for rows that may share cached pages (forked prefixes,
 * e.g. GRPO branches of one root): rows are grouped in aligned blocks of
 * 16 / q_rows; where rows of a block hold a whole 2048-token chunk on the
 * very same pages as the block's first row that has that chunk, one work
 * item reads the chunk's K/V once for all of their queries (the other rows'
 * entries get no item of their own); a row that holds only the chunk's head
 * on those pages (forked inside the chunk) joins the item for the head and
 * reads the rest of the chunk as an extra item of its own. Outputs equal
 * mb_decode_plan's bit for bit for rows holding whole chunks, and within
 * bf16 rounding for a row whose chunk is split (two partials merged instead
 * of one). Requires
 * every query to see every cached slot of its row (q_pos[b, s] >= kv_len[b]
 * - q_rows, as in one-token decode: q_pos = kv_len - 1), and q_rows <= 8 for
 * any sharing to happen. Replaces nothing in the reference, whose decode
 * session copies a forked prefix per row (flex_decode.py:226-229 reads it
 * per row). */
int mb_decode_plan_shared(const int32_t* kv_len, const int32_t* block_table, int max_pages, int page_size,
                          int batch, int kv_heads, int q_rows, int head_dim, int max_kv_len, void* workspace,
                          size_t workspace_bytes, mb_stream_t stream);

/* out = softmax(scale * q k^T, masked to slots <= q_pos) v, per row and
 * q-head (q-head h reads kv-head h / (q_heads / kv_heads)). head_dim 64 or
 * 128; page_size a multiple of 64. plan_ready = 1 reuses the plan already
 * in `workspace` (built by mb_decode_plan for the same kv_len); 0 builds it.
 * Three schedules: split mode (q_rows <= 16: one-token decode; workspace
 * required); the tcgen05 prefill (q_len >= 64 with q and out 16-byte
 * aligned: 128-query tiles over TMEM accumulators, K/V pages gathered by TMA;
 * a workspace, if given, holds the persistent CTAs' tile counter in its first
 * 4 bytes, otherwise one CTA runs per tile); warp-MMA block mode otherwise. */
int mb_decode_attention(const void* q, const void* k_pool, const void* v_pool, int num_pages,
                        const int32_t* block_table, int max_pages, const int32_t* q_pos, const int32_t* kv_len,
                        int batch, int q_len, int q_heads, int kv_heads, int head_dim, int page_size, float scale,
                        int max_kv_len, int plan_ready, void* out, void* workspace, size_t workspace_bytes,
                        mb_stream_t stream);

/* Scratch size built into the library for mb_decode_attention_noalloc. */
#define MB_NOALLOC_SCRATCH_BYTES (32u * 1024u * 1024u)

/* The same attention as mb_decode_attention, for callers that cannot
 * allocate device memory and so cannot pass a workspace: for example an FFI
 * caller (ctypes, cgo, JNI) that only holds the pointers its framework gave
 * it, or a process whose device memory belongs to another framework's
 * allocator. It has no counterpart in the reference (the reference is Python
 * and its FlexAttention call allocates through torch).
 * Its scratch is an array of MB_NOALLOC_SCRATCH_BYTES compiled into the
 * library, held by every GPU that loads it until the process exits; a shape
 * whose workspace (mb_decode_workspace_bytes) exceeds that is rejected with
 * MB_ERR_WORKSPACE. It calls no allocator. The first call on a device looks
 * up the array's device address (cudaGetSymbolAddress) with that device
 * current; make it before capturing any stream. `stream` must belong to the
 * current device (MB_ERR_INVALID_ARG otherwise). Every call shares the one
 * array and rebuilds its work list and merge counters from scratch, so calls
 * that overlap on the GPU (several streams or host threads at once) race and
 * must be serialised by the caller. */
int mb_decode_attention_noalloc(const void* q, const void* k_pool, const void* v_pool, int num_pages,
                                const int32_t* block_table, int max_pages, const int32_t* q_pos,
                                const int32_t* kv_len, int batch, int q_len, int q_heads, int kv_heads, int head_dim,
                                int page_size, float scale, int max_kv_len, void* out, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Fused q/k RMSNorm + RoPE + paged K/V append (K2).
 * Replaces models/backbone/flex_decode.py:212-224 (q/k projections' norm,
 * apply_rotary_pos_emb with cos/sin from rotary_emb at :204, and the cache
 * scatter k_cache[li][real_rows, :, cache_slots] = ...), and the same norm +
 * RoPE of models/backbone/flex_train.py:137-146.
 *   qkv      [tokens, qkv_stride] = q (q_heads*hd) | k (kv_heads*hd) | v
 *   pos      int32 [tokens] RoPE position; slot int32 [tokens] =
 *            page * page_size + offset, or -1 for tokens not cached
 *   q_norm_w / k_norm_w  [head_dim] or NULL (Llama); inv_freq f32 [hd/2]
 *   q_out    [tokens, q_heads, hd]; k_out / v_out [tokens, kv_heads, hd]
 *            or NULL; k_pool / v_pool one layer's pool or NULL
 * ------------------------------------------------------------------- */
int mb_kv_append(const void* qkv, int tokens, int qkv_stride, const int32_t* pos, const int32_t* slot,
                 const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                 float attention_scaling, int q_heads, int kv_heads, int head_dim, int page_size,
                 long long num_pages, void* q_out, void* k_out, void* v_out, void* k_pool, void* v_pool,
                 mb_stream_t stream);
/* The same with an fp32 qkv (the fp32 output of the QKV projection when the
 * decode session keeps its residual stream in fp32); outputs stay bf16. */
int mb_kv_append_f32(const float* qkv, int tokens, int qkv_stride, const int32_t* pos, const int32_t* slot,
                     const void* q_norm_w, const void* k_norm_w, float eps, const float* inv_freq,
                     float attention_scaling, int q_heads, int kv_heads, int head_dim, int page_size,
                     long long num_pages, void* q_out, void* k_out, void* v_out, void* k_pool, void* v_pool,
                     mb_stream_t stream);

/* ---------------------------------------------------------------------
 * QKV projection with the K2 epilogue (K13, tcgen05).
 * Replaces, per layer of a decode step, the q/k/v projections of
 * models/backbone/flex_decode.py:204-224 together with mb_kv_append_f32:
 * y = x w_qkv^T (+ bias) accumulates in fp32 in tensor memory and goes
 * straight into K2's arithmetic (q/k RMSNorm, RoPE, one rounding to bf16),
 * q to q_out and k/v to their page slots; the fp32 projection is never
 * written. Same outputs as the fp32 GEMM followed by mb_kv_append_f32, up to
 * the GEMM's order of summation.
 *   x [tokens, hidden] bf16 (row-major, 16-byte aligned; hidden % 8 == 0);
 *   w_qkv [(q_heads + 2 kv_heads) * head_dim, hidden] bf16 (q | k | v rows),
 *   a multiple of 128 rows; bias bf16 of that length or NULL;
 *   rope_table [tokens, head_dim / 2] (cos, sin) float pairs from
 *   mb_rope_table for the tokens' positions (one table serves every layer);
 *   q/k norm weights bf16 [head_dim] or NULL; slot [tokens] as for
 *   mb_kv_append (k_pool, v_pool and slot NULL together: q only).
 * mb_rope_table writes (cos, sin)(pos[t] * inv_freq[j]) * attention_scaling,
 * j < head_dim / 2: tokens * head_dim floats, 16-byte aligned.
 * ------------------------------------------------------------------- */
int mb_rope_table(const int32_t* pos, int tokens, const float* inv_freq, int head_dim, float attention_scaling,
                  float* table, mb_stream_t stream);
int mb_qkv_append(const void* x, int tokens, int hidden, const void* w_qkv, const void* bias, const float* rope_table,
                  const void* q_norm_w, const void* k_norm_w, float eps, const int32_t* slot, int q_heads,
                  int kv_heads, int head_dim, int page_size, long long num_pages, void* q_out, void* k_pool,
                  void* v_pool, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Page copy (K3): dst_pool[dst_pages[i]] = src_pool[src_pages[i]] for one
 * layer's pool, page_elems = kv_heads * page_size * head_dim elements.
 * Replaces the whole-cache copy of FlexDecodeSession._grow
 * (models/backbone/flex_decode.py:140-149) for the cases paging still needs
 * a copy: copy-on-write of a shared partial page and rebuild-from-cache.
 * ------------------------------------------------------------------- */
int mb_page_copy(const void* src_pool, void* dst_pool, const int32_t* src_pages, const int32_t* dst_pages, int n,
                 long long page_elems, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * One decode step's metadata on the device (each row appends at most one
 * token). Replaces the host-side position and slot bookkeeping of
 * FlexDecodeSession.forward (models/backbone/flex_decode.py:180-195) for
 * steps of lengths 0 or 1: reads each row's current length from kv_len
 * [batch] (left there by the previous step), writes q_pos = length, the new
 * token's cache slot (page * page_size + offset, looked up in block_table
 * [batch, max_pages]) and kv_len = length + 1. new_page [batch] (or NULL:
 * every row -1) holds a code per row: -1 append; a page id >= 0 that the
 * row's token opens (written into the block table first), with
 * MB_STEP_RESTART set when the row was emptied (it restarts at length 0 and
 * the page goes to column 0); -2 the row appends nothing (q_pos =
 * max(length - 1, 0), slot -1, length kept); -3 the row was emptied and
 * appends nothing (q_pos 0, slot -1, length 0). All int32, device memory.
 * ------------------------------------------------------------------- */
#define MB_STEP_RESTART (1 << 30)
int mb_decode_step_meta(int batch, int max_pages, int page_size, const int32_t* new_page, int32_t* block_table,
                        int32_t* q_pos, int32_t* kv_len, int32_t* slot, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Decoder-layer glue.
 * mb_rmsnorm: sum_out = x + residual (bf16), norm_out = RMSNorm(sum) * w;
 *   with residual == NULL it normalises x (sum_out unused). Replaces the
 *   residual adds and input/post_attention_layernorm calls of
 *   flex_decode.py:210, 231-232.
 * mb_silu_mul: out[r, :] = silu(gate_up[r, :I]) * gate_up[r, I:]. Replaces
 *   the activation product inside layer.mlp (flex_decode.py:232).
 * ------------------------------------------------------------------- */
int mb_rmsnorm(const void* x, const void* residual, const void* weight, float eps, int rows, int dim, void* sum_out,
               void* norm_out, mb_stream_t stream);
int mb_silu_mul(const void* gate_up, int rows, int inter, void* out, mb_stream_t stream);
/* The same glue for a residual stream kept in fp32 (the decode session's
 * default): the reference rounds the stream to bf16 at every residual add
 * (flex_decode.py:231, 233); here only the GEMM inputs are rounded, once.
 * mb_rmsnorm_f32: sum_out = x + delta in fp32 (x fp32, or x_bf16 for the
 *   bf16 embeddings entering the first layer; delta fp32 or NULL; sum_out may
 *   be x or NULL), norm_out = bf16(RMSNorm(sum) * w).
 * mb_silu_mul_f32: out = bf16(silu(gate) * up) for an fp32 gate_up [rows, 2I],
 *   I a multiple of 4, gate_up 16-byte aligned. */
int mb_rmsnorm_f32(const float* x, const void* x_bf16, const float* delta, const void* weight, float eps, int rows,
                   int dim, float* sum_out, void* norm_out, mb_stream_t stream);
int mb_silu_mul_f32(const float* gate_up, int rows, int inter, void* out, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Token embedding of a flat TokenBatch (K11). Replaces NumericEmbedder.forward
 * (models/embedding/embedding.py:293-326): embeds[t] = the row ids[t] of the
 * table of type types[t] (kinds[type] = 1), or, for Fourier types (kind 2),
 * fourier_scale * cos(scalars[t] * freqs[ids[t]] + phases[ids[t]])
 * (models/embedding/encoding.py:67-86), else zero. tables is a device array
 * of n_types device pointers to [vocab[type], dim] rows in out's dtype (bf16,
 * or fp32 when out_f32); freqs / phases fp32 [freq_sets, dim]. An id outside
 * its table or bank leaves the token zero and sets status 7. All index arrays
 * int32, device memory; dim * element size a multiple of 16 bytes.
 * ------------------------------------------------------------------- */
int mb_embed_tokens(const int32_t* types, const int32_t* ids, const float* scalars, long long tokens, int dim,
                    const int32_t* kinds, const void* const* tables, const int32_t* vocab, int n_types,
                    const float* fourier_freqs, const float* fourier_phases, int freq_sets, float fourier_scale,
                    void* out, int out_f32, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * One-step TD loss (K12). Replaces DqnObjective.__call__
 * (objectives/dqn.py:116-213) and _valid_transitions (dqn.py:12-39): over
 * the pairs (i, i + 1) with equal sequence_id (all pairs when it is NULL),
 * target = reward[i+1] + gammas[done[i+1]] * max_a q_target[i+1],
 * loss = mean (q[i, action[i+1]] - target)^2 (+ cql_weight * (|target| +
 * cql_eps) * (logsumexp(q[i]) - q[i, action[i+1]])). out (device, 6 floats):
 * loss, valid pairs, then mean / std / min / max over valid pairs of
 * max_a q[i] (the reference's metrics) — no host sync; loss is NaN when no
 * pair is valid. q, q_target f32 [n, actions]; action, done, sequence_id
 * int64 [n]; reward f32 [n]; gammas: host array of 5 (done codes 0..4);
 * scratch of mb_td_loss_scratch_bytes(n), zero-filled once before its first
 * use (calls leave it ready for the next). mb_td_loss_bwd writes
 * dq = grad_out[0] * d loss / d q (grad_out a device scalar or NULL for 1)
 * from the forward's scratch and out. A pair whose action or done code is out
 * of range is left out and sets status 7.
 * ------------------------------------------------------------------- */
size_t mb_td_loss_scratch_bytes(int n);
int mb_td_loss_fwd(const float* q, const float* q_target, const int64_t* action, const float* reward,
                   const int64_t* done, const int64_t* sequence_id, int n, int actions, const float* gammas,
                   float cql_weight, float cql_eps, void* scratch, size_t scratch_bytes, float* out,
                   mb_stream_t stream);
int mb_td_loss_bwd(const float* q, const int64_t* action, int n, int actions, float cql_weight, void* scratch,
                   size_t scratch_bytes, const float* out, const float* grad_out, float* dq, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Packed varlen segment-causal attention forward (K5, tcgen05).
 * Replaces models/backbone/flex_train.py:147 (flex_attention with the mask of
 * flex_train.py:98-102, built at :116-125): out[i, h] = softmax over keys j
 * with run_start[i] <= j <= i of scale * q[i, h] . k[j, h / G], times v.
 *   q [L, q_heads, hd], k/v [L, kv_heads, hd] bf16 (16-byte aligned);
 *   run_start int32 [L] and tile_lo int32 [ceil(L / 128)] from
 *   mb_segment_meta(tile = 128) on ids that are sorted;
 *   out [L, q_heads, hd] bf16; lse f32 [q_heads, L] = log2 of the softmax
 *   denominator of the log2-scaled scores (saved for the backward), in a
 *   buffer of MB_VARLEN_FWD_LSE_FLOATS(q_heads, L) floats whose last 4 are
 *   the persistent kernel's scratch.
 * ------------------------------------------------------------------- */
#define MB_VARLEN_FWD_LSE_FLOATS(q_heads, L) ((size_t)(q_heads) * (size_t)(L) + 4u)
int mb_varlen_attention_fwd(const void* q, const void* k, const void* v, int L, int q_heads, int kv_heads,
                            int head_dim, const int32_t* run_start, const int32_t* tile_lo, float scale, void* out,
                            float* lse, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Packed varlen segment-causal attention backward (K6, tcgen05).
 * The gradient the reference obtains by autograd through flex_attention
 * (models/backbone/flex_train.py:147): given the forward's q, k, v, out, lse
 * and the upstream dout [L, q_heads, hd], writes dq [L, q_heads, hd] and
 * dk, dv [L, kv_heads, hd] (bf16; dk/dv summed over each GQA group).
 * run_start / run_end come from mb_segment_meta. delta is caller scratch of
 * MB_VARLEN_BWD_SCRATCH_FLOATS(q_heads, L) floats (the row sums of dO * O,
 * then the tile counters of the persistent kernels). Deterministic: every
 * output element is written by one CTA, without atomics on the data.
 * ------------------------------------------------------------------- */
#define MB_VARLEN_BWD_SCRATCH_FLOATS(q_heads, L) ((size_t)(q_heads) * (size_t)(L) + 4u)
int mb_varlen_attention_bwd(const void* q, const void* k, const void* v, const void* out, const void* dout,
                            const float* lse, int L, int q_heads, int kv_heads, int head_dim,
                            const int32_t* run_start, const int32_t* run_end, float scale, void* dq, void* dk,
                            void* dv, float* delta, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Packed attention backward without the recompute of S and dP for dQ.
 * Same gradients as mb_varlen_attention_bwd; the dK/dV kernel also stores
 * every bf16 dS^T block (32 KB per q-head and (query tile, key tile) pair)
 * in ds_scratch, and dQ = scale dS K is one GEMM over the stored blocks.
 *   tile_lo: from mb_segment_meta (tile 128).
 *   pair_off int32 [MB_VARLEN_BWD_PAIR_OFFSETS(L)] from
 *   mb_varlen_bwd_pair_offsets; n_pairs = pair_off[ceil(L/128)], the number
 *   of pairs the forward visits (the caller reads it back or computes it
 *   from the segment lengths: sum over query tiles i of i - tile_lo[i]/128 + 1).
 *   ds_scratch: >= MB_VARLEN_BWD_DS_BYTES(q_heads, n_pairs) bytes, 16-byte
 *   aligned.
 * A pair offset that disagrees with n_pairs sets the device status
 * (mb_device_status) instead of writing outside the scratch.
 * ------------------------------------------------------------------- */
#define MB_VARLEN_BWD_PAIR_OFFSETS(L) (((size_t)(L) + 127u) / 128u + 1u)
#define MB_VARLEN_BWD_DS_BYTES(q_heads, n_pairs) ((size_t)(q_heads) * (size_t)(n_pairs) * 32768u)
int mb_varlen_bwd_pair_offsets(const int32_t* tile_lo, int L, int32_t* pair_off, mb_stream_t stream);
int mb_varlen_attention_bwd_stored(const void* q, const void* k, const void* v, const void* out, const void* dout,
                                   const float* lse, int L, int q_heads, int kv_heads, int head_dim,
                                   const int32_t* run_start, const int32_t* run_end, const int32_t* tile_lo,
                                   const int32_t* pair_off, int n_pairs, float scale, void* dq, void* dk, void* dv,
                                   float* delta, void* ds_scratch, size_t ds_bytes, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Decode-step layout glue (K9), byte-for-byte the index maps of
 * models/base.py:1163-1201 (_flat_to_batched_left_pad) and
 * models/embedding/packing.py:8-28 (left_align_content).
 * mb_flat_rank: rank int32 [L] = position of token i among the tokens of its
 *   id (stable; -1 for ids outside [0, batch)); stats int32 [batch + 2] =
 *   tokens per id, their maximum, and a flag (1: a prediction index outside
 *   [-L, L) or past n_pred, written as -1; negative indices count from the
 *   end, as Python indexing does); local_indices int64 [batch, steps]
 *   = rank of row b's prediction tokens in columns steps - n_b .. steps - 1
 *   (n_b = step_counts[b], read from prediction_indices[step_offsets[b] ..]),
 *   0 elsewhere. batch <= MB_FLAT_RANK_MAX_BATCH (one CTA, shared counters).
 * mb_flat_scatter: out [batch, max_len, row_bytes] zeroed, then flat row i
 *   copied to (sequence_ids[i], rank[i]).
 * mb_left_align: with rl = prediction_indices[b, steps-1] + 1 > 0, row b's
 *   first rl columns move to columns L - rl .. L - 1 (the rest zero) and its
 *   indices shift by L - rl; with rl <= 0 the row is zero and the indices
 *   are unchanged.
 * ------------------------------------------------------------------- */
#define MB_FLAT_RANK_MAX_BATCH 49152
int mb_flat_rank(const int64_t* sequence_ids, int L, int batch, const int64_t* prediction_indices, int n_pred,
                 const int32_t* step_counts, const int32_t* step_offsets, int steps, int32_t* rank, int32_t* stats,
                 int64_t* local_indices, mb_stream_t stream);
int mb_flat_scatter(const void* embeds, int L, int row_bytes, const int64_t* sequence_ids, const int32_t* rank,
                    int batch, int max_len, void* out, mb_stream_t stream);
int mb_left_align(const void* embeds, int batch, int L, int row_bytes, const int64_t* prediction_indices, int steps,
                  void* aligned, int64_t* aligned_indices, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Segment metadata of a packed stream (K7).
 * Replaces the position ids of models/backbone/flex_train.py:84-92 (and
 * models/base.py:1226-1236) and the BlockMask build of flex_train.py:116-125.
 *   sequence_ids int64 [L] -> position int64 [L] (restarts at 0 where
 *   sequence_ids[i] != sequence_ids[i-1]), run_start int32 [L],
 *   run_end int32 [L] or NULL (one past the end of i's run),
 *   tile_lo int32 [ceil(L / tile)] = run_start of each tile's first token,
 *   flags int32 [1]: flags[0] = 1 if the ids are not sorted (an id may then
 *   own several runs; the caller reorders tokens so each id is one run).
 * ------------------------------------------------------------------- */
int mb_segment_meta(const int64_t* sequence_ids, int L, int tile, int64_t* position, int32_t* run_start,
                    int32_t* run_end, int32_t* tile_lo, int32_t* flags, mb_stream_t stream);

/* ---------------------------------------------------------------------
 * Packed training layer, element-wise forward and backward (K4).
 * The decoder layer that models/backbone/flex_train.py:128-150 runs on the
 * packed stream (transformers' Qwen3DecoderLayer / LlamaDecoderLayer) in
 * fused passes. All tensors bf16 unless noted; rstd and weight gradients f32.
 *
 * mb_rmsnorm_fwd: y = weight * bf16(x * rstd), rstd[r] = 1 / sqrt(mean(x^2) +
 *   eps) (input_layernorm, post_attention_layernorm and the final norm,
 *   flex_train.py:145-150). dim a multiple of 256, <= 2048.
 * mb_rmsnorm_bwd: dx and dweight (= sum over rows of dy * bf16(x * rstd));
 *   scratch holds mb_rmsnorm_bwd_scratch_floats(rows, dim) floats.
 * mb_qkv_heads_fwd: the attention inputs from one fused projection
 *   qkv [L, qkv_row_stride] = q (q_heads * hd) | k (kv_heads * hd) | v: q and
 *   k through the optional per-head RMSNorm (q_norm / k_norm of
 *   flex_train.py:137-142; both weights or neither) then y = n * cos +
 *   rotate_half(n) * sin (flex_train.py:143-146, cos/sin [L, head_dim] per
 *   token), v copied: q [L, q_heads, hd], k / v [L, kv_heads, hd]; q_rstd
 *   [L * q_heads] and k_rstd [L * kv_heads] f32 with the norm. Row strides
 *   multiples of 8; tensors 16-byte aligned.
 * mb_qkv_heads_bwd: gradient of mb_qkv_heads_fwd for dq, dk, dv: writes the
 *   whole of dqkv (row stride dqkv_row_stride) and, with the norm, the f32
 *   norm-weight gradients [head_dim]; scratch holds
 *   mb_qkv_heads_bwd_scratch_floats(L, head_dim) floats.
 * mb_silu_mul_bwd: gradient of h = silu(gate) * up over gate_up [rows, 2I]:
 *   dgate_up[:, :I] = dh * up * silu'(gate), dgate_up[:, I:] = dh * silu(gate).
 * mb_add_rmsnorm_fwd: the decoder layer's residual add fused in front of the
 *   norm: sum_out = bf16(x + residual) (the module's add), then y and rstd of
 *   mb_rmsnorm_fwd over sum_out.
 * mb_rmsnorm_bwd_add: mb_rmsnorm_bwd with dsum, the gradient that reaches
 *   the normalised input along the residual path, added into dx before its
 *   one rounding (dx is then the gradient of both x and residual).
 * ------------------------------------------------------------------- */
int mb_rmsnorm_fwd(const void* x, const void* weight, float eps, int rows, int dim, void* y, float* rstd,
                   mb_stream_t stream);
int mb_add_rmsnorm_fwd(const void* x, const void* residual, const void* weight, float eps, int rows, int dim,
                       void* sum_out, void* y, float* rstd, mb_stream_t stream);
int mb_rmsnorm_bwd_add(const void* dy, const void* x, const void* weight, const float* rstd, const void* dsum,
                       int rows, int dim, void* dx, float* dweight, float* scratch, size_t scratch_floats,
                       mb_stream_t stream);
size_t mb_rmsnorm_bwd_scratch_floats(int rows, int dim);
int mb_rmsnorm_bwd(const void* dy, const void* x, const void* weight, const float* rstd, int rows, int dim, void* dx,
                   float* dweight, float* scratch, size_t scratch_floats, mb_stream_t stream);
int mb_qkv_heads_fwd(const void* qkv, long long qkv_row_stride, int L, int q_heads, int kv_heads, int head_dim,
                     const void* q_norm_weight, const void* k_norm_weight, float q_eps, float k_eps, const void* cos,
                     const void* sin, void* q, void* k, void* v, float* q_rstd, float* k_rstd, mb_stream_t stream);
size_t mb_qkv_heads_bwd_scratch_floats(int L, int head_dim);
int mb_qkv_heads_bwd(const void* dq, const void* dk, const void* dv, const void* qkv, long long qkv_row_stride,
                     int L, int q_heads, int kv_heads, int head_dim, const void* q_norm_weight,
                     const void* k_norm_weight, const void* cos, const void* sin, const float* q_rstd,
                     const float* k_rstd, void* dqkv, long long dqkv_row_stride, float* dq_norm_weight,
                     float* dk_norm_weight, float* scratch, size_t scratch_floats, mb_stream_t stream);
int mb_silu_mul_bwd(const void* gate_up, const void* dh, int rows, int inter, void* dgate_up, mb_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* MOUSE_B200_H */
