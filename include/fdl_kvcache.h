/*
 * fdl_kvcache.h -- C ABI of the B200 (sm_100a) KV-cache hot path for
 * Fast-dLLM v2 block-diffusion decoding.
 *
 * Every entry point:
 *   - takes raw device pointers, explicit sizes and element strides
 *     (strides are in ELEMENTS of the tensor's own dtype; the innermost
 *     dimension must be contiguous),
 *   - enqueues its kernels on the caller's stream and returns immediately,
 *   - allocates nothing (scratch memory, where needed, is passed in),
 *   - returns 0 on success, a positive FDL_E_* code for a rejected argument
 *     (nothing is launched), or a negative value -(cudaError_t) when a launch
 *     fails.
 *
 * Kernels never trap.  An index or length that is out of range on the device
 * (e.g. a write position beyond the cache) skips that row and records the
 * first such event in a per-device status word; read and clear it with
 * fdl_last_device_error().  Waits inside the attention kernel are bounded and
 * report FDL_DEV_TIMEOUT the same way.
 *
 * Reference interfaces (navneet-13/fast_v2) that each entry point replaces are
 * cited on the declaration as path:line.
 */
#ifndef FDL_KVCACHE_H
#define FDL_KVCACHE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* fdl_stream_t; /* == cudaStream_t */

/* Host-side argument errors (return values > 0).  A call whose sizes
 * describe no work (zero tokens, rows or positions) returns FDL_OK before
 * its data pointers are looked at, so empty buffers may be passed as NULL. */
#define FDL_OK              0
#define FDL_E_NULL          1  /* required pointer is NULL                     */
#define FDL_E_SHAPE         2  /* size out of supported range                  */
#define FDL_E_ALIGN         3  /* pointer / stride not aligned for vector I/O  */
#define FDL_E_DTYPE         4  /* unsupported dtype code                       */
#define FDL_E_WORKSPACE     5  /* workspace too small                          */
#define FDL_E_UNSUPPORTED   6  /* valid but unsupported configuration          */
#define FDL_E_NODEVICE      7  /* no usable sm_100 device / symbol lookup fail */

/* Device-side status codes (fdl_last_device_error). */
#define FDL_DEV_OK          0
#define FDL_DEV_INDEX       1  /* position / index outside the target buffer   */
#define FDL_DEV_LENGTH      2  /* per-sequence length outside [0, capacity]    */
#define FDL_DEV_TIMEOUT     3  /* a pipeline wait exceeded its iteration cap   */

/* dtype codes */
#define FDL_BF16            0
#define FDL_F16             1
#define FDL_F32             2

#define FDL_MAX_LAYERS      64

/* ------------------------------------------------------------------------
 * (a) Committed-block KV append with per-sequence start positions.
 *
 * For every layer l < num_layers, batch row b, new token t < n_new, head h:
 *   k_caches[l][b, start_pos[b] + t, h, :] = k_srcs[l][b, t, h, :]
 *   v_caches[l][b, start_pos[b] + t, h, :] = v_srcs[l][b, t, h, :]
 * Cache layout BSHD [B, max_seq, H, D]; src layout [B, n_new, H, D].
 * start_pos is a device int32[B].  Rows whose position falls outside
 * [0, max_seq) are skipped and reported as FDL_DEV_INDEX.
 * elem_bytes is 2 (bf16/f16) or 4 (f32); the copy is bit-exact.
 *
 * Replaces StaticKVCache.update (utils/static_kv_cache.py:132-160, uniform
 * start = _seq_len) and StaticKVCache.write_scratch_compiled with
 * prepare_write_idx (utils/static_kv_cache.py:180-229, start =
 * kv_write_start); StaticBlockCache.update (utils/static_kv_cache.py:456-462,
 * start = 0) and the sub-block copy at attention_backends.py:862-866.
 * ---------------------------------------------------------------------- */
int fdl_kv_append(void* const* k_caches, void* const* v_caches,
                  const void* const* k_srcs, const void* const* v_srcs,
                  int num_layers, const int32_t* start_pos,
                  int batch, int n_new, int max_seq, int heads, int head_dim,
                  int elem_bytes,
                  int64_t cache_sb, int64_t cache_ss, int64_t cache_sh,
                  int64_t src_sb, int64_t src_ss, int64_t src_sh,
                  fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (a) Row scatter at per-row positions (K and V in one launch).
 *
 *   dst[b, pos[b, i], h, :] = src[b, i, h, :]     for i < n, h < heads
 * applied to (k_dst, k_src) and, when v_dst != NULL, to (v_dst, v_src).
 * pos is a device int64 [B, n] with row stride pos_sb.  dst_len bounds the
 * position axis.  Duplicate positions within a row b resolve to the LAST
 * occurrence (sequential scatter semantics) when n <= 1024.
 * Strides are free, so the same call covers the BSHD cache
 * (StaticKVCache.write_sparse, utils/static_kv_cache.py:231-247), the BHSD
 * block buffer (DynamicBlockKV.write, utils/dynamic_block_kv.py:39-43), the
 * hidden-row caches (BlockSparseCache.scatter_attn_output / _mlp_output,
 * utils/block_sparse_cache.py:112-132; heads = 1) and
 * scatter_and_return_cuda (cuda_bench/fused_gather_norm.cu:79-119).
 * ---------------------------------------------------------------------- */
int fdl_kv_scatter(void* k_dst, void* v_dst,
                   const void* k_src, const void* v_src,
                   const int64_t* pos, int64_t pos_sb,
                   int batch, int n, int dst_len, int heads, int head_dim,
                   int elem_bytes,
                   int64_t dst_sb, int64_t dst_ss, int64_t dst_sh,
                   int64_t src_sb, int64_t src_ss, int64_t src_sh,
                   fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (b) Prefix gather (+ optional appended block, + optional GQA expansion).
 *
 * For batch row b, output token t < len[b] + n_blk, output head ho < heads*rep:
 *   src = t < len[b] ? prefix[b, t, ho / rep, :] : block[b, t - len[b], ho / rep, :]
 *   out[row(b, t), ho, :] = src
 * where row(b, t) = cu_seqlens[b] + t when cu_seqlens != NULL (packed varlen
 * output [sum_b(len[b]+n_blk), heads*rep, D]) and otherwise b*out_sb + t*out_ss
 * (padded output, e.g. the BHSD concat buffer).  len is device int32 [B]
 * bounded by prefix_cap; cu_seqlens is device int32 [B+1] and out_rows the
 * number of rows of the packed output (ignored without cu_seqlens).  A
 * sequence whose packed range [cu_seqlens[b], cu_seqlens[b+1]) is negative,
 * reaches past out_rows or holds fewer than len[b] + n_blk rows is skipped
 * whole and reported as FDL_DEV_INDEX (info = b).
 * Replaces the dynamic-path prefix concat torch.cat(prefix, block)
 * (modeling.py:390-392, :1410-1413, :1494-1495), the prefix views
 * StaticKVCache.get_kv_up_to / __getitem__ (utils/static_kv_cache.py:162-168,
 * 279-284) and repeat_kv (modeling.py:202-211) /
 * AttentionBackend._sdpa_attention's GQA expand (attention_backends.py:366-373).
 * ---------------------------------------------------------------------- */
int fdl_kv_gather_prefix(const void* k_prefix, const void* v_prefix,
                         const int32_t* len, int prefix_cap,
                         const void* k_block, const void* v_block, int n_blk,
                         void* k_out, void* v_out, const int32_t* cu_seqlens,
                         int64_t out_rows,
                         int batch, int heads, int head_dim, int rep,
                         int elem_bytes,
                         int64_t pre_sb, int64_t pre_ss, int64_t pre_sh,
                         int64_t blk_sb, int64_t blk_ss, int64_t blk_sh,
                         int64_t out_sb, int64_t out_ss, int64_t out_sh,
                         fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (b) Row gather by index:  out[b, i, h, :] = src[b, idx[b, i], h, :]
 * for i < n (or i < count[b] when count != NULL).  idx is int64 [B, n]
 * (idx_is_i32 = 0) or int32 (idx_is_i32 = 1) with row stride idx_sb;
 * indices must lie in [0, src_len).  Used for the token-sparse prefix
 * gather and for the hidden-state row gathers of the sparse / FOCUS / dKV
 * forwards (modeling.py:1232-1238, :1590-1592, :1661-1663).
 * ---------------------------------------------------------------------- */
int fdl_kv_gather_rows(const void* k_src, const void* v_src,
                       const void* idx, int idx_is_i32, int64_t idx_sb,
                       const int32_t* count,
                       void* k_out, void* v_out,
                       int batch, int n, int src_len, int heads, int head_dim,
                       int elem_bytes,
                       int64_t src_sb, int64_t src_ss, int64_t src_sh,
                       int64_t out_sb, int64_t out_ss, int64_t out_sh,
                       fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (a) In-place batch compaction (storage and addresses unchanged).
 *
 * For every buffer j < n_bufs and every i < n_keep, in increasing i:
 *   bufs[j][i * batch_stride : + row_bytes] = bufs[j][active[i] * batch_stride : + row_bytes]
 * Each buffer holds `batch` rows of row_bytes bytes, batch_stride bytes
 * apart (batch_stride >= row_bytes).  active is a device int64 [n_keep]
 * with i <= active[i] < batch for every i: every ascending list of distinct
 * slots (torch.nonzero of an active mask, utils/batch_bucketing.py:135)
 * qualifies.  The kernel checks the whole list before moving anything; a
 * list outside that set moves nothing and is reported as FDL_DEV_INDEX
 * (info = the offending entry).  Rows with active[i] == i are not touched;
 * rows >= n_keep keep stale bytes.  n_keep <= 4096; any number of buffers
 * (128 per launch); the copy is bit-exact for any element type.
 *
 * Replaces the batch re-indexing `t[active_indices].contiguous()` of
 * StaticKVCache.compact_batch (utils/static_kv_cache.py:350-398),
 * StaticBlockCache.compact_batch (utils/static_kv_cache.py:473-491),
 * DynamicBlockKV.compact_batch (utils/dynamic_block_kv.py:52-56) and
 * BlockSparseCache.compact_batch (utils/block_sparse_cache.py:141-147),
 * which allocate new tensors: the caches here keep their buffers and shrink
 * to a prefix view, so addresses baked into CUDA graphs stay valid.
 * ---------------------------------------------------------------------- */
int fdl_kv_compact(void* const* bufs, int n_bufs, int64_t row_bytes, int64_t batch_stride,
                   int batch, const int64_t* active, int n_keep, fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (b) Token-sparse prefix selection ("keep the top keep_num/keep_den of the
 * committed prefix tokens by key norm").  No reference counterpart exists;
 * the specification is:
 *   score[b, t] = sqrt( sum over (h, d) of K[b, t, h, d]^2 )  (fp32), t < len[b]
 *   keep[b]     = ceil(len[b] * keep_num / keep_den)
 *   sel[b, :]   = the keep[b] indices of largest score, ties -> lower index,
 *                 written in ascending order; sel[b, i] = -1 for i >= keep[b]
 *   out_len[b]  = keep[b]
 * and, when k_out/v_out are non-NULL, the selected rows are gathered:
 *   k_out[b, i, h, :] = k[b, sel[b, i], h, :]   (likewise V), i < keep[b].
 * K/V are bf16 BSHD [B, cap, H, D]; H*D must be a multiple of 8.
 * workspace: at least fdl_sparse_prefix_workspace_bytes(batch, cap) bytes.
 * ---------------------------------------------------------------------- */
int64_t fdl_sparse_prefix_workspace_bytes(int batch, int cap);
int fdl_kv_sparse_prefix(const void* k, const void* v, const int32_t* len,
                         int batch, int cap, int heads, int head_dim,
                         int64_t kv_sb, int64_t kv_ss, int64_t kv_sh,
                         int keep_num, int keep_den, int max_keep,
                         int32_t* sel, int32_t* out_len,
                         void* k_out, void* v_out,
                         int64_t out_sb, int64_t out_ss, int64_t out_sh,
                         void* workspace, int64_t workspace_bytes,
                         fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * fdl_kv_sparse_prefix without a workspace argument.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory --
 * code running inside another framework's memory pool, hosts that forbid
 * cudaMalloc after start-up, or bindings that only pass the tensors they
 * already own.  Same arguments and results as fdl_kv_sparse_prefix; the
 * per-token score scratch lives in a fixed device array of
 * FDL_NOALLOC_SCORE_MAX floats (4 MiB) inside the library, held by every GPU
 * that loads the library until the process exits.
 *   - batch * cap must not exceed FDL_NOALLOC_SCORE_MAX, else FDL_E_WORKSPACE
 *     is returned and nothing is launched;
 *   - the first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture;
 *   - all calls share the one array: calls that may overlap on the GPU (other
 *     streams, other threads on the same device) race and must be serialised
 *     by the caller.  Nothing in the array needs to start at zero.
 * Allocates nothing (no cudaMalloc / cudaFree, no library allocator).
 * ---------------------------------------------------------------------- */
#define FDL_NOALLOC_SCORE_MAX (1 << 20)
int fdl_kv_sparse_prefix_noalloc(const void* k, const void* v, const int32_t* len,
                                 int batch, int cap, int heads, int head_dim,
                                 int64_t kv_sb, int64_t kv_ss, int64_t kv_sh,
                                 int keep_num, int keep_den, int max_keep,
                                 int32_t* sel, int32_t* out_len,
                                 void* k_out, void* v_out,
                                 int64_t out_sb, int64_t out_ss, int64_t out_sh,
                                 fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (c) Fused gather + RMSNorm.
 *
 * For b < B, t < T:  row = x[b, idx[b, t], :]  (length H)
 *   inv = 1 / sqrt( sum(row^2) / H + eps )        (fp32 accumulate)
 *   gathered[b, t, :] = row                        (optional, may be NULL)
 *   x_dtype == FDL_BF16/F16 (Fast_dLLM_QwenRMSNorm.forward, modeling.py:427-432):
 *       normed[b, t, :] = round( w * round(row * inv) )   two roundings,
 *                         w == NULL -> round(row * inv)
 *   x_dtype == FDL_F32 (select_gather_rmsnorm_kernel, fused_gather_norm.cu:123-175):
 *       normed[b, t, :] = row * inv (* w when w != NULL), fp32
 * idx is int64 [B, T] (row stride idx_sb) with entries in [0, S); w has
 * x's dtype.  Replaces fused_gather_input_rmsnorm_pair
 * (cuda_bench/fused_sparse_extension.py:51-87) and the extension functions
 * gather_rmsnorm_cuda / fused_select_norm / fused_gather_input_rmsnorm_pair
 * (cuda_bench/fused_gather_norm.cu:60-73, 177-209).
 * idx == NULL means the identity gather (plain RMSNorm over T = S rows).
 * ---------------------------------------------------------------------- */
int fdl_gather_rmsnorm(const void* x, const int64_t* idx, int64_t idx_sb,
                       const void* w, float eps,
                       void* gathered, void* normed,
                       int batch, int seq, int n_tok, int hidden, int x_dtype,
                       int64_t x_sb, int64_t x_ss,
                       int64_t out_sb, int64_t out_ss,
                       fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * Residual add fused with RMSNorm (16-bit dtypes): for each of `rows` rows
 *     sum[r, :]    = round(x[r, :] + res[r, :])
 *     normed[r, :] = RMSNorm(sum[r, :]) exactly as fdl_gather_rmsnorm
 * i.e. the decoder layer's `hidden_states = residual + hidden_states`
 * followed by post_attention_layernorm / the next layer's input_layernorm
 * (Qwen2DecoderLayer.forward as used by modeling.py; RMSNorm per
 * modeling.py:427-432).  Row strides x_rs, res_rs, out_rs in elements;
 * sum_out and normed share out_rs.  sum_out may alias res (in-place update
 * of the residual stream); sum_out == NULL skips writing the sum.
 * ---------------------------------------------------------------------- */
int fdl_add_rmsnorm(const void* x, int64_t x_rs, const void* res, int64_t res_rs,
                    const void* w, float eps, void* sum_out, void* normed,
                    int64_t out_rs, int rows, int hidden, int x_dtype,
                    fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * (d) Block attention of the current query block over the KV cache, with
 * the GQA expansion done in-kernel (tcgen05 / TMEM / TMA, sm_100a).
 *
 *   q    : bf16 [B, Sq, Hq, D]  (strides q_sb, q_ss, q_sh; D = 128)
 *   k, v : bf16 [B, cap, Hkv, D] (strides kv_sb, kv_ss, kv_sh), Hq % Hkv == 0
 *   seqlens : device int32 [B]; keys j < seqlens[b] are valid
 *   k_blk, v_blk (optional): a second key source [B, n_blk, Hkv, D] that is
 *     logically appended after the first seqlens[b] keys (the dynamic-block
 *     concat cat(prefix, block) without materialising it)
 *   mask_block > 0 enables the block-causal mask of modeling.py:145-150 /
 *     585-593: query row s with absolute position qpos = q_pos[b, s] (int32,
 *     row stride Sq) may see a key of absolute position kpos only when
 *     qpos / mask_block >= kpos / mask_block.  Keys of the first source sit
 *     at positions j, keys of the block source at seqlens[b] + j.
 *   out  : bf16 [B, Sq, Hq, D] (strides o_sb, o_ss, o_sh)
 *   A query row with no visible key produces zeros.
 *   softmax in fp32 with scale `scale`; num_splits = 0 picks a split-KV
 *   factor; splits > 1 need workspace >= fdl_block_attn_workspace_bytes().
 * Replaces AttentionBackend.flash_kvcache_attention
 * (utils/attention_backends.py:588-640; FA2/FA4 flash_attn_with_kvcache and
 * FlashInfer BatchPrefillWithPagedKVCacheWrapper.run, :624-630, :642-682) and
 * the SDPA over cat(prefix, block) of the dynamic path (modeling.py:390-411).
 * ---------------------------------------------------------------------- */
int64_t fdl_block_attn_workspace_bytes(int batch, int sq, int hq, int head_dim,
                                       int num_splits);
/* Split-KV factor fdl_block_attn picks when num_splits = 0 (given a large
 * enough workspace). */
int fdl_block_attn_auto_splits(int batch, int sq, int hq, int hkv, int cap,
                               int n_blk);
int fdl_block_attn(const void* q, const void* k, const void* v,
                   const int32_t* seqlens, int cap,
                   const void* k_blk, const void* v_blk, int n_blk,
                   const int32_t* q_pos, int mask_block,
                   void* out,
                   int batch, int sq, int hq, int hkv, int head_dim,
                   float scale,
                   int64_t q_sb, int64_t q_ss, int64_t q_sh,
                   int64_t kv_sb, int64_t kv_ss, int64_t kv_sh,
                   int64_t blk_sb, int64_t blk_ss, int64_t blk_sh,
                   int64_t o_sb, int64_t o_ss, int64_t o_sh,
                   int num_splits, void* workspace, int64_t workspace_bytes,
                   fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * Token selection feeding the sparse gathers (one block of seq <= 32 tokens
 * per sequence).  Index outputs are exact: float reductions run in a fixed
 * order, bf16 inputs (dtype FDL_BF16) are rounded to bf16 after every step
 * where the reference's bf16 torch op rounds, FDL_F32 inputs are not; equal
 * values rank by position, lower index first (torch.topk leaves that open).
 * Strides are in elements; rows read as 16-byte vectors must be 16-byte
 * aligned.
 *
 * fdl_cosine_select: for every sequence b and token s < seq,
 *   cos[b, s] = sum_e (x_e / max(|x|, eps)) * (y_e / max(|y|, eps)),
 *   x = hidden[b, s, :], y = cached[b, s, :], eps = 1e-8
 * (F.cosine_similarity); idx[b, :n_select] = the n_select tokens of lowest
 * cos, ascending.  With cache_out != NULL the hidden rows are then copied
 * into cache_out (may be `cached` itself: each row is read before it is
 * overwritten).  cos_out (fp32 [B, seq], optional) returns the similarities.
 * hidden_size % (16 / element bytes) == 0.  Replaces the sparse forward's
 * cosine top-k + sort and the layer-input cache refresh
 * (modeling.py:868-877).
 *
 * fdl_focus_select: _focus_select (modeling.py:240-306) with the retain
 * target k_floor = max(1, min(seq, ceil(...))) computed by the caller:
 * mean + std threshold over the masked deltas, right-neighbour rule, top
 * k_floor masked deltas, decoded tokens retained, frozen ones (optional)
 * dropped; ksel[0] = the batch-uniform count; sel[b, :ksel] = the ksel
 * highest-priority positions (retained first) ascending, sel[b, ksel:seq]
 * = -1.  mask / frozen are bool (one byte) [B, seq].  batch <= 4096.
 *
 * fdl_focus_importance: _focus_importance (modeling.py:214-237): for every
 * sequence the attention mass each masked key receives from masked queries
 * (scores scaled, max-pooled over 3 keys, softmaxed over masked keys),
 * summed over queries and heads.  q [B, hq, seq, D], k [B, hkv, seq, D]
 * (query head h reads key head h / (hq / hkv): no repeat_kv copy); mask bool
 * [B, seq]; imp [B, seq] in the input dtype.  hq <= 128, D <= 128.
 * Floating point: within bf16 tolerance of the reference.
 * ---------------------------------------------------------------------- */
int fdl_cosine_select(const void* hidden, const void* cached, void* cache_out,
                      int batch, int seq, int hidden_size, int dtype,
                      int64_t h_sb, int64_t h_ss, int64_t c_sb, int64_t c_ss,
                      int64_t o_sb, int64_t o_ss,
                      int n_select, int64_t* idx, int64_t idx_sb, float* cos_out,
                      fdl_stream_t stream);
int fdl_focus_select(const void* delta, int64_t delta_sb,
                     const uint8_t* mask, int64_t mask_sb,
                     const uint8_t* frozen, int64_t frozen_sb,
                     int batch, int seq, int k_floor, int dtype,
                     int64_t* sel, int64_t sel_sb, int32_t* ksel,
                     fdl_stream_t stream);
int fdl_focus_importance(const void* q, const void* k, const uint8_t* mask,
                         int batch, int seq, int hq, int hkv, int head_dim, int dtype,
                         int64_t q_sb, int64_t q_sh, int64_t q_ss,
                         int64_t k_sb, int64_t k_sh, int64_t k_ss,
                         int64_t mask_sb, float scaling,
                         void* imp, int64_t imp_sb, fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * Decode-forward elementwise stages next to the KV path (single HBM pass).
 *
 * fdl_rope_qkv: y is the fused q/k/v projection output, bf16
 * [rows, (hq + 2*hkv) * head_dim] with row stride y_rs (elements); pos is
 * device int64 [rows] (absolute positions), inv_freq device fp32
 * [head_dim/2].  Writes q [rows, hq, D], k [rows, hkv, D] (rotary embedding
 * applied) and v [rows, hkv, D], contiguous bf16.  Per element, exactly the
 * reference's bf16 arithmetic: c, s = bf16(cos/sin(fp32(pos * inv_freq)));
 * out = bf16(bf16(x * c) + bf16(rotate_half(x) * s)).  Replaces the q/k/v
 * view + _apply_rotary_pos_emb of the patched attention forward
 * (utils/attention_backends.py:777-788, 829-836) / apply_rotary_pos_emb
 * (modeling.py:186-199) with the rotary table of modeling.py:545-560.
 *
 * fdl_rope_qkv_kv: the same split + rotary embedding for `batch` sequences
 * of n tokens (row b * n + t of y), with q written contiguously and K / V
 * written straight into their cache rows instead of separate buffers:
 *   k_dst[b, p, h, :] / v_dst[b, p, h, :]  (element strides dst_sb, dst_ss,
 *   dst_sh, so BSHD caches and BHSD block buffers both fit)
 *   p = dst_pos[b, t] (int64, row stride dst_pos_sb) when dst_pos != NULL,
 *   else start[b] + t (int32) when start != NULL, else t.
 * Rows whose p falls outside [0, dst_len) store no K/V and are reported as
 * FDL_DEV_INDEX.  Fuses the commit append (StaticKVCache.update /
 * write_sparse at cache_seqlens + arange, utils/static_kv_cache.py:132-160,
 * 231-247) and the block-buffer writes (DynamicBlockKV.write_full / write,
 * utils/dynamic_block_kv.py:34-43) into the RoPE pass after the q/k/v GEMM.
 *
 * fdl_swiglu: gu bf16 [rows, 2F] (gate then up, row stride gu_rs) ->
 * out [rows, F] (row stride out_rs) = bf16(bf16(silu(gate)) * up)
 * (Fast_dLLM_QwenMLP.forward, modeling.py:163-165).  F % 8 == 0.
 * ---------------------------------------------------------------------- */
int fdl_rope_qkv(const void* y, int64_t y_rs, const int64_t* pos,
                 const float* inv_freq, void* q, void* k, void* v,
                 int rows, int hq, int hkv, int head_dim, fdl_stream_t stream);
int fdl_rope_qkv_kv(const void* y, int64_t y_rs, const int64_t* pos,
                    const float* inv_freq, void* q, void* k_dst, void* v_dst,
                    int64_t dst_sb, int64_t dst_ss, int64_t dst_sh, int dst_len,
                    const int32_t* start, const int64_t* dst_pos, int64_t dst_pos_sb,
                    int batch, int n, int hq, int hkv, int head_dim,
                    fdl_stream_t stream);
int fdl_swiglu(const void* gu, int64_t gu_rs, void* out, int64_t out_rs,
               int64_t rows, int ffn, fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * Greedy sampling statistics over the vocabulary (bf16 logits).
 *
 * For every row r < rows of logits [rows, vocab] (row stride in elements):
 *   m = max_v l_v,  s = sum_v exp(l_v - m)   (fp32),
 *   prob[r]  = bf16(exp(0) / s)               (the largest probability),
 *   token[r] = the first v with bf16(exp(l_v - m) / s) == prob[r].
 * That is the argmax of the bf16 softmax with ties to the lower index, and
 * the probability gathered at it: sample_with_top_p at temperature 0
 * (modeling.py:2263-2269) and the x1_p gather of the samplers
 * (generation_functions.py:2290-2291), without the [rows, vocab]
 * probabilities.  prob may be NULL.  A row with no finite logit gets token 0
 * and is reported as FDL_DEV_INDEX (info = row).
 * ---------------------------------------------------------------------- */
int fdl_softmax_argmax(const void* logits, int64_t row_stride, int rows,
                       int vocab, int64_t* token, void* prob,
                       fdl_stream_t stream);

/* ------------------------------------------------------------------------
 * Status.  Copies the calling device's first recorded device-side error
 * code into *code and the offending value into *info (either may be NULL),
 * then clears both.  Synchronises the device.  Returns 0 or -(cudaError_t).
 * The reference has no device-side error channel; its failures surface as
 * Python exceptions (attention_backends.py:637-640).
 * ---------------------------------------------------------------------- */
int fdl_last_device_error(int32_t* code, int64_t* info);

/* Library build identity: "fdl_b200 <version> sm_100a". */
const char* fdl_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FDL_KVCACHE_H */
