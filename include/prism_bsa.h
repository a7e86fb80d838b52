/*
 * prism_bsa.h -- C ABI of the B200 (sm_100a) dynamic block-shape block-sparse
 * attention path of Tencent-Hunyuan/Prism.
 *
 * All tensors are raw DEVICE pointers owned by the caller; every entry point
 * enqueues work on `stream` and returns immediately.  No entry point allocates
 * device memory, synchronises the host or exits the process; workspaces are
 * caller-provided and sized by the matching *_workspace_bytes() query.
 * Errors come back as a prism_status_t; prism_last_error() gives a
 * thread-local message.
 *
 * Layout conventions
 *   THW order   token s = (t*H + h)*W + w over a (T, H, W) latent grid.
 *   padded grid (Tp, Hp, Wp) = (T, H, W) rounded up to multiples of 8 (the
 *               8x8x8 macro-zone, dynamic_block_shape.py:31).
 *   tile order  the per-zone anisotropic rearrangement: zone z holds tokens
 *               [512 z, 512 z + 512), split into 64-token tiles; built by
 *               prism_build_layout (src_idx[r] = padded THW index of row r).
 *               The uniform fixed-shape path instead uses the global 3D-chunk
 *               order of prism_uniform_layout (grid padded to the chunk).
 *   bitmaps     bits_q[h][q_tile][w] bit b set <=> q tile attends key tile
 *               32 w + b; bits_k is its transpose (key tile -> q tiles).
 *               Row length WQ = ceil(N_tiles / 32) 32-bit words.
 *   bf16        tensors are passed as void* holding __nv_bfloat16.
 *
 * Reference paths below are relative to the reference project root.
 */
#ifndef PRISM_BSA_H_
#define PRISM_BSA_H_

#include <stddef.h>
#include <stdint.h>
#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  PRISM_OK = 0,
  PRISM_ERR_INVALID_ARG = 1,
  PRISM_ERR_CUDA = 2,
  PRISM_ERR_UNSUPPORTED = 3,
} prism_status_t;

/* Thread-local text of the last error raised on this host thread. */
const char* prism_last_error(void);
/* ABI version (incremented on any signature change). */
int prism_abi_version(void);
/* Device-side status of the attention kernels: 0 when every bounded wait
 * inside them completed, otherwise the code of the first wait that gave up
 * (the kernel then drained its in-flight copies, released its tensor memory
 * and returned without finishing its outputs).  Reading the status
 * synchronises with the device and resets it to 0; -1 = the read failed.
 * No counterpart in the reference (Triton kernels have no device-side waits). */
int prism_device_status(void);

/* TEST ONLY -- proves that the bounded waits return.  Runs the forward kernel
 * (prism_bsa_fwd, one head, S <= 256 tokens: one CTA) with its producer
 * issuing no load, and the wait limit shortened to wait_limit_ns (0.1 ms..2 s)
 * for this launch only (set and restored by stream-ordered writes around it).
 * The MMA warp's first wait therefore ends at the limit: the kernel sets the
 * device status (prism_device_status: 102 or 103), releases its tensor memory
 * and returns with o / lse unwritten.  Synchronises `stream` before returning.
 * Not for production use; no counterpart in the reference. */
prism_status_t prism_test_fwd_withheld_load(const void* q, const void* k, const void* v, int64_t S,
                                            int D, float sm_scale, const uint32_t* bits_q,
                                            const uint64_t* tile_bits, void* o, float* lse,
                                            uint64_t wait_limit_ns, cudaStream_t stream);

/* Per-token L2 norm of the audio->video bridge residual, bf16 in/out, fp32
 * accumulation.  Replaces `a2v_bridge_residual.norm(dim=-1)`
 * (hymm/models/modules/wan_video_dit.py:742-744).  dim % 8 == 0. */
prism_status_t prism_token_norms(const void* x, int64_t n_tokens, int dim, void* out,
                                 cudaStream_t stream);

/* Zone statistics: head average of V (bf16, dynamic_block_attention.py:236) and
 * the masked per-zone means packed as [Nz, 25*D] fp32 = channel | per-t[8] |
 * per-h[8] | per-w[8] (compute_zone_aggregates, dynamic_block_shape.py:68-129),
 * axis validity [Nz, 24] u8, and the same means of the audio norms [Nz, 25] fp32
 * (compute_audio_directional's masked means, dynamic_block_shape.py:216-229).
 * v [heads, T*H*W, D] bf16 on the source grid (T, H, W) <= (Tp, Hp, Wp) with
 * head stride v_stride_h and token stride v_stride_s (elements); norms [T*H*W]
 * bf16 on the same grid or NULL.  A token of the padded grid is valid iff it
 * lies inside (T, H, W) and valid[padded index] (valid NULL = no extra mask):
 * passing the unpadded tensors fuses the zero padding of
 * wan_video_dit.py:364-395.  workspace: prism_zone_stats_workspace_bytes(). */
size_t prism_zone_stats_workspace_bytes(int Tp, int Hp, int Wp, int D);
prism_status_t prism_zone_stats(const void* v, int heads, int64_t v_stride_h, int64_t v_stride_s,
                                int T, int H, int W, int Tp, int Hp, int Wp, int D,
                                const uint8_t* valid, const void* norms, void* workspace,
                                float* packed, uint8_t* axis_valid, float* audio,
                                cudaStream_t stream);

/* Shape choice per zone from the (SP-averaged) packed statistics:
 * compute_effective_gradient + select_shapes_ivpq (method 0) or
 * select_shapes_penalty (method 1) (dynamic_block_shape.py:248-391).
 * shape_ids [Nz] int64 in [0, 13).  g_out [Nz,3] / rho_out [Nz] optional. */
prism_status_t prism_shape_select(const float* packed, const uint8_t* axis_valid,
                                  const float* audio, int has_audio, int Nz, int D, int method,
                                  float lambda_a, float tau_128, float lambda_128,
                                  int64_t* shape_ids, float* g_out, float* rho_out,
                                  cudaStream_t stream);

/* Permutation and tile/block maps (_precompute_local_orders,
 * _build_rearrange_index, _build_block_tile_maps:
 * dynamic_block_attention.py:21-63, 107-170).
 * src_idx/inv_idx [S] int32; block_of_tile [N_tiles] int32;
 * block_tiles [(N_tiles+1)*2] int32 (rows >= n_blocks hold the sentinel
 * N_tiles); n_blocks [1] int32 (device).  N_tiles = 8 * Nz. */
prism_status_t prism_build_layout(const int64_t* shape_ids, int Tp, int Hp, int Wp,
                                  int32_t* src_idx, int32_t* inv_idx, int32_t* block_of_tile,
                                  int32_t* block_tiles, int32_t* n_blocks, cudaStream_t stream);

/* Key validity of each 64-token tile in tile order: bit i of tile_bits[j] is
 * set iff padded token src_idx[64 j + i] lies inside the source grid
 * (T, H, W) and (valid == NULL or valid[src_idx[64 j + i]]); tile_count[j] is
 * its popcount (the reference's valid_re / tile_counts,
 * dynamic_block_attention.py:253, 260; rearrange_THW_to_3d_block_1d,
 * bsa_interface.py:1117-1121, for the uniform path).  n_rows = length of
 * src_idx, a multiple of 64; entries >= Tp*Hp*Wp are padding rows. */
prism_status_t prism_tile_valid(const int32_t* src_idx, int64_t n_rows, const uint8_t* valid, int T,
                                int H, int W, int Tp, int Hp, int Wp, uint64_t* tile_bits,
                                int32_t* tile_count, cudaStream_t stream);

/* Gather rows into tile order: out[h][r] = x[h][thw(src_idx[r])], where
 * src_idx holds padded-grid THW indices and x is laid out on the grid
 * (T, H, W) <= (Tp, Hp, Wp); rows outside (T, H, W) are written as zeros
 * (the F.pad of wan_video_dit.py:382-389 fused with
 * q.index_select(2, src_idx), dynamic_block_attention.py:250-252; the uniform
 * path's pad, wan_video_dit.py:485-505, and rearrange_THW_to_3d_block,
 * bsa_interface.py:1105-1109).  n_rows = length of src_idx (output rows per
 * head); entries >= Tp*Hp*Wp give zero rows.
 * Strides in elements; rows are D contiguous bf16, D % 8 == 0. */
prism_status_t prism_gather_rows(const void* x, int64_t x_stride_h, int64_t x_stride_s, int heads,
                                 int D, int T, int H, int W, int Tp, int Hp, int Wp,
                                 const int32_t* src_idx, int64_t n_rows, void* out,
                                 int64_t out_stride_h, cudaStream_t stream);

/* Inverse of prism_gather_rows for the tokens inside (T, H, W):
 * out[h][thw] = x_re[h][inv_idx[padded thw]] (o_re.index_select(2, inv_idx)
 * + unpad, dynamic_block_attention.py:329, wan_video_dit.py:429-431). */
prism_status_t prism_scatter_rows(const void* x_re, int64_t x_stride_h, int heads, int D, int T,
                                  int H, int W, int Tp, int Hp, int Wp, const int32_t* inv_idx,
                                  void* out, int64_t out_stride_h, int64_t out_stride_s,
                                  cudaStream_t stream);

/* Strided block copy (the Ulysses exchange's layout changes,
 * communications.py:179-183, 195, 219-225, 235 of the reference): for block o <
 * n_blocks and row r < n_rows, row_bytes bytes from
 * src + o * src_stride_block + r * src_stride_row to
 * dst + o * dst_stride_block + r * dst_stride_row (all byte offsets; pointers, strides
 * and row_bytes multiples of 16; n_blocks <= 65535).  Source and destination must not
 * overlap. */
prism_status_t prism_copy_rows(const void* src, int64_t src_stride_block, int64_t src_stride_row,
                               void* dst, int64_t dst_stride_block, int64_t dst_stride_row,
                               int64_t n_blocks, int64_t n_rows, int64_t row_bytes, cudaStream_t stream);

/* Pooled logical-block scores and hybrid selection, per head
 * (masked_mean_pooling_compression bsa_interface.py:177-201,
 * _logical_block_means dynamic_block_attention.py:173-188, cal_score
 * bsa_interface.py:203-207, get_select_indices_{cdf_topk,cdf,topk}_from_score
 * bsa_interface.py:235-304, tile expansion dynamic_block_attention.py:297-319).
 * mode 0 = top-k + cumulative mass, 1 = cumulative mass only, 2 = top-k only.
 * tile_bits from prism_tile_valid.  Writes every word of bits_q
 * [heads, N_tiles, WQ] and of its transpose bits_k.  Ties in the top-k /
 * cumulative-mass order are broken by lower block index.
 * workspace: prism_block_select_workspace_bytes(). */
size_t prism_block_select_workspace_bytes(int heads, int64_t S, int D);
prism_status_t prism_block_select(const void* q_re, const void* k_re, int heads, int64_t S, int D,
                                  const int32_t* block_tiles, const int32_t* n_blocks,
                                  const uint64_t* tile_bits, int mode, double sparsity,
                                  double cdf_threshold, void* workspace, uint32_t* bits_q,
                                  uint32_t* bits_k, cudaStream_t stream);

/* Uniform fixed-shape path (flash_attn_bsa_3d, bsa_interface.py:1123-1176).
 *
 * prism_uniform_layout: the permutation of rearrange_THW_to_3d_block
 * (bsa_interface.py:1105-1109) for chunk (ct, ch, cw) over the padded grid
 * (Tp, Hp, Wp) (multiples of the chunk): row p of the chunk order holds padded
 * THW token src_idx[p]; inv_idx [Tp*Hp*Wp] is its inverse
 * (rearrange_3d_block_to_THW, :1111-1115).  n_rows >= Tp*Hp*Wp rows are
 * written; rows p >= Tp*Hp*Wp get the sentinel Tp*Hp*Wp (zero rows, padding),
 * so that the attention kernels see whole 128-row tile pairs. */
prism_status_t prism_uniform_layout(int Tp, int Hp, int Wp, int ct, int ch, int cw, int64_t n_rows,
                                    int32_t* src_idx, int32_t* inv_idx, cudaStream_t stream);

/* Chunk pooling, scores and selection of _attention_bsa.forward
 * (bsa_interface.py:600-633: masked_mean_pooling_compression /
 * mean_pooling_compression :164-201, cal_score :203-207,
 * get_select_indices_{topk,cdf,cdf_topk}_from_score :235-304), expanded to
 * 64-token tile bitmaps.  q_re [heads, Sq, D] is in the q chunk order, k_re
 * [heads, Sk, D] in the key chunk order (bf16, Sq and Sk multiples of 64); the
 * first seq_q / seq_k rows are real (multiples of chunk_q / chunk_k, which are
 * multiples of 64).  k_bits [Sk/64]: key validity (64 rows per word); q_bits
 * [Sq/64] or NULL: the rows the q pooling counts (the reference pools q under
 * q_valid_mask if given, else under the key mask when Sq == Sk, else all rows,
 * :606-611; NULL = all rows).  Pooling is fp32 (sequential sums /
 * max(count, 1)); no key chunk is excluded from the ranking; selected tiles
 * without a valid key are dropped (they contribute nothing).
 * bits_q [heads, Sq/64, ceil(Sk/2048)] (rows of padding tiles are zero) and
 * its transpose bits_k [heads, Sk/64, ceil(Sq/2048)].  mode as for
 * prism_block_select.  workspace: prism_block_select_uniform_workspace_bytes(
 * heads, seq_q/chunk_q, seq_k/chunk_k, D).
 * Guided selection (flash_attn_bsa_3d_variance_guided / _audio_guided,
 * bsa_interface.py:1179-1260, 1395-1501): k_weights [seq_k] fp32 or NULL
 * replaces the key validity in the key pooling by per-row weights (sum of
 * x*w / max(sum of w, 1), audio_weighted_mean_pooling_compression :902-970;
 * see prism_audio_pool_weights); col_scale [seq_k/chunk_k] fp32 or NULL
 * multiplies every score of key chunk c by col_scale[c] before the selection
 * (score * score_modifier :626-627, score * (1 + boost) :764; see
 * prism_guidance_scale). */
size_t prism_block_select_uniform_workspace_bytes(int heads, int64_t n_chunks_q, int64_t n_chunks_k,
                                                  int D);
prism_status_t prism_block_select_uniform(const void* q_re, const void* k_re, int heads, int64_t Sq,
                                          int64_t Sk, int D, int64_t seq_q, int64_t seq_k,
                                          int chunk_q, int chunk_k, const uint64_t* q_bits,
                                          const uint64_t* k_bits, const float* k_weights,
                                          const float* col_scale, int mode, double sparsity,
                                          double cdf_threshold, void* workspace, uint32_t* bits_q,
                                          uint32_t* bits_k, cudaStream_t stream);

/* Inputs of the guided selection.  Keys are in the key chunk order of
 * prism_uniform_layout (chunk (ct, ch, cw), chunk_k = ct*ch*cw rows, the first
 * seq_k rows real); k_bits [Sk/64] key validity (NULL = every row valid, the
 * reference's valid_mask = None).
 *
 * prism_gather_values: per-token fp32 values x [T*H*W] on the grid (T, H, W)
 * <= (Tp, Hp, Wp) into the chunk order (out[r] = x at src_idx[r], 0 at padding);
 * the padding of wan_video_dit.py:301-306 fused with
 * rearrange_THW_to_3d_block_1d (bsa_interface.py:1117-1121).
 *
 * prism_variance_density: compute_channel_variance_density
 * (bsa_interface.py:973-1062) of v_re [heads, Sk, D] bf16 -> rho [seq_k/chunk_k]
 * fp32 in [0, 1]: per chunk, the head-averaged V's spatial channel variance
 * (variance over channels of the masked chunk means) plus temporal channel
 * variance (mean over channels of the squared differences of consecutive
 * masked frame means, ct frames of ch*cw rows, pairs with both frames
 * non-empty), normalised by the maximum over chunks (floor 1e-6).  Sums are
 * sequential fp32.  D a multiple of 32 up to 256.
 *
 * prism_audio_saliency: compute_block_audio_saliency (bsa_interface.py:
 * 1065-1102) of the audio norms in chunk order: masked chunk means / their
 * maximum (floor 1e-6).
 *
 * prism_audio_pool_weights: the per-row weights of Path B
 * (audio_weighted_mean_pooling_compression, bsa_interface.py:902-970):
 * w = 1 + lambda_w * a / max(1e-6, chunk max of valid a) on valid rows, 0 on
 * invalid rows; pass to prism_block_select_uniform as k_weights.
 *
 * prism_guidance_scale: scale [n_chunks] = 1 + boost with
 *   ext   = modifier[c] + variance_gamma * rho[c]  (terms present when non-NULL)
 *   boost = audio_gamma * (g * saliency[c] + (1 - g) / n_chunks) + ext
 * in that order of operations (_attention_bsa_audio_guided.forward,
 * bsa_interface.py:744-764, variance term folded as :1467-1470; the
 * variance-only path's 1 + gamma * rho, :1240-1245, is the case with
 * saliency = modifier = NULL).  audio_gate: device scalar g (NULL = 1);
 * saliency NULL = no audio term. */
prism_status_t prism_gather_values(const float* x, int T, int H, int W, int Tp, int Hp, int Wp,
                                   const int32_t* src_idx, int64_t n_rows, float* out,
                                   cudaStream_t stream);
prism_status_t prism_variance_density(const void* v_re, int heads, int64_t Sk, int D, int64_t seq_k,
                                      int ct, int ch, int cw, const uint64_t* k_bits, float* rho,
                                      cudaStream_t stream);
prism_status_t prism_audio_saliency(const float* norms_re, int64_t seq_k, int chunk_k,
                                    const uint64_t* k_bits, float* saliency, cudaStream_t stream);
prism_status_t prism_audio_pool_weights(const float* norms_re, int64_t seq_k, int chunk_k,
                                        const uint64_t* k_bits, float lambda_w, float* weights,
                                        cudaStream_t stream);
/* Chunk means of x_re [heads, S, D] bf16 over chunks of `chunk` consecutive rows
 * (the first seq rows) -> out [heads, seq/chunk, D] fp32: with weights [seq] fp32
 * the Path B form (sum of rounded x*w / max(sum of w, 1),
 * audio_weighted_mean_pooling_compression, bsa_interface.py:902-970), else the
 * mean over the rows valid in bits (NULL = all) / max(count, 1)
 * (masked_mean_pooling_compression, :177-201).  The same pooling as the
 * selection's. */
prism_status_t prism_pool_chunks(const void* x_re, int heads, int64_t S, int D, int64_t seq,
                                int chunk, const uint64_t* bits, const float* weights, float* out,
                                cudaStream_t stream);
prism_status_t prism_guidance_scale(int64_t n_chunks, const float* rho, float variance_gamma,
                                    const float* saliency, const float* audio_gate, float audio_gamma,
                                    const float* modifier, float* scale, cudaStream_t stream);

/* Raw chunk scores (cal_score, bsa_interface.py:203-207): score[h][a][b] = fp32
 * dot product of pooled q chunk a and pooled key chunk b (qc [heads, nq, D], kc
 * [heads, nk, D]), the same products as the selection's, without its col_scale. */
prism_status_t prism_chunk_scores(const float* qc, const float* kc, int heads, int nq, int nk, int D,
                                  float* scores, cudaStream_t stream);

/* Block-sparse attention forward over tile-ordered q/k/v [heads, S, D] bf16
 * (attn_fwd_bsa_varlen_triton + _attn_fwd_bsa_varlen_align,
 * bsa_interface.py:328-385, flash_attn_bsa_varlen_mask.py:193-319).
 * o [heads, S, D] bf16; lse [heads, S] fp32 natural log.  D in {64, 128}.
 * o_lo (optional, same shape as o) receives the bf16 rounding residual of the
 * output (o + o_lo = the fp32 result to ~16 bits); pass it to the backward so
 * that delta = rowsum(O * dO) is not limited by O's bf16 rounding. */
prism_status_t prism_bsa_fwd(const void* q, const void* k, const void* v, int heads, int64_t S,
                             int D, float sm_scale, const uint32_t* bits_q,
                             const uint64_t* tile_bits, void* o, void* o_lo, float* lse,
                             cudaStream_t stream);

/* Key-bias form of the forward (the pooled-key pass of the Taylor merge,
 * _taylor_merge_fwd_kernel, bias_rectification_triton.py:156-293): as
 * prism_bsa_fwd_qk, with the key validity per (head, query tile, key tile),
 * key_masks [heads, Sq/64, Sk/64] u64, and a score offset per key, key_bias [Sk]
 * fp32 added to the raw score q.k before sm_scale (a log-weight w is passed as
 * w / sm_scale).  Rows without a selected key give O = 0, lse = -inf. */
prism_status_t prism_bsa_fwd_keybias(const void* q, const void* k, const void* v, int heads, int64_t Sq,
                                     int64_t Sk, int D, float sm_scale, const uint32_t* bits_q,
                                     const uint64_t* key_masks, const float* key_bias, void* o,
                                     void* o_lo, float* lse, cudaStream_t stream);

/* Bias rectification of the uniform path, inference (bsa_rectified_sparse_attn /
 * bsa_taylor_sparse_attn, bias_rectification.py:261-446; fused kernels
 * bias_rectification_triton.py:9-363).
 *
 * prism_correction_stats: per head h and q chunk a, from the raw chunk scores
 * [heads, nq, nk] fp32, the selection bitmap bits_q [heads, n_qt, ceil(n_kt/32)]
 * (q chunk a = tiles [a*tq, a*tq+tq), key chunk j = tiles [j*tk, j*tk+tk); chunk j
 * is selected iff one of its tiles is set) and the key validity tile_bits [n_kt]
 * (chunk j valid iff one of its tiles holds a valid key):
 *   A_j = softmax over valid j of score * sm_scale (_masked_softmax_along_last :146-152)
 *   R[h][a] = max(1 - sum of A over valid unselected j, 1e-6)           (:435-436)
 *   M[h][a] = variance of A over the valid j (_masked_var_along_last :155-170)
 * nonsel [heads, nq, ceil(nk/64)] u64 (NULL = not written): the valid unselected
 * chunks; a_rect [heads, nq, nk] fp32 (NULL = not written): A on them, 0 elsewhere.
 * Sums in a fixed order (256 strided partials, then a halving tree), deterministic
 * exponentials.
 *
 * prism_taylor_prep: the pooled-key pass inputs for n_ut = Sk_pooled/64 key tiles:
 * masks [heads, n_qt, n_ut] u64 = nonsel of the q tile's chunk where M < *tau
 * (is_flat, :300-303), else 0; bits_t [heads, n_qt, ceil(n_ut/32)] bit u set iff
 * masks[..][u] != 0.  tau: device scalar.
 *
 * prism_key_log_bias: bias [n_pad] = log(max(valid tokens of chunk j, 1)) / sm_scale
 * for j < nk (the log-count offsets of :218-221), 0 beyond.
 *
 * prism_rows_to_bf16: fp32 rows [heads, n, D] -> bf16 [heads, n_pad, D], zero rows past n.
 *
 * prism_taylor_merge: rows r < seq_q of chunk a = r / chunk_q with M[h][a] < *tau:
 * out = w_spa O_spa + w_t O_t with w = exp(lse - lse_total) (natural-log lse,
 * bias_rectification_triton.py:270-292); other rows out = O_spa.  O given as bf16
 * plus an optional bf16 residual (o_lo of the forward).  Rows [heads, S, D].
 *
 * prism_rectified_contract: o_ncri [heads, nq, D] fp32 = a_rect [heads, nq, nk] x
 * v_cmp [heads, nk, D] fp32 (the pooled values of the key chunks), one fmaf per term
 * in increasing key chunk order (deterministic): the A_rect V_cmp product of
 * _rectified_correction_fwd_kernel (bias_rectification_triton.py:9-95).
 *
 * prism_rectified_apply: rows r < seq_q: out = R[h][a] O_spa + o_ncri[h][a][:]
 * (o_ncri [heads, nq, D] fp32 = a_rect V_cmp); other rows out = O_spa
 * (_rectified_correction_fwd_kernel, bias_rectification_triton.py:9-95). */
prism_status_t prism_correction_stats(const float* scores, int heads, int nq, int nk, int tq, int tk,
                                      const uint32_t* bits_q, int64_t n_qt, int64_t n_kt,
                                      const uint64_t* tile_bits, float sm_scale, float* R, float* M,
                                      uint64_t* nonsel, float* a_rect, cudaStream_t stream);
prism_status_t prism_taylor_prep(const uint64_t* nonsel, const float* M, const float* tau, int heads,
                                 int64_t n_qt, int tq, int nq, int nk, int64_t n_ut, uint64_t* masks,
                                 uint32_t* bits_t, cudaStream_t stream);
prism_status_t prism_key_log_bias(const uint64_t* tile_bits, int nk, int tk, int n_pad, float sm_scale,
                                  float* bias, cudaStream_t stream);
prism_status_t prism_rows_to_bf16(const float* x, int heads, int n, int D, int n_pad, void* out,
                                  cudaStream_t stream);
prism_status_t prism_taylor_merge(const void* o_spa, const void* o_spa_lo, const float* lse_spa,
                                  const void* o_t, const void* o_t_lo, const float* lse_t,
                                  const float* M, const float* tau, int heads, int64_t S, int64_t seq_q,
                                  int chunk_q, int D, void* out, cudaStream_t stream);
prism_status_t prism_rectified_contract(const float* a_rect, const float* v_cmp, int heads, int nq, int nk,
                                        int D, float* o_ncri, cudaStream_t stream);
prism_status_t prism_rectified_apply(const void* o_spa, const void* o_spa_lo, const float* R,
                                     const float* o_ncri, int heads, int64_t S, int64_t seq_q, int chunk_q,
                                     int D, void* out, cudaStream_t stream);

/* Dense GEMM on the tensor cores for the layer's projections (self.q / k / v / o,
 * wan_video_dit.py:699-701, 841) and their gradients; replaces F.linear / cuBLAS:
 *   C[M, N] (bf16, row stride ldc) = sum_k A(m, k) B(n, k) (+ bias[n] fp32; with
 *   accumulate != 0 the old C is added), fp32 accumulation.
 * A is K-major (A(m, k) = a[m * lda + k]) or, with a_mn_major, MN-major
 * (a[k * lda + m]); B likewise.  Forward y = x W^T: both K-major; dx = dy W: A
 * K-major, B MN-major; dW = dy^T x: both MN-major.  N, lda, ldb, ldc multiples of 8;
 * 16-byte aligned tensors.  Persistent kernel: 128 x 256 tiles, 4-stage TMA ring,
 * double-buffered TMEM accumulators.  Bounded waits report through
 * prism_device_status (codes 401-403). */
prism_status_t prism_gemm_bf16(const void* a, int64_t lda, int a_mn_major, const void* b, int64_t ldb,
                               int b_mn_major, int M, int N, int K, const float* bias, void* c,
                               int64_t ldc, int accumulate, cudaStream_t stream);

/* Producer side of the self-attention (SelfAttention.forward,
 * wan_video_dit.py:699-705, 764-787), one pass per token row after the q / k / v
 * projections.  x [S, H*D] bf16 rows (stride ld elements) -> out [P, S_pack, hp, D]
 * bf16, all_to_all_4D's send layout (P ranks, hp heads per rank, P*hp >= H: heads
 * h >= H zero; rows s >= S zero, the last rank's padding of an uneven split).
 * norm = 1 (q, k): torch.nn.RMSNorm over the H*D row in fp32 (x rsqrt(mean(x^2) +
 * eps) gamma, gamma [H*D] fp32 or NULL), rounded to bf16, then the 3D RoPE of
 * rope_apply_head_dim (:177-182): each (even, odd) pair rotated by rope_ff
 * [S, D/2, 4] fp32 = (cos_hi, cos_lo, sin_hi, sin_lo), the double cos / sin of
 * precompute_freqs_cis_3d (:125-139, assembled as :1183-1187) split into float
 * hi + lo parts; the rotation is evaluated in float-float arithmetic and rounded to
 * float, then bf16, which equals the reference's double evaluation rounded through
 * float except within ~2^-46 of a float midpoint; rstd [S] receives the norm's
 * rsqrt.  norm = 0 (v): the pack alone.
 * prism_norm_rope_pack_bwd: g [P, S_pack, hp, D] (gradient of out) -> dx [S, H*D]
 * (stride ldx): norm = 1 the conjugate rotation (float-float, rounded to bf16) then the
 * RMSNorm gradient (fp32) with x, rstd of the forward, and dgamma [H*D] fp32 (sum
 * over rows, fixed order); norm = 0 the unpack.  workspace:
 * prism_norm_rope_pack_bwd_workspace_bytes(S, H, D). */
prism_status_t prism_norm_rope_pack(const void* x, int64_t ld, int64_t S, int64_t S_pack, int H, int D,
                                    int P, int hp, const float* gamma, float eps, const float* rope_ff,
                                    int norm, void* out, float* rstd, cudaStream_t stream);
size_t prism_norm_rope_pack_bwd_workspace_bytes(int64_t S, int H, int D);
prism_status_t prism_norm_rope_pack_bwd(const void* g, const void* x, int64_t ld, int64_t S, int64_t S_pack,
                                        int H, int D, int P, int hp, const float* gamma, const float* rstd,
                                        const float* rope_ff, int norm, void* dx, int64_t ldx,
                                        void* workspace, float* dgamma, cudaStream_t stream);

/* Block-sparse attention backward (attn_bwd_bsa_varlen_triton,
 * bsa_interface.py:387-523): delta, then dK/dV over bits_k, then dQ over
 * bits_q.  o_lo: the forward's residual or NULL.
 * workspace: prism_bsa_bwd_workspace_bytes() (holds delta). */
size_t prism_bsa_bwd_workspace_bytes(int heads, int64_t S);
prism_status_t prism_bsa_bwd(const void* q, const void* k, const void* v, const void* o,
                             const void* o_lo, const void* dout, const float* lse, int heads,
                             int64_t S, int D,
                             float sm_scale, const uint32_t* bits_q, const uint32_t* bits_k,
                             const uint64_t* tile_bits, void* workspace, void* dq, void* dk,
                             void* dv, cudaStream_t stream);

/* Attention with different query and key lengths (cross-modal BSA,
 * flash_attn_bsa_cross, bsa_interface.py:1276-1392, and flash_attn_bsa_3d
 * with latent_shape_q != latent_shape_k): q, o, dO, dq [heads, Sq, D];
 * k, v, dk, dv [heads, Sk, D]; lse [heads, Sq]; bits_q [heads, Sq/64,
 * ceil(Sk/2048)], bits_k [heads, Sk/64, ceil(Sq/2048)], tile_bits [Sk/64];
 * workspace prism_bsa_bwd_workspace_bytes(heads, Sq).  Sq and Sk are positive
 * multiples of 128.  prism_bsa_fwd / prism_bsa_bwd are these with Sq == Sk. */
prism_status_t prism_bsa_fwd_qk(const void* q, const void* k, const void* v, int heads, int64_t Sq,
                                int64_t Sk, int D, float sm_scale, const uint32_t* bits_q,
                                const uint64_t* tile_bits, void* o, void* o_lo, float* lse,
                                cudaStream_t stream);
prism_status_t prism_bsa_bwd_qk(const void* q, const void* k, const void* v, const void* o,
                                const void* o_lo, const void* dout, const float* lse, int heads,
                                int64_t Sq, int64_t Sk, int D, float sm_scale,
                                const uint32_t* bits_q, const uint32_t* bits_k,
                                const uint64_t* tile_bits, void* workspace, void* dq, void* dk,
                                void* dv, cudaStream_t stream);

/* The three stages of prism_bsa_bwd, callable one by one:
 * delta[h][s] = sum_d O * dO (_attn_bwd_preprocess, common.py:94-111);
 * dK, dV per key-tile pair over the transposed selection
 * (_attn_bwd_dkdv_bsa_varlen_wrapper, flash_attn_bsa_varlen_mask.py:564-704);
 * dQ per query-tile pair (_attn_bwd_dq_bsa_varlen_align_wrapper, :881-1014). */
prism_status_t prism_bsa_bwd_delta(const void* o, const void* o_lo, const void* dout, int heads,
                                   int64_t S, int D, float* delta, cudaStream_t stream);
prism_status_t prism_bsa_bwd_dkdv(const void* q, const void* k, const void* v, const void* dout,
                                  const float* lse, const float* delta, int heads, int64_t S, int D,
                                  float sm_scale, const uint32_t* bits_k, const uint64_t* tile_bits,
                                  void* dk, void* dv, cudaStream_t stream);
prism_status_t prism_bsa_bwd_dq(const void* q, const void* k, const void* v, const void* dout,
                                const float* lse, const float* delta, int heads, int64_t S, int D,
                                float sm_scale, const uint32_t* bits_q, const uint64_t* tile_bits,
                                void* dq, cudaStream_t stream);

/* Backward without any device allocation -- no counterpart in the reference,
 * which always runs inside PyTorch's allocator.
 *
 * Some callers cannot allocate device memory at the moment they run the
 * backward: an inference or training engine that plans every byte up front
 * and forbids allocation while a step executes, a plugin hosted by a runtime
 * that owns the device pool, or code that must not call cudaMalloc because it
 * would synchronise the device mid-step.  This entry point takes the same
 * inputs and outputs as prism_bsa_bwd (minus `workspace`) and keeps its only
 * scratch, the per-row delta, in a fixed array compiled into the library:
 *   - limit: heads * S <= PRISM_BSA_BWD_NOALLOC_MAX_ROWS query rows (16 MiB of
 *     scratch, reserved on every GPU that loads the library until exit);
 *     larger calls return PRISM_ERR_INVALID_ARG;
 *   - it calls no cudaMalloc / cudaFree and no allocating library routine;
 *   - the first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *     The address is cached per device and per CUDA context: a call made
 *     under another context of the device (or after cudaDeviceReset created a
 *     new one) looks it up again;
 *   - all calls share the one array: calls whose kernels overlap on the GPU
 *     (different streams, or different host threads) race and must be
 *     serialised by the caller.  The array keeps the last call's contents;
 *     every value a call reads is first written by that same call. */
#define PRISM_BSA_BWD_NOALLOC_MAX_ROWS (4u << 20)
prism_status_t prism_bsa_bwd_noalloc(const void* q, const void* k, const void* v, const void* o,
                                     const void* o_lo, const void* dout, const float* lse,
                                     int heads, int64_t S, int D, float sm_scale,
                                     const uint32_t* bits_q, const uint32_t* bits_k,
                                     const uint64_t* tile_bits, void* dq, void* dk, void* dv,
                                     cudaStream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* PRISM_BSA_H_ */
