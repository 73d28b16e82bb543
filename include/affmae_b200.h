/*
 * affmae_b200 — C ABI of the B200 (sm_100a) kernels that replace AFFMAE's
 * custom-kernel hot path (the Triton operators of src/layers/kernels/ in
 * najafian-lab/affmae).
 *
 * Conventions shared by every entry point
 *  - All tensor arguments are device pointers to dense, row-major
 *    (C-contiguous) arrays whose shapes are given in the comment of each
 *    function.  Pointers must be 16-byte aligned where a function says so.
 *  - `dtype` is one of AFFB_F32 / AFFB_F16 / AFFB_BF16 and names the storage
 *    type of the tensors documented as "T".  Arithmetic is fp32 throughout.
 *  - `stream` is a cudaStream_t passed as void*.  Work is only enqueued;
 *    no entry point synchronises the host or allocates device memory.
 *  - Buffers documented as "fp32 accumulator, zeroed by the caller" receive
 *    atomic scatter-adds; the caller clears them before the call.
 *  - Return value: AFFB_OK, or an error code with a message available from
 *    affb_last_error() (thread-local).  Shape/argument errors are detected
 *    before anything is enqueued.
 *
 * Each declaration cites the reference interface it replaces as
 * file:line inside the reference repository.
 */
#ifndef AFFMAE_B200_H_
#define AFFMAE_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { AFFB_F32 = 0, AFFB_F16 = 1, AFFB_BF16 = 2 };
enum { AFFB_OK = 0, AFFB_ERR_INVALID = 1, AFFB_ERR_CUDA = 2 };

/* Last error message of the calling thread ("" if none). */
const char* affb_last_error(void);
/* ABI version, bumped on any signature change. */
int affb_abi_version(void);

/* ------------------------------------------------------------------ KNN --
 * Replaces knn() / KNNFunction / knn_forward
 * (src/layers/kernels/knn.py:1615, :1543, :1368) and the K>8 fallback
 * knn_pytorch_large (knn.py:1312) with one exact kernel for every K.
 * query [B,M,D] T, ref [B,N,D] T, D in {2,3,4}, 1 <= K <= min(N, 256).
 * out_idx [B,M,K] int64: indices of the K nearest refs by fp32 squared
 * Euclidean distance (products and sums rounded separately, no FMA),
 * ascending, ties broken by lower index.                                   */
int affb_knn(const void* query, const void* ref, int dtype, int64_t B, int64_t M,
             int64_t N, int D, int K, int64_t* out_idx, void* stream);
/* 2-D K-nearest neighbours through a uniform grid of the reference points:
 * same contract and result as affb_knn with D = 2, for fp32 points.
 * workspace: affb_knn2d_workspace_bytes(B, N) bytes, 256-byte aligned.    */
int64_t affb_knn2d_workspace_bytes(int64_t B, int64_t N);
int affb_knn2d(const float* query, const float* ref, int64_t B, int64_t M, int64_t N, int K,
               int64_t* out_idx, void* workspace, int64_t workspace_bytes, void* stream);

/* -------------------------------------------------- weighted features --
 * Replaces WeightedFeaturesFunction (src/layers/kernels/weighted_features.py:401)
 * and, with IC = 1, WeightedGatherFunction (weighted_gather.py:329).
 * out[b,i,ic,c] = sum_m w[b,i,m,ic] * feat[b, idx[b,i,m], c]
 * w [B,No,M,IC] T, feat [B,N,C] T, idx [B,No,M] int32, out [B,No,IC,C] T.  */
int affb_weighted_features_fwd(const void* w, const void* feat, const int32_t* idx, int dtype,
                               int64_t B, int64_t No, int64_t M, int64_t IC, int64_t N,
                               int64_t C, void* out, void* stream);
/* Backward (weighted_features.py:164-345, weighted_gather.py:127-276):
 * dw [B,No,M,IC] T (written), dfeat_acc [B,N,C] fp32 accumulator zeroed by
 * the caller (scatter-added).                                              */
int affb_weighted_features_bwd(const void* dout, const void* w, const void* feat,
                               const int32_t* idx, int dtype, int64_t B, int64_t No,
                               int64_t M, int64_t IC, int64_t N, int64_t C, void* dw,
                               float* dfeat_acc, void* stream);

/* ------------------------------------------- neighbourhood attention --
 * Replaces launch_flash_nbhood_attn_fwd (src/layers/kernels/local_attn.py:609)
 * i.e. the forward of FlashLocalAttentionFunction (local_attn.py:843).
 * q,k,v [B,H,N,D] T (D % 8 == 0, D <= 256, 16-byte aligned);
 * member_idx [B,N,M] int32 (M % 8 == 0); bias [B,H,N,M] T or NULL;
 * mask [B,mask_heads,N,M] uint8 (nonzero = attend) or NULL, mask_heads in {1,H};
 * blank_k, blank_v [H,D] T or NULL (both or neither);
 * out [B,H,N,D] T; lse [B,H,N] fp32.                                       */
int affb_nbhd_attn_fwd(const void* q, const void* k, const void* v, const int32_t* member_idx,
                       const void* bias, const uint8_t* mask, int mask_heads,
                       const void* blank_k, const void* blank_v, int dtype, int64_t B,
                       int64_t H, int64_t N, int64_t D, int64_t M, float scale, void* out,
                       float* lse, void* stream);
/* Replaces launch_flash_nbhood_attn_bwd (local_attn.py:711).
 * o, dout [B,H,N,D] T; lse [B,H,N] fp32 from the forward.
 * dq, dk, dv [B,H,N,D] T (written); dbias [B,H,N,M] T (written) or NULL
 * when bias is NULL; dbk_acc, dbv_acc [H,D] fp32 accumulators zeroed by the
 * caller, or NULL when there is no blank token.  workspace: device memory of
 * at least affb_nbhd_attn_bwd_workspace_bytes(...) bytes, 256-byte aligned,
 * no initial contents (the reference allocates its fp32 dK / dV buffers
 * itself, local_attn.py:785-787).  member_idx 16-byte aligned.            */
int64_t affb_nbhd_attn_bwd_workspace_bytes(int dtype, int64_t B, int64_t H, int64_t N,
                                           int64_t D, int64_t M);
int affb_nbhd_attn_bwd(const void* q, const void* k, const void* v, const void* o,
                       const void* dout, const float* lse, const int32_t* member_idx,
                       const void* bias, const uint8_t* mask, int mask_heads,
                       const void* blank_k, const void* blank_v, int dtype, int64_t B,
                       int64_t H, int64_t N, int64_t D, int64_t M, float scale, void* dq,
                       void* dk, void* dv, void* dbias, float* dbk_acc, float* dbv_acc,
                       void* workspace, int64_t workspace_bytes, void* stream);

/* The same forward and backward sharing the tiles' cluster unions (no
 * counterpart in the reference, whose backward re-reads member_idx per query
 * block).  On the tensor-core path (bf16 / fp16, D == 32, M <= 64) the
 * forward builds, per tile of 16 queries, the union of the key clusters they
 * list and a run-offset table; affb_nbhd_attn_fwd_plan also stores them in
 * `tile_plan` (affb_nbhd_tile_plan_bytes(...) bytes, 16-byte aligned; 0
 * bytes off the tensor-core path), and affb_nbhd_attn_bwd_plan's dQ kernel
 * reads them instead of rebuilding them.  The plan is valid for the
 * member_idx and mask of the forward that wrote it.                        */
int64_t affb_nbhd_tile_plan_bytes(int dtype, int64_t B, int64_t N, int64_t D, int64_t M);
int affb_nbhd_attn_fwd_plan(const void* q, const void* k, const void* v, const int32_t* member_idx,
                            const void* bias, const uint8_t* mask, int mask_heads, const void* blank_k,
                            const void* blank_v, int dtype, int64_t B, int64_t H, int64_t N, int64_t D,
                            int64_t M, float scale, void* out, float* lse, void* tile_plan,
                            int64_t tile_plan_bytes, void* stream);
int affb_nbhd_attn_bwd_plan(const void* q, const void* k, const void* v, const void* o,
                            const void* dout, const float* lse, const int32_t* member_idx,
                            const void* bias, const uint8_t* mask, int mask_heads, const void* blank_k,
                            const void* blank_v, int dtype, int64_t B, int64_t H, int64_t N, int64_t D,
                            int64_t M, float scale, void* dq, void* dk, void* dv, void* dbias,
                            float* dbk_acc, float* dbv_acc, const void* tile_plan, int64_t tile_plan_bytes,
                            void* workspace, int64_t workspace_bytes, void* stream);

/* ------------------------------------------------ relative-position bias --
 * Replaces the gather of ClusterAttention._make_pos_bias
 * (src/layers/attention.py:110-124):
 * out[b,h,n,m] = table[pe_idx[b,n,m], h]; table [T,H] T, pe_idx [B,N,M] int64,
 * out [B,H,N,M] T.                                                          */
int affb_pos_bias_fwd(const void* table, const int64_t* pe_idx, int dtype, int64_t T,
                      int64_t H, int64_t B, int64_t N, int64_t M, void* out, void* stream);
/* dtable_acc [T,H] fp32 accumulator zeroed by the caller.                  */
int affb_pos_bias_bwd(const void* dbias, const int64_t* pe_idx, int dtype, int64_t T,
                      int64_t H, int64_t B, int64_t N, int64_t M, float* dtable_acc,
                      void* stream);

/* Relative-position bias evaluated in the kernel (no table): replaces
 * Linear(5 -> H)(pre_table) followed by the gather of _make_pos_bias
 * (src/layers/attention.py:111-124; pre_table of src/utils/pos_embed.py:8-22).
 * out[b,h,n,m] = weight[h,:] . f(pe_idx[b,n,m]) + bias[h] with
 * f(i) = (dx, dy, r, dy/r, dx/r), dx = i % 255 - 127, dy = i / 255 - 127
 * (last three 0 at r = 0).  weight [H,5] fp32, bias [H] fp32, pe_idx
 * [B,N,M] int64 in [0, 65025), out [B,H,N,M] T, H <= 32.                   */
int affb_rel_bias_fwd(const float* weight, const float* bias, const int64_t* pe_idx, int dtype,
                      int64_t H, int64_t B, int64_t N, int64_t M, void* out, void* stream);
/* dweight [H,5], dbias_vec [H]: fp32 accumulators zeroed by the caller.    */
int affb_rel_bias_bwd(const void* dbias, const int64_t* pe_idx, int dtype, int64_t H, int64_t B,
                      int64_t N, int64_t M, float* dweight, float* dbias_vec, void* stream);

/* ------------------------------------------------------- head layout --
 * The per-head splits and merges of ClusterAttention
 * (src/layers/attention.py:126-207: q / kv projections viewed as
 * [B,N,H,d] and permuted to [B,H,N,d], the output permuted back), and their
 * gradients: dst[b,n,h,j] = src[b,n,h,j] for j < d, each side addressed by
 * its own batch / token / head strides in elements, d contiguous.
 * elem_bytes 2 or 4; d * elem_bytes, every stride * elem_bytes and both
 * pointers multiples of 16 bytes.                                          */
int affb_head_copy(const void* src, int64_t src_sb, int64_t src_sn, int64_t src_sh, void* dst,
                   int64_t dst_sb, int64_t dst_sn, int64_t dst_sh, int64_t elem_bytes, int64_t B,
                   int64_t N, int64_t H, int64_t d, void* stream);

/* ------------------------------- fused residual + dropout + LayerNorm --
 * The add / dropout / LayerNorm / dtype-cast sequences around the operators
 * above in the model (decoder blocks, src/layers/decoder.py:114-143, and the
 * encoder pre-norms, src/layers/aff.py:95-115) as one pass per direction.
 * Forward: s = x + dropout_p(delta) (delta may be NULL), y = LN(s) written to
 * y32 (fp32) and/or y16_bf16; rows R of C <= 1536 channels; x and delta fp32
 * or bf16; s_saved [R,C] fp32 (needed with delta), mean/rstd [R] fp32.  The
 * dropout mask is Philox-4x32-10 of (seed, element index); the same seed and
 * p regenerate it in the backward.                                         */
int affb_layer_norm_fwd(const void* x, int x_dtype, const void* delta, int delta_dtype, float p,
                        uint32_t seed, const float* gamma, const float* beta, float eps, int64_t R,
                        int64_t C, float* s_saved, float* mean, float* rstd, float* y32,
                        void* y16_bf16, void* stream);
/* Backward: dy32 and/or dy16_bf16 summed; s = s_saved (fp32) or x (s_dtype);
 * dx written in s_dtype, ddelta (NULL when the forward had no delta) in
 * delta_dtype; dgamma, dbeta [C] fp32 accumulators zeroed by the caller.    */
int affb_layer_norm_bwd(const float* dy32, const void* dy16_bf16, const void* s, int s_dtype,
                        const float* mean, const float* rstd, const float* gamma, float p,
                        uint32_t seed, int64_t R, int64_t C, void* dx, void* ddelta,
                        int delta_dtype, float* dgamma, float* dbeta, void* stream);
/* Pre-norm residual form (ClusterTransformerBlock, src/layers/aff.py:95-115:
 * x = x + drop_path(branch); y = norm(x)): s = x + row_scale[r / rows_per_scale]
 * * dropout_p(delta) (row_scale NULL: factor 1), y = LayerNorm(s).  s is an
 * fp32 result (the residual stream), not only a saved value.  The backward
 * takes ds_in, the fp32 gradient of s from its other uses (or NULL), adds the
 * normalisation's gradient to it and writes dx (fp32) and
 * ddelta = dx * factor * dropout scale.                                      */
int affb_layer_norm_res_fwd(const void* x, int x_dtype, const void* delta, int delta_dtype, float p,
                            uint32_t seed, const float* row_scale, int64_t rows_per_scale,
                            const float* gamma, const float* beta, float eps, int64_t R, int64_t C,
                            float* s, float* mean, float* rstd, float* y32, void* y16_bf16, void* stream);
int affb_layer_norm_res_bwd(const float* dy32, const void* dy16_bf16, const float* ds_in,
                            const float* s, const float* mean, const float* rstd, const float* gamma,
                            float p, uint32_t seed, const float* row_scale, int64_t rows_per_scale,
                            int64_t R, int64_t C, float* dx, void* ddelta, int delta_dtype,
                            float* dgamma, float* dbeta, void* stream);
/* Host-side evaluation of that dropout mask: keep[i] = 1 when element e0 + i
 * survives dropout p under `seed` (the kernels' exact rule).  No GPU.  Part
 * of the model glue; the reference uses torch's dropout here.              */
int affb_dropout_keep_mask(uint32_t seed, float p, int64_t e0, int64_t n, uint8_t* keep);

/* Neighbour lists of an encoder stage (BasicLayer.forward,
 * src/layers/aff.py:426-465) from the ids of every token's nnc nearest
 * clusters: pos [B,n,2] fp32 in cluster order (clusters of 8 consecutive
 * tokens), nearest [B,n,nnc] int64 (e.g. from affb_knn2d against the cluster
 * means).  Writes member_idx [B,n,8 nnc] int32 (8c+r, or 0 past the last
 * token), mask [B,n,8 nnc] uint8 (8c+r < n; NULL to skip) and pe_idx
 * [B,n,8 nnc] int64 = y*255 + x of clamp(pos[member] - pos[q] + 127, 0, 254),
 * with the fp32 rounding of the reference's PyTorch sequence.               */
int affb_nbhd_build(const float* pos, const int64_t* nearest, int64_t B, int64_t n, int64_t nnc,
                    int32_t* member_idx, uint8_t* mask, int64_t* pe_idx, void* stream);

/* Token-mask multiply of the masked-autoencoder patch stem: the re-masking
 * after each stride-2 convolution of AFFPatchEmbed (src/layers/aff.py:591-639)
 * without materialising the upsampled mask.  x, out [B,h,w,C] T
 * (channels-last), token_mask [B,th,tw] uint8 (nonzero = keep), h/th = w/tw
 * an integer s: out[b,y,x,c] = x[b,y,x,c] * token_mask[b,y/s,x/s].  Also the
 * gradient (the same product).                                              */
int affb_token_mask_apply(const void* x, int dtype, int64_t B, int64_t h, int64_t w, int64_t C,
                          const uint8_t* token_mask, int64_t th, int64_t tw, void* out, void* stream);

/* ReLU followed by dropout (the decoder feed-forward network,
 * src/layers/decoder.py:138-141: dropout3(relu(linear1(x)))) in one pass:
 * y[e] = (x[e] > 0 and keep(seed, e)) ? x[e] / (1 - p) : 0 over n elements,
 * keep() being the same Philox-4x32-10 stream as affb_dropout_keep_mask; p = 0
 * gives a plain ReLU.  The gradient needs no mask: dx = (y > 0) ? dy / (1 - p)
 * : 0.  x, y, dy, dx: n elements of dtype. */
/* Normalised sine position embedding (PositionEmbeddingSine,
 * src/layers/decoder.py:16-62, normalize=True): pos [R,2] fp32 -> out [R,D]
 * of dtype, out = [sin(u_x[0::2]), cos(u_x[1::2]), sin(u_y[0::2]),
 * cos(u_y[1::2])] with u = coord / (maxes[axis] + 1e-6) * 2pi / freq;
 * maxes [2] (device, fp32) are the coordinate maxima over all rows, freq
 * [D/2] (device, fp32) the frequency table.  D a multiple of 4. */
int affb_sine_embed(const float* pos, int64_t R, int64_t D, const float* maxes, const float* freq, void* out,
                    int dtype, void* stream);

int affb_relu_dropout_fwd(const void* x, int dtype, int64_t n, float p, uint32_t seed, void* y, void* stream);
int affb_relu_dropout_bwd(const void* dy, const void* y, int dtype, int64_t n, float p, void* dx, void* stream);

/* --------------------------------- fused KNN deformable attention (2-D) --
 * Replaces fused_knn_deform_cross_attn_forward_save
 * (src/layers/kernels/fused_deform_attn.py:2592) and, with kv_pos == query_pos
 * and Nkv == Nq, fused_knn_deform_self_attn_forward_save (:2530).
 * query_pos [B,Nq,2] fp32, kv_pos [B,Nkv,2] fp32, offsets [B,Nq,H,4,2] fp32,
 * attn_w [B,Nq,H,4] fp32, values [B,Nkv,H,C] T (C % 8 == 0, H <= 16),
 * power: 1 fp32 on device (clamped to >= 1e-6 on device).  For every
 * (query, head, point) the sample s = query_pos + offset; its 4 nearest kv
 * positions (fp32 squared distance, ties -> lower index) get Shepard weights
 * softmax(-P*(sqrt(d2)+1e-6)) with +1e-8 in the denominator;
 * out [B,Nq,H,C] T = sum_p attn_w * sum_j w_j v_j.
 * knn_idx [B,Nq,H,4,4] int32 and knn_d2 [B,Nq,H,4,4] fp32 are written for the
 * backward (knn_d2 may be NULL: not written).  `workspace` (device, affb_deform_workspace_bytes(B,Nkv) bytes,
 * 256-byte aligned) receives the spatial grid of kv_pos built by this call. */
int64_t affb_deform_workspace_bytes(int64_t B, int64_t Nkv);
int affb_deform_knn_fwd(const float* query_pos, const float* kv_pos, const float* offsets,
                        const float* attn_w, const void* values, const float* power,
                        int dtype, int64_t B, int64_t Nq, int64_t Nkv, int64_t H, int64_t C,
                        void* out, int32_t* knn_idx, float* knn_d2, void* workspace,
                        void* stream);
/* Allocation-free variant of affb_deform_knn_fwd; it has no counterpart in
 * the reference.  For callers that may not allocate device memory on the
 * call path: hosts whose device memory is owned by another allocator (a
 * framework's caching allocator, an inference engine's memory pool or a
 * plugin interface that only hands over input/output buffers), where a
 * cudaMalloc would synchronise the device and bypass the owner's budget.
 * Same arguments and results as affb_deform_knn_fwd minus `workspace`: the
 * spatial grid is built in a fixed device array of
 * affb_deform_noalloc_max_scratch_bytes() bytes (16 MiB) that every GPU
 * loading the library holds until the process exits.  Sizes whose grid
 * (affb_deform_workspace_bytes(B, Nkv)) exceeds it are rejected with an
 * error.  The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress) and caches it, so make that first call before any
 * stream capture.  Every call on a device shares that device's array, which
 * keeps the last call's contents (each call clears what it needs cleared);
 * calls whose GPU work can overlap (for example on unordered streams) race
 * on it and must be serialised by the caller.  The cached address belongs to
 * the device's primary context: do not use this entry point across a
 * cudaDeviceReset (or a release and re-creation of the primary context) in
 * the same process.                                                        */
int64_t affb_deform_noalloc_max_scratch_bytes(void);
int affb_deform_knn_fwd_noalloc(const float* query_pos, const float* kv_pos,
                                const float* offsets, const float* attn_w, const void* values,
                                const float* power, int dtype, int64_t B, int64_t Nq,
                                int64_t Nkv, int64_t H, int64_t C, void* out, int32_t* knn_idx,
                                float* knn_d2, void* stream);

/* Replaces fused_knn_deform_cross_attn_backward (fused_deform_attn.py:2792)
 * and fused_knn_deform_self_attn_backward (:2661).  dout [B,Nq,H,C] T.
 * Written: d_offsets [B,Nq,H,4,2] fp32, d_attn_w [B,Nq,H,4] fp32.
 * Accumulated (zeroed by the caller): d_qpos [B,Nq,2] fp32,
 * d_kvpos [B,Nkv,2] fp32 (may alias d_qpos for self-attention),
 * d_values_acc [B,Nkv,H,C] fp32, d_power [1] fp32.  knn_d2 may be NULL: the
 * squared distances are then recomputed from the positions with the
 * forward's rounding (the same values bit for bit).                        */
int affb_deform_knn_bwd(const float* query_pos, const float* kv_pos, const float* offsets,
                        const float* attn_w, const void* values, const float* power,
                        const int32_t* knn_idx, const float* knn_d2, const void* dout,
                        int dtype, int64_t B, int64_t Nq, int64_t Nkv, int64_t H, int64_t C,
                        float* d_offsets, float* d_attn_w, float* d_qpos, float* d_kvpos,
                        float* d_values_acc, float* d_power, void* stream);

/* ------------------------ deformable attention with given neighbours --
 * Replaces fused_deform_attn_forward / _backward
 * (src/layers/kernels/fused_deform_attn.py:502-640).
 * sl [B,N,D] fp32, kv_pos [B,Nkv,D] fp32, nb_idx [B,N,K] int32 (K <= 16),
 * power 1 fp32 on device, attn_w [B,N] fp32, values [B,Nkv,C] T,
 * out [B,N,C] T = attn_w * sum_k softmax_k(-P*(sqrt(d2)+1e-6)) values[nb].  */
int affb_deform_nbidx_fwd(const float* sl, const float* kv_pos, const int32_t* nb_idx,
                          const float* power, const float* attn_w, const void* values,
                          int dtype, int64_t B, int64_t N, int64_t Nkv, int64_t K, int D,
                          int64_t C, void* out, void* stream);
/* Written: d_sl [B,N,D] fp32, d_attn_w [B,N] fp32.  Accumulated (zeroed by
 * the caller): d_kvpos [B,Nkv,D] fp32, d_power [1] fp32, d_values_acc
 * [B,Nkv,C] fp32.                                                          */
int affb_deform_nbidx_bwd(const float* sl, const float* kv_pos, const int32_t* nb_idx,
                          const float* power, const float* attn_w, const void* values,
                          const void* dout, int dtype, int64_t B, int64_t N, int64_t Nkv,
                          int64_t K, int D, int64_t C, float* d_sl, float* d_kvpos,
                          float* d_power, float* d_attn_w, float* d_values_acc,
                          void* stream);

/* ------------------------------------------------------------ MSDETRPC --
 * Replaces MSDETRPCFunction (src/layers/kernels/msdetrpc.py:372).
 * out[b,n,c] = sum_m attn[b,n,m] * sum_k w[b,n,m,k] * val[b, idx[b,n,m,k], c]
 * idx [B,N,M,K] int32, w [B,N,M,K] T, attn [B,N,M] T, val [B,Nv,C] T,
 * out [B,N,C] T.                                                            */
int affb_msdetrpc_fwd(const int32_t* idx, const void* w, const void* attn, const void* val,
                      int dtype, int64_t B, int64_t N, int64_t M, int64_t K, int64_t Nv,
                      int64_t C, void* out, void* stream);
/* dw [B,N,M,K] T and dattn [B,N,M] T written; dval_acc [B,Nv,C] fp32
 * accumulator zeroed by the caller.                                        */
int affb_msdetrpc_bwd(const void* dout, const int32_t* idx, const void* w, const void* attn,
                      const void* val, int dtype, int64_t B, int64_t N, int64_t M, int64_t K,
                      int64_t Nv, int64_t C, void* dw, void* dattn, float* dval_acc,
                      void* stream);

/* ------------------------------------------------------------ MSSample --
 * Replaces MSSampleFunction (src/layers/kernels/mssample.py:402).
 * sl [B,N,D] fp32, kv_pos [B,Nkv,D] fp32, nb_idx [B,N,K] int32 (K <= 16),
 * power 1 fp32 on device; w_out [B,N,K] fp32 =
 * softmax_k(-P*sqrt(d2+1e-6)) with +1e-8 in the denominator.               */
int affb_mssample_fwd(const float* sl, const float* kv_pos, const int32_t* nb_idx,
                      const float* power, int64_t B, int64_t N, int64_t Nkv, int64_t K, int D,
                      float* w_out, void* stream);
/* dw [B,N,K] fp32 upstream gradient; w the forward output.  Written: d_sl
 * [B,N,D] fp32.  Accumulated (zeroed by the caller): d_kvpos [B,Nkv,D],
 * d_power [1].                                                              */
int affb_mssample_bwd(const float* dw, const float* sl, const float* kv_pos,
                      const int32_t* nb_idx, const float* power, const float* w, int64_t B,
                      int64_t N, int64_t Nkv, int64_t K, int D, float* d_sl, float* d_kvpos,
                      float* d_power, void* stream);

/* ----------------------------------------------------------- utilities --
 * dst[i] = (T) src[i] for n elements (fp32 accumulator -> storage dtype).
 * No counterpart in the reference (it casts with torch's .to()).           */
int affb_cast_f32(const float* src, void* dst, int dtype, int64_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* AFFMAE_B200_H_ */
