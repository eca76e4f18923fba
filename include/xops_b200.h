/*
 * xops_b200 -- C ABI of the B200 (sm_100a) build of the xLLM GDN
 * linear-attention and normalisation hot path.
 *
 * Every entry point takes raw device pointers, element counts/strides and a
 * cudaStream_t (passed as void*), validates its arguments on the host before
 * launching anything, enqueues its kernels on that stream and returns an
 * xops_status_t.  Nothing synchronises the stream and nothing allocates
 * device memory: where a kernel needs scratch, the caller passes a workspace
 * sized by the matching *_workspace_size query.  On failure the call launches
 * nothing (argument errors) and xops_last_error() holds a message for the
 * calling thread.
 *
 * Each declaration names the reference interface it replaces (paths relative
 * to the reference project root).  Layout conventions follow the reference:
 * token-major [B, T, H, D] tensors, varlen batches as B == 1 plus int32
 * cu_seqlens [N+1], grouped-query heads h -> h / (H / Hg).
 */
#ifndef XOPS_B200_H_
#define XOPS_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define XOPS_API __attribute__((visibility("default")))
#else
#define XOPS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
  XOPS_OK = 0,
  XOPS_ERR_INVALID_ARGUMENT = 1, /* bad shape / pointer / dtype (TORCH_CHECK) */
  XOPS_ERR_UNSUPPORTED = 2,      /* valid request outside the compiled kernels */
  XOPS_ERR_CUDA = 3,             /* launch or runtime error from CUDA */
  XOPS_ERR_WORKSPACE = 4         /* workspace missing or too small */
} xops_status_t;

typedef enum { XOPS_F32 = 0, XOPS_BF16 = 1, XOPS_F16 = 2 } xops_dtype_t;

/* Message of the last failing call on this thread ("" if none). */
XOPS_API const char* xops_last_error(void);
/* Library version string. */
XOPS_API const char* xops_version(void);
/* Number of kernel launches this library has issued (process-wide). */
XOPS_API uint64_t xops_launch_count(void);

/* ---------------------------------------------------------------- norms -- */

/* y = x * rsqrt(sum(x^2) + eps) over the last axis; x, y [rows, cols], bf16
 * or fp32, contiguous.  Replaces npu_l2norm_last_dim
 * (triton_npu/torch_api/npu_triton_l2norm.cpp:52-108). */
XOPS_API int xops_l2norm_last_dim(const void* x, void* y, int64_t rows, int64_t cols, float eps,
                         int dtype, void* stream);

/* Grouped LayerNorm / RMSNorm with optional bias and SiLU gate z.
 * x, z [M, N] with row strides; y [M, N] (row stride stride_y); weight,
 * bias [N]; mean (LayerNorm only, may be NULL for RMSNorm) and rstd are fp32
 * [ngroups * M] indexed group * M + row.  norm_before_gate selects
 * y = norm(x)*w(+b) * silu(z) (1) or norm(x * silu(z))*w(+b) (0).
 * x/z/y dtype x_dtype; weight/bias dtype w_dtype.  Replaces layer_norm_fwd
 * (triton_npu/torch_api/npu_triton_layernorm_fwd.cpp:48-333) and
 * npu_ops::layer_norm_fwd / aclnnLayerNormFwd
 * (ascendc_npu/layer_norm_fwd.cpp:24-82). */
XOPS_API int xops_layer_norm_fwd(const void* x, const void* weight, const void* bias, const void* z,
                        void* y, float* mean, float* rstd, int64_t M, int64_t N,
                        int64_t group_size, int64_t stride_x_row, int64_t stride_z_row,
                        int64_t stride_y_row, float eps, int norm_before_gate,
                        int is_rms_norm, int x_dtype, int w_dtype, void* stream);

/* Gemma RMSNorm y = x * rsqrt(mean(x^2) + eps) * (1 + gamma) over rows of
 * length cols; rstd fp32 [rows].  Replaces npu_ops::npu_gemma_rms_norm /
 * aclnnGemmaRmsNorm (ascendc_npu/gemma_rms_norm.cpp:28-57). */
XOPS_API int xops_gemma_rms_norm(const void* x, const void* gamma, void* y, float* rstd, int64_t rows,
                        int64_t cols, float eps, int x_dtype, int gamma_dtype, void* stream);

/* ----------------------------------------------------------------- rope -- */

/* Split packed [T, q_hidden + 2*kv_hidden] into q, k, v; per-head RMSNorm
 * (weight [head_dim] shared by heads, optional bias) on q and k; NeoX
 * rotate-half RoPE on the first rotary_dim dims with per-token sin/cos
 * [T, rotary_dim]; v copied.  Outputs contiguous in the input dtype.
 * rotary_dim == head_dim is the reference kernel; rotary_dim < head_dim is
 * the partial-rotary extension.  Replaces npu_split_rmsnorm_rope
 * (triton_npu/torch_api/npu_triton_split_rmsnorm_rope.cpp:57-143). */
XOPS_API int xops_split_rmsnorm_rope(const void* input, const void* sin, const void* cos, void* q_out,
                            void* k_out, void* v_out, const void* q_weight, const void* q_bias,
                            const void* k_weight, const void* k_bias, int64_t num_tokens,
                            int64_t q_hidden, int64_t kv_hidden, int64_t head_dim,
                            int64_t rotary_dim, float eps, int dtype, int w_dtype,
                            int sincos_dtype, void* stream);

/* Interleaved RoPE on the last rope_dim dims of x [rows, heads, hidden]
 * (row stride x_stride_row, head stride x_stride_head, unit element
 * stride), in place: pairs (2i, 2i+1) -> (x0 cos0 - x1 sin0, x1 cos1 +
 * x0 sin1).  sin, cos [rows, >= rope_dim] with row stride sincos_stride,
 * shared by a row's heads.  Replaces rope_inplace
 * (triton_npu/torch_api/npu_triton_rope_inplace.cpp:22-66). */
XOPS_API int xops_rope_inplace(void* x, const void* sin, const void* cos, int64_t rows,
                               int64_t heads, int64_t hidden, int64_t rope_dim,
                               int64_t x_stride_row, int64_t x_stride_head,
                               int64_t sincos_stride, int x_dtype, int sincos_dtype,
                               void* stream);

/* --------------------------------------------------------------- conv1d -- */

/* Decode-style depthwise causal conv update.  x [batch, dim, seqlen] with
 * strides (x_stride_b, x_stride_d, x_stride_t); out same shape, contiguous;
 * conv_state [num_cache_lines, dim, state_len] contiguous, updated in place
 * (state <- last state_len columns of cat(state, x)); weight [dim, width];
 * bias [dim] or NULL; conv_state_indices [batch] int32 or NULL (identity);
 * rows whose slot equals pad_slot_id are skipped.  Replaces
 * npu_causal_conv1d_update (triton_npu/torch_api/npu_triton_causal_conv1d_update.cpp:22-137). */
XOPS_API int xops_causal_conv1d_update(const void* x, void* conv_state, const void* weight,
                              const void* bias, const int32_t* conv_state_indices, void* out,
                              int64_t batch, int64_t dim, int64_t seqlen, int64_t width,
                              int64_t state_len, int64_t num_cache_lines, int64_t x_stride_b,
                              int64_t x_stride_d, int64_t x_stride_t, int silu,
                              int32_t pad_slot_id, int dtype, void* stream);

/* Varlen (prefill) depthwise causal conv: x [total_tokens, dim] token-major,
 * out same; query_start_loc [batch+1] int32; conv_state
 * [num_cache_lines, dim, width-1] holds each sequence's history and is
 * updated in place to the last width-1 inputs of cat(history, x_seq).
 * Replaces npu_causal_conv1d_update_v2 with query_start_loc
 * (triton_npu/torch_api/npu_triton_causal_conv1d_update_v2.cpp:99-239). */
XOPS_API int xops_causal_conv1d_varlen(const void* x, void* conv_state, const void* weight,
                              const void* bias, const int32_t* query_start_loc,
                              const int32_t* conv_state_indices, void* out, int64_t batch,
                              int64_t total_tokens, int64_t dim, int64_t width,
                              int64_t num_cache_lines, int silu, int32_t pad_slot_id, int dtype,
                              void* stream);

/* The varlen prefill conv of xops_causal_conv1d_varlen with the GDN layer's
 * q/k L2 normalisation fused into its output: the first l2_channels output
 * channels (whole 128-channel heads: the q and k blocks of the layer's conv
 * output) are written as y / sqrt(sum y^2 + l2_eps) over each head, computed
 * from the bf16-rounded conv output, exactly as npu_l2norm_last_dim would
 * compute it in a separate pass (npu_triton_chunk_gated_delta_rule.cpp:608-609
 * calls it on q and k when use_qk_l2norm_in_kernel).  The chunked rule then
 * runs with use_qk_l2norm_in_kernel = 0 on views of this output.  16-bit
 * activations, dim a multiple of 128.  This fused form has no single
 * counterpart in the reference, which runs the two steps separately. */
XOPS_API int xops_causal_conv1d_varlen_qk_l2norm(
    const void* x, void* conv_state, const void* weight, const void* bias,
    const int32_t* query_start_loc, const int32_t* conv_state_indices, void* out, int64_t batch,
    int64_t total_tokens, int64_t dim, int64_t width, int64_t num_cache_lines, int silu,
    int32_t pad_slot_id, int dtype, int64_t l2_channels, float l2_eps, void* stream);

/* Prefill conv reading the GDN layer's input projection in place:
 * mixed_qkvz [total_tokens, num_k_heads * (2 + 2r) * 128] (row stride x_ld
 * elements), per key head q (128) | k (128) | v (r value heads x 128) | z
 * (r x 128), r = num_v_heads / num_k_heads, the layout
 * fused_qkvzba_split_reshape_cat de-interleaves
 * (triton_npu/triton_src/test_fused_qkvzba_split_reshape.py:463-507).  The
 * conv channels are all q heads, then all k heads, then all v heads
 * (dim = (2 num_k_heads + num_v_heads) * 128, the order of the split's
 * mixed_qkv); weight [dim, width], bias [dim], conv_state and out as
 * xops_causal_conv1d_varlen_qk_l2norm, whose q/k L2 normalisation is applied
 * when qk_l2norm is set.  Equals the split followed by that conv, without
 * the split's read and write of the projection. */
XOPS_API int xops_causal_conv1d_varlen_qkvz(
    const void* mixed_qkvz, int64_t x_ld, int64_t num_k_heads, int64_t num_v_heads,
    void* conv_state, const void* weight, const void* bias, const int32_t* query_start_loc,
    const int32_t* conv_state_indices, void* out, int64_t batch, int64_t total_tokens,
    int64_t width, int64_t num_cache_lines, int silu, int32_t pad_slot_id, int dtype,
    int qk_l2norm, float l2_eps, void* stream);

/* De-interleave of the GDN input projections.  mixed_qkvz [rows, nqk *
 * (2 hqk + 2 r hv)] holds per key head q | k | v (r heads) | z (r heads),
 * r = num_heads_v / num_heads_qk in [1, 4]; mixed_ba [rows, nqk * 2r] holds
 * b (r) | a (r).  Outputs: mixed_qkv [rows, 2 nqk hqk + nv hv] (all q, all
 * k, all v), z [rows, nv, hv] in qkvz_dtype; b, a [rows, nv] in ba_dtype.
 * All contiguous.  Replaces npu_fused_qkvzba_split_reshape_cat
 * (triton_npu/torch_api/npu_triton_fused_qkvzba_split_reshape.cpp:105-206). */
XOPS_API int xops_fused_qkvzba_split_reshape_cat(const void* mixed_qkvz, const void* mixed_ba,
                                                 void* mixed_qkv, void* z, void* b, void* a,
                                                 int64_t rows, int64_t num_heads_qk,
                                                 int64_t num_heads_v, int64_t head_qk,
                                                 int64_t head_v, int qkvz_dtype, int ba_dtype,
                                                 void* stream);

/* npu_causal_conv1d_update_v2 with slot tables: speculative decoding
 * (num_accepted_tokens [batch]) and prefix-cache block tables
 * (conv_state_indices [batch, *] with row stride indices_stride, plus
 * initial_state_idx / block_idx_last_scheduled_token [batch], both or
 * neither).  x, out [num_tokens, dim] token-major with query_start_loc
 * [batch+1]; conv_state [num_cache_lines, dim, state_len], state_len >=
 * width - 1, updated in place.  Sequence b reads line idx[b, init[b]]
 * (idx[b] for a [batch] table, b without one) from column
 * num_accepted_tokens[b] - 1 (0 without), and writes columns [0, L) of line
 * idx[b, last[b]], L = width - 1 + (speculative ? len_b - 1 : 0).  A line
 * equal to pad_slot_id or outside the cache skips the row.  Replaces the
 * slot-table paths of npu_causal_conv1d_update_v2
 * (triton_npu/torch_api/npu_triton_causal_conv1d_update_v2.cpp:99-239). */
XOPS_API int xops_causal_conv1d_update_v2_slots(
    const void* x, void* conv_state, const void* weight, const void* bias,
    const int32_t* conv_state_indices, int64_t indices_stride, const int32_t* num_accepted_tokens,
    const int32_t* initial_state_idx, const int32_t* block_idx_last_scheduled_token,
    const int32_t* query_start_loc, void* out, int64_t batch, int64_t dim, int64_t width,
    int64_t state_len, int64_t num_cache_lines, int silu, int32_t pad_slot_id, int dtype,
    void* stream);

/* ---------------------------------------------------- gated delta rule -- */

/* Token-serial gated delta rule (decode).  q, k [B, T, H, K], v [B, T, HV, V]
 * bf16; g, beta [B, T, HV] fp32 (beta may be NULL = ones); o [B, T, HV, V]
 * bf16; h0 fp32 state slots [*, HV, K, V] with slot stride h0_stride.
 * Sequences: cu_seqlens [N+1] int32, or NULL with N == B rows of T tokens.
 * State slots: ssm_state_indices NULL (slot n), or an int32 table whose
 * entry for (sequence n, token t) is at n * idx_stride_seq + t *
 * idx_stride_tok (idx_stride_tok == 0: one slot per sequence).  The initial
 * state comes from token 0, or from token num_accepted_tokens[n] - 1 when
 * num_accepted_tokens [N] int32 is given (speculative decoding).  ht == h0
 * updates in place: with a per-token table (idx_stride_tok != 0) or under
 * speculative decoding the state after every token t goes to slot (n, t),
 * otherwise the final state goes back to the initial slot.  Any other ht is
 * [N, HV, K, V] (stride ht_stride) indexed by sequence (speculative
 * decoding still stores per token, into ht's slots).  A negative slot reads
 * as a zero state and is never written.  K, V in {64, 128}.  Replaces
 * npu_fused_recurrent_gated_delta_rule
 * (triton_npu/torch_api/npu_triton_recurrent_gated_delta_rule.cpp:54-246). */
XOPS_API int xops_fused_recurrent_gated_delta_rule(const void* q, const void* k, const void* v,
                                          const float* g, const float* beta, void* o,
                                          const float* h0, float* ht,
                                          const int32_t* cu_seqlens,
                                          const int32_t* ssm_state_indices,
                                          int64_t idx_stride_seq, int64_t idx_stride_tok,
                                          const int32_t* num_accepted_tokens, int64_t B,
                                          int64_t T, int64_t N, int64_t H, int64_t HV,
                                          int64_t K, int64_t V, int64_t h0_stride,
                                          int64_t ht_stride, float scale,
                                          int use_qk_l2norm_in_kernel, void* stream);

/* The recurrent step with the gates computed from the projections in the
 * step: g = -exp(A_log[h]) * softplus(a + dt_bias[h]) (torch Softplus with
 * softplus_beta / softplus_threshold), beta = sigmoid(b).  A_log, dt_bias
 * [HV] fp32; a, b [B, T, HV] of ab_dtype; q, k [B, T, H, K], v [B, T, HV, V]
 * bf16; o [B, T, HV, V] bf16.  cu_seqlens [N+1] int32 over the B*T
 * flattened tokens (required).  Sequence n starts from slot
 * initial_state_indices[n] of initial_state_source [slots, HV, K, V] fp32
 * and writes its final state back there; a negative index starts from zeros
 * and writes nothing.  K, V in {64, 128}.  Replaces
 * npu_fused_sigmoid_gating_delta_rule_update
 * (triton_npu/torch_api/npu_triton_fused_sigmoid_gating_delta_rule_update.cpp:54-179). */
XOPS_API int xops_fused_sigmoid_gating_delta_rule_update(
    const float* A_log, const void* a, const float* dt_bias, float softplus_beta,
    float softplus_threshold, const void* q, const void* k, const void* v, const void* b,
    void* o, float* initial_state_source, const int32_t* initial_state_indices,
    const int32_t* cu_seqlens, float scale, int64_t B, int64_t T, int64_t N, int64_t H,
    int64_t HV, int64_t K, int64_t V, int ab_dtype, int use_qk_l2norm_in_kernel, void* stream);

/* GDN gates from the projections: g = -exp(A_log[h]) * softplus(a +
 * dt_bias[h]) fp32, beta_out = sigmoid(b) in b's dtype; a, b, g, beta_out
 * [rows, heads] (rows = batch for decode, tokens for prefill), A_log and
 * dt_bias [heads] fp32.  Replaces npu_fused_gdn_gating
 * (triton_npu/torch_api/npu_triton_fused_gdn_gating.cpp:33-93). */
XOPS_API int xops_fused_gdn_gating(const float* A_log, const void* a, const void* b,
                                   const float* dt_bias, float* g, void* beta_out, int64_t rows,
                                   int64_t heads, int a_dtype, int b_dtype, float softplus_beta,
                                   float softplus_threshold, void* stream);

/* Chunked gated delta rule prefill on the tensor cores.  q, k [B, T, Hg, K],
 * v [B, T, H, V] bf16; g, beta [B, T, H] fp32; h0 [N, H, K, V] fp32 or NULL;
 * o [B, T, H, V] bf16; ht [N, H, K, V] fp32 or NULL.  cu_seqlens [N+1] int32
 * with B == 1, or NULL with N == B.  K == V == 128, chunk 64.  q/k/v rows may
 * be strided views (e.g. slices of a packed conv output): *_token_stride is
 * the element distance between consecutive tokens (0 = contiguous), heads
 * contiguous inside a token.  Two launches: a chunk-parallel preparation
 * kernel (WY factors into `workspace`) and the chunk-serial state kernel
 * (per-chunk states and v_new never leave the SM).  `workspace` must hold
 * xops_chunk_gated_delta_rule_workspace_size() bytes, 16-byte aligned.
 * Replaces npu_chunk_gated_delta_rule
 * (triton_npu/torch_api/npu_triton_chunk_gated_delta_rule.cpp:556-642). */
XOPS_API int xops_chunk_gated_delta_rule(const void* q, const void* k, const void* v, const float* g,
                                const float* beta, const float* h0, void* o, float* ht,
                                const int32_t* cu_seqlens, int64_t B, int64_t T, int64_t N,
                                int64_t Hg, int64_t H, int64_t K, int64_t V,
                                int64_t q_token_stride, int64_t k_token_stride,
                                int64_t v_token_stride, float scale,
                                int use_qk_l2norm_in_kernel, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* The same rule with fused_gdn_gating folded into its prologue: the gates
 * are computed where the kernels read them, from the layer's projections a,
 * b [B, T, H] (fp32, bf16 or fp16 each, a_dtype / b_dtype XOPS_F32 /
 * XOPS_BF16 / XOPS_F16; ab_token_stride elements between tokens, 0 =
 * contiguous) or, with ba_interleaved, from the un-split projection
 * mixed_ba [T, Hg * 2r] itself (a == b; per key head b (r heads) | a (r),
 * r = H / Hg, the layout fused_qkvzba_split_reshape_cat de-interleaves),
 * and A_log, dt_bias [H] fp32:
 *   g = -exp(A_log[h]) * softplus(a + dt_bias[h]),  beta = sigmoid(b) in b's dtype
 * with the arithmetic of xops_fused_gdn_gating, so the result equals
 * xops_fused_gdn_gating followed by xops_chunk_gated_delta_rule (beta widened
 * to fp32) bit for bit, without the g / beta round trip through HBM and
 * the extra launch.  The GDN layer's prefill calls fused_gdn_gating
 * (npu_triton_fused_gdn_gating.cpp:33-93) then npu_chunk_gated_delta_rule
 * (npu_triton_chunk_gated_delta_rule.cpp:556-642); this entry replaces the
 * pair.  Other arguments and the workspace as xops_chunk_gated_delta_rule. */
XOPS_API int xops_chunk_gated_delta_rule_gated(
    const void* q, const void* k, const void* v, const float* A_log, const void* a, const void* b,
    const float* dt_bias, int a_dtype, int b_dtype, int64_t ab_token_stride, int ba_interleaved,
    float softplus_beta, float softplus_threshold,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    void* workspace, int64_t workspace_bytes, void* stream);

/* The rule followed by the GDN layer's output norm, as one operator: each
 * (token, value head) row of V values of o (as the bf16 value
 * xops_chunk_gated_delta_rule would store) becomes
 *   y = ((o * rstd) * w) * silu(z),  rstd = 1 / sqrt(mean(o^2) + eps)
 * inside the chain kernel's output epilogue, so o makes no round trip
 * through HBM.  This is layer_norm_fwd with is_rms_norm, norm_before_gate,
 * no bias and group size V (npu_triton_layernorm_fwd.cpp:48-333), which the
 * layer runs on the rule's output.  z: bf16 rows of H * V per token,
 * z_token_stride elements apart (0 = H * V), 16-byte aligned; norm_weight
 * [V] of weight_dtype XOPS_F32 or XOPS_BF16; y [B, T, H, V] bf16.  o may be
 * NULL (only y is written) or a buffer that also receives o.  Other
 * arguments and the workspace as xops_chunk_gated_delta_rule.  This fusion
 * has no single counterpart in the reference; it replaces the pair
 * npu_chunk_gated_delta_rule -> layer_norm_fwd. */
XOPS_API int xops_chunk_gated_delta_rule_out_norm(
    const void* q, const void* k, const void* v, const float* g, const float* beta,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    const void* z, int64_t z_token_stride, const void* norm_weight, int weight_dtype, float eps,
    void* y, void* workspace, int64_t workspace_bytes, void* stream);

/* xops_chunk_gated_delta_rule_gated with the output norm of
 * xops_chunk_gated_delta_rule_out_norm: the GDN layer's prefill from its
 * projections (fused_gdn_gating -> npu_chunk_gated_delta_rule ->
 * layer_norm_fwd) with gates and norm inside the rule's kernels.  The z row
 * of value head h of token t is read at z + t * z_token_stride +
 * (h / z_heads_per_group) * z_group_stride + (h % z_heads_per_group) * V
 * (elements; all multiples of 8, z 16-byte aligned), so z can be read in
 * place from the layer's projection mixed_qkvz, whose key-head groups
 * interleave their z heads with q, k and v (z_heads_per_group = H / Hg,
 * z_group_stride = the group's width).  0 for z_heads_per_group,
 * z_group_stride or z_token_stride selects 1, V and H * V.  Other arguments
 * as the two entries it combines. */
XOPS_API int xops_chunk_gated_delta_rule_gated_out_norm(
    const void* q, const void* k, const void* v, const float* A_log, const void* a, const void* b,
    const float* dt_bias, int a_dtype, int b_dtype, int64_t ab_token_stride, int ba_interleaved,
    float softplus_beta, float softplus_threshold,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    const void* z, int64_t z_token_stride, int64_t z_heads_per_group, int64_t z_group_stride,
    const void* norm_weight, int weight_dtype, float eps, void* y, void* workspace,
    int64_t workspace_bytes, void* stream);

/* Workspace bytes xops_chunk_gated_delta_rule needs (an upper bound computed
 * from shapes only, no device access); varlen = cu_seqlens given. */
XOPS_API int64_t xops_chunk_gated_delta_rule_workspace_size(int64_t B, int64_t T, int64_t N,
                                                   int64_t Hg, int64_t H, int64_t K,
                                                   int use_qk_l2norm_in_kernel, int varlen);

/* xops_chunk_gated_delta_rule without a caller workspace, for callers that
 * cannot allocate device memory when they run.  This entry has no
 * counterpart in the reference.  Its scratch is one fixed 64 MiB array of
 * the library's own device memory, so problems whose
 * xops_chunk_gated_delta_rule_workspace_size() exceeds 64 MiB are rejected
 * with XOPS_ERR_WORKSPACE.  The array's address is looked up again on every
 * call made outside stream capture (so a reset or a new context on the
 * device is followed); a call made during capture reuses the last address
 * found on that device, so make the first call on each device before any
 * stream capture.  All calls on a device share the array, so calls that may
 * overlap on the GPU (e.g. unordered streams) race; keep them ordered.  The
 * 64 MiB is reserved on every device where the library's chunked-GDN module
 * is loaded, whether or not this entry is called.  Arguments are those of
 * xops_chunk_gated_delta_rule minus the workspace. */
XOPS_API int xops_chunk_gated_delta_rule_noalloc(const void* q, const void* k, const void* v,
                                        const float* g, const float* beta, const float* h0,
                                        void* o, float* ht, const int32_t* cu_seqlens, int64_t B,
                                        int64_t T, int64_t N, int64_t Hg, int64_t H, int64_t K,
                                        int64_t V, int64_t q_token_stride,
                                        int64_t k_token_stride, int64_t v_token_stride,
                                        float scale, int use_qk_l2norm_in_kernel, void* stream);

/* ---- chunk pipeline sub-operators (the reference's decomposition) ---- */
/* All take the same sequence description (cu_seqlens [N+1] int32 with B == 1
 * or NULL with N == B) and chunk_size == 64. */

/* g_cumsum [B, T, H] fp32 = per-chunk inclusive cumsum of g.  Replaces
 * npu_chunk_local_cumsum (npu_triton_chunk_gated_delta_rule.cpp:151-227). */
XOPS_API int xops_chunk_local_cumsum(const float* g, float* g_cumsum, const int32_t* cu_seqlens,
                            int64_t B, int64_t T, int64_t N, int64_t H, int64_t chunk_size,
                            void* stream);

/* A [B, T, H, 64] fp32 = strict_tril(beta_i exp(g_i - g_j) k_i.k_j) per chunk.
 * Replaces npu_chunk_scaled_dot_kkt_fwd (npu_triton_chunk_gated_delta_rule.cpp:229-297). */
XOPS_API int xops_chunk_scaled_dot_kkt_fwd(const void* k, const float* beta, const float* g_cumsum,
                                  float* A, const int32_t* cu_seqlens, int64_t B, int64_t T,
                                  int64_t N, int64_t Hg, int64_t H, int64_t K,
                                  int64_t chunk_size, void* stream);

/* Ai [B, T, H, 64] (out_dtype) = (I + A_c)^-1 per chunk.  Replaces
 * npu_solve_tril (npu_triton_chunk_gated_delta_rule.cpp:299-395). */
XOPS_API int xops_solve_tril(const float* A, void* Ai, const int32_t* cu_seqlens, int64_t B, int64_t T,
                    int64_t N, int64_t H, int64_t chunk_size, int out_dtype, void* stream);

/* w [B, T, H, K] = Ai (beta e^g k), u [B, T, H, V] = Ai (beta v), bf16;
 * Ai in ai_dtype.  Replaces npu_recompute_w_u_fwd
 * (npu_triton_chunk_gated_delta_rule.cpp:397-475). */
XOPS_API int xops_recompute_w_u_fwd(const void* k, const void* v, const float* beta,
                           const float* g_cumsum, const void* Ai, int ai_dtype, void* w, void* u,
                           const int32_t* cu_seqlens, int64_t B, int64_t T, int64_t N,
                           int64_t Hg, int64_t H, int64_t K, int64_t V, void* stream);

/* Chunk-state pass: h [B, NT, H, K, V] bf16 (state at every chunk start),
 * v_new [B, T, H, V] bf16 (may be NULL), ht [N, H, K, V] fp32 (may be NULL);
 * g_cumsum may be NULL (no gating); h0 fp32 or NULL.  NT = total chunks.
 * Replaces npu_chunk_gated_delta_rule_fwd_h
 * (npu_triton_chunk_gated_delta_rule.cpp:644-802). */
XOPS_API int xops_chunk_gated_delta_rule_fwd_h(const void* k, const void* w, const void* u,
                                      const float* g_cumsum, const float* h0, void* h,
                                      void* v_new, float* ht, const int32_t* cu_seqlens,
                                      int64_t B, int64_t T, int64_t N, int64_t Hg, int64_t H,
                                      int64_t K, int64_t V, int64_t NT, void* stream);

/* o [B, T, H, V] bf16 = scale (q h e^g + tril(q k^T e^{g_i-g_j}) v_new).
 * Replaces npu_chunk_fwd_o (npu_triton_chunk_gated_delta_rule.cpp:477-554). */
XOPS_API int xops_chunk_fwd_o(const void* q, const void* k, const void* v_new, const void* h,
                     const float* g_cumsum, void* o, const int32_t* cu_seqlens, int64_t B,
                     int64_t T, int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V,
                     int64_t NT, float scale, void* stream);

/* Number of device-side wait timeouts recorded by the tensor-core and the
 * bulk-copy streaming kernels (chunked GDN, conv1d, the norms, RoPE) since
 * the last call (0 when healthy); synchronises the device and resets the
 * counter.  A kernel that times out on an internal barrier writes no
 * further output and returns instead of hanging. */
XOPS_API int xops_device_error_count(void);

/* Total chunk count of a batch, computed on the host from a HOST copy of
 * cu_seqlens (or B*ceil(T/64) when cu_seqlens_host is NULL). */
XOPS_API int64_t xops_total_chunks(const int32_t* cu_seqlens_host, int64_t B, int64_t T, int64_t N,
                          int64_t chunk_size);

#ifdef __cplusplus
}
#endif

#endif /* XOPS_B200_H_ */
