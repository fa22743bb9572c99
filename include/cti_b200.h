/*
 * cti_b200.h - C ABI of the B200 (sm_100a) hot path of the generative
 * ad-ranking CTR model: the Top-2 sparse MoE layer and the 28-feature
 * embedding-bag pooling that feeds it.
 *
 * Conventions shared by every entry point:
 *   - All tensor arguments are raw device pointers to contiguous row-major
 *     buffers that the caller owns (for example torch tensors); sizes are
 *     element counts.  bf16/fp16 buffers are passed as `void*`.
 *   - `stream` is a cudaStream_t passed as `void*`; all work is enqueued on
 *     it, nothing synchronises the host, and no entry point allocates device
 *     memory.  Scratch needs are met by caller-provided workspaces whose sizes
 *     the *_workspace_bytes queries return.
 *   - The return value is CTI_OK or a CTI_ERR_* code describing a host-side
 *     argument or launch problem.  Problems that only the device can see (an
 *     index outside a buffer, a bounded wait that ran out) are written to the
 *     caller's device status word `status` (int32[2]: code, detail) and the
 *     offending element is skipped; read it with cti_status_read.
 *   - There is no fallback path: an unsupported shape is an error.
 */
#ifndef CTI_B200_H_
#define CTI_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return / status codes. */
#define CTI_OK 0
#define CTI_ERR_INVALID_ARG 1  /* null pointer, bad size, misaligned buffer */
#define CTI_ERR_UNSUPPORTED 2  /* shape outside what the kernels implement   */
#define CTI_ERR_CUDA 3         /* a CUDA runtime/driver call failed           */
#define CTI_ERR_TIMEOUT 4      /* device: a bounded wait ran out              */
#define CTI_ERR_BOUNDS 5       /* device: an index pointed outside a buffer   */

/* Expert activations (fc1 epilogue). */
#define CTI_ACT_NONE 0
#define CTI_ACT_RELU 1 /* reference model: baseline/infer.py:287            */
#define CTI_ACT_GELU 2 /* exact-erf GELU of the benchmark configurations    */

/* Output dtypes of the embedding-bag pooling. */
#define CTI_DTYPE_F32 0
#define CTI_DTYPE_BF16 1
#define CTI_DTYPE_F16 2

/* Tokens handled by one router block; the dispatch scratch holds one
 * E-wide histogram per block. */
#define CTI_ROUTER_BLOCK_TOKENS 128
#define CTI_MAX_EXPERTS 128

/* Library identity and device query. */
const char* cti_version(void);
int cti_num_sms(int device, int* num_sms);

/* Reads (and optionally clears) a device status word int32[2] on `stream`;
 * synchronises that stream. */
int cti_status_read(int32_t* status, int clear, int32_t* code, int32_t* detail, void* stream);

/* Self-test of the failure path (no counterpart in the reference): one
 * thread waits on a shared-memory mbarrier that nothing ever arrives at,
 * with the same bounded wait as every kernel of the library but a limit of
 * limit_ns nanoseconds (1e3 <= limit_ns <= 2e9).  When it runs out the
 * kernel writes CTI_ERR_TIMEOUT (detail 0x7f0) to `status` and returns
 * normally; the context stays usable.  Lets a test watch a wait run out
 * without hanging or faulting the GPU. */
int cti_selftest_wait_timeout(int32_t* status, int64_t limit_ns, void* stream);

/* ------------------------------------------------------------------------
 * Stage 1 - router.
 * Replaces TopKGate.forward (baseline/infer.py:298-309; online_best/infer.py:
 * 1800-1852) and the fused_top2_gate_kernel launch (online_best/infer.py:
 * 1624-1778, launched at :1818 and :2210).
 *
 * logits[t,e] = bg[e] + sum_d x[t,d]*wg[e,d] in fp32 (x is bf16, wg/bg fp32);
 * the sum is one fused-multiply-add chain in increasing d from 0, and the
 * bias is added after it.  Top-2 by logit
 * with ties to the lower expert id.  D % 8 == 0.  renorm=1: gates are the two softmax
 * probabilities renormalised to sum to 1; renorm=0: the raw softmax
 * probabilities (the reference's un-renormalised scores).
 * Outputs: idx2[T,2] int32, gate2[T,2] fp32, route_rank[T,2] int32 (rank of
 * each route among the same-expert routes of its 128-token block, token
 * order), block_hist[ceil(T/128), E] int32 (per-block expert counts; the
 * dispatch scratch).  E <= 128.
 * ---------------------------------------------------------------------- */
int cti_moe_router(const void* x_bf16, const float* wg, const float* bg, int64_t T, int D, int E,
                   int renorm, int32_t* idx2, float* gate2, int32_t* route_rank,
                   int32_t* block_hist, int32_t* status, void* stream);

/* Bytes of dispatch scratch (block_hist) for T tokens and E experts. */
size_t cti_moe_dispatch_workspace_bytes(int64_t T, int E);

/* ------------------------------------------------------------------------
 * Stage 2 - dispatch.
 * Replaces moe_route_count_kernel / moe_prefix8_kernel /
 * moe_route_pack(_chunked)_kernel and SMoE._pack_routes*
 * (online_best/infer.py:1205-1290, :1987-2062) and the per-expert
 * `mask.nonzero()` + `x_flat[token_idx]` gather of baseline/infer.py:336-346.
 *
 * Turns block_hist (from cti_moe_router, rewritten in place into per-block
 * base offsets) into expert offsets[E+1] (int32, exclusive prefix), then
 * places every route r=(t,k) at position pos = offsets[e] + (number of
 * earlier routes to e in token order): perm_inv[t,k] = pos,
 * sorted_token[pos] = t, xperm[pos,:] = x[t,:].  Deterministic.
 * xperm may be NULL (positions only): expert parallelism moves rows
 * itself, and cti_moe_expert_ffn_fused_gather reads them from x.
 * ---------------------------------------------------------------------- */
int cti_moe_dispatch(const void* x_bf16, const int32_t* idx2, const int32_t* route_rank,
                     int32_t* block_hist, int64_t T, int D, int E, int32_t* offsets,
                     int32_t* perm_inv, int32_t* sorted_token, void* xperm_bf16, int32_t* status,
                     void* stream);

/* ------------------------------------------------------------------------
 * Routing + dispatch for callers that cannot allocate device memory.
 * This entry point has no counterpart in the reference.
 *
 * Same results as cti_moe_router followed by cti_moe_dispatch (idx2, gate2,
 * offsets, perm_inv, sorted_token, xperm), but the scratch those two need
 * between them (route ranks and per-block expert counts) lives in a
 * 1.5 MiB array inside the library instead of a caller workspace - for a
 * host that binds only this C library and has no device allocator, or that
 * must stay inside a fixed pre-reserved memory budget.  Limits: T <=
 * CTI_NOALLOC_MAX_TOKENS, E <= CTI_NOALLOC_MAX_EXPERTS (larger sizes return
 * CTI_ERR_UNSUPPORTED).  All calls on a device share the array, so calls
 * that overlap on the GPU race; serialise them.  The first call on each
 * device resolves the array's address and should come before any stream
 * capture.  The address is cached per device together with the CUDA
 * context that was current; a call under another context (one the host
 * made with the driver API) resolves it again, so make the first call
 * under each such context outside any capture as well.
 * ---------------------------------------------------------------------- */
#define CTI_NOALLOC_MAX_TOKENS 131072
#define CTI_NOALLOC_MAX_EXPERTS 128
int cti_moe_route_dispatch_noalloc(const void* x_bf16, const float* wg, const float* bg,
                                   int64_t T, int D, int E, int renorm, int32_t* idx2,
                                   float* gate2, int32_t* offsets, int32_t* perm_inv,
                                   int32_t* sorted_token, void* xperm_bf16, int32_t* status,
                                   void* stream);

/* ------------------------------------------------------------------------
 * Stage 3 - grouped expert GEMM on tcgen05 tensor cores.
 * Replaces moe_sparse_fc1*_kernel and moe_sparse_fc2*_kernel
 * (online_best/infer.py:1293-1600) and Expert.forward (baseline/infer.py:
 * 286-287).
 *
 * For every group g (rows group_offsets[g] .. group_offsets[g+1]-1 of A):
 *   C[rows, :] = act(A[rows, :K] @ W[g % Gw]^T + bias[g % Gw])
 * A [rows_total, K] bf16, W [Gw, N, K] bf16 (the nn.Linear weight layout,
 * stacked), bias [Gw, N] fp32 (may be NULL), C [rows_total, N] bf16.
 * group_offsets is a device int32[G+1] array (non-decreasing, starting at 0);
 * rows_total bounds it.  N % 128 == 0, K % 64 == 0, G <= 1024.
 * ---------------------------------------------------------------------- */
int cti_moe_grouped_gemm(const void* A_bf16, const void* W_bf16, const float* bias,
                         const int32_t* group_offsets, int G, int Gw, int64_t rows_total, int N,
                         int K, int act, void* C_bf16, int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Stage 3 (fused) - expert FFN with the hidden activation kept on chip.
 * Y[rows,:] = (act(Xp[rows,:] @ W1[e]^T + b1[e])) @ W2[e]^T + b2[e]
 * for e = g % Gw; the [rows, F] hidden tile never leaves the SM.
 * Xp [rows_total, D], W1 [Gw, F, D], b1 [Gw, F] fp32, W2 [Gw, D, F],
 * b2 [Gw, D] fp32, Y [rows_total, D] bf16.  D in {128, 256}; F % 128 == 0.
 * Replaces the fc1 -> packed_hidden -> fc2 round trip of
 * SMoE._chunked_compute (online_best/infer.py:2109-2173).
 * ---------------------------------------------------------------------- */
int cti_moe_expert_ffn_fused(const void* Xp_bf16, const void* W1_bf16, const float* b1,
                             const void* W2_bf16, const float* b2, const int32_t* group_offsets,
                             int G, int Gw, int64_t rows_total, int D, int F, int act,
                             void* Y_bf16, int32_t* status, void* stream);

/* The same with the rows gathered in the kernel: row r of the expert-sorted
 * order is x[sorted_token[r], :] (x [T, D] bf16, sorted_token [rows_total]
 * from cti_moe_dispatch), so the dispatch need not write Xp (pass
 * xperm_bf16 = NULL there).  This replaces the fc1 kernel's row gather of
 * online_best/infer.py:1329-1333 as well.  Results equal
 * cti_moe_expert_ffn_fused on the dispatched rows, bit for bit.  One extra
 * warp copies the rows (16-byte cp.async); at the cfg2 shape the layer built
 * on it took 0.279 ms against 0.248 ms with the dispatched copy and TMA, so
 * cti_moe_layer_forward keeps the copy. */
int cti_moe_expert_ffn_fused_gather(const void* x_bf16, int64_t T, const int32_t* sorted_token,
                                    const void* W1_bf16, const float* b1, const void* W2_bf16,
                                    const float* b2, const int32_t* group_offsets, int G, int Gw,
                                    int64_t rows_total, int D, int F, int act, void* Y_bf16,
                                    int32_t* status, void* stream);

/* The same on CTA pairs (thread-block clusters of two SMs, one
 * tcgen05.mma.cta_group::2 stream per pair, 256-row tiles, every MMA
 * 256 x 256 x 16): each SM holds half of every weight K slab, so it streams
 * half the weight bytes per FLOP; d_ff goes in 256-wide chunks whose GELU'd
 * hidden activation passes through shared memory.  D == 256 and
 * F % 256 == 0 (CTI_ERR_UNSUPPORTED otherwise); otherwise the same
 * arguments, shapes and results. */
int cti_moe_expert_ffn_fused_pair(const void* Xp_bf16, const void* W1_bf16, const float* b1,
                                  const void* W2_bf16, const float* b2,
                                  const int32_t* group_offsets, int G, int Gw,
                                  int64_t rows_total, int D, int F, int act, void* Y_bf16,
                                  int32_t* status, void* stream);

/* 1 if the fused kernels take this shape (D in {128, 256}, F % 128 == 0,
 * F <= 1024, G <= 128 groups, rows_total < 2^31 - 256), else 0. */
int cti_moe_expert_ffn_fused_supported(int D, int F, int G, int64_t rows_total);

/* ------------------------------------------------------------------------
 * Stage 4 - gate-weighted combine.
 * Replaces moe_top2_reduce_kernel (online_best/infer.py:1603-1621), the
 * `* score` of the fc2 epilogue (:1465-1473) and the
 * `out_flat[token_idx] += expert_out * weight` of baseline/infer.py:350-353.
 * out[t,:] = bf16( gate2[t,0]*Y[perm_inv[t,0],:] + gate2[t,1]*Y[perm_inv[t,1],:] )
 * in fp32.  Y has Y_rows rows (bounds-checked).
 * ---------------------------------------------------------------------- */
int cti_moe_combine(const void* Y_bf16, int64_t Y_rows, const int32_t* perm_inv,
                    const float* gate2, int64_t T, int D, void* out_bf16, int32_t* status,
                    void* stream);

/* ------------------------------------------------------------------------
 * Whole layer: router -> dispatch -> expert FFN -> combine, one call.
 * The drop-in for SMoE.forward (online_best/infer.py:1910-1954; baseline/
 * infer.py:323-358) for a caller that binds only C.
 * wg/bg fp32 [E,D]/[E]; W1 [E,F,D], b1 [E,F] fp32, W2 [E,D,F], b2 [E,D]
 * fp32; x/out [T,D] bf16.  workspace: cti_moe_layer_workspace_bytes bytes.
 * ---------------------------------------------------------------------- */
size_t cti_moe_layer_workspace_bytes(int64_t T, int D, int E, int F);
int cti_moe_layer_forward(const void* x_bf16, const float* wg, const float* bg,
                          const void* W1_bf16, const float* b1, const void* W2_bf16,
                          const float* b2, int64_t T, int D, int E, int F, int act, int renorm,
                          void* out_bf16, void* workspace, size_t workspace_bytes,
                          int32_t* status, void* stream);

/* ------------------------------------------------------------------------
 * Whole layer between host buffers: the SMoE.forward drop-in
 * (online_best/infer.py:1910-1954) together with the caller's copy of the
 * activations to the device and of the output back (online_best/infer.py:
 * 2513 consumes the output on the host side of the plugin in a host-bound
 * caller).  Tokens are processed in chunks of chunk_tokens; chunk i's
 * host->device copy (copy_stream_in), layer (stream) and device->host copy
 * (copy_stream_out) overlap those of its neighbours.  Each token's output
 * depends only on its own row, so out_host equals cti_moe_layer_forward over
 * all T, bit for bit.
 *   x_host, out_host: [T,D] bf16 host memory (page-locked for the copies to
 *     run asynchronously); x_dev, out_dev: [T,D] bf16 device staging;
 *   workspace: W = cti_moe_layer_workspace_bytes(min(chunk_tokens, T), D, E,
 *     F) bytes; with compute_stream2, W rounded up to 256 bytes plus W.
 * compute_stream2 (may be NULL): odd chunks' layers run on it, on the second
 * half of the workspace, so that the layers of neighbouring chunks overlap.
 * The copies start after the work enqueued on `stream` before the call, and
 * `stream` waits for the last copy back (and for compute_stream2), so
 * synchronising `stream` makes out_host valid.  The copy streams may be
 * `stream` itself (no overlap).
 * ---------------------------------------------------------------------- */
int cti_moe_layer_forward_host(const void* x_host, void* out_host, void* x_dev, void* out_dev,
                               const float* wg, const float* bg, const void* W1_bf16,
                               const float* b1, const void* W2_bf16, const float* b2, int64_t T,
                               int D, int E, int F, int act, int renorm, int64_t chunk_tokens,
                               void* workspace, size_t workspace_bytes, int32_t* status,
                               void* stream, void* copy_stream_in, void* copy_stream_out,
                               void* compute_stream2);

/* ------------------------------------------------------------------------
 * Stage 5 - 28-feature embedding-bag sum pooling.
 * Replaces fused_all_slots_embedding_kernel and its launch
 * (online_best/infer.py:793-827, :1029-1059) and the per-slot
 * `emb(values.clamp(0, V-1))` + `segment_reduce(sum)` loop of
 * RepEncoder.forward (baseline/infer.py:253-263).
 *
 * Flat layout of the reference batch: values int64 [n_values]; row_offsets
 * int64 [F*(B+1)] (per-feature offsets, each feature's block starting at 0);
 * val_offsets int64 [F] (start of each feature's values).  Tables are rows
 * of one fp16 [total_rows, dim] buffer: feature f uses rows
 * table_row_base[f] .. table_row_base[f] + vocab[f] - 1 and clamps ids to
 * [0, vocab[f]-1].  out[b, f*dim + c] = sum over the bag in order, fp32
 * accumulation, stored as out_dtype.  dim in {32, 64, 128, 256, 512}.
 * ---------------------------------------------------------------------- */
int cti_embbag_sum(const int64_t* values, int64_t n_values, const int64_t* row_offsets,
                   const int64_t* val_offsets, const int64_t* table_row_base,
                   const int64_t* vocab, const void* table_f16, int64_t table_rows, int64_t B,
                   int F, int dim, void* out, int out_dtype, int32_t* status, void* stream);

/* ----------------------------------------------------------------------
 * The RepEncoder in one launch: embedding-bag pooling (as cti_embbag_sum,
 * dim 64, bf16-rounded sums), LayerNorm over the F*64 pooled columns and the
 * Linear to N = d_model, never writing the pooled rows
 * (baseline/infer.py:253-265 RepEncoder.forward; online_best/infer.py:793-827,
 * :829-858 and :1061-1085, the pooling, LayerNorm and Linear launches).  The
 * LayerNorm is folded into the weights by the caller:
 *   wg bf16 [N, F*64] = W * gamma;  r1 fp32 [N] = sum_k wg[n, k];
 *   c fp32 [N] = W beta + b;
 *   out[b, n] = rstd_b * (sum_k wg[n, k] x[b, k] - mean_b * r1[n]) + c[n]
 * with mean_b, rstd_b = 1/sqrt(var_b + eps) over the bf16 pooled row x[b].
 * Batch layout, clamping and bounds errors as cti_embbag_sum.  out bf16
 * [B, N] contiguous (16-byte aligned).  dim 64 and N in {128, 256} only
 * (CTI_ERR_UNSUPPORTED otherwise).
 * ---------------------------------------------------------------------- */
int cti_rep_encoder_fused(const int64_t* values, int64_t n_values, const int64_t* row_offsets,
                          const int64_t* val_offsets, const int64_t* table_row_base,
                          const int64_t* vocab, const void* table_f16, int64_t table_rows,
                          int64_t B, int F, int dim, const void* wg_bf16, const float* r1,
                          const float* c, int N, float eps, void* out_bf16, int32_t* status,
                          void* stream);

/* ----------------------------------------------------------------------
 * Causal attention inside packed variable-length sequences (the CTR model's
 * per-layer attention: baseline/infer.py:267-276 scaled_dot_product with the
 * sequence causal mask of :420-427; online_best/infer.py:1132-1202).
 *   out[t, h, :] = softmax over the keys j of t's sequence with j <= t of
 *                  q[t,h,:].k[j,h,:] / sqrt(head_dim), applied to v[j,h,:]
 * q, k, v: bf16 [tokens][heads][head_dim] views with token strides
 * (elements, multiples of 8, >= heads*head_dim; 16-byte aligned bases);
 * cu_seqlens int32 [num_seqs+1] non-decreasing token offsets, cu[0] >= 0;
 * out bf16 [tokens][heads][head_dim] contiguous, written for the tokens
 * [cu[0], min(cu[num_seqs], tokens)) only.  head_dim 32 only
 * (CTI_ERR_UNSUPPORTED otherwise).  Sequences of any length; max_seqlen is
 * the caller's bound (checked >= 0, not needed by the kernel).  `status`
 * (int32[2], may be NULL) receives CTI_ERR_TIMEOUT if a pipeline wait runs
 * out, CTI_ERR_INVALID_ARG if cu[0] < 0.
 * ---------------------------------------------------------------------- */
int cti_varlen_attention(const void* q_bf16, const void* k_bf16, const void* v_bf16,
                         int64_t q_stride, int64_t k_stride, int64_t v_stride,
                         const int32_t* cu_seqlens, int num_seqs, int max_seqlen, int64_t tokens,
                         int heads, int head_dim, void* out_bf16, int32_t* status, void* stream);

/* ----------------------------------------------------------------------
 * Residual add + LayerNorm of the CTR model around the MoE layer: the
 * pre-LN steps of TransformerEncoder.forward (baseline/infer.py:388-409,
 * `residual + y` then nn.LayerNorm) and the RepEncoder LayerNorm over the
 * pooled 28*64 columns (baseline/infer.py:264).
 *   s   = bf16(x + residual)   (residual may be NULL: s = x); written to
 *                              sum if sum is not NULL (needs residual)
 *   out = bf16((s - mean) * rsqrt(var + eps) * gamma + beta), fp32 mean and
 *         biased variance of the bf16 row s
 * bf16 [rows, cols] row-major, gamma / beta bf16 [cols]; cols a multiple of
 * 8, at most 2048 (CTI_ERR_UNSUPPORTED otherwise); every pointer 16-byte
 * aligned.
 * ---------------------------------------------------------------------- */
int cti_add_layernorm(const void* x_bf16, const void* residual_bf16, const void* gamma_bf16,
                      const void* beta_bf16, int64_t rows, int cols, float eps, void* sum_bf16,
                      void* out_bf16, void* stream);

/* ----------------------------------------------------------------------
 * The CTR head in one launch: the configuration's MLP head, then the clamp
 * and sigmoid of the reference head.  Replaces final_linear_clamp_kernel
 * (online_best/infer.py:861-887, launched at :2529-2567) and the separate
 * Linear / ReLU / Linear / clamp / sigmoid launches.
 *   logits[t] = clamp(w2 . relu(W1 h[t] + b1) + b2, -limit, limit)
 *   probs[t]  = 1 / (1 + exp(-logits[t]))
 * h [T, D] bf16, W1 [Hd, D] bf16, b1 [Hd], w2 [Hd], b2 [1] fp32; the hidden
 * activation stays in fp32 on chip.  logits / probs fp32 [T], either may be
 * NULL (not both).  D % 64 == 0, D <= 256, Hd % 32 == 0, Hd <= 128.
 * ---------------------------------------------------------------------- */
int cti_ctr_head(const void* h_bf16, const void* W1_bf16, const float* b1, const float* w2,
                 const float* b2, int64_t T, int D, int Hd, float limit, float* logits,
                 float* probs, int32_t* status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CTI_B200_H_ */
