/*
 * zs.h — C ABI of the B200 (sm_100a) kernels for the Zarelga-Superposition
 * MoE training step.
 *
 * Every entry point takes plain device pointers, element strides and sizes,
 * and a CUDA stream passed as `void*` (a cudaStream_t / CUstream; NULL is the
 * legacy default stream).  Nothing here allocates device memory: callers pass
 * outputs and, where a kernel needs scratch, a workspace whose size the
 * matching *_workspace() function returns.  Calls are asynchronous on the
 * given stream and never synchronise the host, so they can be captured in a
 * CUDA graph.
 *
 * Return value: ZS_OK (0) or one of the ZS_ERR_* codes below for a rejected
 * argument or a failed launch.  Faults detected on the device (a bounded wait
 * that ran out, an index out of range) never trap: they set bits in a
 * device-global error word read with zs_device_error_get().
 *
 * Current device: an entry point makes the device that owns its data current
 * on the calling thread (cudaSetDevice) before it launches, and leaves it
 * current when it returns.  A multi-GPU caller in one process that relies on
 * the current device afterwards (allocations without an explicit device) sets
 * it again itself.
 *
 * Each declaration names the reference function it replaces
 * (CoffeeVampir3/Architecture-Zarelga-Superposition, path:line).
 */
#ifndef ZS_H_
#define ZS_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */
#define ZS_OK 0
#define ZS_ERR_ARG 1         /* null pointer or invalid enum */
#define ZS_ERR_SHAPE 2       /* sizes inconsistent or out of the supported range */
#define ZS_ERR_DTYPE 3       /* unsupported dtype combination */
#define ZS_ERR_ALIGN 4       /* pointer or stride alignment required by TMA not met */
#define ZS_ERR_CUDA 5        /* a CUDA runtime/driver call failed */
#define ZS_ERR_WORKSPACE 6   /* workspace missing or too small */
#define ZS_ERR_LAYOUT 7      /* stride pattern not supported by the kernel */
#define ZS_ERR_SCRATCH_LIMIT 8 /* problem larger than the fixed scratch of an allocation-free entry point */

/* device error bits (zs_device_error_get) */
#define ZS_DEVERR_TIMEOUT_PRODUCER 0x01
#define ZS_DEVERR_TIMEOUT_MMA 0x02
#define ZS_DEVERR_TIMEOUT_EPILOGUE 0x04
#define ZS_DEVERR_TIMEOUT_DRAIN 0x08
#define ZS_DEVERR_INDEX 0x10       /* an index input was out of range; the element was skipped */
#define ZS_DEVERR_TIMEOUT_PEER 0x20 /* a wait for a peer GPU's flag expired (zs_ce_allreduce) */

/* dtype codes */
#define ZS_F32 0
#define ZS_BF16 1
#define ZS_F16 2

/* ------------------------------------------------------------------ misc */
int zs_version(void);
const char* zs_error_string(int code);
/* Synchronously read (stream-ordered) the device error word of the current device. */
int zs_device_error_get(int* out, void* stream);
/* Clear the device error word (stream-ordered). */
int zs_device_error_clear(void* stream);
/* The cudaError_t of the last failed CUDA runtime call behind a ZS_ERR_CUDA
 * return on this host thread (driver CUresult codes are reported + 100000). */
int zs_last_cuda_error(void);

/* ------------------------------------------------------------- routing (a1-a3) */

/*
 * MoEGate.forward after the router GEMM and sigmoid
 * (modeling/moe_gate.py:29-34):
 *   biased = gate_probs + expert_biases           (f32)
 *   topk_idx = topk(biased, top_k, sorted=False)  (CUDA torch.topk order:
 *              values above the k-th value in index order, then ties equal to
 *              the k-th value in index order)
 *   topk_weight = L1-normalise(gate_probs[topk_idx])  (F.normalize p=1, eps=1e-12)
 * gate_probs: [num_tokens, num_experts] row-major, dtype probs_dtype.
 * topk_idx: int64 [num_tokens, top_k]; topk_weight: probs_dtype [num_tokens, top_k].
 * Limits: num_experts <= 1024, top_k <= 32, top_k <= num_experts.
 */
int zs_moe_gate_topk(const void* gate_probs, int probs_dtype, const float* expert_biases, int64_t num_tokens,
                     int num_experts, int top_k, int64_t* topk_idx, void* topk_weight, void* stream);

/*
 * Backward of the differentiable part of MoEGate.forward
 * (modeling/moe_gate.py:33-34: gather of gate_probs at topk_idx, then
 * F.normalize(p=1, eps=1e-12)): grad_probs [T, E] (fully written, zeros off
 * the selected experts) from grad_weight [T, k].  f32 arithmetic; grad and
 * probs share one dtype.
 */
int zs_moe_gate_topk_backward(const void* gate_probs, int probs_dtype, const int64_t* topk_idx,
                              const void* grad_weight, int grad_dtype, int64_t num_tokens, int num_experts, int top_k,
                              void* grad_probs, void* stream);

/*
 * flatten_sort_count (scattermoe/parallel_experts.py:21-28): stable counting
 * sort of the flat expert ids.
 *   sorted_expert_idxs[i]    expert id of the i-th sorted slot
 *   sorted_scattered_idxs[i] flat index (token * k + j) of that slot; ties keep
 *                            ascending flat index
 *   expert_offsets[e]        inclusive cumulative count (int64)
 * expert_idxs values must lie in [0, num_experts); others raise ZS_DEVERR_INDEX
 * and are dropped.  Workspace: zs_flatten_sort_count_workspace(n, num_experts) bytes.
 */
size_t zs_flatten_sort_count_workspace(int64_t n, int num_experts);
int zs_flatten_sort_count(const int64_t* expert_idxs, int64_t n, int num_experts, int64_t* sorted_expert_idxs,
                          int64_t* sorted_scattered_idxs, int64_t* expert_offsets, void* workspace,
                          size_t workspace_bytes, void* stream);

/*
 * Allocation-free variant of zs_flatten_sort_count.  No counterpart in the
 * reference: it exists for callers that cannot allocate device memory where
 * they route tokens (runtimes that own a fixed device memory pool and forbid
 * cudaMalloc after start-up, C callers without an allocator).  Same inputs, outputs and results as zs_flatten_sort_count; the
 * scratch lives in a fixed 1 MiB device array inside the library (held on
 * every GPU that loads the library until the process exits), so the problem
 * must satisfy ceil(n / 4096) * (num_experts + 1) <= 262144 (the value of
 * zs_flatten_sort_count_noalloc_max_scratch_ints()); larger problems return
 * ZS_ERR_SCRATCH_LIMIT without launching anything.  It allocates nothing.
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress, with that device current); make that first call
 * before any stream capture.  All calls on a device share the array, so calls
 * whose kernels overlap on the GPU (different streams without ordering) race;
 * serialise them.
 */
int64_t zs_flatten_sort_count_noalloc_max_scratch_ints(void);
int zs_flatten_sort_count_noalloc(const int64_t* expert_idxs, int64_t n, int num_experts,
                                  int64_t* sorted_expert_idxs, int64_t* sorted_scattered_idxs,
                                  int64_t* expert_offsets, void* stream);

/* compileable_bincount (scattermoe/parallel_experts.py:6-15): int64 counts of
 * x[0..n) over [0, minlength). */
int zs_bincount(const int64_t* x, int64_t n, int minlength, int64_t* out, void* stream);

/*
 * auxillary_loss_free_update (main.py:161-175), split so that a data-parallel
 * caller can all-reduce the counts between the two halves.
 *   zs_expert_counts: counts[e] += #{(t, j) : valid[t] && topk_idx[t, j] == e}
 *     (valid may be NULL = all tokens valid; counts is accumulated, not cleared)
 *   zs_bias_sign_update: bias[e] += update_rate * sign(mean(counts) - counts[e]),
 *     skipped entirely when sum(counts) == 0 (the reference's `numel() == 0`).
 */
int zs_expert_counts(const int64_t* topk_idx, const uint8_t* valid, int64_t num_tokens, int top_k,
                     int num_experts, int64_t* counts, void* stream);
int zs_bias_sign_update(const int64_t* counts, int num_experts, float update_rate, float* expert_biases,
                        void* stream);

/* ------------------------------------------------ grouped expert GEMMs (a5-a9) */

/*
 * scatter2scatter (scattermoe/kernels/ops.py:192-255, kernel :128-190):
 *   for each sorted slot i with expert e = sorted_expert_idxs[i]:
 *     in_row  = x_grouped ? i : sorted_scattered_idxs[i] / fan_out
 *     out_row = y_grouped ? i : sorted_scattered_idxs[i]
 *     out[out_row, :] = X[in_row, :] @ W[e] (+ b[e])
 * W is addressed as W[e, k, n] = W + e*w_se + k*w_sk + n*w_sn and must have
 * either w_sk == 1 (K contiguous, e.g. the reference's weight.permute(0,2,1))
 * or w_sn == 1 (N contiguous); w_se must equal the packed expert size.
 * X: [x_rows, K] with row stride x_sm; out: [n, N] with row stride out_sm.
 * dtype: ZS_BF16 or ZS_F16 for X, W and out; bias same dtype or NULL.
 * expert_offsets (inclusive cumsum) may be NULL, in which case expert
 * boundaries are found from sorted_expert_idxs.
 * Workspace: zs_scatter2scatter_workspace(n, K, dtype, x_grouped) bytes
 * (the gathered input rows when x_grouped == 0).
 */
size_t zs_scatter2scatter_workspace(int64_t n, int64_t K, int dtype, int x_grouped);
int zs_scatter2scatter(void* out, int64_t out_sm, const void* W, int64_t num_experts, int64_t K, int64_t N,
                       int64_t w_se, int64_t w_sk, int64_t w_sn, const void* X, int64_t x_rows, int64_t x_sm,
                       const void* bias, int64_t b_se, int64_t b_sn, int fan_out, const int64_t* sorted_expert_idxs,
                       const int64_t* sorted_scattered_idxs, const int64_t* expert_offsets, int64_t n, int x_grouped,
                       int y_grouped, int dtype, void* workspace, size_t workspace_bytes, void* stream);

/*
 * groupXtY (scattermoe/kernels/ops.py:263-311, kernel :320-438):
 *   for each expert e with sorted rows [start_e, end_e) (from expert_offsets,
 *   inclusive cumsum):  DW[e] = X[start_e:end_e]^T @ DY[start_e:end_e]
 *   and, when Db != NULL, Db[e] = column sums of DY[start_e:end_e].
 * DW[e, k, n] = DW + e*dw_se + k*dw_sk + n*dw_sn, with dw_sk == 1 or dw_sn == 1.
 * Experts with no rows get zeros.  X: [n, K], DY: [n, N], grouped (sorted) rows.
 */
int zs_group_xty(int num_experts, void* DW, int64_t dw_se, int64_t dw_sk, int64_t dw_sn, void* Db, int64_t db_se,
                 int64_t db_sn, const void* DY, int64_t dy_sm, const void* X, int64_t x_sm, int64_t n, int64_t K,
                 int64_t N, const int64_t* expert_offsets, int dtype, void* stream);

/*
 * Upper bound on the CTAs of the persistent tensor-core GEMMs (0: one per SM,
 * the default).  A data-parallel step lowers it so the all-reduce kernels of
 * gradients already computed find free SMs and overlap the GEMMs that follow.
 * Process-wide; applies to launches made after the call.
 */
int zs_set_gemm_cta_limit(int max_ctas);

/*
 * groupXtY with an f32 result written straight into a weight-gradient buffer:
 * DW[e] = X_e^T DY_e (accumulate == 0) or DW[e] += X_e^T DY_e (accumulate != 0),
 * DW f32 with the same addressing as zs_group_xty; X and DY in dtype.  This is
 * the autograd step "dW (bf16) -> .to(f32) -> param.grad += dW" of the
 * reference's ParallelLinear backward under autocast (parallel_experts.py:
 * 106-120) in one pass, used when the caller accumulates into param.grad itself.
 */
int zs_group_xty_f32(int num_experts, float* DW, int64_t dw_se, int64_t dw_sk, int64_t dw_sn, const void* DY,
                     int64_t dy_sm, const void* X, int64_t x_sm, int64_t n, int64_t K, int64_t N,
                     const int64_t* expert_offsets, int dtype, int accumulate, void* stream);

/*
 * group (scattermoe/kernels/ops.py:449-482, kernel :490-529):
 *   Y[i, :] = A[sorted_scattered_idxs[i] / fan_out, :] (* coeff[sorted_scattered_idxs[i]])
 * A: [n / fan_out, K] row stride a_sm; Y: [n, K] row stride y_sm; coeff may be NULL.
 */
int zs_group(const void* A, int64_t a_sm, int64_t K, void* Y, int64_t y_sm, int64_t n, const void* coeff,
             int coeff_dtype, int fan_out, const int64_t* sorted_scattered_idxs, int dtype, void* stream);

/*
 * rowwise_sum_product (scattermoe/kernels/ops.py:9-46, kernel :50-80):
 *   out[t, f] = sum_h A[t, f, h] * B[t, h]   (f32 accumulation)
 * Strides in elements.
 */
int zs_rowwise_sum_product(void* out, int out_dtype, int64_t o_s0, int64_t o_s1, const void* A, int a_dtype,
                           int64_t a_s0, int64_t a_s1, int64_t a_s2, const void* B, int b_dtype, int64_t b_s0,
                           int64_t b_s1, int64_t T, int64_t F, int64_t H, void* stream);

/*
 * k-way row combine that closes the expert layer:
 *   out[t, c] = sum_j w[t, j] * in[t*k + j, c]
 * With weights it is the gate-weighted sum `gates.unsqueeze(1) @ output_expanded`
 * (scattermoe/parallel_experts.py:50-52); with weights == NULL it is the
 * `.view(T, k, d).sum(-2)` of the input gradient (parallel_experts.py:122-125).
 * f32 accumulation; in/out dtype ZS_BF16 or ZS_F16, weights any dtype code.
 */
int zs_weighted_row_sum(void* out, int64_t o_sm, const void* in, int64_t i_sm, const void* weights, int w_dtype,
                        int64_t T, int k, int64_t C, int dtype, void* stream);

/*
 * The MoE layer's close added into the f32 residual stream (the transformer
 * block's `h + (shared_experts(x) + routed_experts(x))`,
 * modeling/transformer_block.py:39-45 with modeling/moe_layer.py:44-58):
 *   out[t, c] = residual[t, c] + (shared[t, c] + round(sum_j w[t, j] * rows[t*k + j, c]))
 * in f32, the routed sum rounded to the rows' dtype (bf16 / f16) first as the
 * unfused path stores it.  shared (rows' dtype) and residual (f32) may be NULL.
 * k <= 8; C % 8 == 0; 16-byte aligned rows.
 */
int zs_moe_combine(float* out, int64_t o_sm, const void* rows, int64_t i_sm, const void* weights, int w_dtype,
                   int64_t T, int k, int64_t C, int dtype, const void* shared, int64_t s_sm, const float* residual,
                   int64_t r_sm, void* stream);

/*
 * The same k-way sum with the slot rows stored in another order (no
 * counterpart in the reference; the combine of the expert-parallel layer,
 * whose output rows return in expert order):
 *   out[t, c] = sum_j in[row_of_slot[t*k + j], c]
 * row_of_slot int64 [T*k]; a row outside [0, n_rows) contributes zero and
 * records ZS_DEVERR_INDEX.
 */
int zs_gathered_row_sum(void* out, int64_t o_sm, const void* in, int64_t i_sm, int64_t n_rows,
                        const int64_t* row_of_slot, int64_t T, int k, int64_t C, int dtype, void* stream);

/*
 * GLUMLP up projection with the SwiGLU activation fused into the GEMM
 * epilogue (scattermoe/mlp.py:80-87: experts(...) then chunk(2) into
 * h = first half, gates = second half, then silu(gates) * h):
 *   hfull[i, :] = Xg[i, :] @ W1[e_i]^T          ([n, 2F]; written when hfull != NULL)
 *   act[i, c]   = silu(hfull[i, F + c]) * hfull[i, c]   ([n, F])
 * W1: the experts.weight tensor [E, 2F, K], contiguous.  Xg: grouped rows
 * [n, K] with row stride xg_sm.  act/hfull contiguous.  Intermediates are
 * rounded to the storage dtype exactly where the reference stores them.
 */
int zs_expert_up_swiglu(void* act, void* hfull, const void* W1, int64_t num_experts, int64_t K, int64_t F,
                        const void* Xg, int64_t xg_sm, const int64_t* sorted_expert_idxs, const int64_t* expert_offsets,
                        int64_t n, int dtype, void* stream);

/*
 * Backward of act = silu(g) * h (autograd of scattermoe/mlp.py:87):
 *   dhfull[:, :F] = dact * silu(g);  dhfull[:, F:] = (dact * h) * silu'(g)
 * with hfull = [h | g] rows [n, 2F]; all contiguous, one dtype.
 */
int zs_swiglu_backward(void* dhfull, const void* dact, const void* hfull, int64_t n, int64_t F, int dtype,
                       void* stream);

/*
 * GLUMLP down-projection input gradient with the SwiGLU backward fused into
 * the GEMM epilogue (ParallelLinear.backward's grouped scatter2scatter with
 * the transposed weight, scattermoe/parallel_experts.py:112-120, followed by
 * the autograd of scattermoe/mlp.py:87):
 *   dact[i, :]  = dyg[i, :] @ W2[e_i]                 (never stored)
 *   dhfull[i,:] = zs_swiglu_backward(dact, hfull) rows
 * W2: output_experts.weight [E, K, F] contiguous (K = d_model); dyg: grouped
 * gate-scaled output gradient [n, K], row stride dyg_sm; hfull/dhfull [n, 2F].
 */
int zs_expert_down_dswiglu(void* dhfull, const void* hfull, const void* W2, int64_t num_experts, int64_t K, int64_t F,
                           const void* dyg, int64_t dyg_sm, const int64_t* sorted_expert_idxs,
                           const int64_t* expert_offsets, int64_t n, int dtype, void* stream);

/* ------------------------------------------------ norm and RoPE (a12, a14) */

/*
 * ZeroCenteredRMSNorm.forward (modeling/zRMSNorm.py:13-17), rows of length d:
 *   y = x * rsqrt(mean(x^2) + eps) * (1 + w)   in f32, stored in x's dtype.
 * rstd (f32 [rows], nullable) keeps rsqrt(...) for the backward.
 * Dtypes: x/y ZS_BF16 | ZS_F16 | ZS_F32; weight ZS_F32 (or ZS_BF16 with bf16 x).
 */
int zs_zrmsnorm_forward(const void* x, const void* weight, void* y, float* rstd, int64_t rows, int d, float eps,
                        int x_dtype, int w_dtype, void* stream);
/*
 * Backward of zs_zrmsnorm_forward (autograd of modeling/zRMSNorm.py:13-17):
 *   dx = r * (dn - n * mean(dn * n)),  n = x * r,  dn = dy * (1 + w)   (x's dtype)
 *   dweight = sum over rows of dy * n                                   (f32 [d])
 * d <= 12288; workspace: zs_zrmsnorm_backward_workspace(rows, d) bytes.
 */
size_t zs_zrmsnorm_backward_workspace(int64_t rows, int d);
/*
 * The transformer block's residual add fused with the next zRMSNorm (no
 * counterpart as one function in the reference; it computes
 * modeling/transformer_block.py:19-46's `h = x + branch` and the norm of
 * modeling/zRMSNorm.py:13-17 with the output cast that the following autocast
 * GEMM applies).  x f32 [rows, d], r bf16 [rows, d] or NULL, d = 128 * {1, 2, 4,
 * 8, 12, 16}, 16-byte aligned:
 *   forward:  h = x + r (f32, written to h_out when both are given), y = bf16 of
 *             zRMSNorm(h) (or of x without r), rstd as zs_zrmsnorm_forward;
 *   backward: dy bf16 (gradient of y), h the saved norm input, dh_in f32 or NULL
 *             (gradient reaching h from the residual path); dx = dh_in + the
 *             norm's input gradient (f32), dr = bf16 of dx (or NULL), dweight
 *             f32 [d]; workspace zs_zrmsnorm_backward_workspace(rows, d) bytes.
 */
int zs_add_zrmsnorm_forward(const float* x, const void* r, const float* weight, float* h_out, void* y, float* rstd,
                            int64_t rows, int d, float eps, void* stream);
int zs_add_zrmsnorm_backward(const void* dy, const float* h, const float* weight, const float* rstd,
                             const float* dh_in, float* dx, void* dr, float* dweight, int64_t rows, int d,
                             void* workspace, size_t workspace_bytes, void* stream);
int zs_zrmsnorm_backward(const void* dy, const void* x, const void* weight, const float* rstd, void* dx,
                         float* dweight, int64_t rows, int d, int x_dtype, int w_dtype, void* workspace,
                         size_t workspace_bytes, void* stream);

/*
 * LigerRopeFunction forward / backward (modeling/liger_rope.py:20-119, 183-206),
 * in place on q [batch, seq, n_q_heads, head_dim] and k [batch, seq,
 * n_kv_heads, head_dim] (row strides q_row_stride / k_row_stride per
 * (batch, position) row; heads contiguous).  Pair (i, i + head_dim/2) of each
 * head is rotated by the angle whose cos/sin are the tables' row entry i;
 * tables [cos_batch (1 or batch), seq, head_dim/2] with row stride
 * cos_row_stride.  backward != 0 rotates by the negative angle (the
 * gradient).  Arithmetic in f32.
 */
int zs_rope(void* q, int64_t q_row_stride, void* k, int64_t k_row_stride, const void* q_cos, const void* q_sin,
            const void* k_cos, const void* k_sin, int64_t cos_row_stride, int batch, int seq_len, int cos_batch,
            int n_q_heads, int n_kv_heads, int head_dim, int dtype, int table_dtype, int backward, void* stream);
/* zs_rope restricted to the first rot_pairs pairs of every head (0 <= rot_pairs
 * <= head_dim/2; the tables hold rot_pairs entries per row, cos_row_stride
 * apart): the partial RoPE of GatedAttention, whose remaining pairs have cos 1
 * and sin 0 (modeling/attention.py:85-104), so they are left untouched. */
int zs_rope_partial(void* q, int64_t q_row_stride, void* k, int64_t k_row_stride, const void* q_cos,
                    const void* q_sin, const void* k_cos, const void* k_sin, int64_t cos_row_stride, int batch,
                    int seq_len, int cos_batch, int n_q_heads, int n_kv_heads, int head_dim, int rot_pairs, int dtype,
                    int table_dtype, int backward, void* stream);

/*
 * GatedAttention's QK normalisation and partial position RoPE fused
 * (modeling/attention.py:140-150: q_norm / k_norm = zero-centred RMSNorm per
 * head, modeling/zRMSNorm.py:4-20, then the rotate-half RoPE of the first
 * rot pairs, modeling/liger_rope.py).  x: bf16 rows of ldx elements (one row
 * per token, tokens = batch * seq_len) whose leading (Hq + Hk) * hd columns
 * are the Hq query heads then the Hk key heads (the fused q/k/v/gate
 * projection's output); wq / wk: f32 [hd] norm weights (the gain is 1 + w).
 * forward: y (bf16, rows of ldy, same column order) = rope(x * rsqrt(mean(x^2)
 *   + eps) * (1 + w)) per head in f32, rounded once; rstd f32 [tokens *
 *   (Hq + Hk)].  Tables as zs_rope_partial: [cos_bs (1 or batch), seq_len,
 *   rot] with row stride cos_row_stride, f32 or bf16 (table_dtype).
 * backward: dx (bf16, rows of lddx; may be the q/k columns of the projection's
 *   gradient) from dy (rows of lddy); dwq / dwk (f32 [hd]) overwritten with the
 *   weight gradients, reduced in a fixed order (workspace:
 *   zs_qk_norm_rope_backward_workspace(hd) bytes).
 * hd 64 or 128; row strides multiples of 4 elements, rows 8-byte aligned.
 */
int zs_qk_norm_rope_forward(const void* x, int64_t ldx, const float* wq, const float* wk, const void* cos,
                            const void* sin, int table_dtype, int64_t cos_row_stride, int cos_bs, int rot, void* y,
                            int64_t ldy, float* rstd, int64_t tokens, int seq_len, int Hq, int Hk, int hd, float eps,
                            void* stream);
size_t zs_qk_norm_rope_backward_workspace(int hd);
int zs_qk_norm_rope_backward(const void* dy, int64_t lddy, const void* x, int64_t ldx, const float* wq,
                             const float* wk, const void* cos, const void* sin, int table_dtype,
                             int64_t cos_row_stride, int cos_bs, int rot, const float* rstd, void* dx, int64_t lddx,
                             float* dwq, float* dwk, int64_t tokens, int seq_len, int Hq, int Hk, int hd,
                             void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------ attention core (a13, a15) */

/*
 * Causal grouped-query attention as GatedAttention calls flash_attn_varlen_func
 * (modeling/attention.py:131-169, window_size = (W-1, 0) at :31), with the
 * optional per-head sink key of modeling/hca.py:138-144,264-298 (an extra
 * always-visible key k_sink[h] whose value is zero):
 *   o[b, q, h]  = sum_{k visible} softmax_k(scale * q.k) v[b, k, h / (H/Hkv)]
 *   lse[b, h, q] = natural log of the softmax denominator (sink included)
 * Key k is visible to query q when k <= q, q - k < window (window <= 0: no
 * window) and, with seg_start, seg_start[q] >= 0 and k >= seg_start[q]
 * (packed sequences: seg_start[b*S + i] is the first position of token i's
 * sequence in batch row b, -1 marks padding).
 * q [B*S, H*hd], k/v [B*S, Hkv*hd], o [B*S, H*hd]: bf16, rows contiguous;
 * lse f32 [B, H, S]; hd 64 or 128; k_sink [H, hd] f32 or bf16 (sink_dtype) or NULL.
 */
int zs_attention_forward(const void* q, const void* k, const void* v, void* o, float* lse, int B, int S, int H,
                         int Hkv, int hd, int window, const int* seg_start, const void* k_sink, int sink_dtype,
                         float softmax_scale, void* stream);

/*
 * Backward of zs_attention_forward (flash_attn's backward as autograd runs it
 * for attention.py:131-169).  Inputs: q, k, v, o, dout (bf16, layouts as in
 * the forward), lse from the forward.  Outputs: dq, dk, dv (bf16, same
 * layouts; dk/dv sum over the heads of a GQA group), D (f32 [B, H, S]
 * scratch: rowsum(dout * o)), and with k_sink: ds_sink (f32 [B, H, S]) =
 * d loss / d (sink logit) per query row; the sink's own gradient is
 * scale * sum_{b,q} ds_sink[b, h, q] * q[b, q, h, :].  dq already holds the
 * sink key's share.
 */
int zs_attention_backward(const void* q, const void* k, const void* v, const void* o, const void* dout,
                          const float* lse, void* dq, void* dk, void* dv, float* D, int B, int S, int H, int Hkv,
                          int hd, int window, const int* seg_start, const void* k_sink, int sink_dtype,
                          float* ds_sink, float softmax_scale, void* stream);

/*
 * zs_attention_forward / _backward with row strides and GatedAttention's
 * per-head output gate fused (modeling/attention.py:151-154: o * sigmoid(
 * head_gate_proj(x)) per head).  Every bf16 operand is rows of ld* elements
 * (multiples of 8, 16-byte aligned), so q, k, v and the gate logits can be
 * column ranges of one fused projection output.
 * forward: with gate_logits (bf16 [B*S, H] rows of ldg, or NULL for no gate)
 *   o = sigmoid(gate) * attention (sigmoid in f32, one rounding to bf16).
 * backward: dout is the gradient of the (gated) o; with a gate the kernel
 *   writes dgate_logits (bf16 [B*S, H] rows of lddg, followed by gate_pad < 32
 *   zeroed columns) and needs zs_gated_attention_backward_workspace(B, S, H,
 *   hd, 1) bytes of workspace (the ungated dO of the attention core).
 *   D = rowsum(dout * o) as before.
 */
int zs_gated_attention_forward(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                               void* o, int64_t ldo, float* lse, const void* gate_logits, int64_t ldg, int B, int S,
                               int H, int Hkv, int hd, int window, const int* seg_start, const void* k_sink,
                               int sink_dtype, float softmax_scale, void* stream);
size_t zs_gated_attention_backward_workspace(int B, int S, int H, int hd, int gated);
int zs_gated_attention_backward(const void* q, int64_t ldq, const void* k, int64_t ldk, const void* v, int64_t ldv,
                                const void* o, int64_t ldo, const void* dout, int64_t lddo, const float* lse,
                                const void* gate_logits, int64_t ldg, void* dq, int64_t lddq, void* dk, int64_t lddk,
                                void* dv, int64_t lddv, void* dgate_logits, int64_t lddg, int gate_pad, float* D,
                                int B, int S, int H, int Hkv, int hd, int window, const int* seg_start,
                                const void* k_sink, int sink_dtype, float* ds_sink, float softmax_scale,
                                void* workspace, size_t workspace_bytes, void* stream);

/*
 * Gradient of the sink key (modeling/hca.py:138-144: the sink logit of query
 * row (b, s, h) is scale * q[b, s, h, :] . k_sink[h]):
 *   dk_sink[h, :] = scale * sum_{b, s} ds_sink[b, h, s] * q[b, s, h, :]
 * with ds_sink from zs_attention_backward / zs_gated_attention_backward and q
 * the (normalised, rotated) bf16 queries, rows of ldq elements with head h at
 * column h * hd.  dk_sink f32 [H, hd].  Fixed-order sums (bit-identical runs);
 * workspace: zs_attention_sink_grad_workspace(B, S, H, hd) bytes.
 */
size_t zs_attention_sink_grad_workspace(int B, int S, int H, int hd);
int zs_attention_sink_grad(const float* ds_sink, const void* q, int64_t ldq, int B, int S, int H, int hd,
                           float softmax_scale, float* dk_sink, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------ cross entropy (a16-a18) */

/*
 * Multi-target cut cross entropy, raw-token mean (modeling/mcce_fast.py:21-31,
 * mcce_fast_v2.py:329-408) and, with s_max = 1 and s = 0 on ignored rows, the
 * standard next-token CE of linear_cross_entropy(e, c, targets,
 * ignore_index) as main.py:761 calls it:
 *   lse_t  = logsumexp_v(hidden[t] . classifier[v])
 *   loss   = (sum_t s_t * lse_t - sum_t sum_{j<s_t} z[t, labels[t, j]]) / sum_t s_t
 * The logits are never stored: one tensor-core GEMM pass keeps per-tile
 * (max, sum exp) partials and the target logits (workspace:
 * zs_xent_forward_workspace(T, V) bytes).  hidden [T, D], classifier [V, D]
 * (row strides h_sm / c_sm), labels int64 [T, s_max] (s_max <= 8; only the
 * first s_t of a row are read), s_count int32 [T].  Outputs (f32, device):
 * lse [T], row_loss [T], loss [1], denom [1] = sum_t s_t.
 */
size_t zs_xent_forward_workspace(int64_t T, int64_t V);
int zs_xent_forward(const void* hidden, int64_t T, int64_t D, int64_t h_sm, const void* classifier, int64_t V,
                    int64_t c_sm, const int64_t* labels, int s_max, const int* s_count, float* lse, float* row_loss,
                    float* loss, float* denom, void* workspace, size_t workspace_bytes, int dtype, void* stream);

/*
 * Backward of zs_xent_forward: dz[t, v] = (grad_loss / denom) * (s_t * softmax_t[v] - count_t(v))
 * recomputed per vocabulary slice of v_chunk columns (a multiple of 256); the
 * slice's dz lives only in the workspace (zs_xent_backward_workspace bytes):
 *   d_hidden     (f32 [T, D])  = dz @ classifier   (either output may be NULL)
 *   d_classifier (f32 [V, D])  = dz^T @ hidden
 * grad_loss and denom are device scalars (f32).
 */
size_t zs_xent_backward_workspace(int64_t T, int64_t v_chunk, int dtype);
int zs_xent_backward(const void* hidden, int64_t T, int64_t D, int64_t h_sm, const void* classifier, int64_t V,
                     int64_t c_sm, const int64_t* labels, int s_max, const int* s_count, const float* lse,
                     const float* grad_loss, const float* denom, float* d_hidden, float* d_classifier, int64_t v_chunk,
                     void* workspace, size_t workspace_bytes, int dtype, void* stream);

/* ------------------------------------------------ Muon (a22) */

/*
 * zeropower_via_newtonschulz5 (optimizer/muon.py:6-32) on a batch of
 * matrices already oriented with m <= n (the caller transposes taller ones):
 *   X = G / (||G||_F + 1e-7);  repeat `steps` times:
 *     A = X X^T;  B = b*A + c*A A;  X = a*X + B X
 * G, X_out: [batch, m, n] contiguous, bf16 or f16 (m and n multiples of 8).
 * Each product is a batched tcgen05 GEMM; the linear combinations are fused
 * into the GEMM epilogues.  Workspace: zs_newton_schulz5_workspace bytes.
 */
size_t zs_newton_schulz5_workspace(int64_t batch, int64_t m, int64_t n, int dtype);
int zs_newton_schulz5(const void* G, void* X_out, int64_t batch, int64_t m, int64_t n, int steps, float a, float b,
                      float c, void* workspace, size_t workspace_bytes, int dtype, void* stream);

/* ------------------------------------------------ MuonMD step (a23, a24) */

/*
 * md_decoupled_step (optimizer/muon.py:398-508) around the Newton-Schulz call,
 * for one weight stack W [L, m, n] (f32, contiguous) with gradient G and
 * momentum buffer buf (f32, same layout) and raw gains g_scalar [L], g_row
 * [L, m], g_col [L, n] (f32, each NULL when the gain mode lacks it; the
 * effective gain is softplus(scalar) * softplus(row) * softplus(col)).
 *
 * zs_muonmd_pre:  buf = lerp(buf, g*G, 1 - momentum);
 *                 x_out (bf16 [L, m, n], or [L, n, m] when x_transposed: the
 *                 layout Newton-Schulz runs a tall stack in) = lerp(g*G, buf,
 *                 momentum);
 *                 red_* = the gain-gradient reductions of (W/g)*G times the
 *                 other gains over the axes each gain does not span (red_*
 *                 f32, same shapes as the gains, overwritten; NULL exactly
 *                 where the gain is NULL).  The reductions add per-block
 *                 partial sums in a fixed order (no atomics): results are
 *                 bit-identical from run to run.  Workspace (only when a
 *                 gain is present): zs_muonmd_pre_workspace bytes.
 * zs_muonmd_post: with U the orthogonalised update (bf16 [L, m, n], or
 *                 [L, n, m] when u_transposed):
 *                 W' = W/g - lr * rescale * U, projected to target_norm
 *                 per matrix (norm_axis 0, target [L]), row (1, [L, m]) or
 *                 column (2, [L, n]); gain Adam (betas b1, b2, eps, step from
 *                 step_dev (f32 device scalar, already incremented) or
 *                 step_host) on dL/draw = red * sigmoid(raw), raw -= gain_lr
 *                 * update; p_out (f32 or bf16 by p_dtype, may alias W) =
 *                 g_new * W', and with shadow_bf16 (f32 p_out only) the same
 *                 values in bf16 in p_out's layout (the weight copy the next
 *                 forward's GEMMs read).  lr from lr_dev (f32 device scalar)
 *                 or lr_host.
 *                 Workspace: zs_muonmd_post_workspace bytes.
 */
size_t zs_muonmd_pre_workspace(int64_t L, int64_t m, int64_t n);
int zs_muonmd_pre(const float* W, const float* G, float* buf, const float* g_scalar, const float* g_row,
                  const float* g_col, void* x_out, int x_transposed, float* red_scalar, float* red_row,
                  float* red_col, int64_t L, int64_t m, int64_t n, float momentum, void* workspace,
                  size_t workspace_bytes, void* stream);
size_t zs_muonmd_post_workspace(int64_t L, int64_t m, int64_t n);
int zs_muonmd_post(const float* W, const void* U, int u_transposed, void* p_out, int p_dtype, void* shadow_bf16,
                   float* g_scalar, float* g_row, float* g_col, float* m1_scalar, float* m2_scalar, float* m1_row, float* m2_row,
                   float* m1_col, float* m2_col, const float* red_scalar, const float* red_row, const float* red_col,
                   const float* step_dev, float step_host, float b1, float b2, float eps, float gain_lr,
                   const float* lr_dev, float lr_host, float rescale, int norm_axis, const float* target_norm,
                   int64_t L, int64_t m, int64_t n, void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------ AdamW step (a23) */

/*
 * The aux-Adam groups of SingleDeviceMuonMDWithAuxAdam (optimizer/muon.py:
 * 616-650, adam_update :131-136) over a list of f32 parameters in one launch:
 *   m1 = lerp(m1, g, 1-b1); m2 = lerp(m2, g*g, 1-b2);
 *   u  = (m1 / (1 - b1^t)) / (sqrt(m2 / (1 - b2^t)) + eps);
 *   p  = p * (1 - lr*wd) - lr * u;   shadow_bf16 (optional) = bf16(p).
 * Per tensor: step_dev (f32 device scalar, already incremented for this step)
 * or, when NULL, the host step given as the f32 reciprocals of its bias
 * corrections (inv_bc*_host = 1 / (1 - b^t) computed in double).  lr from
 * lr_dev (f32 device scalar; decay = 1 - lr*wd in f32) or lr_host with
 * decay_host.  one_minus_b* are the lerp weights as the host computes them.
 * p, g, m1, m2 contiguous, n elements each; any number of tensors (launched
 * 96 per kernel).
 */
typedef struct {
  float* p;
  const float* g;
  float* m1;
  float* m2;
  const float* step_dev;
  float inv_bc1_host;
  float inv_bc2_host;
  void* shadow_bf16;
  int64_t n;
} zs_adamw_tensor;

int zs_adamw_step(const zs_adamw_tensor* tensors, int count, const float* lr_dev, float lr_host, float decay_host,
                  float b1, float b2, double one_minus_b1, double one_minus_b2, float eps, float weight_decay,
                  void* stream);

/*
 * Data-parallel all-reduce over NVLink peer memory with the copy engines (no
 * counterpart in the reference, which trains on one device; replaces the NCCL
 * all-reduce of data-parallel gradients).  Buffers are shared between the
 * processes of one node through CUDA IPC:
 *   zs_ipc_export: IPC handle (zs_ipc_handle_size() bytes) of the allocation
 *                  holding ptr, and ptr's byte offset in it;
 *   zs_ipc_open:   map a peer's handle on `device`; *ptr_out = mapping +
 *                  offset, *base_out = the mapping for zs_ipc_close.
 * zs_ce_allreduce: data (count elements, bf16 or f32, 16-byte aligned) =
 *   scale * the sum over the `world` ranks' data, bit-identical on every rank
 *   (rank r sums chunk r in rank order in f32).  recv[p], red[p], flags[p]:
 *   rank p's receive buffer (world * zs_ce_allreduce_chunk(count, world)
 *   elements), reduced-chunk buffer (one chunk) and int32 flag table [3 *
 *   world] (zeroed before the first call), as mapped in this process (own
 *   entries local).  `step` starts at 1 and grows by one per call on the same
 *   buffers.  Every rank makes the same calls in the same order.  The copies run
 *   on the copy engines; waits for peers are bounded and record
 *   ZS_DEVERR_TIMEOUT_PEER when they expire.
 */
int zs_ipc_handle_size(void);
int zs_ipc_export(const void* ptr, void* handle_out, int64_t* offset_out);
int zs_ipc_open(const void* handle, int64_t offset, int device, void** ptr_out, void** base_out);
int zs_ipc_close(void* base);
int64_t zs_ce_allreduce_chunk(int64_t count, int world);
int zs_ce_allreduce(void* data, int64_t count, int dtype, int rank, int world, void* const* recv, void* const* red,
                    int* const* flags, int step, float scale, void* stream);

/*
 * Sparse input embedding (modeling/model.py:71-86: nn.Embedding(sparse=True),
 * bag mean in f32 for token-superposition ids, x sqrt(d) when untied):
 *   zs_embedding_bag_forward:  out[t, :] = scale * mean_{j < bag} table[ids[t*bag + j], :]
 *     table f32 [num_rows, d] (row stride d), ids int64 [num_bags * bag],
 *     out f32 [num_bags, d]; bag = 1 is the plain lookup.  Out-of-range ids
 *     contribute nothing and record ZS_DEVERR_INDEX.
 *   zs_embedding_bag_backward: the COO values of the table gradient, one row
 *     per lookup in lookup order: values[t*bag + j, :] = (dy[t, :] * scale) / bag
 *     (the indices are the ids themselves).  d % 4 == 0, 16-byte aligned rows.
 */
int zs_embedding_bag_forward(const float* table, int64_t num_rows, int64_t d, const int64_t* ids, int64_t num_bags,
                             int bag, float scale, float* out, void* stream);
int zs_embedding_bag_backward(const float* dy, int64_t num_bags, int bag, int64_t d, float scale, float* values,
                              void* stream);

/*
 * GramReaperSparse.step (engram/GramReaperSparse.py:18-66) on one table: the
 * COO gradient (rows int64 [n], values f32 [n, d], duplicates allowed, in any
 * order) is summed per distinct row in lookup order (coalesce), then for each
 * touched row r:
 *   v[r] = beta * v[r] + (1 - beta) * sum(g_r^2)
 *   p[r] -= lr / (sqrt(v[r] / (1 - beta^t)) + eps) * g_r
 *   p[r] /= max(||p[r]||, eps)                       (unit_norm != 0)
 * t is the device counter *step_counter, incremented once per call with n > 0
 * (n == 0 leaves everything untouched, as the reference skips).  lr is *lr_ptr
 * when lr_ptr is not NULL (a device f32, read when the kernels run), else lr.
 * No host synchronisation; deterministic (a stable radix sort by row, one CTA
 * per distinct row).  d <= 4096, d % 4 == 0.  Rows outside [0, num_rows) are
 * skipped and record ZS_DEVERR_INDEX.
 */
size_t zs_sparse_rmsprop_workspace(int64_t n, int64_t num_rows);
int zs_sparse_rmsprop_step(float* param, int64_t num_rows, int64_t d, int64_t ld_param, float* v_state,
                           long long* step_counter, const int64_t* rows, const float* values, int64_t ld_values,
                           int64_t n, const float* lr_ptr, float lr, double beta, float eps, int unit_norm,
                           void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ZS_H_ */
