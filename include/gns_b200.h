/*
 * gns_b200.h - C ABI of the B200 (sm_100a) Gram Newton-Schulz library.
 *
 * Plain pointers, element strides and sizes; no framework types. Every call is
 * asynchronous on the given CUDA stream, allocates no device memory (callers
 * pass a workspace where one is needed), performs no host synchronisation and
 * returns GNS_OK (0) or a negative error code. gns_last_error() returns the
 * message of the most recent failure on the calling host thread.
 *
 * Element type codes: GNS_F16 = 0, GNS_BF16 = 1, GNS_F32 = 2.
 * Matrices are batched [batch, rows, cols] with element strides
 * (batch_stride, row_stride, col_stride). Interface citations refer to files of
 * the reference project afrenkai/Gram-Newton-Schulz-Ampere.
 */
#ifndef GNS_B200_H_
#define GNS_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GNS_API __attribute__((visibility("default")))
#else
#define GNS_API
#endif

typedef struct CUstream_st* gns_stream_t;

enum {
  GNS_F16 = 0,
  GNS_BF16 = 1,
  GNS_F32 = 2,
};

enum {
  GNS_OK = 0,
  GNS_ERR_ARGUMENT = -1,   /* invalid shape, dtype or scalar */
  GNS_ERR_LAYOUT = -2,     /* strides/alignment a TMA tile load cannot express */
  GNS_ERR_WORKSPACE = -3,  /* workspace missing or too small */
  GNS_ERR_CUDA = -4,       /* a CUDA runtime/driver call failed */
  GNS_ERR_DEVICE = -5,     /* device is not sm_100 */
  GNS_ERR_UNSUPPORTED = -6 /* size beyond a documented kernel limit */
};

/* Library version, e.g. 100 for 0.1.0. */
GNS_API int gns_version(void);

/* Message of the last failing call on this host thread ("" if none). */
GNS_API const char* gns_last_error(void);

/* Reads (and optionally clears) the device status word that kernels set when a
 * bounded wait gives up (0 = no failure). Synchronises the current device. */
GNS_API int gns_device_status(int* status, int clear);

/* Per-launch timing of the tcgen05 GEMM (no counterpart in the reference; used by
 * bench.py for the live roofline). gns_profile_enable(n) records a CUDA event pair
 * and the algorithmic flop count (2mnk, or mnk for symmetric products) for each of
 * the next n GEMM launches on any stream; gns_profile_collect synchronises those
 * events, writes up to `capacity` records, frees them and stops recording. */
GNS_API int gns_profile_enable(int capacity);
GNS_API int gns_profile_collect(int capacity, int* count, float* ms, double* flops, int* symmetric);

/* ------------------------------------------------------------------ GEMM
 * D = alpha * A @ B + beta * C, batched, fp32 accumulation on tcgen05.
 * A is [batch, m, k], B is [batch, k, n], C and D are [batch, m, n] with unit
 * column stride. A and B share one dtype (F16 or BF16); each may be stored with
 * either unit column stride (row-major) or unit row stride (a transposed view).
 * C (dtype c_dtype) is read only when beta != 0; it may alias D.
 * symmetric != 0 asserts the result is symmetric (m == n): only column >= row
 * is computed and mirrored, so D is exactly symmetric.
 * Replaces: TorchBackend.symmetric_matmul / symmetric_batch_matrix_matrix_product /
 * matmul / matmul_add (kernels/torch_ns.py:6-35, protocols.py:36-61) and the
 * CUTLASS exports cutlass_baddbmm / cutlass_symmetric_baddbmm
 * (kernels/cutlass_ns.cu:380-384, cutlass_ns.py:117-204). */
GNS_API int gns_gemm(int ab_dtype, int64_t batch, int64_t m, int64_t n, int64_t k,
             const void* a, int64_t a_bstride, int64_t a_rstride, int64_t a_cstride,
             const void* b, int64_t b_bstride, int64_t b_rstride, int64_t b_cstride,
             const void* c, int c_dtype, int64_t c_bstride, int64_t c_rstride,
             void* d, int d_dtype, int64_t d_bstride, int64_t d_rstride,
             float alpha, float beta, int symmetric, gns_stream_t stream);

/* ------------------------------------------------------- normalisation
 * out[b] = fp16(x[b] / (||x[b]||_F + eps)) with the norm taken in fp32.
 * x has unit column stride; out is [batch, rows, out_ld] fp16.
 * Replaces: the input normalisation of newton_schulz.py:81-84 / :141-144 / :304-307. */
GNS_API size_t gns_normalize_workspace_size(int64_t batch, int64_t rows, int64_t cols);
GNS_API int gns_frobenius_normalize(int x_dtype, int64_t batch, int64_t rows, int64_t cols,
                            const void* x, int64_t x_bstride, int64_t x_rstride,
                            void* out_f16, int64_t out_ld, float eps,
                            void* workspace, size_t workspace_bytes, gns_stream_t stream);

/* Same result as gns_frobenius_normalize, but it allocates nothing and takes no
 * workspace: for callers that cannot allocate device memory when they normalise
 * (their memory is owned by another pool or allocator, or an allocation could
 * block or fail in the middle of a step). Its scratch is a 64 KiB array inside
 * the library, held on every GPU that loads it until the process exits; it
 * serves at most 8192 matrices per call, and larger batches return
 * GNS_ERR_UNSUPPORTED with a message. Each call asks the runtime for the
 * array's device address on the current device (no allocation); the first call
 * on a device also loads the library's device code there, so make that first
 * call before any stream capture. Every call shares the one array and the
 * previous call's contents remain in it (the counters that must start at zero
 * are cleared by each call), so calls that can overlap on the GPU (different
 * streams, or concurrent host threads) race and must be serialised by the caller.
 * No counterpart in the reference. */
GNS_API int gns_frobenius_normalize_noalloc(int x_dtype, int64_t batch, int64_t rows, int64_t cols,
                                            const void* x, int64_t x_bstride, int64_t x_rstride,
                                            void* out_f16, int64_t out_ld, float eps, gns_stream_t stream);

/* Failure path of the normalisation's bounded wait (no counterpart in the
 * reference). Each normalisation CTA waits for the other row slices of its
 * matrix; a wait still unfinished after the limit (default 2 s) records status
 * 4 for gns_device_status and fills the CTA's slice of the output with NaN.
 * gns_set_wait_limit_ns sets that limit process-wide (1 ms to 10 s) and returns
 * the previous one. gns_selftest_normalize_timeout launches the normalisation
 * on a small contiguous fp32 batch (at most 64 matrices, 2^20 elements each;
 * out is [batch, rows, cols] fp16, workspace as for gns_frobenius_normalize)
 * waiting for one arrival more than it launches, so every wait runs out: the
 * call returns GNS_OK, the device status reads 4 afterwards and the output is
 * NaN. It exists so that tests can exercise the failure path without a fault. */
GNS_API int gns_set_wait_limit_ns(unsigned long long limit_ns, unsigned long long* previous);
GNS_API int gns_selftest_normalize_timeout(int64_t batch, int64_t rows, int64_t cols, const float* x,
                                           void* out_f16, void* workspace, size_t workspace_bytes,
                                           gns_stream_t stream);

/* ---------------------------------------------------- Newton-Schulz chains
 * Whole orthogonalisation of a batch in one call: normalise, iterate with the
 * given (a, b, c) coefficient triples (coeffs[3*i + 0..2]), cast to out_dtype.
 * x and out have unit column stride and may not alias. Internal products run
 * in fp16 with fp32 accumulation, like the reference's fp16 torch path.
 *
 * gns_gram_newton_schulz follows build_gram_newton_schulz_operation
 * (newton_schulz.py:124-223); reset_mask bit i restarts from X at iteration i
 * (gram_newton_schulz_reset_iterations, default (2,)). Square inputs are
 * dispatched to the standard chain by the caller, as NewtonSchulz.__call__
 * does (newton_schulz.py:308-318).
 * gns_standard_newton_schulz follows build_standard_newton_schulz_operation
 * (newton_schulz.py:66-121). */
GNS_API size_t gns_newton_schulz_workspace_size(int64_t batch, int64_t rows, int64_t cols);
GNS_API int gns_gram_newton_schulz(int x_dtype, int64_t batch, int64_t rows, int64_t cols,
                           const void* x, int64_t x_bstride, int64_t x_rstride,
                           void* out, int out_dtype, int64_t out_bstride, int64_t out_rstride,
                           const double* coeffs, int n_iters, uint32_t reset_mask, float eps,
                           void* workspace, size_t workspace_bytes, gns_stream_t stream);
GNS_API int gns_standard_newton_schulz(int x_dtype, int64_t batch, int64_t rows, int64_t cols,
                               const void* x, int64_t x_bstride, int64_t x_rstride,
                               void* out, int out_dtype, int64_t out_bstride, int64_t out_rstride,
                               const double* coeffs, int n_iters, float eps,
                               void* workspace, size_t workspace_bytes, gns_stream_t stream);

/* Tactic switch of gns_gram_newton_schulz (process-wide; returns the previous
 * setting). Enabled (the default): non-square matrices whose short side is at
 * most 128 and whose long side is at most 3072 run as ONE fused kernel per call after
 * the normalisation: a CTA per matrix keeps G, P, GP and Q in shared memory and
 * runs every product of the chain without a launch boundary; the same kernel
 * runs gns_standard_newton_schulz for square matrices of side at most 128 (X, G
 * and P in shared memory). Disabled: every product is its own GEMM launch. Both tactics compute the same products in the
 * same order and rounding. The reference's CUTLASS backend picks among its
 * kernels the same way, by size (select_cutlass_tactic, kernels/cutlass_ns.py:109-114). */
GNS_API int gns_set_small_chain(int enabled);

/* Caps the SMs one GEMM launch occupies (process-wide; 0, the default, means
 * all; returns the previous cap). The GEMM's grid is persistent and assigns
 * tiles statically, so a CTA that cannot start because another kernel (a
 * collective running beside it) holds its SM delays the whole launch; with a
 * cap the launch leaves those SMs free. No counterpart in the reference. */
GNS_API int gns_set_gemm_sm_limit(int sms);

/* ------------------------------------- pieces of a column-sharded Gram chain
 * For a matrix whose long dimension is split across ranks (a wide matrix sharded
 * by columns, or a tall one by rows), Gram Newton-Schulz only needs the m x m
 * Gram matrix summed over ranks. The distributed layer runs:
 *   s  = gns_frobenius_sumsq(shard);  all-reduce(s);  Xh = gns_frobenius_scale(shard, s)
 *   G  = gns_gemm(Xh, Xh^T, symmetric, fp32 out);  all-reduce(G)
 *   Q  = gns_gram_iterations(G, iterations [begin, end) up to the next restart)
 *   restart: Xh = Q Xh (gns_gemm);  G = all-reduce(Xh Xh^T);  next segment
 *   out = Q Xh (gns_gemm)
 * The arithmetic follows newton_schulz.py:139-217; the reference itself has no
 * such entry points (it assembles whole matrices on owner ranks with an
 * all-to-all, distributed_orthogonalization.py:278-349).
 * gns_frobenius_sumsq writes sum(x^2) per matrix in fp32 (fixed summation order;
 * workspace: gns_normalize_workspace_size bytes). gns_frobenius_scale writes
 * fp16(x / (sqrt(sumsq[b]) + eps)). gns_gram_iterations takes G (fp32 or fp16,
 * m x m, symmetric), rounds it to fp16 and runs the Gram iterations
 * [it_begin, it_end) of the given schedule as one restart-free segment (G is
 * advanced after every iteration but the last), writing Q in fp16. */
GNS_API int gns_frobenius_sumsq(int x_dtype, int64_t batch, int64_t rows, int64_t cols,
                                const void* x, int64_t x_bstride, int64_t x_rstride, float* sumsq_out,
                                void* workspace, size_t workspace_bytes, gns_stream_t stream);
GNS_API int gns_frobenius_scale(int x_dtype, int64_t batch, int64_t rows, int64_t cols,
                                const void* x, int64_t x_bstride, int64_t x_rstride, const float* sumsq,
                                float eps, void* out_f16, int64_t out_ld, gns_stream_t stream);
GNS_API size_t gns_gram_iterations_workspace_size(int64_t batch, int64_t m);
GNS_API int gns_gram_iterations(int64_t batch, int64_t m, const void* gram, int gram_f32,
                                int64_t g_bstride, int64_t g_rstride, const double* coeffs, int n_iters,
                                int it_begin, int it_end, void* q_out,
                                int64_t q_bstride, int64_t q_rstride, void* workspace,
                                size_t workspace_bytes, gns_stream_t stream);

/* ----------------------------------------------------------- Muon (K5)
 * Multi-tensor momentum for `count` tensors of numel[i] elements each:
 *   m <- g + mu * m            (torch.add(g, m, alpha=mu, out=m), muon.py:429-434)
 *   u <- g + mu * m   if nesterov (muon.py:435-436), else u is not written
 *   mu == 0: m <- g            (muon.py:425-427)
 * grads/moms/updates are arrays of device pointers held in HOST memory; every
 * grad has g_dtype, every momentum m_dtype, every update u_dtype (torch's type
 * promotion of g_dtype and m_dtype). The gradient is first rounded to m_dtype
 * (muon.py:424). With nesterov, updates[i] may be NULL: that tensor's momentum
 * is advanced and no update is written (a rank that does not orthogonalise the
 * matrix needs only the momentum). */
GNS_API int gns_muon_momentum(int count, const void* const* grads, void* const* moms, void* const* updates,
                      const int64_t* numel, int g_dtype, int m_dtype, int u_dtype, float mu,
                      int nesterov, gns_stream_t stream);

/* Multi-tensor parameter update (muon.py:471-476):
 *   p <- p * decay            (only when apply_decay != 0; decay = 1 - lr * wd)
 *   p <- p - lr_adj[i] * o    (o read with its own dtype)
 * Each step rounds to the parameter dtype, as the two torch in-place ops do. */
GNS_API int gns_muon_apply(int count, void* const* params, const void* const* updates, const int64_t* numel,
                   int p_dtype, int o_dtype, float decay, int apply_decay, const float* lr_adj,
                   gns_stream_t stream);

/* ---------------------------------------------------------- Dion3 (K6-K8)
 * Row selection for one [batch, rows, cols] matrix stack (contiguous):
 *   m <- m + g;  p <- p * parameter_decay (if != 1);  row L1 norms of m;
 *   top-`selected` rows per matrix by L1 norm, emitted as ascending int64 indices;
 *   selected <- bf16(m[idx]);  m[idx] <- m[idx] * decay.
 * selected == rows selects every row (identity indices). selected must be in [1, rows].
 * m, g and p share `dtype`. Replaces select_rows (kernels/dion3_cuda.cu:336-351) and its
 * torch twin select_dion3_rows (dion3_update.py:14-70); at::topk is replaced by a
 * radix select whose index order is ascending. */
GNS_API size_t gns_dion3_select_workspace_size(int64_t batch, int64_t rows);
GNS_API int gns_dion3_select_rows(int dtype, int64_t batch, int64_t rows, int64_t cols, void* momentum,
                          const void* gradient, void* parameter, int64_t selected, float decay,
                          float parameter_decay, void* selected_out_bf16, int64_t* indices_out,
                          void* workspace, size_t workspace_bytes, gns_stream_t stream);

/* gns_dion3_select_rows over a list of `count` separate same-shape tensors
 * (rows x cols each, contiguous, one dtype): momenta[i], gradients[i] and
 * parameters[i] (parameters may be NULL when parameter_decay == 1) are the i-th
 * matrices; the outputs are one contiguous stack, selected_out_bf16 as
 * [count, selected, cols] and indices_out as [count, selected]; workspace:
 * gns_dion3_select_workspace_size(count, rows) bytes. The same kernels run over
 * all matrices in a few launches, so a Dion3 bucket costs three launches
 * instead of three per matrix. Replaces the per-tensor loop of
 * select_dion3_rows_cuda_batch (kernels/dion3_cuda.py:111-149). */
GNS_API int gns_dion3_select_rows_multi(int dtype, int count, int64_t rows, int64_t cols, void* const* momenta,
                                        const void* const* gradients, void* const* parameters, int64_t selected,
                                        float decay, float parameter_decay, void* selected_out_bf16,
                                        int64_t* indices_out, void* workspace, size_t workspace_bytes,
                                        gns_stream_t stream);

/* NorMuon normalisation + scatter update (kernels/dion3_cuda.cu:353-503,
 * dion3_update.py:73-148) for one [batch, rows, cols] parameter stack:
 *   v[idx] <- beta2 * v[idx] + (1 - beta2) * mean(u^2)        (fp32 variance [batch, rows])
 *   n = u / (sqrt(v[idx]) + eps), rescaled by ||u||_F / max(||n||_F, eps) per matrix
 *   p[idx] <- p[idx] - lr_adj * n   (p *= 1 - lr * wd first when wd != 0)
 * u is [batch, selected, cols] with dtype u_dtype and row stride u_rstride. */
GNS_API size_t gns_dion3_normalize_workspace_size(int64_t batch, int64_t selected);
GNS_API int gns_dion3_normalize_apply(int p_dtype, int u_dtype, int64_t batch, int64_t rows, int64_t cols,
                              int64_t selected, void* parameter, const void* update,
                              int64_t u_bstride, int64_t u_rstride, float* variance,
                              const int64_t* indices, float beta2, float eps, float lr, float wd,
                              float lr_adj, void* workspace, size_t workspace_bytes,
                              gns_stream_t stream);

/* gns_dion3_normalize_apply over a list of `count` separate same-shape
 * parameters (parameters[i], rows x cols, contiguous) and their variances
 * (variances[i], rows fp32); the update is one [count, selected, cols] stack
 * with strides (u_bstride, u_rstride) and indices one [count, selected] stack;
 * workspace: gns_dion3_normalize_workspace_size(count, selected) bytes.
 * Replaces the per-tensor loop of normalize_apply_rows_cuda_batch
 * (kernels/dion3_cuda.py:220-253). */
GNS_API int gns_dion3_normalize_apply_multi(int p_dtype, int u_dtype, int count, int64_t rows, int64_t cols,
                                            int64_t selected, void* const* parameters, const void* update,
                                            int64_t u_bstride, int64_t u_rstride, float* const* variances,
                                            const int64_t* indices, float beta2, float eps, float lr, float wd,
                                            float lr_adj, void* workspace, size_t workspace_bytes,
                                            gns_stream_t stream);

/* ------------------------------------------------------ AdamW / Lion groups
 * Multi-tensor replacements of Muon's per-parameter AdamW and Lion groups
 * (muon.py:516-583), same roundings as the torch sequence there (every
 * intermediate rounded to its tensor's dtype; division by a host scalar as a
 * multiplication by its float reciprocal). Tensors of one call share
 * p_dtype (parameters), g_dtype (gradients) and s_dtype (state), are
 * contiguous, and are updated in place. AdamW takes per-tensor bias
 * corrections computed on the host in double: lr_bc1[i] = float(lr / (1 -
 * beta1^step_i)) and inv_bc2[i] = float(1 / sqrt(1 - beta2^step_i)) (reciprocal in double).
 * Every scalar is the float rounding of the host's double value, as torch
 * passes scalars: one_minus_beta = float(1 - beta) is computed from the double
 * beta, decay = float(1 - lr * weight_decay), applied when apply_decay is set. */
GNS_API int gns_adamw_step(int count, void* const* params, const void* const* grads, void* const* exp_avgs,
                           void* const* exp_avg_sqs, const int64_t* numel, int p_dtype, int g_dtype, int s_dtype,
                           const float* lr_bc1, const float* inv_bc2, float beta1, float beta2,
                           float one_minus_beta1, float one_minus_beta2, float epsilon, float decay,
                           int apply_decay, gns_stream_t stream);
GNS_API int gns_lion_step(int count, void* const* params, const void* const* grads, void* const* buffers,
                          const int64_t* numel, int p_dtype, int g_dtype, int s_dtype, float lr, float beta1,
                          float beta2, float one_minus_beta1, float one_minus_beta2, float decay, int apply_decay,
                          gns_stream_t stream);

/* The two halves of gns_dion3_normalize_apply as separate calls, for callers of
 * the reference's normalize_rows / apply_rows (kernels/dion3_cuda.py:151-192,
 * kernels/dion3_cuda.cu:353-470):
 * gns_dion3_normalize_rows updates the variance of the selected rows and writes
 * normalized (fp32, [batch * selected][cols], contiguous) = u / (sqrt(v) + eps)
 * and squared_norms (fp32, [batch][2]) = (sum |u|^2, sum |normalized|^2) per
 * matrix; workspace: gns_dion3_normalize_workspace_size bytes.
 * gns_dion3_apply_rows decays the parameter by (1 - lr * wd) and adds
 * -lr_adj * normalized * sqrt(sum |u|^2) / max(sqrt(sum |n|^2), eps) to the
 * selected rows, with the same roundings as the fused call. */
GNS_API int gns_dion3_normalize_rows(int u_dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected,
                                     const void* update, int64_t u_bstride, int64_t u_rstride, float* variance,
                                     const int64_t* indices, float beta2, float eps, float* normalized,
                                     float* squared_norms, void* workspace, size_t workspace_bytes,
                                     gns_stream_t stream);
GNS_API int gns_dion3_apply_rows(int p_dtype, int64_t batch, int64_t rows, int64_t cols, int64_t selected,
                                 void* parameter, const float* normalized, const int64_t* indices,
                                 const float* squared_norms, float lr, float wd, float lr_adj, float eps,
                                 gns_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GNS_B200_H_ */
