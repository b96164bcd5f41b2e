/*
 * sumac_b200.h — C ABI of libsumac_b200.so, the B200 (sm_100a) implementation of the hot path of
 * flatironinstitute/sumac: the fused masked product ReLU(A B^T) with the sparse S subtracted on its
 * support, the SALSA block step and the GD block step built on it, and the per-block CSR
 * preprocessing they read.
 *
 * Conventions
 *  - Every pointer is device memory of the current CUDA device unless stated otherwise.
 *  - Matrices are row-major fp32. "Padded" factors have Dp = sumac_padded_rank(d) columns whose
 *    entries d..Dp-1 are zero; their rows are 16-byte aligned.
 *  - Nothing here allocates device memory or synchronises: callers pass workspaces sized by the
 *    matching *_workspace_bytes query, and all work is enqueued on `stream`.
 *  - Every entry point returns SUMAC_OK (0) or a negative status; sumac_last_error() gives the
 *    message of the last failure on the calling thread. Kernels never trap: a device-side wait that
 *    runs out of time writes a nonzero code into *dev_err (device int) and returns.
 *  - precision: SUMAC_TF32 (1) = one TF32 tensor-core pass; SUMAC_3XTF32 (3) = the split
 *    hi/lo 3xTF32 scheme, fp32-accurate (the reference's default fp32 path, allow_tf32=False).
 */
#ifndef SUMAC_B200_H
#define SUMAC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* sumac_stream_t; /* a cudaStream_t */

enum {
  SUMAC_OK = 0,
  SUMAC_ERR_ARG = -1,         /* bad shape / pointer / alignment */
  SUMAC_ERR_UNSUPPORTED = -2, /* rank / precision combination not built */
  SUMAC_ERR_WORKSPACE = -3,   /* workspace too small */
  SUMAC_ERR_CUDA = -4,        /* a CUDA runtime call failed */
};
enum { SUMAC_TF32 = 1, SUMAC_3XTF32 = 3 };

/* Library version, number of SMs of `device`, padded rank for a rank d, last error message. */
int sumac_version(void);
int sumac_num_sms(int device);
int sumac_padded_rank(int d);
const char* sumac_last_error(void);
/* Time limit for device-side waits (nanoseconds, default 2e9). */
void sumac_set_timeout_ns(unsigned long long ns);
/* Number of kernels this library has launched since it was loaded (all threads and devices). */
long long sumac_kernel_launches(void);

/*
 * The fused product alone on prepared operands (the benchmark view of the hot kernel, as the
 * reference's kernel_benchmarks/relu_bat_c_bench.py times relu_bat_c alone):
 * partials[s][M][Dp] = sum over the chunks of split s of ReLU(X F^T) C, with X[M][Dp],
 * F{hi,lo}[N][Dp], Ct{hi,lo}[Dp][ldct] = C^T (tf32 hi / lo split for SUMAC_3XTF32; for SUMAC_TF32
 * lo may be NULL and Fhi holds F rounded to tf32 values: the kernel rounds X itself). The number of splits s is sumac_relu_product_splits(M, N, Dp, precision);
 * `partials` must hold s*M*Dp floats plus 4 more (scratch for the operand maxima of SUMAC_TF32).
 */
int sumac_relu_product_splits(int64_t M, int64_t N, int Dp, int precision);
int sumac_relu_product(const float* X, int64_t M, const float* Fhi, const float* Flo,
                       const float* Cthi, const float* Ctlo, int64_t ldct, int64_t N, int Dp,
                       int precision, float* partials, int* dev_err, sumac_stream_t stream);

/*
 * relu_bat_c: Y[M][D] = ReLU(B[M][D] A[N][D]^T) C[N][D], plain (unpadded) row-major inputs.
 * Replaces the custom op sumac::relu_bat_c_fused
 * (src/sumac/kernels/relu_batc_jit/custom_op.py:7-42 -> jit_kernel.py:91-135) and the TF32 op
 * sumac::relu_bat_c_tf32_mma_sync (src/sumac/kernels/relu_batc_tf32_jit/custom_op.py:33-79).
 */
size_t sumac_relu_bat_c_workspace_bytes(int64_t M, int64_t N, int D, int precision);
int sumac_relu_bat_c(const float* A, const float* B, const float* C, int64_t M, int64_t N, int D,
                     float* Y, int precision, void* ws, size_t ws_bytes, int* dev_err,
                     sumac_stream_t stream);

/*
 * relu_bat_c with a choice of the elementwise map applied to S = B A^T before the contraction:
 * SUMAC_RELU gives relu_bat_c; SUMAC_STEP gives Y = step(B A^T) C with step(s) = 1 for s > 0 and
 * 0 otherwise, the mask product in the gradient of sum ReLU(A B^T) that the reference forms densely
 * in src/sumac/kernels/relu_bat_reduce_jit/custom_op.py:74-82 (relu_mask @ B, relu_mask.T @ A).
 * Same workspace as sumac_relu_bat_c.
 */
enum { SUMAC_RELU = 0, SUMAC_STEP = 1 };
int sumac_relu_bat_c_mode(const float* A, const float* B, const float* C, int64_t M, int64_t N,
                          int D, float* Y, int precision, int mode, void* ws, size_t ws_bytes,
                          int* dev_err, sumac_stream_t stream);

/*
 * relu_bat_reduce: out[0] = sum ReLU(A B^T), out[1] = sum ReLU(A B^T)^2 (double, device), with
 * A[M][D], B[N][D] unpadded. Replaces sumac::relu_bat_reduce_fused
 * (src/sumac/kernels/relu_bat_reduce_jit/custom_op.py:7-18 -> jit_kernel.py:87-132).
 */
size_t sumac_relu_bat_reduce_workspace_bytes(int64_t M, int64_t N, int D, int precision);
int sumac_relu_bat_reduce(const float* A, const float* B, int64_t M, int64_t N, int D,
                          double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                          sumac_stream_t stream);

/*
 * relu_bat_reduce without a caller workspace. No counterpart in the reference: it exists for
 * callers that cannot give this library device memory (a host whose allocator owns every byte of
 * the GPU, such as a MATLAB gpuArray binding or a serving process that reserved the device, or a
 * path where cudaMalloc / cudaFree must not run because they can synchronise the device). Its
 * scratch is a fixed 16 MiB array (sumac_noalloc_scratch_bytes()) that lives in the library's
 * device image on every GPU that loads it until the process exits; larger problems are rejected
 * with SUMAC_ERR_WORKSPACE. All calls share the array, so calls that overlap on the GPU race. The
 * first call on a device looks up the array's address and should come before any stream capture.
 * Same inputs, output and checks as sumac_relu_bat_reduce; it allocates nothing.
 */
size_t sumac_noalloc_scratch_bytes(void);
int sumac_relu_bat_reduce_noalloc(const float* A, const float* B, int64_t M, int64_t N, int D,
                                  double* out, int precision, int* dev_err,
                                  sumac_stream_t stream);

/*
 * Masked product on padded operands: Y[M][Dp] = R C with R[j][i] = ReLU(L_ji) off the support and
 * L_ji - S_ij on it, L = X F^T (X: M rows, F and C: N rows). The support of row j is
 * ent[rowptr[j] .. rowptr[j+1]) with int pairs {i, bits of S_ij}. rowptr may be NULL (no support).
 * Semantics of the sparse fused kernel (src/sumac/kernels/relu_batc_jit/kernel_fused.cu:117-133,
 * matlab/sumac/relu_bat_c_sparse_fused_nvrtc_mex.cu).
 */
size_t sumac_masked_product_workspace_bytes(int64_t M, int64_t N, int Dp, int precision);
int sumac_masked_product(const float* X, const float* F, const float* C, int64_t M, int64_t N,
                         int Dp, const int32_t* rowptr, const int32_t* ent, float* Y,
                         int precision, void* ws, size_t ws_bytes, int* dev_err,
                         sumac_stream_t stream);

/*
 * One SALSA least-squares block update of the padded factor X[M][Dp] (in place, with its momentum
 * buffer dX) against rows `rows[0..b)` of the padded fixed factor F[m_fixed][Dp]:
 *   P = F_I (F_I^T F_I)^{-1};  X' per training/salsa.py:84-116 (lsq_update_single_gpu) with the
 *   block's support in CSR form (rowptr[M+1] absolute into ent; entries {local row in rows, S}).
 * Replaces batch_update_single_gpu (training/salsa.py:119-166) and its kernel call.
 * unbias is a device float (1 - momentum^step).
 */
size_t sumac_salsa_update_workspace_bytes(int64_t M, int64_t b_max, int d, int precision);
int sumac_salsa_block_update(const float* F, int64_t m_fixed, const int64_t* rows, int64_t b,
                             float* X, float* dX, int64_t M, int d, const int32_t* rowptr,
                             const int32_t* ent, float momentum, float lrate,
                             const float* unbias, int precision, void* ws, size_t ws_bytes,
                             int* dev_err, sumac_stream_t stream);

/*
 * Per-block CSR of one update direction after a reshuffle (datasets.py:37-58 partition, layout of
 * matlab/sumac/salsa_loop_cuda.m:143-208). Edges (e_fixed[e], e_out[e], e_val[e]) must be sorted
 * by e_out (stable). For the permutation perm[m_fixed] (int64, as torch.randperm returns) the
 * block of an edge is perm^-1[e_fixed] / ceil(m_fixed / num_blocks). Output: rowptr[num_blocks*M+1]
 * over keys block*M + out_row, ent[2*nnz] = {local fixed row, value bits}; stable, bit-exact.
 */
size_t sumac_block_csr_workspace_bytes(int64_t m_fixed, int64_t nnz, int num_blocks, int64_t M);
int sumac_block_csr_build(const int64_t* perm, int64_t m_fixed, int num_blocks,
                          const int32_t* e_fixed, const int32_t* e_out, const float* e_val,
                          int64_t nnz, int64_t M, int32_t* rowptr, int32_t* ent, void* ws,
                          size_t ws_bytes, sumac_stream_t stream);

/*
 * GD block gradient (errZ of eval.py:24-38 differentiated as in
 * kernels/relu_bat_reduce_jit/custom_op.py:39-85 plus the support terms): with L = A_I B^T and R
 * the masked residual, gA[rows[i]] (+)= 2 (R B)_i and gB (+)= 2 R^T A_I. A[m][Dp], B[n][Dp].
 * rowptr_b[n+1]/ent_b: block support by column j (entries {local row i, S}); rowptr_a[b+1]/ent_a:
 * the same support by local row i (entries {j, S}).
 */
size_t sumac_gd_grad_workspace_bytes(int64_t n, int64_t b_max, int d, int precision);
int sumac_gd_block_grad(const float* A, const float* B, int64_t n, int d, const int64_t* rows,
                        int64_t b, const int32_t* rowptr_b, const int32_t* ent_b,
                        const int32_t* rowptr_a, const int32_t* ent_a, float* gA, float* gB,
                        int accumulate, int precision, void* ws, size_t ws_bytes, int* dev_err,
                        sumac_stream_t stream);

/*
 * Metric terms (eval.py:14-38, 111-157) over the whole factorisation: out[8] doubles (device):
 * {sum ReLU(L), sum ReLU(L)^2, sum_S ReLU(L)^2, sum_S (S-ReLU(L))^2, sum_S (S-L)^2,
 *  sum_S min(S, ReLU(L)), sum_S S, sum_S S^2} with L = A B^T, S given as COO (ei, ej, v).
 * A[m][Dp], B[n][Dp] padded.
 */
size_t sumac_eval_terms_workspace_bytes(int64_t m, int64_t n, int64_t nnz, int d, int precision);
int sumac_eval_terms(const float* A, const float* B, int64_t m, int64_t n, int d,
                     const int32_t* ei, const int32_t* ej, const float* v, int64_t nnz,
                     double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                     sumac_stream_t stream);
/* The eight terms of sumac_eval_terms plus out[8] = the number of positive entries of A B^T,
 * the numerator of the MATLAB implementation's fnnz = nnz(ReLU(A B^T)) / nnz(S)
 * (matlab/sumac/compute_errors.m:62, counted by src/sumac/kernels/relu_bat_reduce_jit/
 * kernel_nnz.cu:11-119). out has 9 doubles; same workspace as sumac_eval_terms. */
int sumac_eval_terms_fnnz(const float* A, const float* B, int64_t m, int64_t n, int d,
                          const int32_t* ei, const int32_t* ej, const float* v, int64_t nnz,
                          double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                          sumac_stream_t stream);
/* The same eight terms for one GD row block (rows of A, support by column as in
 * sumac_gd_block_grad); out (+)= when accumulate. */
size_t sumac_block_loss_workspace_bytes(int64_t n, int64_t b_max, int d, int precision);
int sumac_block_loss_terms(const float* A, const float* B, int64_t n, int d, const int64_t* rows,
                           int64_t b, const int32_t* rowptr_b, const int32_t* ent_b, double* out,
                           int accumulate, int precision, void* ws, size_t ws_bytes, int* dev_err,
                           sumac_stream_t stream);

/*
 * Optimizer steps over a flat fp32 buffer of n entries (training/gd.py:20-46):
 * Adam / AdamW(weight_decay=0) as torch.optim.Adam; lr_over_bc1 = lr / (1 - beta1^t),
 * inv_sqrt_bc2 = 1 / sqrt(1 - beta2^t).
 */
int sumac_adam_step(float* p, const float* g, float* m, float* v, int64_t n, float lr_over_bc1,
                    float inv_sqrt_bc2, float beta1, float beta2, float eps, sumac_stream_t stream);
/* SGD with momentum after clip_grad_norm_(max_norm) over the squared norm *sumsq (device). */
int sumac_grad_sumsq(const float* g, int64_t n, double* sumsq, sumac_stream_t stream);
int sumac_sgd_step(float* p, float* g, float* buf, int64_t n, float lr, float momentum, int first,
                   const double* sumsq, float max_norm, sumac_stream_t stream);
int sumac_fill_zero(float* p, int64_t n, sumac_stream_t stream);

/*
 * Row exchange of the row-sharded multi-GPU SALSA step over NVLink peer memory (no counterpart
 * kernel in the reference, which moves whole factors between devices, training/salsa.py:169-209).
 * peer_bufs: device array [world] of every rank's exchange buffer (two slots of slot_floats floats);
 * peer_flags: device array [world] of every rank's flag array (world unsigned ints, zero at start);
 * epoch: this rank's exchange counter on the device (zero at start). The call stores the rows
 * rows[p] that this rank owns (lo <= rows[p] < hi, local = its rows [lo, hi)) into row p of slot
 * (epoch + 1) & 1 of every rank's buffer, signals every rank and waits for every rank's signal
 * (bounded; a timeout writes code 8 into dev_err). Every rank must make the same
 * sequence of calls; between two calls that use the same slot, the readers of that slot must have
 * been enqueued on `stream` before the intervening call.
 */
int sumac_assemble_rows_p2p(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                            int64_t nrows, int Dp, int64_t slot_floats, float* const* peer_bufs,
                            unsigned int* const* peer_flags, unsigned int* epoch, int rank,
                            int world, int* dev_err, sumac_stream_t stream);

/*
 * Initial SALSA factors (replaces the sparse products and the gathered dot products of
 * init_salsa_factors, src/sumac/training/salsa.py:36-78).
 * sumac_init_factor: out[r][c] = sign * sqrt(sum_{e in [rowptr[r], rowptr[r+1])} val[e] R[col[e]][c])
 * for r < M, c < d (R and out row-major with d columns): sqrt(S R_A) and -sqrt(S^T R_B) from the
 * edges sorted by row, summed in edge order.
 * sumac_init_scale_terms: out[0..2] = (sum v^2, sum v L, sum L^2) in float64 over the nnz entries,
 * L = <A[ei], B[ej]> in float32 (A, B row-major, d columns); ws of
 * sumac_init_scale_workspace_bytes() bytes. Both enqueue on `stream`.
 */
int sumac_init_factor(const int32_t* rowptr, const int32_t* col, const float* val, int64_t M,
                      const float* R, int d, float sign, float* out, sumac_stream_t stream);
size_t sumac_init_scale_workspace_bytes(void);
int sumac_init_scale_terms(const float* A, const float* B, int d, const int32_t* ei,
                           const int32_t* ej, const float* v, int64_t nnz, double* out, void* ws,
                           size_t ws_bytes, sumac_stream_t stream);

/*
 * Row-sharded factors (multi-GPU SALSA): out[p] = local[rows[p] - lo] (Dp floats) when this rank
 * owns global row rows[p] (lo <= rows[p] < hi), zero otherwise. An allreduce(sum) of `out` over the
 * ranks then yields the block rows F[rows] exactly. No counterpart kernel in the reference, whose
 * multi-GPU SALSA moves whole factors between devices (training/salsa.py:169-209).
 */
int sumac_gather_owned_rows(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                            int64_t nrows, int Dp, float* out, sumac_stream_t stream);

/* Test hook for the bounded-wait path: waits on *flag (device) for at most timeout_ns and writes
 * a timeout code into *dev_err when nobody sets it. The kernel returns normally either way. */
int sumac_wait_flag(const int* flag, int* dev_err, unsigned long long timeout_ns,
                    sumac_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* SUMAC_B200_H */
