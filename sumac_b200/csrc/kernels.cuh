// kernels.cuh — launch interfaces of the non-tensor-core kernels (kernels.cu) and of the fused
// product (product.cu). All functions enqueue on `stream`, never allocate and never synchronise.
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_runtime.h>

namespace sb {

// Number of kernels this library has launched (all threads, all devices).
void count_launch();

// Programmatic dependent launch: a kernel launched with launch_pdl may start while the previous
// kernel of its stream drains; it calls pdl_wait() before it reads anything that kernel wrote
// (a no-op when the launch had no programmatic dependency). pdl_trigger() lets the next
// programmatic launch of the stream start before this kernel ends.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t stream, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}
long long launch_count();

// ---- fused product / reduce (product.cu) ---------------------------------------------------
// X [M][Dp], F{hi,lo} [N][Dp], Ct{hi,lo} [Dp][ldct] (row-major, 16-byte aligned rows).
// Writes ws[splits][M][Dp] partial products (splits = product_split_count(...)); step = 1 replaces
// ReLU(S) by the 0/1 step of S. f_rounded = 1 declares that F already holds tf32 values (TF32
// mode rounds X and, unless declared, every F chunk in shared memory). Returns 0 or a
// cudaError_t value; -1 for an unsupported (Dp, x3) combination, -5 bad sizes, -6 tensor map.
int launch_relu_product(const float* X, int64_t M, const float* Fhi, const float* Flo,
                        const float* Cthi, const float* Ctlo, int64_t ldct, int64_t N, int Dp,
                        bool x3, float* ws, int* err, int num_sms, unsigned long long timeout_ns,
                        cudaStream_t stream, const unsigned int* stats, int step = 0,
                        int f_rounded = 0, int nstats = 1);
// stats[0] = bits of max_r |F[r]| (row norm over Dp), stats[1] = bits of max |C| over nC values
// (atomicMax on non-negative float bits; the words must be zero beforehand). The TF32 product
// (fp16 second MMA) reads them to pick exact power-of-two scales.
void launch_operand_stats(const float* F, int64_t N, int Dp, const float* C, int64_t nC,
                          unsigned int* stats, cudaStream_t stream);
// Reduce mode: partials[grid][2] (grid <= num_sms) hold per-CTA (sum ReLU, sum ReLU^2).
// With count = 1 the partials are [grid][3]: (sum, sum^2, number of positive entries).
int launch_relu_reduce(const float* X, int64_t M, const float* Fhi, const float* Flo, int64_t N,
                       int Dp, bool x3, double* partials, int* grid_out, int* err, int num_sms,
                       unsigned long long timeout_ns, cudaStream_t stream, int count = 0,
                       int f_rounded = 0);
int product_split_count(int64_t M, int64_t N, int Dp, bool x3, int num_sms);
bool product_supported(int Dp, bool x3);
bool reduce_supported(int Dp, bool x3);

// ---- packing ------------------------------------------------------------------------------
// dst[r][0:Dp] = src[rows ? rows[r] : r][0:d] (zero padded), optional tf32 hi / lo copies.
void launch_gather_pad(const float* src, int64_t ld_src, int d, const int64_t* rows, int64_t nrows,
                       int Dp, float* dst, float* dst_hi, float* dst_lo, cudaStream_t stream);
// dst{hi,lo}[c][r] = split(src[r][c]) for c < Dp, r < nrows; dst rows have stride ld_dst.
// With dst_lo == nullptr, dst_hi receives the plain fp32 values.
void launch_transpose_split(const float* src, int64_t nrows, int Dp, float* dst_hi, float* dst_lo,
                            int64_t ld_dst, cudaStream_t stream);

// ---- SALSA least-squares prep -------------------------------------------------------------
// Gram partials of FI[b][Dp] (first d columns) into gram_ws[nparts][d*d] (double).
int gram_parts(int64_t b);
void launch_gram(const float* FI, int64_t b, int d, int Dp, double* gram_ws, cudaStream_t stream);
// P = FI G^{-1} via an LU with partial pivoting of G = sum of partials; writes P[b][Dp] and
// Ct{hi,lo}[Dp][ldct] = P^T (plain values in Cthi when Ctlo is null).
void launch_solve(const float* FI, int64_t b, int d, int Dp, const double* gram_ws, int nparts,
                  float* P, float* Cthi, float* Ctlo, int64_t ldct, int* err, cudaStream_t stream);

int salsa_gram_parts(int64_t b);

// SALSA block step with C = F_I (d <= 32): gather F_I = Ffix[rows] (and its tf32 halves, its
// transpose C^T = F_I^T split in 3xTF32 mode, and each CTA's operand maxima into its own pair
// stats[2 * cta .. 2 * cta + 1], salsa_gather_ctas(b) pairs, no zeroing needed) in one launch,
// which also zeroes the Gram-inverse counter; then G^{-1} of G = F_I^T F_I into ginv [Dp][Dp]
// (fp32) in one launch whose last CTA factors G. scratch: salsa_ginv_scratch_bytes(b, d).
int salsa_gather_ctas(int64_t b);
// SMs the Gram-inverse launch uses beside the fused product, which then runs on num_sms - kGinvSms
constexpr int kGinvSms = 11;
size_t salsa_ginv_scratch_bytes(int64_t b, int d);
void launch_salsa_gather(const float* Ffix, const int64_t* rows, int64_t b, int Dp, float* FI,
                         float* Fhi, float* Flo, float* Cthi, float* Ctlo, int64_t ldct,
                         unsigned int* stats, unsigned int* ginv_counter, cudaStream_t stream);
void launch_salsa_ginv(const float* FI, int64_t b, int d, int Dp, void* scratch,
                       unsigned int* counter, float* ginv, int* err, cudaStream_t stream);

// Row exchange over NVLink peer memory (see kernels.cu): the owned rows of rows[0..nrows) into
// slot (epoch & 1) of every rank's buffer, then a flag barrier with a bounded wait.
void launch_assemble_rows_p2p(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                              int64_t nrows, int Dp, int64_t slot_floats, float* const* peer_bufs,
                              unsigned* const* peer_flags, unsigned* epoch, int rank, int world,
                              int* err, unsigned long long timeout_ns, cudaStream_t stream);
// out[p] = local[rows[p] - lo] if lo <= rows[p] < hi else 0 (Dp floats per row).
void launch_gather_owned_rows(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                              int64_t nrows, int Dp, float* out, cudaStream_t stream);

// ---- finalize: sparse correction + update -------------------------------------------------
enum FinalizeMode { FIN_STORE = 0, FIN_SALSA = 1, FIN_GRAD = 2 };
struct FinalizeArgs {
  int mode;
  int64_t M;              // output rows
  int Dp;
  int splits;
  const float* ws;        // [splits][M][Dp]
  float* X;               // [M][Dp] row operand (read; updated in place in FIN_SALSA)
  float* dX;              // [M][Dp] momentum buffer (FIN_SALSA)
  const float* F;         // [N][Dp] fixed rows (fp32) for the on-support dot products
  const float* Cm;        // [N][Dp] rows of C
  const int32_t* rowptr;  // [M+1] (may be null: no sparse term)
  const int2* ent;        // {local fixed row, value bits}
  float* out;             // FIN_STORE / FIN_GRAD output rows
  int out_d;              // FIN_STORE: columns written (<= Dp); rows of `out` have ld_out floats
  int64_t ld_out;
  const int64_t* out_rows;// FIN_GRAD: output row of local row j (null = j)
  float scale;            // FIN_GRAD scale
  int accumulate;         // FIN_GRAD: out += instead of out =
  float momentum, lrate;  // FIN_SALSA
  const float* unbias;    // FIN_SALSA: device scalar
  const float* ginv;      // FIN_SALSA, Dp <= 32: [Dp][Dp] G^{-1}; ws and Cm were formed with F_I
};
void launch_finalize(const FinalizeArgs& a, cudaStream_t stream);

// ---- per-block CSR builder ----------------------------------------------------------------
size_t csr_workspace_bytes(int64_t m_fixed, int64_t nnz, int num_blocks, int64_t M);
int launch_block_csr(const int64_t* perm, int64_t m_fixed, int num_blocks, const int32_t* e_fixed,
                     const int32_t* e_out, const float* e_val, int64_t nnz, int64_t M,
                     int32_t* rowptr, int2* ent, void* ws, size_t ws_bytes, cudaStream_t stream);

// ---- initial factors ----------------------------------------------------------------------
void launch_init_spmm_sqrt(const int32_t* rowptr, const int32_t* col, const float* val, int64_t M,
                           const float* R, int d, float sign, float* out, cudaStream_t stream);
size_t init_scale_workspace_bytes();
void launch_init_scale_terms(const float* A, const float* B, int d, const int32_t* ei,
                             const int32_t* ej, const float* v, int64_t nnz, double* partials,
                             double* out, cudaStream_t stream);

// ---- metrics / loss -----------------------------------------------------------------------
// partials[grid][6] doubles:
//   sum M^2, sum (v-M)^2, sum (v-L)^2, sum min(v, M), sum v, sum v^2    (M = ReLU(L))
int sparse_terms_grid(int64_t n);
void launch_sparse_terms_coo(const float* A, const float* B, int Dp, const int32_t* ei,
                             const int32_t* ej, const float* v, int64_t nnz, double* partials,
                             int grid, cudaStream_t stream);
// CSR form (rows j of X, entries {local row of F, value}).
void launch_sparse_terms_csr(const float* X, const float* F, int Dp, const int32_t* rowptr,
                             int64_t M, const int2* ent, double* partials, int grid,
                             cudaStream_t stream);
// out[w] (+)= sum_n partials[n][w], fixed order.
void launch_sum_partials(const double* partials, int n, int w, double* out, int accumulate,
                         cudaStream_t stream);

// ---- optimizers ---------------------------------------------------------------------------
void launch_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr_over_bc1,
                 float inv_sqrt_bc2, float beta1, float beta2, float eps, cudaStream_t stream);
void launch_fill_zero(float* p, int64_t n, cudaStream_t stream);
void launch_sumsq(const float* g, int64_t n, double* out, cudaStream_t stream);
void launch_sgd(float* p, float* g, float* buf, int64_t n, float lr, float momentum, int first,
                const double* sumsq, float max_norm, cudaStream_t stream);

// test hook: a kernel that waits (bounded) for a flag nobody sets and reports the timeout
void launch_wait_flag(const int* flag, int* err, unsigned long long timeout_ns, cudaStream_t s);

}  // namespace sb
