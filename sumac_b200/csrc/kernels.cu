// kernels.cu — HBM / latency-bound kernels around the fused product: packing, the SALSA
// Gram + solve, the finalize pass (sparse correction + momentum update or gradient store), the
// deterministic per-block CSR builder, loss / metric terms and the optimizer steps.
#include <atomic>
#include <cstdint>

#include <algorithm>

#include "kernels.cuh"
#include "sm100.cuh"

namespace sb {

static std::atomic<long long> g_launches{0};
void count_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
long long launch_count() { return g_launches.load(std::memory_order_relaxed); }

static inline int cdiv64(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }
static inline unsigned grid_cap(int64_t work, int threads, int64_t cap) {
  int64_t g = (work + threads - 1) / threads;
  if (g < 1) g = 1;
  if (g > cap) g = cap;
  return (unsigned)g;
}

// ============================================================================================
// packing
// ============================================================================================
__global__ void gather_pad_kernel(const float* __restrict__ src, int64_t ld_src, int d,
                                  const int64_t* __restrict__ rows, int64_t nrows, int Dp,
                                  float* __restrict__ dst, float* __restrict__ dhi,
                                  float* __restrict__ dlo) {
  const int64_t total = nrows * Dp;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / Dp;
    const int c = (int)(i - r * Dp);
    const int64_t sr = rows ? rows[r] : r;
    const float x = c < d ? src[sr * ld_src + c] : 0.f;
    if (dst) dst[i] = x;
    if (dhi) {
      const float h = tf32_hi(x);
      dhi[i] = h;
      if (dlo) dlo[i] = tf32_lo(x, h);
    }
  }
}

void launch_gather_pad(const float* src, int64_t ld_src, int d, const int64_t* rows, int64_t nrows,
                       int Dp, float* dst, float* dst_hi, float* dst_lo, cudaStream_t stream) {
  const int64_t total = nrows * Dp;
  if (total == 0) return;
  count_launch();
  gather_pad_kernel<<<grid_cap(total, 256, 148 * 16), 256, 0, stream>>>(src, ld_src, d, rows,
                                                                         nrows, Dp, dst, dst_hi,
                                                                         dst_lo);
}

// 32 x 32 tiles through shared memory: dst[c][r] = src[r][c]
__global__ void transpose_split_kernel(const float* __restrict__ src, int64_t nrows, int Dp,
                                       float* __restrict__ dhi, float* __restrict__ dlo,
                                       int64_t ld_dst) {
  __shared__ float tile[32][33];
  const int64_t r0 = (int64_t)blockIdx.x * 32;
  const int c0 = blockIdx.y * 32;
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int64_t r = r0 + i;
    const int c = c0 + threadIdx.x;
    tile[i][threadIdx.x] = (r < nrows && c < Dp) ? src[r * Dp + c] : 0.f;
  }
  __syncthreads();
  for (int i = threadIdx.y; i < 32; i += 8) {
    const int c = c0 + i;
    const int64_t r = r0 + threadIdx.x;
    if (c < Dp && r < nrows) {
      const float x = tile[threadIdx.x][i];
      if (dlo) {
        const float h = tf32_hi(x);
        dhi[c * ld_dst + r] = h;
        dlo[c * ld_dst + r] = tf32_lo(x, h);
      } else {
        dhi[c * ld_dst + r] = x;
      }
    }
  }
}

void launch_transpose_split(const float* src, int64_t nrows, int Dp, float* dst_hi, float* dst_lo,
                            int64_t ld_dst, cudaStream_t stream) {
  if (nrows == 0) return;
  dim3 grid((unsigned)((nrows + 31) / 32), (unsigned)((Dp + 31) / 32));
  count_launch();
  transpose_split_kernel<<<grid, dim3(32, 8), 0, stream>>>(src, nrows, Dp, dst_hi, dst_lo, ld_dst);
}

// ============================================================================================
// SALSA prep: Gram matrix and P = F_I G^{-1}
// (training/salsa.py:138-140: GramA = Ar^T Ar; pinvAt = solve(GramA, Ar^T)^T)
// ============================================================================================
static constexpr int GRAM_ROWS_PER_PART = 256;

int gram_parts(int64_t b) {
  int p = cdiv64(b, GRAM_ROWS_PER_PART);
  return p < 1 ? 1 : p;
}

// One CTA per (256-row slice, 2048-entry group): partial[i*d + j] = sum_r FI[r][i] FI[r][j]
__global__ void gram_kernel(const float* __restrict__ FI, int64_t b, int d, int Dp,
                            double* __restrict__ parts) {
  extern __shared__ float srow[];  // [64][d]
  const int64_t r0 = (int64_t)blockIdx.x * GRAM_ROWS_PER_PART;
  const int64_t r1 = min(b, r0 + GRAM_ROWS_PER_PART);
  const int dd = d * d;
  const int ebase = blockIdx.y * 2048;
  double acc[8];
#pragma unroll
  for (int k = 0; k < 8; ++k) acc[k] = 0.0;
  for (int64_t rs = r0; rs < r1; rs += 64) {
    const int nr = (int)min((int64_t)64, r1 - rs);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * d; i += blockDim.x) {
      const int rr = i / d, c = i - rr * d;
      srow[i] = FI[(rs + rr) * Dp + c];
    }
    __syncthreads();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int e = ebase + threadIdx.x + k * 256;
      if (e < dd) {
        const int i = e / d, j = e - i * d;
        double s = 0.0;
        for (int rr = 0; rr < nr; ++rr) s += (double)srow[rr * d + i] * (double)srow[rr * d + j];
        acc[k] += s;
      }
    }
  }
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const int e = ebase + threadIdx.x + k * 256;
    if (e < dd) parts[(size_t)blockIdx.x * dd + e] = acc[k];
  }
}

void launch_gram(const float* FI, int64_t b, int d, int Dp, double* gram_ws, cudaStream_t stream) {
  dim3 grid(gram_parts(b), (d * d + 2047) / 2048);
  count_launch();
  gram_kernel<<<grid, 256, 64 * d * sizeof(float), stream>>>(FI, b, d, Dp, gram_ws);
}

// Every CTA redundantly sums the partials (fixed order), factors G = P L U with partial pivoting
// (first maximal |pivot| wins, as LAPACK getrf) and solves its rows: P[r] = G^{-1} FI[r]
// (G is symmetric, so (G^{-1} FI^T)^T = FI G^{-1}).
__global__ void solve_kernel(const float* __restrict__ FI, int64_t b, int d, int Dp,
                             const double* __restrict__ parts, int nparts, float* __restrict__ P,
                             float* __restrict__ Cthi, float* __restrict__ Ctlo, int64_t ldct,
                             int* err) {
  extern __shared__ double sG[];  // [d][d] then piv[d]
  int* piv = reinterpret_cast<int*>(sG + d * d);
  __shared__ int s_piv_row;
  const int dd = d * d;
  for (int e = threadIdx.x; e < dd; e += blockDim.x) {
    double s = 0.0;
    for (int q = 0; q < nparts; ++q) s += parts[(size_t)q * dd + e];
    sG[e] = s;
  }
  __syncthreads();
  for (int k = 0; k < d; ++k) {
    if (threadIdx.x < 32) {
      double best = -1.0;
      int bi = k;
      for (int i = k + threadIdx.x; i < d; i += 32) {
        const double a = fabs(sG[i * d + k]);
        if (a > best) { best = a; bi = i; }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const double ob = __shfl_xor_sync(0xffffffffu, best, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ob > best || (ob == best && oi < bi)) { best = ob; bi = oi; }
      }
      if (threadIdx.x == 0) {
        s_piv_row = bi;
        piv[k] = bi;
        if (best == 0.0 && err && blockIdx.x == 0) atomicCAS(err, 0, DEV_SINGULAR);
      }
    }
    __syncthreads();
    const int pr = s_piv_row;
    if (pr != k) {
      for (int j = threadIdx.x; j < d; j += blockDim.x) {
        const double t = sG[k * d + j];
        sG[k * d + j] = sG[pr * d + j];
        sG[pr * d + j] = t;
      }
    }
    __syncthreads();
    const double inv = 1.0 / sG[k * d + k];
    for (int i = k + 1 + threadIdx.x; i < d; i += blockDim.x) sG[i * d + k] *= inv;
    __syncthreads();
    const int rem = d - k - 1;
    for (int e = threadIdx.x; e < rem * rem; e += blockDim.x) {
      const int i = k + 1 + e / rem, j = k + 1 + e % rem;
      sG[i * d + j] -= sG[i * d + k] * sG[k * d + j];
    }
    __syncthreads();
  }
  const int64_t r = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= b) return;
  double x[256];
  for (int c = 0; c < d; ++c) x[c] = (double)FI[r * Dp + c];
  for (int k = 0; k < d; ++k) {
    const int p = piv[k];
    if (p != k) { const double t = x[k]; x[k] = x[p]; x[p] = t; }
  }
  for (int i = 0; i < d; ++i) {
    double s = x[i];
    for (int j = 0; j < i; ++j) s -= sG[i * d + j] * x[j];
    x[i] = s;
  }
  for (int i = d - 1; i >= 0; --i) {
    double s = x[i];
    for (int j = i + 1; j < d; ++j) s -= sG[i * d + j] * x[j];
    x[i] = s / sG[i * d + i];
  }
  for (int c = 0; c < Dp; ++c) {
    const float v = c < d ? (float)x[c] : 0.f;
    P[r * Dp + c] = v;
    if (Ctlo) {
      const float h = tf32_hi(v);
      Cthi[c * ldct + r] = h;
      Ctlo[c * ldct + r] = tf32_lo(v, h);
    } else {
      Cthi[c * ldct + r] = v;
    }
  }
}

void launch_solve(const float* FI, int64_t b, int d, int Dp, const double* gram_ws, int nparts,
                  float* P, float* Cthi, float* Ctlo, int64_t ldct, int* err, cudaStream_t stream) {
  const int grid = cdiv64(b, 128);
  const size_t smem = (size_t)d * d * sizeof(double) + (size_t)d * sizeof(int) + 16;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(solve_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  count_launch();
  solve_kernel<<<grid, 128, smem, stream>>>(FI, b, d, Dp, gram_ws, nparts, P, Cthi, Ctlo, ldct, err);
}


// ============================================================================================
// SALSA least-squares helpers (training/salsa.py:138-140)
// ============================================================================================
static constexpr int PREP_ROWS = 64;

int salsa_gram_parts(int64_t b) { return cdiv64(b, PREP_ROWS) < 1 ? 1 : cdiv64(b, PREP_ROWS); }


// ============================================================================================
// SALSA block step without the least-squares map P (training/salsa.py:138-140 rewritten):
// since P = F_I G^{-1}, the product R P equals (R F_I) G^{-1} and the support term
// sum_i c_ji P_i equals (sum_i c_ji F_i) G^{-1}. So the fused product contracts with C = F_I
// directly, the finalize pass applies G^{-1} to each row once, and the Gram matrix and its inverse
// are needed only by the finalize pass: they are computed on a side stream while the product runs.
//   salsa_gather_kernel  F_I = F[rows] (fp32, tf32 hi / lo halves), C^T = F_I^T (split in 3xTF32
//                        mode) and the operand maxima of the TF32 product, 32 rows per CTA
//   salsa_ginv_kernel    partial Grams (fp64) of the block rows split over at most kGinvSms CTAs;
//                        the last CTA sums them in CTA order and inverts G by Gauss-Jordan
//                        elimination (getrf's pivot choice): G^{-1} [Dp][Dp] (fp32, zero
//                        outside d x d)
// ============================================================================================
__global__ void __launch_bounds__(256) salsa_gather_kernel(
    const float* __restrict__ Ffix, const int64_t* __restrict__ rows, int64_t b, int Dp,
    float* __restrict__ FI, float* __restrict__ Fhi, float* __restrict__ Flo,
    float* __restrict__ Cthi, float* __restrict__ Ctlo, int64_t ldct, unsigned int* stats,
    unsigned int* ginv_counter) {
  extern __shared__ float tile[];  // [32][Dp + 1]
  __shared__ float wmax[2][8];
  pdl_wait();     // launched programmatically behind the previous block update
  pdl_trigger();  // the product may launch now; it waits for this grid before reading its output
  // the Gram-inverse launch of this update runs after this grid; the previous one has finished
  if (blockIdx.x == 0 && threadIdx.x == 0 && ginv_counter) *ginv_counter = 0u;
  const int64_t r0 = (int64_t)blockIdx.x * 32;
  const int nr = (int)min((int64_t)32, b - r0);
  const int ld = Dp + 1;
  float amax = 0.f;
  for (int i = threadIdx.x; i < nr * Dp; i += blockDim.x) {
    const int rr = i / Dp, c = i - rr * Dp;
    const float v = Ffix[rows[r0 + rr] * Dp + c];
    tile[rr * ld + c] = v;
    amax = fmaxf(amax, fabsf(v));
    const int64_t o = (r0 + rr) * Dp + c;
    FI[o] = v;
    if (Fhi) {  // tf32 hi / lo halves (3xTF32), or the value rounded to tf32 (TF32: no Flo)
      const float h = tf32_hi(v);
      Fhi[o] = h;
      if (Flo) Flo[o] = tf32_lo(v, h);
    }
  }
  __syncthreads();
  // transposed copy: for column c, the CTA's 32 rows are 32 consecutive floats
  for (int i = threadIdx.x; i < Dp * 32; i += blockDim.x) {
    const int c = i >> 5, rr = i & 31;
    if (rr < nr) {
      const float v = tile[rr * ld + c];
      if (Ctlo) {
        const float h = tf32_hi(v);
        Cthi[c * ldct + r0 + rr] = h;
        Ctlo[c * ldct + r0 + rr] = tf32_lo(v, h);
      } else {
        Cthi[c * ldct + r0 + rr] = v;
      }
    }
  }
  if (stats) {
    float n2 = 0.f;
    if ((int)threadIdx.x < nr)
      for (int c = 0; c < Dp; ++c) n2 = fmaf(tile[threadIdx.x * ld + c], tile[threadIdx.x * ld + c], n2);
    float fm = sqrtf(n2);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      fm = fmaxf(fm, __shfl_xor_sync(0xffffffffu, fm, o));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    }
    // this CTA's pair: maxima over its warps (no atomics, so no zeroing before the launch)
    if ((threadIdx.x & 31) == 0) {
      wmax[0][threadIdx.x >> 5] = fm;
      wmax[1][threadIdx.x >> 5] = amax;
    }
    __syncthreads();
    if (threadIdx.x < 2) {
      float m = 0.f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, wmax[threadIdx.x][w]);
      stats[2 * blockIdx.x + threadIdx.x] = __float_as_uint(m);
    }
  }
}

int salsa_gather_ctas(int64_t b) { return (int)cdiv64(b > 0 ? b : 1, 32); }

// G^{-1} by Gauss-Jordan elimination of [G | I] (a0: D x 2D, fp64) held in one warp's registers:
// lane l keeps column l of the 32 columns, all D rows. At step k column k is broadcast from its
// lane, every lane picks the pivot row (largest |entry| at or below k, the first on ties:
// getrf's choice, with magnitudes compared in fp32) and updates its column: row k <- pivot row /
// pivot, row pr <- old row k, other rows r <- r - r[k] * (new row k). No CTA barrier inside the
// elimination; the step's dependent chain is short because fp64 operations have long latency.
__device__ __forceinline__ void warp_gauss_jordan16(const double (*a0)[32], int d, int Dp,
                                                    float* ginv, int* err) {
  constexpr int D = 16;
  const int lane = threadIdx.x & 31;
  double c[D];
#pragma unroll
  for (int i = 0; i < D; ++i) c[i] = a0[i][lane];
  for (int k = 0; k < d; ++k) {
    double colk[D];
    float mag[D];
    int id[D];
#pragma unroll
    for (int i = 0; i < D; ++i) {
      colk[i] = __shfl_sync(0xffffffffu, c[i], k);
      mag[i] = (i >= k && i < d) ? fabsf((float)colk[i]) : -1.f;
      id[i] = i;
    }
    // pivot: largest magnitude (compared in fp32), the first on ties, by a tree over the rows
    // (the lower-index half always on the left) instead of a chain of dependent fp64 compares
#pragma unroll
    for (int w = 1; w < D; w <<= 1) {
#pragma unroll
      for (int i = 0; i + w < D; i += 2 * w) {
        if (mag[i + w] > mag[i]) { mag[i] = mag[i + w]; id[i] = id[i + w]; }
      }
    }
    const int idx = id[0];
    if (lane == 0 && mag[0] == 0.f && err) atomicCAS(err, 0, DEV_SINGULAR);
    double pv = 0.0, ck = 0.0, cpr = 0.0, ckk = 0.0;
#pragma unroll
    for (int i = 0; i < D; ++i) {
      if (i == idx) { pv = colk[i]; cpr = c[i]; }
      if (i == k) { ckk = colk[i]; ck = c[i]; }
    }
    // 1 / pv: fp32 seed refined by two Newton-Raphson steps r <- r + r (1 - pv r) (each doubles
    // the correct bits: 2^-23 -> 2^-46 -> fp64 rounding); IEEE division where the seed is not
    // finite (|pv| outside the fp32 range)
    double inv = (double)(1.0f / (float)pv);
    if (isfinite(inv) && inv != 0.0) {
      inv = fma(inv, fma(-pv, inv, 1.0), inv);
      inv = fma(inv, fma(-pv, inv, 1.0), inv);
    } else {
      inv = 1.0 / pv;
    }
    const double rowk = cpr * inv;  // this lane's entry of the pivot row, moved to k and scaled
#pragma unroll
    for (int i = 0; i < D; ++i) {
      const double sv = (i == idx) ? ck : c[i];      // row pr takes the old row k
      const double sk = (i == idx) ? ckk : colk[i];
      c[i] = (i == k) ? rowk : sv - sk * rowk;
    }
  }
  // columns D..2D-1 hold G^{-1}: lane D + col writes column col
  if (lane >= D) {
    const int col = lane - D;
    for (int k = 0; k < Dp; ++k) {
      double v = 0.0;
#pragma unroll
      for (int i = 0; i < D; ++i)
        if (i == k) v = c[i];
      ginv[k * Dp + col] = (k < d && col < d) ? (float)v : 0.f;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256) salsa_ginv_kernel(
    const float* __restrict__ FI, int64_t b, int d, int Dp, int64_t rows_per_cta,
    double* __restrict__ parts, unsigned int* counter, double* __restrict__ LU,
    int* __restrict__ piv, float* __restrict__ ginv, int* err) {
  __shared__ float srow[PREP_ROWS * (D + 1)];
  __shared__ double aug[2][D][2 * D];  // [G | I] and its Gauss-Jordan iterates (double-buffered)
  __shared__ bool last;
  const int dd = d * d;
  // this CTA's rows [r0, r1), staged PREP_ROWS at a time; each thread keeps its entries' sums
  constexpr int EPT = (D * D + 255) / 256;  // Gram entries per thread
  double acc[EPT];
#pragma unroll
  for (int q = 0; q < EPT; ++q) acc[q] = 0.0;
  const int64_t r0 = (int64_t)blockIdx.x * rows_per_cta;
  const int64_t r1 = min(b, r0 + rows_per_cta);
  for (int64_t c0 = r0; c0 < r1; c0 += PREP_ROWS) {
    const int nr = (int)min((int64_t)PREP_ROWS, r1 - c0);
    __syncthreads();
    for (int i = threadIdx.x; i < nr * D; i += blockDim.x) {
      const int rr = i / D, c = i - rr * D;
      srow[rr * (D + 1) + c] = c < d ? FI[(c0 + rr) * Dp + c] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < EPT; ++q) {
      const int e = threadIdx.x + q * 256;
      if (e < dd) {
        const int i = e / d, j = e - i * d;
        // four independent fp64 chains (fp64 latency, not throughput, bounds this loop)
        double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
        int rr = 0;
        for (; rr + 3 < nr; rr += 4) {
          s0 += (double)srow[rr * (D + 1) + i] * (double)srow[rr * (D + 1) + j];
          s1 += (double)srow[(rr + 1) * (D + 1) + i] * (double)srow[(rr + 1) * (D + 1) + j];
          s2 += (double)srow[(rr + 2) * (D + 1) + i] * (double)srow[(rr + 2) * (D + 1) + j];
          s3 += (double)srow[(rr + 3) * (D + 1) + i] * (double)srow[(rr + 3) * (D + 1) + j];
        }
        for (; rr < nr; ++rr) s0 += (double)srow[rr * (D + 1) + i] * (double)srow[rr * (D + 1) + j];
        acc[q] += (s0 + s1) + (s2 + s3);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < EPT; ++q) {
    const int e = threadIdx.x + q * 256;
    if (e < dd) parts[(size_t)blockIdx.x * dd + e] = acc[q];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) last = atomicAdd(counter, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int e = threadIdx.x; e < D * 2 * D; e += blockDim.x) {
    const int i = e / (2 * D), j = e - i * (2 * D);
    double v = 0.0;
    if (j < D) {
      if (i < d && j < d) {
#pragma unroll 8
        for (int q = 0; q < (int)gridDim.x; ++q) v += __ldcg(&parts[(size_t)q * dd + i * d + j]);
      }
    } else {
      v = (j - D == i) ? 1.0 : 0.0;
    }
    aug[0][i][j] = v;
  }
  __syncthreads();
  if constexpr (D == 16) {
    if (threadIdx.x < 32) warp_gauss_jordan16(aug[0], d, Dp, ginv, err);
    if (threadIdx.x == 0) *counter = 0u;  // ready for the next launch (graph replays included)
    return;
  }
  // G^{-1} by Gauss-Jordan elimination of [G | I] with partial pivoting (at step k the row, at or
  // below k, of largest |entry| in column k, the first on ties: getrf's pivot choice). Every
  // thread updates its elements of the augmented matrix from the previous iterate; one barrier
  // per step. Rows and columns beyond d stay the identity.
  (void)LU;
  (void)piv;
  int piv_row = 0;
  for (int k = 0; k < d; ++k) {
    double(*cur)[2 * D] = aug[k & 1];
    double(*nxt)[2 * D] = aug[(k + 1) & 1];
    {
      // every warp finds the pivot row itself (no extra barrier)
      const int i = threadIdx.x & 31;
      double v = (i >= k && i < d) ? fabs(cur[i][k]) : -1.0;
      int idx = i;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const double ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) { v = ov; idx = oi; }
      }
      if (threadIdx.x == 0 && v == 0.0 && err) atomicCAS(err, 0, DEV_SINGULAR);
      piv_row = idx;
    }
    const int pr = piv_row;
    const double inv = 1.0 / cur[pr][k];
    for (int e = threadIdx.x; e < D * 2 * D; e += blockDim.x) {
      const int i = e / (2 * D), j = e - i * (2 * D);
      const double rowk = cur[pr][j] * inv;  // the pivot row, moved to k and scaled
      if (i == k) {
        nxt[i][j] = rowk;
      } else {
        const int src = i == pr ? k : i;      // row pr takes the old row k
        nxt[i][j] = cur[src][j] - cur[src][k] * rowk;
      }
    }
    __syncthreads();
  }
  {
    double(*fin)[2 * D] = aug[d & 1];
    for (int e = threadIdx.x; e < Dp * Dp; e += blockDim.x) {
      const int k = e / Dp, c = e - k * Dp;
      ginv[e] = (k < d && c < d) ? (float)fin[k][D + c] : 0.f;
    }
  }
  if (threadIdx.x == 0) *counter = 0u;  // ready for the next launch (graph replays included)
}

size_t salsa_ginv_scratch_bytes(int64_t b, int d) {
  return (size_t)salsa_gram_parts(b) * d * d * sizeof(double) + 32 * 32 * sizeof(double) +
         64 * sizeof(int) + 64;
}

void launch_salsa_gather(const float* Ffix, const int64_t* rows, int64_t b, int Dp, float* FI,
                         float* Fhi, float* Flo, float* Cthi, float* Ctlo, int64_t ldct,
                         unsigned int* stats, unsigned int* ginv_counter,
                         cudaStream_t stream) {
  const size_t smem = (size_t)32 * (Dp + 1) * sizeof(float);
  count_launch();
  launch_pdl(salsa_gather_kernel, dim3((unsigned)cdiv64(b, 32)), dim3(256), smem, stream, Ffix,
             rows, b, Dp, FI, Fhi, Flo, Cthi, Ctlo, ldct, stats, ginv_counter);
}

void launch_salsa_ginv(const float* FI, int64_t b, int d, int Dp, void* scratch,
                       unsigned int* counter, float* ginv, int* err, cudaStream_t stream) {
  // at most kGinvSms CTAs (one per SM: a 256-thread CTA cannot share an SM with a product CTA),
  // on the SMs the concurrent fused product leaves free
  const int64_t rpc = std::max<int64_t>(PREP_ROWS, cdiv64(b > 0 ? b : 1, kGinvSms));
  const int np = (int)cdiv64(b > 0 ? b : 1, rpc);
  double* parts = reinterpret_cast<double*>(scratch);
  double* LU = parts + (size_t)salsa_gram_parts(b) * d * d;
  int* piv = reinterpret_cast<int*>(LU + 32 * 32);
  count_launch();
  if (Dp == 16)
    salsa_ginv_kernel<16><<<np, 256, 0, stream>>>(FI, b, d, Dp, rpc, parts, counter, LU, piv,
                                                  ginv, err);
  else
    salsa_ginv_kernel<32><<<np, 256, 0, stream>>>(FI, b, d, Dp, rpc, parts, counter, LU, piv,
                                                  ginv, err);
}

// ============================================================================================
// operand maxima for the fp16 second MMA: max row norm of F, max |C|
// ============================================================================================
__global__ void operand_stats_kernel(const float* __restrict__ F, int64_t N, int Dp,
                                     const float* __restrict__ C, int64_t nC, unsigned int* stats) {
  float fm = 0.f, cm = 0.f;
  for (int64_t r = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; r < N;
       r += (int64_t)gridDim.x * blockDim.x) {
    const float4* fr = reinterpret_cast<const float4*>(F + r * Dp);
    float n2 = 0.f;
    for (int c = 0; c < Dp / 4; ++c) {
      const float4 v = fr[c];
      n2 = fmaf(v.x, v.x, fmaf(v.y, v.y, fmaf(v.z, v.z, fmaf(v.w, v.w, n2))));
    }
    fm = fmaxf(fm, sqrtf(n2));
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < nC;
       i += (int64_t)gridDim.x * blockDim.x)
    cm = fmaxf(cm, fabsf(C[i]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    fm = fmaxf(fm, __shfl_xor_sync(0xffffffffu, fm, o));
    cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, o));
  }
  if ((threadIdx.x & 31) == 0) {
    atomicMax(&stats[0], __float_as_uint(fm));
    atomicMax(&stats[1], __float_as_uint(cm));
  }
}

void launch_operand_stats(const float* F, int64_t N, int Dp, const float* C, int64_t nC,
                          unsigned int* stats, cudaStream_t stream) {
  cudaMemsetAsync(stats, 0, 2 * sizeof(unsigned int), stream);
  count_launch();
  const int64_t work = N > nC ? N : nC;
  operand_stats_kernel<<<grid_cap(work, 256, 148 * 4), 256, 0, stream>>>(F, N, Dp, C, nC, stats);
}

// ============================================================================================
// finalize: Y = sum of split partials + sparse correction, then the per-mode update.
// Sparse term per entry (i local fixed row, value v), L = <X_j, F_i> in fp32:
//   SALSA (training/salsa.py:100-115): Ct = v - L + ReLU(L); stepC_j += Ct P_i;
//          lsq = X - Y + stepC; dX' = (lsq - X)(1-mu) + dX mu; X' = X + lr dX' / unbias
//   GRAD / STORE: corr_j += (L - v - ReLU(L)) C_i; out_j (+)= scale (Y + corr)
// One group of G = min(32, Dp/4) lanes owns a row, one float4 slice (or two) per lane.
// ============================================================================================
// Entries of a row beyond this many are shared by the whole warp in finalize_kernel.
constexpr int FIN_K0 = 8;

// <x, f> over V float4 slices (this lane's part of a row)
template <int V>
__device__ __forceinline__ float dot4v(const float4* x, const float4* f) {
  float s = 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    s = fmaf(x[v].x, f[v].x, s);
    s = fmaf(x[v].y, f[v].y, s);
    s = fmaf(x[v].z, f[v].z, s);
    s = fmaf(x[v].w, f[v].w, s);
  }
  return s;
}

// acc += coef * c over V float4 slices
template <int V>
__device__ __forceinline__ void axpy4v(float coef, const float4* c, float4* acc) {
#pragma unroll
  for (int v = 0; v < V; ++v) {
    acc[v].x = fmaf(coef, c[v].x, acc[v].x);
    acc[v].y = fmaf(coef, c[v].y, acc[v].y);
    acc[v].z = fmaf(coef, c[v].z, acc[v].z);
    acc[v].w = fmaf(coef, c[v].w, acc[v].w);
  }
}

// Support correction coefficient of one entry (value val, prediction L): SALSA adds
// (S - L + ReLU(L)) C_i (training/salsa.py:100-111), the gradient modes (L - S - ReLU(L)) C_i.
__device__ __forceinline__ float support_coef(int mode, float val, float L) {
  return (mode == FIN_SALSA) ? (val - L + fmaxf(L, 0.f)) : (L - val - fmaxf(L, 0.f));
}

template <int DP, bool GINV>
// 80 registers (3 CTAs of 256 threads per SM): room for the heavy rows' entries in flight
__global__ void __launch_bounds__(256, 3) finalize_kernel(FinalizeArgs a) {
  pdl_wait();  // launched programmatically behind the product: its partials must be complete
  constexpr int G = DP / 4 < 32 ? DP / 4 : 32;  // lanes per row
  constexpr int V = DP / 4 / G;                  // float4 slices per lane
  constexpr int RPW = 32 / G;                    // rows per warp
  const int lane = threadIdx.x & 31;
  const int gl = lane % G;
  const int gw = lane / G;
  const int64_t warp_id = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nwarps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  const float mu = a.momentum;
  const float one_m_mu = 1.0f - mu;
  const float ub = (a.mode == FIN_SALSA) ? *a.unbias : 1.f;
  // GINV: y and the support term were contracted with F_I instead of P = F_I G^{-1}; the row's
  // (y - cor) is multiplied by G^{-1} (fp32, [DP][DP]) before the update
  __shared__ __align__(16) float sginv[GINV ? DP * DP : 4];
  if constexpr (GINV) {
    for (int i = threadIdx.x; i < DP * DP; i += blockDim.x) sginv[i] = a.ginv[i];
    __syncthreads();
  }
  // all lanes of a warp run the same iterations (shuffles below use the full mask)
  for (int64_t base = warp_id * RPW; base < a.M; base += nwarps * RPW) {
    const int64_t j = base + gw;
    const bool active = j < a.M;
    const int64_t jr = active ? j : base;
    float4 y[V], x[V], cor[V], dxv[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c4 = gl + v * G;
      // the momentum row is loaded with the others, ahead of the dependent sparse loads
      dxv[v] = a.mode == FIN_SALSA ? reinterpret_cast<const float4*>(a.dX + jr * DP)[c4]
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
      float4 s = reinterpret_cast<const float4*>(a.ws + jr * DP)[c4];
      for (int q = 1; q < a.splits; ++q) {
        const float4 t = reinterpret_cast<const float4*>(a.ws + ((int64_t)q * a.M + jr) * DP)[c4];
        s.x += t.x; s.y += t.y; s.z += t.z; s.w += t.w;
      }
      y[v] = s;
      x[v] = reinterpret_cast<const float4*>(a.X + jr * DP)[c4];
      cor[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (a.rowptr) {
      const int e0 = active ? a.rowptr[j] : 0;
      const int ne = active ? a.rowptr[j + 1] - e0 : 0;
      // light part: each row's own lane group takes its first FIN_K0 entries, four per round
      // (independent loads, fixed accumulation order)
      const int nl = (RPW == 1 || ne < FIN_K0) ? ne : FIN_K0;
      int nmax = nl;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) nmax = max(nmax, __shfl_xor_sync(0xffffffffu, nmax, o));
      for (int q0 = 0; q0 < nmax; q0 += 4) {
        int2 en[4];
        float4 f[4][V], c[4][V];
        float part[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool has = q0 + u < nl;
          en[u] = has ? a.ent[e0 + q0 + u] : make_int2(0, 0);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const bool has = q0 + u < nl;
          const float4* frow = reinterpret_cast<const float4*>(a.F + (int64_t)en[u].x * DP);
          const float4* crow = reinterpret_cast<const float4*>(a.Cm + (int64_t)en[u].x * DP);
#pragma unroll
          for (int v = 0; v < V; ++v) {
            f[u][v] = has ? frow[gl + v * G] : make_float4(0.f, 0.f, 0.f, 0.f);
            c[u][v] = has ? crow[gl + v * G] : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) part[u] = dot4v<V>(x, f[u]);
#pragma unroll
        for (int o = G / 2; o > 0; o >>= 1) {
#pragma unroll
          for (int u = 0; u < 4; ++u) part[u] += __shfl_xor_sync(0xffffffffu, part[u], o);
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (q0 + u < nl) axpy4v<V>(support_coef(a.mode, __int_as_float(en[u].y), part[u]), c[u], cor);
      }
      // heavy part (power-law rows): the whole warp shares the rest of one row at a time, one
      // entry per lane group and round, then the groups' partial corrections are summed
      if (RPW > 1) {
        unsigned heavy = __ballot_sync(0xffffffffu, gl == 0 && ne > FIN_K0);
        while (heavy) {
          const int src = __ffs(heavy) - 1;
          heavy &= heavy - 1;
          const int hg = src / G;
          const int hb = __shfl_sync(0xffffffffu, e0, src) + FIN_K0;
          const int hn = __shfl_sync(0xffffffffu, ne, src) - FIN_K0;
          float4 hx[V], hcor[V];
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const int sl = hg * G + gl;
            hx[v] = make_float4(__shfl_sync(0xffffffffu, x[v].x, sl), __shfl_sync(0xffffffffu, x[v].y, sl),
                                __shfl_sync(0xffffffffu, x[v].z, sl), __shfl_sync(0xffffffffu, x[v].w, sl));
            hcor[v] = make_float4(0.f, 0.f, 0.f, 0.f);
          }
          // HU entries per lane group and round (entry q0 + u * RPW + gw; 2 measured faster than 1
          // or 4: 20.2 against 21.3 / 21.1 us at C4), the next round's
          // entries loaded before this round's F / C gathers
          constexpr int HU = 2;
          int2 en[HU];
#pragma unroll
          for (int u = 0; u < HU; ++u) {
            const int q = u * RPW + gw;
            en[u] = q < hn ? a.ent[hb + q] : make_int2(0, 0);
          }
          for (int q0 = 0; q0 < hn; q0 += HU * RPW) {
            float4 f[HU][V], c[HU][V];
            float part[HU];
#pragma unroll
            for (int u = 0; u < HU; ++u) {
              const bool has = q0 + u * RPW + gw < hn;
              const float4* frow = reinterpret_cast<const float4*>(a.F + (int64_t)en[u].x * DP);
              const float4* crow = reinterpret_cast<const float4*>(a.Cm + (int64_t)en[u].x * DP);
#pragma unroll
              for (int v = 0; v < V; ++v) {
                f[u][v] = has ? frow[gl + v * G] : make_float4(0.f, 0.f, 0.f, 0.f);
                c[u][v] = has ? crow[gl + v * G] : make_float4(0.f, 0.f, 0.f, 0.f);
              }
            }
            int2 enx[HU];
#pragma unroll
            for (int u = 0; u < HU; ++u) {
              const int q = q0 + HU * RPW + u * RPW + gw;
              enx[u] = q < hn ? a.ent[hb + q] : make_int2(0, 0);
            }
#pragma unroll
            for (int u = 0; u < HU; ++u) part[u] = dot4v<V>(hx, f[u]);
#pragma unroll
            for (int o = G / 2; o > 0; o >>= 1) {
#pragma unroll
              for (int u = 0; u < HU; ++u) part[u] += __shfl_xor_sync(0xffffffffu, part[u], o);
            }
#pragma unroll
            for (int u = 0; u < HU; ++u) {
              if (q0 + u * RPW + gw < hn)
                axpy4v<V>(support_coef(a.mode, __int_as_float(en[u].y), part[u]), c[u], hcor);
              en[u] = enx[u];
            }
          }
#pragma unroll
          for (int o = G; o < 32; o <<= 1) {
#pragma unroll
            for (int v = 0; v < V; ++v) {
              hcor[v].x += __shfl_xor_sync(0xffffffffu, hcor[v].x, o);
              hcor[v].y += __shfl_xor_sync(0xffffffffu, hcor[v].y, o);
              hcor[v].z += __shfl_xor_sync(0xffffffffu, hcor[v].z, o);
              hcor[v].w += __shfl_xor_sync(0xffffffffu, hcor[v].w, o);
            }
          }
          if (gw == hg) {
#pragma unroll
            for (int v = 0; v < V; ++v) {
              cor[v].x += hcor[v].x; cor[v].y += hcor[v].y;
              cor[v].z += hcor[v].z; cor[v].w += hcor[v].w;
            }
          }
        }
      }
    }
    if constexpr (GINV) {
      // u = (y - cor) G^{-1}: the row's DP values live in its G lanes (slice k4 of 4 columns in
      // lane k4 % G, register k4 / G); every lane forms its own output columns
      float4 t[V], u[V];
#pragma unroll
      for (int v = 0; v < V; ++v) {
        t[v] = make_float4(y[v].x - cor[v].x, y[v].y - cor[v].y, y[v].z - cor[v].z,
                           y[v].w - cor[v].w);
        u[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      const int gbase = lane - gl;
#pragma unroll
      for (int k4 = 0; k4 < DP / 4; ++k4) {
        const int src = gbase + k4 % G;
        const float4 tk = make_float4(__shfl_sync(0xffffffffu, t[k4 / G].x, src),
                                      __shfl_sync(0xffffffffu, t[k4 / G].y, src),
                                      __shfl_sync(0xffffffffu, t[k4 / G].z, src),
                                      __shfl_sync(0xffffffffu, t[k4 / G].w, src));
        const float tks[4] = {tk.x, tk.y, tk.z, tk.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float* grow = sginv + (4 * k4 + q) * DP;
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const float4 g4 = reinterpret_cast<const float4*>(grow)[gl + v * G];
            u[v].x = fmaf(tks[q], g4.x, u[v].x);
            u[v].y = fmaf(tks[q], g4.y, u[v].y);
            u[v].z = fmaf(tks[q], g4.z, u[v].z);
            u[v].w = fmaf(tks[q], g4.w, u[v].w);
          }
        }
      }
#pragma unroll
      for (int v = 0; v < V; ++v) {
        y[v] = u[v];
        cor[v] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
    if (!active) continue;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int c4 = gl + v * G;
      if (a.mode == FIN_SALSA) {
        const float4 dx = dxv[v];
        float4 nx, ndx;
#define SB_SALSA_COMPONENT(comp)                                   \
  {                                                                \
    const float lsq = (x[v].comp - y[v].comp) + cor[v].comp;       \
    ndx.comp = (lsq - x[v].comp) * one_m_mu + dx.comp * mu;        \
    nx.comp = x[v].comp + a.lrate * ndx.comp / ub;                 \
  }
        SB_SALSA_COMPONENT(x) SB_SALSA_COMPONENT(y) SB_SALSA_COMPONENT(z) SB_SALSA_COMPONENT(w)
#undef SB_SALSA_COMPONENT
        reinterpret_cast<float4*>(a.X + j * DP)[c4] = nx;
        reinterpret_cast<float4*>(a.dX + j * DP)[c4] = ndx;
      } else if (a.mode == FIN_STORE) {
        const int64_t orow = a.out_rows ? a.out_rows[j] : j;
        float* o = a.out + orow * a.ld_out + 4 * c4;
        const float r[4] = {y[v].x + cor[v].x, y[v].y + cor[v].y, y[v].z + cor[v].z,
                            y[v].w + cor[v].w};
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (4 * c4 + u < a.out_d) o[u] = r[u];
      } else {
        const int64_t orow = a.out_rows ? a.out_rows[j] : j;
        float4* o = reinterpret_cast<float4*>(a.out + orow * DP) + c4;
        float4 r;
        r.x = a.scale * (y[v].x + cor[v].x);
        r.y = a.scale * (y[v].y + cor[v].y);
        r.z = a.scale * (y[v].z + cor[v].z);
        r.w = a.scale * (y[v].w + cor[v].w);
        if (a.accumulate) {
          const float4 old = *o;
          r.x += old.x; r.y += old.y; r.z += old.z; r.w += old.w;
        }
        *o = r;
      }
    }
  }
}

void launch_finalize(const FinalizeArgs& a, cudaStream_t stream) {
  if (a.M == 0) return;
  const int threads = 256;
  const int G = a.Dp / 4 < 32 ? a.Dp / 4 : 32;
  // one wave: 3 resident CTAs per SM (80 registers)
  const unsigned grid = grid_cap(a.M * G, threads, 148 * 3);
  count_launch();
  if (a.ginv) {
    switch (a.Dp) {
      case 16: launch_pdl(finalize_kernel<16, true>, grid, threads, 0, stream, a); break;
      case 32: launch_pdl(finalize_kernel<32, true>, grid, threads, 0, stream, a); break;
      default: break;
    }
    return;
  }
  switch (a.Dp) {
    case 16: launch_pdl(finalize_kernel<16, false>, grid, threads, 0, stream, a); break;
    case 32: launch_pdl(finalize_kernel<32, false>, grid, threads, 0, stream, a); break;
    case 64: launch_pdl(finalize_kernel<64, false>, grid, threads, 0, stream, a); break;
    case 128: launch_pdl(finalize_kernel<128, false>, grid, threads, 0, stream, a); break;
    case 256: launch_pdl(finalize_kernel<256, false>, grid, threads, 0, stream, a); break;
    default: break;
  }
}

// ============================================================================================
// Per-block CSR builder (datasets.py:37-58 partition; matlab/sumac/salsa_loop_cuda.m:143-208
// layout). Input edges are sorted by output row (stable). For a permutation `perm` of the fixed
// rows: pos = perm^-1[i], block = pos / bs, local = pos - block * bs. A stable partition by block
// (one radix pass with per-CTA histograms) keeps the output-row order inside each block, so the
// result is sorted by key = block * M + out_row and is bit-identical from run to run.
// ============================================================================================
static constexpr int CSR_THREADS = 256;
static constexpr int CSR_LONG_GAP = 64;

struct CsrLayout {
  int ncta;
  int64_t chunk;
  size_t off_perm_inv, off_hist, off_totals, off_keys, off_ntask, off_tasks, total;
  int64_t max_tasks;
};

static CsrLayout csr_layout(int64_t m_fixed, int64_t nnz, int num_blocks, int64_t M) {
  CsrLayout L;
  int64_t nc = (nnz + 4095) / 4096;
  if (nc < 1) nc = 1;
  if (nc > 1024) nc = 1024;
  L.ncta = (int)nc;
  L.chunk = (nnz + nc - 1) / nc;
  if (L.chunk < 1) L.chunk = 1;
  auto al = [](size_t x) { return (x + 255) & ~size_t(255); };
  size_t o = 0;
  L.off_perm_inv = o; o = al(o + sizeof(int32_t) * (size_t)(m_fixed > 0 ? m_fixed : 1));
  L.off_hist = o; o = al(o + sizeof(int32_t) * (size_t)num_blocks * L.ncta);
  L.off_totals = o; o = al(o + sizeof(int32_t) * (size_t)num_blocks);
  L.off_keys = o; o = al(o + sizeof(int32_t) * (size_t)(nnz > 0 ? nnz : 1));
  L.off_ntask = o; o = al(o + 16);
  L.max_tasks = ((int64_t)num_blocks * M) / CSR_LONG_GAP + 4;
  L.off_tasks = o; o = al(o + sizeof(int4) * (size_t)L.max_tasks);
  L.total = o;
  return L;
}

size_t csr_workspace_bytes(int64_t m_fixed, int64_t nnz, int num_blocks, int64_t M) {
  return csr_layout(m_fixed, nnz, num_blocks, M).total;
}

__global__ void perm_inv_kernel(const int64_t* __restrict__ perm, int64_t m, int32_t* __restrict__ inv,
                                int* ntask) {
  for (int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; p < m;
       p += (int64_t)gridDim.x * blockDim.x)
    inv[perm[p]] = (int32_t)p;
  if (blockIdx.x == 0 && threadIdx.x == 0) *ntask = 0;
}

// The lanes of the warp holding the same value v (0 <= v < 2^nbits): one ballot per bit (warp
// multisplit). Every lane must call it.
__device__ __forceinline__ unsigned warp_peers(int v, int nbits) {
  unsigned peers = 0xffffffffu;
  for (int i = 0; i < nbits; ++i) {
    const bool bit = (v >> i) & 1;
    const unsigned bal = __ballot_sync(0xffffffffu, bit);
    peers &= bit ? bal : ~bal;
  }
  return peers;
}

// Bits of the block index, with nb itself as the value of a missing edge.
static int csr_block_bits(int nb) { return 32 - __builtin_clz((unsigned)nb); }

__global__ void csr_hist_kernel(const int32_t* __restrict__ e_fixed, int64_t nnz, int64_t chunk,
                                const int32_t* __restrict__ inv, int bs, int nb, int nbits,
                                int32_t* __restrict__ hist) {
  extern __shared__ int sh[];
  for (int k = threadIdx.x; k < nb; k += blockDim.x) sh[k] = 0;
  __syncthreads();
  const int64_t e0 = (int64_t)blockIdx.x * chunk;
  const int64_t e1 = min(nnz, e0 + chunk);
  constexpr int IT = 4;  // edges per thread in flight
  const unsigned lane_lt = (1u << (threadIdx.x & 31)) - 1u;
  for (int64_t rb = e0; rb < e1; rb += (int64_t)blockDim.x * IT) {
    int fx[IT];
#pragma unroll
    for (int j = 0; j < IT; ++j) {
      const int64_t e = rb + (int64_t)j * blockDim.x + threadIdx.x;
      fx[j] = e < e1 ? e_fixed[e] : -1;
    }
#pragma unroll
    for (int j = 0; j < IT; ++j) {
      const int blk = fx[j] >= 0 ? inv[fx[j]] / bs : nb;
      // one shared-memory atomic per distinct block in the warp
      const unsigned peers = warp_peers(blk, nbits);
      if (blk < nb && (peers & lane_lt) == 0) atomicAdd(&sh[blk], __popc(peers));
    }
  }
  __syncthreads();
  for (int k = threadIdx.x; k < nb; k += blockDim.x) hist[(int64_t)k * gridDim.x + blockIdx.x] = sh[k];
}

// Exclusive scan of hist[nb][ncta] in row-major (block-major) order, in two launches: each CTA
// of csr_scan_rows_kernel scans one row k in place (ncta <= 1024 entries, one per thread) and
// writes its total; each CTA of csr_scan_add_kernel adds the sum of the totals of the rows before
// its row (computed by the CTA itself, in a fixed order).
__device__ __forceinline__ int32_t block_exclusive_scan_1024(int32_t v, int32_t* total) {
  __shared__ int32_t wsum[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int32_t incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    const int32_t ws = lane < nw ? wsum[lane] : 0;
    int32_t wi = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t t = __shfl_up_sync(0xffffffffu, wi, o);
      if (lane >= o) wi += t;
    }
    if (lane < nw) wsum[lane] = wi - ws;
    if (lane == 31) *total = wi;
  }
  __syncthreads();
  return wsum[w] + incl - v;
}

__global__ void csr_scan_rows_kernel(int32_t* __restrict__ hist, int ncta,
                                     int32_t* __restrict__ totals) {
  __shared__ int32_t tot;
  int32_t* row = hist + (int64_t)blockIdx.x * ncta;
  const int32_t v = (int)threadIdx.x < ncta ? row[threadIdx.x] : 0;
  const int32_t ex = block_exclusive_scan_1024(v, &tot);
  if ((int)threadIdx.x < ncta) row[threadIdx.x] = ex;
  if (threadIdx.x == 0) totals[blockIdx.x] = tot;
}

__global__ void csr_scan_add_kernel(int32_t* __restrict__ hist, int ncta,
                                    const int32_t* __restrict__ totals) {
  __shared__ int32_t part[32];
  const int k = blockIdx.x;
  int32_t s = 0;
  for (int i = threadIdx.x; i < k; i += blockDim.x) s += totals[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
  __syncthreads();
  int32_t base = 0;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) base += part[w];
  int32_t* row = hist + (int64_t)k * ncta;
  for (int i = threadIdx.x; i < ncta; i += blockDim.x) row[i] += base;
}

// Exclusive scan over the 256 threads of a CTA; *total gets the sum. Two barriers.
__device__ __forceinline__ int block_exclusive_scan_256(int v, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ws = wsum[i];
    before += i < w ? ws : 0;
    all += ws;
  }
  *total = all;
  __syncthreads();  // wsum is reused by the next call
  return before + incl - v;
}

// Stable partition of the edges by block, IT edges per thread per round (256 * IT edges per CTA
// and round). Within a round the edges are ordered item-major (edge rb + j * 256 + t is item j of
// thread t): segment s = j * 8 + warp holds 32 consecutive edges. Warp multisplit gives each
// edge its rank among the segment's edges of its block and the segment's count per block; one
// CTA-wide exclusive scan of the counts in block-major order [block][segment] then gives every
// edge its position behind the block's earlier rounds. Same order (and output) as
// csr_scatter_kernel.
template <int IT>
__global__ void __launch_bounds__(256)
    csr_scatter_tile_kernel(const int32_t* __restrict__ e_fixed, const int32_t* __restrict__ e_out,
                            const float* __restrict__ e_val, int64_t nnz, int64_t chunk,
                            const int32_t* __restrict__ inv, int bs, int nb, int nbits, int64_t M,
                            const int32_t* __restrict__ offs, int32_t* __restrict__ keys,
                            int2* __restrict__ ent) {
  constexpr int S = IT * 8;
  extern __shared__ int sm[];
  int* base = sm;        // [nb] next free position of each block
  int* cnt = sm + nb;    // [nb][S] segment counts, then their exclusive prefix
  __shared__ int wsum[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ns = nb * S;
  const int per = (ns + 255) / 256;  // scan elements per thread (contiguous)
  const int k0 = min(ns, (int)threadIdx.x * per), k1 = min(ns, k0 + per);
  for (int k = threadIdx.x; k < nb; k += blockDim.x) base[k] = offs[(int64_t)k * gridDim.x + blockIdx.x];
  for (int k = threadIdx.x; k < ns; k += blockDim.x) cnt[k] = 0;
  __syncthreads();
  const int64_t e0 = (int64_t)blockIdx.x * chunk;
  const int64_t e1 = min(nnz, e0 + chunk);
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t rb = e0; rb < e1; rb += 256 * IT) {
    int blk[IT], loc[IT], rank[IT];
#pragma unroll
    for (int j = 0; j < IT; ++j) {
      const int64_t e = rb + j * 256 + threadIdx.x;
      blk[j] = e < e1 ? e_fixed[e] : -1;
    }
#pragma unroll
    for (int j = 0; j < IT; ++j) {
      if (blk[j] >= 0) {
        const int pos = inv[blk[j]];
        blk[j] = pos / bs;
        loc[j] = pos - blk[j] * bs;
      } else {
        blk[j] = nb;
        loc[j] = 0;
      }
    }
#pragma unroll
    for (int j = 0; j < IT; ++j) {
      const unsigned peers = warp_peers(blk[j], nbits);
      rank[j] = __popc(peers & lt_mask);
      if (blk[j] < nb && rank[j] == 0) cnt[blk[j] * S + j * 8 + warp] = __popc(peers);
    }
    __syncthreads();
    int tsum = 0;
    for (int k = k0; k < k1; ++k) tsum += cnt[k];
    int total;
    int run = block_exclusive_scan_256(tsum, wsum, &total);
    for (int k = k0; k < k1; ++k) {
      const int v = cnt[k];
      cnt[k] = run;
      run += v;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < IT; ++j) {
      if (blk[j] < nb) {
        const int64_t e = rb + j * 256 + threadIdx.x;
        const int b = blk[j];
        const int pos = base[b] + cnt[b * S + j * 8 + warp] - cnt[b * S] + rank[j];
        keys[pos] = (int32_t)((int64_t)b * M + e_out[e]);
        ent[pos] = make_int2(loc[j], __float_as_int(e_val[e]));
      }
    }
    // the blocks' new bases (read before any thread rewrites base or cnt)
    int nbase[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int b = threadIdx.x + q * 256;
      nbase[q] = b < nb ? base[b] + (b + 1 < nb ? cnt[(b + 1) * S] : total) - cnt[b * S] : 0;
    }
    __syncthreads();
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int b = threadIdx.x + q * 256;
      if (b < nb) base[b] = nbase[q];
    }
    for (int k = k0; k < k1; ++k) cnt[k] = 0;
    __syncthreads();
  }
}

// Exclusive scan over the 1024 threads of a CTA; *total gets the sum.
__device__ __forceinline__ int block_exclusive_scan_1024i(int v, int* wsum, int* total) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  int incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int t = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += t;
  }
  if (lane == 31) wsum[w] = incl;
  __syncthreads();
  if (w == 0) {
    const int ws = wsum[lane];
    int x = ws;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, x, o);
      if (lane >= o) x += t;
    }
    wsum[lane] = x - ws;
    if (lane == 31) wsum[32] = x;
  }
  __syncthreads();
  const int r = wsum[w] + incl - v;
  *total = wsum[32];
  __syncthreads();  // wsum is reused by the next call
  return r;
}

// Stable partition by block with the output staged in shared memory: per round of 8192 edges
// (1024 threads x 8), warp w takes 256 consecutive edges (item-major) and ranks each within its
// span and block (warp multisplit plus the warp's running count per block); one CTA-wide scan of
// the [block][warp] counts orders the round by block, the round's (key, entry) pairs are written
// to shared memory in that order, and then copied out so that consecutive threads write
// consecutive positions of each block's run: coalesced stores, where the scatter kernels above
// write 12-byte pieces into ~100 regions per round. Same output as csr_scatter_kernel.
constexpr int CSR_STAGE_IT = 8;
constexpr int CSR_STAGE_ROUND = 1024 * CSR_STAGE_IT;
static size_t csr_stage_smem(int nb) {
  return (size_t)CSR_STAGE_ROUND * (sizeof(int2) + sizeof(int32_t)) +
         (size_t)(1 + 32 + 32 + 1) * nb * sizeof(int) + 64 * sizeof(int);
}

__global__ void __launch_bounds__(1024, 1)
    csr_scatter_stage_kernel(const int32_t* __restrict__ e_fixed, const int32_t* __restrict__ e_out,
                             const float* __restrict__ e_val, int64_t nnz, int64_t chunk,
                             const int32_t* __restrict__ inv, int bs, int nb, int nbits, int64_t M,
                             const int32_t* __restrict__ offs, int32_t* __restrict__ keys,
                             int2* __restrict__ ent) {
  extern __shared__ __align__(16) uint8_t smraw[];
  int2* sent = reinterpret_cast<int2*>(smraw);                       // [ROUND]
  int* skey = reinterpret_cast<int*>(sent + CSR_STAGE_ROUND);        // [ROUND]
  int* base = skey + CSR_STAGE_ROUND;                                // [nb]
  int* wcnt = base + nb;                                             // [32][nb]
  int* pre = wcnt + 32 * nb;                                         // [nb][32]
  int* off = pre + 32 * nb;                                          // [nb + 1]
  int* wsum = off + nb + 1;                                          // [33]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int k = threadIdx.x; k < nb; k += blockDim.x) base[k] = offs[(int64_t)k * gridDim.x + blockIdx.x];
  const int64_t e0 = (int64_t)blockIdx.x * chunk;
  const int64_t e1 = min(nnz, e0 + chunk);
  const unsigned lt_mask = (1u << lane) - 1u;
  const int ns = nb * 32;
  const int per = (ns + 1023) / 1024;
  const int q0 = min(ns, (int)threadIdx.x * per), q1 = min(ns, q0 + per);
  for (int64_t rb = e0; rb < e1; rb += CSR_STAGE_ROUND) {
    for (int k = lane; k < nb; k += 32) wcnt[warp * nb + k] = 0;
    __syncwarp();
    int blk[CSR_STAGE_IT], loc[CSR_STAGE_IT], rnk[CSR_STAGE_IT];
#pragma unroll
    for (int j = 0; j < CSR_STAGE_IT; ++j) {
      const int64_t e = rb + warp * (32 * CSR_STAGE_IT) + j * 32 + lane;
      blk[j] = e < e1 ? e_fixed[e] : -1;
    }
#pragma unroll
    for (int j = 0; j < CSR_STAGE_IT; ++j) {
      if (blk[j] >= 0) {
        const int pos = inv[blk[j]];
        blk[j] = pos / bs;
        loc[j] = pos - blk[j] * bs;
      } else {
        blk[j] = nb;
        loc[j] = 0;
      }
    }
#pragma unroll
    for (int j = 0; j < CSR_STAGE_IT; ++j) {
      const unsigned peers = warp_peers(blk[j], nbits);
      const int rank = __popc(peers & lt_mask);
      const int run = blk[j] < nb ? wcnt[warp * nb + blk[j]] : 0;
      rnk[j] = run + rank;
      __syncwarp();
      if (blk[j] < nb && rank == 0) wcnt[warp * nb + blk[j]] = run + __popc(peers);
      __syncwarp();
    }
    __syncthreads();
    // exclusive scan of the counts in [block][warp] order
    int tsum = 0;
    for (int q = q0; q < q1; ++q) tsum += wcnt[(q & 31) * nb + (q >> 5)];
    int total;
    int run = block_exclusive_scan_1024i(tsum, wsum, &total);
    for (int q = q0; q < q1; ++q) {
      pre[q] = run;
      run += wcnt[(q & 31) * nb + (q >> 5)];
    }
    __syncthreads();
    for (int k = threadIdx.x; k < nb; k += blockDim.x) off[k] = pre[k * 32];
    if (threadIdx.x == 0) off[nb] = total;
#pragma unroll
    for (int j = 0; j < CSR_STAGE_IT; ++j) {
      if (blk[j] < nb) {
        const int64_t e = rb + warp * (32 * CSR_STAGE_IT) + j * 32 + lane;
        const int sp = pre[blk[j] * 32 + warp] + rnk[j];
        skey[sp] = (int32_t)((int64_t)blk[j] * M + e_out[e]);
        sent[sp] = make_int2(loc[j], __float_as_int(e_val[e]));
      }
    }
    __syncthreads();
    for (int t = threadIdx.x; t < total; t += blockDim.x) {
      int lo = 0, hi = nb;  // the block b with off[b] <= t < off[b + 1]
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (off[mid] <= t) lo = mid; else hi = mid;
      }
      const int gp = base[lo] + t - off[lo];
      keys[gp] = skey[t];
      ent[gp] = sent[t];
    }
    __syncthreads();
    for (int k = threadIdx.x; k < nb; k += blockDim.x) base[k] += off[k + 1] - off[k];
    __syncthreads();
  }
}

__global__ void csr_scatter_kernel(const int32_t* __restrict__ e_fixed, const int32_t* __restrict__ e_out,
                                   const float* __restrict__ e_val, int64_t nnz, int64_t chunk,
                                   const int32_t* __restrict__ inv, int bs, int nb, int64_t M,
                                   const int32_t* __restrict__ offs, int32_t* __restrict__ keys,
                                   int2* __restrict__ ent) {
  extern __shared__ int sm[];
  int* base = sm;            // [nb]
  int* wcnt = sm + nb;       // [8][nb]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int k = threadIdx.x; k < nb; k += blockDim.x) base[k] = offs[(int64_t)k * gridDim.x + blockIdx.x];
  for (int k = threadIdx.x; k < 8 * nb; k += blockDim.x) wcnt[k] = 0;
  __syncthreads();
  const int64_t e0 = (int64_t)blockIdx.x * chunk;
  const int64_t e1 = min(nnz, e0 + chunk);
  const unsigned lt_mask = (1u << lane) - 1u;
  for (int64_t rb = e0; rb < e1; rb += CSR_THREADS) {
    const int64_t e = rb + threadIdx.x;
    const bool valid = e < e1;
    int blk = 0x7fffffff, loc = 0;
    if (valid) {
      const int pos = inv[e_fixed[e]];
      blk = pos / bs;
      loc = pos - blk * bs;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, blk);
    const int rank = __popc(peers & lt_mask);
    const int cnt = __popc(peers);
    if (valid && rank == 0) wcnt[warp * nb + blk] = cnt;
    __syncthreads();
    if (valid) {
      int pos = base[blk] + rank;
      for (int w = 0; w < warp; ++w) pos += wcnt[w * nb + blk];
      keys[pos] = (int32_t)((int64_t)blk * M + e_out[e]);
      ent[pos] = make_int2(loc, __float_as_int(e_val[e]));
    }
    __syncthreads();
    if (valid && rank == 0) {
      atomicAdd(&base[blk], cnt);
      wcnt[warp * nb + blk] = 0;
    }
    __syncthreads();
  }
}

// rowptr[q] = first sorted position whose key >= q, for q in [0, nb*M]. Gaps longer than
// CSR_LONG_GAP are queued as tasks and filled by csr_fill_tasks_kernel (one CTA per task).
__global__ void csr_rowptr_kernel(const int32_t* __restrict__ keys, int64_t nnz, int64_t nkeys,
                                  int32_t* __restrict__ rowptr, int* ntask, int4* tasks,
                                  int64_t max_tasks) {
  const int64_t p = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  auto fill = [&](int64_t lo, int64_t hi, int32_t val) {  // rowptr[lo..hi] = val (inclusive)
    if (hi < lo) return;
    if (hi - lo + 1 <= CSR_LONG_GAP) {
      for (int64_t q = lo; q <= hi; ++q) rowptr[q] = val;
    } else {
      const int t = atomicAdd(ntask, 1);
      if (t < max_tasks) tasks[t] = make_int4((int)lo, (int)hi, val, 0);
    }
  };
  if (nnz == 0) {
    if (p == 0) fill(0, nkeys, 0);
    return;
  }
  if (p >= nnz) return;
  const int64_t k = keys[p];
  const int64_t kp = p == 0 ? -1 : keys[p - 1];
  fill(kp + 1, k, (int32_t)p);
  if (p == nnz - 1) fill(k + 1, nkeys, (int32_t)nnz);
}

// The same with four consecutive edges per thread (one 16-byte load of keys) and a grid-stride
// loop over a grid sized to the GPU, for large nnz (keys must be 16-byte aligned).
__global__ void __launch_bounds__(256) csr_rowptr4_kernel(const int32_t* __restrict__ keys,
                                                          int64_t nnz, int64_t nkeys,
                                                          int32_t* __restrict__ rowptr, int* ntask,
                                                          int4* tasks, int64_t max_tasks) {
  auto fill = [&](int64_t lo, int64_t hi, int32_t val) {  // rowptr[lo..hi] = val (inclusive)
    if (hi < lo) return;
    if (hi - lo + 1 <= CSR_LONG_GAP) {
      for (int64_t q = lo; q <= hi; ++q) rowptr[q] = val;
    } else {
      const int t = atomicAdd(ntask, 1);
      if (t < max_tasks) tasks[t] = make_int4((int)lo, (int)hi, val, 0);
    }
  };
  const int64_t nq = (nnz + 3) / 4;
  for (int64_t q = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; q < nq;
       q += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p0 = 4 * q;
    int k[4];
    if (p0 + 3 < nnz) {
      const int4 v = reinterpret_cast<const int4*>(keys)[q];
      k[0] = v.x; k[1] = v.y; k[2] = v.z; k[3] = v.w;
    } else {
      for (int u = 0; u < 4; ++u) k[u] = p0 + u < nnz ? keys[p0 + u] : 0;
    }
    int64_t prev = p0 == 0 ? -1 : keys[p0 - 1];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int64_t p = p0 + u;
      if (p < nnz) {
        fill(prev + 1, k[u], (int32_t)p);
        if (p == nnz - 1) fill((int64_t)k[u] + 1, nkeys, (int32_t)nnz);
        prev = k[u];
      }
    }
  }
}

__global__ void csr_fill_tasks_kernel(const int* ntask, const int4* tasks, int64_t max_tasks,
                                      int32_t* __restrict__ rowptr) {
  const int nt = (int)min((int64_t)*ntask, max_tasks);
  for (int t = blockIdx.x; t < nt; t += gridDim.x) {
    const int4 tk = tasks[t];
    for (int64_t q = (int64_t)tk.x + threadIdx.x; q <= tk.y; q += blockDim.x) rowptr[q] = tk.z;
  }
}

int launch_block_csr(const int64_t* perm, int64_t m_fixed, int num_blocks, const int32_t* e_fixed,
                     const int32_t* e_out, const float* e_val, int64_t nnz, int64_t M,
                     int32_t* rowptr, int2* ent, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const CsrLayout L = csr_layout(m_fixed, nnz, num_blocks, M);
  if (ws_bytes < L.total) return -2;
  if ((int64_t)num_blocks * M >= (int64_t)INT32_MAX || nnz >= (int64_t)INT32_MAX) return -3;
  if (num_blocks > 4096 || num_blocks < 1) return -4;
  uint8_t* w = static_cast<uint8_t*>(ws);
  int32_t* inv = reinterpret_cast<int32_t*>(w + L.off_perm_inv);
  int32_t* hist = reinterpret_cast<int32_t*>(w + L.off_hist);
  int32_t* totals = reinterpret_cast<int32_t*>(w + L.off_totals);
  int32_t* keys = reinterpret_cast<int32_t*>(w + L.off_keys);
  int* ntask = reinterpret_cast<int*>(w + L.off_ntask);
  int4* tasks = reinterpret_cast<int4*>(w + L.off_tasks);
  const int bs = (int)((m_fixed + num_blocks - 1) / num_blocks);
  count_launch();
  perm_inv_kernel<<<grid_cap(m_fixed, 256, 148 * 8), 256, 0, stream>>>(perm, m_fixed, inv, ntask);
  if (nnz > 0) {
    const int nbits = csr_block_bits(num_blocks);
    count_launch();
    csr_hist_kernel<<<L.ncta, CSR_THREADS, num_blocks * sizeof(int), stream>>>(
        e_fixed, nnz, L.chunk, inv, bs, num_blocks, nbits, hist);
    count_launch();
    csr_scan_rows_kernel<<<num_blocks, 1024, 0, stream>>>(hist, L.ncta, totals);
    count_launch();
    csr_scan_add_kernel<<<num_blocks, 256, 0, stream>>>(hist, L.ncta, totals);
    // four (one) edges per thread per round while the block table fits in 48 KB of shared memory
    // (up to 1024 blocks: the new bases are formed four per thread)
    const size_t smem4 = (size_t)(1 + 32) * num_blocks * sizeof(int);
    const size_t smem1 = (size_t)(1 + 8) * num_blocks * sizeof(int);
    const size_t smem_st = csr_stage_smem(num_blocks);
    if (smem_st <= 200 * 1024) {
      // largest opt-in so far per device (set on the first, eager, call of a shape)
      static int stage_smem_set[64] = {};
      int dev = 0;
      cudaGetDevice(&dev);
      if (dev < 0 || dev >= 64 || (int)smem_st > stage_smem_set[dev]) {
        cudaFuncSetAttribute(csr_scatter_stage_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)smem_st);
        if (dev >= 0 && dev < 64) stage_smem_set[dev] = (int)smem_st;
      }
      count_launch();
      csr_scatter_stage_kernel<<<L.ncta, 1024, smem_st, stream>>>(
          e_fixed, e_out, e_val, nnz, L.chunk, inv, bs, num_blocks, nbits, M, hist, keys, ent);
      goto scattered;
    }
    if (smem4 <= 48 * 1024) {
      count_launch();
      csr_scatter_tile_kernel<4><<<L.ncta, CSR_THREADS, smem4, stream>>>(
          e_fixed, e_out, e_val, nnz, L.chunk, inv, bs, num_blocks, nbits, M, hist, keys, ent);
      goto scattered;
    }
    if (smem1 <= 48 * 1024 && num_blocks <= 1024) {
      count_launch();
      csr_scatter_tile_kernel<1><<<L.ncta, CSR_THREADS, smem1, stream>>>(
          e_fixed, e_out, e_val, nnz, L.chunk, inv, bs, num_blocks, nbits, M, hist, keys, ent);
      goto scattered;
    }
    {
    const size_t smem = (size_t)9 * num_blocks * sizeof(int);
    static int scatter_smem_set = 0;  // largest opt-in so far (set eagerly before any capture)
    if (smem > 48 * 1024 && (int)smem > scatter_smem_set) {
      cudaFuncSetAttribute(csr_scatter_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      scatter_smem_set = (int)smem;
    }
    count_launch();
    csr_scatter_kernel<<<L.ncta, CSR_THREADS, smem, stream>>>(e_fixed, e_out, e_val, nnz, L.chunk,
                                                             inv, bs, num_blocks, M, hist, keys, ent);
    }
  scattered:;
  }
  const int64_t nkeys = (int64_t)num_blocks * M;
  count_launch();
  if (nnz >= 4 * 148 * 256)
    csr_rowptr4_kernel<<<grid_cap((nnz + 3) / 4, 256, 148 * 16), 256, 0, stream>>>(
        keys, nnz, nkeys, rowptr, ntask, tasks, L.max_tasks);
  else
    csr_rowptr_kernel<<<grid_cap(nnz > 0 ? nnz : 1, 256, INT32_MAX), 256, 0, stream>>>(
        keys, nnz, nkeys, rowptr, ntask, tasks, L.max_tasks);
  count_launch();
  csr_fill_tasks_kernel<<<148 * 2, 256, 0, stream>>>(ntask, tasks, L.max_tasks, rowptr);
  return (int)cudaGetLastError();
}

// ============================================================================================
// metric / loss terms on the support (eval.py:24-36), fp64 accumulation
// ============================================================================================
static constexpr int TERMS = 6;

__device__ __forceinline__ void block_reduce_terms(double (&t)[TERMS], double* out) {
  __shared__ double sh[TERMS][8];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < TERMS; ++k) {
    double v = t[k];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) sh[k][w] = v;
  }
  __syncthreads();
  if (threadIdx.x < TERMS) {
    double s = 0.0;
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) s += sh[threadIdx.x][i];
    out[blockIdx.x * TERMS + threadIdx.x] = s;
  }
}

__device__ __forceinline__ void add_terms(double (&t)[TERMS], double L, double v) {
  const double Mv = L > 0.0 ? L : 0.0;
  t[0] += Mv * Mv;
  t[1] += (v - Mv) * (v - Mv);
  t[2] += (v - L) * (v - L);
  t[3] += v < Mv ? v : Mv;
  t[4] += v;
  t[5] += v * v;
}

int sparse_terms_grid(int64_t n) { return (int)grid_cap(n, 256, 148 * 4); }

__global__ void sparse_terms_coo_kernel(const float* __restrict__ A, const float* __restrict__ B, int Dp,
                                        const int32_t* __restrict__ ei, const int32_t* __restrict__ ej,
                                        const float* __restrict__ v, int64_t nnz, double* partials) {
  double t[TERMS] = {0, 0, 0, 0, 0, 0};
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float4* a = reinterpret_cast<const float4*>(A + (int64_t)ei[e] * Dp);
    const float4* b = reinterpret_cast<const float4*>(B + (int64_t)ej[e] * Dp);
    double L = 0.0;
    for (int c = 0; c < Dp / 4; ++c) {
      const float4 x = a[c], y = b[c];
      L += (double)x.x * y.x + (double)x.y * y.y + (double)x.z * y.z + (double)x.w * y.w;
    }
    add_terms(t, L, (double)v[e]);
  }
  block_reduce_terms(t, partials);
}

void launch_sparse_terms_coo(const float* A, const float* B, int Dp, const int32_t* ei,
                             const int32_t* ej, const float* v, int64_t nnz, double* partials,
                             int grid, cudaStream_t stream) {
  count_launch();
  sparse_terms_coo_kernel<<<grid, 256, 0, stream>>>(A, B, Dp, ei, ej, v, nnz, partials);
}

__global__ void sparse_terms_csr_kernel(const float* __restrict__ X, const float* __restrict__ F, int Dp,
                                        const int32_t* __restrict__ rowptr, int64_t M,
                                        const int2* __restrict__ ent, double* partials) {
  double t[TERMS] = {0, 0, 0, 0, 0, 0};
  for (int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; j < M;
       j += (int64_t)gridDim.x * blockDim.x) {
    const float4* x = reinterpret_cast<const float4*>(X + j * Dp);
    for (int e = rowptr[j]; e < rowptr[j + 1]; ++e) {
      const int2 en = ent[e];
      const float4* f = reinterpret_cast<const float4*>(F + (int64_t)en.x * Dp);
      double L = 0.0;
      for (int c = 0; c < Dp / 4; ++c) {
        const float4 a = x[c], b = f[c];
        L += (double)a.x * b.x + (double)a.y * b.y + (double)a.z * b.z + (double)a.w * b.w;
      }
      add_terms(t, L, (double)__int_as_float(en.y));
    }
  }
  block_reduce_terms(t, partials);
}

void launch_sparse_terms_csr(const float* X, const float* F, int Dp, const int32_t* rowptr,
                             int64_t M, const int2* ent, double* partials, int grid,
                             cudaStream_t stream) {
  count_launch();
  sparse_terms_csr_kernel<<<grid, 256, 0, stream>>>(X, F, Dp, rowptr, M, ent, partials);
}

__global__ void sum_partials_kernel(const double* __restrict__ partials, int n, int w,
                                    double* __restrict__ out, int accumulate) {
  const int k = threadIdx.x;
  if (k >= w) return;
  double s = 0.0;
  for (int i = 0; i < n; ++i) s += partials[(int64_t)i * w + k];
  out[k] = accumulate ? out[k] + s : s;
}

void launch_sum_partials(const double* partials, int n, int w, double* out, int accumulate,
                         cudaStream_t stream) {
  count_launch();
  sum_partials_kernel<<<1, 32, 0, stream>>>(partials, n, w, out, accumulate);
}

// ============================================================================================
// initial factors (training/salsa.py:36-78): out_r = sign sqrt(sum_e val_e R[col_e]) over the
// entries e of row r (rows sorted, rowptr), i.e. sign sqrt(S R) row by row; and the three sums of
// the closed-form scale: sum v^2, sum v L, sum L^2 with L_e = <A_i, B_j> over the entries (i, j, v)
// ============================================================================================
__global__ void __launch_bounds__(256) init_spmm_sqrt_kernel(const int32_t* __restrict__ rowptr,
                                                             const int32_t* __restrict__ col,
                                                             const float* __restrict__ val, int64_t M,
                                                             const float* __restrict__ R, int d,
                                                             float sign, float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t w0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t nw = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t r = w0; r < M; r += nw) {
    const int e0 = rowptr[r], e1 = rowptr[r + 1];
    for (int c0 = 0; c0 < d; c0 += 32) {
      const int c = c0 + lane;
      const bool on = c < d;
      float acc = 0.f;
      int e = e0;
      for (; e + 4 <= e1; e += 4) {
        int j[4];
        float v[4], x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) { j[u] = col[e + u]; v[u] = val[e + u]; }
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = on ? R[(int64_t)j[u] * d + c] : 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) acc = fmaf(v[u], x[u], acc);
      }
      for (; e < e1; ++e) acc = fmaf(val[e], on ? R[(int64_t)col[e] * d + c] : 0.f, acc);
      if (on) out[r * d + c] = sign * sqrtf(acc);
    }
  }
}

constexpr int INIT_SCALE_GRID = 148 * 4;

__global__ void __launch_bounds__(256) init_scale_terms_kernel(
    const float* __restrict__ A, const float* __restrict__ B, int d, const int32_t* __restrict__ ei,
    const int32_t* __restrict__ ej, const float* __restrict__ v, int64_t nnz,
    double* __restrict__ partials) {
  double s_vv = 0.0, s_vl = 0.0, s_ll = 0.0;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < nnz;
       e += (int64_t)gridDim.x * blockDim.x) {
    const float* a = A + (int64_t)ei[e] * d;
    const float* b = B + (int64_t)ej[e] * d;
    float L = 0.f;
#pragma unroll 4
    for (int k = 0; k < d; ++k) L = fmaf(a[k], b[k], L);
    const double x = v[e], l = L;
    s_vv += x * x;
    s_vl += x * l;
    s_ll += l * l;
  }
  __shared__ double red[3][8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s_vv += __shfl_xor_sync(0xffffffffu, s_vv, o);
    s_vl += __shfl_xor_sync(0xffffffffu, s_vl, o);
    s_ll += __shfl_xor_sync(0xffffffffu, s_ll, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s_vv;
    red[1][threadIdx.x >> 5] = s_vl;
    red[2][threadIdx.x >> 5] = s_ll;
  }
  __syncthreads();
  if (threadIdx.x < 3) {
    double t = 0.0;
    for (int w = 0; w < 8; ++w) t += red[threadIdx.x][w];
    partials[(int64_t)blockIdx.x * 3 + threadIdx.x] = t;
  }
}

void launch_init_spmm_sqrt(const int32_t* rowptr, const int32_t* col, const float* val, int64_t M,
                           const float* R, int d, float sign, float* out, cudaStream_t stream) {
  if (M <= 0) return;
  count_launch();
  init_spmm_sqrt_kernel<<<grid_cap(M * 32, 256, 148 * 8), 256, 0, stream>>>(rowptr, col, val, M, R,
                                                                            d, sign, out);
}

size_t init_scale_workspace_bytes() { return (size_t)INIT_SCALE_GRID * 3 * sizeof(double); }

void launch_init_scale_terms(const float* A, const float* B, int d, const int32_t* ei,
                             const int32_t* ej, const float* v, int64_t nnz, double* partials,
                             double* out, cudaStream_t stream) {
  count_launch();
  init_scale_terms_kernel<<<INIT_SCALE_GRID, 256, 0, stream>>>(A, B, d, ei, ej, v, nnz, partials);
  launch_sum_partials(partials, INIT_SCALE_GRID, 3, out, 0, stream);
}

// ============================================================================================
// optimizers (training/gd.py:20-46 through torch.optim)
// ============================================================================================
__global__ void adam_kernel(float* __restrict__ p, const float* __restrict__ g, float* __restrict__ m,
                            float* __restrict__ v, int64_t n, float lr_over_bc1, float inv_sqrt_bc2,
                            float beta1, float beta2, float eps) {
  const float w1 = 1.0f - beta1, w2 = 1.0f - beta2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i];
    float mi = m[i];
    mi = mi + w1 * (gi - mi);                // lerp(m, g, 1 - beta1)
    float vi = v[i] * beta2;
    vi = fmaf(w2 * gi, gi, vi);              // v * beta2 + (1 - beta2) g g
    const float denom = sqrtf(vi) * inv_sqrt_bc2 + eps;
    p[i] = p[i] - lr_over_bc1 * (mi / denom);
    m[i] = mi;
    v[i] = vi;
  }
}

void launch_adam(float* p, const float* g, float* m, float* v, int64_t n, float lr_over_bc1,
                 float inv_sqrt_bc2, float beta1, float beta2, float eps, cudaStream_t stream) {
  if (n == 0) return;
  count_launch();
  adam_kernel<<<grid_cap(n, 256, 148 * 16), 256, 0, stream>>>(p, g, m, v, n, lr_over_bc1,
                                                               inv_sqrt_bc2, beta1, beta2, eps);
}

__global__ void fill_zero_kernel(float* __restrict__ p, int64_t n) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = 0.f;
}

void launch_fill_zero(float* p, int64_t n, cudaStream_t stream) {
  if (n == 0) return;
  count_launch();
  fill_zero_kernel<<<grid_cap(n, 256, 148 * 16), 256, 0, stream>>>(p, n);
}

__global__ void sumsq_kernel(const float* __restrict__ g, int64_t n, double* out) {
  double s = 0.0;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    s += (double)g[i] * g[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) atomicAdd(out, s);
}

void launch_sumsq(const float* g, int64_t n, double* out, cudaStream_t stream) {
  if (n == 0) return;
  count_launch();
  sumsq_kernel<<<grid_cap(n, 256, 148 * 4), 256, 0, stream>>>(g, n, out);
}

// torch.nn.utils.clip_grad_norm_(max_norm) then torch.optim.SGD(momentum, dampening 0)
__global__ void sgd_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ buf,
                           int64_t n, float lr, float momentum, int first, const double* sumsq,
                           float max_norm) {
  float coef = 1.f;
  if (sumsq) {
    const float total = (float)sqrt(*sumsq);
    const float c = max_norm / (total + 1e-6f);
    coef = c < 1.f ? c : 1.f;
  }
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    const float gi = g[i] * coef;
    float b = gi;
    if (momentum != 0.f) {
      b = first ? gi : fmaf(momentum, buf[i], gi);
      buf[i] = b;
    }
    p[i] = p[i] - lr * b;
  }
}

void launch_sgd(float* p, float* g, float* buf, int64_t n, float lr, float momentum, int first,
                const double* sumsq, float max_norm, cudaStream_t stream) {
  if (n == 0) return;
  count_launch();
  sgd_kernel<<<grid_cap(n, 256, 148 * 16), 256, 0, stream>>>(p, g, buf, n, lr, momentum, first,
                                                              sumsq, max_norm);
}

// ============================================================================================
// bounded wait on a flag nobody sets: exercises the timeout path without faulting the GPU
// ============================================================================================
__global__ void wait_flag_kernel(const volatile int* flag, int* err, unsigned long long timeout_ns) {
  const uint64_t t0 = globaltimer_ns();
  while (*flag == 0) {
    if (globaltimer_ns() - t0 > timeout_ns) {
      atomicCAS(err, 0, DEV_TIMEOUT_FLAG);
      return;
    }
  }
}

void launch_wait_flag(const int* flag, int* err, unsigned long long timeout_ns, cudaStream_t s) {
  count_launch();
  wait_flag_kernel<<<1, 1, 0, s>>>(flag, err, timeout_ns);
}

// ============================================================================================
// Rows of a row-sharded factor: out[p] = local[rows[p] - lo] when this rank owns rows[p]
// (lo <= rows[p] < hi), zero otherwise; one float4 per thread. An allreduce(sum) over the ranks
// then completes the block rows exactly (one nonzero term per element).
// ============================================================================================
__global__ void gather_owned_rows_kernel(const float* __restrict__ local, int64_t lo, int64_t hi,
                                         const int64_t* __restrict__ rows, int64_t nrows, int Dp,
                                         float* __restrict__ out) {
  const int q4 = Dp / 4;
  const int64_t total = nrows * q4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = i / q4;
    const int c4 = (int)(i - p * q4);
    const int64_t r = rows[p];
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r >= lo && r < hi) v = reinterpret_cast<const float4*>(local + (r - lo) * Dp)[c4];
    reinterpret_cast<float4*>(out)[i] = v;
  }
}

// Row exchange of the row-sharded SALSA step over NVLink peer memory: every rank stores the block
// rows it owns (rows[p] in [lo, hi)) into slot (epoch & 1) of every rank's buffer (itself
// included; each row has exactly one owner, so the slot is complete once all ranks have written),
// then sets its flag in every rank's flag array to the new epoch (release, system scope) and waits
// (acquire, bounded) until every rank's flag in its own array has reached it. One CTA. Slot reuse:
// a peer writes slot s for exchange e only after passing exchange e - 1, for which this rank
// signalled only once everything it had enqueued before exchange e - 1 (the readers of slot s from
// exchange e - 2) had completed.
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(512) assemble_rows_p2p_kernel(
    const float* __restrict__ local, int64_t lo, int64_t hi, const int64_t* __restrict__ rows,
    int64_t nrows, int Dp, int64_t slot_floats, float* const* __restrict__ peer_bufs,
    unsigned* const* __restrict__ peer_flags, unsigned* epoch, int rank, int world, int* err,
    unsigned long long timeout_ns) {
  const unsigned ep = *epoch + 1u;
  const int64_t slot_off = (int64_t)(ep & 1u) * slot_floats;
  const int v4 = Dp / 4;
  for (int64_t e = threadIdx.x; e < nrows * v4; e += blockDim.x) {
    const int64_t p = e / v4;
    const int v = (int)(e - p * v4);
    const int64_t g = rows[p];
    if (g >= lo && g < hi) {
      const float4 val = reinterpret_cast<const float4*>(local)[(g - lo) * v4 + v];
      for (int q = 0; q < world; ++q)
        reinterpret_cast<float4*>(peer_bufs[q] + slot_off)[p * v4 + v] = val;
    }
  }
  __threadfence_system();
  __syncthreads();
  if ((int)threadIdx.x < world) {
    st_release_sys(peer_flags[threadIdx.x] + rank, ep);
    const unsigned* mine = peer_flags[rank] + threadIdx.x;
    const uint64_t t0 = globaltimer_ns();
    while ((int)(ld_acquire_sys(mine) - ep) < 0) {
      if (globaltimer_ns() - t0 > timeout_ns) {
        if (err) atomicCAS(err, 0, DEV_TIMEOUT_PEER);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) *epoch = ep;
}

void launch_assemble_rows_p2p(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                              int64_t nrows, int Dp, int64_t slot_floats, float* const* peer_bufs,
                              unsigned* const* peer_flags, unsigned* epoch, int rank, int world,
                              int* err, unsigned long long timeout_ns, cudaStream_t stream) {
  count_launch();
  assemble_rows_p2p_kernel<<<1, 512, 0, stream>>>(local, lo, hi, rows, nrows, Dp, slot_floats,
                                                   peer_bufs, peer_flags, epoch, rank, world, err,
                                                   timeout_ns);
}

void launch_gather_owned_rows(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                              int64_t nrows, int Dp, float* out, cudaStream_t stream) {
  if (nrows <= 0) return;
  count_launch();
  gather_owned_rows_kernel<<<grid_cap(nrows * (Dp / 4), 256, 148 * 4), 256, 0, stream>>>(
      local, lo, hi, rows, nrows, Dp, out);
}

}  // namespace sb
