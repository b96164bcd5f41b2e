// product.cu — tensor maps, the (Dp, precision) configuration table and launchers of the fused
// ReLU product / reduce kernel (relu_product.cuh).
#include <cstring>

#include "kernels.cuh"
#include "relu_product.cuh"

namespace sb {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 2-D fp32 map over a row-major [rows][inner] array with `ld` floats per row. Out-of-range boxes
// read as zero.
static bool make_map(CUtensorMap* m, const float* base, uint64_t inner, uint64_t rows, uint64_t ld,
                     uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t gdim[2] = {inner, rows};
  cuuint64_t gstride[1] = {ld * sizeof(float)};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estride[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), gdim, gstride,
                  box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

struct ProdCfgRt {
  int bn, stages, g;  // chunk rows, pipeline stages, row tiles per group
  bool ok;
  bool simt = false;  // fp32 CUDA-core kernel (relu_simt_kernel) instead of tcgen05
};

// Per (Dp, precision): the TMEM budget is NBUF * BN (x2 for 3xTF32) S columns plus G * Dp Y
// columns <= 512; shared memory holds G X slots and the stages.
static ProdCfgRt product_cfg(int Dp, bool x3) {
  // TMEM: (MS sets of) G Dp Y columns + NBUF S buffers of BN columns within 512 columns
  if (!x3) {
    switch (Dp) {
      case 16: return {128, 4, 8, true};
      case 32: return {128, 3, 4, true};
      case 64: return {128, 2, 1, true};
      case 128: return {64, 2, 1, true};
      case 256: return {32, 1, 1, true};  // tf32 second MMA (no room for an fp16 C copy)
    }
  } else {
    switch (Dp) {
      case 16: return {64, 4, 8, true};
      case 32: return {64, 2, 4, true};
      case 64: return {64, 2, 1, true};
      case 128: return {32, 1, 1, true};
      // a 128-row X tile in hi + lo halves is 256 KB at Dp = 256: more than shared memory
      case 256: return {0, 0, 0, true, true};
    }
  }
  return {0, 0, 0, false};
}

static ProdCfgRt reduce_cfg(int Dp, bool x3) {
  if (!x3) {
    switch (Dp) {
      case 16: return {128, 6, 8, true};
      case 32: return {128, 4, 8, true};
      case 64: return {128, 3, 4, true};
      case 128: return {64, 2, 2, true};
      case 256: return {32, 2, 1, true};
    }
  } else {
    switch (Dp) {
      case 16: return {128, 4, 8, true};
      case 32: return {128, 3, 4, true};
      case 64: return {64, 3, 2, true};
      case 128: return {32, 2, 1, true};
      case 256: return {0, 0, 0, true, true};
    }
  }
  return {0, 0, 0, false};
}

bool product_supported(int Dp, bool x3) { return product_cfg(Dp, x3).ok; }
bool reduce_supported(int Dp, bool x3) { return reduce_cfg(Dp, x3).ok; }

// Work plan. With fewer row tiles than SMs: one tile per group and split-K over the chunk range
// so that every SM gets work (at least ~4 chunks per split, no empty split). Otherwise: no
// split, and the tiles are cut into balanced contiguous groups of at most G tiles, as many
// groups as fill whole rounds of the persistent grid.
static void plan_work(int64_t M, int64_t N, int bn, int G, int num_sms, ProductParams* p) {
  const int64_t tiles = (M + 127) / 128;
  const int64_t nc = (N + bn - 1) / bn;
  int64_t s = 1, groups = tiles;
  if (tiles < num_sms) {
    s = (num_sms + tiles - 1) / tiles;
    int64_t max_s = nc / 4;
    if (max_s < 1) max_s = 1;
    if (s > max_s) s = max_s;
  } else {
    const int64_t need = (tiles + G - 1) / G;
    const int64_t rounds = (need + num_sms - 1) / num_sms;
    groups = rounds * num_sms < tiles ? rounds * num_sms : tiles;
  }
  int64_t c = (nc + s - 1) / s;
  s = (nc + c - 1) / c;
  p->splits = (int)s;
  p->chunks_per_split = (int)c;
  p->n_chunks = (int)nc;
  p->n_tiles = (int)tiles;
  p->n_groups = (int)groups;
}

int product_split_count(int64_t M, int64_t N, int Dp, bool x3, int num_sms) {
  ProdCfgRt c = product_cfg(Dp, x3);
  if (!c.ok) return 0;
  if (c.simt) return 1;
  ProductParams p;
  plan_work(M, N, c.bn, c.g, num_sms, &p);
  return p.splits;
}

template <int DP, int BN, int STAGES, bool X3, bool REDUCE, int G>
static int run_kernel(const CUtensorMap& mx, const CUtensorMap& mfh, const CUtensorMap& mfl,
                      const CUtensorMap& mch, const CUtensorMap& mcl, const ProductParams& p,
                      int grid, cudaStream_t stream) {
  using Cfg = ProductCfg<DP, BN, STAGES, X3, REDUCE, G>;
  auto kern = relu_product_kernel<DP, BN, STAGES, X3, REDUCE, G>;
  // once per device (and before any stream capture: the first call of a shape runs eagerly)
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  count_launch();
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(Cfg::THREADS), Cfg::SMEM_BYTES, stream,
                                   mx, mfh, mfl, mch, mcl, p);
  return e != cudaSuccess ? (int)e : (int)cudaGetLastError();
}

#define SB_PRODUCT_CASE(DPV, BNV, STV, X3V, REDV, GV)                                          \
  if (Dp == DPV && c.bn == BNV && c.stages == STV && x3 == X3V && c.g == GV)                   \
    return run_kernel<DPV, BNV, STV, X3V, REDV, GV>(mx, mfh, mfl, mch, mcl, p, grid, stream);

static int dispatch_product(int Dp, const ProdCfgRt& c, bool x3, const CUtensorMap& mx,
                            const CUtensorMap& mfh, const CUtensorMap& mfl, const CUtensorMap& mch,
                            const CUtensorMap& mcl, const ProductParams& p, int grid,
                            cudaStream_t stream) {
  SB_PRODUCT_CASE(16, 128, 4, false, false, 8)
  SB_PRODUCT_CASE(32, 128, 3, false, false, 4)
  SB_PRODUCT_CASE(64, 128, 2, false, false, 1)
  SB_PRODUCT_CASE(128, 64, 2, false, false, 1)
  SB_PRODUCT_CASE(256, 32, 1, false, false, 1)
  SB_PRODUCT_CASE(16, 64, 4, true, false, 8)
  SB_PRODUCT_CASE(32, 64, 2, true, false, 4)
  SB_PRODUCT_CASE(64, 64, 2, true, false, 1)
  SB_PRODUCT_CASE(128, 32, 1, true, false, 1)
  return -1;
}

static int dispatch_reduce(int Dp, const ProdCfgRt& c, bool x3, const CUtensorMap& mx,
                           const CUtensorMap& mfh, const CUtensorMap& mfl, const CUtensorMap& mch,
                           const CUtensorMap& mcl, const ProductParams& p, int grid,
                           cudaStream_t stream) {
  SB_PRODUCT_CASE(16, 128, 6, false, true, 8)
  SB_PRODUCT_CASE(32, 128, 4, false, true, 8)
  SB_PRODUCT_CASE(64, 128, 3, false, true, 4)
  SB_PRODUCT_CASE(128, 64, 2, false, true, 2)
  SB_PRODUCT_CASE(256, 32, 2, false, true, 1)
  SB_PRODUCT_CASE(16, 128, 4, true, true, 8)
  SB_PRODUCT_CASE(32, 128, 3, true, true, 4)
  SB_PRODUCT_CASE(64, 64, 3, true, true, 2)
  SB_PRODUCT_CASE(128, 32, 2, true, true, 1)
  return -1;
}
#undef SB_PRODUCT_CASE

static CUtensorMapSwizzle row_swizzle(int Dp) {
  return Dp * 4 >= 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
}

// ------------------------------------------------------------------------------------------
// fp32 CUDA-core path for the 3xTF32 (fp32-accurate) mode at Dp = 256, where a 128-row X tile in
// tf32 hi + lo halves (256 KB) does not fit shared memory. Persistent CTAs of 256 threads take
// 64-row blocks of X; per 32-row chunk of F: S = X F^T (each thread 8 entries, K = Dp in fp32
// FMAs from shared memory), R = ReLU(S) to shared memory, then Y += R C (each thread 64 of the
// block's 64 x Dp outputs in registers) or the (sum R, sum R^2) accumulation. F = Fhi + Flo and
// C^T = Cthi + Ctlo are reassembled exactly (the halves of a tf32 split add up to the fp32 value).
template <int DP, bool REDUCE>
__global__ void __launch_bounds__(256, 1)
    relu_simt_kernel(const float* __restrict__ X, int M, const float* __restrict__ Fhi,
                     const float* __restrict__ Flo, int N, const float* __restrict__ Cthi,
                     const float* __restrict__ Ctlo, int64_t ldct, float* __restrict__ Y,
                     double* __restrict__ partials, int step, int count) {
  constexpr int RB = 64, CB = 32, LDS = DP + 4;   // rows per block, chunk rows, padded stride
  constexpr int YC = DP / 4;                      // output columns per thread
  extern __shared__ __align__(16) float sm[];
  float* sX = sm;                        // [RB][LDS]
  float* sF = sX + RB * LDS;             // [CB][LDS]
  float* sC = sF + CB * LDS;             // [CB][DP]   (product mode)
  float* sR = sC + (REDUCE ? 0 : CB * DP);  // [RB][CB + 1]
  const int t = threadIdx.x;
  const int r = t >> 2, q = t & 3;
  double acc_s = 0.0, acc_s2 = 0.0, acc_n = 0.0;
  for (int rb = blockIdx.x; rb * RB < M; rb += gridDim.x) {
    const int row0 = rb * RB;
    __syncthreads();
    for (int i = t; i < RB * DP / 4; i += 256) {
      const int rr = i / (DP / 4), kk = (i % (DP / 4)) * 4;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (row0 + rr < M) v = *reinterpret_cast<const float4*>(X + (size_t)(row0 + rr) * DP + kk);
      *reinterpret_cast<float4*>(sX + rr * LDS + kk) = v;
    }
    float y[YC];
#pragma unroll
    for (int j = 0; j < YC; ++j) y[j] = 0.f;
    for (int c0 = 0; c0 < N; c0 += CB) {
      __syncthreads();
      for (int i = t; i < CB * DP / 4; i += 256) {
        const int jj = i / (DP / 4), kk = (i % (DP / 4)) * 4;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (c0 + jj < N) {
          const float4 h = *reinterpret_cast<const float4*>(Fhi + (size_t)(c0 + jj) * DP + kk);
          const float4 l = *reinterpret_cast<const float4*>(Flo + (size_t)(c0 + jj) * DP + kk);
          v = make_float4(h.x + l.x, h.y + l.y, h.z + l.z, h.w + l.w);
        }
        *reinterpret_cast<float4*>(sF + jj * LDS + kk) = v;
      }
      if constexpr (!REDUCE) {
        for (int i = t; i < CB * DP; i += 256) {
          const int k = i / CB, jj = i % CB;
          float v = 0.f;
          if (c0 + jj < N) v = Cthi[(size_t)k * ldct + c0 + jj] + Ctlo[(size_t)k * ldct + c0 + jj];
          sC[jj * DP + k] = v;
        }
      }
      __syncthreads();
      // S[r][q*8 .. q*8+7]
      float s[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] = 0.f;
      for (int k = 0; k < DP; k += 4) {
        const float4 xv = *reinterpret_cast<const float4*>(sX + r * LDS + k);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 fv = *reinterpret_cast<const float4*>(sF + (q * 8 + j) * LDS + k);
          s[j] = fmaf(xv.x, fv.x, fmaf(xv.y, fv.y, fmaf(xv.z, fv.z, fmaf(xv.w, fv.w, s[j]))));
        }
      }
      if constexpr (REDUCE) {
        float cs = 0.f, cs2 = 0.f, cn = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const bool valid = row0 + r < M && c0 + q * 8 + j < N;
          const float v = valid ? fmaxf(s[j], 0.f) : 0.f;
          cs += v;
          cs2 = fmaf(v, v, cs2);
          cn += v > 0.f ? 1.f : 0.f;
        }
        acc_s += (double)cs;
        acc_s2 += (double)cs2;
        acc_n += (double)cn;
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          sR[r * (CB + 1) + q * 8 + j] = step ? (s[j] > 0.f ? 1.f : 0.f) : fmaxf(s[j], 0.f);
        __syncthreads();
        for (int jj = 0; jj < CB; ++jj) {
          const float rv = sR[r * (CB + 1) + jj];
          const float* cr = sC + jj * DP + q * YC;
#pragma unroll
          for (int j = 0; j < YC; j += 4) {
            const float4 cv = *reinterpret_cast<const float4*>(cr + j);
            y[j] = fmaf(rv, cv.x, y[j]);
            y[j + 1] = fmaf(rv, cv.y, y[j + 1]);
            y[j + 2] = fmaf(rv, cv.z, y[j + 2]);
            y[j + 3] = fmaf(rv, cv.w, y[j + 3]);
          }
        }
      }
    }
    if constexpr (!REDUCE) {
      if (row0 + r < M) {
        float* out = Y + (size_t)(row0 + r) * DP + q * YC;
#pragma unroll
        for (int j = 0; j < YC; j += 4)
          *reinterpret_cast<float4*>(out + j) = make_float4(y[j], y[j + 1], y[j + 2], y[j + 3]);
      }
    }
  }
  if constexpr (REDUCE) {
    __shared__ double red[3][8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      acc_s += __shfl_xor_sync(0xffffffffu, acc_s, o);
      acc_s2 += __shfl_xor_sync(0xffffffffu, acc_s2, o);
      acc_n += __shfl_xor_sync(0xffffffffu, acc_n, o);
    }
    __syncthreads();
    if ((t & 31) == 0) { red[0][t >> 5] = acc_s; red[1][t >> 5] = acc_s2; red[2][t >> 5] = acc_n; }
    __syncthreads();
    if (t == 0) {
      double a = 0.0, b = 0.0, c = 0.0;
      for (int w = 0; w < 8; ++w) { a += red[0][w]; b += red[1][w]; c += red[2][w]; }
      const int stride = count ? 3 : 2;
      partials[stride * blockIdx.x] = a;
      partials[stride * blockIdx.x + 1] = b;
      if (count) partials[stride * blockIdx.x + 2] = c;
    }
  }
}

template <bool REDUCE>
static int launch_simt(const float* X, int64_t M, const float* Fhi, const float* Flo, int64_t N,
                       const float* Cthi, const float* Ctlo, int64_t ldct, float* Y,
                       double* partials, int num_sms, cudaStream_t stream, int* grid_out,
                       int step, int count = 0) {
  constexpr int DP = 256, LDS = DP + 4;
  constexpr size_t smem = sizeof(float) * (64 * LDS + 32 * LDS + (REDUCE ? 0 : 32 * DP) +
                                           (REDUCE ? 0 : 64 * 33));
  auto kern = relu_simt_kernel<DP, REDUCE>;
  static bool attr_set[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return (int)e;
    if (dev >= 0 && dev < 64) attr_set[dev] = true;
  }
  const int64_t blocks = (M + 63) / 64;
  const int grid = (int)(blocks < num_sms ? blocks : num_sms);
  if (grid_out) *grid_out = grid;
  count_launch();
  kern<<<grid, 256, smem, stream>>>(X, (int)M, Fhi, Flo ? Flo : Fhi, (int)N, Cthi, Ctlo, ldct, Y,
                                    partials, step, count);
  return (int)cudaGetLastError();
}

int launch_relu_product(const float* X, int64_t M, const float* Fhi, const float* Flo,
                        const float* Cthi, const float* Ctlo, int64_t ldct, int64_t N, int Dp,
                        bool x3, float* ws, int* err, int num_sms, unsigned long long timeout_ns,
                        cudaStream_t stream, const unsigned int* stats, int step, int f_rounded,
                        int nstats) {
  ProdCfgRt c = product_cfg(Dp, x3);
  if (!c.ok) return -1;
  if (M <= 0 || N <= 0 || M >= INT32_MAX || N >= INT32_MAX) return -5;
  if (!x3 && !stats) return -7;  // the fp16 second MMA needs the operand maxima
  if (c.simt) return launch_simt<false>(X, M, Fhi, Flo, N, Cthi, Ctlo, ldct, ws, nullptr, num_sms,
                                        stream, nullptr, step);
  const uint32_t box_k = Dp * 4 <= 128 ? Dp : 32;
  CUtensorMap mx, mfh, mfl, mch, mcl;
  const CUtensorMapSwizzle sw = row_swizzle(Dp);
  if (!make_map(&mx, X, Dp, M, Dp, box_k, 128, sw)) return -6;
  if (!make_map(&mfh, Fhi, Dp, N, Dp, box_k, c.bn, sw)) return -6;
  if (!make_map(&mfl, x3 ? Flo : Fhi, Dp, N, Dp, box_k, c.bn, sw)) return -6;
  if (!make_map(&mch, Cthi, N, Dp, ldct, 32, Dp, CU_TENSOR_MAP_SWIZZLE_128B)) return -6;
  if (!make_map(&mcl, x3 ? Ctlo : Cthi, N, Dp, ldct, 32, Dp, CU_TENSOR_MAP_SWIZZLE_128B)) return -6;
  ProductParams p;
  p.M = (int)M;
  p.N = (int)N;
  plan_work(M, N, c.bn, c.g, num_sms, &p);
  p.ws = ws;
  p.partials = nullptr;
  p.err = err;
  p.timeout_ns = timeout_ns;
  p.Xg = X;
  p.stats = stats;
  p.nstats = nstats;
  p.step = step;
  p.count = 0;
  p.f_rounded = f_rounded;
  const int64_t items = (int64_t)p.n_groups * p.splits;
  const int grid = (int)(items < num_sms ? items : num_sms);
  return dispatch_product(Dp, c, x3, mx, mfh, mfl, mch, mcl, p, grid, stream);
}

int launch_relu_reduce(const float* X, int64_t M, const float* Fhi, const float* Flo, int64_t N,
                       int Dp, bool x3, double* partials, int* grid_out, int* err, int num_sms,
                       unsigned long long timeout_ns, cudaStream_t stream, int count,
                       int f_rounded) {
  ProdCfgRt c = reduce_cfg(Dp, x3);
  if (!c.ok) return -1;
  if (M <= 0 || N <= 0 || M >= INT32_MAX || N >= INT32_MAX) return -5;
  if (c.simt) return launch_simt<true>(X, M, Fhi, Flo, N, nullptr, nullptr, 0, nullptr, partials,
                                       num_sms, stream, grid_out, 0, count);
  const uint32_t box_k = Dp * 4 <= 128 ? Dp : 32;
  CUtensorMap mx, mfh, mfl;
  const CUtensorMapSwizzle sw = row_swizzle(Dp);
  if (!make_map(&mx, X, Dp, M, Dp, box_k, 128, sw)) return -6;
  if (!make_map(&mfh, Fhi, Dp, N, Dp, box_k, c.bn, sw)) return -6;
  if (!make_map(&mfl, x3 ? Flo : Fhi, Dp, N, Dp, box_k, c.bn, sw)) return -6;
  ProductParams p;
  p.M = (int)M;
  p.N = (int)N;
  plan_work(M, N, c.bn, c.g, num_sms, &p);
  p.ws = nullptr;
  p.Xg = X;
  p.stats = nullptr;
  p.nstats = 0;
  p.step = 0;
  p.count = count;
  p.f_rounded = f_rounded;
  p.partials = partials;
  p.err = err;
  p.timeout_ns = timeout_ns;
  const int64_t items = (int64_t)p.n_groups * p.splits;
  const int grid = (int)(items < num_sms ? items : num_sms);
  *grid_out = grid;
  return dispatch_reduce(Dp, c, x3, mx, mfh, mfl, mfh, mfh, p, grid, stream);
}

}  // namespace sb

#ifdef SB_TRACE
// Copy the CTA-0 timeline of the last product / reduce launch (28 x 512 clock64 stamps).
extern "C" int sumac_debug_trace(unsigned long long* host_dst) {
  cudaDeviceSynchronize();
  return (int)cudaMemcpyFromSymbol(host_dst, sb::g_sb_trace, sizeof(sb::g_sb_trace));
}
extern "C" int sumac_debug_trace_clear(void) {
  static unsigned long long zero[28][512];
  return (int)cudaMemcpyToSymbol(sb::g_sb_trace, zero, sizeof(zero));
}
#endif
