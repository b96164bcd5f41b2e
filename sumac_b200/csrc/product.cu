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
};

// Per (Dp, precision): the TMEM budget is NBUF * BN (x2 for 3xTF32) S columns plus G * Dp Y
// columns <= 512; shared memory holds G X slots and the stages.
static ProdCfgRt product_cfg(int Dp, bool x3) {
  if (!x3) {
    switch (Dp) {
      case 16: return {128, 4, 8, true};
      case 32: return {128, 3, 4, true};
      case 64: return {128, 2, 2, true};
      case 128: return {64, 2, 1, true};
    }
  } else {
    switch (Dp) {
      case 16: return {64, 4, 8, true};
      case 32: return {64, 2, 4, true};
      case 64: return {64, 2, 1, true};
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
  kern<<<grid, Cfg::THREADS, Cfg::SMEM_BYTES, stream>>>(mx, mfh, mfl, mch, mcl, p);
  return (int)cudaGetLastError();
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
  SB_PRODUCT_CASE(64, 128, 2, false, false, 2)
  SB_PRODUCT_CASE(128, 64, 2, false, false, 1)
  SB_PRODUCT_CASE(16, 64, 4, true, false, 8)
  SB_PRODUCT_CASE(32, 64, 2, true, false, 4)
  SB_PRODUCT_CASE(64, 64, 2, true, false, 1)
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

int launch_relu_product(const float* X, int64_t M, const float* Fhi, const float* Flo,
                        const float* Cthi, const float* Ctlo, int64_t ldct, int64_t N, int Dp,
                        bool x3, float* ws, int* err, int num_sms, unsigned long long timeout_ns,
                        cudaStream_t stream, const unsigned int* stats) {
  ProdCfgRt c = product_cfg(Dp, x3);
  if (!c.ok) return -1;
  if (M <= 0 || N <= 0 || M >= INT32_MAX || N >= INT32_MAX) return -5;
  if (!x3 && !stats) return -7;  // the fp16 second MMA needs the operand maxima
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
  const int64_t items = (int64_t)p.n_groups * p.splits;
  const int grid = (int)(items < num_sms ? items : num_sms);
  return dispatch_product(Dp, c, x3, mx, mfh, mfl, mch, mcl, p, grid, stream);
}

int launch_relu_reduce(const float* X, int64_t M, const float* Fhi, const float* Flo, int64_t N,
                       int Dp, bool x3, double* partials, int* grid_out, int* err, int num_sms,
                       unsigned long long timeout_ns, cudaStream_t stream) {
  ProdCfgRt c = reduce_cfg(Dp, x3);
  if (!c.ok) return -1;
  if (M <= 0 || N <= 0 || M >= INT32_MAX || N >= INT32_MAX) return -5;
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
// Copy the CTA-0 timeline of the last product / reduce launch (16 x 512 clock64 stamps).
extern "C" int sumac_debug_trace(unsigned long long* host_dst) {
  cudaDeviceSynchronize();
  return (int)cudaMemcpyFromSymbol(host_dst, sb::g_sb_trace, sizeof(sb::g_sb_trace));
}
extern "C" int sumac_debug_trace_clear(void) {
  static unsigned long long zero[16][512];
  return (int)cudaMemcpyToSymbol(sb::g_sb_trace, zero, sizeof(zero));
}
#endif
