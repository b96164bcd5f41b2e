// relu_product.cuh — the fused ReLU(X F^T) contraction on tcgen05 (sm_100a).
//
// One persistent, warp-specialised kernel computes, for a group of up to G row tiles of X
// (128 rows each) and a range of chunks of the fixed operand F (BN rows each):
//
//   product mode:  Y[rows, :Dp] = sum_chunks ReLU(X_tile F_chunk^T) C_chunk          (C = Ct^T)
//   reduce  mode:  (sum ReLU(X F^T), sum ReLU(X F^T)^2)  over the whole X x F product
//
// which is relu_bat_c (src/sumac/kernels/tuning/relu_bat_c/relu_bat_c_base.py:4-6, with
// B -> X, A -> F) and relu_bat_reduce (src/sumac/kernels/tuning/relu_bat_reduce/
// relu_bat_reduce.py:11-22, with A -> X, B -> F). The m x n intermediate never leaves the SM.
//
// Schedule: the row tiles of a group stay resident in shared memory (one X slot each) and every
// (F, C) chunk is loaded once per group and used by all of its tiles, so the chunk stream per SM
// is G times shorter than with one tile at a time. MMA "pairs" (first + second MMA of one tile
// and one chunk) run chunk-major: (c0, tile 0), (c0, tile 1), ..., (c1 - 1, last tile). Each
// tile has its own Y accumulator in TMEM (G x Dp columns), next to NBUF S buffers.
//
//   warp 0       TMA producer of the chunks: lanes 0..15 fill each stage (F chunk, C^T chunk)
//                together, one copy per lane (copies issued by one thread complete one after
//                another, copies from different lanes overlap)
//   warp 1       first-MMA issuer (one thread): S = X_g F_c^T into the next of NBUF TMEM
//                buffers (kind::tf32); with an even NBUF >= 4 in TF32 mode a second issuer takes
//                the odd pairs
//   warps 2..9   epilogue, two warps per TMEM lane quadrant, each on half of the columns: they
//                prepare the group's X tiles in shared memory (round / scale / split) two pairs
//                ahead of the first chunk's pairs, then per pair tcgen05.ld S -> ReLU ->
//                tcgen05.st R (or accumulate the sums), and in the last chunk tcgen05.ld of each
//                Y_g -> global behind the next tile's pair
//   warp 10      TF32: chunk prep (fp16 copy of the C chunk in product mode; rounding of F where
//                it was not packed as tf32 values)
//   warps 11-12  second-MMA issuers (one thread each, product mode, even / odd tiles of the
//                group): Y_g += R C_c with R read from TMEM once the epilogue has rewritten
//                that S as R = ReLU(S); the commit hands the S buffer back to warp 1.
//   X loader     (last warp; warp 10 in 3xTF32 mode) loads each group's row tiles into its X
//                slot set (two sets where they fit, so the next group's tiles land early)
//
// Cost model (measured on B200 with in-kernel timestamps): at small rank the kernel is bound by
// serial latencies, not by tensor throughput or HBM: ~50 ns per tcgen05 MMA or commit issued by
// one thread (whatever N <= 64; the second MMA has N = Dp and needs BN / 16 fp16 or BN / 8 tf32
// instructions per pair), the epilogue's TMEM round trip (~350 ns per pair), and at Dp = 64 with
// 2-tile groups the per-chunk fp16 conversion of C. Resident tile groups (a chunk copy from L2
// takes 1.5-4 us to land), two second-MMA issuers and batched conversion keep these apart.
//
// Precision: X3=false is TF32 for S = X F^T (the tensor core reads the fp32 bits as tf32), and
// the second MMA runs in fp16 (same 10-bit mantissa) with R and C scaled by exact powers of two
// so that no value overflows. X3=true is the 3xTF32 split (x = hi + lo, hi = x with the low 13
// mantissa bits cleared), giving fp32 accuracy: S = Xlo Fhi + Xhi Flo + Xhi Fhi and
// Y += Rlo Chi + Rhi Clo + Rhi Chi.
//
// Shared-memory operands are K-major with the TMA swizzle matching the row width (64 B rows:
// SWIZZLE_64B, 128 B rows: SWIZZLE_128B; wider rows are split in 128 B sub-tiles).
// No TMA multicast is used anywhere. Every wait is bounded (see mbar_wait).
#pragma once
#include "kernels.cuh"
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace sb {

// Optional in-kernel timeline (build with -DSB_TRACE): CTA 0 stamps clock64() at each hand-off of
// the pipeline into g_sb_trace[event][index]; sumac_debug_trace copies it out. Off by default.
#ifdef SB_TRACE
__device__ unsigned long long g_sb_trace[28][512];
#define SB_TR(ev, i)                                                         \
  do {                                                                       \
    if (blockIdx.x == 0 && (unsigned)(i) < 512u) g_sb_trace[ev][i] = clock64(); \
  } while (0)
#else
#define SB_TR(ev, i) \
  do {               \
  } while (0)
#endif

// max over the p.nstats pairs of stats entry k (0: max_i |F_i|, 1: max |C|)
struct ProductParams;
__device__ __forceinline__ float stats_max(const unsigned int* stats, int nstats, int k) {
  unsigned int m = 0u;
#pragma unroll 4
  for (int i = 0; i < nstats; ++i) m = max(m, stats[2 * i + k]);
  return __uint_as_float(m);
}

struct ProductParams {
  int M;                 // rows of X
  int N;                 // rows of F (columns of C^T)
  int n_chunks;          // ceil(N / BN)
  int splits;            // chunk ranges per group (split-K); items = n_groups * splits
  int chunks_per_split;  // ceil(n_chunks / splits)
  int n_tiles;           // ceil(M / 128)
  int n_groups;          // group k holds tiles [k n_tiles / n_groups, (k+1) n_tiles / n_groups)
  float* ws;             // product mode: [splits][M][DP] partial outputs
  double* partials;      // reduce mode: [gridDim.x][2] per-CTA (sum, sum of squares)
  int* err;              // device error word (0 = ok)
  unsigned long long timeout_ns;
  // TF32 product mode: stats[0] = bits of max_i |F_i| (row norm), stats[1] = bits of max |C|;
  // Xg is X in global memory (row norms for the per-row scale of R).
  // stats holds nstats such pairs (one per CTA of the launch that wrote them); the product takes
  // their maxima (non-negative float bits compare as unsigned integers).
  const float* Xg;
  const unsigned int* stats;
  int nstats;
  // product mode: 0 = R = ReLU(S); 1 = R = step(S) (1 where S > 0, else 0), the mask term of the
  // gradient of sum ReLU(A B^T) (relu_bat_reduce_jit/custom_op.py:74-82)
  int step;
  // reduce mode: 1 = also count the positive entries (relu_bat_reduce_jit/kernel_nnz.cu); the
  // per-CTA partials then hold (sum, sum of squares, count), stride 3
  int count;
  // TF32 mode: 1 = the F operand in global memory already holds tf32 values (rounded to nearest
  // when it was packed), so its chunks are not rounded again in shared memory
  int f_rounded;
};

template <int DP, int BN, int STAGES, bool X3, bool REDUCE, int G>
struct ProductCfg {
  static_assert(DP == 16 || DP == 32 || DP == 64 || DP == 128 || DP == 256, "DP");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(G >= 1 && G <= 8, "tiles per group");
  static_assert(STAGES >= 1 && STAGES <= 16, "stages");
  static constexpr int TM = 128;                          // rows per tile (MMA M)
  static constexpr int XW = DP * 4 <= 128 ? DP * 4 : 128; // K-major row width in bytes
  static constexpr int KSUB = DP * 4 / XW;                // 128 B sub-tiles along K
  static constexpr uint32_t XLAYOUT = XW == 64 ? UMMA_SW64 : UMMA_SW128;
  static constexpr int BOX_K = XW / 4;                    // TMA box inner extent (floats)
  static constexpr int X_BYTES = TM * DP * 4;
  static constexpr int F_BYTES = BN * DP * 4;
  static constexpr int C_BYTES = REDUCE ? 0 : DP * BN * 4;
  static constexpr int NPREC = X3 ? 2 : 1;
  static constexpr int STAGE_BYTES = NPREC * (F_BYTES + C_BYTES);   // bytes the TMA fills
  // TMA copies per stage: per precision half, KSUB sub-tiles of F and BN / 32 of C^T; lanes
  // 0..NLOADS-1 of the producer warp issue one each
  static constexpr int LOADS_PER_PREC = KSUB + (REDUCE ? 0 : BN / 32);
  static constexpr int NLOADS = NPREC * LOADS_PER_PREC;
  static_assert(NLOADS <= 16, "one producer lane per copy");
  // TF32 product mode runs the second MMA in fp16 (half the instructions of kind::tf32) up to
  // Dp = 128; at Dp = 256 the stage has no room for the fp16 copy of C, and R stays fp32 (tf32)
  static constexpr bool H16 = !X3 && !REDUCE && DP <= 128;        // fp16 second MMA
  static constexpr int C16_BYTES = H16 ? DP * BN * 2 : 0;         // fp16 copy of the C chunk
  static constexpr int STAGE_ALLOC = STAGE_BYTES + C16_BYTES;
  static constexpr int XBUF_BYTES = NPREC * X_BYTES;      // one X slot (hi [, lo])
  // Beside the barriers: TMEM slot, abort flag, the epilogue's reduction scratch and (TF32
  // product) the per-row scale exponents of two groups
  static constexpr int aux_bytes(int xb) {
    return ((3 * STAGES + 3 * 8 + 3 * xb * G + 2 * G + 4) * 8 + 16 + 8 * 3 * 8 +
            (H16 ? 2 * G * 128 : 0) + 127) / 128 * 128;
  }
  // X slot sets: two when they fit next to the stages, so that the X loader brings in the next
  // group's tiles while the current group runs; one otherwise
  static constexpr int XB =
      2 * G * XBUF_BYTES + STAGES * STAGE_ALLOC + aux_bytes(2) + 1024 <= 232448 ? 2 : 1;
  static constexpr int AUX_BYTES = aux_bytes(XB);
  static constexpr int NXS = XB * G;                      // X slots
  static constexpr int X_TOTAL = NXS * XBUF_BYTES;
  static constexpr int SMEM_DATA = X_TOTAL + STAGES * STAGE_ALLOC;
  static constexpr int SMEM_BYTES_RAW = SMEM_DATA + AUX_BYTES + 1024 /*align slack*/;
  // at least 120 KB so that only one CTA (and one 512-column TMEM allocation) lives on an SM
  static constexpr int SMEM_BYTES = SMEM_BYTES_RAW < 122880 ? 122880 : SMEM_BYTES_RAW;
  static_assert(SMEM_BYTES_RAW <= 232448, "shared memory budget");
  // S buffers in TMEM: as many as the 512 columns hold next to the Y accumulators (3xTF32
  // product mode keeps a lo half per buffer), at most 8. More buffers in flight hide the round
  // trip of a buffer (first MMA -> epilogue -> second MMA -> free), which bounds small ranks.
  // product mode, MS = 2 (when two sets of Y accumulators fit next to three S buffers): the two
  // second-MMA issuers each take half of every pair's K range into their own set of Y
  // accumulators (the epilogue sums the two), which halves the second MMA's share of the S
  // buffer's round trip; MS = 1: each issuer takes whole pairs, of the tiles gi % 2 == issuer.
  // Measured at d = 16: 8 resident tiles with MS = 1 beat 4 tiles with MS = 2 (56 vs 64 us); at
  // d = 64 one tile with MS = 2 beats MS = 1 (80 vs 96 us)
  static constexpr int MS =
      (!REDUCE && 2 * G * DP + 3 * ((X3 && !REDUCE) ? 2 : 1) * BN <= 512) ? 2 : 1;
  static constexpr int NBUF_FIT =
      (512 - (REDUCE ? 0 : MS * G * DP)) / (((X3 && !REDUCE) ? 2 : 1) * BN);
  static constexpr int NBUF = NBUF_FIT < 8 ? NBUF_FIT : 8;
  static_assert(NBUF >= 2, "at least two S buffers");
  static constexpr int TMEM_S_LO = NBUF * BN;             // lo halves of R (3xTF32)
  static constexpr int TMEM_Y = (X3 ? 2 : 1) * NBUF * BN; // G Y accumulators follow
  static_assert(REDUCE ? NBUF * BN <= 512 : TMEM_Y + MS * G * DP <= 512, "TMEM budget");
  static constexpr uint32_t IDESC1 = umma_idesc_tf32(TM, BN);
  static constexpr uint32_t IDESC2 = umma_idesc_tf32(TM, DP);
  // kind::f16: f32 accumulate, A and B f16, both K-major
  static constexpr uint32_t IDESC2_F16 =
      (1u << 4) | ((uint32_t)(DP >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
  static constexpr int EPI_WARPS = 8;                     // two per TMEM lane quadrant
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  // TF32 mode rounds every operand to the nearest tf32 value in shared memory before the tensor
  // core reads it (the tensor core itself would drop the low 13 mantissa bits, a bias of about
  // -2^-12 per operand): the X tiles by the epilogue warps when a group starts, each (F, C) chunk
  // by the chunk-prep warp, which in product mode also builds the fp16 copy of C
  static constexpr bool ROUND = !X3;
  static constexpr int CPREP_WARP = REDUCE ? 11 : 10;     // chunk-prep warp (ROUND)
  static_assert(!H16 || BN % 64 == 0, "the fp16 C chunk is built of 64-element sub-tiles");
  // product mode: second-MMA issuers, warp MMA2_WARP + i takes the tiles gi with gi % N2 == i
  static constexpr int MMA2_WARP = 11;
  static constexpr int N2 = 2;
  // first-MMA issuers: in TF32 mode with an even number of S buffers, warp 1 issues the even
  // pairs and warp MMA1B_WARP the odd ones (a thread issues one tcgen05.mma every ~100-200
  // cycles whatever its size, so two issuers double the rate); elsewhere warp 1 alone
  static constexpr int N1 = (!X3 && NBUF % 2 == 0 && NBUF >= 4) ? 2 : 1;
  static constexpr int MMA1B_WARP = N1 == 1 ? 1 : (REDUCE ? 10 : MMA2_WARP + N2);
  // The S buffers are split between the first-MMA issuers: pair p belongs to issuer p % N1 and,
  // as that issuer's k-th pair (k = p / N1), to buffer p % N1 + N1 (k % NB1) in its use k / NB1
  // (pair_slot). Each buffer is then filled by one issuer in order, so its wait for the buffer's
  // previous use is at most one phase ahead of the barrier: mbarrier parity waits are only sound
  // then. A buffer is reused every NBUF pairs in the global order. A second-MMA issuer owns the
  // tiles gi % N2 == me, so two of its consecutive pairs can lie up to 2 N2 - 1 pairs apart (one
  // owned tile in a group of 2 N2 - 1 tiles); its wait on r_ready of the later pair needs the
  // epilogue to have released the buffer's previous use, NBUF pairs earlier: NBUF >= 2 N2 - 1.
  static constexpr int NB1 = NBUF / N1;
  static_assert(NBUF % N1 == 0, "S buffers split evenly between the first-MMA issuers");
  static_assert(REDUCE || MS == 2 || NBUF >= 2 * N2 - 1, "barrier phase lag");
  static_assert(MS == 1 || MS == N2, "one accumulator set per second-MMA issuer");
  // X-loader warp: loads each group's row tiles into its X slot set (the epilogue warps prepare
  // them); warp 10 in 3xTF32 mode (no chunk prep there), else the last warp
  static constexpr int XLOAD_WARP =
      X3 ? 10 : (REDUCE ? 12 : MMA2_WARP + N2 + (N1 == 2 ? 1 : 0));
  static constexpr int THREADS =
      32 * (REDUCE ? (X3 ? 11 : 13) : MMA2_WARP + N2 + (N1 == 2 ? 1 : 0) + (X3 ? 0 : 1));
  static_assert(XLOAD_WARP < THREADS / 32, "X-loader warp");
  // mbarriers (below +BAR_BYTES), then TMEM slot and abort flag, the epilogue's reduction scratch
  // and the row exponents
  static constexpr int NBARS = 3 * STAGES + 3 * NBUF + 3 * NXS + 2 * G + N1 + N2;
  static constexpr int BAR_BYTES = (NBARS * 8 + 15) / 16 * 16;
  static constexpr int RED_OFF = BAR_BYTES + 16;
  static constexpr int ER_OFF = RED_OFF + EPI_WARPS * 3 * 8;
  static constexpr bool ROW_SCALE = H16;  // per-row exponents kept for the Y readout
  static_assert(ER_OFF + (ROW_SCALE ? 2 * G * TM : 0) <= AUX_BYTES, "auxiliary area");
  static constexpr int EPI_COLS = BN / 2;                 // S columns per epilogue warp
  static_assert(EPI_COLS % 16 == 0, "epilogue column split");
  static constexpr int LDW = EPI_COLS % 32 == 0 ? 32 : 16;  // tcgen05.ld/st width used
};

// The S buffer of pair `pair` and which use of that buffer it is (see ProductCfg::NB1).
template <class Cfg>
__device__ __forceinline__ void pair_slot(uint32_t pair, uint32_t& buf, uint32_t& use) {
  const uint32_t k = pair / Cfg::N1;
  buf = pair % Cfg::N1 + Cfg::N1 * (k % Cfg::NB1);
  use = k / Cfg::NB1;
}

// One work item: tiles [tile0, tile0 + ntiles) of a group and chunks [c0, c1) of a split.
struct WorkItem {
  int tile0, ntiles, c0, c1;
};

__device__ __forceinline__ WorkItem work_item(const ProductParams& p, int item) {
  const int group = item / p.splits, split = item % p.splits;
  WorkItem w;
  w.tile0 = (int)(((int64_t)group * p.n_tiles) / p.n_groups);
  w.ntiles = (int)(((int64_t)(group + 1) * p.n_tiles) / p.n_groups) - w.tile0;
  w.c0 = split * p.chunks_per_split;
  w.c1 = min(p.n_chunks, w.c0 + p.chunks_per_split);
  return w;
}

// The ci-th chunk of an item in this CTA's order: the chunk range rotated by the CTA index, so
// that at any moment the SMs read different chunks (the same chunk from every SM at once
// concentrates all loads on a few L2 slices). Every role walks the same order.
__device__ __forceinline__ int chunk_at(const WorkItem& w, int ci) {
  const int nc = w.c1 - w.c0;
  return w.c0 + (int)((ci + blockIdx.x) % (unsigned)nc);
}

// Round NV 16-byte units of shared memory at `base` in place, unit i by thread i % NT.
template <int NV, int NT>
__device__ __forceinline__ void round_tf32_smem(uint8_t* base, int t) {
  uint4* q = reinterpret_cast<uint4*>(base);
#pragma unroll 4
  for (int i = t; i < NV; i += NT) {
    uint4 v = q[i];
    v.x = tf32_rne_bits(v.x);
    v.y = tf32_rne_bits(v.y);
    v.z = tf32_rne_bits(v.z);
    v.w = tf32_rne_bits(v.w);
    q[i] = v;
  }
}

// One arrival per warp on an mbarrier whose count is the number of arriving warps (an arrival
// per thread serialises 256 atomic updates of one shared-memory word on the critical path). The
// lanes' earlier shared-memory and tcgen05 work is ordered before lane 0's release-arrive by the
// fences each lane executes before calling this and by __syncwarp.
__device__ __forceinline__ void warp_arrive(uint64_t* bar, int lane) {
  __syncwarp();
  if (lane == 0) mbar_arrive(bar);
}

// A bounded wait whose outcome is the same in every lane of the warp (the .sync.aligned tcgen05
// instructions that follow need the whole warp).
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code, uint64_t timeout_ns) {
  const bool ok = mbar_wait(bar, parity, abort_flag, err, code, timeout_ns);
  return __all_sync(0xffffffffu, ok);
}

// fp16x2 of (ReLU(lo), ReLU(hi)), round to nearest; lo in the low half.
__device__ __forceinline__ uint32_t pack_relu_h2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <int DP, int BN, int STAGES, bool X3, bool REDUCE, int G>
__global__ void __launch_bounds__(ProductCfg<DP, BN, STAGES, X3, REDUCE, G>::THREADS, 1)
    relu_product_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmFhi,
                        const __grid_constant__ CUtensorMap tmFlo,
                        const __grid_constant__ CUtensorMap tmChi,
                        const __grid_constant__ CUtensorMap tmClo, const ProductParams p) {
  using Cfg = ProductCfg<DP, BN, STAGES, X3, REDUCE, G>;
  constexpr int NBUF = Cfg::NBUF;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem;                                   // [NXS][NPREC][X_BYTES]
  uint8_t* sStage = smem + Cfg::X_TOTAL;                // [STAGES][STAGE_ALLOC]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_DATA);
  uint64_t* full = bars;                    // [STAGES] TMA landed
  uint64_t* empty = full + STAGES;          // [STAGES] last MMA reading the stage completed
  uint64_t* c16_ready = empty + STAGES;     // [STAGES] chunk rounded / C converted (ROUND)
  uint64_t* s_full = c16_ready + STAGES;    // [NBUF] S = X F^T computed
  uint64_t* r_ready = s_full + NBUF;        // [NBUF] epilogue done with the S buffer
  uint64_t* s_free = r_ready + NBUF;        // [NBUF] second MMA done with the S buffer
  uint64_t* x_full = s_free + NBUF;         // [NXS] X slot landed
  uint64_t* x_ready = x_full + Cfg::NXS;    // [NXS] X slot prepared (rounded / scaled / split)
  uint64_t* x_empty = x_ready + Cfg::NXS;   // [NXS] last MMA reading the X slot completed
  uint64_t* y_full = x_empty + Cfg::NXS;    // [G] Y accumulator complete
  uint64_t* y_empty = y_full + G;           // [G] Y accumulator read out
  uint64_t* drain = y_empty + G;            // [N1 + N2] each MMA thread's own MMAs completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + Cfg::SMEM_DATA + Cfg::BAR_BYTES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  double* red = reinterpret_cast<double*>(smem + Cfg::SMEM_DATA + Cfg::RED_OFF);  // [EPI_WARPS][3]
  int8_t* er_s = reinterpret_cast<int8_t*>(smem + Cfg::SMEM_DATA + Cfg::ER_OFF);  // [2][G][128]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.n_groups * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], REDUCE ? Cfg::N1 : Cfg::N2);
      mbar_init(&c16_ready[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&r_ready[b], Cfg::EPI_WARPS);
      mbar_init(&s_free[b], Cfg::MS);
    }
    for (int xs = 0; xs < Cfg::NXS; ++xs) {
      mbar_init(&x_full[xs], 1);
      mbar_init(&x_ready[xs], Cfg::EPI_WARPS);
      mbar_init(&x_empty[xs], Cfg::N1);
    }
    for (int g = 0; g < G; ++g) {
      mbar_init(&y_full[g], Cfg::MS);
      mbar_init(&y_empty[g], Cfg::EPI_WARPS);
    }
    for (int i = 0; i < Cfg::N1 + Cfg::N2; ++i) mbar_init(&drain[i], 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tmX);
    tma_prefetch_desc(&tmFhi);
    if (X3) tma_prefetch_desc(&tmFlo);
    if (!REDUCE) {
      tma_prefetch_desc(&tmChi);
      if (X3) tma_prefetch_desc(&tmClo);
    }
  }
  // launched programmatically behind the operand gather: its output is read from here on, and
  // the TMEM allocation waits too (so it never overlaps a previous product of the stream)
  pdl_wait();
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;
  if (threadIdx.x == 0) SB_TR(15, 0);

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // lanes 0..15 fill the stages together: lane 0 waits for the stage to be free and posts the
    // expected bytes, lane j < NLOADS issues copy j of the chunk (copies issued by one thread
    // complete one after another, copies from different lanes overlap). The X tiles are loaded by
    // the first epilogue warp, so that they do not queue behind the chunk copies of this warp.
    if (lane < 16) {
      bool ok = true;
      uint32_t gch = 0;     // chunks issued
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const WorkItem w = work_item(p, item);
        for (int ci = 0; ci < w.c1 - w.c0; ++ci, ++gch) {
          const int c = chunk_at(w, ci);
          const int stage = gch % STAGES;
          const uint32_t round = gch / STAGES;
          int go = 1;
          if (lane == 0) {
            // a stage is free once the empty barrier completed its previous round
            if (round > 0 && !mbar_wait(&empty[stage], (round - 1) & 1, abort_flag, p.err,
                                        DEV_TIMEOUT_EMPTY, p.timeout_ns)) go = 0;
            else mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          }
          go = __shfl_sync(0xffffu, go, 0);
          if (!go) { ok = false; break; }
          if (lane == 0) SB_TR(0, gch);
          if (lane < Cfg::NLOADS) {
            uint8_t* st = sStage + stage * Cfg::STAGE_ALLOC;
            const int h = lane / Cfg::LOADS_PER_PREC, r = lane % Cfg::LOADS_PER_PREC;
            if (r < Cfg::KSUB) {
              tma_load_2d(st + h * Cfg::F_BYTES + r * BN * Cfg::XW, h == 0 ? &tmFhi : &tmFlo,
                          r * Cfg::BOX_K, c * BN, &full[stage]);
            } else {
              const int sc = r - Cfg::KSUB;
              tma_load_2d(st + Cfg::NPREC * Cfg::F_BYTES + h * Cfg::C_BYTES + sc * DP * 128,
                          h == 0 ? &tmChi : &tmClo, c * BN + sc * 32, 0, &full[stage]);
            }
          }
        }
      }
      if (*abort_flag && lane == 0) {
        // wait (bounded) for the copies still in flight: the last fill of every stage
        for (uint32_t u = 1; u <= (uint32_t)STAGES && u <= gch; ++u) {
          const uint32_t g = gch - u;
          mbar_drain(&full[g % STAGES], (g / STAGES) & 1);
        }
      }
    }
  } else if (warp == 1 || warp == Cfg::MMA1B_WARP) {
    // ------------------------------------------------------------------ first MMA (S = X F^T)
    // issuer me1 takes the pairs with pair % N1 == me1; the stage and X-slot release barriers
    // count one commit per issuer
    const int me1 = warp == 1 ? 0 : 1;
    if (lane == 0) {
      const uint32_t sX_addr = smem_u32(sX);
      const uint32_t sSt_addr = smem_u32(sStage);
      uint32_t pair = 0, chunk = 0;
      uint32_t slot_par = 0;  // bit xs: parity of the number of earlier uses of X slot xs
      bool ok = true;
      uint32_t li = 0;        // groups of this CTA so far
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++li) {
        const WorkItem w = work_item(p, item);
        const int xs0 = (int)(li % Cfg::XB) * G;  // this group's X slots: xs0 + gi
        // a tile's slot is waited for right before its first pair; every issuer also waits for
        // the slots it issues no pair on before its release commit below (the slot's barrier
        // must not see a commit for this group before the previous group's phase completed)
        uint32_t waited = 0;
        for (int ci = 0; ci < w.c1 - w.c0 && ok; ++ci, ++chunk) {
          const int c = chunk_at(w, ci);
          const int stage = chunk % STAGES;
          const bool prepped = Cfg::ROUND && (!REDUCE || !p.f_rounded);
          if (!mbar_wait(prepped ? &c16_ready[stage] : &full[stage], (chunk / STAGES) & 1,
                         abort_flag, p.err, DEV_TIMEOUT_FULL, p.timeout_ns)) { ok = false; break; }
          const uint32_t fbase = sSt_addr + stage * Cfg::STAGE_ALLOC;
          for (int gi = 0; gi < w.ntiles; ++gi, ++pair) {
            if ((int)(pair % Cfg::N1) != me1) continue;
            uint32_t buf, use;
            pair_slot<Cfg>(pair, buf, use);
            // the S buffer is free once the epilogue (reduce) or the second MMA (product) is
            // done with its previous use
            if (use > 0 &&
                !mbar_wait(REDUCE ? &r_ready[buf] : &s_free[buf], (use - 1) & 1,
                           abort_flag, p.err, DEV_TIMEOUT_RREADY, p.timeout_ns)) {
              ok = false;
              break;
            }
            if (!((waited >> gi) & 1u)) {
              if (!mbar_wait(&x_ready[xs0 + gi], (slot_par >> (xs0 + gi)) & 1u, abort_flag, p.err,
                             DEV_TIMEOUT_X, p.timeout_ns)) { ok = false; break; }
              waited |= 1u << gi;
            }
            tc_fence_after();
            SB_TR(1, pair);
            const uint32_t xaddr = sX_addr + (xs0 + gi) * Cfg::XBUF_BYTES;
            const uint32_t s_tm = tbase + buf * BN;
#pragma unroll
            for (int kk = 0; kk < DP / 8; ++kk) {
              const int sub = kk / (Cfg::XW / 32);
              const uint32_t off = (kk % (Cfg::XW / 32)) * 32;
              const uint64_t ahi = umma_sdesc(xaddr + sub * Cfg::TM * Cfg::XW + off, 16,
                                              8 * Cfg::XW, Cfg::XLAYOUT);
              const uint64_t bhi = umma_sdesc(fbase + sub * BN * Cfg::XW + off, 16, 8 * Cfg::XW,
                                              Cfg::XLAYOUT);
              if (X3) {
                const uint64_t alo = umma_sdesc(xaddr + Cfg::X_BYTES + sub * Cfg::TM * Cfg::XW + off,
                                                16, 8 * Cfg::XW, Cfg::XLAYOUT);
                const uint64_t blo = umma_sdesc(fbase + Cfg::F_BYTES + sub * BN * Cfg::XW + off,
                                                16, 8 * Cfg::XW, Cfg::XLAYOUT);
                mma_tf32_ss(s_tm, alo, bhi, Cfg::IDESC1, kk == 0 ? 0u : 1u);
                mma_tf32_ss(s_tm, ahi, blo, Cfg::IDESC1, 1u);
                mma_tf32_ss(s_tm, ahi, bhi, Cfg::IDESC1, 1u);
              } else {
                mma_tf32_ss(s_tm, ahi, bhi, Cfg::IDESC1, kk == 0 ? 0u : 1u);
              }
            }
            mma_commit(&s_full[buf]);
            SB_TR(2, pair);
          }
          // reduce mode: the first MMAs are the stage's only readers
          if (REDUCE && ok) mma_commit(&empty[stage]);
        }
        for (int gi = 0; gi < w.ntiles && ok; ++gi) {
          if (!((waited >> gi) & 1u) &&
              !mbar_wait(&x_ready[xs0 + gi], (slot_par >> (xs0 + gi)) & 1u, abort_flag, p.err,
                         DEV_TIMEOUT_X, p.timeout_ns)) { ok = false; break; }
          mma_commit(&x_empty[xs0 + gi]);  // X slot done
        }
        slot_par ^= ((1u << w.ntiles) - 1u) << xs0;
      }
      // make sure every MMA this thread issued has completed before TMEM is released
      mma_commit(&drain[me1]);
      mbar_drain(&drain[me1], 0);
    }
  } else if (!REDUCE && warp >= Cfg::MMA2_WARP && warp < Cfg::MMA2_WARP + Cfg::N2) {
    // ------------------------------------------------------------------ second MMA (Y += R C)
    // issuer `me` owns the Y slots gi with gi % N2 == me
    const int me = warp - Cfg::MMA2_WARP;
    if (lane == 0) {
      const uint32_t sSt_addr = smem_u32(sStage);
      uint32_t pair = 0, chunk = 0;
      uint32_t slot_par = 0;   // bit g: parity of the number of earlier uses of Y slot g
      uint32_t slot_used = 0;  // bit g: Y slot g used by an earlier item
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
        const WorkItem w = work_item(p, item);
        for (int ci = 0; ci < w.c1 - w.c0 && ok; ++ci, ++chunk) {
          const int stage = chunk % STAGES;
          const uint32_t stg = sSt_addr + stage * Cfg::STAGE_ALLOC;
          // every issuer waits for the chunk, even one that owns no tile of this group: its
          // commit on `empty` below must not run ahead into a later phase of the barrier
          if (!mbar_wait(Cfg::ROUND ? &c16_ready[stage] : &full[stage], (chunk / STAGES) & 1,
                         abort_flag, p.err, DEV_TIMEOUT_FULL, p.timeout_ns)) { ok = false; break; }
          for (int gi = 0; gi < w.ntiles; ++gi, ++pair) {
            if (Cfg::MS == 1 && gi % Cfg::N2 != me) continue;
            uint32_t buf, use;
            pair_slot<Cfg>(pair, buf, use);
            const bool first = ci == 0;
            if (!mbar_wait(&r_ready[buf], use & 1, abort_flag, p.err, DEV_TIMEOUT_RREADY,
                           p.timeout_ns)) { ok = false; break; }
            if (first && ((slot_used >> gi) & 1u) &&
                !mbar_wait(&y_empty[gi], ((slot_par >> gi) & 1u) ^ 1u, abort_flag, p.err,
                           DEV_TIMEOUT_Y, p.timeout_ns)) { ok = false; break; }
            tc_fence_after();
            SB_TR(7 + 2 * me, pair);
            const uint32_t s_hi = tbase + buf * BN;
            // this issuer's accumulator set (MS = 2) and its share of the K steps
            const uint32_t ytm = tbase + Cfg::TMEM_Y + (Cfg::MS == 2 ? me : 0) * G * DP + gi * DP;
            if constexpr (Cfg::H16) {
              // R packed as fp16 pairs: warp half h holds k in [h*EPI_COLS, (h+1)*EPI_COLS) in
              // its own first EPI_COLS/2 columns; C in fp16, 64-element 128 B swizzled sub-tiles
              const uint32_t c16 = stg + Cfg::STAGE_BYTES;
              constexpr int KK = BN / 16, K0 = Cfg::MS == 2 ? KK / 2 : KK;
#pragma unroll
              for (int k = 0; k < K0; ++k) {
                const int kk = (Cfg::MS == 2 ? me * K0 : 0) + k;
                const int hh = (16 * kk) / Cfg::EPI_COLS;
                const uint32_t acol = hh * Cfg::EPI_COLS + (16 * kk - hh * Cfg::EPI_COLS) / 2;
                const uint32_t off = (kk >> 2) * (DP * 128) + (kk & 3) * 32;
                const uint64_t bd = umma_sdesc(c16 + off, 16, 1024, UMMA_SW128);
                mma_f16_ts(ytm, s_hi + acol, bd, Cfg::IDESC2_F16, (first && k == 0) ? 0u : 1u);
              }
            } else {
              const uint32_t s_lo = tbase + Cfg::TMEM_S_LO + buf * BN;
              const uint32_t cbase = stg + Cfg::NPREC * Cfg::F_BYTES;
              constexpr int KK = BN / 8, K0 = Cfg::MS == 2 ? KK / 2 : KK;
#pragma unroll
              for (int k = 0; k < K0; ++k) {
                const int kk = (Cfg::MS == 2 ? me * K0 : 0) + k;
                const uint32_t off = (kk >> 2) * (DP * 128) + (kk & 3) * 32;
                const uint64_t bhi = umma_sdesc(cbase + off, 16, 1024, UMMA_SW128);
                const uint32_t acc0 = (first && k == 0) ? 0u : 1u;
                if (X3) {
                  const uint64_t blo = umma_sdesc(cbase + Cfg::C_BYTES + off, 16, 1024, UMMA_SW128);
                  mma_tf32_ts(ytm, s_lo + kk * 8, bhi, Cfg::IDESC2, acc0);
                  mma_tf32_ts(ytm, s_hi + kk * 8, blo, Cfg::IDESC2, 1u);
                  mma_tf32_ts(ytm, s_hi + kk * 8, bhi, Cfg::IDESC2, 1u);
                } else {
                  mma_tf32_ts(ytm, s_hi + kk * 8, bhi, Cfg::IDESC2, acc0);
                }
              }
            }
            mma_commit(&s_free[buf]);
            SB_TR(8 + 2 * me, pair);
            if (ci == w.c1 - w.c0 - 1) mma_commit(&y_full[gi]);
          }
          // every first MMA of this chunk completed before the epilogue released its S, so the
          // N2 issuers' commits together cover the last readers of the stage
          if (ok) mma_commit(&empty[stage]);
        }
        const uint32_t mask = (1u << w.ntiles) - 1u;
        slot_par ^= mask;
        slot_used |= mask;
      }
      mma_commit(&drain[Cfg::N1 + me]);
      mbar_drain(&drain[Cfg::N1 + me], 0);
    }
  } else if (warp >= 2 && warp < 2 + Cfg::EPI_WARPS) {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    // warp w reads TMEM lane quadrant w % 4 (hardware rule) and half (w - 2) / 4 of the columns
    const int qd = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = qd * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
    uint32_t pair = 0;
    uint32_t slot_par = 0;       // bit g: parity of the earlier uses of Y slot g
    uint32_t xslot_par = 0;      // bit xs: parity of the earlier uses of X slot xs
    double acc_s = 0.0, acc_s2 = 0.0, acc_n = 0.0;
    bool ok = true;
    // fp16 second MMA: C is scaled by 2^ec (fixed per launch), row j of R by 2^er(j)
    int ec = 0;
    float fmax = 0.f;  // max_i |F_i| (row norms), for the row scales
    if constexpr (Cfg::H16) {
      fmax = stats_max(p.stats, p.nstats, 0);
      const float cmax = stats_max(p.stats, p.nstats, 1);
      int ex = 0;
      if (cmax > 0.f) frexpf(cmax, &ex);
      ec = 14 - ex;
    }
    uint32_t li = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++li) {
      const WorkItem w = work_item(p, item);
      const int xs0 = (int)(li % Cfg::XB) * G;
      const int split = item % p.splits;
      // Prepare tile g of the group in shared memory, all 256 epilogue threads on it: 3xTF32
      // splits X into tf32 hi / lo halves, TF32 rounds it to tf32; the TF32 product first scales
      // row j by 2^er(j) so that S and R come out inside the fp16 range of the second MMA
      // (|S_ji| <= |x_j| max_i |F_i| < 2^15 after scaling) and keeps er(j) for the Y readout (two
      // sets of exponents, by group parity).
      auto prep_tile = [&](int g) -> bool {
        const int xs = xs0 + g;
        if (!warp_wait(&x_full[xs], (xslot_par >> xs) & 1u, abort_flag, p.err, DEV_TIMEOUT_X,
                       p.timeout_ns)) return false;
        uint8_t* xt = sX + xs * Cfg::XBUF_BYTES;
        const int et = threadIdx.x - 64;  // epilogue thread 0..255
        if constexpr (X3) {
          float4* xh = reinterpret_cast<float4*>(xt);
          float4* xl = reinterpret_cast<float4*>(xt + Cfg::X_BYTES);
#pragma unroll 2
          for (int i = et; i < Cfg::X_BYTES / 16; i += Cfg::EPI_THREADS) {
            const float4 v = xh[i];
            const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
            xh[i] = h;
            xl[i] = make_float4(tf32_lo(v.x, h.x), tf32_lo(v.y, h.y), tf32_lo(v.z, h.z),
                                tf32_lo(v.w, h.w));
          }
        } else if constexpr (Cfg::ROW_SCALE) {
          // UPR consecutive threads share a row, one 16-byte unit each (within a row the swizzle
          // only permutes the units)
          constexpr int UPR = DP / 4;
          constexpr int UPS = Cfg::XW / 16;  // units per row of one 128 B sub-tile
          static_assert(UPR <= 32 && 32 % UPR == 0 && (Cfg::TM * UPR) % Cfg::EPI_THREADS == 0,
                        "units per row");
          const int ers = ((li & 1) * G + g) * Cfg::TM;
#pragma unroll
          for (int i = et; i < Cfg::TM * UPR; i += Cfg::EPI_THREADS) {
            const int row = i / UPR, u = i % UPR;
            uint4* q = reinterpret_cast<uint4*>(xt + (u / UPS) * Cfg::TM * Cfg::XW + row * Cfg::XW) +
                       u % UPS;
            uint4 v = *q;
            const float a = __uint_as_float(v.x), b = __uint_as_float(v.y);
            const float c = __uint_as_float(v.z), d = __uint_as_float(v.w);
            float n2 = fmaf(a, a, fmaf(b, b, fmaf(c, c, d * d)));
#pragma unroll
            for (int o = 1; o < UPR; o <<= 1) n2 += __shfl_xor_sync(0xffffffffu, n2, o);
            // frexp exponent of the bound (zero: none); 2^er and 2^-er stay normal floats
            const float bound = sqrtf(n2) * fmax * 1.001f;
            const int ex = bound > 0.f ? ((__float_as_int(bound) >> 23) & 0xff) - 126 : 0;
            const int e = p.step ? 0 : min(120, max(-120, 14 - ex));  // step values: 0 or 1
            const float sc = __int_as_float((127 + e) << 23);
            v.x = tf32_rne_bits(__float_as_uint(a * sc));
            v.y = tf32_rne_bits(__float_as_uint(b * sc));
            v.z = tf32_rne_bits(__float_as_uint(c * sc));
            v.w = tf32_rne_bits(__float_as_uint(d * sc));
            *q = v;
            if (u == 0) er_s[ers + row] = (int8_t)e;
          }
        } else if constexpr (Cfg::ROUND) {
          round_tf32_smem<Cfg::X_BYTES / 16, Cfg::EPI_THREADS>(xt, et);
        }
        fence_proxy_async_smem();
        warp_arrive(&x_ready[xs], lane);
        if (lane == 0 && warp == 2) SB_TR(24, li * G + g);
        return true;
      };
      // Y readout of tile gi (product mode): scaled back, written to this split's partial rows
      auto readout = [&](int gi) -> bool {
        if constexpr (!REDUCE) {
          if (!warp_wait(&y_full[gi], (slot_par >> gi) & 1u, abort_flag, p.err, DEV_TIMEOUT_Y,
                         p.timeout_ns)) return false;
          tc_fence_after();
          if (warp == 2 && lane == 0) SB_TR(12, gi);
          const int row = (w.tile0 + gi) * Cfg::TM + row_in_tile;
          float inv = 1.f;
          if constexpr (Cfg::ROW_SCALE) {
            // the row's exponent, written by whichever thread prepared the row: every warp's
            // x_ready arrival for the slot is complete by now (the wait orders the exponent's
            // write before this read); the next group writes the other set
            const int xs = xs0 + gi;
            if (!warp_wait(&x_ready[xs], (xslot_par >> xs) & 1u, abort_flag, p.err, DEV_TIMEOUT_X,
                           p.timeout_ns)) return false;
            const int er = er_s[((li & 1) * G + gi) * Cfg::TM + row_in_tile];
            inv = __int_as_float((127 - er - ec) << 23);
          }
          float* out = p.ws + ((size_t)split * p.M + (size_t)(row < p.M ? row : 0)) * DP;
          // the two warps of a quadrant share the 16-column pieces of Y
#pragma unroll 1
          for (int col = half * 16; col < DP; col += 32) {
            float y[16];
            tmem_ld16(tbase + lane_addr + Cfg::TMEM_Y + gi * DP + col, y);
            tmem_ld_wait_regs16(y);
            if constexpr (Cfg::MS == 2) {
              float y2[16];
              tmem_ld16(tbase + lane_addr + Cfg::TMEM_Y + (G + gi) * DP + col, y2);
              tmem_ld_wait_regs16(y2);
#pragma unroll
              for (int i = 0; i < 16; ++i) y[i] += y2[i];
            }
            if (row < p.M) {
              float4* o4 = reinterpret_cast<float4*>(out + col);
#pragma unroll
              for (int i = 0; i < 4; ++i)
                o4[i] = make_float4(y[4 * i] * inv, y[4 * i + 1] * inv, y[4 * i + 2] * inv,
                                    y[4 * i + 3] * inv);
            }
          }
          tc_fence_before();
          warp_arrive(&y_empty[gi], lane);
          if (warp == 2 && lane == 0) SB_TR(13, gi);
        }
        return true;
      };
      // In the first chunk the tiles are prepared XPRE_AHEAD pairs ahead of the pair being read
      // (the first MMA starts on a tile as soon as it is ready, and the next tiles are prepared
      // while it runs); in the last chunk each tile's Y is read out behind the next tile's pair,
      // so that the readout overlaps the last MMAs.
      constexpr int XPRE_AHEAD = 2;
      int prepped = 0;
      for (int c = w.c0; c < w.c1 && ok; ++c) {
        for (int gi = 0; gi < w.ntiles; ++gi, ++pair) {
          for (; prepped < w.ntiles && prepped <= gi + XPRE_AHEAD; ++prepped)
            if (!prep_tile(prepped)) { ok = false; break; }
          if (!ok) break;
          uint32_t buf, use;
          pair_slot<Cfg>(pair, buf, use);
          if (!warp_wait(&s_full[buf], use & 1, abort_flag, p.err, DEV_TIMEOUT_SFULL,
                         p.timeout_ns)) { ok = false; break; }
          tc_fence_after();
          if (warp == 2 && lane == 0) SB_TR(3, pair);
          const uint32_t s_tm = tbase + lane_addr + buf * BN + half * Cfg::EPI_COLS;
          float v[Cfg::EPI_COLS];
          if constexpr (Cfg::LDW == 32) {
#pragma unroll
            for (int col = 0; col < Cfg::EPI_COLS; col += 32) tmem_ld32(s_tm + col, v + col);
            tmem_ld_wait_all<Cfg::EPI_COLS>(v);
          } else {
            tmem_ld16(s_tm, v);
            tmem_ld_wait_regs16(v);
          }
          if constexpr (REDUCE) {
            float cs = 0.f, cs2 = 0.f;
            if (p.count) {
              float cn = 0.f;
#pragma unroll
              for (int i = 0; i < Cfg::EPI_COLS; ++i) {
                const float r = fmaxf(v[i], 0.f);
                cs += r;
                cs2 = fmaf(r, r, cs2);
                cn += v[i] > 0.f ? 1.f : 0.f;
              }
              acc_n += (double)cn;
            } else {
#pragma unroll
              for (int i = 0; i < Cfg::EPI_COLS; ++i) {
                const float r = fmaxf(v[i], 0.f);
                cs += r;
                cs2 = fmaf(r, r, cs2);
              }
            }
            acc_s += (double)cs;
            acc_s2 += (double)cs2;
          } else if constexpr (X3) {
            const uint32_t lo_tm =
                tbase + lane_addr + Cfg::TMEM_S_LO + buf * BN + half * Cfg::EPI_COLS;
#pragma unroll
            for (int col = 0; col < Cfg::EPI_COLS; col += Cfg::LDW) {
              float lo[Cfg::LDW];
#pragma unroll
              for (int i = 0; i < Cfg::LDW; ++i) {
                const float r = p.step ? (v[col + i] > 0.f ? 1.f : 0.f) : fmaxf(v[col + i], 0.f);
                const float h = tf32_hi(r);
                lo[i] = tf32_lo(r, h);
                v[col + i] = h;
              }
              if constexpr (Cfg::LDW == 32) {
                tmem_st32(s_tm + col, v + col);
                tmem_st32(lo_tm + col, lo);
              } else {
                tmem_st16(s_tm + col, v + col);
                tmem_st16(lo_tm + col, lo);
              }
            }
            tmem_st_wait();
          } else if constexpr (!Cfg::H16) {
            // plain TF32 second MMA: R = ReLU(S) in place (the tensor core reads it as tf32)
#pragma unroll
            for (int col = 0; col < Cfg::EPI_COLS; col += Cfg::LDW) {
#pragma unroll
              for (int i = 0; i < Cfg::LDW; ++i)
                v[col + i] = p.step ? (v[col + i] > 0.f ? 1.f : 0.f) : fmaxf(v[col + i], 0.f);
              if constexpr (Cfg::LDW == 32) tmem_st32(s_tm + col, v + col);
              else tmem_st16(s_tm + col, v + col);
            }
            tmem_st_wait();
          } else {
            // pack ReLU(R) (scaled) as fp16 pairs (even k in the low half) into this warp's own
            // first EPI_COLS / 2 columns
            // S is already scaled by 2^er (X was scaled in shared memory)
            uint32_t pk[Cfg::EPI_COLS / 2];
            if (p.step) {
#pragma unroll
              for (int i = 0; i < Cfg::EPI_COLS / 2; ++i)
                pk[i] = (v[2 * i] > 0.f ? 0x3C00u : 0u) | (v[2 * i + 1] > 0.f ? 0x3C000000u : 0u);
            } else {
#pragma unroll
              for (int i = 0; i < Cfg::EPI_COLS / 2; ++i)
                pk[i] = pack_relu_h2(v[2 * i], v[2 * i + 1]);
            }
            if constexpr (Cfg::EPI_COLS / 2 == 32) tmem_st32(s_tm, reinterpret_cast<const float*>(pk));
            else tmem_st16(s_tm, reinterpret_cast<const float*>(pk));
            tmem_st_wait();
          }
          tc_fence_before();
          warp_arrive(&r_ready[buf], lane);
          if (lane == 0 && warp == 2) SB_TR(5, pair);
          if (lane == 0 && warp == 9) SB_TR(6, pair);
          if (lane == 0) SB_TR(16 + warp - 2, pair);
          if (c == w.c1 - 1 && gi > 0 && !readout(gi - 1)) { ok = false; break; }
        }
      }
      if (!ok) break;
      if (!readout(w.ntiles - 1)) { ok = false; break; }
      slot_par ^= (1u << w.ntiles) - 1u;
      xslot_par ^= ((1u << w.ntiles) - 1u) << xs0;
    }
    if constexpr (REDUCE) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc_s += __shfl_xor_sync(0xffffffffu, acc_s, o);
        acc_s2 += __shfl_xor_sync(0xffffffffu, acc_s2, o);
        acc_n += __shfl_xor_sync(0xffffffffu, acc_n, o);
      }
      if (lane == 0) {
        red[(warp - 2) * 3 + 0] = acc_s;
        red[(warp - 2) * 3 + 1] = acc_s2;
        red[(warp - 2) * 3 + 2] = acc_n;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(Cfg::EPI_THREADS) : "memory");
      if (threadIdx.x == 64) {
        double a = 0.0, b = 0.0, c = 0.0;
        for (int wi = 0; wi < Cfg::EPI_WARPS; ++wi) {
          a += red[3 * wi];
          b += red[3 * wi + 1];
          c += red[3 * wi + 2];
        }
        const int stride = p.count ? 3 : 2;
        p.partials[stride * blockIdx.x + 0] = a;
        p.partials[stride * blockIdx.x + 1] = b;
        if (p.count) p.partials[stride * blockIdx.x + 2] = c;
      }
    }
  } else if (Cfg::ROUND && warp == Cfg::CPREP_WARP) {
    if constexpr (Cfg::ROUND) {
    // ------------------------------------------------------------------ chunk prep (TF32 mode)
    // rounds the F chunk to tf32 in place; product mode: fp32 C chunk (32-float SW128 sub-tiles)
    // -> fp16 scaled by 2^ec (64-element SW128 sub-tiles), or (Dp = 256) C rounded in place
    float cscale = 1.f;
    const bool idle = REDUCE && p.f_rounded;  // nothing to prepare: the MMA waits the TMA
    if constexpr (Cfg::H16) {
      const float cmax = stats_max(p.stats, p.nstats, 1);
      int ex = 0;
      if (cmax > 0.f) frexpf(cmax, &ex);
      cscale = ldexpf(1.f, 14 - ex);
    }
    uint32_t gch = 0;
    bool ok = !idle;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x) {
      const WorkItem w = work_item(p, item);
      for (int c = w.c0; c < w.c1; ++c, ++gch) {
        const int stage = gch % STAGES;
        const uint32_t round = gch / STAGES;
        if (!warp_wait(&full[stage], round & 1, abort_flag, p.err, DEV_TIMEOUT_FULL, p.timeout_ns)) {
          ok = false;
          break;
        }
        uint8_t* stg = sStage + stage * Cfg::STAGE_ALLOC;
        if (!p.f_rounded) round_tf32_smem<Cfg::F_BYTES / 16, 32>(stg, lane);
        if constexpr (!REDUCE && !Cfg::H16) round_tf32_smem<Cfg::C_BYTES / 16, 32>(stg + Cfg::F_BYTES, lane);
        if constexpr (Cfg::H16) {
        const uint8_t* src = stg + Cfg::F_BYTES;
        uint8_t* dst = stg + Cfg::STAGE_BYTES;
        constexpr int UNITS = (BN / 64) * DP * 8;  // 16-byte fp16 units
        static_assert(UNITS % 32 == 0, "whole rounds of the converter warp");
        // batches of UB units per lane: all loads of a batch are issued before its stores, so
        // they are in flight together (source and destination share the shared-memory array,
        // so the compiler would not hoist loads above earlier stores by itself); at Dp = 64
        // with 2-tile groups the converter otherwise paces the kernel
        constexpr int PER_LANE = UNITS / 32;
        constexpr int UB = PER_LANE < 8 ? PER_LANE : 8;
        static_assert(PER_LANE % UB == 0, "converter batches");
        for (int b0 = 0; b0 < PER_LANE; b0 += UB) {
          float4 va[UB], vb[UB];
#pragma unroll
          for (int q = 0; q < UB; ++q) {
            const int uidx = lane + 32 * (b0 + q);
            const int u = uidx & 7;
            const int r = (uidx >> 3) % DP;
            const int k0 = 64 * ((uidx >> 3) / DP) + 8 * u;
            const int s32 = k0 >> 5, v0 = (k0 & 31) >> 2;
            const uint8_t* rowp = src + s32 * (DP * 128) + r * 128;
            va[q] = *reinterpret_cast<const float4*>(rowp + ((v0 ^ (r & 7)) << 4));
            vb[q] = *reinterpret_cast<const float4*>(rowp + (((v0 + 1) ^ (r & 7)) << 4));
          }
#pragma unroll
          for (int q = 0; q < UB; ++q) {
            const int uidx = lane + 32 * (b0 + q);
            const int u = uidx & 7;
            const int r = (uidx >> 3) % DP;
            const int s16 = (uidx >> 3) / DP;
            __half2 h[4] = {__floats2half2_rn(va[q].x * cscale, va[q].y * cscale),
                            __floats2half2_rn(va[q].z * cscale, va[q].w * cscale),
                            __floats2half2_rn(vb[q].x * cscale, vb[q].y * cscale),
                            __floats2half2_rn(vb[q].z * cscale, vb[q].w * cscale)};
            *reinterpret_cast<uint4*>(dst + s16 * (DP * 128) + r * 128 + ((u ^ (r & 7)) << 4)) =
                *reinterpret_cast<const uint4*>(h);
          }
        }
        }
        fence_proxy_async_smem();
        warp_arrive(&c16_ready[stage], lane);
        if (lane == 0) SB_TR(11, gch);
      }
    }
    }
  } else if (warp == Cfg::XLOAD_WARP) {
    // ------------------------------------------------------------------ X loader
    // Group k's tiles go to X slot set k % XB; lane g loads tile g as soon as the MMAs of the
    // slot's previous group have completed (with two sets, while the previous group still runs)
    uint32_t slot_par = 0;    // bit xs: parity of the number of earlier uses of X slot xs
    uint32_t slot_used = 0;   // bit xs: slot used by an earlier group
    uint32_t issued = 0, issued_par = 0;  // this lane's copies (drained on abort)
    bool ok = true;
    uint32_t li = 0;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++li) {
      const WorkItem w = work_item(p, item);
      const int xs0 = (int)(li % Cfg::XB) * G;
      bool lok = true;
      if (lane < w.ntiles) {
        const int xs = xs0 + lane;
        if ((slot_used >> xs) & 1u)
          lok = mbar_wait(&x_empty[xs], ((slot_par >> xs) & 1u) ^ 1u, abort_flag, p.err,
                          DEV_TIMEOUT_X, p.timeout_ns);
        if (lok) {
          uint8_t* xdst = sX + xs * Cfg::XBUF_BYTES;
          mbar_arrive_expect_tx(&x_full[xs], Cfg::X_BYTES);
#pragma unroll
          for (int sub = 0; sub < Cfg::KSUB; ++sub)
            tma_load_2d(xdst + sub * Cfg::TM * Cfg::XW, &tmX, sub * Cfg::BOX_K,
                        (w.tile0 + lane) * Cfg::TM, &x_full[xs]);
          issued |= 1u << xs;
          issued_par = (issued_par & ~(1u << xs)) | (((slot_par >> xs) & 1u) << xs);
          SB_TR(14, li * G + lane);
        }
      }
      if (!__all_sync(0xffffffffu, lok)) { ok = false; break; }
      const uint32_t mask = ((1u << w.ntiles) - 1u) << xs0;
      slot_par ^= mask;
      slot_used |= mask;
    }
    if (*abort_flag) {
      // wait (bounded) for this lane's copies still in flight before leaving
      for (int xs = 0; xs < Cfg::NXS; ++xs)
        if ((issued >> xs) & 1u) mbar_drain(&x_full[xs], (issued_par >> xs) & 1u);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) SB_TR(15, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace sb
