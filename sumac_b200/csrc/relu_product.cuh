// relu_product.cuh — the fused ReLU(X F^T) contraction on tcgen05 (sm_100a).
//
// One persistent, warp-specialised kernel computes, for a row tile of X (128 rows) and a range
// of chunks of the fixed operand F (BN rows each):
//
//   product mode:  Y[rows, :Dp] = sum_chunks ReLU(X_tile F_chunk^T) C_chunk          (C = Ct^T)
//   reduce  mode:  (sum ReLU(X F^T), sum ReLU(X F^T)^2)  over the whole X x F product
//
// which is relu_bat_c (src/sumac/kernels/tuning/relu_bat_c/relu_bat_c_base.py:4-6, with
// B -> X, A -> F) and relu_bat_reduce (src/sumac/kernels/tuning/relu_bat_reduce/
// relu_bat_reduce.py:11-22, with A -> X, B -> F). The m x n intermediate never leaves the SM:
//
//   warp 0       TMA producer: X tile per work item (double-buffered where shared memory
//                allows), (F chunk, C^T chunk) per pipeline stage
//   warp 1       MMA issuer (one thread): S = X F^T into one of NBUF TMEM buffers (kind::tf32);
//                NBUF-1 chunks later, once the epilogue has rewritten S as R = ReLU(S) in place,
//                Y += R C with R read straight from TMEM (the [d], [a_tmem], b_desc form). Y is
//                double-buffered across work items.
//   warps 2..9   epilogue, two warps per TMEM lane quadrant, each on half of the columns:
//                tcgen05.ld S -> ReLU -> tcgen05.st R (or accumulate the sums), and the final
//                tcgen05.ld of Y -> global
//   warp 10      (3xTF32 only) splits each X tile into tf32 hi / lo halves in shared memory
//
// Cost model (measured on B200, tf32, M=128, K=8): an MMA costs ~45-50 cycles for N <= 64 and
// reaches the full rate only at N >= 128; it is bound by streaming ~4.5 KB of operands per
// instruction. The second MMA (N = Dp) therefore streams R (128 x BN fp32 per chunk) at operand
// bandwidth and dominates at small rank; everything else is kept off its critical path.
//
// Precision: X3=false is plain TF32 (the tensor core reads the fp32 bits as tf32). X3=true is
// the 3xTF32 split (x = hi + lo with hi = x with the low 13 mantissa bits cleared), giving fp32
// accuracy: S = Xlo Fhi + Xhi Flo + Xhi Fhi and Y += Rlo Chi + Rhi Clo + Rhi Chi.
//
// Shared-memory operands are K-major with the TMA swizzle matching the row width (64 B rows:
// SWIZZLE_64B, 128 B rows: SWIZZLE_128B; wider rows are split in 128 B sub-tiles).
// No TMA multicast is used anywhere. Every wait is bounded (see mbar_wait).
#pragma once
#include "kernels.cuh"
#include <cuda_fp16.h>

#include "sm100.cuh"

namespace sb {

struct ProductParams {
  int M;                 // rows of X
  int N;                 // rows of F (columns of C^T)
  int n_chunks;          // ceil(N / BN)
  int splits;            // chunk ranges per row tile (split-K); items = tiles * splits
  int chunks_per_split;  // ceil(n_chunks / splits)
  int n_tiles;           // ceil(M / 128)
  float* ws;             // product mode: [splits][M][DP] partial outputs
  double* partials;      // reduce mode: [gridDim.x][2] per-CTA (sum, sum of squares)
  int* err;              // device error word (0 = ok)
  unsigned long long timeout_ns;
  // Fused finalize (product mode, splits == 1, DP <= 32): when fin.mode != FIN_NONE the epilogue
  // applies the support correction and the per-mode update of kernels.cu's finalize pass to each
  // row as soon as its Y is complete, instead of writing Y to `ws`.
  int fuse;              // 0: write ws; 1: apply `fin` in the epilogue
  FinalizeArgs fin;
  // TF32 product mode: the second MMA runs in fp16 (kind::f16, same 10-bit mantissa as tf32,
  // K = 16 per instruction). stats[0] = bits of max_i |F_i| (row norm), stats[1] = bits of
  // max |C|; R rows and C are scaled by exact powers of two so that no fp16 value overflows.
  const float* Xg;                // X in global memory (row norms for the R scale)
  const unsigned int* stats;
};

template <int DP, int BN, int STAGES, bool X3, bool REDUCE, int NXB>
struct ProductCfg {
  static_assert(DP == 16 || DP == 32 || DP == 64 || DP == 128 || DP == 256, "DP");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static_assert(NXB == 1 || NXB == 2, "X buffers");
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
  static constexpr bool H16 = !X3 && !REDUCE;                     // fp16 second MMA
  static constexpr int C16_BYTES = H16 ? DP * BN * 2 : 0;         // fp16 copy of the C chunk
  static constexpr int STAGE_ALLOC = STAGE_BYTES + C16_BYTES;
  static constexpr int XBUF_BYTES = NPREC * X_BYTES;      // one X buffer (hi [, lo])
  static constexpr int X_TOTAL = NXB * XBUF_BYTES;
  static constexpr int SMEM_DATA = X_TOTAL + STAGES * STAGE_ALLOC;
  static constexpr int SMEM_BYTES_RAW = SMEM_DATA + 1024 /*barriers*/ + 1024 /*align slack*/;
  // at least 120 KB so that only one CTA (and one 512-column TMEM allocation) lives on an SM
  static constexpr int SMEM_BYTES = SMEM_BYTES_RAW < 122880 ? 122880 : SMEM_BYTES_RAW;
  static_assert(SMEM_BYTES_RAW <= 232448, "shared memory budget");
  static constexpr int NBUF = 3;                          // S buffers in TMEM
  // chunks by which the second MMA trails the first; the stage of chunk c is released by the
  // second MMA of c, which is issued after the first MMA of c + LAG, so LAG < STAGES
  static constexpr int LAG = (NBUF < STAGES ? NBUF : STAGES) - 1;
  static constexpr int TMEM_S_LO = NBUF * BN;             // lo halves of R (3xTF32)
  static constexpr int TMEM_Y = (X3 ? 2 : 1) * NBUF * BN; // two Y accumulators follow
  static_assert(REDUCE ? NBUF * BN <= 512 : TMEM_Y + 2 * DP <= 512, "TMEM budget");
  static_assert(REDUCE || STAGES >= 2, "product mode needs two stages (MMA2 lags MMA1)");
  static constexpr uint32_t IDESC1 = umma_idesc_tf32(TM, BN);
  static constexpr uint32_t IDESC2 = umma_idesc_tf32(TM, DP);
  // kind::f16: f32 accumulate, A and B f16, both K-major
  static constexpr uint32_t IDESC2_F16 =
      (1u << 4) | ((uint32_t)(DP >> 3) << 17) | ((uint32_t)(TM >> 4) << 24);
  static constexpr int EPI_WARPS = 8;                     // two per TMEM lane quadrant
  static constexpr int EPI_THREADS = 32 * EPI_WARPS;
  static constexpr int THREADS = 64 + EPI_THREADS + ((X3 || H16) ? 32 : 0);
  static constexpr int EPI_COLS = BN / 2;                 // S columns per epilogue warp
  static_assert(EPI_COLS % 16 == 0, "epilogue column split");
  static constexpr int LDW = EPI_COLS % 32 == 0 ? 32 : 16;  // tcgen05.ld/st width used
};

// The finalize pass of kernels.cu for one row j whose Y (DP values) is in registers: support
// correction with L = <X_j, F_i> (fp32) and the FIN_SALSA / FIN_GRAD / FIN_STORE update.
template <int DP>
__device__ __forceinline__ void epilogue_finalize(const FinalizeArgs& a, int64_t j, const float* y) {
  float x[DP], cor[DP];
  const float4* xr = reinterpret_cast<const float4*>(a.X + j * DP);
#pragma unroll
  for (int c = 0; c < DP / 4; ++c) {
    const float4 v = xr[c];
    x[4 * c] = v.x; x[4 * c + 1] = v.y; x[4 * c + 2] = v.z; x[4 * c + 3] = v.w;
  }
#pragma unroll
  for (int c = 0; c < DP; ++c) cor[c] = 0.f;
  if (a.rowptr) {
    const int e0 = a.rowptr[j], e1 = a.rowptr[j + 1];
    for (int e = e0; e < e1; ++e) {
      const int2 en = a.ent[e];
      const float4* fr = reinterpret_cast<const float4*>(a.F + (int64_t)en.x * DP);
      const float4* cr = reinterpret_cast<const float4*>(a.Cm + (int64_t)en.x * DP);
      float L = 0.f;
#pragma unroll
      for (int c = 0; c < DP / 4; ++c) {
        const float4 f = fr[c];
        L = fmaf(x[4 * c], f.x, L);
        L = fmaf(x[4 * c + 1], f.y, L);
        L = fmaf(x[4 * c + 2], f.z, L);
        L = fmaf(x[4 * c + 3], f.w, L);
      }
      const float val = __int_as_float(en.y);
      const float coef = (a.mode == FIN_SALSA) ? (val - L + fmaxf(L, 0.f)) : (L - val - fmaxf(L, 0.f));
#pragma unroll
      for (int c = 0; c < DP / 4; ++c) {
        const float4 cv = cr[c];
        cor[4 * c] = fmaf(coef, cv.x, cor[4 * c]);
        cor[4 * c + 1] = fmaf(coef, cv.y, cor[4 * c + 1]);
        cor[4 * c + 2] = fmaf(coef, cv.z, cor[4 * c + 2]);
        cor[4 * c + 3] = fmaf(coef, cv.w, cor[4 * c + 3]);
      }
    }
  }
  if (a.mode == FIN_SALSA) {
    const float mu = a.momentum, one_m_mu = 1.0f - mu, ub = *a.unbias;
    float4* xw = reinterpret_cast<float4*>(a.X + j * DP);
    float4* dw = reinterpret_cast<float4*>(a.dX + j * DP);
#pragma unroll
    for (int c = 0; c < DP / 4; ++c) {
      const float4 dx = dw[c];
      const float dxv[4] = {dx.x, dx.y, dx.z, dx.w};
      float nx[4], ndx[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = 4 * c + u;
        const float lsq = (x[i] - y[i]) + cor[i];
        ndx[u] = (lsq - x[i]) * one_m_mu + dxv[u] * mu;
        nx[u] = x[i] + a.lrate * ndx[u] / ub;
      }
      xw[c] = make_float4(nx[0], nx[1], nx[2], nx[3]);
      dw[c] = make_float4(ndx[0], ndx[1], ndx[2], ndx[3]);
    }
  } else if (a.mode == FIN_STORE) {
    const int64_t orow = a.out_rows ? a.out_rows[j] : j;
    float* o = a.out + orow * a.ld_out;
#pragma unroll
    for (int c = 0; c < DP; ++c)
      if (c < a.out_d) o[c] = y[c] + cor[c];
  } else {
    const int64_t orow = a.out_rows ? a.out_rows[j] : j;
    float4* o = reinterpret_cast<float4*>(a.out + orow * DP);
#pragma unroll
    for (int c = 0; c < DP / 4; ++c) {
      float4 r = make_float4(a.scale * (y[4 * c] + cor[4 * c]), a.scale * (y[4 * c + 1] + cor[4 * c + 1]),
                             a.scale * (y[4 * c + 2] + cor[4 * c + 2]), a.scale * (y[4 * c + 3] + cor[4 * c + 3]));
      if (a.accumulate) {
        const float4 old = o[c];
        r.x += old.x; r.y += old.y; r.z += old.z; r.w += old.w;
      }
      o[c] = r;
    }
  }
}

template <int DP, int BN, int STAGES, bool X3, bool REDUCE, int NXB>
__global__ void __launch_bounds__(ProductCfg<DP, BN, STAGES, X3, REDUCE, NXB>::THREADS, 1)
    relu_product_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmFhi,
                        const __grid_constant__ CUtensorMap tmFlo,
                        const __grid_constant__ CUtensorMap tmChi,
                        const __grid_constant__ CUtensorMap tmClo, const ProductParams p) {
  using Cfg = ProductCfg<DP, BN, STAGES, X3, REDUCE, NXB>;
  constexpr int NBUF = Cfg::NBUF;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem;                                   // [NXB][NPREC][X_BYTES]
  uint8_t* sStage = smem + Cfg::X_TOTAL;                // [STAGES][STAGE_ALLOC]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_DATA);
  uint64_t* full = bars;                    // [STAGES]
  uint64_t* empty = full + STAGES;          // [STAGES]
  uint64_t* s_full = empty + STAGES;        // [NBUF]
  uint64_t* r_ready = s_full + NBUF;        // [NBUF]
  uint64_t* x_full = r_ready + NBUF;        // [2]
  uint64_t* x_empty = x_full + 2;           // [2]
  uint64_t* x_ready = x_empty + 2;          // [2]
  uint64_t* y_full = x_ready + 2;           // [2]
  uint64_t* y_empty = y_full + 2;           // [2]
  uint64_t* drain = y_empty + 2;
  uint64_t* c16_ready = drain + 1;          // [STAGES] fp16 C chunk converted (H16)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(c16_ready + STAGES);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  double* red = reinterpret_cast<double*>(smem + Cfg::SMEM_DATA + 512);  // [EPI_WARPS][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.n_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&r_ready[b], Cfg::EPI_THREADS);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&x_full[b], 1);
      mbar_init(&x_empty[b], 1);
      mbar_init(&x_ready[b], 32);
      mbar_init(&y_full[b], 1);
      mbar_init(&y_empty[b], Cfg::EPI_THREADS);
    }
    mbar_init(drain, 1);
    for (int s = 0; s < STAGES; ++s) mbar_init(&c16_ready[s], 32);
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
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    // Copies issued by one thread complete one after another (~600 cycles each from L2 on
    // B200), copies from different threads overlap: lane s owns pipeline stage s and issues its
    // loads, lane 31 loads the X tiles, so STAGES + 1 copy streams are in flight.
    const bool x_lane = lane == 31;
    const bool stage_lane = lane < STAGES;
    uint32_t fills = 0;   // loads this lane issued into its stage (stage lanes)
    int t = 0;
    bool ok = true;
    uint32_t g = 0;       // global chunk counter, identical in every lane
    if (stage_lane || x_lane) {
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++t) {
        const int tile = item / p.splits, split = item % p.splits;
        const int c0 = split * p.chunks_per_split;
        const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
        if (x_lane) {
          const int xb = t % NXB;
          if (t >= NXB && !mbar_wait(&x_empty[xb], ((t / NXB) - 1) & 1, abort_flag, p.err,
                                     DEV_TIMEOUT_X, p.timeout_ns)) { ok = false; break; }
          uint8_t* xdst = sX + xb * Cfg::XBUF_BYTES;
          mbar_arrive_expect_tx(&x_full[xb], Cfg::X_BYTES);
#pragma unroll
          for (int s = 0; s < Cfg::KSUB; ++s)
            tma_load_2d(xdst + s * Cfg::TM * Cfg::XW, &tmX, s * Cfg::BOX_K, tile * Cfg::TM,
                        &x_full[xb]);
          continue;
        }
        for (int c = c0; c < c1; ++c, ++g) {
          const int stage = g % STAGES;
          if (stage != lane) continue;
          const uint32_t round = g / STAGES;
          // a stage is free once the empty barrier completed its previous round
          if (round > 0 && !mbar_wait(&empty[stage], (round - 1) & 1, abort_flag, p.err,
                                      DEV_TIMEOUT_EMPTY, p.timeout_ns)) { ok = false; break; }
          uint8_t* st = sStage + stage * Cfg::STAGE_ALLOC;
          mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
#pragma unroll
          for (int h = 0; h < Cfg::NPREC; ++h) {
            const CUtensorMap* tf = h == 0 ? &tmFhi : &tmFlo;
            uint8_t* fdst = st + h * Cfg::F_BYTES;
#pragma unroll
            for (int s = 0; s < Cfg::KSUB; ++s)
              tma_load_2d(fdst + s * BN * Cfg::XW, tf, s * Cfg::BOX_K, c * BN, &full[stage]);
            if (!REDUCE) {
              const CUtensorMap* tc = h == 0 ? &tmChi : &tmClo;
              uint8_t* cdst = st + Cfg::NPREC * Cfg::F_BYTES + h * Cfg::C_BYTES;
#pragma unroll
              for (int s = 0; s < BN / 32; ++s)
                tma_load_2d(cdst + s * DP * 128, tc, c * BN + s * 32, 0, &full[stage]);
            }
          }
          ++fills;
        }
      }
      if (*abort_flag) {
        // wait (bounded) for this lane's own copies still in flight before leaving
        if (stage_lane && fills > 0) mbar_drain(&full[lane], (fills - 1) & 1);
        if (x_lane)
          for (int u = 1; u <= NXB && u <= t; ++u)
            mbar_drain(&x_full[(t - u) % NXB], ((t - u) / NXB) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      uint32_t buf_uses[NBUF];
#pragma unroll
      for (int b = 0; b < NBUF; ++b) buf_uses[b] = 0;
      uint32_t gchunk = 0;  // global chunk counter -> S buffer = gchunk % NBUF
      bool ok = true;
      const uint32_t sX_addr = smem_u32(sX);
      const uint32_t sSt_addr = smem_u32(sStage);
      // FIFO of chunks whose second MMA is still to be issued (product mode)
      struct Pend {
        int stage, buf, t;
        uint32_t use, sphase;
        bool first, last;
      };
      Pend q[NBUF];
      int qh = 0, qn = 0;
      auto issue_second = [&](const Pend& e) -> bool {
        if (!mbar_wait(&r_ready[e.buf], e.use & 1, abort_flag, p.err, DEV_TIMEOUT_RREADY,
                       p.timeout_ns)) return false;
        const int yb = e.t & 1;
        if (e.first && e.t >= 2) {
          if (!mbar_wait(&y_empty[yb], ((e.t >> 1) - 1) & 1, abort_flag, p.err, DEV_TIMEOUT_Y,
                         p.timeout_ns)) return false;
        }
        if (Cfg::H16 && !mbar_wait(&c16_ready[e.stage], e.sphase, abort_flag, p.err,
                                   DEV_TIMEOUT_FULL, p.timeout_ns)) return false;
        tc_fence_after();
        const uint32_t cbase = sSt_addr + e.stage * Cfg::STAGE_ALLOC + Cfg::NPREC * Cfg::F_BYTES;
        const uint32_t s_hi = tbase + e.buf * BN;
        const uint32_t s_lo = tbase + Cfg::TMEM_S_LO + e.buf * BN;
        const uint32_t ytm = tbase + Cfg::TMEM_Y + yb * DP;
        if constexpr (Cfg::H16) {
          // R packed as fp16 pairs: warp half h holds k in [h*EPI_COLS, (h+1)*EPI_COLS) in its
          // own first EPI_COLS/2 columns; C in fp16, 64-element 128 B swizzled sub-tiles
          const uint32_t c16 = sSt_addr + e.stage * Cfg::STAGE_ALLOC + Cfg::STAGE_BYTES;
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk) {
            const int hh = (16 * kk) / Cfg::EPI_COLS;
            const uint32_t acol = hh * Cfg::EPI_COLS + (16 * kk - hh * Cfg::EPI_COLS) / 2;
            const uint32_t off = (kk >> 2) * (DP * 128) + (kk & 3) * 32;
            const uint64_t bd = umma_sdesc(c16 + off, 16, 1024, UMMA_SW128);
            mma_f16_ts(ytm, s_hi + acol, bd, Cfg::IDESC2_F16, (e.first && kk == 0) ? 0u : 1u);
          }
          mma_commit(&empty[e.stage]);
          if (e.last) mma_commit(&y_full[yb]);
          return true;
        }
#pragma unroll
        for (int kk = 0; kk < BN / 8; ++kk) {
          const uint32_t off = (kk >> 2) * (DP * 128) + (kk & 3) * 32;
          const uint64_t bhi = umma_sdesc(cbase + off, 16, 1024, UMMA_SW128);
          const uint32_t acc0 = (e.first && kk == 0) ? 0u : 1u;
          if (X3) {
            const uint64_t blo = umma_sdesc(cbase + Cfg::C_BYTES + off, 16, 1024, UMMA_SW128);
            mma_tf32_ts(ytm, s_lo + kk * 8, bhi, Cfg::IDESC2, acc0);
            mma_tf32_ts(ytm, s_hi + kk * 8, blo, Cfg::IDESC2, 1u);
            mma_tf32_ts(ytm, s_hi + kk * 8, bhi, Cfg::IDESC2, 1u);
          } else {
            mma_tf32_ts(ytm, s_hi + kk * 8, bhi, Cfg::IDESC2, acc0);
          }
        }
        mma_commit(&empty[e.stage]);  // the stage (F and C chunk) is free once these complete
        if (e.last) mma_commit(&y_full[yb]);
        return true;
      };

      int t = 0;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++t) {
        const int split = item % p.splits;
        const int c0 = split * p.chunks_per_split;
        const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
        const int xb = t % NXB;
        uint64_t* xbar = X3 ? &x_ready[xb] : &x_full[xb];
        if (!mbar_wait(xbar, (t / NXB) & 1, abort_flag, p.err, DEV_TIMEOUT_X, p.timeout_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t xaddr = sX_addr + xb * Cfg::XBUF_BYTES;
        for (int c = c0; c < c1; ++c) {
          if (!mbar_wait(&full[stage], phase, abort_flag, p.err, DEV_TIMEOUT_FULL,
                         p.timeout_ns)) { ok = false; break; }
          const int buf = gchunk % NBUF;
          if (REDUCE && buf_uses[buf] > 0) {
            // the epilogue must have drained this S buffer before it is overwritten
            if (!mbar_wait(&r_ready[buf], (buf_uses[buf] - 1) & 1, abort_flag, p.err,
                           DEV_TIMEOUT_RREADY, p.timeout_ns)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t fbase = sSt_addr + stage * Cfg::STAGE_ALLOC;
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
              const uint64_t blo = umma_sdesc(fbase + Cfg::F_BYTES + sub * BN * Cfg::XW + off, 16,
                                              8 * Cfg::XW, Cfg::XLAYOUT);
              mma_tf32_ss(s_tm, alo, bhi, Cfg::IDESC1, kk == 0 ? 0u : 1u);
              mma_tf32_ss(s_tm, ahi, blo, Cfg::IDESC1, 1u);
              mma_tf32_ss(s_tm, ahi, bhi, Cfg::IDESC1, 1u);
            } else {
              mma_tf32_ss(s_tm, ahi, bhi, Cfg::IDESC1, kk == 0 ? 0u : 1u);
            }
          }
          mma_commit(&s_full[buf]);
          if (REDUCE) mma_commit(&empty[stage]);
          if (c == c1 - 1) mma_commit(&x_empty[xb]);  // last use of this X tile
          if (!REDUCE) {
            q[(qh + qn) % NBUF] = Pend{stage, buf, t, buf_uses[buf], phase, c == c0, c == c1 - 1};
            ++qn;
            if (qn > Cfg::LAG) {  // keep LAG chunks of lookahead
              if (!issue_second(q[qh])) { ok = false; break; }
              qh = (qh + 1) % NBUF;
              --qn;
            }
          }
          ++buf_uses[buf];
          ++gchunk;
          if (++stage == STAGES) { stage = 0; phase ^= 1; }
        }
      }
      while (ok && qn > 0) {
        if (!issue_second(q[qh])) { ok = false; break; }
        qh = (qh + 1) % NBUF;
        --qn;
      }
      // make sure every MMA this thread issued has completed before TMEM is released
      mma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else if (warp < 2 + Cfg::EPI_WARPS) {
    // ------------------------------------------------------------------ epilogue (warps 2..9)
    // warp w reads TMEM lane quadrant w % 4 (hardware rule) and half (w - 2) / 4 of the columns
    const int qd = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = qd * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(qd * 32) << 16;
    uint32_t buf_uses[NBUF];
#pragma unroll
    for (int b = 0; b < NBUF; ++b) buf_uses[b] = 0;
    uint32_t gchunk = 0;
    double acc_s = 0.0, acc_s2 = 0.0;
    int t = 0;
    bool ok = true;
    // fp16 second MMA: C is scaled by 2^ec (fixed per launch), row j of R by 2^er(j)
    int ec = 0;
    float fmax = 0.f;
    if constexpr (Cfg::H16) {
      fmax = __uint_as_float(p.stats[0]);
      const float cmax = __uint_as_float(p.stats[1]);
      int ex = 0;
      if (cmax > 0.f) frexpf(cmax, &ex);
      ec = 14 - ex;
    }
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++t) {
      const int tile = item / p.splits, split = item % p.splits;
      const int c0 = split * p.chunks_per_split;
      const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
      int er = 0;
      float rscale = 1.f;
      if constexpr (Cfg::H16) {
        // |S_ji| <= |x_j| max_i |F_i|: scale the row so that |R| < 2^15
        const int row = tile * Cfg::TM + row_in_tile;
        if (row < p.M) {
          const float4* xr = reinterpret_cast<const float4*>(p.Xg + (size_t)row * DP);
          float n2 = 0.f;
#pragma unroll
          for (int c = 0; c < DP / 4; ++c) {
            const float4 xv = xr[c];
            n2 = fmaf(xv.x, xv.x, fmaf(xv.y, xv.y, fmaf(xv.z, xv.z, fmaf(xv.w, xv.w, n2))));
          }
          const float bound = sqrtf(n2) * fmax * 1.001f;
          int ex = 0;
          if (bound > 0.f) frexpf(bound, &ex);
          er = 14 - ex;
          rscale = ldexpf(1.f, er);
        }
      }
      for (int c = c0; c < c1; ++c) {
        const int buf = gchunk % NBUF;
        if (!mbar_wait(&s_full[buf], buf_uses[buf] & 1, abort_flag, p.err, DEV_TIMEOUT_SFULL,
                       p.timeout_ns)) { ok = false; break; }
        tc_fence_after();
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
#pragma unroll
        for (int i = 0; i < Cfg::EPI_COLS; ++i) v[i] = fmaxf(v[i], 0.f);
        if (REDUCE) {
          float cs = 0.f, cs2 = 0.f;
#pragma unroll
          for (int i = 0; i < Cfg::EPI_COLS; ++i) {
            cs += v[i];
            cs2 = fmaf(v[i], v[i], cs2);
          }
          acc_s += (double)cs;
          acc_s2 += (double)cs2;
        } else if (X3) {
          const uint32_t lo_tm =
              tbase + lane_addr + Cfg::TMEM_S_LO + buf * BN + half * Cfg::EPI_COLS;
#pragma unroll
          for (int col = 0; col < Cfg::EPI_COLS; col += Cfg::LDW) {
            float lo[Cfg::LDW];
#pragma unroll
            for (int i = 0; i < Cfg::LDW; ++i) {
              const float h = tf32_hi(v[col + i]);
              lo[i] = v[col + i] - h;
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
        } else if constexpr (Cfg::H16) {
          // pack R (scaled) as fp16 pairs (even k in the low half) into this warp's own columns
          uint32_t pk[Cfg::EPI_COLS / 2];
#pragma unroll
          for (int i = 0; i < Cfg::EPI_COLS / 2; ++i) {
            const __half2 h2 = __floats2half2_rn(v[2 * i] * rscale, v[2 * i + 1] * rscale);
            pk[i] = *reinterpret_cast<const uint32_t*>(&h2);
          }
          if constexpr (Cfg::EPI_COLS / 2 == 32) tmem_st32(s_tm, reinterpret_cast<const float*>(pk));
          else tmem_st16(s_tm, reinterpret_cast<const float*>(pk));
          tmem_st_wait();
        } else {
#pragma unroll
          for (int col = 0; col < Cfg::EPI_COLS; col += Cfg::LDW) {
            if constexpr (Cfg::LDW == 32) tmem_st32(s_tm + col, v + col);
            else tmem_st16(s_tm + col, v + col);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&r_ready[buf]);
        ++buf_uses[buf];
        ++gchunk;
      }
      if (!ok) break;
      if (!REDUCE) {
        const int yb = t & 1;
        if (!mbar_wait(&y_full[yb], (t >> 1) & 1, abort_flag, p.err, DEV_TIMEOUT_Y,
                       p.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        const int row = tile * Cfg::TM + row_in_tile;
        if constexpr (DP <= 32) {
          if (p.fuse) {
            // warps of half 0 own full rows: read all of Y, release the accumulator, finalize
            float y[DP];
            if (half == 0) {
#pragma unroll
              for (int col = 0; col < DP; col += 16) {
                tmem_ld16(tbase + lane_addr + Cfg::TMEM_Y + yb * DP + col, y + col);
                tmem_ld_wait_regs16(y + col);
              }
              if constexpr (Cfg::H16) {
                const float inv = ldexpf(1.f, -(er + ec));
#pragma unroll
                for (int i = 0; i < DP; ++i) y[i] *= inv;
              }
            }
            tc_fence_before();
            mbar_arrive(&y_empty[yb]);
            if (half == 0 && row < p.M) epilogue_finalize<DP>(p.fin, row, y);
            continue;
          }
        }
        float* out = p.ws + ((size_t)split * p.M + (size_t)(row < p.M ? row : 0)) * DP;
        // the two warps of a quadrant share the 16-column pieces of Y
#pragma unroll 1
        for (int col = half * 16; col < DP; col += 32) {
          float y[16];
          tmem_ld16(tbase + lane_addr + Cfg::TMEM_Y + yb * DP + col, y);
          tmem_ld_wait_regs16(y);
          if constexpr (Cfg::H16) {
            const float inv = ldexpf(1.f, -(er + ec));
#pragma unroll
            for (int i = 0; i < 16; ++i) y[i] *= inv;
          }
          if (row < p.M) {
            float4* o4 = reinterpret_cast<float4*>(out + col);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              o4[i] = make_float4(y[4 * i], y[4 * i + 1], y[4 * i + 2], y[4 * i + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(&y_empty[yb]);
      }
    }
    if (REDUCE) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        acc_s += __shfl_xor_sync(0xffffffffu, acc_s, o);
        acc_s2 += __shfl_xor_sync(0xffffffffu, acc_s2, o);
      }
      if (lane == 0) {
        red[(warp - 2) * 2 + 0] = acc_s;
        red[(warp - 2) * 2 + 1] = acc_s2;
      }
      asm volatile("bar.sync 1, %0;" ::"r"(Cfg::EPI_THREADS) : "memory");
      if (threadIdx.x == 64) {
        double a = 0.0, b = 0.0;
        for (int w = 0; w < Cfg::EPI_WARPS; ++w) { a += red[2 * w]; b += red[2 * w + 1]; }
        p.partials[2 * blockIdx.x + 0] = a;
        p.partials[2 * blockIdx.x + 1] = b;
      }
    }
  } else if (Cfg::H16) {
    // ------------------------------------------------------------------ C converter (warp 10)
    // fp32 C chunk (32-float SW128 sub-tiles) -> fp16, scaled by 2^ec (64-element SW128 sub-tiles)
    const float cmax = __uint_as_float(p.stats[1]);
    int ex = 0;
    if (cmax > 0.f) frexpf(cmax, &ex);
    const float cscale = ldexpf(1.f, 14 - ex);
    uint32_t g = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
      const int split = item % p.splits;
      const int c0 = split * p.chunks_per_split;
      const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
      bool ok = true;
      for (int c = c0; c < c1; ++c, ++g) {
        const int stage = g % STAGES;
        const uint32_t round = g / STAGES;
        if (!mbar_wait(&full[stage], round & 1, abort_flag, p.err, DEV_TIMEOUT_FULL, p.timeout_ns)) {
          ok = false;
          break;
        }
        const uint8_t* src = sStage + stage * Cfg::STAGE_ALLOC + Cfg::F_BYTES;
        uint8_t* dst = sStage + stage * Cfg::STAGE_ALLOC + Cfg::STAGE_BYTES;
        constexpr int UNITS = (BN / 64) * DP * 8;  // 16-byte fp16 units
        for (int uidx = lane; uidx < UNITS; uidx += 32) {
          const int u = uidx & 7;
          const int r = (uidx >> 3) % DP;
          const int s16 = (uidx >> 3) / DP;
          const int k0 = 64 * s16 + 8 * u;
          const int s32 = k0 >> 5, v0 = (k0 & 31) >> 2;
          const uint8_t* rowp = src + s32 * (DP * 128) + r * 128;
          const float4 a = *reinterpret_cast<const float4*>(rowp + ((v0 ^ (r & 7)) << 4));
          const float4 b = *reinterpret_cast<const float4*>(rowp + (((v0 + 1) ^ (r & 7)) << 4));
          __half2 h[4] = {__floats2half2_rn(a.x * cscale, a.y * cscale),
                          __floats2half2_rn(a.z * cscale, a.w * cscale),
                          __floats2half2_rn(b.x * cscale, b.y * cscale),
                          __floats2half2_rn(b.z * cscale, b.w * cscale)};
          *reinterpret_cast<uint4*>(dst + s16 * (DP * 128) + r * 128 + ((u ^ (r & 7)) << 4)) =
              *reinterpret_cast<const uint4*>(h);
        }
        fence_proxy_async_smem();
        mbar_arrive(&c16_ready[stage]);
      }
      if (!ok) break;
    }
  } else if (X3) {
    // ------------------------------------------------------------------ X splitter (warp 10)
    int t = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++t) {
      const int xb = t % NXB;
      if (!mbar_wait(&x_full[xb], (t / NXB) & 1, abort_flag, p.err, DEV_TIMEOUT_X, p.timeout_ns))
        break;
      float4* xs = reinterpret_cast<float4*>(sX + xb * Cfg::XBUF_BYTES);
      float4* xl = reinterpret_cast<float4*>(sX + xb * Cfg::XBUF_BYTES + Cfg::X_BYTES);
      for (int i = lane; i < Cfg::X_BYTES / 16; i += 32) {
        const float4 v = xs[i];
        const float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
        xs[i] = h;
        xl[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
      }
      fence_proxy_async_smem();
      mbar_arrive(&x_ready[xb]);
    }
  }

  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tbase, 512);
  }
}

}  // namespace sb
