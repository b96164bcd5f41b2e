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
//   warp 0      TMA producer: X tile once per work item, then (F chunk, Ct chunk) per stage
//   warp 1      MMA issuer (one thread): S = X F^T into a TMEM buffer (kind::tf32), then,
//               once the epilogue has rewritten S as R = ReLU(S) in place, Y += R C with R read
//               straight from TMEM (the .kind::tf32 [d], [a_tmem], b_desc form)
//   warps 2..5  epilogue: tcgen05.ld S -> ReLU -> tcgen05.st R (or accumulate the sums), and the
//               final tcgen05.ld of Y -> global
//
// Precision: X3=false is plain TF32 (the tensor core reads the fp32 bits as tf32). X3=true is
// the 3xTF32 split (x = hi + lo with hi = x with the low 13 mantissa bits cleared), giving fp32
// accuracy: S = Xlo Fhi + Xhi Flo + Xhi Fhi and Y += Rlo Chi + Rhi Clo + Rhi Chi.
//
// Shared-memory operands are K-major with the TMA swizzle matching the row width (64 B rows:
// SWIZZLE_64B, 128 B rows: SWIZZLE_128B; wider rows are split in 128 B sub-tiles).
// No TMA multicast is used anywhere.
#pragma once
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
};

template <int DP, int BN, int STAGES, bool X3, bool REDUCE>
struct ProductCfg {
  static_assert(DP == 16 || DP == 32 || DP == 64 || DP == 128 || DP == 256, "DP");
  static_assert(BN % 32 == 0 && BN >= 32 && BN <= 256, "BN");
  static constexpr int TM = 128;                          // rows per tile (MMA M)
  static constexpr int XW = DP * 4 <= 128 ? DP * 4 : 128; // K-major row width in bytes
  static constexpr int KSUB = DP * 4 / XW;                // 128 B sub-tiles along K
  static constexpr uint32_t XLAYOUT = XW == 64 ? UMMA_SW64 : UMMA_SW128;
  static constexpr int BOX_K = XW / 4;                    // TMA box inner extent (floats)
  static constexpr int X_BYTES = TM * DP * 4;
  static constexpr int F_BYTES = BN * DP * 4;
  static constexpr int C_BYTES = REDUCE ? 0 : DP * BN * 4;
  static constexpr int NPREC = X3 ? 2 : 1;
  static constexpr int STAGE_BYTES = NPREC * (F_BYTES + C_BYTES);
  static constexpr int X_TOTAL = NPREC * X_BYTES;
  static constexpr int SMEM_DATA = X_TOTAL + STAGES * STAGE_BYTES;
  static constexpr int SMEM_BYTES_RAW = SMEM_DATA + 1024 /*barriers*/ + 1024 /*align slack*/;
  // at least 120 KB so that only one CTA (and one 512-column TMEM allocation) lives on an SM
  static constexpr int SMEM_BYTES = SMEM_BYTES_RAW < 122880 ? 122880 : SMEM_BYTES_RAW;
  static_assert(SMEM_BYTES_RAW <= 232448, "shared memory budget");
  static constexpr int TMEM_S_LO = 2 * BN;                // lo halves of R (3xTF32)
  static constexpr int TMEM_Y = X3 ? 4 * BN : 2 * BN;
  static_assert(TMEM_Y + (REDUCE ? 0 : DP) <= 512, "TMEM budget");
  static_assert(REDUCE || STAGES >= 2, "product mode needs two stages (MMA2 lags MMA1)");
  static constexpr uint32_t IDESC1 = umma_idesc_tf32(TM, BN);
  static constexpr uint32_t IDESC2 = umma_idesc_tf32(TM, DP);
  static constexpr int THREADS = 192;
};

template <int DP, int BN, int STAGES, bool X3, bool REDUCE>
__global__ void __launch_bounds__(192, 1)
    relu_product_kernel(const __grid_constant__ CUtensorMap tmX,
                        const __grid_constant__ CUtensorMap tmFhi,
                        const __grid_constant__ CUtensorMap tmFlo,
                        const __grid_constant__ CUtensorMap tmChi,
                        const __grid_constant__ CUtensorMap tmClo, const ProductParams p) {
  using Cfg = ProductCfg<DP, BN, STAGES, X3, REDUCE>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  uint8_t* sX = smem;                                   // [NPREC][X_BYTES]   (hi, lo)
  uint8_t* sStage = smem + Cfg::X_TOTAL;                // [STAGES][STAGE_BYTES]
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::SMEM_DATA);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* s_full = bars + 2 * STAGES;  // [2]
  uint64_t* r_ready = s_full + 2;        // [2]
  uint64_t* x_full = r_ready + 2;
  uint64_t* x_empty = x_full + 1;
  uint64_t* x_ready = x_empty + 1;
  uint64_t* y_full = x_ready + 1;
  uint64_t* y_empty = y_full + 1;
  uint64_t* drain = y_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  double* red = reinterpret_cast<double*>(smem + Cfg::SMEM_DATA + 512);  // [4][2]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.n_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&r_ready[b], 128);
    }
    mbar_init(x_full, 1);
    mbar_init(x_empty, 1);
    mbar_init(x_ready, 128);
    mbar_init(y_full, 1);
    mbar_init(y_empty, 128);
    mbar_init(drain, 1);
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
    if (lane == 0) {
      uint32_t stage = 0;
      int t = 0;
      uint32_t uses[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) uses[s] = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++t) {
        const int tile = item / p.splits, split = item % p.splits;
        const int c0 = split * p.chunks_per_split;
        const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
        if (t > 0 && !mbar_wait(x_empty, (t - 1) & 1, abort_flag, p.err, DEV_TIMEOUT_X,
                                p.timeout_ns)) { ok = false; break; }
        mbar_arrive_expect_tx(x_full, Cfg::X_BYTES);
#pragma unroll
        for (int s = 0; s < Cfg::KSUB; ++s)
          tma_load_2d(sX + s * Cfg::TM * Cfg::XW, &tmX, s * Cfg::BOX_K, tile * Cfg::TM, x_full);
        for (int c = c0; c < c1; ++c) {
          if (uses[stage] > 0) {
            if (!mbar_wait(&empty[stage], (uses[stage] - 1) & 1, abort_flag, p.err,
                           DEV_TIMEOUT_EMPTY, p.timeout_ns)) { ok = false; break; }
          }
          uint8_t* st = sStage + stage * Cfg::STAGE_BYTES;
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
          ++uses[stage];
          if (++stage == STAGES) stage = 0;
        }
      }
      if (*abort_flag) {
        // wait (bounded) for this CTA's own copies still in flight before leaving
#pragma unroll
        for (int s = 0; s < STAGES; ++s)
          if (uses[s] > 0) mbar_drain(&full[s], (uses[s] - 1) & 1);
        if (t > 0) mbar_drain(x_full, (t - 1) & 1);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t stage = 0;
      uint32_t uses[STAGES];
#pragma unroll
      for (int s = 0; s < STAGES; ++s) uses[s] = 0;
      uint32_t buf_uses[2] = {0, 0};
      uint32_t gchunk = 0;  // global chunk counter -> S buffer = gchunk & 1
      int t = 0;
      bool ok = true;
      const uint32_t sX_addr = smem_u32(sX);
      const uint32_t sSt_addr = smem_u32(sStage);
      // pending second MMA (product mode)
      int pend_stage = -1, pend_buf = 0, pend_first = 0;
      uint32_t pend_use = 0;
      auto issue_second = [&](int st, int buf, uint32_t buse, int first_of_item) -> bool {
        if (!mbar_wait(&r_ready[buf], buse & 1, abort_flag, p.err, DEV_TIMEOUT_RREADY,
                       p.timeout_ns)) return false;
        if (first_of_item && t > 0) {
          if (!mbar_wait(y_empty, (t - 1) & 1, abort_flag, p.err, DEV_TIMEOUT_Y, p.timeout_ns))
            return false;
        }
        tc_fence_after();
        const uint32_t cbase = sSt_addr + st * Cfg::STAGE_BYTES + Cfg::NPREC * Cfg::F_BYTES;
        const uint32_t s_hi = tbase + buf * BN;
        const uint32_t s_lo = tbase + Cfg::TMEM_S_LO + buf * BN;
        const uint32_t ytm = tbase + Cfg::TMEM_Y;
#pragma unroll
        for (int kk = 0; kk < BN / 8; ++kk) {
          const uint32_t off = (kk >> 2) * (DP * 128) + (kk & 3) * 32;
          const uint64_t bhi = umma_sdesc(cbase + off, 16, 1024, UMMA_SW128);
          const uint32_t acc0 = (first_of_item && kk == 0) ? 0u : 1u;
          if (X3) {
            const uint64_t blo = umma_sdesc(cbase + Cfg::C_BYTES + off, 16, 1024, UMMA_SW128);
            mma_tf32_ts(ytm, s_lo + kk * 8, bhi, Cfg::IDESC2, acc0);
            mma_tf32_ts(ytm, s_hi + kk * 8, blo, Cfg::IDESC2, 1u);
            mma_tf32_ts(ytm, s_hi + kk * 8, bhi, Cfg::IDESC2, 1u);
          } else {
            mma_tf32_ts(ytm, s_hi + kk * 8, bhi, Cfg::IDESC2, acc0);
          }
        }
        mma_commit(&empty[st]);  // the stage (F and C chunk) is free once these complete
        return true;
      };

      for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++t) {
        const int split = item % p.splits;
        const int c0 = split * p.chunks_per_split;
        const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
        uint64_t* xb = X3 ? x_ready : x_full;
        if (!mbar_wait(xb, t & 1, abort_flag, p.err, DEV_TIMEOUT_X, p.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        for (int c = c0; c < c1; ++c) {
          if (!mbar_wait(&full[stage], uses[stage] & 1, abort_flag, p.err, DEV_TIMEOUT_FULL,
                         p.timeout_ns)) { ok = false; break; }
          const int buf = gchunk & 1;
          if (REDUCE && buf_uses[buf] > 0) {
            // the epilogue must have drained this S buffer before it is overwritten
            if (!mbar_wait(&r_ready[buf], (buf_uses[buf] - 1) & 1, abort_flag, p.err,
                           DEV_TIMEOUT_RREADY, p.timeout_ns)) { ok = false; break; }
          }
          tc_fence_after();
          const uint32_t fbase = sSt_addr + stage * Cfg::STAGE_BYTES;
          const uint32_t s_tm = tbase + buf * BN;
#pragma unroll
          for (int kk = 0; kk < DP / 8; ++kk) {
            const int sub = kk / (Cfg::XW / 32);
            const uint32_t off = (kk % (Cfg::XW / 32)) * 32;
            const uint64_t ahi = umma_sdesc(sX_addr + sub * Cfg::TM * Cfg::XW + off, 16,
                                            8 * Cfg::XW, Cfg::XLAYOUT);
            const uint64_t bhi = umma_sdesc(fbase + sub * BN * Cfg::XW + off, 16, 8 * Cfg::XW,
                                            Cfg::XLAYOUT);
            if (X3) {
              const uint64_t alo = umma_sdesc(sX_addr + Cfg::X_BYTES + sub * Cfg::TM * Cfg::XW + off,
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
          if (c == c1 - 1) mma_commit(x_empty);  // last use of this X tile
          if (!REDUCE) {
            if (pend_stage >= 0) {
              if (!issue_second(pend_stage, pend_buf, pend_use, pend_first)) { ok = false; break; }
            }
            pend_stage = stage; pend_buf = buf; pend_use = buf_uses[buf]; pend_first = (c == c0);
          }
          ++buf_uses[buf];
          ++gchunk;
          ++uses[stage];
          if (++stage == STAGES) stage = 0;
        }
        if (!ok) break;
        if (!REDUCE) {
          if (pend_stage >= 0 && !issue_second(pend_stage, pend_buf, pend_use, pend_first)) {
            ok = false; break;
          }
          pend_stage = -1;
          mma_commit(y_full);
        }
      }
      // make sure every MMA this thread issued has completed before TMEM is released
      mma_commit(drain);
      mbar_drain(drain, 0);
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;  // TMEM lane quadrant this warp may access
    const int row_in_tile = q * 32 + lane;
    const uint32_t lane_addr = (uint32_t)(q * 32) << 16;
    uint32_t buf_uses[2] = {0, 0};
    uint32_t gchunk = 0;
    double acc_s = 0.0, acc_s2 = 0.0;
    int t = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < n_items && ok; item += gridDim.x, ++t) {
      const int tile = item / p.splits, split = item % p.splits;
      const int c0 = split * p.chunks_per_split;
      const int c1 = min(p.n_chunks, c0 + p.chunks_per_split);
      if (X3) {
        // split the X tile into hi (in place) and lo halves
        if (!mbar_wait(x_full, t & 1, abort_flag, p.err, DEV_TIMEOUT_X, p.timeout_ns)) { ok = false; break; }
        float4* xs = reinterpret_cast<float4*>(sX);
        float4* xl = reinterpret_cast<float4*>(sX + Cfg::X_BYTES);
        for (int i = threadIdx.x - 64; i < Cfg::X_BYTES / 16; i += 128) {
          float4 v = xs[i];
          float4 h = make_float4(tf32_hi(v.x), tf32_hi(v.y), tf32_hi(v.z), tf32_hi(v.w));
          xs[i] = h;
          xl[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);
        }
        fence_proxy_async_smem();
        mbar_arrive(x_ready);
      }
      for (int c = c0; c < c1; ++c) {
        const int buf = gchunk & 1;
        if (!mbar_wait(&s_full[buf], buf_uses[buf] & 1, abort_flag, p.err, DEV_TIMEOUT_SFULL,
                       p.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        const uint32_t s_tm = tbase + lane_addr + buf * BN;
        float cs = 0.f, cs2 = 0.f;
#pragma unroll 1
        for (int col = 0; col < BN; col += 32) {
          float v[32];
          tmem_ld16(s_tm + col, v);
          tmem_ld16(s_tm + col + 16, v + 16);
          tmem_ld_wait_regs32(v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.f);
          if (REDUCE) {
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              cs += v[i];
              cs2 = fmaf(v[i], v[i], cs2);
            }
          } else if (X3) {
            float lo[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              const float h = tf32_hi(v[i]);
              lo[i] = v[i] - h;
              v[i] = h;
            }
            tmem_st16(s_tm + col, v);
            tmem_st16(s_tm + col + 16, v + 16);
            const uint32_t lo_tm = tbase + lane_addr + Cfg::TMEM_S_LO + buf * BN;
            tmem_st16(lo_tm + col, lo);
            tmem_st16(lo_tm + col + 16, lo + 16);
          } else {
            tmem_st16(s_tm + col, v);
            tmem_st16(s_tm + col + 16, v + 16);
          }
        }
        if (REDUCE) {
          acc_s += (double)cs;
          acc_s2 += (double)cs2;
        } else {
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&r_ready[buf]);
        ++buf_uses[buf];
        ++gchunk;
      }
      if (!ok) break;
      if (!REDUCE) {
        if (!mbar_wait(y_full, t & 1, abort_flag, p.err, DEV_TIMEOUT_Y, p.timeout_ns)) { ok = false; break; }
        tc_fence_after();
        const int row = tile * Cfg::TM + row_in_tile;
        float* out = p.ws + ((size_t)split * p.M + (size_t)(row < p.M ? row : 0)) * DP;
#pragma unroll 1
        for (int col = 0; col < DP; col += 16) {
          float v[16];
          tmem_ld16(tbase + lane_addr + Cfg::TMEM_Y + col, v);
          tmem_ld_wait_regs16(v);
          if (row < p.M) {
            float4* o4 = reinterpret_cast<float4*>(out + col);
#pragma unroll
            for (int i = 0; i < 4; ++i)
              o4[i] = make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]);
          }
        }
        tc_fence_before();
        mbar_arrive(y_empty);
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
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (threadIdx.x == 64) {
        double a = 0.0, b = 0.0;
        for (int w = 0; w < 4; ++w) { a += red[2 * w]; b += red[2 * w + 1]; }
        p.partials[2 * blockIdx.x + 0] = a;
        p.partials[2 * blockIdx.x + 1] = b;
      }
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
