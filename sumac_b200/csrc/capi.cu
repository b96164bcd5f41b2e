// capi.cu — the extern "C" entry points declared in include/sumac_b200.h. Argument checks,
// workspace layout (a bump allocator over the caller's buffer; the *_workspace_bytes queries run
// the same plan with a null base) and kernel sequencing. Nothing here allocates or synchronises.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/sumac_b200.h"
#include "kernels.cuh"

using namespace sb;

namespace {

thread_local std::string g_last_error;
unsigned long long g_timeout_ns = 2000000000ull;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_status(int rc, const char* what) {
  if (rc == 0) return SUMAC_OK;
  if (rc == -1) return fail(SUMAC_ERR_UNSUPPORTED, "%s: unsupported rank/precision", what);
  if (rc == -5) return fail(SUMAC_ERR_ARG, "%s: bad sizes", what);
  if (rc == -6) return fail(SUMAC_ERR_CUDA, "%s: cuTensorMapEncodeTiled failed", what);
  if (rc == -7) return fail(SUMAC_ERR_ARG, "%s: operand maxima missing", what);
  if (rc < 0) return fail(SUMAC_ERR_ARG, "%s: error %d", what, rc);
  return fail(SUMAC_ERR_CUDA, "%s: %s", what, cudaGetErrorString((cudaError_t)rc));
}

int launched(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(SUMAC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return SUMAC_OK;
}

struct Bump {
  uint8_t* base;
  size_t off = 0;
  explicit Bump(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t count) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += count * sizeof(T);
    return p;
  }
};

int padded(int d) {
  if (d <= 0) return 0;
  if (d <= 16) return 16;
  if (d <= 32) return 32;
  if (d <= 64) return 64;
  if (d <= 128) return 128;
  if (d <= 256) return 256;
  return 0;
}

int num_sms_current() {
  static int cache[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0)
      n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Per device: a side stream and two events that fork work off the caller's stream and join it
// back (stream-ordered, so it is captured into CUDA graphs as a parallel branch). Created on the
// first use on a device; SALSA runs its first iteration eagerly, so creation precedes capture.
struct SideStream {
  cudaStream_t stream = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
std::mutex g_side_mutex;
SideStream g_side[64];

SideStream* side_stream() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(g_side_mutex);
  SideStream& ss = g_side[dev];
  if (!ss.stream) {
    if (cudaStreamCreateWithFlags(&ss.stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
      ss = SideStream{};
      return nullptr;
    }
  }
  return &ss;
}
int64_t round4(int64_t x) { return (x + 3) & ~int64_t(3); }

}  // namespace

namespace sb {
// Record a message for sumac_last_error() from another translation unit of this library.
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace sb

extern "C" {

int sumac_version(void) { return 1; }
const char* sumac_last_error(void) { return g_last_error.c_str(); }
int sumac_padded_rank(int d) { return padded(d); }
long long sumac_kernel_launches(void) { return launch_count(); }

int sumac_relu_product(const float* X, int64_t M, const float* Fhi, const float* Flo,
                       const float* Cthi, const float* Ctlo, int64_t ldct, int64_t N, int Dp,
                       int precision, float* partials, int* dev_err, sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  if (!X || !Fhi || !Cthi || !partials || !dev_err || (x3 && (!Flo || !Ctlo)))
    return fail(SUMAC_ERR_ARG, "relu_product: null pointer");
  if (!aligned16(X) || !aligned16(Fhi) || !aligned16(Cthi) || (ldct & 3))
    return fail(SUMAC_ERR_ARG, "relu_product: operands must be 16-byte aligned");
  // the TF32 product's fp16 second MMA needs the operand maxima: they go to the 16 bytes that
  // follow the partial outputs in `partials`
  unsigned int* stats = nullptr;
  const int splits_p = product_split_count(M, N, Dp, x3, num_sms_current());
  if (!x3) {
    stats = reinterpret_cast<unsigned int*>(partials + (size_t)splits_p * M * Dp);
    launch_operand_stats(Fhi, N, Dp, Cthi, (int64_t)Dp * ldct, stats,
                         reinterpret_cast<cudaStream_t>(stream));
  }
  int rc = launch_relu_product(X, M, Fhi, Flo, Cthi, Ctlo, ldct, N, Dp, x3, partials, dev_err,
                               num_sms_current(), g_timeout_ns,
                               reinterpret_cast<cudaStream_t>(stream), stats, 0, 1);
  return cuda_status(rc, "relu_product");
}
int sumac_relu_product_splits(int64_t M, int64_t N, int Dp, int precision) {
  return product_split_count(M, N, Dp, precision == SUMAC_3XTF32, num_sms_current());
}
void sumac_set_timeout_ns(unsigned long long ns) { g_timeout_ns = ns; }
int sumac_num_sms(int device) {
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return -1;
  return n;
}

// ------------------------------------------------------------------------------ relu_bat_c
struct RbcPlan {
  float *Xp, *Fp, *Flo, *Cp, *Cthi, *Ctlo, *part;
  unsigned int* stats;
  int64_t ldct;
  size_t bytes;
};
static RbcPlan plan_relu_bat_c(void* ws, int64_t M, int64_t N, int Dp, bool x3, int sms) {
  Bump b(ws);
  RbcPlan p;
  p.ldct = round4(N);
  const int splits = product_split_count(M, N, Dp, x3, sms);
  p.Xp = b.take<float>((size_t)M * Dp);
  p.Fp = b.take<float>((size_t)N * Dp);
  p.Flo = x3 ? b.take<float>((size_t)N * Dp) : nullptr;
  p.Cp = b.take<float>((size_t)N * Dp);
  p.Cthi = b.take<float>((size_t)Dp * p.ldct);
  p.Ctlo = x3 ? b.take<float>((size_t)Dp * p.ldct) : nullptr;
  p.part = b.take<float>((size_t)(splits > 0 ? splits : 1) * M * Dp);
  p.stats = b.take<unsigned int>(4);
  p.bytes = b.off + 256;
  return p;
}

size_t sumac_relu_bat_c_workspace_bytes(int64_t M, int64_t N, int D, int precision) {
  const int Dp = padded(D);
  if (!Dp) return 0;
  return plan_relu_bat_c(nullptr, M, N, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

int sumac_relu_bat_c(const float* A, const float* B, const float* C, int64_t M, int64_t N, int D,
                     float* Y, int precision, void* ws, size_t ws_bytes, int* dev_err,
                     sumac_stream_t stream) {
  return sumac_relu_bat_c_mode(A, B, C, M, N, D, Y, precision, SUMAC_RELU, ws, ws_bytes, dev_err,
                               stream);
}

int sumac_relu_bat_c_mode(const float* A, const float* B, const float* C, int64_t M, int64_t N,
                          int D, float* Y, int precision, int mode, void* ws, size_t ws_bytes,
                          int* dev_err, sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  if (mode != SUMAC_RELU && mode != SUMAC_STEP)
    return fail(SUMAC_ERR_ARG, "relu_bat_c: mode %d is neither SUMAC_RELU nor SUMAC_STEP", mode);
  const int Dp = padded(D);
  if (M <= 0 || N <= 0 || D <= 0) return fail(SUMAC_ERR_ARG, "relu_bat_c: empty shape M=%lld N=%lld D=%d", (long long)M, (long long)N, D);
  if (!A || !B || !C || !Y || !dev_err) return fail(SUMAC_ERR_ARG, "relu_bat_c: null pointer");
  if (!Dp || !product_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "relu_bat_c: D=%d not supported with precision %d", D, precision);
  const int sms = num_sms_current();
  RbcPlan p = plan_relu_bat_c(ws, M, N, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes) return fail(SUMAC_ERR_WORKSPACE, "relu_bat_c: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  launch_gather_pad(B, D, D, nullptr, M, Dp, p.Xp, nullptr, nullptr, s);
  // F as tf32 hi / lo halves (3xTF32) or rounded to tf32 (TF32)
  launch_gather_pad(A, D, D, nullptr, N, Dp, nullptr, p.Fp, x3 ? p.Flo : nullptr, s);
  launch_gather_pad(C, D, D, nullptr, N, Dp, p.Cp, nullptr, nullptr, s);
  launch_transpose_split(p.Cp, N, Dp, p.Cthi, p.Ctlo, p.ldct, s);
  if (!x3) launch_operand_stats(p.Fp, N, Dp, p.Cthi, (int64_t)Dp * p.ldct, p.stats, s);
  int rc = launch_relu_product(p.Xp, M, p.Fp, p.Flo, p.Cthi, p.Ctlo, p.ldct, N, Dp, x3, p.part,
                               dev_err, sms, g_timeout_ns, s, p.stats, mode == SUMAC_STEP, 1);
  if (rc) return cuda_status(rc, "relu_bat_c");
  FinalizeArgs f{};
  f.mode = FIN_STORE; f.M = M; f.Dp = Dp; f.splits = product_split_count(M, N, Dp, x3, sms);
  f.ws = p.part; f.X = p.Xp; f.out = Y; f.out_d = D; f.ld_out = D;
  launch_finalize(f, s);
  return launched("relu_bat_c");
}

// ------------------------------------------------------------------------------ relu_bat_reduce
struct RedPlan {
  float *Xp, *Fp, *Flo;
  double* part;
  size_t bytes;
};
static RedPlan plan_reduce(void* ws, int64_t M, int64_t N, int Dp, bool x3, int sms) {
  Bump b(ws);
  RedPlan p;
  p.Xp = b.take<float>((size_t)M * Dp);
  p.Fp = b.take<float>((size_t)N * Dp);
  p.Flo = x3 ? b.take<float>((size_t)N * Dp) : nullptr;
  p.part = b.take<double>((size_t)sms * 2);
  p.bytes = b.off + 256;
  return p;
}

size_t sumac_relu_bat_reduce_workspace_bytes(int64_t M, int64_t N, int D, int precision) {
  const int Dp = padded(D);
  if (!Dp) return 0;
  return plan_reduce(nullptr, M, N, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

int sumac_relu_bat_reduce(const float* A, const float* B, int64_t M, int64_t N, int D,
                          double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                          sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  const int Dp = padded(D);
  if (M <= 0 || N <= 0 || D <= 0) return fail(SUMAC_ERR_ARG, "relu_bat_reduce: empty shape");
  if (!A || !B || !out || !dev_err) return fail(SUMAC_ERR_ARG, "relu_bat_reduce: null pointer");
  if (!Dp || !reduce_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "relu_bat_reduce: D=%d not supported with precision %d", D, precision);
  const int sms = num_sms_current();
  RedPlan p = plan_reduce(ws, M, N, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes) return fail(SUMAC_ERR_WORKSPACE, "relu_bat_reduce: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  launch_gather_pad(A, D, D, nullptr, M, Dp, p.Xp, nullptr, nullptr, s);
  launch_gather_pad(B, D, D, nullptr, N, Dp, nullptr, p.Fp, x3 ? p.Flo : nullptr, s);
  int grid = 0;
  int rc = launch_relu_reduce(p.Xp, M, p.Fp, p.Flo, N, Dp, x3, p.part, &grid, dev_err, sms,
                              g_timeout_ns, s, 0, 1);
  if (rc) return cuda_status(rc, "relu_bat_reduce");
  launch_sum_partials(p.part, grid, 2, out, 0, s);
  return launched("relu_bat_reduce");
}

// ------------------------------------------------------------------------------ masked product
struct MpPlan {
  float *Fhi, *Flo, *Cthi, *Ctlo, *part;
  unsigned int* stats;
  int64_t ldct;
  size_t bytes;
};
static MpPlan plan_masked(void* ws, int64_t M, int64_t N, int Dp, bool x3, int sms) {
  Bump b(ws);
  MpPlan p;
  p.ldct = round4(N);
  p.Fhi = b.take<float>((size_t)N * Dp);
  p.Flo = x3 ? b.take<float>((size_t)N * Dp) : nullptr;
  p.Cthi = b.take<float>((size_t)Dp * p.ldct);
  p.Ctlo = x3 ? b.take<float>((size_t)Dp * p.ldct) : nullptr;
  const int splits = product_split_count(M, N, Dp, x3, sms);
  p.part = b.take<float>((size_t)(splits > 0 ? splits : 1) * M * Dp);
  p.stats = b.take<unsigned int>(4);
  p.bytes = b.off + 256;
  return p;
}

size_t sumac_masked_product_workspace_bytes(int64_t M, int64_t N, int Dp, int precision) {
  return plan_masked(nullptr, M, N, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

int sumac_masked_product(const float* X, const float* F, const float* C, int64_t M, int64_t N,
                         int Dp, const int32_t* rowptr, const int32_t* ent, float* Y,
                         int precision, void* ws, size_t ws_bytes, int* dev_err,
                         sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  if (M <= 0 || N <= 0) return fail(SUMAC_ERR_ARG, "masked_product: empty shape");
  if (!X || !F || !C || !Y || !dev_err || (rowptr && !ent))
    return fail(SUMAC_ERR_ARG, "masked_product: null pointer");
  if (padded(Dp) != Dp || !product_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "masked_product: Dp=%d not supported with precision %d", Dp, precision);
  if (!aligned16(X) || !aligned16(F) || !aligned16(C) || !aligned16(Y))
    return fail(SUMAC_ERR_ARG, "masked_product: operands must be 16-byte aligned");
  const int sms = num_sms_current();
  MpPlan p = plan_masked(ws, M, N, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes) return fail(SUMAC_ERR_WORKSPACE, "masked_product: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  launch_gather_pad(F, Dp, Dp, nullptr, N, Dp, nullptr, p.Fhi, x3 ? p.Flo : nullptr, s);
  launch_transpose_split(C, N, Dp, p.Cthi, p.Ctlo, p.ldct, s);
  if (!x3) launch_operand_stats(F, N, Dp, p.Cthi, (int64_t)Dp * p.ldct, p.stats, s);
  FinalizeArgs f{};
  f.mode = FIN_STORE; f.M = M; f.Dp = Dp; f.splits = product_split_count(M, N, Dp, x3, sms);
  f.ws = p.part; f.X = const_cast<float*>(X); f.F = F; f.Cm = C;
  f.rowptr = rowptr; f.ent = reinterpret_cast<const int2*>(ent);
  f.out = Y; f.out_d = Dp; f.ld_out = Dp;
  int rc = launch_relu_product(X, M, p.Fhi, p.Flo, p.Cthi, p.Ctlo, p.ldct, N, Dp, x3,
                               p.part, dev_err, sms, g_timeout_ns, s, p.stats, 0, 1);
  if (rc) return cuda_status(rc, "masked_product");
  launch_finalize(f, s);
  return launched("masked_product");
}

// ------------------------------------------------------------------------------ SALSA update
struct SalsaPlan {
  float *FI, *Fhi, *Flo, *P, *Cthi, *Ctlo, *part, *ginv;
  double* gram;
  unsigned int* counter;
  int64_t ldct;
  size_t bytes;
};
static SalsaPlan plan_salsa(void* ws, int64_t M, int64_t b, int d, int Dp, bool x3, int sms) {
  Bump bp(ws);
  SalsaPlan p;
  p.ldct = round4(b);
  p.FI = bp.take<float>((size_t)b * Dp);
  p.Fhi = bp.take<float>((size_t)b * Dp);
  p.Flo = x3 ? bp.take<float>((size_t)b * Dp) : nullptr;
  p.P = bp.take<float>((size_t)b * Dp);
  p.Cthi = bp.take<float>((size_t)Dp * p.ldct);
  p.Ctlo = x3 ? bp.take<float>((size_t)Dp * p.ldct) : nullptr;
  const size_t gbytes = (size_t)gram_parts(b) * d * d * sizeof(double);
  const size_t pbytes = d <= 32 ? salsa_ginv_scratch_bytes(b, d) : 0;
  p.gram = bp.take<double>(((gbytes > pbytes ? gbytes : pbytes) + 7) / 8);
  p.ginv = bp.take<float>((size_t)Dp * Dp);
  // [0] Gram-inverse done-CTA counter; from [2]: one (max |F_i|, max |C|) pair per gather CTA
  // (the d > 32 path: one atomically maxed pair at [1..2])
  p.counter = bp.take<unsigned int>(4 + 2 * (size_t)salsa_gather_ctas(b));
  // the split count grows as b shrinks; size for the worst case over b' <= b
  int smax = 1;
  for (int64_t bb = b; bb > 0; bb = bb / 2) {
    const int s = product_split_count(M, bb, Dp, x3, sms);
    if (s > smax) smax = s;
    if (bb == 1) break;
  }
  p.part = bp.take<float>((size_t)smax * M * Dp);
  p.bytes = bp.off + 256;
  return p;
}

size_t sumac_salsa_update_workspace_bytes(int64_t M, int64_t b_max, int d, int precision) {
  const int Dp = padded(d);
  if (!Dp) return 0;
  return plan_salsa(nullptr, M, b_max, d, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

int sumac_salsa_block_update(const float* F, int64_t m_fixed, const int64_t* rows, int64_t b,
                             float* X, float* dX, int64_t M, int d, const int32_t* rowptr,
                             const int32_t* ent, float momentum, float lrate,
                             const float* unbias, int precision, void* ws, size_t ws_bytes,
                             int* dev_err, sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  const int Dp = padded(d);
  if (b <= 0 || M <= 0 || m_fixed <= 0) return fail(SUMAC_ERR_ARG, "salsa_block_update: empty shape");
  if (!F || !rows || !X || !dX || !unbias || !dev_err || (rowptr && !ent))
    return fail(SUMAC_ERR_ARG, "salsa_block_update: null pointer");
  // the solve of the least-squares map keeps the d x d Gram matrix (fp64) in shared memory
  if (!Dp || d > 128 || !product_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "salsa_block_update: rank %d not supported with precision %d (SALSA takes rank <= 128)", d, precision);
  if (!aligned16(F) || !aligned16(X) || !aligned16(dX))
    return fail(SUMAC_ERR_ARG, "salsa_block_update: factors must be 16-byte aligned");
  const int sms = num_sms_current();
  SalsaPlan p = plan_salsa(ws, M, b, d, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes)
    return fail(SUMAC_ERR_WORKSPACE, "salsa_block_update: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (d <= 32) {
    // C = F_I: the product and the support term contract with the gathered rows themselves and
    // the finalize pass applies G^{-1}, which a side stream computes while the product runs
    SideStream* side = side_stream();
    if (!side) return fail(SUMAC_ERR_CUDA, "salsa_block_update: side stream creation failed");
    // no memset: the gather writes every CTA's pair of operand maxima and zeroes the counter
    launch_salsa_gather(F, rows, b, Dp, p.FI, p.Fhi, p.Flo, p.Cthi, p.Ctlo, p.ldct,
                        x3 ? nullptr : p.counter + 2, p.counter, s);
    cudaEventRecord(side->fork, s);
    cudaStreamWaitEvent(side->stream, side->fork, 0);
    launch_salsa_ginv(p.FI, b, d, Dp, p.gram, p.counter, p.ginv, dev_err, side->stream);
    cudaEventRecord(side->join, side->stream);
    // the product leaves kGinvSms SMs to the Gram-inverse launch, which then runs at full speed
    // instead of sharing issue slots with product CTAs
    const int psms = sms > 2 * kGinvSms ? sms - kGinvSms : sms;
    int rc = launch_relu_product(X, M, p.Fhi, p.Flo, p.Cthi, p.Ctlo, p.ldct, b, Dp,
                                 x3, p.part, dev_err, psms, g_timeout_ns, s, p.counter + 2, 0, 1,
                                 salsa_gather_ctas(b));
    cudaStreamWaitEvent(s, side->join, 0);
    if (rc) return cuda_status(rc, "salsa_block_update");
    FinalizeArgs f{};
    f.mode = FIN_SALSA; f.M = M; f.Dp = Dp; f.splits = product_split_count(M, b, Dp, x3, psms);
    f.ws = p.part; f.X = X; f.dX = dX; f.F = p.FI; f.Cm = p.FI; f.ginv = p.ginv;
    f.rowptr = rowptr; f.ent = reinterpret_cast<const int2*>(ent);
    f.momentum = momentum; f.lrate = lrate; f.unbias = unbias;
    launch_finalize(f, s);
    return launched("salsa_block_update");
  }
  // d > 32: P = F_I G^{-1} from a block-parallel Gram and a per-row solve, then C = P
  launch_gather_pad(F, Dp, Dp, rows, b, Dp, p.FI, p.Fhi, x3 ? p.Flo : nullptr, s);
  launch_gram(p.FI, b, d, Dp, p.gram, s);
  launch_solve(p.FI, b, d, Dp, p.gram, gram_parts(b), p.P, p.Cthi, p.Ctlo, p.ldct, dev_err, s);
  if (!x3) launch_operand_stats(p.FI, b, Dp, p.Cthi, (int64_t)Dp * p.ldct, p.counter + 1, s);
  FinalizeArgs f{};
  f.mode = FIN_SALSA; f.M = M; f.Dp = Dp; f.splits = product_split_count(M, b, Dp, x3, sms);
  f.ws = p.part; f.X = X; f.dX = dX; f.F = p.FI; f.Cm = p.P;
  f.rowptr = rowptr; f.ent = reinterpret_cast<const int2*>(ent);
  f.momentum = momentum; f.lrate = lrate; f.unbias = unbias;
  int rc = launch_relu_product(X, M, p.Fhi, p.Flo, p.Cthi, p.Ctlo, p.ldct, b, Dp, x3,
                               p.part, dev_err, sms, g_timeout_ns, s, p.counter + 1, 0, 1);
  if (rc) return cuda_status(rc, "salsa_block_update");
  launch_finalize(f, s);
  return launched("salsa_block_update");
}

// ------------------------------------------------------------------------------ block CSR
size_t sumac_block_csr_workspace_bytes(int64_t m_fixed, int64_t nnz, int num_blocks, int64_t M) {
  return csr_workspace_bytes(m_fixed, nnz, num_blocks, M);
}

int sumac_block_csr_build(const int64_t* perm, int64_t m_fixed, int num_blocks,
                          const int32_t* e_fixed, const int32_t* e_out, const float* e_val,
                          int64_t nnz, int64_t M, int32_t* rowptr, int32_t* ent, void* ws,
                          size_t ws_bytes, sumac_stream_t stream) {
  if (m_fixed <= 0 || M <= 0 || num_blocks < 1 || num_blocks > m_fixed || nnz < 0)
    return fail(SUMAC_ERR_ARG, "block_csr_build: bad sizes");
  if (!perm || !rowptr || !ws || (nnz > 0 && (!e_fixed || !e_out || !e_val || !ent)))
    return fail(SUMAC_ERR_ARG, "block_csr_build: null pointer");
  int rc = launch_block_csr(perm, m_fixed, num_blocks, e_fixed, e_out, e_val, nnz, M, rowptr,
                            reinterpret_cast<int2*>(ent), ws, ws_bytes,
                            reinterpret_cast<cudaStream_t>(stream));
  if (rc == -2) return fail(SUMAC_ERR_WORKSPACE, "block_csr_build: workspace too small");
  if (rc == -3) return fail(SUMAC_ERR_ARG, "block_csr_build: num_blocks*M or nnz exceeds int32");
  if (rc == -4) return fail(SUMAC_ERR_UNSUPPORTED, "block_csr_build: num_blocks > 4096");
  return cuda_status(rc, "block_csr_build");
}

// ------------------------------------------------------------------------------ GD block gradient
struct GdPlan {
  float *AI, *AIhi, *AIlo, *AIthi, *AItlo, *Bhi, *Blo, *Bthi, *Btlo, *part;
  unsigned int* stats;
  int64_t ldb, ldn;
  size_t bytes;
};
static GdPlan plan_gd(void* ws, int64_t n, int64_t b, int Dp, bool x3, int sms) {
  Bump bp(ws);
  GdPlan p;
  p.ldb = round4(b);
  p.ldn = round4(n);
  p.AI = bp.take<float>((size_t)b * Dp);
  p.AIhi = bp.take<float>((size_t)b * Dp);
  p.AIlo = x3 ? bp.take<float>((size_t)b * Dp) : nullptr;
  p.AIthi = bp.take<float>((size_t)Dp * p.ldb);
  p.AItlo = x3 ? bp.take<float>((size_t)Dp * p.ldb) : nullptr;
  p.Bhi = x3 ? bp.take<float>((size_t)n * Dp) : nullptr;
  p.Blo = x3 ? bp.take<float>((size_t)n * Dp) : nullptr;
  p.Bthi = bp.take<float>((size_t)Dp * p.ldn);
  p.Btlo = x3 ? bp.take<float>((size_t)Dp * p.ldn) : nullptr;
  size_t need = 0;
  for (int64_t bb = b; bb > 0; bb /= 2) {
    const size_t s1 = (size_t)product_split_count(n, bb, Dp, x3, sms) * n * Dp;
    const size_t s2 = (size_t)product_split_count(bb, n, Dp, x3, sms) * bb * Dp;
    if (s1 > need) need = s1;
    if (s2 > need) need = s2;
    if (bb == 1) break;
  }
  p.part = bp.take<float>(need);
  p.stats = bp.take<unsigned int>(8);
  p.bytes = bp.off + 256;
  return p;
}

size_t sumac_gd_grad_workspace_bytes(int64_t n, int64_t b_max, int d, int precision) {
  const int Dp = padded(d);
  if (!Dp) return 0;
  return plan_gd(nullptr, n, b_max, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

int sumac_gd_block_grad(const float* A, const float* B, int64_t n, int d, const int64_t* rows,
                        int64_t b, const int32_t* rowptr_b, const int32_t* ent_b,
                        const int32_t* rowptr_a, const int32_t* ent_a, float* gA, float* gB,
                        int accumulate, int precision, void* ws, size_t ws_bytes, int* dev_err,
                        sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  const int Dp = padded(d);
  if (b <= 0 || n <= 0) return fail(SUMAC_ERR_ARG, "gd_block_grad: empty shape");
  if (!A || !B || !rows || !gA || !gB || !dev_err || (rowptr_b && !ent_b) || (rowptr_a && !ent_a))
    return fail(SUMAC_ERR_ARG, "gd_block_grad: null pointer");
  if (!Dp || !product_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "gd_block_grad: rank %d not supported with precision %d", d, precision);
  if (!aligned16(A) || !aligned16(B) || !aligned16(gA) || !aligned16(gB))
    return fail(SUMAC_ERR_ARG, "gd_block_grad: factors must be 16-byte aligned");
  const int sms = num_sms_current();
  GdPlan p = plan_gd(ws, n, b, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes) return fail(SUMAC_ERR_WORKSPACE, "gd_block_grad: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // pass B: rows j of B, contraction over the b block rows; C = A_I
  launch_gather_pad(A, Dp, Dp, rows, b, Dp, p.AI, p.AIhi, x3 ? p.AIlo : nullptr, s);
  launch_transpose_split(p.AI, b, Dp, p.AIthi, p.AItlo, p.ldb, s);
  if (!x3) launch_operand_stats(p.AI, b, Dp, p.AIthi, (int64_t)Dp * p.ldb, p.stats, s);
  FinalizeArgs f{};
  f.mode = FIN_GRAD; f.M = n; f.Dp = Dp; f.splits = product_split_count(n, b, Dp, x3, sms);
  f.ws = p.part; f.X = const_cast<float*>(B); f.F = p.AI; f.Cm = p.AI;
  f.rowptr = rowptr_b; f.ent = reinterpret_cast<const int2*>(ent_b);
  f.out = gB; f.scale = 2.f; f.accumulate = accumulate;
  int rc = launch_relu_product(B, n, p.AIhi, p.AIlo, p.AIthi, p.AItlo, p.ldb, b, Dp,
                               x3, p.part, dev_err, sms, g_timeout_ns, s, p.stats, 0, 1);
  if (rc) return cuda_status(rc, "gd_block_grad (B pass)");
  launch_finalize(f, s);
  // pass A: rows i of A_I, contraction over all n rows of B; C = B
  if (x3) launch_gather_pad(B, Dp, Dp, nullptr, n, Dp, nullptr, p.Bhi, p.Blo, s);
  launch_transpose_split(B, n, Dp, p.Bthi, p.Btlo, p.ldn, s);
  if (!x3) launch_operand_stats(B, n, Dp, p.Bthi, (int64_t)Dp * p.ldn, p.stats + 4, s);
  rc = launch_relu_product(p.AI, b, x3 ? p.Bhi : B, p.Blo, p.Bthi, p.Btlo, p.ldn, n, Dp, x3,
                           p.part, dev_err, sms, g_timeout_ns, s, p.stats + 4);
  if (rc) return cuda_status(rc, "gd_block_grad (A pass)");
  FinalizeArgs g{};
  g.mode = FIN_GRAD; g.M = b; g.Dp = Dp; g.splits = product_split_count(b, n, Dp, x3, sms);
  g.ws = p.part; g.X = p.AI; g.F = B; g.Cm = B;
  g.rowptr = rowptr_a; g.ent = reinterpret_cast<const int2*>(ent_a);
  g.out = gA; g.out_rows = rows; g.scale = 2.f; g.accumulate = accumulate;
  launch_finalize(g, s);
  return launched("gd_block_grad");
}

// ------------------------------------------------------------------------------ metrics / loss
struct EvalPlan {
  float *Fhi, *Flo;
  double *red, *sp;
  size_t bytes;
};
static EvalPlan plan_eval(void* ws, int64_t nf, int64_t nsparse, int Dp, bool x3, int sms) {
  Bump bp(ws);
  EvalPlan p;
  p.Fhi = x3 ? bp.take<float>((size_t)nf * Dp) : nullptr;
  p.Flo = x3 ? bp.take<float>((size_t)nf * Dp) : nullptr;
  p.red = bp.take<double>((size_t)sms * 3 + 3);
  p.sp = bp.take<double>((size_t)sparse_terms_grid(nsparse) * 6);
  p.bytes = bp.off + 256;
  return p;
}

size_t sumac_eval_terms_workspace_bytes(int64_t m, int64_t n, int64_t nnz, int d, int precision) {
  const int Dp = padded(d);
  if (!Dp) return 0;
  return plan_eval(nullptr, m < n ? m : n, nnz, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

static int eval_terms_impl(const float* A, const float* B, int64_t m, int64_t n, int d,
                           const int32_t* ei, const int32_t* ej, const float* v, int64_t nnz,
                           double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                           sumac_stream_t stream, bool count) {
  const bool x3 = precision == SUMAC_3XTF32;
  const int Dp = padded(d);
  if (m <= 0 || n <= 0 || nnz < 0) return fail(SUMAC_ERR_ARG, "eval_terms: empty shape");
  if (!A || !B || !out || !dev_err || (nnz > 0 && (!ei || !ej || !v)))
    return fail(SUMAC_ERR_ARG, "eval_terms: null pointer");
  if (!Dp || !reduce_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "eval_terms: rank %d not supported with precision %d", d, precision);
  const int sms = num_sms_current();
  // sum ReLU(A B^T) is symmetric in the roles: stream the larger factor as the row tiles
  const float* X = m >= n ? A : B;
  const float* F = m >= n ? B : A;
  const int64_t MX = m >= n ? m : n, NF = m >= n ? n : m;
  EvalPlan p = plan_eval(ws, NF, nnz, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes) return fail(SUMAC_ERR_WORKSPACE, "eval_terms: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (x3) launch_gather_pad(F, Dp, Dp, nullptr, NF, Dp, nullptr, p.Fhi, p.Flo, s);
  int grid = 0;
  int rc = launch_relu_reduce(X, MX, x3 ? p.Fhi : F, p.Flo, NF, Dp, x3, p.red, &grid, dev_err, sms,
                              g_timeout_ns, s, count ? 1 : 0);
  if (rc) return cuda_status(rc, "eval_terms");
  if (count) {
    // (sum, sum^2, count) partials: the count goes to out[8]
    launch_sum_partials(p.red, grid, 3, p.red + (size_t)grid * 3, 0, s);
    cudaMemcpyAsync(out, p.red + (size_t)grid * 3, 2 * sizeof(double), cudaMemcpyDeviceToDevice, s);
    cudaMemcpyAsync(out + 8, p.red + (size_t)grid * 3 + 2, sizeof(double),
                    cudaMemcpyDeviceToDevice, s);
  } else {
    launch_sum_partials(p.red, grid, 2, out, 0, s);
  }
  const int g2 = sparse_terms_grid(nnz);
  launch_sparse_terms_coo(A, B, Dp, ei, ej, v, nnz, p.sp, g2, s);
  launch_sum_partials(p.sp, g2, 6, out + 2, 0, s);
  return launched("eval_terms");
}

int sumac_eval_terms(const float* A, const float* B, int64_t m, int64_t n, int d,
                     const int32_t* ei, const int32_t* ej, const float* v, int64_t nnz,
                     double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                     sumac_stream_t stream) {
  return eval_terms_impl(A, B, m, n, d, ei, ej, v, nnz, out, precision, ws, ws_bytes, dev_err,
                         stream, false);
}

int sumac_eval_terms_fnnz(const float* A, const float* B, int64_t m, int64_t n, int d,
                          const int32_t* ei, const int32_t* ej, const float* v, int64_t nnz,
                          double* out, int precision, void* ws, size_t ws_bytes, int* dev_err,
                          sumac_stream_t stream) {
  return eval_terms_impl(A, B, m, n, d, ei, ej, v, nnz, out, precision, ws, ws_bytes, dev_err,
                         stream, true);
}

struct LossPlan {
  float *AI, *AIhi, *AIlo;
  double *red, *sp;
  size_t bytes;
};
static LossPlan plan_loss(void* ws, int64_t n, int64_t b, int Dp, bool x3, int sms) {
  Bump bp(ws);
  LossPlan p;
  p.AI = bp.take<float>((size_t)b * Dp);
  p.AIhi = bp.take<float>((size_t)b * Dp);
  p.AIlo = x3 ? bp.take<float>((size_t)b * Dp) : nullptr;
  p.red = bp.take<double>((size_t)sms * 2);
  p.sp = bp.take<double>((size_t)sparse_terms_grid(n) * 6);
  p.bytes = bp.off + 256;
  return p;
}

size_t sumac_block_loss_workspace_bytes(int64_t n, int64_t b_max, int d, int precision) {
  const int Dp = padded(d);
  if (!Dp) return 0;
  return plan_loss(nullptr, n, b_max, Dp, precision == SUMAC_3XTF32, num_sms_current()).bytes;
}

int sumac_block_loss_terms(const float* A, const float* B, int64_t n, int d, const int64_t* rows,
                           int64_t b, const int32_t* rowptr_b, const int32_t* ent_b, double* out,
                           int accumulate, int precision, void* ws, size_t ws_bytes, int* dev_err,
                           sumac_stream_t stream) {
  const bool x3 = precision == SUMAC_3XTF32;
  const int Dp = padded(d);
  if (b <= 0 || n <= 0) return fail(SUMAC_ERR_ARG, "block_loss_terms: empty shape");
  if (!A || !B || !rows || !out || !dev_err || !rowptr_b || !ent_b)
    return fail(SUMAC_ERR_ARG, "block_loss_terms: null pointer");
  if (!Dp || !reduce_supported(Dp, x3))
    return fail(SUMAC_ERR_UNSUPPORTED, "block_loss_terms: rank %d not supported", d);
  const int sms = num_sms_current();
  LossPlan p = plan_loss(ws, n, b, Dp, x3, sms);
  if (!ws || ws_bytes < p.bytes) return fail(SUMAC_ERR_WORKSPACE, "block_loss_terms: workspace %zu < %zu", ws_bytes, p.bytes);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  launch_gather_pad(A, Dp, Dp, rows, b, Dp, p.AI, p.AIhi, x3 ? p.AIlo : nullptr, s);
  int grid = 0;
  int rc = launch_relu_reduce(B, n, p.AIhi, p.AIlo, b, Dp, x3, p.red, &grid, dev_err,
                              sms, g_timeout_ns, s, 0, 1);
  if (rc) return cuda_status(rc, "block_loss_terms");
  launch_sum_partials(p.red, grid, 2, out, accumulate, s);
  const int g2 = sparse_terms_grid(n);
  launch_sparse_terms_csr(B, p.AI, Dp, rowptr_b, n, reinterpret_cast<const int2*>(ent_b), p.sp, g2, s);
  launch_sum_partials(p.sp, g2, 6, out + 2, accumulate, s);
  return launched("block_loss_terms");
}

// ------------------------------------------------------------------------------ optimizers
int sumac_adam_step(float* p, const float* g, float* m, float* v, int64_t n, float lr_over_bc1,
                    float inv_sqrt_bc2, float beta1, float beta2, float eps, sumac_stream_t stream) {
  if (n < 0 || (n > 0 && (!p || !g || !m || !v))) return fail(SUMAC_ERR_ARG, "adam_step: bad args");
  launch_adam(p, g, m, v, n, lr_over_bc1, inv_sqrt_bc2, beta1, beta2, eps,
              reinterpret_cast<cudaStream_t>(stream));
  return launched("adam_step");
}
int sumac_grad_sumsq(const float* g, int64_t n, double* sumsq, sumac_stream_t stream) {
  if (n < 0 || !sumsq || (n > 0 && !g)) return fail(SUMAC_ERR_ARG, "grad_sumsq: bad args");
  launch_sumsq(g, n, sumsq, reinterpret_cast<cudaStream_t>(stream));
  return launched("grad_sumsq");
}
int sumac_sgd_step(float* p, float* g, float* buf, int64_t n, float lr, float momentum, int first,
                   const double* sumsq, float max_norm, sumac_stream_t stream) {
  if (n < 0 || (n > 0 && (!p || !g || (momentum != 0.f && !buf))))
    return fail(SUMAC_ERR_ARG, "sgd_step: bad args");
  launch_sgd(p, g, buf, n, lr, momentum, first, sumsq, max_norm,
             reinterpret_cast<cudaStream_t>(stream));
  return launched("sgd_step");
}
int sumac_gather_owned_rows(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                            int64_t nrows, int Dp, float* out, sumac_stream_t stream) {
  if (nrows < 0 || hi < lo || padded(Dp) != Dp || (nrows > 0 && (!rows || !out)) ||
      (nrows > 0 && hi > lo && !local))
    return fail(SUMAC_ERR_ARG, "gather_owned_rows: bad args");
  if (!aligned16(local) || !aligned16(out))
    return fail(SUMAC_ERR_ARG, "gather_owned_rows: rows must be 16-byte aligned");
  launch_gather_owned_rows(local, lo, hi, rows, nrows, Dp, out, reinterpret_cast<cudaStream_t>(stream));
  return launched("gather_owned_rows");
}

int sumac_assemble_rows_p2p(const float* local, int64_t lo, int64_t hi, const int64_t* rows,
                            int64_t nrows, int Dp, int64_t slot_floats, float* const* peer_bufs,
                            unsigned int* const* peer_flags, unsigned int* epoch, int rank,
                            int world, int* dev_err, sumac_stream_t stream) {
  if (nrows < 0 || hi < lo || padded(Dp) != Dp || world < 1 || world > 512 || rank < 0 ||
      rank >= world || !peer_bufs || !peer_flags || !epoch || slot_floats < nrows * Dp ||
      (nrows > 0 && !rows) || (nrows > 0 && hi > lo && !local))
    return fail(SUMAC_ERR_ARG, "assemble_rows_p2p: bad args");
  if (!aligned16(local)) return fail(SUMAC_ERR_ARG, "assemble_rows_p2p: rows must be 16-byte aligned");
  launch_assemble_rows_p2p(local, lo, hi, rows, nrows, Dp, slot_floats, peer_bufs, peer_flags,
                           epoch, rank, world, dev_err, g_timeout_ns,
                           reinterpret_cast<cudaStream_t>(stream));
  return launched("assemble_rows_p2p");
}

int sumac_fill_zero(float* p, int64_t n, sumac_stream_t stream) {
  if (n < 0 || (n > 0 && !p)) return fail(SUMAC_ERR_ARG, "fill_zero: bad args");
  launch_fill_zero(p, n, reinterpret_cast<cudaStream_t>(stream));
  return launched("fill_zero");
}

// ------------------------------------------------------------------------------ initial factors
int sumac_init_factor(const int32_t* rowptr, const int32_t* col, const float* val, int64_t M,
                      const float* R, int d, float sign, float* out, sumac_stream_t stream) {
  if (M < 0 || d <= 0 || (M > 0 && (!rowptr || !R || !out)))
    return fail(SUMAC_ERR_ARG, "init_factor: bad args");
  launch_init_spmm_sqrt(rowptr, col, val, M, R, d, sign, out, reinterpret_cast<cudaStream_t>(stream));
  return launched("init_factor");
}
size_t sumac_init_scale_workspace_bytes(void) { return init_scale_workspace_bytes(); }
int sumac_init_scale_terms(const float* A, const float* B, int d, const int32_t* ei,
                           const int32_t* ej, const float* v, int64_t nnz, double* out, void* ws,
                           size_t ws_bytes, sumac_stream_t stream) {
  if (d <= 0 || nnz < 0 || !out || (nnz > 0 && (!A || !B || !ei || !ej || !v)))
    return fail(SUMAC_ERR_ARG, "init_scale_terms: bad args");
  if (!ws || ws_bytes < init_scale_workspace_bytes())
    return fail(SUMAC_ERR_WORKSPACE, "init_scale_terms: workspace too small");
  launch_init_scale_terms(A, B, d, ei, ej, v, nnz, static_cast<double*>(ws), out,
                          reinterpret_cast<cudaStream_t>(stream));
  return launched("init_scale_terms");
}

int sumac_wait_flag(const int* flag, int* dev_err, unsigned long long timeout_ns,
                    sumac_stream_t stream) {
  if (!flag || !dev_err) return fail(SUMAC_ERR_ARG, "wait_flag: null pointer");
  launch_wait_flag(flag, dev_err, timeout_ns, reinterpret_cast<cudaStream_t>(stream));
  return launched("wait_flag");
}

}  // extern "C"
