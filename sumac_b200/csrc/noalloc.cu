// noalloc.cu — sumac_relu_bat_reduce_noalloc: the relu_bat_reduce entry point for callers that
// cannot hand this library a workspace they allocated.
//
// Who needs it: a host that owns all device memory through its own pool (a MATLAB gpuArray / MEX
// binding, a serving process that reserved the whole GPU at start-up) and therefore cannot
// cudaMalloc a scratch buffer for us, or code on a latency-sensitive path where cudaMalloc and
// cudaFree are off limits because they may synchronise the device. This variant keeps its scratch
// in a fixed array in device memory that is part of the library image, so a call allocates
// nothing: the caller still passes the inputs A, B and the output `out`.
//
// Limits and rules:
//  - the scratch holds at most SCRATCH_BYTES (16 MiB); larger problems are rejected with
//    SUMAC_ERR_WORKSPACE and a message (use sumac_relu_bat_reduce with a caller workspace then);
//  - every GPU that loads the library holds the 16 MiB until the process exits;
//  - all calls on a device share the one array and it keeps the last call's contents; calls that
//    overlap on the GPU (different streams without ordering, or different host threads) race on
//    it. Nothing in it has to start at zero: each call writes every scratch byte it reads;
//  - the first call on a device looks up the array's device address (cudaGetSymbolAddress with
//    that device current); make that first call before any stream capture.
#include <cstdio>
#include <mutex>

#include "../../include/sumac_b200.h"
#include "kernels.cuh"

namespace {

constexpr size_t SCRATCH_BYTES = size_t(16) << 20;
static __device__ __align__(256) unsigned char g_scratch[SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
void* g_scratch_ptr[MAX_DEVICES] = {};
std::mutex g_scratch_mutex;

int scratch_for_current_device(void** out, const char** why) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= MAX_DEVICES) {
    *why = "no current CUDA device";
    return SUMAC_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    // g_scratch names a host-side stand-in here; the device address comes from the runtime.
    cudaError_t e = cudaGetSymbolAddress(&p, g_scratch);
    if (e != cudaSuccess || !p) {
      *why = cudaGetErrorString(e);
      return SUMAC_ERR_CUDA;
    }
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return SUMAC_OK;
}

}  // namespace

namespace sb {
int set_last_error(int code, const char* msg);
}

extern "C" {

size_t sumac_noalloc_scratch_bytes(void) { return SCRATCH_BYTES; }

int sumac_relu_bat_reduce_noalloc(const float* A, const float* B, int64_t M, int64_t N, int D,
                                  double* out, int precision, int* dev_err,
                                  sumac_stream_t stream) {
  // shape and pointer checks come first, so that a bad argument is reported as such (a negative
  // M or N would otherwise wrap to a huge scratch size and read as "too large")
  if (M <= 0 || N <= 0 || D <= 0)
    return sb::set_last_error(SUMAC_ERR_ARG, "relu_bat_reduce_noalloc: empty or negative shape");
  if (!A || !B || !out || !dev_err)
    return sb::set_last_error(SUMAC_ERR_ARG, "relu_bat_reduce_noalloc: null pointer");
  const size_t need = sumac_relu_bat_reduce_workspace_bytes(M, N, D, precision);
  if (need > SCRATCH_BYTES) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "relu_bat_reduce_noalloc: M=%lld N=%lld D=%d needs %zu bytes of scratch but the "
             "fixed scratch holds %zu; use sumac_relu_bat_reduce with a workspace",
             (long long)M, (long long)N, D, need, SCRATCH_BYTES);
    return sb::set_last_error(SUMAC_ERR_WORKSPACE, msg);
  }
  void* ws = nullptr;
  const char* why = "";
  if (scratch_for_current_device(&ws, &why) != SUMAC_OK) {
    char msg[256];
    snprintf(msg, sizeof(msg), "relu_bat_reduce_noalloc: scratch address lookup failed: %s", why);
    return sb::set_last_error(SUMAC_ERR_CUDA, msg);
  }
  // argument checks (shapes, pointers, supported rank) are those of the regular entry point
  return sumac_relu_bat_reduce(A, B, M, N, D, out, precision, ws, SCRATCH_BYTES, dev_err, stream);
}

}  // extern "C"
