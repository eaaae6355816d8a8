// ccv_forward_noalloc: the reference-ABI forward (KRSC weights, TF32) for
// callers that cannot allocate device memory.
//
// Who needs this: code that runs inside another framework's execute/enqueue
// callback (an inference-server backend, a plugin of a graph runtime, a
// real-time loop) often may not call cudaMalloc at all: the host framework
// owns the device memory pool, and cudaMalloc/cudaFree can synchronize the
// device and stall every other stream.  ccv_forward needs scratch for the
// packed weight image, which such callers cannot provide.  This entry point
// keeps that scratch in a fixed, file-scope device array instead.
//
// Limits and sharing rules:
//   * The scratch holds one packed TF32 weight image of at most
//     CCV_NOALLOC_MAX_WEIGHT_BYTES (16 MiB: 3 planes x R*S*K*C fp32, e.g.
//     3x3 filters with K*C <= 155,344).  Larger problems are rejected with
//     CCV_ERR_WORKSPACE before any device work.
//   * Every GPU that loads this library reserves the 16 MiB when the module
//     is loaded and keeps it until the process exits.
//   * All calls on a device share the one array, and it keeps the last
//     call's contents.  Each call rewrites every element it reads (the
//     prepack fills the whole image), so nothing needs clearing, but calls
//     whose work overlaps on the GPU (different streams without ordering, or
//     several host threads) race on the array: order them on one stream.
//   * The first call on each device looks up the array's device address with
//     cudaGetSymbolAddress (with that device current) and caches it; make
//     that first call before any stream capture begins.
#include <cuda_runtime.h>

#include <mutex>
#include <string>

#include "ccv_internal.h"

// The scratch: one packed weight image, reserved on every device that loads
// this library.
static __device__ __align__(256) float g_noalloc_weights[CCV_NOALLOC_MAX_WEIGHT_BYTES / sizeof(float)];

namespace ccv {
namespace {

constexpr size_t kNoAllocMaxWeightBytes = CCV_NOALLOC_MAX_WEIGHT_BYTES;
constexpr int kMaxDev = 64;
std::mutex g_noalloc_mutex;
void* g_noalloc_addr[kMaxDev] = {};

// Device address of g_noalloc_weights on the current device (set-up on the
// first call per device).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev) return set_error(CCV_ERR_DEVICE, "device index out of range");
  std::lock_guard<std::mutex> lk(g_noalloc_mutex);
  if (g_noalloc_addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_weights);
    if (e != cudaSuccess) return cuda_error(e, "cudaGetSymbolAddress(no-alloc scratch)");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return CCV_OK;
}

}  // namespace
}  // namespace ccv

using namespace ccv;

extern "C" int ccv_forward_noalloc(const float* x_real, const float* x_imag,
                                   const float* w_real_krsc, const float* w_imag_krsc,
                                   float* y_real, float* y_imag, const ccv_conv_shape* shape,
                                   ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  const size_t need = ccv_packed_weight_bytes(shape, CCV_PRECISION_TF32);
  if (need > kNoAllocMaxWeightBytes) {
    return set_error(CCV_ERR_WORKSPACE,
                     "ccv_forward_noalloc: packed weights need " + std::to_string(need) +
                         " bytes, above the fixed scratch of " +
                         std::to_string(kNoAllocMaxWeightBytes) + " bytes; use ccv_forward");
  }
  void* scratch = nullptr;
  rc = noalloc_scratch(&scratch);
  if (rc != CCV_OK) return rc;
  // The entry-point bodies without the public functions' one-time pinned
  // allocation of the host-visible status mirror.
  rc = prepack_weights_impl(w_real_krsc, w_imag_krsc, CCV_WEIGHT_KRSC, shape, CCV_PRECISION_TF32,
                            scratch, kNoAllocMaxWeightBytes, stream);
  if (rc != CCV_OK) return rc;
  return fprop_planar_impl(x_real, x_imag, scratch, nullptr, nullptr, y_real, y_imag, shape,
                           CCV_PRECISION_TF32, nullptr, 0, stream);
}
