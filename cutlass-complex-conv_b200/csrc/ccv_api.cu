// extern "C" entry points of libccv_b200.so (declared in include/ccv_b200.h):
// argument checking with the reference's error texts, per-device state
// (status word, SM count, architecture check), tensor-map encoding, and the
// composition of layout kernels with the fprop kernel.
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ccv_internal.h"

#define CCV_VERSION_STRING "ccv_b200 0.1.0 (sm_100a tcgen05/TMA)"

namespace ccv {

// Per-device status block.  Word 0: bounded in-kernel waits that run out
// write a CCV_ERR_* code here; fprop kernels read it at start and exit
// without work while it is set.  Words 2-3: device address of the host-mapped
// mirror of word 0 (null until the host sets it up), which the same waits
// also write, so that host code sees a timeout without synchronizing.
__device__ __align__(16) int g_ccv_status[4] = {0, 0, 0, 0};
// Counter sets (see acquire_counter_set); zero-initialized.
__device__ unsigned g_ccv_sk_counters[kCounterSets * kSkCounterWords];

namespace {

thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
int* g_status_ptr[kMaxDevices] = {};
volatile int* g_status_host[kMaxDevices] = {};  // host-mapped mirror of word 0
int g_sm_count[kMaxDevices] = {};
int g_arch_ok[kMaxDevices] = {};  // 0 unknown, 1 ok, -1 not sm_100

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode_tiled = nullptr;
std::once_flag g_encode_once;

int current_device(int* dev) {
  const cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return cuda_error(e, "cudaGetDevice");
  if (*dev < 0 || *dev >= kMaxDevices) return set_error(CCV_ERR_DEVICE, "device index out of range");
  return CCV_OK;
}

int check_device() {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != CCV_OK) return rc;
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  if (g_arch_ok[dev] == 0) {
    int major = 0, minor = 0, sms = 0;
    cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_error(e, "cudaDeviceGetAttribute");
    g_sm_count[dev] = sms;
    g_arch_ok[dev] = (major == 10 && minor == 0) ? 1 : -1;
  }
  if (g_arch_ok[dev] != 1) {
    return set_error(CCV_ERR_DEVICE,
                     "complex_conv2d B200 kernels need an sm_100 (B200/GB200) device");
  }
  return CCV_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Bytes of one fp32 NHWC input plane, rounded up to 256.
size_t plane_bytes_aligned(const Problem& pb) {
  const size_t plane = static_cast<size_t>(pb.n) * pb.h * pb.w * pb.c * sizeof(float);
  return (plane + 255) & ~static_cast<size_t>(255);
}

}  // namespace

int set_error(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_error(cudaError_t e, const char* what) {
  return set_error(CCV_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

namespace {

int env_int(const char* name, int dflt) {
  const char* v = getenv(name);
  return v != nullptr && *v != '\0' ? atoi(v) : dflt;
}

Knobs parse_knobs() {
  Knobs k;
  k.pdl = env_int("CCV_PDL", 1);
  k.kt = env_int("CCV_KT", 0);
  k.force_kernel = env_int("CCV_FORCE_KERNEL", 0);
  k.halo = env_int("CCV_HALO", -1);
  k.splitk = env_int("CCV_SPLITK", 0);
  k.lw = env_int("CCV_LW", -1);
  k.lw_prefix = env_int("CCV_LW_PREFIX", -1);
  k.lw_tma = env_int("CCV_LW_TMA", 1);
  k.lw_tma_images = env_int("CCV_LW_TMA_IMAGES", 0);
  k.lw_tma_bufs = env_int("CCV_LW_TMA_BUFS", 0);
  k.subbox = env_int("CCV_SUBBOX", 1);
  k.streamk = env_int("CCV_STREAMK", -1);
  k.max_clusters = env_int("CCV_MAX_CLUSTERS", 0);
  k.tma_store = env_int("CCV_TMA_STORE", 1);
  return k;
}

// Readers may hold a reference across a reload, so replaced snapshots are
// kept (a reload is a testing/benchmarking action, a few per process).
std::atomic<const Knobs*> g_knobs{nullptr};
std::mutex g_knobs_mutex;

// Counter sets per device: the set's completion event (created on first
// use), whether it has been handed out, and whether a captured graph owns
// it for good.
struct CounterSlot {
  cudaEvent_t done = nullptr;
  bool used = false;
  bool reserved = false;
};
CounterSlot g_slots[kMaxDevices][kCounterSets];
unsigned g_next_slot[kMaxDevices] = {};
unsigned* g_sk_base[kMaxDevices] = {};

// Sets this host thread took since its innermost CounterScope began.
struct PendingSets {
  int dev = -1;
  int slots[8];
  int count = 0;
  int depth = 0;
};
thread_local PendingSets t_pending;

}  // namespace

const Knobs& knobs() {
  const Knobs* k = g_knobs.load(std::memory_order_acquire);
  if (k == nullptr) {
    reload_knobs();
    k = g_knobs.load(std::memory_order_acquire);
  }
  return *k;
}

void reload_knobs() {
  std::lock_guard<std::mutex> lk(g_knobs_mutex);
  g_knobs.store(new Knobs(parse_knobs()), std::memory_order_release);
}

unsigned* acquire_counter_set(cudaStream_t stream) {
  int dev = 0;
  if (current_device(&dev) != CCV_OK) return nullptr;
  if (t_pending.depth == 0 || t_pending.count >= 8) return nullptr;
  if (t_pending.count > 0 && t_pending.dev != dev) return nullptr;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  const bool capturing = cap != cudaStreamCaptureStatusNone;
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  if (g_sk_base[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ccv_sk_counters);
    if (e != cudaSuccess) {
      cuda_error(e, "cudaGetSymbolAddress(counter sets)");
      return nullptr;
    }
    g_sk_base[dev] = static_cast<unsigned*>(p);
  }
  for (int i = 0; i < kCounterSets; ++i) {
    const int slot = static_cast<int>((g_next_slot[dev] + i) % kCounterSets);
    CounterSlot& cs = g_slots[dev][slot];
    if (cs.reserved) continue;
    bool pending_here = false;
    for (int j = 0; j < t_pending.count; ++j) pending_here |= t_pending.slots[j] == slot;
    if (pending_here) continue;
    if (cs.used) {
      // Querying events is not allowed while a stream captures; a set
      // that has been used is then skipped.
      if (capturing) continue;
      const cudaError_t q = cudaEventQuery(cs.done);
      if (q == cudaErrorNotReady) continue;
      if (q != cudaSuccess) {
        cudaGetLastError();
        continue;
      }
    }
    if (cs.done == nullptr && !capturing) {
      if (cudaEventCreateWithFlags(&cs.done, cudaEventDisableTiming) != cudaSuccess) {
        cudaGetLastError();
        cs.done = nullptr;
        return nullptr;
      }
    }
    if (cs.done == nullptr && !capturing) return nullptr;
    cs.used = true;
    if (capturing) cs.reserved = true;
    g_next_slot[dev] = static_cast<unsigned>(slot + 1);
    t_pending.dev = dev;
    t_pending.slots[t_pending.count++] = capturing ? -1 - slot : slot;
    return g_sk_base[dev] + static_cast<size_t>(slot) * kSkCounterWords;
  }
  return nullptr;
}

CounterScope::CounterScope(cudaStream_t stream) : stream_(stream) {
  if (t_pending.depth++ == 0) t_pending.count = 0;
}

CounterScope::~CounterScope() {
  if (--t_pending.depth != 0) return;
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  for (int j = 0; j < t_pending.count; ++j) {
    const int slot = t_pending.slots[j];
    if (slot < 0) continue;  // owned by a captured graph
    CounterSlot& cs = g_slots[t_pending.dev][slot];
    if (cudaEventRecord(cs.done, stream_) != cudaSuccess) {
      // Without an event the set cannot be known free again: keep it out.
      cudaGetLastError();
      cs.reserved = true;
    }
  }
  t_pending.count = 0;
}

int* device_status_ptr() {
  int dev = 0;
  if (current_device(&dev) != CCV_OK) return nullptr;
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_ccv_status);
    if (e != cudaSuccess) {
      cuda_error(e, "cudaGetSymbolAddress(status)");
      return nullptr;
    }
    g_status_ptr[dev] = static_cast<int*>(p);
  }
  return g_status_ptr[dev];
}

namespace {

// Sets up the host-mapped mirror of the current device's status word (once
// per device; a pinned host allocation, skipped while `stream` captures).
void ensure_status_mirror(cudaStream_t stream) {
  int dev = 0;
  if (current_device(&dev) != CCV_OK) return;
  {
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if (g_status_host[dev] != nullptr) return;
  }
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone) {
    cudaGetLastError();
    return;
  }
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  if (g_status_host[dev] != nullptr) return;
  int* h = nullptr;
  if (cudaHostAlloc(reinterpret_cast<void**>(&h), sizeof(int),
                    cudaHostAllocMapped | cudaHostAllocPortable) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  *h = 0;
  void* d = nullptr;
  if (cudaHostGetDevicePointer(&d, h, 0) != cudaSuccess ||
      cudaMemcpyToSymbol(g_ccv_status, &d, sizeof(d), 2 * sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    cudaFreeHost(h);
    return;
  }
  g_status_host[dev] = h;
}

// CCV_ERR_DEVICE when a kernel on the current device has reported a timeout
// that the host can see (the status mirror is set): the library's kernels
// would skip their work, so nothing is launched.
int check_status_clear() {
  int dev = 0;
  const int rc = current_device(&dev);
  if (rc != CCV_OK) return rc;
  const volatile int* h = g_status_host[dev];
  if (h != nullptr && *h != 0) {
    return set_error(CCV_ERR_DEVICE,
                     "a library kernel on this device gave up a bounded wait (status " +
                         std::to_string(*h) +
                         "); outputs since then are invalid - call ccv_clear_device_status");
  }
  return CCV_OK;
}

}  // namespace

int device_sm_count() {
  int dev = 0;
  if (current_device(&dev) != CCV_OK) return 148;
  std::lock_guard<std::mutex> lk(g_dev_mutex);
  return g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
}

int encode_tiled(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, const uint32_t* elem_strides,
                 int swizzle_bytes) {
  return encode_tiled_ex(map, base, rank, dims, strides_bytes, box, elem_strides,
                         swizzle_bytes == 128 ? kSwizzle128 : kSwizzle64, false);
}

int encode_tiled_ex(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box,
                    const uint32_t* elem_strides, TmaSwizzle swizzle, bool elem8) {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode_tiled = reinterpret_cast<EncodeTiledFn>(fn);
    }
  });
  if (g_encode_tiled == nullptr) {
    return set_error(CCV_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  }
  cuuint64_t d[5];
  cuuint64_t st[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    es[i] = elem_strides[i];
    if (i + 1 < rank) st[i] = strides_bytes[i];
  }
  const CUtensorMapSwizzle sw = swizzle == kSwizzle128   ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle == kSwizzleNone ? CU_TENSOR_MAP_SWIZZLE_NONE
                                                          : CU_TENSOR_MAP_SWIZZLE_64B;
  // 8-byte elements (complex64 moved as opaque 64-bit words) or fp32.
  const CUresult r = g_encode_tiled(
      map, elem8 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT64 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank,
      const_cast<void*>(base), d, st, bx, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
      CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return set_error(CCV_ERR_UNSUPPORTED,
                     "cuTensorMapEncodeTiled rejected the problem (error " + std::to_string(r) + ")");
  }
  return CCV_OK;
}

int make_problem(const ccv_conv_shape* shape, Problem* out) {
  if (shape == nullptr) return set_error(CCV_ERR_INVALID_ARGUMENT, "shape is null");
  const ccv_conv_shape& s = *shape;
  if (s.n <= 0 || s.h <= 0 || s.w <= 0 || s.c <= 0 || s.k <= 0) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor dimensions must be positive");
  }
  if (s.r <= 0 || s.s <= 0) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "kernel dimensions must be positive");
  }
  if (s.stride_h <= 0 || s.stride_w <= 0) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "stride must be positive");
  }
  if (s.pad_h < 0 || s.pad_w < 0) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "padding must be non-negative");
  }
  const int64_t lim = 0x7fffffffLL;
  if (s.n > lim || s.h > lim || s.w > lim || s.c > lim || s.k > lim || s.r > lim || s.s > lim ||
      s.pad_h > (1 << 20) || s.pad_w > (1 << 20) || s.stride_h > lim || s.stride_w > lim) {
    return set_error(CCV_ERR_UNSUPPORTED, "cannot implement this convolution configuration: "
                                          "dimension exceeds 32-bit range");
  }
  const int64_t p = (s.h + 2 * s.pad_h - s.r) / s.stride_h + 1;
  const int64_t q = (s.w + 2 * s.pad_w - s.s) / s.stride_w + 1;
  if (s.h + 2 * s.pad_h - s.r < 0 || s.w + 2 * s.pad_w - s.s < 0 || p <= 0 || q <= 0) {
    return set_error(CCV_ERR_INVALID_ARGUMENT,
                     "invalid convolution configuration: output spatial size must be positive");
  }
  if (s.c % 4 != 0 || s.k % 4 != 0) {
    return set_error(CCV_ERR_UNSUPPORTED,
                     "cannot implement this convolution configuration: input and output "
                     "channel counts must be multiples of 4");
  }
  if (s.stride_h > 8 || s.stride_w > 8) {
    return set_error(CCV_ERR_UNSUPPORTED,
                     "cannot implement this convolution configuration: stride above 8");
  }
  if (s.n * s.h * s.w * s.c * 4 >= (1LL << 40) || s.n * p * q * s.k * 8 >= (1LL << 40)) {
    return set_error(CCV_ERR_UNSUPPORTED,
                     "cannot implement this convolution configuration: tensor too large");
  }
  Problem pb;
  pb.n = static_cast<int>(s.n); pb.h = static_cast<int>(s.h); pb.w = static_cast<int>(s.w);
  pb.c = static_cast<int>(s.c); pb.k = static_cast<int>(s.k); pb.r = static_cast<int>(s.r);
  pb.s = static_cast<int>(s.s); pb.p = static_cast<int>(p); pb.q = static_cast<int>(q);
  pb.sh = static_cast<int>(s.stride_h); pb.sw = static_cast<int>(s.stride_w);
  pb.ph = static_cast<int>(s.pad_h); pb.pw = static_cast<int>(s.pad_w);
  *out = pb;
  return CCV_OK;
}

}  // namespace ccv

using namespace ccv;

extern "C" {

const char* ccv_version(void) { return CCV_VERSION_STRING; }

const char* ccv_last_error_message(void) { return g_last_error.c_str(); }

int ccv_output_size(const ccv_conv_shape* shape, int64_t* p, int64_t* q) {
  Problem pb;
  const int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (p) *p = pb.p;
  if (q) *q = pb.q;
  return CCV_OK;
}

int ccv_check_shape(const ccv_conv_shape* shape) {
  Problem pb;
  return make_problem(shape, &pb);
}

size_t ccv_packed_weight_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  const size_t img = packed_image_floats(pb) * sizeof(float);
  return precision == CCV_PRECISION_3XTF32 ? 2 * img : img;
}

int ccv_prepack_weights(const float* w_real, const float* w_imag, int layout,
                        const ccv_conv_shape* shape, int precision, void* packed,
                        size_t packed_bytes, ccv_stream_t stream) {
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  return prepack_weights_impl(w_real, w_imag, layout, shape, precision, packed, packed_bytes,
                              stream);
}

}  // extern "C"

namespace ccv {

int prepack_weights_impl(const float* w_real, const float* w_imag, int layout,
                         const ccv_conv_shape* shape, int precision, void* packed,
                         size_t packed_bytes, ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (layout != CCV_WEIGHT_KCRS && layout != CCV_WEIGHT_KRSC) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown weight layout");
  }
  if (precision != CCV_PRECISION_TF32 && precision != CCV_PRECISION_3XTF32) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown precision");
  }
  if (w_real == nullptr || w_imag == nullptr || packed == nullptr) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null weight pointer");
  }
  if (!aligned16(packed)) return set_error(CCV_ERR_INVALID_ARGUMENT, "packed weights must be 16-byte aligned");
  if (packed_bytes < ccv_packed_weight_bytes(shape, precision)) {
    return set_error(CCV_ERR_WORKSPACE, "packed weight buffer too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  return launch_prepack(w_real, w_imag, layout, pb, precision, static_cast<float*>(packed),
                        reinterpret_cast<cudaStream_t>(stream));
}

namespace {

size_t align256(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

// Workspace a planar call cannot run without: 3xTF32 splits the input planes
// into TF32 parts and remainders (4 planes).
size_t planar_required_bytes(const Problem& pb, int precision) {
  return precision == CCV_PRECISION_3XTF32 ? 4 * plane_bytes_aligned(pb) : 0;
}

// Workspace a complex call cannot run without: fp32 NHWC planes of the
// input (real, imaginary; 3xTF32: also remainders).
size_t complex_required_bytes(const Problem& pb, int precision) {
  return (precision == CCV_PRECISION_3XTF32 ? 4 : 2) * plane_bytes_aligned(pb);
}

// The part of a caller's workspace past the required bytes, handed to the
// kernels as stream-K scratch (null when nothing usable is left).
void split_scratch(void* workspace, size_t workspace_bytes, size_t required, void** ws,
                   size_t* ws_bytes) {
  *ws = nullptr;
  *ws_bytes = 0;
  if (workspace == nullptr) return;
  const uintptr_t base = reinterpret_cast<uintptr_t>(workspace);
  const uintptr_t start = (base + align256(required) + 255) & ~static_cast<uintptr_t>(255);
  const uintptr_t end = base + workspace_bytes;
  if (start >= end) return;
  *ws = reinterpret_cast<void*>(start);
  *ws_bytes = end - start;
}

int check_precision(int precision) {
  if (precision != CCV_PRECISION_TF32 && precision != CCV_PRECISION_3XTF32) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown precision");
  }
  return CCV_OK;
}

int make_epilogue(const float* bias_real, const float* bias_imag, Epilogue* ep) {
  if ((bias_real == nullptr) != (bias_imag == nullptr)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "bias_real and bias_imag must both be set or both null");
  }
  if (bias_real != nullptr && (!aligned16(bias_real) || !aligned16(bias_imag))) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "bias pointers must be 16-byte aligned");
  }
  ep->bias_r = bias_real;
  ep->bias_i = bias_imag;
  return CCV_OK;
}

}  // namespace

int fprop_planar_impl(const float* x_real, const float* x_imag, const void* w_packed,
                      const float* bias_real, const float* bias_imag, float* y_real,
                      float* y_imag, const ccv_conv_shape* shape, int precision, void* workspace,
                      size_t workspace_bytes, ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if ((rc = check_precision(precision)) != CCV_OK) return rc;
  if (!x_real || !x_imag || !w_packed || !y_real || !y_imag) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  }
  if (!aligned16(x_real) || !aligned16(x_imag) || !aligned16(w_packed) || !aligned16(y_real) ||
      !aligned16(y_imag)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  Epilogue ep;
  if ((rc = make_epilogue(bias_real, bias_imag, &ep)) != CCV_OK) return rc;
  const size_t need = planar_required_bytes(pb, precision);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CounterScope scope(st);
  void* sk = nullptr;
  size_t sk_bytes = 0;
  split_scratch(workspace, workspace_bytes, need, &sk, &sk_bytes);
  const float* wp = static_cast<const float*>(w_packed);
  if (precision == CCV_PRECISION_3XTF32) {
    const size_t pl = plane_bytes_aligned(pb);
    char* ws = static_cast<char*>(workspace);
    float* hr = reinterpret_cast<float*>(ws);
    float* hi = reinterpret_cast<float*>(ws + pl);
    float* lr = reinterpret_cast<float*>(ws + 2 * pl);
    float* li = reinterpret_cast<float*>(ws + 3 * pl);
    if (use_layout_warps_planar(pb, precision)) {
      rc = launch_fprop_planar_lw(x_real, x_imag, hr, hi, lr, li, wp, y_real, y_imag, pb, ep, sk,
                                  sk_bytes, st);
      if (rc != kNoCounterSet) return rc;
    }
    rc = launch_split_planes(x_real, x_imag, hr, hi, lr, li,
                             static_cast<size_t>(pb.n) * pb.h * pb.w * pb.c, st);
    if (rc != CCV_OK) return rc;
    return launch_fprop(hr, hi, lr, li, wp, y_real, y_imag, pb, precision, OUT_PLANAR_NHWC, ep, sk,
                        sk_bytes, st);
  }
  return launch_fprop(x_real, x_imag, nullptr, nullptr, wp, y_real, y_imag, pb, precision,
                      OUT_PLANAR_NHWC, ep, sk, sk_bytes, st);
}

int fprop_complex_impl(const void* x, const int64_t* x_strides, const void* w_packed,
                       const float* bias_real, const float* bias_imag, void* y,
                       const ccv_conv_shape* shape, int precision, void* workspace,
                       size_t workspace_bytes, ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if ((rc = check_precision(precision)) != CCV_OK) return rc;
  if (!x || !w_packed || !y) return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  // Dense NCHW input, unless strides say otherwise.
  bool dense = true;
  if (x_strides != nullptr) {
    const int64_t hw = static_cast<int64_t>(pb.h) * pb.w;
    dense = x_strides[0] == hw * pb.c && x_strides[1] == hw && x_strides[2] == pb.w &&
            x_strides[3] == 1;
    for (int i = 0; i < 4; ++i) {
      if (x_strides[i] < 0) return set_error(CCV_ERR_INVALID_ARGUMENT, "negative input stride");
    }
  }
  if ((reinterpret_cast<uintptr_t>(x) & 7u) != 0) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "complex input must be 8-byte aligned");
  }
  // The layout-warp path reads dense input in 16-byte pieces; a dense input
  // at an 8-byte boundary goes through the layout kernels (8-byte loads).
  if (x_strides == nullptr && !aligned16(x)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  dense = dense && aligned16(x);
  if (!aligned16(w_packed) || !aligned16(y)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  Epilogue ep;
  if ((rc = make_epilogue(bias_real, bias_imag, &ep)) != CCV_OK) return rc;
  const size_t need = complex_required_bytes(pb, precision);
  if (workspace == nullptr || workspace_bytes < need || !aligned16(workspace)) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  CounterScope scope(st);
  void* sk = nullptr;
  size_t sk_bytes = 0;
  split_scratch(workspace, workspace_bytes, need, &sk, &sk_bytes);
  const size_t pl = plane_bytes_aligned(pb);
  char* ws = static_cast<char*>(workspace);
  float* xr = reinterpret_cast<float*>(ws);
  float* xi = reinterpret_cast<float*>(ws + pl);
  const bool split = precision == CCV_PRECISION_3XTF32;
  float* lr = split ? reinterpret_cast<float*>(ws + 2 * pl) : nullptr;
  float* li = split ? reinterpret_cast<float*>(ws + 3 * pl) : nullptr;
  const float* wp = static_cast<const float*>(w_packed);
  if (dense && use_layout_warps(pb, precision)) {
    rc = launch_fprop_complex_lw(static_cast<const float*>(x), xr, xi, lr, li, wp,
                                 static_cast<float*>(y), pb, precision, ep, sk, sk_bytes, st);
    if (rc != kNoCounterSet) return rc;
  }
  rc = dense ? launch_nchw_complex_to_planar(static_cast<const float*>(x), xr, xi, lr, li, pb, st)
             : launch_strided_complex_to_planar(static_cast<const float*>(x), x_strides, xr, xi,
                                                lr, li, pb, st);
  if (rc != CCV_OK) return rc;
  return launch_fprop(xr, xi, lr, li, wp, static_cast<float*>(y), nullptr, pb, precision,
                      OUT_COMPLEX_NCHW, ep, sk, sk_bytes, st);
}

}  // namespace ccv

extern "C" {

size_t ccv_fprop_planar_workspace_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  const size_t split = split_workspace_bytes(pb, precision, false);
  const size_t req = planar_required_bytes(pb, precision);
  return split > 0 ? align256(req) + 256 + split : req;
}

size_t ccv_fprop_complex_workspace_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  const size_t split = split_workspace_bytes(pb, precision, true);
  const size_t req = complex_required_bytes(pb, precision);
  return split > 0 ? align256(req) + 256 + split : req;
}

size_t ccv_fprop_planar_min_workspace_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  return planar_required_bytes(pb, precision);
}

size_t ccv_fprop_complex_min_workspace_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  return complex_required_bytes(pb, precision);
}

int ccv_fprop_planar(const float* x_real, const float* x_imag, const void* w_packed,
                     float* y_real, float* y_imag, const ccv_conv_shape* shape, int precision,
                     void* workspace, size_t workspace_bytes, ccv_stream_t stream) {
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  return fprop_planar_impl(x_real, x_imag, w_packed, nullptr, nullptr, y_real, y_imag, shape,
                           precision, workspace, workspace_bytes, stream);
}

int ccv_fprop_planar_bias(const float* x_real, const float* x_imag, const void* w_packed,
                          const float* bias_real, const float* bias_imag, float* y_real,
                          float* y_imag, const ccv_conv_shape* shape, int precision,
                          void* workspace, size_t workspace_bytes, ccv_stream_t stream) {
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  return fprop_planar_impl(x_real, x_imag, w_packed, bias_real, bias_imag, y_real, y_imag, shape,
                           precision, workspace, workspace_bytes, stream);
}

int ccv_fprop_complex(const void* x, const void* w_packed, void* y, const ccv_conv_shape* shape,
                      int precision, void* workspace, size_t workspace_bytes,
                      ccv_stream_t stream) {
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  return fprop_complex_impl(x, nullptr, w_packed, nullptr, nullptr, y, shape, precision,
                            workspace, workspace_bytes, stream);
}

int ccv_fprop_complex_bias(const void* x, const void* w_packed, const float* bias_real,
                           const float* bias_imag, void* y, const ccv_conv_shape* shape,
                           int precision, void* workspace, size_t workspace_bytes,
                           ccv_stream_t stream) {
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  return fprop_complex_impl(x, nullptr, w_packed, bias_real, bias_imag, y, shape, precision,
                            workspace, workspace_bytes, stream);
}

int ccv_fprop_complex_strided(const void* x, const int64_t* x_strides, const void* w_packed,
                              const float* bias_real, const float* bias_imag, void* y,
                              const ccv_conv_shape* shape, int precision, void* workspace,
                              size_t workspace_bytes, ccv_stream_t stream) {
  if (x_strides == nullptr) return set_error(CCV_ERR_INVALID_ARGUMENT, "null strides");
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  return fprop_complex_impl(x, x_strides, w_packed, bias_real, bias_imag, y, shape, precision,
                            workspace, workspace_bytes, stream);
}

int ccv_fprop_planar_to_complex(const float* x_real, const float* x_imag, const void* w_packed,
                                void* y, const ccv_conv_shape* shape, int precision,
                                void* workspace, size_t workspace_bytes, ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if ((rc = check_precision(precision)) != CCV_OK) return rc;
  if (!x_real || !x_imag || !w_packed || !y) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  }
  if (!aligned16(x_real) || !aligned16(x_imag) || !aligned16(w_packed) || !aligned16(y)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  const size_t need = planar_required_bytes(pb, precision);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ensure_status_mirror(st);
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  CounterScope scope(st);
  void* sk = nullptr;
  size_t sk_bytes = 0;
  split_scratch(workspace, workspace_bytes, need, &sk, &sk_bytes);
  const float* xr = x_real;
  const float* xi = x_imag;
  const float* lr = nullptr;
  const float* li = nullptr;
  if (precision == CCV_PRECISION_3XTF32) {
    const size_t pl = plane_bytes_aligned(pb);
    char* ws = static_cast<char*>(workspace);
    float* hr = reinterpret_cast<float*>(ws);
    float* hi = reinterpret_cast<float*>(ws + pl);
    float* wlr = reinterpret_cast<float*>(ws + 2 * pl);
    float* wli = reinterpret_cast<float*>(ws + 3 * pl);
    rc = launch_split_planes(x_real, x_imag, hr, hi, wlr, wli,
                             static_cast<size_t>(pb.n) * pb.h * pb.w * pb.c, st);
    if (rc != CCV_OK) return rc;
    xr = hr;
    xi = hi;
    lr = wlr;
    li = wli;
  }
  return launch_fprop(xr, xi, lr, li, static_cast<const float*>(w_packed), static_cast<float*>(y),
                      nullptr, pb, precision, OUT_COMPLEX_NCHW, Epilogue(), sk, sk_bytes, st);
}

int ccv_fprop_kernel_launches(const ccv_conv_shape* shape, int precision, int complex_input,
                              int* kernels) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (kernels == nullptr) return set_error(CCV_ERR_INVALID_ARGUMENT, "null output pointer");
  const bool split = precision == CCV_PRECISION_3XTF32;
  if (complex_input) {
    const char* name = complex_kernel_name(pb, precision);
    *kernels = strncmp(name, "layout_pass", 11) == 0 ? 2 : 1;
  } else {
    *kernels = split && !use_layout_warps_planar(pb, precision) ? 2 : 1;
  }
  return CCV_OK;
}

const char* ccv_fprop_complex_kernel(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return "invalid";
  if (precision != CCV_PRECISION_TF32 && precision != CCV_PRECISION_3XTF32) return "invalid";
  return complex_kernel_name(pb, precision);
}

size_t ccv_forward_workspace_bytes(const ccv_conv_shape* shape) {
  const size_t b = align256(ccv_packed_weight_bytes(shape, CCV_PRECISION_TF32));
  if (b == 0) return 0;
  return b + ccv_fprop_planar_workspace_bytes(shape, CCV_PRECISION_TF32);
}

int ccv_forward(const float* x_real, const float* x_imag, const float* w_real_krsc,
                const float* w_imag_krsc, float* y_real, float* y_imag,
                const ccv_conv_shape* shape, void* workspace, size_t workspace_bytes,
                ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  const size_t packed = align256(ccv_packed_weight_bytes(shape, CCV_PRECISION_TF32));
  if (workspace == nullptr || workspace_bytes < packed) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing or too small");
  }
  rc = ccv_prepack_weights(w_real_krsc, w_imag_krsc, CCV_WEIGHT_KRSC, shape, CCV_PRECISION_TF32,
                           workspace, packed, stream);
  if (rc != CCV_OK) return rc;
  // Past the packed weights: optional scratch for the fprop kernels.
  void* rest = workspace_bytes > packed ? static_cast<char*>(workspace) + packed : nullptr;
  return ccv_fprop_planar(x_real, x_imag, workspace, y_real, y_imag, shape, CCV_PRECISION_TF32,
                          rest, rest ? workspace_bytes - packed : 0, stream);
}

int ccv_get_device_status(int* status) {
  if (status == nullptr) return set_error(CCV_ERR_INVALID_ARGUMENT, "status is null");
  int v = 0;
  const cudaError_t e = cudaMemcpyFromSymbol(&v, g_ccv_status, sizeof(int));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyFromSymbol(status)");
  *status = v;
  return CCV_OK;
}

int ccv_clear_device_status(void) {
  const int zero = 0;
  cudaError_t e = cudaMemcpyToSymbol(g_ccv_status, &zero, sizeof(int));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyToSymbol(status)");
  // A kernel that gave up may have left counters counted.
  static const std::vector<unsigned> zeros(static_cast<size_t>(kCounterSets) * kSkCounterWords,
                                           0u);
  e = cudaMemcpyToSymbol(g_ccv_sk_counters, zeros.data(), zeros.size() * sizeof(unsigned));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyToSymbol(counter sets)");
  int dev = 0;
  if (current_device(&dev) == CCV_OK && g_status_host[dev] != nullptr) *g_status_host[dev] = 0;
  return CCV_OK;
}

int ccv_selftest_bounded_wait(int* status_dev, ccv_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ensure_status_mirror(st);
  const int rc = check_device();
  if (rc != CCV_OK) return rc;
  if (status_dev == nullptr) {
    int* lib = device_status_ptr();
    if (lib == nullptr) return CCV_ERR_CUDA;
    return launch_selftest_wait(lib, true, st);
  }
  return launch_selftest_wait(status_dev, false, st);
}

int ccv_reload_config(void) {
  reload_knobs();
  return CCV_OK;
}

}  // extern "C"

// ------------------------------------------------------------------ backward
namespace ccv {
namespace {

// Phase (a, b) of the data gradient as a forward problem: dy with the
// phase's zero border (y.out + y.taps - 1 rows), the phase's sub-filter
// (y.taps x x.taps taps), stride 1, no padding; its output is the phase's
// y.out x x.out positions of dx.
struct DgradPhase {
  DgradAxis y, x;
  ccv_conv_shape shape;
  bool live = false;         // some filter tap reaches this phase
  size_t filter_floats = 0;  // floats of its packed image(s)
};

DgradPhase dgrad_phase(const Problem& pb, int a, int b, int precision) {
  DgradPhase ph;
  ph.y = dgrad_axis(a, pb.sh, pb.ph, pb.r, pb.h);
  ph.x = dgrad_axis(b, pb.sw, pb.pw, pb.s, pb.w);
  ph.filter_floats = static_cast<size_t>(ph.y.taps) * ph.x.taps * 3 * pb.k * pb.c *
                     (precision == CCV_PRECISION_3XTF32 ? 2 : 1);
  ph.live = ph.y.taps > 0 && ph.x.taps > 0 && ph.y.out > 0 && ph.x.out > 0;
  ccv_conv_shape d;
  d.n = pb.n;
  d.h = ph.y.out + ph.y.taps - 1;
  d.w = ph.x.out + ph.x.taps - 1;
  d.c = pb.k;
  d.k = pb.c;
  d.r = ph.y.taps;
  d.s = ph.x.taps;
  d.stride_h = 1;
  d.stride_w = 1;
  d.pad_h = 0;
  d.pad_w = 0;
  ph.shape = d;
  return ph;
}

// Stride 1 with padding <= kernel size - 1: one phase whose zero border is
// the forward's own padding, so dy is convolved in place (no copy).
bool dgrad_direct(const Problem& pb) {
  return pb.sh == 1 && pb.sw == 1 && pb.ph <= pb.r - 1 && pb.pw <= pb.s - 1;
}

ccv_conv_shape dgrad_direct_shape(const Problem& pb) {
  ccv_conv_shape d;
  d.n = pb.n;
  d.h = pb.p;
  d.w = pb.q;
  d.c = pb.k;
  d.k = pb.c;
  d.r = pb.r;
  d.s = pb.s;
  d.stride_h = 1;
  d.stride_w = 1;
  d.pad_h = pb.r - 1 - pb.ph;
  d.pad_w = pb.s - 1 - pb.pw;
  return d;
}

// Scratch of the phase path: every phase's output (dx-sized in total), the
// largest phase copy of dy and the largest forward workspace of a phase.
struct DgradScratch {
  size_t outputs = 0, pad = 0, fprop = 0;
  size_t total() const { return outputs + pad + fprop; }
};

// planar: the phase copies are two fp32 planes (each half of `pad`, 256-byte
// aligned) and the forward workspace is the planar one.
int dgrad_scratch(const Problem& pb, int precision, DgradScratch* out, bool planar = false) {
  DgradScratch sc;
  sc.outputs = align256(static_cast<size_t>(pb.n) * pb.c * pb.h * pb.w * 8);
  for (int a = 0; a < pb.sh; ++a) {
    for (int b = 0; b < pb.sw; ++b) {
      const DgradPhase ph = dgrad_phase(pb, a, b, precision);
      if (!ph.live) continue;
      Problem pp;
      const int rc = make_problem(&ph.shape, &pp);
      if (rc != CCV_OK) return rc;
      sc.pad = std::max(sc.pad, 2 * align256(static_cast<size_t>(pb.n) * pb.k * ph.shape.h *
                                             ph.shape.w * 4));
      sc.fprop = std::max(sc.fprop, planar ? ccv_fprop_planar_workspace_bytes(&ph.shape, precision)
                                           : ccv_fprop_complex_workspace_bytes(&ph.shape, precision));
    }
  }
  *out = sc;
  return CCV_OK;
}

}  // namespace
}  // namespace ccv

extern "C" {

int ccv_prepack_weights_dgrad(const float* w_real, const float* w_imag, int layout,
                              const ccv_conv_shape* shape, int precision, void* packed,
                              size_t packed_bytes, ccv_stream_t stream) {
  ensure_status_mirror(reinterpret_cast<cudaStream_t>(stream));
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (layout != CCV_WEIGHT_KCRS && layout != CCV_WEIGHT_KRSC) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown weight layout");
  }
  if ((rc = check_precision(precision)) != CCV_OK) return rc;
  if (w_real == nullptr || w_imag == nullptr || packed == nullptr) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null weight pointer");
  }
  if (!aligned16(packed)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "packed weights must be 16-byte aligned");
  }
  if (packed_bytes < ccv_packed_weight_bytes(shape, precision)) {
    return set_error(CCV_ERR_WORKSPACE, "packed weight buffer too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  return launch_prepack_dgrad(w_real, w_imag, layout, pb, precision, static_cast<float*>(packed),
                              reinterpret_cast<cudaStream_t>(stream));
}

size_t ccv_dgrad_complex_workspace_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  if (dgrad_direct(pb)) {
    const ccv_conv_shape d = dgrad_direct_shape(pb);
    return ccv_fprop_complex_workspace_bytes(&d, precision);
  }
  DgradScratch sc;
  if (dgrad_scratch(pb, precision, &sc) != CCV_OK) return 0;
  return sc.total();
}

int ccv_dgrad_complex(const void* dy, const void* w_packed_dgrad, void* dx,
                      const ccv_conv_shape* shape, int precision, void* workspace,
                      size_t workspace_bytes, ccv_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ensure_status_mirror(st);
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if ((rc = check_precision(precision)) != CCV_OK) return rc;
  if (!dy || !w_packed_dgrad || !dx) return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned16(dy) || !aligned16(w_packed_dgrad) || !aligned16(dx)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  if (workspace == nullptr || !aligned16(workspace)) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing or misaligned");
  }
  if (dgrad_direct(pb)) {
    const ccv_conv_shape d = dgrad_direct_shape(pb);
    return fprop_complex_impl(dy, nullptr, w_packed_dgrad, nullptr, nullptr, dx, &d, precision,
                              workspace, workspace_bytes, stream);
  }
  DgradScratch sc;
  if ((rc = dgrad_scratch(pb, precision, &sc)) != CCV_OK) return rc;
  if (workspace_bytes < sc.total()) {
    return set_error(CCV_ERR_WORKSPACE, "workspace too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  char* ws = static_cast<char*>(workspace);
  char* outputs = ws;
  char* padded = ws + sc.outputs;
  char* fws = padded + sc.pad;
  const float* filt = static_cast<const float*>(w_packed_dgrad);
  size_t out_off = 0;  // bytes into `outputs`
  for (int a = 0; a < pb.sh; ++a) {
    for (int b = 0; b < pb.sw; ++b) {
      const DgradPhase ph = dgrad_phase(pb, a, b, precision);
      if (ph.live) {
        if ((rc = launch_dgrad_phase_pad(dy, padded, pb, static_cast<int>(ph.shape.h),
                                         static_cast<int>(ph.shape.w), ph.y.offset,
                                         ph.x.offset, st)) != CCV_OK) {
          return rc;
        }
        rc = fprop_complex_impl(padded, nullptr, filt, nullptr, nullptr, outputs + out_off,
                                &ph.shape, precision, fws, sc.fprop, stream);
        if (rc != CCV_OK) return rc;
      }
      filt += ph.filter_floats;
      out_off += static_cast<size_t>(pb.n) * pb.c * ph.y.out * ph.x.out * 8;
    }
  }
  return launch_dgrad_interleave(outputs, dx, pb, st);
}

size_t ccv_wgrad_complex_workspace_bytes(const ccv_conv_shape* shape) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  return wgrad_workspace_bytes(pb);
}

int ccv_wgrad_complex(const void* x, const void* dy, float* dw_real, float* dw_imag,
                      const ccv_conv_shape* shape, void* workspace, size_t workspace_bytes,
                      ccv_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ensure_status_mirror(st);
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (!x || !dy || !dw_real || !dw_imag) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  }
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dw_real) || !aligned16(dw_imag)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < wgrad_workspace_bytes(pb)) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  WgradSource src;
  src.x = x;
  src.dy = dy;
  return launch_wgrad(src, dw_real, dw_imag, pb, workspace, st);
}

size_t ccv_wgrad_planar_workspace_bytes(const ccv_conv_shape* shape) {
  return ccv_wgrad_complex_workspace_bytes(shape);
}

int ccv_wgrad_planar(const float* x_real, const float* x_imag, const float* dy_real,
                     const float* dy_imag, float* dw_real, float* dw_imag,
                     const ccv_conv_shape* shape, void* workspace, size_t workspace_bytes,
                     ccv_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ensure_status_mirror(st);
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (!x_real || !x_imag || !dy_real || !dy_imag || !dw_real || !dw_imag) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  }
  if (!aligned16(x_real) || !aligned16(x_imag) || !aligned16(dy_real) || !aligned16(dy_imag) ||
      !aligned16(dw_real) || !aligned16(dw_imag)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  if (workspace == nullptr || !aligned16(workspace) ||
      workspace_bytes < wgrad_workspace_bytes(pb)) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  WgradSource src;
  src.x_real = x_real;
  src.x_imag = x_imag;
  src.dy_real = dy_real;
  src.dy_imag = dy_imag;
  return launch_wgrad(src, dw_real, dw_imag, pb, workspace, st);
}

size_t ccv_dgrad_planar_workspace_bytes(const ccv_conv_shape* shape, int precision) {
  Problem pb;
  if (make_problem(shape, &pb) != CCV_OK) return 0;
  if (dgrad_direct(pb)) {
    const ccv_conv_shape d = dgrad_direct_shape(pb);
    return ccv_fprop_planar_workspace_bytes(&d, precision);
  }
  DgradScratch sc;
  if (dgrad_scratch(pb, precision, &sc, true) != CCV_OK) return 0;
  return sc.total();
}

int ccv_dgrad_planar(const float* dy_real, const float* dy_imag, const void* w_packed_dgrad,
                     float* dx_real, float* dx_imag, const ccv_conv_shape* shape, int precision,
                     void* workspace, size_t workspace_bytes, ccv_stream_t stream) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  ensure_status_mirror(st);
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if ((rc = check_precision(precision)) != CCV_OK) return rc;
  if (!dy_real || !dy_imag || !w_packed_dgrad || !dx_real || !dx_imag) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  }
  if (!aligned16(dy_real) || !aligned16(dy_imag) || !aligned16(w_packed_dgrad) ||
      !aligned16(dx_real) || !aligned16(dx_imag)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  if (dgrad_direct(pb)) {
    const ccv_conv_shape d = dgrad_direct_shape(pb);
    return fprop_planar_impl(dy_real, dy_imag, w_packed_dgrad, nullptr, nullptr, dx_real, dx_imag,
                             &d, precision, workspace, workspace_bytes, stream);
  }
  if (workspace == nullptr || !aligned16(workspace)) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing or misaligned");
  }
  DgradScratch sc;
  if ((rc = dgrad_scratch(pb, precision, &sc, true)) != CCV_OK) return rc;
  if (workspace_bytes < sc.total()) return set_error(CCV_ERR_WORKSPACE, "workspace too small");
  if ((rc = check_device()) != CCV_OK) return rc;
  if ((rc = check_status_clear()) != CCV_OK) return rc;
  char* ws = static_cast<char*>(workspace);
  float* outputs = reinterpret_cast<float*>(ws);
  float* pad_r = reinterpret_cast<float*>(ws + sc.outputs);
  float* pad_i = reinterpret_cast<float*>(ws + sc.outputs + sc.pad / 2);
  char* fws = ws + sc.outputs + sc.pad;
  const float* filt = static_cast<const float*>(w_packed_dgrad);
  size_t out_off = 0;  // floats into `outputs`
  for (int a = 0; a < pb.sh; ++a) {
    for (int b = 0; b < pb.sw; ++b) {
      const DgradPhase ph = dgrad_phase(pb, a, b, precision);
      const size_t plane = static_cast<size_t>(pb.n) * ph.y.out * ph.x.out * pb.c;
      if (ph.live) {
        if ((rc = launch_dgrad_phase_pad_planar(dy_real, dy_imag, pad_r, pad_i, pb,
                                                static_cast<int>(ph.shape.h),
                                                static_cast<int>(ph.shape.w), ph.y.offset,
                                                ph.x.offset, st)) != CCV_OK) {
          return rc;
        }
        rc = fprop_planar_impl(pad_r, pad_i, filt, nullptr, nullptr, outputs + out_off,
                               outputs + out_off + plane, &ph.shape, precision, fws, sc.fprop,
                               stream);
        if (rc != CCV_OK) return rc;
      }
      filt += ph.filter_floats;
      out_off += 2 * plane;
    }
  }
  return launch_dgrad_interleave_planar(outputs, dx_real, dx_imag, pb, st);
}

}  // extern "C"
