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

// Per-device status word.  Bounded in-kernel waits that run out write a
// CCV_ERR_* code here; fprop kernels read it at start and exit without work
// while it is set.
__device__ int g_ccv_status = 0;
// Stream-K counter sets (see stream_k_counters); zero-initialized.
constexpr int kSkRing = 32;
__device__ unsigned g_ccv_sk_counters[kSkRing * kSkCounterWords];

namespace {

thread_local std::string g_last_error;

constexpr int kMaxDevices = 64;
std::mutex g_dev_mutex;
int* g_status_ptr[kMaxDevices] = {};
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
std::atomic<unsigned> g_sk_epoch[kMaxDevices];
unsigned* g_sk_base[kMaxDevices] = {};
}  // namespace

unsigned* stream_k_counters() {
  int dev = 0;
  if (current_device(&dev) != CCV_OK) return nullptr;
  {
    std::lock_guard<std::mutex> lk(g_dev_mutex);
    if (g_sk_base[dev] == nullptr) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_ccv_sk_counters);
      if (e != cudaSuccess) {
        cuda_error(e, "cudaGetSymbolAddress(stream-K counters)");
        return nullptr;
      }
      g_sk_base[dev] = static_cast<unsigned*>(p);
    }
  }
  const unsigned slot = g_sk_epoch[dev].fetch_add(1u) % kSkRing;
  return g_sk_base[dev] + static_cast<size_t>(slot) * kSkCounterWords;
}

bool pdl_enabled() {
  static const bool on = [] {
    const char* env = getenv("CCV_PDL");
    return env == nullptr || atoi(env) != 0;
  }();
  return on;
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
  const CUtensorMapSwizzle sw = swizzle == kSwizzle128        ? CU_TENSOR_MAP_SWIZZLE_128B
                                : swizzle == kSwizzle128Atom32 ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B
                                : swizzle == kSwizzleNone      ? CU_TENSOR_MAP_SWIZZLE_NONE
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

// Workspace a complex call cannot run without: none for the fused kernel
// (it reads complex64 directly); otherwise fp32 NHWC planes of the input
// (real, imaginary; 3xTF32: also remainders).
size_t complex_required_bytes(const Problem& pb, int precision) {
  if (fused_complex_available(pb, precision)) return 0;
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

}  // namespace

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
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (precision != CCV_PRECISION_TF32 && precision != CCV_PRECISION_3XTF32) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown precision");
  }
  if (!x_real || !x_imag || !w_packed || !y_real || !y_imag) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  }
  if (!aligned16(x_real) || !aligned16(x_imag) || !aligned16(w_packed) || !aligned16(y_real) ||
      !aligned16(y_imag)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  const size_t need = planar_required_bytes(pb, precision);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* sk = nullptr;
  size_t sk_bytes = 0;
  split_scratch(workspace, workspace_bytes, need, &sk, &sk_bytes);
  if (precision == CCV_PRECISION_3XTF32) {
    const size_t pl = plane_bytes_aligned(pb);
    char* ws = static_cast<char*>(workspace);
    float* hr = reinterpret_cast<float*>(ws);
    float* hi = reinterpret_cast<float*>(ws + pl);
    float* lr = reinterpret_cast<float*>(ws + 2 * pl);
    float* li = reinterpret_cast<float*>(ws + 3 * pl);
    if (use_layout_warps_planar(pb, precision)) {
      return launch_fprop_planar_lw(x_real, x_imag, hr, hi, lr, li,
                                    static_cast<const float*>(w_packed), y_real, y_imag, pb, sk,
                                    sk_bytes, st);
    }
    rc = launch_split_planes(x_real, x_imag, hr, hi, lr, li,
                             static_cast<size_t>(pb.n) * pb.h * pb.w * pb.c, st);
    if (rc != CCV_OK) return rc;
    return launch_fprop(hr, hi, lr, li, static_cast<const float*>(w_packed), y_real, y_imag, pb,
                        precision, OUT_PLANAR_NHWC, sk, sk_bytes, st);
  }
  return launch_fprop(x_real, x_imag, nullptr, nullptr, static_cast<const float*>(w_packed),
                      y_real, y_imag, pb, precision, OUT_PLANAR_NHWC, sk, sk_bytes, st);
}

int ccv_fprop_planar_to_complex(const float* x_real, const float* x_imag, const void* w_packed,
                                void* y, const ccv_conv_shape* shape, int precision,
                                void* workspace, size_t workspace_bytes, ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (precision != CCV_PRECISION_TF32 && precision != CCV_PRECISION_3XTF32) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown precision");
  }
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
  if ((rc = check_device()) != CCV_OK) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
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
                      nullptr, pb, precision, OUT_COMPLEX_NCHW, sk, sk_bytes, st);
}

int ccv_fprop_complex(const void* x, const void* w_packed, void* y, const ccv_conv_shape* shape,
                      int precision, void* workspace, size_t workspace_bytes,
                      ccv_stream_t stream) {
  Problem pb;
  int rc = make_problem(shape, &pb);
  if (rc != CCV_OK) return rc;
  if (precision != CCV_PRECISION_TF32 && precision != CCV_PRECISION_3XTF32) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "unknown precision");
  }
  if (!x || !w_packed || !y) return set_error(CCV_ERR_INVALID_ARGUMENT, "null tensor pointer");
  if (!aligned16(x) || !aligned16(w_packed) || !aligned16(y)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "tensor pointers must be 16-byte aligned");
  }
  const size_t need = complex_required_bytes(pb, precision);
  if (need > 0 && (workspace == nullptr || workspace_bytes < need || !aligned16(workspace))) {
    return set_error(CCV_ERR_WORKSPACE, "workspace missing, misaligned or too small");
  }
  if ((rc = check_device()) != CCV_OK) return rc;
  void* sk = nullptr;
  size_t sk_bytes = 0;
  split_scratch(workspace, workspace_bytes, need, &sk, &sk_bytes);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (need == 0) {
    return launch_fprop_fused_complex(static_cast<const float*>(x),
                                      static_cast<const float*>(w_packed), static_cast<float*>(y),
                                      pb, precision, sk, sk_bytes, st);
  }
  const size_t pl = plane_bytes_aligned(pb);
  char* ws = static_cast<char*>(workspace);
  float* xr = reinterpret_cast<float*>(ws);
  float* xi = reinterpret_cast<float*>(ws + pl);
  if (use_in_kernel_conversion(pb, precision)) {
    return launch_fprop_complex_cvt(static_cast<const float*>(x), xr, xi,
                                    static_cast<const float*>(w_packed), static_cast<float*>(y),
                                    pb, st);
  }
  const bool split = precision == CCV_PRECISION_3XTF32;
  float* lr = split ? reinterpret_cast<float*>(ws + 2 * pl) : nullptr;
  float* li = split ? reinterpret_cast<float*>(ws + 3 * pl) : nullptr;
  if (use_layout_warps(pb, precision)) {
    return launch_fprop_complex_lw(static_cast<const float*>(x), xr, xi, lr, li,
                                   static_cast<const float*>(w_packed), static_cast<float*>(y), pb,
                                   precision, sk, sk_bytes, st);
  }
  rc = launch_nchw_complex_to_planar(static_cast<const float*>(x), xr, xi, lr, li, pb, st);
  if (rc != CCV_OK) return rc;
  return launch_fprop(xr, xi, lr, li, static_cast<const float*>(w_packed), static_cast<float*>(y),
                      nullptr, pb, precision, OUT_COMPLEX_NCHW, sk, sk_bytes, st);
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
  // A kernel that gave up may have left stream-K counters counted.
  static const std::vector<unsigned> zeros(static_cast<size_t>(kSkRing) * kSkCounterWords, 0u);
  e = cudaMemcpyToSymbol(g_ccv_sk_counters, zeros.data(), zeros.size() * sizeof(unsigned));
  if (e != cudaSuccess) return cuda_error(e, "cudaMemcpyToSymbol(stream-K counters)");
  return CCV_OK;
}

int ccv_selftest_bounded_wait(int* status_dev, ccv_stream_t stream) {
  if (status_dev == nullptr) return set_error(CCV_ERR_INVALID_ARGUMENT, "status is null");
  const int rc = check_device();
  if (rc != CCV_OK) return rc;
  return launch_selftest_wait(status_dev, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
