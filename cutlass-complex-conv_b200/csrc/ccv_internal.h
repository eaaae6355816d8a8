// Internal declarations shared by the translation units of libccv_b200.so.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>

#include "ccv_b200.h"

namespace ccv {

// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);

// Converts a CUDA runtime error into CCV_ERR_CUDA with context.
int cuda_error(cudaError_t e, const char* what);

// Device pointer of the per-device status word (the current device).
int* device_status_ptr();

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Validated problem with derived sizes.
struct Problem {
  int n, h, w, c, k, r, s, p, q;
  int sh, sw, ph, pw;
};

int make_problem(const ccv_conv_shape* shape, Problem* out);

// Packed weight image: per precision "image" of [R*S][3][K][C] floats.
inline size_t packed_image_floats(const Problem& pb) {
  return static_cast<size_t>(pb.r) * pb.s * 3ull * pb.k * pb.c;
}

// Kernels of ccv_layout.cu.
int launch_prepack(const float* w_real, const float* w_imag, int layout, const Problem& pb,
                   int precision, float* packed, cudaStream_t stream);
// complex64 NCHW -> fp32 NHWC planes.  With xr_lo/xi_lo non-null (3xTF32),
// xr/xi receive tf32(x) and xr_lo/xi_lo the remainders x - tf32(x).
int launch_nchw_complex_to_planar(const float* x, float* xr, float* xi, float* xr_lo,
                                  float* xi_lo, const Problem& pb, cudaStream_t stream);
// fp32 planes -> (tf32(x), x - tf32(x)) planes, for 3xTF32 on planar inputs.
int launch_split_planes(const float* xr, const float* xi, float* hr, float* hi, float* lr,
                        float* li, size_t count, cudaStream_t stream);

// Kernels of ccv_fprop.cu.
enum OutLayout { OUT_PLANAR_NHWC = 0, OUT_COMPLEX_NCHW = 1 };
// For 3xTF32, xr/xi are the TF32-rounded activation planes and xr_lo/xi_lo
// the remainders (x - tf32(x)); for TF32 the *_lo pointers are ignored.
// ws/ws_bytes: optional scratch (256-byte aligned) for the stream-K split of
// the pair kernels' last partial wave; null runs every tile whole.
int launch_fprop(const float* xr, const float* xi, const float* xr_lo, const float* xi_lo,
                 const float* w_packed, float* y0, float* y1, const Problem& pb, int precision,
                 OutLayout out_layout, void* ws, size_t ws_bytes, cudaStream_t stream);

// Scratch bytes the stream-K split of this problem's kernel can use (0 when
// the problem runs on a kernel without the split).
size_t split_workspace_bytes(const Problem& pb, int precision, bool complex_input);

// Fused complex path: complex64 NCHW in, complex64 NKPQ out, one launch, no
// required workspace.  Available when the problem runs on the halo pair kernel.
bool fused_complex_available(const Problem& pb, int precision);
// forward() with the layout conversion done by converter clusters inside
// the halo pair kernel (one launch; xr/xi: workspace planes it fills).
bool use_in_kernel_conversion(const Problem& pb, int precision);
int launch_fprop_complex_cvt(const float* x, float* xr, float* xi, const float* w_packed, float* y,
                             const Problem& pb, cudaStream_t stream);
// forward() with the layout conversion done by layout warps inside the halo
// pair kernel (one launch; xr/xi and, for 3xTF32, xr_lo/xi_lo: workspace
// planes it fills).  The default complex path where it applies.
bool use_layout_warps(const Problem& pb, int precision);
int launch_fprop_complex_lw(const float* x, float* xr, float* xi, float* xr_lo, float* xi_lo,
                            const float* w_packed, float* y, const Problem& pb, int precision,
                            void* ws, size_t ws_bytes, cudaStream_t stream);
// Whether the layout-warp variant pays for this problem (dispatch rule,
// complex or planar source).
bool layout_warps_pay(const Problem& pb, int precision);
// 3xTF32 forward_planar() with the TF32 split of the input planes done by
// layout warps inside the pair kernel (one launch; hr/hi/lr/li: workspace
// planes it fills from x_real/x_imag).
bool use_layout_warps_planar(const Problem& pb, int precision);
int launch_fprop_planar_lw(const float* x_real, const float* x_imag, float* hr, float* hi,
                           float* lr, float* li, const float* w_packed, float* y_real,
                           float* y_imag, const Problem& pb, void* ws, size_t ws_bytes,
                           cudaStream_t stream);
// Name of the kernel path a complex (forward()) call takes.
const char* complex_kernel_name(const Problem& pb, int precision);
int launch_fprop_fused_complex(const float* xc, const float* w_packed, float* y,
                               const Problem& pb, int precision, void* ws, size_t ws_bytes,
                               cudaStream_t stream);

// Encodes a tiled tensor map through the driver entry point.
// `swizzle_bytes` is 64 or 128 (the box's inner extent in bytes).
int encode_tiled(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, const uint32_t* elem_strides,
                 int swizzle_bytes = 64);
// Same, with the swizzle mode named and optionally 8-byte elements.
// kSwizzle128Atom32 swizzles 32-byte chunks within 128-byte rows (the
// shared-memory layout of MN-major 32-bit tensor-core operands).
enum TmaSwizzle { kSwizzle64 = 0, kSwizzle128 = 1, kSwizzle128Atom32 = 2, kSwizzleNone = 3 };
int encode_tiled_ex(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box,
                    const uint32_t* elem_strides, TmaSwizzle swizzle, bool elem8);

int launch_selftest_wait(int* status_dev, cudaStream_t stream);

// Stream-K tile counters for one launch: a zeroed set of kSkCounterWords
// words in library-owned device memory (a ring of sets, so launches in
// flight at the same time use different sets).  Each split tile's counter is
// reset by the piece that completes it, so a set is zero again when its
// kernel ends; ccv_clear_device_status re-zeroes the ring after an abort.
constexpr int kSkCounterWords = 1024;
unsigned* stream_k_counters();

// Programmatic dependent launch for the library's kernels (each calls
// griddepcontrol.wait before its first global-memory access, so its prologue
// may overlap the previous kernel's tail).  CCV_PDL=0 turns it off.
bool pdl_enabled();

// cudaLaunchKernelEx with PDL (when enabled) and, for cluster_x > 1, a
// runtime cluster size.
template <typename... KArgs, typename... Args>
cudaError_t launch_kernel(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                          cudaStream_t stream, int cluster_x, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  unsigned na = 0;
  if (cluster_x > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    ++na;
  }
  if (pdl_enabled()) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<Args&&>(args)...);
}

}  // namespace ccv
