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

// Testing/benchmarking switches read from CCV_* environment variables: read
// once, on first use (ccv_reload_config re-reads them).  Each field's
// default is the tuned behaviour.
struct Knobs {
  int pdl = 1;            // CCV_PDL: programmatic dependent launch
  int kt = 0;             // CCV_KT=32|64|128: single-CTA channel tile (0 auto)
  int force_kernel = 0;   // CCV_FORCE_KERNEL=1|2: single-CTA / pair family (0 auto)
  int halo = -1;          // CCV_HALO=0|1: pair variant (-1 auto)
  int splitk = 0;         // CCV_SPLITK=n: cap of the single-CTA split (0 none)
  int lw = -1;            // CCV_LW=0|1: layout warps off / wherever possible (-1 auto)
  int lw_prefix = -1;     // CCV_LW_PREFIX=0: no prefix phase
  int lw_tma = 1;         // CCV_LW_TMA=0: warp prefix instead of the TMA prefix
  int lw_tma_images = 0;  // CCV_LW_TMA_IMAGES=n: images of the TMA prefix (0 auto)
  int lw_tma_bufs = 0;    // CCV_LW_TMA_BUFS=2..4: TMA prefix boxes in flight (0 default)
  int subbox = 1;         // CCV_SUBBOX=0: no two-sub-box halo tiles
  int streamk = -1;       // CCV_STREAMK=0|1: never / whenever possible (-1 model)
  int max_clusters = 0;   // CCV_MAX_CLUSTERS=n: persistent grid cap (0 none)
  int tma_store = 1;      // CCV_TMA_STORE=0: planar epilogue without TMA stores
};
const Knobs& knobs();
void reload_knobs();

// Epilogue options of an fprop launch: complex bias per output channel
// (K fp32 real parts and K imaginary parts), or none.
struct Epilogue {
  const float* bias_r = nullptr;
  const float* bias_i = nullptr;
};

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
// Same from complex64 input with element strides (n, c, h, w): any layout,
// including slices and channels-last; the dense NCHW case takes the kernel
// above.  x must be 8-byte aligned.
int launch_strided_complex_to_planar(const float* x, const int64_t* strides, float* xr,
                                     float* xi, float* xr_lo, float* xi_lo, const Problem& pb,
                                     cudaStream_t stream);
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
                 OutLayout out_layout, const Epilogue& ep, void* ws, size_t ws_bytes,
                 cudaStream_t stream);

// Scratch bytes the stream-K split of this problem's kernel can use (0 when
// the problem runs on a kernel without the split).
size_t split_workspace_bytes(const Problem& pb, int precision, bool complex_input);

// forward() with the layout conversion done by layout warps inside the
// pair kernel (one launch; xr/xi and, for 3xTF32, xr_lo/xi_lo: workspace
// planes it fills).  The default complex path where it applies.
bool use_layout_warps(const Problem& pb, int precision);
int launch_fprop_complex_lw(const float* x, float* xr, float* xi, float* xr_lo, float* xi_lo,
                            const float* w_packed, float* y, const Problem& pb, int precision,
                            const Epilogue& ep, void* ws, size_t ws_bytes, cudaStream_t stream);
// Whether the layout-warp variant pays for this problem (dispatch rule,
// complex or planar source).
bool layout_warps_pay(const Problem& pb, int precision);
// 3xTF32 forward_planar() with the TF32 split of the input planes done by
// layout warps inside the pair kernel (one launch; hr/hi/lr/li: workspace
// planes it fills from x_real/x_imag).
bool use_layout_warps_planar(const Problem& pb, int precision);
int launch_fprop_planar_lw(const float* x_real, const float* x_imag, float* hr, float* hi,
                           float* lr, float* li, const float* w_packed, float* y_real,
                           float* y_imag, const Problem& pb, const Epilogue& ep, void* ws,
                           size_t ws_bytes, cudaStream_t stream);
// Name of the kernel path a complex (forward()) call takes.
const char* complex_kernel_name(const Problem& pb, int precision);

// Kernels of ccv_backward.cu.
// One axis of one phase of the data gradient: output positions
// a, a + stride, ... (`out` of them) meet filter taps first, first + stride,
// ... (`taps` of them, 0: none), and the phase's convolution reads dy with
// its index shifted by `offset` (a copy of dy whose element i is dy[i - offset]).
struct DgradAxis {
  int first = 0, taps = 0, offset = 0, out = 0;
};
DgradAxis dgrad_axis(int a, int stride, int pad, int taps, int in_size);
// Packed images of the data-gradient filter (transposed K <-> C, flipped,
// conjugated), one per phase of the stride grid in (a, b) order (one for
// stride 1), for the forward kernels, from the forward's KCRS/KRSC planes.
// Their total size is the forward image's.
int launch_prepack_dgrad(const float* w_real, const float* w_imag, int layout, const Problem& pb,
                         int precision, float* packed, cudaStream_t stream);
// dy (complex64 [N][K][P][Q]) with a phase's zero border: [N][K][hp][wp],
// element (i, j) = dy[i - oh][j - ow].
int launch_dgrad_phase_pad(const void* dy, void* out, const Problem& pb, int hp, int wp, int oh,
                           int ow, cudaStream_t stream);
// dx from the phases' outputs ([N][C][Ha][Wb] blocks in (a, b) order).
int launch_dgrad_interleave(const void* phases, void* dx, const Problem& pb, cudaStream_t stream);
// Weight gradient: scratch bytes, and the launch (layout kernels, the
// tcgen05 kernel and, when the reduction is split, the split-order sum).
size_t wgrad_workspace_bytes(const Problem& pb);
// Inputs of the weight gradient: complex64 x (NCHW) and dy (NKPQ), or fp32
// planes x_real/x_imag (NHWC) and dy_real/dy_imag (NPQK).
struct WgradSource {
  const void* x = nullptr;
  const void* dy = nullptr;
  const float* x_real = nullptr;
  const float* x_imag = nullptr;
  const float* dy_real = nullptr;
  const float* dy_imag = nullptr;
};
int launch_wgrad(const WgradSource& src, float* dw_r, float* dw_i, const Problem& pb, void* ws,
                 cudaStream_t stream);
// Planar data gradient pieces: dy planes with a phase's zero border, and dx
// planes from the phases' planar outputs (real block, then imaginary block,
// per phase in (a, b) order).
int launch_dgrad_phase_pad_planar(const float* dy_r, const float* dy_i, float* out_r,
                                  float* out_i, const Problem& pb, int hp, int wp, int oh, int ow,
                                  cudaStream_t stream);
int launch_dgrad_interleave_planar(const float* phases, float* dx_r, float* dx_i, const Problem& pb,
                                   cudaStream_t stream);

// Encodes a tiled tensor map through the driver entry point.
// `swizzle_bytes` is 64 or 128 (the box's inner extent in bytes).
int encode_tiled(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                 const uint64_t* strides_bytes, const uint32_t* box, const uint32_t* elem_strides,
                 int swizzle_bytes = 64);
// Same, with the swizzle mode named and optionally 8-byte elements.
enum TmaSwizzle { kSwizzle64 = 0, kSwizzle128 = 1, kSwizzleNone = 3 };
int encode_tiled_ex(CUtensorMap* map, const void* base, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box,
                    const uint32_t* elem_strides, TmaSwizzle swizzle, bool elem8);

// One CTA waits on an mbarrier nothing arrives on; the bounded wait writes
// CCV_ERR_DEVICE_TIMEOUT into *status_dev (and, with `mirror`, into the
// host-mapped mirror of the library's status block that status_dev points to).
int launch_selftest_wait(int* status_dev, bool mirror, cudaStream_t stream);

// Entry-point bodies without the one-time set-up of the host-mapped status
// mirror (a pinned host allocation): the public functions add that set-up;
// the no-allocation entry point calls these directly.
int prepack_weights_impl(const float* w_real, const float* w_imag, int layout,
                         const ccv_conv_shape* shape, int precision, void* packed,
                         size_t packed_bytes, ccv_stream_t stream);
int fprop_planar_impl(const float* x_real, const float* x_imag, const void* w_packed,
                      const float* bias_real, const float* bias_imag, float* y_real,
                      float* y_imag, const ccv_conv_shape* shape, int precision, void* workspace,
                      size_t workspace_bytes, ccv_stream_t stream);
// x_strides: element strides (n, c, h, w) of the complex64 input, or null
// for dense NCHW.
int fprop_complex_impl(const void* x, const int64_t* x_strides, const void* w_packed,
                       const float* bias_real, const float* bias_imag, void* y,
                       const ccv_conv_shape* shape, int precision, void* workspace,
                       size_t workspace_bytes, ccv_stream_t stream);

// Counter sets (stream-K tile counters, layout-warp tickets) for one launch:
// kSkCounterWords zeroed words in library-owned device memory.  A kernel
// leaves its set zero when it ends (each split tile's counter is reset by
// the piece that completes it; the last layout-warp CTA resets the rest), so
// no memset precedes a launch.  A set is handed to one launch at a time:
// sets taken by an entry point are marked in flight by a CUDA event
// recorded on the launch's stream when the entry point returns (see
// CounterScope), and a set is reused only once its event has completed.
// Sets taken during stream capture stay with the captured graph for good.
// When every set is in flight acquire_counter_set returns nullptr and the
// caller runs a path without counters (no split, layout pass).
// ccv_clear_device_status re-zeroes every set after an abort.
constexpr int kSkCounterWords = 1024;
constexpr int kCounterSets = 64;
unsigned* acquire_counter_set(cudaStream_t stream);
// Internal return code of the pair launchers: no counter set was free for
// the layout warps (nothing was launched; the caller takes another path).
constexpr int kNoCounterSet = -100;

// Marks the counter sets this host thread acquired since the scope began as
// in flight on `stream` when the scope ends (records their events).  Every
// C-ABI entry point that may launch with counters opens one.
class CounterScope {
 public:
  explicit CounterScope(cudaStream_t stream);
  ~CounterScope();
  CounterScope(const CounterScope&) = delete;
  CounterScope& operator=(const CounterScope&) = delete;

 private:
  cudaStream_t stream_;
};

// Programmatic dependent launch for the library's kernels (each calls
// griddepcontrol.wait before its first global-memory access, so its prologue
// may overlap the previous kernel's tail).  CCV_PDL=0 turns it off.
inline bool pdl_enabled() { return knobs().pdl != 0; }

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
