// Python extension `complex_conv2d._C`.
//
// Keeps the reference's pybind surface (csrc/bindings.cpp:16-29 of the
// reference: `forward(x_real, x_imag, w_real, w_imag, stride_h, stride_w,
// pad_h, pad_w) -> [y_real, y_imag]`, with the argument checks and messages
// of csrc/complex_conv2d.cu:94-159) and adds the entry points the module
// uses with cached packed weights.  Every call goes through the C ABI of
// libccv_b200.so (include/ccv_b200.h); this file only validates torch
// tensors, allocates outputs/scratch from the caching allocator and picks
// the current stream.
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include <string>
#include <vector>

#include "ccv_b200.h"

namespace {

#define CHECK_CUDA(x) TORCH_CHECK(x.is_cuda(), #x " must be CUDA")
#define CHECK_FLOAT(x) TORCH_CHECK(x.scalar_type() == at::kFloat, #x " must be float32")
#define CHECK_CONTIGUOUS(x) TORCH_CHECK(x.is_contiguous(), #x " must be contiguous")

void check_rc(int rc, const char* what) {
  if (rc == CCV_OK) return;
  const char* msg = ccv_last_error_message();
  if (rc == CCV_ERR_UNSUPPORTED) {
    TORCH_CHECK(false, "complex_conv2d cannot implement this convolution configuration (", what,
                "): ", msg);
  }
  TORCH_CHECK(false, what, " failed (status ", rc, "): ", msg);
}

ccv_stream_t current_stream() {
  return reinterpret_cast<ccv_stream_t>(at::cuda::getCurrentCUDAStream().stream());
}

// Checks an optional complex bias (two K-element fp32 CUDA tensors) and
// returns its device pointers (null, null without bias).
std::pair<const float*, const float*> bias_ptrs(const c10::optional<torch::Tensor>& br,
                                               const c10::optional<torch::Tensor>& bi,
                                               int64_t K, const torch::Tensor& like) {
  const bool has_r = br.has_value() && br->defined();
  const bool has_i = bi.has_value() && bi->defined();
  TORCH_CHECK(has_r == has_i, "bias_real and bias_imag must both be given or both be None");
  if (!has_r) return {nullptr, nullptr};
  for (const auto* b : {&*br, &*bi}) {
    TORCH_CHECK(b->is_cuda() && b->scalar_type() == at::kFloat && b->is_contiguous(),
                "bias must be a contiguous CUDA float32 tensor");
    TORCH_CHECK(b->dim() == 1 && b->size(0) == K, "bias must have out_channels elements");
    TORCH_CHECK(b->device() == like.device(), "bias must be on the input's CUDA device");
  }
  return {br->data_ptr<float>(), bi->data_ptr<float>()};
}

ccv_conv_shape make_shape(int64_t n, int64_t h, int64_t w, int64_t c, int64_t k, int64_t r,
                          int64_t s, int64_t sh, int64_t sw, int64_t ph, int64_t pw) {
  ccv_conv_shape shp;
  shp.n = n; shp.h = h; shp.w = w; shp.c = c; shp.k = k; shp.r = r; shp.s = s;
  shp.stride_h = sh; shp.stride_w = sw; shp.pad_h = ph; shp.pad_w = pw;
  return shp;
}

// Reference-compatible entry: KRSC weights, fresh NHWC outputs.
std::vector<torch::Tensor> forward(torch::Tensor x_real, torch::Tensor x_imag,
                                   torch::Tensor w_real, torch::Tensor w_imag, int64_t stride_h,
                                   int64_t stride_w, int64_t pad_h, int64_t pad_w) {
  CHECK_CUDA(x_real); CHECK_CUDA(x_imag); CHECK_CUDA(w_real); CHECK_CUDA(w_imag);
  CHECK_FLOAT(x_real); CHECK_FLOAT(x_imag); CHECK_FLOAT(w_real); CHECK_FLOAT(w_imag);
  CHECK_CONTIGUOUS(x_real); CHECK_CONTIGUOUS(x_imag);
  CHECK_CONTIGUOUS(w_real); CHECK_CONTIGUOUS(w_imag);
  TORCH_CHECK(x_real.dim() == 4, "x_real must be a 4D NHWC tensor");
  TORCH_CHECK(x_imag.dim() == 4, "x_imag must be a 4D NHWC tensor");
  TORCH_CHECK(w_real.dim() == 4, "w_real must be a 4D KRSC tensor");
  TORCH_CHECK(w_imag.dim() == 4, "w_imag must be a 4D KRSC tensor");
  TORCH_CHECK(x_real.sizes() == x_imag.sizes(), "x_real and x_imag must have identical shapes");
  TORCH_CHECK(w_real.sizes() == w_imag.sizes(), "w_real and w_imag must have identical shapes");
  TORCH_CHECK(x_real.device() == x_imag.device() && x_real.device() == w_real.device() &&
                  x_real.device() == w_imag.device(),
              "all inputs and weights must be on the same CUDA device");
  TORCH_CHECK(stride_h > 0 && stride_w > 0, "stride must be positive");
  TORCH_CHECK(pad_h >= 0 && pad_w >= 0, "padding must be non-negative");
  c10::cuda::CUDAGuard guard(x_real.device());
  const int64_t N = x_real.size(0), H = x_real.size(1), W = x_real.size(2), C = x_real.size(3);
  const int64_t K = w_real.size(0), R = w_real.size(1), S = w_real.size(2);
  TORCH_CHECK(w_real.size(3) == C, "input channel count must match the weight channel count");
  TORCH_CHECK(R > 0 && S > 0, "kernel dimensions must be positive");
  const int64_t P = (H + 2 * pad_h - R) / stride_h + 1;
  const int64_t Q = (W + 2 * pad_w - S) / stride_w + 1;
  TORCH_CHECK(H + 2 * pad_h - R >= 0 && W + 2 * pad_w - S >= 0 && P > 0 && Q > 0,
              "invalid convolution configuration: output spatial size must be positive");
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  check_rc(ccv_check_shape(&shp), "shape check");
  auto y_real = torch::empty({N, P, Q, K}, x_real.options());
  auto y_imag = torch::empty({N, P, Q, K}, x_real.options());
  const size_t ws_bytes = ccv_forward_workspace_bytes(&shp);
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)},
                         x_real.options().dtype(torch::kUInt8));
  check_rc(ccv_forward(x_real.data_ptr<float>(), x_imag.data_ptr<float>(),
                       w_real.data_ptr<float>(), w_imag.data_ptr<float>(),
                       y_real.data_ptr<float>(), y_imag.data_ptr<float>(), &shp, ws.data_ptr(),
                       ws_bytes, current_stream()),
           "ccv_forward");
  return {y_real, y_imag};
}

// Packs KCRS (layout 0) or KRSC (layout 1) weights into the kernel image.
torch::Tensor prepack(torch::Tensor w_real, torch::Tensor w_imag, int64_t layout,
                      int64_t precision) {
  CHECK_CUDA(w_real); CHECK_CUDA(w_imag); CHECK_FLOAT(w_real); CHECK_FLOAT(w_imag);
  CHECK_CONTIGUOUS(w_real); CHECK_CONTIGUOUS(w_imag);
  TORCH_CHECK(w_real.dim() == 4 && w_real.sizes() == w_imag.sizes(),
              "weights must be two 4D tensors of identical shape");
  TORCH_CHECK(w_real.device() == w_imag.device(), "weights must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(w_real.device());
  int64_t K = w_real.size(0), C, R, S;
  if (layout == CCV_WEIGHT_KCRS) {
    C = w_real.size(1); R = w_real.size(2); S = w_real.size(3);
  } else {
    R = w_real.size(1); S = w_real.size(2); C = w_real.size(3);
  }
  // A shape with a 1x1 image and padding that keeps the output positive.
  ccv_conv_shape shp = make_shape(1, R, S, C, K, R, S, 1, 1, 0, 0);
  const size_t bytes = ccv_packed_weight_bytes(&shp, static_cast<int>(precision));
  check_rc(bytes == 0 ? ccv_check_shape(&shp) : CCV_OK, "weight shape check");
  auto packed = torch::empty({static_cast<int64_t>(bytes / 4)}, w_real.options());
  check_rc(ccv_prepack_weights(w_real.data_ptr<float>(), w_imag.data_ptr<float>(),
                               static_cast<int>(layout), &shp, static_cast<int>(precision),
                               packed.data_ptr(), bytes, current_stream()),
           "ccv_prepack_weights");
  return packed;
}

std::vector<torch::Tensor> forward_planar_packed(torch::Tensor x_real, torch::Tensor x_imag,
                                                 torch::Tensor w_packed, int64_t in_channels,
                                                 int64_t K, int64_t R, int64_t S,
                                                 int64_t stride_h, int64_t stride_w,
                                                 int64_t pad_h, int64_t pad_w, int64_t precision,
                                                 c10::optional<torch::Tensor> bias_real,
                                                 c10::optional<torch::Tensor> bias_imag) {
  CHECK_CUDA(x_real); CHECK_CUDA(x_imag); CHECK_CUDA(w_packed);
  CHECK_FLOAT(x_real); CHECK_FLOAT(x_imag); CHECK_FLOAT(w_packed);
  CHECK_CONTIGUOUS(x_real); CHECK_CONTIGUOUS(x_imag); CHECK_CONTIGUOUS(w_packed);
  TORCH_CHECK(x_real.dim() == 4, "x_real must be a 4D NHWC tensor");
  TORCH_CHECK(x_imag.dim() == 4, "x_imag must be a 4D NHWC tensor");
  TORCH_CHECK(x_real.sizes() == x_imag.sizes(), "x_real and x_imag must have identical shapes");
  TORCH_CHECK(x_real.device() == x_imag.device() && x_real.device() == w_packed.device(),
              "all inputs and weights must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(x_real.device());
  const int64_t N = x_real.size(0), H = x_real.size(1), W = x_real.size(2), C = x_real.size(3);
  TORCH_CHECK(C == in_channels, "input channel count must match the weight channel count");
  TORCH_CHECK(stride_h > 0 && stride_w > 0, "stride must be positive");
  TORCH_CHECK(pad_h >= 0 && pad_w >= 0, "padding must be non-negative");
  const int64_t P0 = (H + 2 * pad_h - R) / stride_h + 1;
  const int64_t Q0 = (W + 2 * pad_w - S) / stride_w + 1;
  TORCH_CHECK(H + 2 * pad_h - R >= 0 && W + 2 * pad_w - S >= 0 && P0 > 0 && Q0 > 0,
              "invalid convolution configuration: output spatial size must be positive");
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(static_cast<size_t>(w_packed.numel()) * 4 >=
                  ccv_packed_weight_bytes(&shp, static_cast<int>(precision)),
              "packed weights do not match the problem");
  const auto bias = bias_ptrs(bias_real, bias_imag, K, x_real);
  auto y_real = torch::empty({N, P, Q, K}, x_real.options());
  auto y_imag = torch::empty({N, P, Q, K}, x_real.options());
  const size_t ws_bytes = ccv_fprop_planar_workspace_bytes(&shp, static_cast<int>(precision));
  torch::Tensor ws;
  void* ws_ptr = nullptr;
  if (ws_bytes > 0) {
    ws = torch::empty({static_cast<int64_t>(ws_bytes)}, x_real.options().dtype(torch::kUInt8));
    ws_ptr = ws.data_ptr();
  }
  check_rc(ccv_fprop_planar_bias(x_real.data_ptr<float>(), x_imag.data_ptr<float>(),
                                 w_packed.data_ptr(), bias.first, bias.second,
                                 y_real.data_ptr<float>(), y_imag.data_ptr<float>(), &shp,
                                 static_cast<int>(precision), ws_ptr, ws_bytes, current_stream()),
           "ccv_fprop_planar");
  return {y_real, y_imag};
}

torch::Tensor forward_complex_packed(torch::Tensor x, torch::Tensor w_packed, int64_t K,
                                     int64_t R, int64_t S, int64_t stride_h, int64_t stride_w,
                                     int64_t pad_h, int64_t pad_w, int64_t precision,
                                     c10::optional<torch::Tensor> bias_real,
                                     c10::optional<torch::Tensor> bias_imag, bool strided) {
  CHECK_CUDA(x); CHECK_CUDA(w_packed);
  TORCH_CHECK(x.scalar_type() == at::kComplexFloat, "x must be complex64");
  CHECK_FLOAT(w_packed);
  CHECK_CONTIGUOUS(w_packed);
  TORCH_CHECK(x.dim() == 4, "x must be a 4D NCHW tensor");
  TORCH_CHECK(x.device() == w_packed.device(),
              "input and weights must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(x.device());
  const int64_t N = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3);
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(static_cast<size_t>(w_packed.numel()) * 4 >=
                  ccv_packed_weight_bytes(&shp, static_cast<int>(precision)),
              "packed weights do not match the problem");
  const auto bias = bias_ptrs(bias_real, bias_imag, K, x);
  auto y = torch::empty({N, K, P, Q}, x.options());
  const size_t ws_bytes = ccv_fprop_complex_workspace_bytes(&shp, static_cast<int>(precision));
  torch::Tensor ws;
  void* ws_ptr = nullptr;
  if (ws_bytes > 0) {
    ws = torch::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(torch::kUInt8));
    ws_ptr = ws.data_ptr();
  }
  if (x.is_contiguous() && !strided) {
    check_rc(ccv_fprop_complex_bias(x.data_ptr(), w_packed.data_ptr(), bias.first, bias.second,
                                    y.data_ptr(), &shp, static_cast<int>(precision), ws_ptr,
                                    ws_bytes, current_stream()),
             "ccv_fprop_complex");
  } else {
    // Any other layout (channels-last, slices, steps; or strided=true):
    // the layout kernel reads the strides; no contiguous copy of the input.
    const int64_t strides[4] = {x.stride(0), x.stride(1), x.stride(2), x.stride(3)};
    check_rc(ccv_fprop_complex_strided(x.data_ptr(), strides, w_packed.data_ptr(), bias.first,
                                       bias.second, y.data_ptr(), &shp,
                                       static_cast<int>(precision), ws_ptr, ws_bytes,
                                       current_stream()),
             "ccv_fprop_complex");
  }
  return y;
}

// Packed images of the data-gradient filter (transposed, flipped,
// conjugated; one per phase of the stride grid) from KCRS weight planes, for
// the layer's stride and padding; size as the forward image.
torch::Tensor prepack_dgrad(torch::Tensor w_real, torch::Tensor w_imag, int64_t stride_h,
                            int64_t stride_w, int64_t pad_h, int64_t pad_w, int64_t precision) {
  CHECK_CUDA(w_real); CHECK_CUDA(w_imag); CHECK_FLOAT(w_real); CHECK_FLOAT(w_imag);
  CHECK_CONTIGUOUS(w_real); CHECK_CONTIGUOUS(w_imag);
  TORCH_CHECK(w_real.dim() == 4 && w_real.sizes() == w_imag.sizes(),
              "weights must be two 4D tensors of identical shape");
  TORCH_CHECK(w_real.device() == w_imag.device(), "weights must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(w_real.device());
  const int64_t K = w_real.size(0), C = w_real.size(1), R = w_real.size(2), S = w_real.size(3);
  // The image depends on the filter, stride and padding only; an input of
  // R x S pixels keeps the shape valid for every filter size.
  ccv_conv_shape shp = make_shape(1, R, S, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  const size_t bytes = ccv_packed_weight_bytes(&shp, static_cast<int>(precision));
  check_rc(bytes == 0 ? ccv_check_shape(&shp) : CCV_OK, "weight shape check");
  auto packed = torch::empty({static_cast<int64_t>(bytes / 4)}, w_real.options());
  check_rc(ccv_prepack_weights_dgrad(w_real.data_ptr<float>(), w_imag.data_ptr<float>(),
                                     CCV_WEIGHT_KCRS, &shp, static_cast<int>(precision),
                                     packed.data_ptr(), bytes, current_stream()),
           "ccv_prepack_weights_dgrad");
  return packed;
}

// Data gradient: dy complex64 [N][K][P][Q] -> dx complex64 [N][C][H][W]
// (H, W: the forward input's size).
torch::Tensor dgrad_complex_packed(torch::Tensor dy, torch::Tensor w_packed_dgrad, int64_t C,
                                   int64_t H, int64_t W, int64_t R, int64_t S, int64_t stride_h,
                                   int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                   int64_t precision) {
  CHECK_CUDA(dy); CHECK_CUDA(w_packed_dgrad); CHECK_FLOAT(w_packed_dgrad);
  CHECK_CONTIGUOUS(w_packed_dgrad);
  TORCH_CHECK(dy.scalar_type() == at::kComplexFloat, "dy must be complex64");
  TORCH_CHECK(dy.dim() == 4, "dy must be a 4D NCHW tensor");
  TORCH_CHECK(dy.device() == w_packed_dgrad.device(),
              "gradient and weights must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(dy.device());
  dy = dy.contiguous();
  const int64_t N = dy.size(0), K = dy.size(1);
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(dy.size(2) == P && dy.size(3) == Q, "dy does not match the forward output size");
  TORCH_CHECK(static_cast<size_t>(w_packed_dgrad.numel()) * 4 >=
                  ccv_packed_weight_bytes(&shp, static_cast<int>(precision)),
              "packed weights do not match the problem");
  const size_t ws_bytes = ccv_dgrad_complex_workspace_bytes(&shp, static_cast<int>(precision));
  check_rc(ws_bytes == 0 ? CCV_ERR_UNSUPPORTED : CCV_OK, "data gradient");
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, dy.options().dtype(torch::kUInt8));
  auto dx = torch::empty({N, C, H, W}, dy.options());
  check_rc(ccv_dgrad_complex(dy.data_ptr(), w_packed_dgrad.data_ptr(), dx.data_ptr(), &shp,
                             static_cast<int>(precision), ws.data_ptr(), ws_bytes,
                             current_stream()),
           "ccv_dgrad_complex");
  return dx;
}

// Weight gradient: x complex64 NCHW and dy complex64 NKPQ -> (dW_real,
// dW_imag) fp32 KCRS.
std::vector<torch::Tensor> wgrad_complex(torch::Tensor x, torch::Tensor dy, int64_t R, int64_t S,
                                         int64_t stride_h, int64_t stride_w, int64_t pad_h,
                                         int64_t pad_w) {
  CHECK_CUDA(x); CHECK_CUDA(dy);
  TORCH_CHECK(x.scalar_type() == at::kComplexFloat && dy.scalar_type() == at::kComplexFloat,
              "x and dy must be complex64");
  TORCH_CHECK(x.dim() == 4 && dy.dim() == 4, "x and dy must be 4D NCHW tensors");
  TORCH_CHECK(x.device() == dy.device(), "x and dy must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(x.device());
  x = x.contiguous();
  dy = dy.contiguous();
  const int64_t N = x.size(0), C = x.size(1), H = x.size(2), W = x.size(3), K = dy.size(1);
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(dy.size(0) == N && dy.size(2) == P && dy.size(3) == Q,
              "dy does not match the forward output size");
  const size_t ws_bytes = ccv_wgrad_complex_workspace_bytes(&shp);
  check_rc(ws_bytes == 0 ? ccv_check_shape(&shp) : CCV_OK, "weight gradient");
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, x.options().dtype(torch::kUInt8));
  auto fo = x.options().dtype(torch::kFloat);
  auto dwr = torch::empty({K, C, R, S}, fo);
  auto dwi = torch::empty({K, C, R, S}, fo);
  check_rc(ccv_wgrad_complex(x.data_ptr(), dy.data_ptr(), dwr.data_ptr<float>(),
                             dwi.data_ptr<float>(), &shp, ws.data_ptr(), ws_bytes,
                             current_stream()),
           "ccv_wgrad_complex");
  return {dwr, dwi};
}

// Planar data gradient: dy planes NPQK -> dx planes NHWC [N][H][W][C].
std::vector<torch::Tensor> dgrad_planar_packed(torch::Tensor dy_real, torch::Tensor dy_imag,
                                               torch::Tensor w_packed_dgrad, int64_t C, int64_t H,
                                               int64_t W, int64_t R, int64_t S,
                                               int64_t stride_h, int64_t stride_w, int64_t pad_h,
                                               int64_t pad_w, int64_t precision) {
  CHECK_CUDA(dy_real); CHECK_CUDA(dy_imag); CHECK_CUDA(w_packed_dgrad);
  CHECK_FLOAT(dy_real); CHECK_FLOAT(dy_imag); CHECK_FLOAT(w_packed_dgrad);
  CHECK_CONTIGUOUS(w_packed_dgrad);
  TORCH_CHECK(dy_real.dim() == 4 && dy_real.sizes() == dy_imag.sizes(),
              "dy_real and dy_imag must be 4D NHWC tensors of identical shape");
  c10::cuda::CUDAGuard guard(dy_real.device());
  dy_real = dy_real.contiguous();
  dy_imag = dy_imag.contiguous();
  const int64_t N = dy_real.size(0), K = dy_real.size(3);
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(dy_real.size(1) == P && dy_real.size(2) == Q,
              "dy does not match the forward output size");
  const size_t ws_bytes = ccv_dgrad_planar_workspace_bytes(&shp, static_cast<int>(precision));
  torch::Tensor ws;
  void* ws_ptr = nullptr;
  if (ws_bytes > 0) {
    ws = torch::empty({static_cast<int64_t>(ws_bytes)}, dy_real.options().dtype(torch::kUInt8));
    ws_ptr = ws.data_ptr();
  }
  auto dxr = torch::empty({N, H, W, C}, dy_real.options());
  auto dxi = torch::empty({N, H, W, C}, dy_real.options());
  check_rc(ccv_dgrad_planar(dy_real.data_ptr<float>(), dy_imag.data_ptr<float>(),
                            w_packed_dgrad.data_ptr(), dxr.data_ptr<float>(),
                            dxi.data_ptr<float>(), &shp, static_cast<int>(precision), ws_ptr,
                            ws_bytes, current_stream()),
           "ccv_dgrad_planar");
  return {dxr, dxi};
}

// Planar weight gradient: x planes NHWC and dy planes NPQK -> (dW_real,
// dW_imag) fp32 KCRS.
std::vector<torch::Tensor> wgrad_planar(torch::Tensor x_real, torch::Tensor x_imag,
                                        torch::Tensor dy_real, torch::Tensor dy_imag, int64_t R,
                                        int64_t S, int64_t stride_h, int64_t stride_w,
                                        int64_t pad_h, int64_t pad_w) {
  for (const auto* t : {&x_real, &x_imag, &dy_real, &dy_imag}) {
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == at::kFloat && t->dim() == 4,
                "inputs must be 4D CUDA float32 tensors");
  }
  TORCH_CHECK(x_real.sizes() == x_imag.sizes() && dy_real.sizes() == dy_imag.sizes(),
              "real and imaginary planes must have identical shapes");
  c10::cuda::CUDAGuard guard(x_real.device());
  x_real = x_real.contiguous(); x_imag = x_imag.contiguous();
  dy_real = dy_real.contiguous(); dy_imag = dy_imag.contiguous();
  const int64_t N = x_real.size(0), H = x_real.size(1), W = x_real.size(2), C = x_real.size(3);
  const int64_t K = dy_real.size(3);
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(dy_real.size(0) == N && dy_real.size(1) == P && dy_real.size(2) == Q,
              "dy does not match the forward output size");
  const size_t ws_bytes = ccv_wgrad_planar_workspace_bytes(&shp);
  check_rc(ws_bytes == 0 ? ccv_check_shape(&shp) : CCV_OK, "weight gradient");
  auto ws = torch::empty({static_cast<int64_t>(ws_bytes)}, x_real.options().dtype(torch::kUInt8));
  auto dwr = torch::empty({K, C, R, S}, x_real.options());
  auto dwi = torch::empty({K, C, R, S}, x_real.options());
  check_rc(ccv_wgrad_planar(x_real.data_ptr<float>(), x_imag.data_ptr<float>(),
                            dy_real.data_ptr<float>(), dy_imag.data_ptr<float>(),
                            dwr.data_ptr<float>(), dwi.data_ptr<float>(), &shp, ws.data_ptr(),
                            ws_bytes, current_stream()),
           "ccv_wgrad_planar");
  return {dwr, dwi};
}

// Planar NHWC planes in, complex64 NKPQ out (the conv launch of forward()
// without its layout pass).
torch::Tensor forward_planar_to_complex_packed(torch::Tensor x_real, torch::Tensor x_imag,
                                               torch::Tensor w_packed, int64_t in_channels,
                                               int64_t K, int64_t R, int64_t S, int64_t stride_h,
                                               int64_t stride_w, int64_t pad_h, int64_t pad_w,
                                               int64_t precision) {
  CHECK_CUDA(x_real); CHECK_CUDA(x_imag); CHECK_CUDA(w_packed);
  CHECK_FLOAT(x_real); CHECK_FLOAT(x_imag); CHECK_FLOAT(w_packed);
  CHECK_CONTIGUOUS(x_real); CHECK_CONTIGUOUS(x_imag); CHECK_CONTIGUOUS(w_packed);
  TORCH_CHECK(x_real.dim() == 4 && x_real.sizes() == x_imag.sizes(),
              "x_real and x_imag must be 4D NHWC tensors of identical shape");
  c10::cuda::CUDAGuard guard(x_real.device());
  const int64_t N = x_real.size(0), H = x_real.size(1), W = x_real.size(2), C = x_real.size(3);
  TORCH_CHECK(C == in_channels, "input channel count must match the weight channel count");
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  int64_t P = 0, Q = 0;
  check_rc(ccv_output_size(&shp, &P, &Q), "shape check");
  TORCH_CHECK(static_cast<size_t>(w_packed.numel()) * 4 >=
                  ccv_packed_weight_bytes(&shp, static_cast<int>(precision)),
              "packed weights do not match the problem");
  auto y = torch::empty({N, K, P, Q}, x_real.options().dtype(at::kComplexFloat));
  const size_t ws_bytes = ccv_fprop_planar_workspace_bytes(&shp, static_cast<int>(precision));
  torch::Tensor ws;
  void* ws_ptr = nullptr;
  if (ws_bytes > 0) {
    ws = torch::empty({static_cast<int64_t>(ws_bytes)}, x_real.options().dtype(torch::kUInt8));
    ws_ptr = ws.data_ptr();
  }
  check_rc(ccv_fprop_planar_to_complex(x_real.data_ptr<float>(), x_imag.data_ptr<float>(),
                                       w_packed.data_ptr(), y.data_ptr(), &shp,
                                       static_cast<int>(precision), ws_ptr, ws_bytes,
                                       current_stream()),
           "ccv_fprop_planar_to_complex");
  return y;
}

// Name of the kernel path forward_complex_packed takes.
std::string complex_forward_kernel(int64_t N, int64_t C, int64_t H, int64_t W, int64_t K,
                                   int64_t R, int64_t S, int64_t stride_h, int64_t stride_w,
                                   int64_t pad_h, int64_t pad_w, int64_t precision) {
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  return std::string(ccv_fprop_complex_kernel(&shp, static_cast<int>(precision)));
}

// Kernel launches of one forward_complex_packed call: 1 for the one-launch
// kernels, 2 with the layout pass (3 for 3xTF32 with a split pass).
int64_t complex_forward_launches(int64_t N, int64_t C, int64_t H, int64_t W, int64_t K, int64_t R,
                                 int64_t S, int64_t stride_h, int64_t stride_w, int64_t pad_h,
                                 int64_t pad_w, int64_t precision) {
  ccv_conv_shape shp = make_shape(N, H, W, C, K, R, S, stride_h, stride_w, pad_h, pad_w);
  check_rc(ccv_check_shape(&shp), "shape check");
  int kernels = 0;
  check_rc(ccv_fprop_kernel_launches(&shp, static_cast<int>(precision), 1, &kernels),
           "ccv_fprop_kernel_launches");
  return kernels;
}

int64_t device_status(int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  int st = 0;
  check_rc(ccv_get_device_status(&st), "ccv_get_device_status");
  return st;
}

void clear_device_status(int64_t device) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  check_rc(ccv_clear_device_status(), "ccv_clear_device_status");
}

// Runs the bounded-wait self-test.  library=false: into a fresh device int,
// returned; library=true: into the library's own status word, as a real
// in-kernel timeout would (returns 0; read it with device_status).
int64_t selftest_bounded_wait(int64_t device, bool library) {
  c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  if (library) {
    check_rc(ccv_selftest_bounded_wait(nullptr, current_stream()), "ccv_selftest_bounded_wait");
    return 0;
  }
  auto st = torch::zeros({1}, torch::TensorOptions()
                                  .dtype(torch::kInt32)
                                  .device(torch::kCUDA, static_cast<c10::DeviceIndex>(device)));
  check_rc(ccv_selftest_bounded_wait(st.data_ptr<int>(), current_stream()),
           "ccv_selftest_bounded_wait");
  return st.item<int>();
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &forward, "B200 tcgen05 planar-complex Conv2d forward (KRSC weights)",
        pybind11::arg("x_real"), pybind11::arg("x_imag"), pybind11::arg("w_real"),
        pybind11::arg("w_imag"), pybind11::arg("stride_h"), pybind11::arg("stride_w"),
        pybind11::arg("pad_h"), pybind11::arg("pad_w"));
  m.def("prepack", &prepack, "Pack weights into the kernel image", pybind11::arg("w_real"),
        pybind11::arg("w_imag"), pybind11::arg("layout"), pybind11::arg("precision"));
  m.def("forward_planar_packed", &forward_planar_packed, "Planar NHWC forward, packed weights",
        pybind11::arg("x_real"), pybind11::arg("x_imag"), pybind11::arg("w_packed"),
        pybind11::arg("in_channels"), pybind11::arg("out_channels"), pybind11::arg("kernel_h"), pybind11::arg("kernel_w"),
        pybind11::arg("stride_h"), pybind11::arg("stride_w"), pybind11::arg("pad_h"),
        pybind11::arg("pad_w"), pybind11::arg("precision"),
        pybind11::arg("bias_real") = pybind11::none(), pybind11::arg("bias_imag") = pybind11::none());
  m.def("forward_complex_packed", &forward_complex_packed,
        "complex64 NCHW forward, packed weights", pybind11::arg("x"), pybind11::arg("w_packed"),
        pybind11::arg("out_channels"), pybind11::arg("kernel_h"), pybind11::arg("kernel_w"),
        pybind11::arg("stride_h"), pybind11::arg("stride_w"), pybind11::arg("pad_h"),
        pybind11::arg("pad_w"), pybind11::arg("precision"),
        pybind11::arg("bias_real") = pybind11::none(), pybind11::arg("bias_imag") = pybind11::none(),
        pybind11::arg("strided") = false);
  m.def("forward_planar_to_complex_packed", &forward_planar_to_complex_packed,
        "planar NHWC in, complex64 NCHW out, packed weights", pybind11::arg("x_real"),
        pybind11::arg("x_imag"), pybind11::arg("w_packed"), pybind11::arg("in_channels"),
        pybind11::arg("out_channels"), pybind11::arg("kernel_h"), pybind11::arg("kernel_w"),
        pybind11::arg("stride_h"), pybind11::arg("stride_w"), pybind11::arg("pad_h"),
        pybind11::arg("pad_w"), pybind11::arg("precision"));
  m.def("complex_forward_kernel", &complex_forward_kernel, pybind11::arg("n"),
        pybind11::arg("c"), pybind11::arg("h"), pybind11::arg("w"), pybind11::arg("k"),
        pybind11::arg("r"), pybind11::arg("s"), pybind11::arg("stride_h"),
        pybind11::arg("stride_w"), pybind11::arg("pad_h"), pybind11::arg("pad_w"),
        pybind11::arg("precision"));
  m.def("complex_forward_launches", &complex_forward_launches, pybind11::arg("n"),
        pybind11::arg("c"), pybind11::arg("h"), pybind11::arg("w"), pybind11::arg("k"),
        pybind11::arg("r"), pybind11::arg("s"), pybind11::arg("stride_h"),
        pybind11::arg("stride_w"), pybind11::arg("pad_h"), pybind11::arg("pad_w"),
        pybind11::arg("precision"));
  m.def("prepack_dgrad", &prepack_dgrad, "Pack the data-gradient filter (KCRS planes)",
        pybind11::arg("w_real"), pybind11::arg("w_imag"), pybind11::arg("stride_h"),
        pybind11::arg("stride_w"), pybind11::arg("pad_h"), pybind11::arg("pad_w"),
        pybind11::arg("precision"));
  m.def("dgrad_complex_packed", &dgrad_complex_packed, "Data gradient, complex64 NCHW",
        pybind11::arg("dy"), pybind11::arg("w_packed_dgrad"), pybind11::arg("in_channels"),
        pybind11::arg("in_h"), pybind11::arg("in_w"), pybind11::arg("kernel_h"),
        pybind11::arg("kernel_w"), pybind11::arg("stride_h"), pybind11::arg("stride_w"),
        pybind11::arg("pad_h"), pybind11::arg("pad_w"), pybind11::arg("precision"));
  m.def("dgrad_planar_packed", &dgrad_planar_packed, "Data gradient, fp32 NHWC planes",
        pybind11::arg("dy_real"), pybind11::arg("dy_imag"), pybind11::arg("w_packed_dgrad"),
        pybind11::arg("in_channels"), pybind11::arg("in_h"), pybind11::arg("in_w"),
        pybind11::arg("kernel_h"), pybind11::arg("kernel_w"), pybind11::arg("stride_h"),
        pybind11::arg("stride_w"), pybind11::arg("pad_h"), pybind11::arg("pad_w"),
        pybind11::arg("precision"));
  m.def("wgrad_planar", &wgrad_planar, "Weight gradient from planes -> (dW_real, dW_imag)",
        pybind11::arg("x_real"), pybind11::arg("x_imag"), pybind11::arg("dy_real"),
        pybind11::arg("dy_imag"), pybind11::arg("kernel_h"), pybind11::arg("kernel_w"),
        pybind11::arg("stride_h"), pybind11::arg("stride_w"), pybind11::arg("pad_h"),
        pybind11::arg("pad_w"));
  m.def("wgrad_complex", &wgrad_complex, "Weight gradient -> (dW_real, dW_imag) KCRS",
        pybind11::arg("x"), pybind11::arg("dy"), pybind11::arg("kernel_h"),
        pybind11::arg("kernel_w"), pybind11::arg("stride_h"), pybind11::arg("stride_w"),
        pybind11::arg("pad_h"), pybind11::arg("pad_w"));
  m.def("device_status", &device_status, pybind11::arg("device"));
  m.def("clear_device_status", &clear_device_status, pybind11::arg("device"));
  m.def("selftest_bounded_wait", &selftest_bounded_wait, pybind11::arg("device"),
        pybind11::arg("library") = false);
  m.def("reload_config", []() { check_rc(ccv_reload_config(), "ccv_reload_config"); },
        "re-read the CCV_* environment switches");
  m.def("version", []() { return std::string(ccv_version()); });
}
