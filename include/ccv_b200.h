/*
 * ccv_b200.h - C ABI of the B200 (sm_100a) complex-valued Conv2d forward.
 *
 * This is the drop-in boundary that replaces the reference's compiled
 * extension `complex_conv2d._C` (pybind module defined in
 * csrc/bindings.cpp:16-29 of jaeeunHwang/cutlass-complex-conv, whose body is
 * `complex_conv2d_cuda` in csrc/complex_conv2d.cu:84-309).  All entry points
 * take plain device pointers and sizes and allocate no device memory.
 * Scratch memory comes from the caller: the *_workspace_bytes queries give
 * the size that enables every optimisation, *_min_workspace_bytes the size a
 * call cannot run without.  The first launching call on a device makes one
 * 4-byte pinned host allocation (the host copy of the device status word,
 * see ccv_get_device_status); ccv_forward_noalloc makes none.  Every launch
 * is asynchronous on the given stream.
 *
 * Conventions
 *   - Activation planes x_real/x_imag: fp32 NHWC, contiguous
 *     (reference: modules.py:153-174, complex_conv2d.cu:134-138).
 *   - Complex activations: complex64 NCHW, interleaved (re, im) fp32 pairs
 *     (reference: modules.py:176-207).
 *   - Output planes y_real/y_imag: fp32 NPQK (NHWC), contiguous
 *     (reference: complex_conv2d.cu:161-165).  Complex output: complex64
 *     NKPQ (NCHW) interleaved.
 *   - Cross-correlation, zero padding, dilation 1, groups 1
 *     (reference: complex_conv2d.cu:173-195).
 *   - P = (H + 2*pad_h - R) / stride_h + 1, Q likewise
 *     (reference: complex_conv2d.cu:151-155).
 *   - Constraints (reference: device/implicit_planar_cgemm_convolution.h
 *     can_implement, :71-187): C % 4 == 0, K % 4 == 0, every tensor below
 *     2^31 bytes per plane; additionally stride <= 8 (TMA traversal stride).
 *   - All pointers 16-byte aligned.
 *
 * Return value of every int function: CCV_OK or a CCV_ERR_* code; the text
 * of the last error on the calling thread is ccv_last_error_message().
 */
#ifndef CCV_B200_H_
#define CCV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream. */
typedef struct CUstream_st* ccv_stream_t;

enum ccv_status {
  CCV_OK = 0,
  CCV_ERR_INVALID_ARGUMENT = 1, /* bad shape, pointer, alignment or size  */
  CCV_ERR_UNSUPPORTED = 2,      /* reference: "CUTLASS cannot implement"   */
  CCV_ERR_WORKSPACE = 3,        /* workspace missing or too small          */
  CCV_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed       */
  CCV_ERR_DEVICE = 5,           /* device not sm_100 or status word set    */
  CCV_ERR_DEVICE_TIMEOUT = 6    /* a bounded in-kernel wait ran out        */
};

enum ccv_precision {
  CCV_PRECISION_TF32 = 0,  /* TF32 tensor-core products, FP32 accumulate   */
  CCV_PRECISION_3XTF32 = 1 /* split-TF32 (hi*hi + hi*lo + lo*hi), ~FP32  */
};

enum ccv_weight_layout {
  CCV_WEIGHT_KCRS = 0, /* nn.Module parameter layout (modules.py:93-107)   */
  CCV_WEIGHT_KRSC = 1  /* extension layout (complex_conv2d.cu:140-143)     */
};

typedef struct ccv_conv_shape {
  int64_t n, h, w, c; /* input batch, height, width, channels */
  int64_t k, r, s;    /* output channels, filter height, filter width */
  int64_t stride_h, stride_w;
  int64_t pad_h, pad_w;
} ccv_conv_shape;

/* Output spatial size; reference complex_conv2d.cu:151-159. */
int ccv_output_size(const ccv_conv_shape* shape, int64_t* p, int64_t* q);

/* Validate a problem the way can_implement does (complex_conv2d.cu:94-159,
 * device/implicit_planar_cgemm_convolution.h:71-187). */
int ccv_check_shape(const ccv_conv_shape* shape);

/* Bytes of the packed weight image used by the fprop kernels. */
size_t ccv_packed_weight_bytes(const ccv_conv_shape* shape, int precision);

/* Repack real/imag weight planes (KCRS or KRSC fp32) into the kernel's
 * packed image: per filter tap, planes (-W_im, W_re, W_im) of [K][C], each
 * value rounded to TF32 (3xTF32 adds a second image of the rounding
 * remainders).  Replaces the KCRS->KRSC prepack of modules.py:127-151. */
int ccv_prepack_weights(const float* w_real, const float* w_imag, int layout,
                        const ccv_conv_shape* shape, int precision,
                        void* packed, size_t packed_bytes, ccv_stream_t stream);

/* Scratch bytes for the fprop entry points below.  *_workspace_bytes: the
 * recommended size - the required scratch plus room for the stream-K split
 * of the last partial wave of output tiles (partial sums and counters; an
 * upper bound for the current device).  *_min_workspace_bytes: the required
 * part alone; a call given only that runs every tile whole.  The required
 * part is 0 for TF32 planar calls. */
size_t ccv_fprop_planar_workspace_bytes(const ccv_conv_shape* shape, int precision);
size_t ccv_fprop_complex_workspace_bytes(const ccv_conv_shape* shape, int precision);
size_t ccv_fprop_planar_min_workspace_bytes(const ccv_conv_shape* shape, int precision);
size_t ccv_fprop_complex_min_workspace_bytes(const ccv_conv_shape* shape, int precision);

/* Number of library kernels one ccv_fprop_planar (complex_input = 0) or
 * ccv_fprop_complex (complex_input = 1) call launches: the conv kernel plus
 * any layout/split pass. */
int ccv_fprop_kernel_launches(const ccv_conv_shape* shape, int precision, int complex_input,
                              int* kernels);

/* Name of the kernel path ccv_fprop_complex takes for this problem (static
 * string): "halo_pair_layout_warps" / "tap_pair_layout_warps" (one launch:
 * warps of the convolution kernel convert the complex64 input into the
 * workspace planes it reads) or "layout_pass+<kernel>" (a complex64 ->
 * planar pass, then the kernel). */
const char* ccv_fprop_complex_kernel(const ccv_conv_shape* shape, int precision);

/* Planar fprop: fp32 NHWC planes in, fp32 NPQK planes out, packed weights.
 * Replaces complex_conv2d_cuda (csrc/complex_conv2d.cu:84-309) behind
 * ComplexConv2d.forward_planar (modules.py:153-174).  TF32 needs no
 * workspace; 3xTF32 needs ccv_fprop_planar_min_workspace_bytes() (the inputs
 * split into TF32 parts and remainders) and weights packed for 3xTF32.
 * Workspace past the required part (256-byte aligned) is used for the
 * stream-K split.  Results do not depend on whether the split is taken
 * beyond fp32 summation order (deterministic for a given workspace size). */
int ccv_fprop_planar(const float* x_real, const float* x_imag, const void* w_packed,
                     float* y_real, float* y_imag, const ccv_conv_shape* shape,
                     int precision, void* workspace, size_t workspace_bytes,
                     ccv_stream_t stream);

/* Complex fprop: complex64 NCHW in, complex64 NKPQ out, packed weights.
 * Replaces the layout conversions plus kernel of ComplexConv2d.forward
 * (modules.py:176-207).  Needs ccv_fprop_complex_min_workspace_bytes() of
 * workspace (fp32 planes of the input). */
int ccv_fprop_complex(const void* x, const void* w_packed, void* y,
                      const ccv_conv_shape* shape, int precision, void* workspace,
                      size_t workspace_bytes, ccv_stream_t stream);

/* ccv_fprop_planar / ccv_fprop_complex with a complex bias per output
 * channel: y[n, k, p, q] += bias_real[k] + i * bias_imag[k], added once to
 * the final sums in the kernels' epilogue.  bias_real and bias_imag are K
 * fp32 values each on the device, 16-byte aligned; both null is the call
 * without bias.  The reference rejects bias=True (modules.py:73-74), so
 * these have no reference counterpart; the bias is the one of
 * torch.nn.Conv2d on complex64 tensors. */
int ccv_fprop_planar_bias(const float* x_real, const float* x_imag, const void* w_packed,
                          const float* bias_real, const float* bias_imag, float* y_real,
                          float* y_imag, const ccv_conv_shape* shape, int precision,
                          void* workspace, size_t workspace_bytes, ccv_stream_t stream);
int ccv_fprop_complex_bias(const void* x, const void* w_packed, const float* bias_real,
                           const float* bias_imag, void* y, const ccv_conv_shape* shape,
                           int precision, void* workspace, size_t workspace_bytes,
                           ccv_stream_t stream);

/* ccv_fprop_complex_bias on a complex64 input of any layout: x_strides[4]
 * are the element strides of dimensions (n, c, h, w) - a channels-last
 * tensor, a slice, a view with a step.  Replaces the .contiguous() copy that
 * ComplexConv2d.forward makes of such inputs (modules.py:198-199): the
 * layout kernel reads the strides directly.  x 8-byte aligned; strides >= 0.
 * Dense NCHW strides take the ccv_fprop_complex path.  Output, workspace
 * and bias as ccv_fprop_complex_bias (bias pointers may be null). */
int ccv_fprop_complex_strided(const void* x, const int64_t* x_strides, const void* w_packed,
                              const float* bias_real, const float* bias_imag, void* y,
                              const ccv_conv_shape* shape, int precision, void* workspace,
                              size_t workspace_bytes, ccv_stream_t stream);

/* Planar fp32 NHWC in, complex64 NKPQ out: the convolution launch of
 * ccv_fprop_complex without its layout pass (for callers that hold planar
 * activations but want complex output).  Workspace as ccv_fprop_planar. */
int ccv_fprop_planar_to_complex(const float* x_real, const float* x_imag, const void* w_packed,
                                void* y, const ccv_conv_shape* shape, int precision,
                                void* workspace, size_t workspace_bytes, ccv_stream_t stream);

/* The reference extension call itself: `_C.forward(x_real, x_imag, w_real,
 * w_imag, stride_h, stride_w, pad_h, pad_w)` (csrc/bindings.cpp:16-29) with
 * KRSC weights, TF32.  Needs the packed weight bytes (256-byte aligned) of
 * scratch; ccv_forward_workspace_bytes() adds the stream-K room. */
size_t ccv_forward_workspace_bytes(const ccv_conv_shape* shape);
int ccv_forward(const float* x_real, const float* x_imag, const float* w_real_krsc,
                const float* w_imag_krsc, float* y_real, float* y_imag,
                const ccv_conv_shape* shape, void* workspace, size_t workspace_bytes,
                ccv_stream_t stream);

/* ccv_forward without scratch allocation - no counterpart in the reference.
 * For callers that may not allocate device memory at all (code running in
 * another framework's enqueue/execute callback, where that framework owns
 * the memory pool and a cudaMalloc/cudaFree could synchronize the device).
 * Same contract and results as ccv_forward, but the packed weights live in
 * a fixed device array of CCV_NOALLOC_MAX_WEIGHT_BYTES inside the library
 * (reserved on every GPU that loads it, until process exit).  Problems whose
 * packed weights (3 * R*S*K*C * 4 bytes) exceed it return CCV_ERR_WORKSPACE.
 * All calls on a device share that array: calls that overlap on the GPU race,
 * so order them on one stream.  The first call on a device looks up the
 * array's address and must come before any stream capture. */
#define CCV_NOALLOC_MAX_WEIGHT_BYTES (16u * 1024u * 1024u)
int ccv_forward_noalloc(const float* x_real, const float* x_imag,
                        const float* w_real_krsc, const float* w_imag_krsc,
                        float* y_real, float* y_imag, const ccv_conv_shape* shape,
                        ccv_stream_t stream);

/* Backward - no counterpart in the reference, whose extension is forward
 * only (README.md:143 lists backward as absent).  The gradients are those
 * torch autograd gives for the reference's four-conv module
 * (benchmarks/baseline.py:12-45) with upstream gradient dy, in PyTorch's
 * complex convention:
 *   dx[n,c,h,w] = sum_{k,r,s} conj(W[k,c,r,s]) dy[n,k,p,q]
 *   dW[k,c,r,s] = sum_{n,p,q} dy[n,k,p,q] conj(x[n,c,h,w])
 * (h = p*stride_h - pad_h + r, w = q*stride_w - pad_w + s); dw_real and
 * dw_imag are the gradients of weight_real and weight_imag.  `shape` is the
 * FORWARD problem.  dy: complex64 NKPQ, dx: complex64 NCHW, x: complex64
 * NCHW, dw_real/dw_imag: fp32 KCRS; all dense.
 *
 * Data gradient: forward convolutions of dy with the transposed, flipped,
 * conjugated filter - one per phase of the stride grid (stride 1: one, run
 * on dy in place when pad <= kernel size - 1) - whose packed images
 * ccv_prepack_weights_dgrad builds (total size
 * ccv_packed_weight_bytes(shape, precision)).  TF32 or 3xTF32. */
int ccv_prepack_weights_dgrad(const float* w_real, const float* w_imag, int layout,
                              const ccv_conv_shape* shape, int precision, void* packed,
                              size_t packed_bytes, ccv_stream_t stream);
size_t ccv_dgrad_complex_workspace_bytes(const ccv_conv_shape* shape, int precision);
int ccv_dgrad_complex(const void* dy, const void* w_packed_dgrad, void* dx,
                      const ccv_conv_shape* shape, int precision, void* workspace,
                      size_t workspace_bytes, ccv_stream_t stream);

/* Weight gradient (TF32 products, FP32 accumulation; the operands are
 * rounded to TF32 first).  Writes every element of dw_real and dw_imag;
 * deterministic. */
size_t ccv_wgrad_complex_workspace_bytes(const ccv_conv_shape* shape);
int ccv_wgrad_complex(const void* x, const void* dy, float* dw_real, float* dw_imag,
                      const ccv_conv_shape* shape, void* workspace, size_t workspace_bytes,
                      ccv_stream_t stream);

/* The same gradients for the planar path (forward_planar): dy_real/dy_imag
 * fp32 NPQK planes, dx_real/dx_imag fp32 NHWC planes, x_real/x_imag fp32
 * NHWC planes; the packed filter of ccv_prepack_weights_dgrad. */
size_t ccv_dgrad_planar_workspace_bytes(const ccv_conv_shape* shape, int precision);
int ccv_dgrad_planar(const float* dy_real, const float* dy_imag, const void* w_packed_dgrad,
                     float* dx_real, float* dx_imag, const ccv_conv_shape* shape, int precision,
                     void* workspace, size_t workspace_bytes, ccv_stream_t stream);
size_t ccv_wgrad_planar_workspace_bytes(const ccv_conv_shape* shape);
int ccv_wgrad_planar(const float* x_real, const float* x_imag, const float* dy_real,
                     const float* dy_imag, float* dw_real, float* dw_imag,
                     const ccv_conv_shape* shape, void* workspace, size_t workspace_bytes,
                     ccv_stream_t stream);

/* Device status word of the current device: nonzero after an in-kernel
 * bounded wait ran out (a CCV_ERR_* code).  While it is set, fprop kernels
 * on that device exit without work.  The kernel that gives up also writes a
 * host-mapped copy of the word (set up by the first allocating call on the
 * device), and every entry point that launches work reads that copy first:
 * once a timeout has reached it, they return CCV_ERR_DEVICE and launch
 * nothing until ccv_clear_device_status.  (A call enqueued before the
 * timeout happened returns CCV_OK and its kernels exit without work.)
 * get copies the device word to the host (synchronizes the device); clear
 * resets the word, its host copy and the library's counter sets. */
int ccv_get_device_status(int* status);
int ccv_clear_device_status(void);

/* Self-test of the bounded wait: launches one CTA that waits on an mbarrier
 * nothing arrives on.  The wait gives up after its time limit and the
 * kernel writes CCV_ERR_DEVICE_TIMEOUT into *status_dev (a device int the
 * caller zeroed), leaving the context usable.  status_dev == NULL: into the
 * library's own status word (and its host copy), as a real timeout would. */
int ccv_selftest_bounded_wait(int* status_dev, ccv_stream_t stream);

/* Re-reads the CCV_* environment switches (testing and benchmarking knobs,
 * read once on first use otherwise). */
int ccv_reload_config(void);

/* Text of the last error raised on the calling host thread. */
const char* ccv_last_error_message(void);

/* Library version string. */
const char* ccv_version(void);

#ifdef __cplusplus
}
#endif

#endif /* CCV_B200_H_ */
