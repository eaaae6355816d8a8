// Backward of the complex Conv2d: data gradient (dgrad) and weight gradient
// (wgrad).  The reference is forward-only (its README lists backward as
// absent); the gradients here are those torch autograd gives for the
// reference's own four-conv module (benchmarks/baseline.py:12-45), in
// PyTorch's complex convention (conjugate Wirtinger):
//
//     dx[n,c,h,w] = sum_{k,r,s} conj(W[k,c,r,s]) * dy[n,k,p,q]
//     dW[k,c,r,s] = sum_{n,p,q} dy[n,k,p,q] * conj(x[n,c,h,w])
//
// over h = p*sh - ph + r, w = q*sw - pw + s.
//
// dgrad is a forward convolution of dy with the filter transposed (K <-> C),
// flipped (r -> R-1-r, s -> S-1-s) and conjugated, padding R-1-ph / S-1-pw,
// on the forward kernels (ccv_fprop*.cu) with a packed image of that filter
// (ccv_prepack_dgrad_kernel).  For stride > 1 the output splits into the
// sh*sw phases of the stride grid (rows h = sh*i + a, columns w = sw*j + b):
// phase (a, b) only meets filter rows r = ra + sh*t and columns
// s = rb + sw*u, so it is a stride-1 convolution of dy with that sub-filter
// (a copy of dy with the phase's zero border, ccv_dgrad_phase_pad_kernel);
// ccv_dgrad_interleave_kernel writes the phases into dx.  Every filter tap
// belongs to exactly one phase, so the phases together do the forward's MACs.
//
// wgrad is an implicit GEMM per filter tap (r, s): M = output channels k
// (128-row tiles), N = input channels c, reduction over the output pixels
// (n, p, q) in steps of 32 consecutive q.  Its operands come from two
// layout kernels: dy as fp32 planes [N][K][P][Q] (q contiguous) and x as
// fp32 planes [S][N][C][H][Q], the input column q*sw - pw + s that filter
// column s reads for output column q (zero outside the image) - one copy
// per filter column, so that every TMA box starts at a multiple of 32
// pixels (a tiled TMA copy must start on a 16-byte boundary) - both
// TF32-rounded.  Two
// tcgen05 MMAs per 8-deep slice share the x operand [x_re; x_im]:
//     D1 += dy_re * [x_re; x_im]^T,   D2 += dy_im * [x_re; x_im]^T
// and the epilogue forms Re dW = D1[:, :CT] + D2[:, CT:],
// Im dW = D2[:, :CT] - D1[:, CT:].  The reduction is split over CTAs; the
// partial sums are added in split order by a second kernel (deterministic).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <mutex>

#include "ccv_internal.h"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

__device__ __forceinline__ float to_tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// ------------------------------------------------------------------ dgrad
// Packed image of one phase's dgrad filter: taps (u, v) of a TA x TB
// sub-filter, W'[c][k][u][v] = conj(W[k][c][ra + sh*(TA-1-u)][rb + sw*(TB-1-v)])
// (transposed, flipped, conjugated), in the forward's packed layout for the
// problem (K' = C, C' = K): [tap'][plane][C][K], plane 0 = -W'_im = W_im,
// 1 = W'_re = W_re, 2 = W'_im = -W_im (TF32-rounded; with `split`, the
// remainders follow as a second image).  Stride 1: one phase, TA = R, TB = S.
__global__ void ccv_prepack_dgrad_kernel(const float* __restrict__ wr,
                                         const float* __restrict__ wi, float* __restrict__ out,
                                         int K, int C, int R, int S, int krsc, int split, int TA,
                                         int TB, int ra, int rb, int sh, int sw) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const long long total = static_cast<long long>(TA) * TB * K * C;
  const long long image = total * 3;
  const long long ck = static_cast<long long>(C) * K;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    // Output order: tap', c (row), k (innermost).
    const int k = static_cast<int>(i % K);
    long long t = i / K;
    const int c = static_cast<int>(t % C);
    const int tap = static_cast<int>(t / C);
    const int r = ra + sh * (TA - 1 - tap / TB);
    const int s = rb + sw * (TB - 1 - tap % TB);
    const long long src = krsc ? ((static_cast<long long>(k) * R + r) * S + s) * C + c
                               : ((static_cast<long long>(k) * C + c) * R + r) * S + s;
    const float xr = wr[src];
    const float xi = wi[src];
    const float hr = to_tf32_rna(xr);
    const float hi = to_tf32_rna(xi);
    const long long o = static_cast<long long>(tap) * 3 * ck + static_cast<long long>(c) * K + k;
    out[o] = hi;
    out[o + ck] = hr;
    out[o + 2 * ck] = -hi;
    if (split) {
      const float lr = to_tf32_rna(xr - hr);
      const float li = to_tf32_rna(xi - hi);
      out[image + o] = li;
      out[image + o + ck] = lr;
      out[image + o + 2 * ck] = -li;
    }
  }
}

// complex64 [planes][P][Q] -> complex64 [planes][Hp][Wp], element (i, j) =
// dy[i - oh][j - ow] (zero outside dy): the phase's zero border.
__global__ void ccv_dgrad_phase_pad_kernel(const float2* __restrict__ dy, float2* __restrict__ out,
                                           long long planes, int P, int Q, int Hp, int Wp,
                                           int oh, int ow) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  // One warp per output row: the row's plane and dy row are derived once,
  // the lanes copy along the row.
  const int lane = threadIdx.x & 31;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const long long rows = planes * Hp;
  for (long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       row < rows; row += nwarps) {
    const long long pl = row / Hp;
    const int p = static_cast<int>(row - pl * Hp) - oh;
    float2* dst = out + row * Wp;
    if (p < 0 || p >= P) {
      for (int j = lane; j < Wp; j += 32) dst[j] = make_float2(0.f, 0.f);
      continue;
    }
    const float2* src = dy + (pl * P + p) * Q;
    for (int j = lane; j < Wp; j += 32) {
      const int q = j - ow;
      dst[j] = (q >= 0 && q < Q) ? __ldg(src + q) : make_float2(0.f, 0.f);
    }
  }
}

// dx[n][c][h][w] = phase (h % sh, w % sw)'s output at (h / sh, w / sw), or 0
// for a phase no filter tap reaches.  Phase outputs are [N][C][Ha][Wb]
// complex64 blocks, back to back in (a, b) order at `phase_off` (elements).
struct DgradPhaseTable {
  long long off[64];
  int ha[8], wb[8];
  int live[64];
};
__global__ void ccv_dgrad_interleave_kernel(const float2* __restrict__ phases,
                                            float2* __restrict__ dx, long long planes, int H,
                                            int W, int sh, int sw,
                                            const __grid_constant__ DgradPhaseTable tab) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  // One warp per dx row: the row's plane and phase row are derived once,
  // the lanes fill the row column by column.
  const int lane = threadIdx.x & 31;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  const long long rows = planes * H;
  for (long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       row < rows; row += nwarps) {
    const long long pl = row / H;
    const int h = static_cast<int>(row - pl * H);
    const int a = h % sh, hh = h / sh;
    const long long prow = pl * tab.ha[a] + hh;
    float2* dst = dx + row * W;
    for (int w = lane; w < W; w += 32) {
      const int b = w % sw;
      const int ph = a * sw + b;
      float2 v = make_float2(0.f, 0.f);
      if (tab.live[ph]) v = phases[tab.off[ph] + prow * tab.wb[b] + w / sw];
      dst[w] = v;
    }
  }
}

}  // namespace

DgradAxis dgrad_axis(int a, int stride, int pad, int taps, int in_size) {
  DgradAxis x;
  x.first = (a + pad) % stride;
  x.taps = x.first < taps ? (taps - x.first + stride - 1) / stride : 0;
  const int d = (a + pad - x.first) / stride;  // dy index offset of the phase's first tap
  x.offset = x.taps - 1 - d;
  x.out = a < in_size ? (in_size - a + stride - 1) / stride : 0;
  return x;
}

int launch_prepack_dgrad(const float* w_real, const float* w_imag, int layout, const Problem& pb,
                         int precision, float* packed, cudaStream_t stream) {
  const int split = precision == CCV_PRECISION_3XTF32 ? 1 : 0;
  const int block = 256;
  float* out = packed;
  for (int a = 0; a < pb.sh; ++a) {
    const DgradAxis ya = dgrad_axis(a, pb.sh, pb.ph, pb.r, pb.h);
    for (int b = 0; b < pb.sw; ++b) {
      const DgradAxis xb = dgrad_axis(b, pb.sw, pb.pw, pb.s, pb.w);
      const long long total = static_cast<long long>(ya.taps) * xb.taps * pb.k * pb.c;
      if (total == 0) continue;
      const int grid = static_cast<int>(std::min<long long>((total + block - 1) / block, 4096));
      const cudaError_t e =
          launch_kernel(ccv_prepack_dgrad_kernel, dim3(grid), dim3(block), 0, stream, 1, w_real,
                        w_imag, out, pb.k, pb.c, pb.r, pb.s, layout == CCV_WEIGHT_KRSC ? 1 : 0,
                        split, ya.taps, xb.taps, ya.first, xb.first, pb.sh, pb.sw);
      if (e != cudaSuccess) return cuda_error(e, "dgrad weight prepack launch");
      out += total * 3 * (split ? 2 : 1);
    }
  }
  return CCV_OK;
}

int launch_dgrad_phase_pad(const void* dy, void* out, const Problem& pb, int hp, int wp, int oh,
                           int ow, cudaStream_t stream) {
  const long long planes = static_cast<long long>(pb.n) * pb.k;
  const long long rows = planes * hp;  // one warp per row
  const int block = 256;
  const int grid = static_cast<int>(std::min<long long>((rows * 32 + block - 1) / block, 148 * 16));
  const cudaError_t e =
      launch_kernel(ccv_dgrad_phase_pad_kernel, dim3(grid), dim3(block), 0, stream, 1,
                    static_cast<const float2*>(dy), static_cast<float2*>(out), planes, pb.p, pb.q,
                    hp, wp, oh, ow);
  return e == cudaSuccess ? CCV_OK : cuda_error(e, "dgrad phase copy launch");
}

int launch_dgrad_interleave(const void* phases, void* dx, const Problem& pb, cudaStream_t stream) {
  DgradPhaseTable tab;
  memset(&tab, 0, sizeof(tab));
  long long off = 0;
  for (int a = 0; a < pb.sh; ++a) {
    const DgradAxis ya = dgrad_axis(a, pb.sh, pb.ph, pb.r, pb.h);
    tab.ha[a] = ya.out;
    for (int b = 0; b < pb.sw; ++b) {
      const DgradAxis xb = dgrad_axis(b, pb.sw, pb.pw, pb.s, pb.w);
      tab.wb[b] = xb.out;
      const int ph = a * pb.sw + b;
      tab.off[ph] = off;
      tab.live[ph] = ya.taps > 0 && xb.taps > 0 && ya.out > 0 && xb.out > 0;
      off += static_cast<long long>(pb.n) * pb.c * ya.out * xb.out;
    }
  }
  const long long planes = static_cast<long long>(pb.n) * pb.c;
  const long long rows = planes * pb.h;  // one warp per row
  const int block = 256;
  const int grid = static_cast<int>(std::min<long long>((rows * 32 + block - 1) / block, 148 * 16));
  const cudaError_t e = launch_kernel(ccv_dgrad_interleave_kernel, dim3(grid), dim3(block), 0,
                                      stream, 1, static_cast<const float2*>(phases),
                                      static_cast<float2*>(dx), planes, pb.h, pb.w, pb.sh, pb.sw,
                                      tab);
  return e == cudaSuccess ? CCV_OK : cuda_error(e, "dgrad interleave launch");
}

// Planar (forward_planar) data gradient: the same phases on fp32 NHWC planes.
namespace {

// fp32 planes [N][P][Q][K] -> [N][Hp][Wp][K]: pixel (i, j) = dy[i - oh][j - ow]
// (zero outside dy); 4 channels per thread.
__global__ void ccv_dgrad_phase_pad_planar_kernel(const float4* __restrict__ yr,
                                                  const float4* __restrict__ yi,
                                                  float4* __restrict__ outr,
                                                  float4* __restrict__ outi, long long n, int P,
                                                  int Q, int K4, int Hp, int Wp, int oh, int ow) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const long long total = n * Hp * Wp * K4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int k4 = static_cast<int>(i % K4);
    long long t = i / K4;
    const int j = static_cast<int>(t % Wp);
    t /= Wp;
    const int r = static_cast<int>(t % Hp);
    const long long img = t / Hp;
    const int p = r - oh, q = j - ow;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f), b = a;
    if (p >= 0 && p < P && q >= 0 && q < Q) {
      const long long src = ((img * P + p) * Q + q) * K4 + k4;
      a = yr[src];
      b = yi[src];
    }
    outr[i] = a;
    outi[i] = b;
  }
}

// dx planes [N][H][W][C] from the phases' planar outputs ([N][Ha][Wb][C] per
// phase and plane: for each phase its real block, then its imaginary block,
// in (a, b) order at `tab.off`, counted in float4).
__global__ void ccv_dgrad_interleave_planar_kernel(const float4* __restrict__ phases,
                                                   float4* __restrict__ dxr,
                                                   float4* __restrict__ dxi, long long n, int H,
                                                   int W, int C4, int sh, int sw,
                                                   const __grid_constant__ DgradPhaseTable tab) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const long long total = n * H * W * C4;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c4 = static_cast<int>(i % C4);
    long long t = i / C4;
    const int w = static_cast<int>(t % W);
    t /= W;
    const int h = static_cast<int>(t % H);
    const long long img = t / H;
    const int a = h % sh, b = w % sw;
    const int ph = a * sw + b;
    float4 vr = make_float4(0.f, 0.f, 0.f, 0.f), vi = vr;
    if (tab.live[ph]) {
      const int ha = tab.ha[a], wb = tab.wb[b];
      const long long plane = n * ha * wb * C4;
      const long long e = ((img * ha + h / sh) * wb + w / sw) * C4 + c4;
      vr = phases[tab.off[ph] + e];
      vi = phases[tab.off[ph] + plane + e];
    }
    dxr[i] = vr;
    dxi[i] = vi;
  }
}

}  // namespace

int launch_dgrad_phase_pad_planar(const float* dy_r, const float* dy_i, float* out_r,
                                  float* out_i, const Problem& pb, int hp, int wp, int oh, int ow,
                                  cudaStream_t stream) {
  const long long total = static_cast<long long>(pb.n) * hp * wp * (pb.k / 4);
  const int block = 256;
  const int grid = static_cast<int>(std::min<long long>((total + block - 1) / block, 148 * 16));
  const cudaError_t e = launch_kernel(
      ccv_dgrad_phase_pad_planar_kernel, dim3(grid), dim3(block), 0, stream, 1,
      reinterpret_cast<const float4*>(dy_r), reinterpret_cast<const float4*>(dy_i),
      reinterpret_cast<float4*>(out_r), reinterpret_cast<float4*>(out_i),
      static_cast<long long>(pb.n), pb.p, pb.q, pb.k / 4, hp, wp, oh, ow);
  return e == cudaSuccess ? CCV_OK : cuda_error(e, "dgrad planar phase copy launch");
}

int launch_dgrad_interleave_planar(const float* phases, float* dx_r, float* dx_i, const Problem& pb,
                                   cudaStream_t stream) {
  DgradPhaseTable tab;
  memset(&tab, 0, sizeof(tab));
  long long off = 0;  // float4
  for (int a = 0; a < pb.sh; ++a) {
    const DgradAxis ya = dgrad_axis(a, pb.sh, pb.ph, pb.r, pb.h);
    tab.ha[a] = ya.out;
    for (int b = 0; b < pb.sw; ++b) {
      const DgradAxis xb = dgrad_axis(b, pb.sw, pb.pw, pb.s, pb.w);
      tab.wb[b] = xb.out;
      const int ph = a * pb.sw + b;
      tab.off[ph] = off;
      tab.live[ph] = ya.taps > 0 && xb.taps > 0 && ya.out > 0 && xb.out > 0;
      off += 2LL * pb.n * ya.out * xb.out * (pb.c / 4);
    }
  }
  const long long total = static_cast<long long>(pb.n) * pb.h * pb.w * (pb.c / 4);
  const int block = 256;
  const int grid = static_cast<int>(std::min<long long>((total + block - 1) / block, 148 * 16));
  const cudaError_t e = launch_kernel(
      ccv_dgrad_interleave_planar_kernel, dim3(grid), dim3(block), 0, stream, 1,
      reinterpret_cast<const float4*>(phases), reinterpret_cast<float4*>(dx_r),
      reinterpret_cast<float4*>(dx_i), static_cast<long long>(pb.n), pb.h, pb.w, pb.c / 4, pb.sh,
      pb.sw, tab);
  return e == cudaSuccess ? CCV_OK : cuda_error(e, "dgrad planar interleave launch");
}

// ------------------------------------------------------------------ wgrad
namespace {

constexpr int kWgThreads = 192;
constexpr int kWgRowBytes = 128;  // one K-major operand row: 32 fp32 (32 pixels)
constexpr int kWgM = 128;         // output channels per tile (MMA M)

template <int CT>
struct WgCfg {
  static constexpr int kABytes = kWgM * kWgRowBytes;  // one dy plane per stage
  static constexpr int kBBytes = CT * kWgRowBytes;    // one x plane per stage
  static constexpr int kStageBytes = 2 * kABytes + 2 * kBBytes;
  static constexpr int kStages = (192 * 1024) / kStageBytes;  // 3 / 4 / 5 for CT 128 / 64 / 32
  static_assert(kStages >= 2, "pipeline too shallow");
  static constexpr int kTmemCols = 4 * CT;  // D1 | D2, 2*CT columns each
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;
};

struct WgradParams {
  CUtensorMap tm_dyr, tm_dyi;  // fp32 [N][K][P][Q] planes: dims (Q, P, K, N)
  CUtensorMap tm_xr, tm_xi;    // fp32 [S][N][C][H][Q] planes: dims (Q, H, C, N, S)
  float* partial;              // [tile][split][128][2*CT] or null (splits == 1)
  float* dw_r;
  float* dw_i;
  int* status;
  int k, c, r, s, sh, sw, ph, pw, p, q;
  int tiles_c, splits, qblocks;
  long long steps;  // reduction steps of a tile: N * P * qblocks
};

// Complex64 [rows][Q] -> TF32-rounded fp32 planes [rows][Qa] (rows = N*K*P).
// One warp per row, lanes along q (32-bit index math inside a row).
__global__ void ccv_wgrad_dy_planes_kernel(const float2* __restrict__ dy, float* __restrict__ yr,
                                           float* __restrict__ yi, long long rows, int Q,
                                           int Qa) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const int lane = threadIdx.x & 31;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       row < rows; row += nwarps) {
    const float2* src = dy + row * Q;
    float* dr = yr + row * Qa;
    float* di = yi + row * Qa;
    for (int q = lane; q < Q; q += 32) {
      const float2 v = __ldg(src + q);
      dr[q] = to_tf32_rna(v.x);
      di[q] = to_tf32_rna(v.y);
    }
  }
}

// Complex64 NCHW -> TF32-rounded fp32 planes [S][N][C][H][Qa], element
// (s, .., q) = x[.., w = q*sw - pw + s] (0 outside the image), for q < Q.
// One warp per input row (n, c, h): the row is read once from DRAM (the S
// shifted copies re-read it from L1) and each copy is written with
// consecutive lanes on consecutive q.
__global__ void ccv_wgrad_x_planes_kernel(const float2* __restrict__ x, float* __restrict__ xr,
                                          float* __restrict__ xi, long long rows, int W, int S,
                                          int Q, int Qa, int sw, int pw) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  // One warp per input row; a lane writes two adjacent output columns per
  // pass as one 8-byte store (64 columns per warp pass; Qa is a multiple of
  // 4, so every pair starts 8-byte aligned).  Columns Q..Qa-1 get zeros
  // (the weight-gradient kernel's tensor map ends at Q, so they are never
  // read).
  const int lane = threadIdx.x & 31;
  const long long nwarps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long row = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       row < rows; row += nwarps) {
    const float2* src = x + row * W;
    for (int q = 2 * lane; q < Qa; q += 64) {
#pragma unroll 1
      for (int s = 0; s < S; ++s) {
        const int w0 = q * sw - pw + s;
        const int w1 = w0 + sw;
        const float2 v0 = (q < Q && w0 >= 0 && w0 < W) ? __ldg(src + w0) : make_float2(0.f, 0.f);
        const float2 v1 =
            (q + 1 < Q && w1 >= 0 && w1 < W) ? __ldg(src + w1) : make_float2(0.f, 0.f);
        const long long o = (static_cast<long long>(s) * rows + row) * Qa + q;
        *reinterpret_cast<float2*>(xr + o) = make_float2(to_tf32_rna(v0.x), to_tf32_rna(v1.x));
        *reinterpret_cast<float2*>(xi + o) = make_float2(to_tf32_rna(v0.y), to_tf32_rna(v1.y));
      }
    }
  }
}

// fp32 planes [N][R][Win][Cn] (channels innermost: NHWC x, NPQK dy) ->
// TF32-rounded planes [S][N][Cn][R][Qa], element (s, n, c, r, q) =
// src[n][r][q*sw - pw + s][c] (0 outside 0..Win-1), for q < Q - the layout
// the weight-gradient kernel reads, from planar inputs.  One block per
// (row r, n, s) and tile of 32 columns x 32 channels, through shared memory:
// loads coalesced along c, stores along q.
__global__ void __launch_bounds__(256) ccv_wgrad_planar_transpose_kernel(
    const float* __restrict__ sr, const float* __restrict__ si, float* __restrict__ dr,
    float* __restrict__ di, int N, int R, int Win, int Cn, int Q, int Qa, int S, int sw, int pw) {
  __shared__ float tr[32][33];
  __shared__ float ti[32][33];
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const int qt = (Q + 31) / 32;
  const int q0 = (blockIdx.x % qt) * 32;
  const int c0 = (blockIdx.x / qt) * 32;
  const int r = blockIdx.y;
  const int n = blockIdx.z / S;
  const int s = blockIdx.z - n * S;
  const int tx = threadIdx.x, ty = threadIdx.y;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ql = ty + 8 * i;
    const int q = q0 + ql;
    const int w = q * sw - pw + s;
    const int c = c0 + tx;
    float a = 0.f, b = 0.f;
    if (q < Q && w >= 0 && w < Win && c < Cn) {
      const long long src = ((static_cast<long long>(n) * R + r) * Win + w) * Cn + c;
      a = __ldg(sr + src);
      b = __ldg(si + src);
    }
    tr[ql][tx] = a;
    ti[ql][tx] = b;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = c0 + ty + 8 * i;
    const int q = q0 + tx;
    if (c < Cn && q < Q) {
      const long long o =
          (((static_cast<long long>(s) * N + n) * Cn + c) * R + r) * Qa + q;
      dr[o] = to_tf32_rna(tr[tx][ty + 8 * i]);
      di[o] = to_tf32_rna(ti[tx][ty + 8 * i]);
    }
  }
}

__device__ __forceinline__ float4 f4(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return make_float4(__uint_as_float(a), __uint_as_float(b), __uint_as_float(c),
                     __uint_as_float(d));
}

// One CTA: tile (k block, c block, tap) x split (a contiguous range of its
// reduction steps).  Warps: 0 TMA producer, 1 TMEM allocation + MMA issue,
// 2..5 epilogue (one output channel k per thread).
template <int CT>
__global__ void __launch_bounds__(kWgThreads, 1)
    ccv_wgrad_tf32_kernel(const __grid_constant__ WgradParams prm) {
  using Cf = WgCfg<CT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cf::kBarOffset);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * Cf::kStages + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] skip, [1] abort

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t smem_base = ptx::smem_u32(smem);
  const uint32_t bar_base = ptx::smem_u32(bars);
  auto full_bar = [&](int i) { return bar_base + 8u * i; };
  auto empty_bar = [&](int i) { return bar_base + 8u * (Cf::kStages + i); };
  const uint32_t acc_bar = bar_base + 8u * (2 * Cf::kStages);

  const int splits = prm.splits;
  const int tile = blockIdx.x / splits;
  const int split = blockIdx.x - tile * splits;
  const int rs = prm.r * prm.s;
  const int tap = tile % rs;
  const int rest = tile / rs;
  const int ct = rest % prm.tiles_c;
  const int kt = rest / prm.tiles_c;
  const int rr = tap / prm.s;
  const int ss = tap - rr * prm.s;
  const long long b0 = static_cast<long long>(split) * prm.steps / splits;
  const long long b1 = static_cast<long long>(split + 1) * prm.steps / splits;

  if (threadIdx.x == 0) {
    flags[1] = 0;
    for (int i = 0; i < Cf::kStages; ++i) {
      ptx::mbar_init(full_bar(i), 1);
      ptx::mbar_init(empty_bar(i), 1);
    }
    ptx::mbar_init(acc_bar, 1);
    ptx::fence_mbar_init();
    ptx::prefetch_tmap(&prm.tm_dyr);
    ptx::prefetch_tmap(&prm.tm_dyi);
    ptx::prefetch_tmap(&prm.tm_xr);
    ptx::prefetch_tmap(&prm.tm_xi);
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), Cf::kTmemCols);
    ptx::tmem_relinquish();
  }
  if (threadIdx.x == 0) flags[0] = *reinterpret_cast<volatile int*>(prm.status) != 0 ? 1 : 0;
  ptx::tc_fence_before();
  ptx::cta_sync();
  ptx::tc_fence_after();
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_holder;
  const bool skip = flags[0] != 0 || b1 <= b0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      for (long long t = b0; t < b1; ++t) {
        if (!ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, prm.status,
                                    CCV_ERR_DEVICE_TIMEOUT)) {
          flags[1] = 1;
          break;
        }
        if (flags[1]) break;
        const uint32_t fb = full_bar(stage);
        ptx::mbar_arrive_expect_tx(fb, Cf::kStageBytes);
        const int qb = static_cast<int>(t % prm.qblocks);
        const long long pr = t / prm.qblocks;
        const int pp = static_cast<int>(pr % prm.p);
        const int nn = static_cast<int>(pr / prm.p);
        const uint32_t a_r = smem_base + stage * Cf::kStageBytes;
        const uint32_t a_i = a_r + Cf::kABytes;
        const uint32_t b_r = a_i + Cf::kABytes;
        const uint32_t b_i = b_r + Cf::kBBytes;
        // dy rows k of output row pp, columns 32*qb.. (zero past Q and K).
        ptx::tma_load_4d(a_r, &prm.tm_dyr, fb, qb * 32, pp, kt * kWgM, nn);
        ptx::tma_load_4d(a_i, &prm.tm_dyi, fb, qb * 32, pp, kt * kWgM, nn);
        // x rows c of input row pp*sh - ph + rr (zero outside the image:
        // the padding), the columns filter column ss reads for output
        // columns 32*qb..
        const int hh = pp * prm.sh - prm.ph + rr;
        ptx::tma_load_5d(b_r, &prm.tm_xr, fb, qb * 32, hh, ct * CT, nn, ss);
        ptx::tma_load_5d(b_i, &prm.tm_xi, fb, qb * 32, hh, ct * CT, nn, ss);
        ++issued;
        if (++stage == Cf::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // No TMA write may be in flight into this CTA's shared memory when it
      // exits (matters only after an abort).
      for (int j = 0; j < Cf::kStages && j < issued; ++j) {
        const long long u = issued - 1 - j;
        ptx::mbar_wait_bounded(full_bar(static_cast<int>(u % Cf::kStages)),
                               static_cast<uint32_t>((u / Cf::kStages) & 1), prm.status,
                               CCV_ERR_DEVICE_TIMEOUT);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && !skip) {
      constexpr uint32_t idesc = ptx::idesc_tf32(kWgM, 2 * CT, false);
      int stage = 0;
      uint32_t phase = 0;
      for (long long t = b0; t < b1; ++t) {
        if (!ptx::mbar_wait_bounded(full_bar(stage), phase, prm.status, CCV_ERR_DEVICE_TIMEOUT)) {
          flags[1] = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t a_r = smem_base + stage * Cf::kStageBytes;
        const uint32_t a_i = a_r + Cf::kABytes;
        const uint32_t b_r = a_i + Cf::kABytes;  // [x_re; x_im]: 2*CT rows
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint32_t koff = kk * 32;
          const uint64_t da_r = ptx::desc_kmajor_sw128(a_r + koff);
          const uint64_t da_i = ptx::desc_kmajor_sw128(a_i + koff);
          const uint64_t db = ptx::desc_kmajor_sw128(b_r + koff);
          const uint32_t acc = (t != b0 || kk != 0) ? 1u : 0u;
          ptx::mma_tf32_ss(tmem_base, da_r, db, idesc, acc);           // D1
          ptx::mma_tf32_ss(tmem_base + 2 * CT, da_i, db, idesc, acc);  // D2
        }
        ptx::mma_commit(empty_bar(stage));
        if (++stage == Cf::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      ptx::mma_commit(acc_bar);
      ptx::mbar_wait_bounded(acc_bar, 0, prm.status, CCV_ERR_DEVICE_TIMEOUT);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const int k = kt * kWgM + row;
    bool ok = false;
    if (!skip) {
      ok = ptx::mbar_wait_bounded_backoff(acc_bar, 0, prm.status, CCV_ERR_DEVICE_TIMEOUT);
      ptx::tc_fence_after();
    }
    if (flags[1]) ok = false;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    float* part = prm.partial != nullptr
                      ? prm.partial + ((static_cast<long long>(tile) * splits + split) * kWgM +
                                       row) * (2 * CT)
                      : nullptr;
#pragma unroll 1
    for (int c16 = 0; c16 < CT; c16 += 16) {
      uint32_t a[16], b[16], e[16], f[16];
      if (ok) {
        ptx::tmem_ld_32x32b_x16(t_row + c16, a);               // dy_re * x_re
        ptx::tmem_ld_32x32b_x16(t_row + CT + c16, b);          // dy_re * x_im
        ptx::tmem_ld_32x32b_x16(t_row + 2 * CT + c16, e);      // dy_im * x_re
        ptx::tmem_ld_32x32b_x16(t_row + 3 * CT + c16, f);      // dy_im * x_im
        ptx::tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j) a[j] = b[j] = e[j] = f[j] = 0u;
      }
      uint32_t re[16], im[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        re[j] = __float_as_uint(__uint_as_float(a[j]) + __uint_as_float(f[j]));
        im[j] = __float_as_uint(__uint_as_float(e[j]) - __uint_as_float(b[j]));
      }
      if (part != nullptr) {
        // A split CTA writes its partial even when it has no steps (zeros),
        // so the reduction reads defined values.
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          *reinterpret_cast<float4*>(part + c16 + j) = f4(re[j], re[j + 1], re[j + 2], re[j + 3]);
          *reinterpret_cast<float4*>(part + CT + c16 + j) =
              f4(im[j], im[j + 1], im[j + 2], im[j + 3]);
        }
      } else if (ok && k < prm.k) {
        const long long base = static_cast<long long>(k) * prm.c;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int c = ct * CT + c16 + j;
          if (c < prm.c) {
            const long long o = (base + c) * rs + tap;
            prm.dw_r[o] = __uint_as_float(re[j]);
            prm.dw_i[o] = __uint_as_float(im[j]);
          }
        }
      }
    }
    ptx::tc_fence_before();
  }
  ptx::cta_sync();
  if (warp == 1) {
    __syncwarp();  // tcgen05.dealloc is warp-collective
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, Cf::kTmemCols);
  }
}

// Sums the splits' partials of every tile in split order and scatters the
// result to dW (KCRS planes).  One thread per (tile, row, 4 channels).
__global__ void ccv_wgrad_reduce_kernel(const float* __restrict__ partial, float* __restrict__ dw_r,
                                        float* __restrict__ dw_i, int tiles, int splits, int ct_w,
                                        int tiles_c, int K, int C, int RS) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const int groups = ct_w / 4;
  const long long total = static_cast<long long>(tiles) * kWgM * groups;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int g = static_cast<int>(i % groups);
    long long t = i / groups;
    const int row = static_cast<int>(t % kWgM);
    const int tile = static_cast<int>(t / kWgM);
    float4 sr = make_float4(0.f, 0.f, 0.f, 0.f), si = sr;
    for (int sp = 0; sp < splits; ++sp) {
      const float* p =
          partial + ((static_cast<long long>(tile) * splits + sp) * kWgM + row) * (2 * ct_w);
      const float4 a = *reinterpret_cast<const float4*>(p + 4 * g);
      const float4 b = *reinterpret_cast<const float4*>(p + ct_w + 4 * g);
      sr.x += a.x; sr.y += a.y; sr.z += a.z; sr.w += a.w;
      si.x += b.x; si.y += b.y; si.z += b.z; si.w += b.w;
    }
    const int tap = tile % RS;
    const int rest = tile / RS;
    const int ct = rest % tiles_c;
    const int kt = rest / tiles_c;
    const int k = kt * kWgM + row;
    if (k >= K) continue;
    const float vr[4] = {sr.x, sr.y, sr.z, sr.w};
    const float vi[4] = {si.x, si.y, si.z, si.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int c = ct * ct_w + 4 * g + j;
      if (c < C) {
        const long long o = (static_cast<long long>(k) * C + c) * RS + tap;
        dw_r[o] = vr[j];
        dw_i[o] = vi[j];
      }
    }
  }
}

}  // namespace

// ------------------------------------------------------------ wgrad host side
namespace {

size_t align256b(size_t b) { return (b + 255) & ~static_cast<size_t>(255); }

struct WgradPlan {
  int ct = 128;
  int tiles_c = 1, tiles = 1, splits = 1, qblocks = 1, qa = 4;
  long long steps = 1;
  size_t dy_plane = 0, x_plane = 0, partial = 0;
};

// Channel tile CT (N = 2*CT), tiles (k block, c block, tap) and the split of
// each tile's reduction: about one CTA per SM in total, each split a
// contiguous range of (n, p, 32-column block) steps.
WgradPlan plan_wgrad(const Problem& pb) {
  WgradPlan w;
  w.ct = pb.c > 64 ? 128 : (pb.c > 32 ? 64 : 32);
  w.tiles_c = (pb.c + w.ct - 1) / w.ct;
  const int tiles_k = (pb.k + kWgM - 1) / kWgM;
  w.tiles = tiles_k * w.tiles_c * pb.r * pb.s;
  w.qblocks = (pb.q + 31) / 32;
  w.steps = static_cast<long long>(pb.n) * pb.p * w.qblocks;
  const int sms = device_sm_count();
  w.splits = static_cast<int>(std::max<long long>(1, std::min<long long>(w.steps, sms / w.tiles)));
  w.qa = (pb.q + 3) & ~3;
  w.dy_plane = align256b(static_cast<size_t>(pb.n) * pb.k * pb.p * w.qa * 4);
  w.x_plane = align256b(static_cast<size_t>(pb.s) * pb.n * pb.c * pb.h * w.qa * 4);
  w.partial = w.splits > 1
                  ? align256b(static_cast<size_t>(w.tiles) * w.splits * kWgM * 2 * w.ct * 4)
                  : 0;
  return w;
}

template <int CT>
cudaError_t prepare_wgrad_variant() {
  static std::once_flag once[64];
  static cudaError_t err[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  const int slot = dev & 63;
  std::call_once(once[slot], [&]() {
    err[slot] = cudaFuncSetAttribute(ccv_wgrad_tf32_kernel<CT>,
                                     cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     WgCfg<CT>::kSmemBytes);
  });
  return err[slot];
}

template <int CT>
int launch_wgrad_kernel(const WgradParams& prm, int ctas, cudaStream_t stream) {
  cudaError_t e = prepare_wgrad_variant<CT>();
  if (e == cudaSuccess) {
    e = launch_kernel(ccv_wgrad_tf32_kernel<CT>, dim3(ctas), dim3(kWgThreads),
                      WgCfg<CT>::kSmemBytes, stream, 1, prm);
  }
  return e == cudaSuccess ? CCV_OK : cuda_error(e, "wgrad kernel launch");
}

}  // namespace

size_t wgrad_workspace_bytes(const Problem& pb) {
  const WgradPlan w = plan_wgrad(pb);
  return 2 * w.dy_plane + 2 * w.x_plane + w.partial;
}

int launch_wgrad(const WgradSource& src, float* dw_r, float* dw_i, const Problem& pb, void* ws,
                 cudaStream_t stream) {
  const WgradPlan w = plan_wgrad(pb);
  char* base = static_cast<char*>(ws);
  float* dyr = reinterpret_cast<float*>(base);
  float* dyi = reinterpret_cast<float*>(base + w.dy_plane);
  float* xr = reinterpret_cast<float*>(base + 2 * w.dy_plane);
  float* xi = reinterpret_cast<float*>(base + 2 * w.dy_plane + w.x_plane);
  float* partial = w.splits > 1
                       ? reinterpret_cast<float*>(base + 2 * w.dy_plane + 2 * w.x_plane)
                       : nullptr;
  const int block = 256;
  const int sms = device_sm_count();
  if (src.x_real != nullptr) {
    // Planar inputs: dy NPQK and x NHWC planes, transposed through shared memory.
    if (pb.n > 65535 / pb.s || pb.p > 65535 || pb.h > 65535) {
      return set_error(CCV_ERR_UNSUPPORTED, "problem too large for the planar weight gradient");
    }
    const int qt = (pb.q + 31) / 32;
    cudaError_t e = launch_kernel(
        ccv_wgrad_planar_transpose_kernel,
        dim3(static_cast<unsigned>(qt * ((pb.k + 31) / 32)), pb.p, pb.n), dim3(32, 8), 0, stream,
        1, src.dy_real, src.dy_imag, dyr, dyi, pb.n, pb.p, pb.q, pb.k, pb.q, w.qa, 1, 1, 0);
    if (e != cudaSuccess) return cuda_error(e, "wgrad planar dy layout launch");
    e = launch_kernel(ccv_wgrad_planar_transpose_kernel,
                      dim3(static_cast<unsigned>(qt * ((pb.c + 31) / 32)), pb.h, pb.n * pb.s),
                      dim3(32, 8), 0, stream, 1, src.x_real, src.x_imag, xr, xi, pb.n, pb.h, pb.w,
                      pb.c, pb.q, w.qa, pb.s, pb.sw, pb.pw);
    if (e != cudaSuccess) return cuda_error(e, "wgrad planar x layout launch");
  } else {
    // Complex64 inputs: dy NKPQ and x NCHW, one warp per row.
    const long long dy_rows = static_cast<long long>(pb.n) * pb.k * pb.p;
    int grid = static_cast<int>(std::min<long long>((dy_rows * 32 + block - 1) / block, sms * 16LL));
    cudaError_t e =
        launch_kernel(ccv_wgrad_dy_planes_kernel, dim3(grid), dim3(block), 0, stream, 1,
                      static_cast<const float2*>(src.dy), dyr, dyi, dy_rows, pb.q, w.qa);
    if (e != cudaSuccess) return cuda_error(e, "wgrad dy layout launch");
    const long long x_rows = static_cast<long long>(pb.n) * pb.c * pb.h;
    grid = static_cast<int>(std::min<long long>((x_rows * 32 + block - 1) / block, sms * 16LL));
    e = launch_kernel(ccv_wgrad_x_planes_kernel, dim3(grid), dim3(block), 0, stream, 1,
                      static_cast<const float2*>(src.x), xr, xi, x_rows, pb.w, pb.s, pb.q, w.qa,
                      pb.sw, pb.pw);
    if (e != cudaSuccess) return cuda_error(e, "wgrad x layout launch");
  }
  WgradParams prm;
  memset(&prm, 0, sizeof(prm));
  int rc;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.q), static_cast<uint64_t>(pb.p),
                              static_cast<uint64_t>(pb.k), static_cast<uint64_t>(pb.n)};
    const uint64_t row = static_cast<uint64_t>(w.qa) * 4;
    const uint64_t strides[3] = {row, row * pb.p, row * pb.p * pb.k};
    const uint32_t box[4] = {32, 1, kWgM, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled_ex(&prm.tm_dyr, dyr, 4, dims, strides, box, es, kSwizzle128, false)) !=
            CCV_OK ||
        (rc = encode_tiled_ex(&prm.tm_dyi, dyi, 4, dims, strides, box, es, kSwizzle128, false)) !=
            CCV_OK) {
      return rc;
    }
  }
  {
    const uint64_t dims[5] = {static_cast<uint64_t>(pb.q), static_cast<uint64_t>(pb.h),
                              static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.n),
                              static_cast<uint64_t>(pb.s)};
    const uint64_t row = static_cast<uint64_t>(w.qa) * 4;
    const uint64_t strides[4] = {row, row * pb.h, row * pb.h * pb.c, row * pb.h * pb.c * pb.n};
    const uint32_t box[5] = {32, 1, static_cast<uint32_t>(w.ct), 1, 1};
    const uint32_t es[5] = {1, 1, 1, 1, 1};
    if ((rc = encode_tiled_ex(&prm.tm_xr, xr, 5, dims, strides, box, es, kSwizzle128, false)) !=
            CCV_OK ||
        (rc = encode_tiled_ex(&prm.tm_xi, xi, 5, dims, strides, box, es, kSwizzle128, false)) !=
            CCV_OK) {
      return rc;
    }
  }
  prm.partial = partial;
  prm.dw_r = dw_r;
  prm.dw_i = dw_i;
  prm.status = device_status_ptr();
  if (prm.status == nullptr) return CCV_ERR_CUDA;
  prm.k = pb.k; prm.c = pb.c; prm.r = pb.r; prm.s = pb.s;
  prm.sh = pb.sh; prm.sw = pb.sw; prm.ph = pb.ph; prm.pw = pb.pw;
  prm.p = pb.p; prm.q = pb.q;
  prm.tiles_c = w.tiles_c;
  prm.splits = w.splits;
  prm.qblocks = w.qblocks;
  prm.steps = w.steps;
  const int ctas = w.tiles * w.splits;
  switch (w.ct) {
    case 32: rc = launch_wgrad_kernel<32>(prm, ctas, stream); break;
    case 64: rc = launch_wgrad_kernel<64>(prm, ctas, stream); break;
    default: rc = launch_wgrad_kernel<128>(prm, ctas, stream); break;
  }
  if (rc != CCV_OK || w.splits == 1) return rc;
  const long long total = static_cast<long long>(w.tiles) * kWgM * (w.ct / 4);
  const int grid = static_cast<int>(std::min<long long>((total + block - 1) / block, sms * 16LL));
  const cudaError_t e = launch_kernel(ccv_wgrad_reduce_kernel, dim3(grid), dim3(block), 0, stream,
                                      1, static_cast<const float*>(partial), dw_r, dw_i, w.tiles,
                                      w.splits, w.ct, w.tiles_c, pb.k, pb.c, pb.r * pb.s);
  return e == cudaSuccess ? CCV_OK : cuda_error(e, "wgrad reduce launch");
}

}  // namespace ccv
