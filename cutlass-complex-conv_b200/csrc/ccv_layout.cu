// Layout kernels around the fprop kernel:
//   * weight prepack: KCRS or KRSC real/imag planes -> per-tap (-Wi, Wr, Wi)
//     planes of [K][C], TF32-rounded (and, for 3xTF32, the rounding
//     remainders as a second image).  Replaces the per-version KCRS->KRSC
//     copy of the reference module (modules.py:127-151).
//   * complex64 NCHW -> fp32 NHWC planes (the two permute+contiguous copies
//     of modules.py:198-199), used by the complex entry point.
#include <cuda_runtime.h>

#include <algorithm>

#include "ccv_internal.h"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

// Round-to-nearest (ties away from zero) conversion to TF32, kept in an fp32
// container with the 13 low mantissa bits cleared.
__device__ __forceinline__ float to_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// out image layout: [tap = r*S + s][plane][K][C], plane 0 = -Wi, 1 = Wr, 2 = Wi.
__global__ void ccv_prepack_kernel(const float* __restrict__ wr, const float* __restrict__ wi,
                                   float* __restrict__ out, int K, int C, int R, int S, int krsc,
                                   int split) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const long long total = static_cast<long long>(R) * S * K * C;
  const long long image = total * 3;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % C);
    long long t = i / C;
    const int k = static_cast<int>(t % K);
    const int tap = static_cast<int>(t / K);
    const int r = tap / S;
    const int s = tap - r * S;
    const long long src = krsc ? ((static_cast<long long>(k) * R + r) * S + s) * C + c
                               : ((static_cast<long long>(k) * C + c) * R + r) * S + s;
    const float xr = wr[src];
    const float xi = wi[src];
    const float hr = to_tf32(xr);
    const float hi = to_tf32(xi);
    const long long kc = static_cast<long long>(K) * C;
    const long long o = static_cast<long long>(tap) * 3 * kc + static_cast<long long>(k) * C + c;
    out[o] = -hi;
    out[o + kc] = hr;
    out[o + 2 * kc] = hi;
    if (split) {
      const float lr = to_tf32(xr - hr);
      const float li = to_tf32(xi - hi);
      out[image + o] = -li;
      out[image + o + kc] = lr;
      out[image + o + 2 * kc] = li;
    }
  }
}

// fp32 planes -> TF32-rounded parts and exact remainders (x - tf32(x)), the
// activation split of 3xTF32.
__global__ void ccv_split_planes_kernel(const float4* __restrict__ xr, const float4* __restrict__ xi,
                                        float4* __restrict__ hr, float4* __restrict__ hi,
                                        float4* __restrict__ lr, float4* __restrict__ li,
                                        long long count4) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = xr[i];
    const float4 b = xi[i];
    const float4 ah = make_float4(to_tf32(a.x), to_tf32(a.y), to_tf32(a.z), to_tf32(a.w));
    const float4 bh = make_float4(to_tf32(b.x), to_tf32(b.y), to_tf32(b.z), to_tf32(b.w));
    hr[i] = ah;
    hi[i] = bh;
    lr[i] = make_float4(a.x - ah.x, a.y - ah.y, a.z - ah.z, a.w - ah.w);
    li[i] = make_float4(b.x - bh.x, b.y - bh.y, b.z - bh.z, b.w - bh.w);
  }
}

// complex64 NCHW -> two fp32 NHWC planes.  One block per image and a
// 32-channel x 64-pixel tile of the image's H*W pixels taken as one row (a
// channel's pixels are contiguous in NCHW), so narrow images fill every
// tile: every thread issues its 8 loads (256-byte runs per warp) before
// touching shared memory, then writes 8 channel-contiguous runs (128 bytes
// per warp and plane).  With xr_lo/xi_lo set, writes tf32(x) and
// x - tf32(x) instead (3xTF32).
constexpr int kLayoutW = 64;

__global__ void __launch_bounds__(256) ccv_nchw_to_planar_kernel(
    const float2* __restrict__ x, float* __restrict__ xr, float* __restrict__ xi,
    float* __restrict__ xr_lo, float* __restrict__ xi_lo, int C, long long HW) {
  __shared__ float tr[32][kLayoutW + 1];
  __shared__ float ti[32][kLayoutW + 1];
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const long long n = blockIdx.z;
  const long long w0 = static_cast<long long>(blockIdx.x) * kLayoutW;  // first pixel of the tile
  const int c0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  float2 v[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int c = c0 + ty + 8 * (i & 3);
    const long long w = w0 + tx + 32 * (i >> 2);
    v[i] = (c < C && w < HW) ? __ldg(x + (n * C + c) * HW + w) : make_float2(0.f, 0.f);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int cl = ty + 8 * (i & 3);
    const int wl = tx + 32 * (i >> 2);
    tr[cl][wl] = v[i].x;
    ti[cl][wl] = v[i].y;
  }
  __syncthreads();
  const int c = c0 + tx;
  if (c >= C) return;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int wl = ty + 8 * i;
    const long long w = w0 + wl;
    if (w < HW) {
      const long long o = (n * HW + w) * C + c;
      const float a = tr[tx][wl];
      const float b = ti[tx][wl];
      if (xr_lo != nullptr) {
        const float ah = to_tf32(a);
        const float bh = to_tf32(b);
        xr[o] = ah;
        xi[o] = bh;
        xr_lo[o] = a - ah;
        xi_lo[o] = b - bh;
      } else {
        xr[o] = a;
        xi[o] = b;
      }
    }
  }
}

// Strided complex64 input (element strides sn, sc, sh, sw; any layout, e.g.
// a slice or a channels-last tensor) -> fp32 NHWC planes.  One thread per
// output element pair (two consecutive channels of one pixel): the stores
// are coalesced along C; the loads follow the input's layout.
__global__ void __launch_bounds__(256) ccv_strided_to_planar_kernel(
    const float2* __restrict__ x, float* __restrict__ xr, float* __restrict__ xi,
    float* __restrict__ xr_lo, float* __restrict__ xi_lo, int C, int H, int W, long long sn,
    long long sc, long long sh, long long sw, long long total2) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total2;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long o = 2 * i;  // NHWC element index of channel pair (c, c + 1)
    const int c = static_cast<int>(o % C);
    long long t = o / C;
    const int w = static_cast<int>(t % W);
    t /= W;
    const int h = static_cast<int>(t % H);
    const long long n = t / H;
    const long long a = n * sn + static_cast<long long>(c) * sc + h * sh + w * sw;
    const float2 v0 = __ldg(x + a);
    const float2 v1 = __ldg(x + a + sc);
    if (xr_lo != nullptr) {
      const float r0 = to_tf32(v0.x), r1 = to_tf32(v1.x), i0 = to_tf32(v0.y), i1 = to_tf32(v1.y);
      *reinterpret_cast<float2*>(xr + o) = make_float2(r0, r1);
      *reinterpret_cast<float2*>(xi + o) = make_float2(i0, i1);
      *reinterpret_cast<float2*>(xr_lo + o) = make_float2(v0.x - r0, v1.x - r1);
      *reinterpret_cast<float2*>(xi_lo + o) = make_float2(v0.y - i0, v1.y - i1);
    } else {
      *reinterpret_cast<float2*>(xr + o) = make_float2(v0.x, v1.x);
      *reinterpret_cast<float2*>(xi + o) = make_float2(v0.y, v1.y);
    }
  }
}

// Channels-last complex64 input (C innermost, dense NHWC): the planes are a
// plain de-interleave, four complex values per thread and step.
__global__ void __launch_bounds__(256) ccv_nhwc_complex_to_planar_kernel(
    const float4* __restrict__ x, float4* __restrict__ xr, float4* __restrict__ xi,
    float4* __restrict__ xr_lo, float4* __restrict__ xi_lo, long long count4) {
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < count4;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float4 a = __ldg(x + 2 * i);      // (re0, im0, re1, im1)
    const float4 b = __ldg(x + 2 * i + 1);  // (re2, im2, re3, im3)
    float4 r = make_float4(a.x, a.z, b.x, b.z);
    float4 m = make_float4(a.y, a.w, b.y, b.w);
    if (xr_lo != nullptr) {
      const float4 rh = make_float4(to_tf32(r.x), to_tf32(r.y), to_tf32(r.z), to_tf32(r.w));
      const float4 mh = make_float4(to_tf32(m.x), to_tf32(m.y), to_tf32(m.z), to_tf32(m.w));
      xr_lo[i] = make_float4(r.x - rh.x, r.y - rh.y, r.z - rh.z, r.w - rh.w);
      xi_lo[i] = make_float4(m.x - mh.x, m.y - mh.y, m.z - mh.z, m.w - mh.w);
      r = rh;
      m = mh;
    }
    xr[i] = r;
    xi[i] = m;
  }
}

}  // namespace

int launch_strided_complex_to_planar(const float* x, const int64_t* strides, float* xr,
                                     float* xi, float* xr_lo, float* xi_lo, const Problem& pb,
                                     cudaStream_t stream) {
  const long long C = pb.c, H = pb.h, W = pb.w;
  const long long sn = strides[0], sc = strides[1], sh = strides[2], sw = strides[3];
  if (sn == C * H * W && sc == H * W && sh == W && sw == 1) {
    return launch_nchw_complex_to_planar(x, xr, xi, xr_lo, xi_lo, pb, stream);
  }
  const long long total = static_cast<long long>(pb.n) * H * W * C;
  const int threads = 256;
  cudaError_t e;
  if (sc == 1 && sw == C && sh == W * C && sn == H * W * C &&
      (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const long long c4 = total / 4;  // C % 4 == 0
    const long long blocks = std::min<long long>((c4 + threads - 1) / threads, 148LL * 16);
    e = launch_kernel(ccv_nhwc_complex_to_planar_kernel, dim3(static_cast<unsigned>(blocks)),
                      dim3(threads), 0, stream, 0, reinterpret_cast<const float4*>(x),
                      reinterpret_cast<float4*>(xr), reinterpret_cast<float4*>(xi),
                      reinterpret_cast<float4*>(xr_lo), reinterpret_cast<float4*>(xi_lo), c4);
  } else {
    const long long t2 = total / 2;  // C % 4 == 0: channel pairs never straddle pixels
    const long long blocks = std::min<long long>((t2 + threads - 1) / threads, 148LL * 16);
    e = launch_kernel(ccv_strided_to_planar_kernel, dim3(static_cast<unsigned>(blocks)),
                      dim3(threads), 0, stream, 0, reinterpret_cast<const float2*>(x), xr, xi,
                      xr_lo, xi_lo, pb.c, pb.h, pb.w, sn, sc, sh, sw, t2);
  }
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "strided layout kernel launch");
  return CCV_OK;
}

int launch_prepack(const float* w_real, const float* w_imag, int layout, const Problem& pb,
                   int precision, float* packed, cudaStream_t stream) {
  const long long total = static_cast<long long>(pb.r) * pb.s * pb.k * pb.c;
  const int threads = 256;
  const long long blocks = std::min<long long>((total + threads - 1) / threads, 148LL * 16);
  cudaError_t e = launch_kernel(ccv_prepack_kernel, dim3(static_cast<unsigned>(blocks)),
                                dim3(threads), 0, stream, 0, w_real, w_imag, packed, pb.k, pb.c,
                                pb.r, pb.s, layout == CCV_WEIGHT_KRSC ? 1 : 0,
                                precision == CCV_PRECISION_3XTF32 ? 1 : 0);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "prepack kernel launch");
  return CCV_OK;
}

int launch_nchw_complex_to_planar(const float* x, float* xr, float* xi, float* xr_lo,
                                  float* xi_lo, const Problem& pb, cudaStream_t stream) {
  if (pb.n > 65535) return set_error(CCV_ERR_UNSUPPORTED, "batch too large for the layout kernel");
  const long long hw = static_cast<long long>(pb.h) * pb.w;
  const long long tiles = (hw + kLayoutW - 1) / kLayoutW;
  if (tiles > 0x7fffffffLL) return set_error(CCV_ERR_UNSUPPORTED, "image too large for the layout kernel");
  dim3 grid(static_cast<unsigned>(tiles), (pb.c + 31) / 32, static_cast<unsigned>(pb.n));
  dim3 block(32, 8);
  cudaError_t e = launch_kernel(ccv_nchw_to_planar_kernel, grid, block, 0, stream, 0,
                                reinterpret_cast<const float2*>(x), xr, xi, xr_lo, xi_lo, pb.c, hw);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "layout kernel launch");
  return CCV_OK;
}

int launch_split_planes(const float* xr, const float* xi, float* hr, float* hi, float* lr,
                        float* li, size_t count, cudaStream_t stream) {
  // count is a multiple of 4 (C % 4 == 0); all pointers 16-byte aligned.
  const long long c4 = static_cast<long long>(count / 4);
  const int threads = 256;
  const long long blocks = std::min<long long>((c4 + threads - 1) / threads, 148LL * 16);
  cudaError_t e = launch_kernel(
      ccv_split_planes_kernel, dim3(static_cast<unsigned>(std::max<long long>(blocks, 1))),
      dim3(threads), 0, stream, 0, reinterpret_cast<const float4*>(xr),
      reinterpret_cast<const float4*>(xi), reinterpret_cast<float4*>(hr),
      reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lr), reinterpret_cast<float4*>(li),
      c4);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "split kernel launch");
  return CCV_OK;
}

}  // namespace ccv
