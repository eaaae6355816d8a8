// In-kernel layout conversion for forward(): a few clusters of a persistent
// pair kernel turn complex64 NCHW images into the fp32 NHWC planes that the
// other clusters' TMA loads read, image by image, so forward() needs no
// separate layout pass and the conversion overlaps the convolution.
//
// Roles are dynamic: the first prm.cvt_clusters clusters to start (an
// atomic ticket) convert, the others convolve - a cluster only ever waits
// for clusters that are already running.  Per image, every converter CTA
// adds 1 to the image's counter after its share of tiles is stored; the
// image is ready when the count reaches the number of converter CTAs.  The
// last CTA to finish resets the counters (a zeroed library-owned set).
//
// Opt-in (CCV_CVT=1).  Measured on B200, a converting SM sustains only about
// 20-25 GB/s (in + out) through this 3-deep ring of 32 KB boxes - even with
// the transpose and stores taken out the loads alone run at that rate - while
// hiding a 64 x 128 x 56 x 56 conversion behind its convolution needs about
// 120 GB/s per converting SM.  forward() of that shape: 1444-1750 us with the
// modelled cluster count, 692-830 us with 12 converter clusters, against
// 422 us for the layout pass (at the HBM copy rate) plus the same kernel.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "ccv_fprop_common.cuh"
#include "ccv_ptx.cuh"

namespace ccv {

// Counter set layout.
constexpr int kCvtTicket = 0;   // cluster role tickets
constexpr int kCvtDone = 1;     // CTAs finished
constexpr int kCvtFlag0 = 8;    // image i: converter CTAs done with it
// Conversion tile: 8 rows x 16 pixels x 32 channels (32 KB of complex64 in,
// two 16 KB fp32 planes out).
constexpr int kCvtRows = 8;
constexpr int kCvtPx = 16;
constexpr int kCvtCh = 32;
constexpr uint32_t kCvtInBytes = kCvtRows * kCvtCh * kCvtPx * 8u;
constexpr uint32_t kCvtOutPlane = kCvtRows * kCvtPx * kCvtCh * 4u;
constexpr int kCvtInBufs = 4;
// Shared memory the converter role needs (input ring + two output buffers).
constexpr uint32_t kCvtSmemBytes = kCvtInBufs * kCvtInBytes + 2u * 2u * kCvtOutPlane;

// Converter CTA `me` of `nme`: converts its share of every image's tiles.
// `buf`: 1024-byte-aligned shared memory of kCvtSmemBytes; `full`: kCvtInBufs
// mbarriers (count 1).  Returns false if a wait ran out (status is set).
__device__ __forceinline__ bool cvt_role(const FpropParams& prm, int me, int nme, uint8_t* buf,
                                         uint32_t full0, int nthreads) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nwarps = nthreads >> 5;
  const int th = (prm.h + kCvtRows - 1) / kCvtRows;
  const int tw = (prm.w + kCvtPx - 1) / kCvtPx;
  const int tc = (prm.c + kCvtCh - 1) / kCvtCh;
  const int per_img = th * tw * tc;
  // This CTA's tiles of one image: j = me, me + nme, ...
  const int mine = per_img > me ? (per_img - me + nme - 1) / nme : 0;
  const long long total = static_cast<long long>(mine) * prm.n;
  uint8_t* in = buf;
  uint8_t* out = buf + kCvtInBufs * kCvtInBytes;
  const uint32_t in_u = ptx::smem_u32(in);
  const uint32_t out_u = ptx::smem_u32(out);
  auto coords = [&](long long k, int& img, int& c0, int& w0, int& h0) {
    img = static_cast<int>(k / (mine > 0 ? mine : 1));
    const int j = me + static_cast<int>(k - static_cast<long long>(img) * mine) * nme;
    const int cb = j % tc;
    const int rest = j / tc;
    c0 = cb * kCvtCh;
    w0 = (rest % tw) * kCvtPx;
    h0 = (rest / tw) * kCvtRows;
  };
  auto issue_load = [&](long long k) {
    int img, c0, w0, h0;
    coords(k, img, c0, w0, h0);
    const int b = static_cast<int>(k % kCvtInBufs);
    const uint32_t bar = full0 + 8u * static_cast<uint32_t>(b);
    ptx::mbar_arrive_expect_tx(bar, kCvtInBytes);
    ptx::tma_load_4d(in_u + static_cast<uint32_t>(b) * kCvtInBytes, &prm.tm_cin, bar, w0, c0, h0,
                     img);
  };
  unsigned* flags = prm.cvt_ctrs + kCvtFlag0;
  bool ok = true;
  if (tid == 0) {
    for (long long k = 0; k < kCvtInBufs && k < total; ++k) issue_load(k);
  }
  int img_done = 0;  // images announced so far
  for (long long k = 0; k < total; ++k) {
    int img, c0, w0, h0;
    coords(k, img, c0, w0, h0);
    const int b = static_cast<int>(k % kCvtInBufs);
    const bool got = ptx::mbar_wait_bounded_backoff(full0 + 8u * static_cast<uint32_t>(b),
                                                    static_cast<uint32_t>(k / kCvtInBufs) & 1u,
                                                    prm.status, CCV_ERR_DEVICE_TIMEOUT);
    const int ob = static_cast<int>(k & 1);
    if (tid == 0 && k >= 2) ptx::bulk_wait_read_le1();  // store of k-2 has read its buffer
    // Every thread takes the same exit if any wait ran out.
    if (__syncthreads_or(!got)) {
      ok = false;
      break;
    }
    // Transpose: lane = channel, (row, pixel pair) spread over the warps.
    const uint8_t* src = in + static_cast<uint32_t>(b) * kCvtInBytes;
    float* orr = reinterpret_cast<float*>(out + static_cast<uint32_t>(ob) * 2u * kCvtOutPlane);
    float* oii = orr + kCvtOutPlane / 4;
    for (int idx = warp; idx < kCvtRows * (kCvtPx / 2); idx += nwarps) {
      const int r = idx / (kCvtPx / 2);
      const int q = idx % (kCvtPx / 2);
      const int line = r * kCvtCh + lane;
      // 128-byte swizzle: 16-byte chunk q of line `line` is at chunk q ^ (line & 7).
      const float4 v = *reinterpret_cast<const float4*>(
          src + static_cast<uint32_t>(line) * 128u + (static_cast<uint32_t>(q ^ (line & 7)) << 4));
      const int p0 = (r * kCvtPx + 2 * q) * kCvtCh + lane;
      orr[p0] = v.x;
      oii[p0] = v.y;
      orr[p0 + kCvtCh] = v.z;
      oii[p0 + kCvtCh] = v.w;
    }
    ptx::fence_proxy_async_shared();
    __syncthreads();
    if (tid == 0) {
      if (k + kCvtInBufs < total) issue_load(k + kCvtInBufs);
      const uint32_t o = out_u + static_cast<uint32_t>(ob) * 2u * kCvtOutPlane;
      ptx::tma_store_4d(&prm.tm_pr, o, c0, w0, h0, img);
      ptx::tma_store_4d(&prm.tm_pi, o + kCvtOutPlane, c0, w0, h0, img);
      ptx::bulk_commit_group();
      // Last tile of this image for this CTA: publish once its stores landed.
      if (k == total - 1 || (k + 1) % mine == 0) {
        ptx::bulk_wait_all();
        ptx::fence_proxy_async_all();
        __threadfence();
        for (; img_done <= img; ++img_done) {
          asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(flags + img_done), "r"(1u)
                       : "memory");
        }
      }
    }
  }
  if (tid == 0) {
    ptx::bulk_wait_all();
    ptx::fence_proxy_async_all();
    __threadfence();
    // Images this CTA had no tile of (or that an abort skipped).
    for (; img_done < prm.n; ++img_done) {
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(flags + img_done), "r"(1u)
                   : "memory");
    }
  }
  return ok;
}

// Waits until image `img` is converted (bounded); then orders the caller's
// later TMA (async-proxy) reads after the converters' stores.
__device__ __forceinline__ bool cvt_wait_image(const FpropParams& prm, int img) {
  const unsigned* f = prm.cvt_ctrs + kCvtFlag0 + img;
  const unsigned need = static_cast<unsigned>(2 * prm.cvt_clusters);
  const uint64_t t0 = ptx::globaltimer();
  uint32_t ns = 64;
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v >= need) break;
    if (ptx::globaltimer() - t0 > CCV_WAIT_TIMEOUT_NS) {
      atomicCAS(prm.status, 0, CCV_ERR_DEVICE_TIMEOUT);
      return false;
    }
    ptx::nanosleep(ns);
    if (ns < 1024) ns <<= 1;
  }
  ptx::fence_proxy_async_all();
  return true;
}

}  // namespace ccv
