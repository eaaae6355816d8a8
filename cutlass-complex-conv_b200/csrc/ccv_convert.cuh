// Converter warps of the fused complex path: read complex64 NCHW activations
// straight from global memory and write the planar, K-major, 128-byte-swizzled
// A tiles the tensor cores read (the layout a TMA load with 128-byte swizzle
// would produce from fp32 NHWC planes).  This replaces the two
// x.real/x.imag permute+contiguous copies of the reference's forward()
// (modules.py:198-199) with work inside the conv kernel.
#pragma once

#include <cuda.h>

#include <cstdint>

namespace ccv {

// Round to nearest TF32 (ties away), kept in an fp32 container.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// Values written per precision pass: raw (TF32 path), tf32(x) or the
// remainder x - tf32(x) (3xTF32 path; same arithmetic as the split kernel).
enum ConvertMode { kConvRaw = 0, kConvHi = 1, kConvLo = 2 };

// One A-slot fill job: rows [0, rows) (rows % 8 == 0) x 32 channels [c0,
// c0+32) of the two planes of an A slot (1024-byte aligned, 128-byte rows).
// Row `row` reads input pixel (img, h0 + row / box_q, w0 + row % box_q);
// pixels outside the image and channels >= C read as zero (padding).
struct SlotJob {
  int img, h0, w0, c0, mode;
};

// Work split: a unit is (block of 32 consecutive rows, channel quad j); lane
// l of the warp takes row 32 * block + l and the 4 channels 4j..4j+3 of it:
// 4 global loads (for box_q = 8, a warp's loads cover 4 runs of 64 contiguous
// bytes per channel) and one 16-byte shared store per plane at the swizzled
// chunk j ^ (row & 7).  Warp `wid` of `nwarps` takes units wid, wid + nwarps,
// ...; UNITS units per lane cover a slot of up to UNITS * nwarps * 4 rows
// (the host checks this).  The fill is split into a load phase (all loads of
// the job issued back to back into registers) and a store phase, so the
// loads of the next job can be in flight while the converter waits for its
// slot to be free.
template <int UNITS>
__device__ __forceinline__ void slot_job_load(float2 (&v)[UNITS][4], const SlotJob& jb,
                                              const float2* __restrict__ x, int C, int H, int W,
                                              int rows, int qlog, int wid, int nwarps,
                                              int lane) {
  const int units = ((rows + 31) >> 5) * 8;
  const int qmask = (1 << qlog) - 1;
  const long long plane = static_cast<long long>(H) * W;
#pragma unroll
  for (int u = 0; u < UNITS; ++u) {
    const int gu = wid + u * nwarps;
    const int row = ((gu >> 3) << 5) + lane;
    const int c = jb.c0 + ((gu & 7) << 2);
    const int h = jb.h0 + (row >> qlog);
    const int w = jb.w0 + (row & qmask);
    const bool ok = gu < units && row < rows && static_cast<unsigned>(h) < static_cast<unsigned>(H) &&
                    static_cast<unsigned>(w) < static_cast<unsigned>(W);
    const float2* src = x + (static_cast<long long>(jb.img) * C + c) * plane +
                        static_cast<long long>(h) * W + w;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      v[u][e] = (ok && c + e < C) ? __ldg(src + e * plane) : make_float2(0.f, 0.f);
    }
  }
}

__device__ __forceinline__ float conv_value(float x, int mode) {
  if (mode == kConvHi) return tf32_rna(x);
  if (mode == kConvLo) return x - tf32_rna(x);
  return x;
}

template <int UNITS>
__device__ __forceinline__ void slot_job_store(const float2 (&v)[UNITS][4], int mode, int rows,
                                               uint8_t* plane_r, uint8_t* plane_i, int wid,
                                               int nwarps, int lane) {
  const int units = ((rows + 31) >> 5) * 8;
#pragma unroll
  for (int u = 0; u < UNITS; ++u) {
    const int gu = wid + u * nwarps;
    const int row = ((gu >> 3) << 5) + lane;
    if (gu < units && row < rows) {
      const uint32_t off =
          static_cast<uint32_t>(row) * 128u + (static_cast<uint32_t>((gu & 7) ^ (row & 7)) << 4);
      *reinterpret_cast<float4*>(plane_r + off) =
          make_float4(conv_value(v[u][0].x, mode), conv_value(v[u][1].x, mode),
                      conv_value(v[u][2].x, mode), conv_value(v[u][3].x, mode));
      *reinterpret_cast<float4*>(plane_i + off) =
          make_float4(conv_value(v[u][0].y, mode), conv_value(v[u][1].y, mode),
                      conv_value(v[u][2].y, mode), conv_value(v[u][3].y, mode));
    }
  }
}

}  // namespace ccv
