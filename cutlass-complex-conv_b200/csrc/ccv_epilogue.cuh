// Epilogue helpers shared by the persistent CTA-pair kernels: map a GEMM row
// of a 128-row tile to its output pixel, and move one TMEM accumulator
// ([re | im], 2*KT fp32 columns) of one row to global memory as fp32 NPQK
// planes or complex64 NKPQ.
#pragma once

#include <cuda.h>

#include <cstdint>

#include "ccv_fprop_common.cuh"
#include "ccv_ptx.cuh"

namespace ccv {

// Output pixel (img, op, oq) of GEMM row `row` of the 128-row tile `half`;
// false when the row lies outside the output.
template <bool FLAT>
__device__ __forceinline__ bool tile_row_pixel(const FpropParams& prm, int half, int row,
                                               int& img, int& op, int& oq) {
  if constexpr (FLAT) {
    const long long m = static_cast<long long>(half) * kBlockM + row;
    const long long pq = static_cast<long long>(prm.p) * prm.q;
    img = static_cast<int>(m / pq);
    const long long rem = m - static_cast<long long>(img) * pq;
    op = static_cast<int>(rem / prm.q);
    oq = static_cast<int>(rem - static_cast<long long>(op) * prm.q);
    return m < prm.m_total;
  } else {
    const int per_img = prm.tiles_bp * prm.tiles_bq;
    const int b = row >> prm.box_px_log2;
    const int local = row & ((1 << prm.box_px_log2) - 1);
    const int gb = half * prm.nb + b;
    img = gb / per_img;
    const int rem = gb - img * per_img;
    const int bp = rem / prm.tiles_bq;
    const int bq = rem - bp * prm.tiles_bq;
    op = bp * prm.box_p + (local >> prm.box_q_log2);
    oq = bq * prm.box_q + (local & ((1 << prm.box_q_log2) - 1));
    return gb < prm.total_boxes && op < prm.p && oq < prm.q;
  }
}

// Reads the accumulator row of this thread (TMEM address `t_acc`: lane of
// the thread, column 0 of the [re | im] block) in 32-column chunks and stores
// output channels [k0, k0 + KT) of pixel (img, op, oq).  Every thread of the
// warp must call this (tcgen05.ld is warp-collective); `valid` masks stores.
template <int KT, bool OUT_COMPLEX>
__device__ __forceinline__ void store_accumulator(const FpropParams& prm, uint32_t t_acc, int k0,
                                                  bool valid, int img, int op, int oq) {
  const long long pix = (static_cast<long long>(img) * prm.p + op) * prm.q + oq;
#pragma unroll 1
  for (int ch = 0; ch < KT; ch += 32) {
    uint32_t vr[32], vi[32];
    ptx::tmem_ld_32x32b_x32(t_acc + ch, vr);
    ptx::tmem_ld_32x32b_x32(t_acc + KT + ch, vi);
    ptx::tmem_wait_ld();
    const int kb = k0 + ch;
    if (!valid || kb >= prm.k) continue;
    if constexpr (!OUT_COMPLEX) {
      float* dr = prm.y0 + pix * prm.k + kb;
      float* di = prm.y1 + pix * prm.k + kb;
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        if (kb + j < prm.k) {
          *reinterpret_cast<float4*>(dr + j) =
              make_float4(__uint_as_float(vr[j]), __uint_as_float(vr[j + 1]),
                          __uint_as_float(vr[j + 2]), __uint_as_float(vr[j + 3]));
          *reinterpret_cast<float4*>(di + j) =
              make_float4(__uint_as_float(vi[j]), __uint_as_float(vi[j + 1]),
                          __uint_as_float(vi[j + 2]), __uint_as_float(vi[j + 3]));
        }
      }
    } else {
      const long long pq = static_cast<long long>(prm.p) * prm.q;
      float2* y = reinterpret_cast<float2*>(prm.y0);
      const long long base =
          static_cast<long long>(img) * prm.k * pq + static_cast<long long>(op) * prm.q + oq;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if (kb + j < prm.k) {
          y[base + static_cast<long long>(kb + j) * pq] =
              make_float2(__uint_as_float(vr[j]), __uint_as_float(vi[j]));
        }
      }
    }
  }
}

}  // namespace ccv
