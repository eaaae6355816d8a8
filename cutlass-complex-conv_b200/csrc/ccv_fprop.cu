// Complex Conv2d forward as an implicit planar-complex GEMM on sm_100a.
//
// GEMM view (same as the reference kernel, csrc/cutlass_ext/cutlass/conv/
// kernel/implicit_planar_cgemm_convolution.h:286-505): M = N*P*Q output
// pixels, N = K output channels, reduction = R*S*C.  The reference's
// mainloop (threadblock/implicit_planar_cgemm_multistage.h:251-271) issues
// four real products per fragment:
//     re += Ar*Br,  re += Ai*(-Bi),  im += Ar*Bi,  im += Ai*Br.
// Here the same four products are two tcgen05 MMAs per 8-deep K step, each
// M=128 x N=2*KT, sharing one weight operand and accumulating into two
// Tensor Memory accumulators:
//     D1 += Ar * [Wr ; Wi]^T,   D2 += Ai * [Wr ; Wi]^T
// (planes 1 and 2 of the packed tap), and the epilogue forms
// re = D1[:, :KT] - D2[:, KT:], im = D1[:, KT:] + D2[:, :KT].  Every
// activation and weight byte is loaded into shared memory once.
//
// Warp roles (192 threads, one CTA per SM):
//   warp 0      TMA producer: activation boxes (both planes) + weight box
//   warp 1      TMEM allocator and single-thread MMA issuer
//   warps 2..5  epilogue: tcgen05.ld -> registers -> global (NHWC planes or
//               complex64 NCHW), one output pixel per thread
//
// Activation tiles: the 128 GEMM rows of a tile are NB spatial boxes of
// box_p x box_q output pixels (box_p*box_q*NB = 128).  For tap (r, s) the
// box is one strided TMA load of the NHWC plane; TMA's out-of-bounds zero
// fill provides the padding (the reference uses cp.async zero-fill,
// threadblock/implicit_planar_cgemm_multistage.h:170-239).  1x1/stride-1/
// pad-0 problems use a flat 2-D view instead (128 consecutive pixels).
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "ccv_internal.h"
#include "ccv_fprop_common.cuh"
#include "ccv_layout_role.cuh"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

constexpr int kThreads = 192;
constexpr int kMaxSplits = 16;  // CTAs per cluster (non-portable above 8)
constexpr int kBlockC = 32;      // input channels per K step (128-byte rows)
constexpr int kRowBytes = kBlockC * 4;
constexpr int kABytes = kBlockM * kRowBytes;  // one activation plane per stage

// Error codes written into the device status word by bounded waits.
constexpr int kTimeoutProducer = CCV_ERR_DEVICE_TIMEOUT;
constexpr int kTimeoutMma = CCV_ERR_DEVICE_TIMEOUT;
constexpr int kTimeoutEpilogue = CCV_ERR_DEVICE_TIMEOUT;



// The weight stage holds two planes, [W_re; W_im] (KT rows each), which
// both MMAs of a K slice share: D1 += A_re * [W_re; W_im]^T and
// D2 += A_im * [W_re; W_im]^T, two TMEM accumulators of 2*KT columns; the
// epilogue forms re = D1[:, :KT] - D2[:, KT:] and im = D1[:, KT:] + D2[:, :KT]
// (each thread holds its whole row).  Two planes instead of the three of the
// one-accumulator form (-W_im, W_re, W_im) cut this kernel's weight bytes by
// a third; its batch-1 layers stream the weights from HBM.
template <int KT>
struct Cfg {
  static constexpr int kWBytes = 2 * KT * kRowBytes;
  static constexpr int kStageBytes = 2 * kABytes + kWBytes;
  static constexpr int kStages = (200 * 1024) / kStageBytes;  // 3 / 4 / 5 for KT 128 / 64 / 32
  static_assert(kStages >= 2, "pipeline too shallow");
  static constexpr int kTmemCols = 4 * KT;  // D1 | D2, 2*KT columns each
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
};

__device__ __forceinline__ float4 u4f(uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  return make_float4(__uint_as_float(a), __uint_as_float(b), __uint_as_float(c),
                     __uint_as_float(d));
}

// Output channels [ch, ch + 16) of this thread's accumulator row (TMEM
// address t_row: its lane, column 0) as fp32 bits: re = D1 - D2 (imag
// weights), im = D1 (imag weights) + D2 (real weights).  Warp-collective.
template <int KT>
__device__ __forceinline__ void load_complex16(uint32_t t_row, int ch, uint32_t (&re)[16],
                                               uint32_t (&im)[16]) {
  uint32_t a[16], b[16];
  ptx::tmem_ld_32x32b_x16(t_row + ch, re);           // sum x_re * W_re
  ptx::tmem_ld_32x32b_x16(t_row + KT + ch, im);      // sum x_re * W_im
  ptx::tmem_ld_32x32b_x16(t_row + 2 * KT + ch, a);   // sum x_im * W_re
  ptx::tmem_ld_32x32b_x16(t_row + 3 * KT + ch, b);   // sum x_im * W_im
  ptx::tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    re[j] = __float_as_uint(__uint_as_float(re[j]) - __uint_as_float(b[j]));
    im[j] = __float_as_uint(__uint_as_float(im[j]) + __uint_as_float(a[j]));
  }
}

template <int KT, bool FLAT, bool OUT_COMPLEX>
__global__ void __launch_bounds__(kThreads, 1)
    ccv_fprop_tf32_kernel(const __grid_constant__ FpropParams prm) {
  using C = Cfg<KT>;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment keeps every stage buffer on a swizzle-pattern boundary.
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  // bars[0..S) full, bars[S..2S) empty, bars[2S] accumulator ready
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 1);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] skip, [1] abort

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t smem_base = ptx::smem_u32(smem);
  const uint32_t bar_base = ptx::smem_u32(bars);
  auto full_bar = [&](int i) { return bar_base + 8u * i; };
  auto empty_bar = [&](int i) { return bar_base + 8u * (C::kStages + i); };
  const uint32_t acc_bar = bar_base + 8u * (2 * C::kStages);

  // Split-K: a cluster of `splits` CTAs shares one output tile; CTA `split`
  // runs K steps [kbeg, kend) and the partial sums are reduced after the
  // mainloop (splits == 1: no cluster).
  const int splits = prm.splits;
  const int tile = blockIdx.x / splits;
  const int split = blockIdx.x - tile * splits;
  const int kbeg = static_cast<int>(static_cast<long long>(split) * prm.ksteps / splits);
  const int kend = static_cast<int>(static_cast<long long>(split + 1) * prm.ksteps / splits);
  const int n_tile = tile % prm.tiles_n;
  const int m_tile = tile / prm.tiles_n;
  const int k0 = n_tile * KT;
  const int rs = prm.r * prm.s;

  // Prologue, spread over warps so that its latencies overlap: thread 0
  // asks for the tensor-map descriptors first (the first TMA issue waits for
  // them otherwise) and initialises the barriers, warp 1 allocates TMEM,
  // warp 3 reads the status word.
  if (threadIdx.x == 0) {
    ptx::prefetch_tmap(&prm.tm_w);
    ptx::prefetch_tmap(&prm.tm_xr);
    ptx::prefetch_tmap(&prm.tm_xi);
    flags[1] = 0;
    for (int i = 0; i < C::kStages; ++i) {
      ptx::mbar_init(full_bar(i), 1);
      ptx::mbar_init(empty_bar(i), 1);
    }
    ptx::mbar_init(acc_bar, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    ptx::tmem_alloc(ptx::smem_u32(tmem_holder), C::kTmemCols);
    ptx::tmem_relinquish();
  }
  // The status word is read before the wait below, so its latency overlaps
  // the previous kernel's tail (programmatic dependent launch).  No kernel
  // writes it except on a timeout, which the host also sees through the
  // word's host copy before it launches again.
  if (warp == 3 && lane == 0) {
    flags[0] = *reinterpret_cast<volatile int*>(prm.status) != 0 ? 1 : 0;
  }
  ptx::tc_fence_before();
  ptx::cta_sync();
  ptx::tc_fence_after();
  if (warp == 2 && lane == 0) {
    // Every weight byte of this CTA's K range is read once, from HBM: ask
    // for all of it now, before the wait for the previous kernel, so the
    // stream of the whole grid is in flight at once instead of `kStages`
    // boxes per CTA at a time; the producer's loads then hit L2.  An
    // epilogue warp issues it: it is idle until the accumulator is ready.
    for (int t = kbeg; t < kend; ++t) {
      const int cb = t / rs;
      ptx::tma_prefetch_l2_4d(&prm.tm_w, cb * kBlockC, k0, 1, t - cb * rs);
    }
  }
  // Everything above may overlap the previous kernel on the stream
  // (programmatic dependent launch); the operands and outputs are touched
  // only below.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  const uint32_t tmem_base = *tmem_holder;
  const bool skip = flags[0] != 0;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int t = kbeg; t < kend; ++t) {
        if (!ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, prm.status, kTimeoutProducer)) {
          flags[1] = 1;
          break;
        }
        if (flags[1]) break;
        const uint32_t fb = full_bar(stage);
        // Boxes of the tile past the last box of the problem are not loaded:
        // their rows hold whatever the stage held before, and the MMA rows
        // they feed are never stored or summed (a 7x7 image is one 8x8 box of
        // a two-box tile).
        int nload = 1;
        if constexpr (!FLAT) nload = max(1, min(prm.nb, prm.total_boxes - m_tile * prm.nb));
        const uint32_t a_bytes =
            FLAT ? static_cast<uint32_t>(kABytes)
                 : static_cast<uint32_t>(nload) * ((1u << prm.box_px_log2) * kRowBytes);
        ptx::mbar_arrive_expect_tx(fb, 2u * a_bytes + static_cast<uint32_t>(C::kWBytes));
        const int cb = t / rs;
        const int tap = t - cb * rs;
        const int rr = tap / prm.s;
        const int ss = tap - rr * prm.s;
        const int c0 = cb * kBlockC;
        const uint32_t a_r = smem_base + stage * C::kStageBytes;
        const uint32_t a_i = a_r + kABytes;
        const uint32_t w_s = a_i + kABytes;
        if constexpr (FLAT) {
          ptx::tma_load_2d(a_r, &prm.tm_xr, fb, c0, m_tile * kBlockM);
          ptx::tma_load_2d(a_i, &prm.tm_xi, fb, c0, m_tile * kBlockM);
        } else {
          const int per_img = prm.tiles_bp * prm.tiles_bq;
          const uint32_t box_bytes = (1u << prm.box_px_log2) * kRowBytes;
          for (int b = 0; b < nload; ++b) {
            const int gb = m_tile * prm.nb + b;
            const int img = gb / per_img;
            const int rem = gb - img * per_img;
            const int bp = rem / prm.tiles_bq;
            const int bq = rem - bp * prm.tiles_bq;
            const int wc = bq * prm.box_q * prm.sw - prm.pw + ss;
            const int hc = bp * prm.box_p * prm.sh - prm.ph + rr;
            ptx::tma_load_4d(a_r + b * box_bytes, &prm.tm_xr, fb, c0, wc, hc, img);
            ptx::tma_load_4d(a_i + b * box_bytes, &prm.tm_xi, fb, c0, wc, hc, img);
          }
        }
        // Planes 1 and 2 of the packed tap: [W_re; W_im].
        ptx::tma_load_4d(w_s, &prm.tm_w, fb, c0, k0, 1, tap);
        ++issued;
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Drain: make sure no TMA write into this CTA's shared memory is still
      // in flight before the CTA can exit (matters only after an abort).
      const int last = issued;
      for (int j = 0; j < C::kStages && j < last; ++j) {
        const int t = last - 1 - j;  // issue index (0-based within this CTA)
        const int st = t % C::kStages;
        const uint32_t ph = static_cast<uint32_t>((t / C::kStages) & 1);
        ptx::mbar_wait_bounded(full_bar(st), ph, prm.status, kTimeoutProducer);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && !skip) {
      constexpr uint32_t idesc = ptx::idesc_tf32(kBlockM, 2 * KT, false);
      int stage = 0;
      uint32_t phase = 0;
      for (int t = kbeg; t < kend; ++t) {
        if (!ptx::mbar_wait_bounded(full_bar(stage), phase, prm.status, kTimeoutMma)) {
          flags[1] = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t a_r = smem_base + stage * C::kStageBytes;
        const uint32_t a_i = a_r + kABytes;
        const uint32_t w_s = a_i + kABytes;
#pragma unroll
        for (int kk = 0; kk < kBlockC / 8; ++kk) {
          const uint32_t koff = kk * 32;
          const uint64_t da_r = ptx::desc_kmajor_sw128(a_r + koff);
          const uint64_t da_i = ptx::desc_kmajor_sw128(a_i + koff);
          const uint64_t db = ptx::desc_kmajor_sw128(w_s + koff);  // [Wr; Wi]
          const uint32_t acc = (t != kbeg || kk != 0) ? 1u : 0u;
          ptx::mma_tf32_ss(tmem_base, da_r, db, idesc, acc);           // D1
          ptx::mma_tf32_ss(tmem_base + 2 * KT, da_i, db, idesc, acc);  // D2
        }
        ptx::mma_commit(empty_bar(stage));
        if (++stage == C::kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      // Accumulator complete (or abandoned): release the epilogue, then wait
      // ourselves so no MMA is in flight when TMEM is freed.
      ptx::mma_commit(acc_bar);
      ptx::mbar_wait_bounded(acc_bar, 0, prm.status, kTimeoutMma);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lane quarter this warp may access
    const int row = quarter * 32 + lane;
    bool ok = false;
    if (!skip) {
      ok = ptx::mbar_wait_bounded(acc_bar, 0, prm.status, kTimeoutEpilogue);
      ptx::tc_fence_after();
    }
    // Map the GEMM row to an output pixel.
    bool valid = ok;
    int img = 0, op = 0, oq = 0;
    if constexpr (FLAT) {
      const long long m = static_cast<long long>(m_tile) * kBlockM + row;
      valid = valid && (m < prm.m_total);
      const long long pq = static_cast<long long>(prm.p) * prm.q;
      img = static_cast<int>(m / pq);
      const long long rem = m - static_cast<long long>(img) * pq;
      op = static_cast<int>(rem / prm.q);
      oq = static_cast<int>(rem - static_cast<long long>(op) * prm.q);
    } else {
      const int b = row >> prm.box_px_log2;
      const int local = row & ((1 << prm.box_px_log2) - 1);
      const int pi = local >> prm.box_q_log2;
      const int qi = local & ((1 << prm.box_q_log2) - 1);
      const int gb = m_tile * prm.nb + b;
      valid = valid && (gb < prm.total_boxes);
      const int per_img = prm.tiles_bp * prm.tiles_bq;
      img = gb / per_img;
      const int rem = gb - img * per_img;
      const int bp = rem / prm.tiles_bq;
      const int bq = rem - bp * prm.tiles_bq;
      op = bp * prm.box_p + pi;
      oq = bq * prm.box_q + qi;
      valid = valid && (op < prm.p) && (oq < prm.q);
    }
    if (flags[1]) valid = false;
    if (!skip && splits > 1 && prm.split_ws != nullptr) {
      // Split-K through L2: this warp's 32 rows, when one of them holds an
      // output pixel, go to this CTA's partial block in the workspace as
      // 2 KB granules - granule g holds channels 8g..8g+7, its float4 j
      // (re 0-3, re 4-7, im 0-3, im 4-7) of row `lane` at g*128 + j*32 +
      // lane - so a warp stores 512 contiguous bytes at a time.
      if (__any_sync(0xffffffffu, valid)) {
        const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
        float4* dst = reinterpret_cast<float4*>(prm.split_ws) +
                      ((static_cast<long long>(tile) * splits + split) * 4 + quarter) * (16 * KT) +
                      lane;
#pragma unroll 1
        for (int ch = 0; ch < KT; ch += 16) {
          uint32_t vr[16], vi[16];
          load_complex16<KT>(t_row, ch, vr, vi);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float4* gd = dst + (ch / 8 + h) * 128;
            __stcg(gd, u4f(vr[8 * h], vr[8 * h + 1], vr[8 * h + 2], vr[8 * h + 3]));
            __stcg(gd + 32, u4f(vr[8 * h + 4], vr[8 * h + 5], vr[8 * h + 6], vr[8 * h + 7]));
            __stcg(gd + 64, u4f(vi[8 * h], vi[8 * h + 1], vi[8 * h + 2], vi[8 * h + 3]));
            __stcg(gd + 96, u4f(vi[8 * h + 4], vi[8 * h + 5], vi[8 * h + 6], vi[8 * h + 7]));
          }
        }
        // No fence: the cluster barrier below (arrive.release / wait.acquire
        // at cluster scope, by every thread) orders these stores before the
        // other CTAs of the cluster - the only readers - load them.
      }
    } else if (!skip && splits > 1) {
      // Split-K: park this CTA's partial accumulator row in shared memory
      // (the pipeline buffers are idle now) for the cluster reduction;
      // 16-byte columns XOR-swizzled by row to spread banks.
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      float4* part = reinterpret_cast<float4*>(smem) + static_cast<size_t>(row) * (KT / 2);
#pragma unroll 1
      for (int ch = 0; ch < KT; ch += 16) {
        uint32_t vr[16], vi[16];
        load_complex16<KT>(t_row, ch, vr, vi);
#pragma unroll
        for (int j = 0; j < 16; j += 4) {
          part[((ch + j) >> 2) ^ (row & 7)] = u4f(vr[j], vr[j + 1], vr[j + 2], vr[j + 3]);
          part[((KT + ch + j) >> 2) ^ (row & 7)] = u4f(vi[j], vi[j + 1], vi[j + 2], vi[j + 3]);
        }
      }
    } else if (!skip) {
      const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
      const long long pix = (static_cast<long long>(img) * prm.p + op) * prm.q + oq;
#pragma unroll 1
      for (int ch = 0; ch < KT; ch += 16) {
        uint32_t vr[16], vi[16];
        load_complex16<KT>(t_row, ch, vr, vi);
        const int kb = k0 + ch;
        if (valid && kb < prm.k) {
          add_bias<16>(prm, kb, vr, vi);
          if constexpr (!OUT_COMPLEX) {
            float* dr = prm.y0 + pix * prm.k + kb;
            float* di = prm.y1 + pix * prm.k + kb;
            if (kb + 16 <= prm.k) {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                *reinterpret_cast<float4*>(dr + j) = u4f(vr[j], vr[j + 1], vr[j + 2], vr[j + 3]);
                *reinterpret_cast<float4*>(di + j) = u4f(vi[j], vi[j + 1], vi[j + 2], vi[j + 3]);
              }
            } else {
#pragma unroll
              for (int j = 0; j < 16; j += 4) {
                if (kb + j < prm.k) {
                  *reinterpret_cast<float4*>(dr + j) = u4f(vr[j], vr[j + 1], vr[j + 2], vr[j + 3]);
                  *reinterpret_cast<float4*>(di + j) = u4f(vi[j], vi[j + 1], vi[j + 2], vi[j + 3]);
                }
              }
            }
          } else {
            // complex64 NKPQ: element (img, k, op, oq) as (re, im)
            const long long pq = static_cast<long long>(prm.p) * prm.q;
            float2* y = reinterpret_cast<float2*>(prm.y0);
            const long long base = static_cast<long long>(img) * prm.k * pq +
                                   static_cast<long long>(op) * prm.q + oq;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (kb + j < prm.k) {
                y[base + static_cast<long long>(kb + j) * pq] =
                    make_float2(__uint_as_float(vr[j]), __uint_as_float(vi[j]));
              }
            }
          }
        }
      }
    }
    ptx::tc_fence_before();
  }

  ptx::cta_sync();
  if (splits > 1) {
    // ---------------------------------------------------------- cluster reduce
    // Every partial is parked.  Only the tile rows that hold an output pixel
    // are summed (a 7x7 image fills 49 of a 128-row tile): the CTAs list
    // them in the same order, and CTA `split` sums an equal share of the
    // (row, 4-channel group) items over the S partials in rank order
    // (deterministic), reading the other CTAs' partials through distributed
    // shared memory, and writes them out.
    __shared__ int vrows[kBlockM];
    __shared__ unsigned vmask[kBlockM / 32];
    bool v = false;
    unsigned vm = 0;
    if (threadIdx.x < kBlockM) {
      const int row = threadIdx.x;
      if constexpr (FLAT) {
        v = static_cast<long long>(m_tile) * kBlockM + row < prm.m_total;
      } else {
        const int b = row >> prm.box_px_log2;
        const int local = row & ((1 << prm.box_px_log2) - 1);
        const int gb = m_tile * prm.nb + b;
        const int per_img = prm.tiles_bp * prm.tiles_bq;
        const int rem = gb - (gb / per_img) * per_img;
        const int bp = rem / prm.tiles_bq;
        const int bq = rem - bp * prm.tiles_bq;
        v = gb < prm.total_boxes && bp * prm.box_p + (local >> prm.box_q_log2) < prm.p &&
            bq * prm.box_q + (local & ((1 << prm.box_q_log2) - 1)) < prm.q;
      }
      vm = __ballot_sync(0xffffffffu, v);
      if (lane == 0) vmask[warp] = vm;
    }
    ptx::cta_sync();
    if (v) {
      int idx = __popc(vm & ((1u << lane) - 1u));
      for (int w2 = 0; w2 < warp; ++w2) idx += __popc(vmask[w2]);
      vrows[idx] = threadIdx.x;
    }
    ptx::cluster_sync();
    int nvalid = 0;
#pragma unroll
    for (int w2 = 0; w2 < kBlockM / 32; ++w2) nvalid += __popc(vmask[w2]);
    const bool do_store = !skip && !flags[1];
    // Stores the sums (sr, si) of channels kb..kb+3 of tile row `row`.
    auto store4 = [&](int row, int kb, float4 sr, float4 si) {
      int img = 0, op = 0, oq = 0;
      if constexpr (FLAT) {
        const long long m = static_cast<long long>(m_tile) * kBlockM + row;
        const long long pq = static_cast<long long>(prm.p) * prm.q;
        img = static_cast<int>(m / pq);
        const long long rem = m - static_cast<long long>(img) * pq;
        op = static_cast<int>(rem / prm.q);
        oq = static_cast<int>(rem - static_cast<long long>(op) * prm.q);
      } else {
        const int b = row >> prm.box_px_log2;
        const int local = row & ((1 << prm.box_px_log2) - 1);
        const int gb = m_tile * prm.nb + b;
        const int per_img = prm.tiles_bp * prm.tiles_bq;
        img = gb / per_img;
        const int rem = gb - img * per_img;
        const int bp = rem / prm.tiles_bq;
        const int bq = rem - bp * prm.tiles_bq;
        op = bp * prm.box_p + (local >> prm.box_q_log2);
        oq = bq * prm.box_q + (local & ((1 << prm.box_q_log2) - 1));
      }
      if (prm.bias_r != nullptr) {
        const float4 br = __ldg(reinterpret_cast<const float4*>(prm.bias_r + kb));
        const float4 bi = __ldg(reinterpret_cast<const float4*>(prm.bias_i + kb));
        sr.x += br.x; sr.y += br.y; sr.z += br.z; sr.w += br.w;
        si.x += bi.x; si.y += bi.y; si.z += bi.z; si.w += bi.w;
      }
      const long long pix = (static_cast<long long>(img) * prm.p + op) * prm.q + oq;
      if constexpr (!OUT_COMPLEX) {
        *reinterpret_cast<float4*>(prm.y0 + pix * prm.k + kb) = sr;
        *reinterpret_cast<float4*>(prm.y1 + pix * prm.k + kb) = si;
      } else {
        const long long pq = static_cast<long long>(prm.p) * prm.q;
        float2* y = reinterpret_cast<float2*>(prm.y0) + static_cast<long long>(img) * prm.k * pq +
                    static_cast<long long>(op) * prm.q + oq;
        y[static_cast<long long>(kb) * pq] = make_float2(sr.x, si.x);
        y[static_cast<long long>(kb + 1) * pq] = make_float2(sr.y, si.y);
        y[static_cast<long long>(kb + 2) * pq] = make_float2(sr.z, si.z);
        y[static_cast<long long>(kb + 3) * pq] = make_float2(sr.w, si.w);
      }
    };
    if (prm.split_ws != nullptr) {
      // L2 partials: items are (32-row block with outputs, granule, half,
      // lane), lane fastest, so a warp loads 512 contiguous bytes from each
      // partial; the S partials are summed in rank order.
      int qlist[kBlockM / 32];
      int nq = 0;
#pragma unroll
      for (int w2 = 0; w2 < kBlockM / 32; ++w2) {
        if (vmask[w2] != 0u) qlist[nq++] = w2;
      }
      constexpr int kGran = KT / 8;
      const int items = nq * kGran * 64;
      const int i0 = items * split / splits;
      const int i1 = items * (split + 1) / splits;
      const float4* ws4 = reinterpret_cast<const float4*>(prm.split_ws);
      for (int it = i0 + threadIdx.x; it < i1; it += kThreads) {
        const int ln = it & 31;
        const int h = (it >> 5) & 1;
        const int rest = it >> 6;
        const int g = rest % kGran;
        const int qb = qlist[rest / kGran];
        const int row = qb * 32 + ln;
        if (!((vmask[qb] >> ln) & 1u)) continue;
        const long long base =
            ((static_cast<long long>(tile) * splits) * 4 + qb) * (16 * KT) + g * 128 + ln;
        float4 pa[16], pb[16];
#pragma unroll
        for (int s2 = 0; s2 < 16; ++s2) {
          if (s2 < splits) {
            const float4* src = ws4 + base + static_cast<long long>(s2) * 4 * (16 * KT);
            pa[s2] = __ldcg(src + h * 32);
            pb[s2] = __ldcg(src + (2 + h) * 32);
          }
        }
        float4 sr = make_float4(0.f, 0.f, 0.f, 0.f), si = sr;
#pragma unroll
        for (int s2 = 0; s2 < 16; ++s2) {
          if (s2 < splits) {
            sr.x += pa[s2].x; sr.y += pa[s2].y; sr.z += pa[s2].z; sr.w += pa[s2].w;
            si.x += pb[s2].x; si.y += pb[s2].y; si.z += pb[s2].z; si.w += pb[s2].w;
          }
        }
        const int kb = k0 + 8 * g + 4 * h;
        if (do_store && kb < prm.k) store4(row, kb, sr, si);
      }
    } else {
      const int quads = KT / 4;
      const long long items = static_cast<long long>(nvalid) * quads;
      const int i0 = static_cast<int>(items * split / splits);
      const int i1 = static_cast<int>(items * (split + 1) / splits);
      const uint32_t part_base = smem_base;
      for (int it = i0 + threadIdx.x; it < i1; it += kThreads) {
        const int row = vrows[it / quads];
        const int q = it - (it / quads) * quads;
        const uint32_t off_r =
            static_cast<uint32_t>(row * (KT / 2) + (q ^ (row & 7))) * 16u;
        const uint32_t off_i =
            static_cast<uint32_t>(row * (KT / 2) + ((quads + q) ^ (row & 7))) * 16u;
        // All remote loads first (they overlap), then the sums in rank order.
        float4 pa[16], pb[16];
#pragma unroll
        for (int s2 = 0; s2 < 16; ++s2) {
          if (s2 < splits) {
            pa[s2] = ptx::ld_shared_cluster_v4(ptx::mapa_shared(part_base + off_r, s2));
            pb[s2] = ptx::ld_shared_cluster_v4(ptx::mapa_shared(part_base + off_i, s2));
          }
        }
        float4 sr = make_float4(0.f, 0.f, 0.f, 0.f), si = sr;
#pragma unroll
        for (int s2 = 0; s2 < 16; ++s2) {
          if (s2 < splits) {
            sr.x += pa[s2].x; sr.y += pa[s2].y; sr.z += pa[s2].z; sr.w += pa[s2].w;
            si.x += pb[s2].x; si.y += pb[s2].y; si.z += pb[s2].z; si.w += pb[s2].w;
          }
        }
        const int kb = k0 + 4 * q;
        if (do_store && kb < prm.k) store4(row, kb, sr, si);
      }
      // Keep every partial alive until all CTAs finished reading.
      ptx::cluster_sync();
    }
  }
  if (warp == 1) {
    __syncwarp();  // tcgen05.dealloc is warp-collective
    ptx::tc_fence_after();
    ptx::tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

// ------------------------------------------------------------------ host side
// Function attributes of one single-CTA kernel variant (once per device).
template <int KT, bool FLAT, bool OUT_COMPLEX>
cudaError_t prepare_variant() {
  using C = Cfg<KT>;
  auto kern = ccv_fprop_tf32_kernel<KT, FLAT, OUT_COMPLEX>;
  static std::once_flag once[64];
  static cudaError_t err[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&]() {
    err[dev & 63] = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         C::kSmemBytes);
    if (err[dev & 63] != cudaSuccess) return;
    cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    cudaGetLastError();
  });
  return err[dev & 63];
}

// Clusters of 1..16 CTAs of the KT-wide single-CTA kernel the device can
// hold at once (index = cluster size; 0: that size cannot be launched),
// queried once per device.  A cluster takes its SMs from one GPC, so B200
// holds only about 7 clusters of 16 - fewer than it has SMs for.
template <int KT>
const int* cluster_capacity() {
  using C = Cfg<KT>;
  auto kern = ccv_fprop_tf32_kernel<KT, false, false>;
  static std::once_flag once[64];
  static int caps[64][kMaxSplits + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  std::call_once(once[dev & 63], [&]() {
    if (prepare_variant<KT, false, false>() != cudaSuccess) return;
    for (int size = 1; size <= kMaxSplits; ++size) {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(size), 1, 1);
      cfg.blockDim = dim3(kThreads, 1, 1);
      cfg.dynamicSmemBytes = C::kSmemBytes;
      cudaLaunchAttribute attr[1];
      attr[0].id = cudaLaunchAttributeClusterDimension;
      attr[0].val.clusterDim.x = static_cast<unsigned>(size);
      attr[0].val.clusterDim.y = 1;
      attr[0].val.clusterDim.z = 1;
      cfg.attrs = attr;
      cfg.numAttrs = 1;
      int n = 0;
      if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) {
        caps[dev & 63][size] = n;
      } else {
        cudaGetLastError();
      }
    }
  });
  return caps[dev & 63];
}

template <int KT, bool FLAT, bool OUT_COMPLEX>
int launch_variant(FpropParams& prm, int tiles, int splits, cudaStream_t stream) {
  using C = Cfg<KT>;
  auto kern = ccv_fprop_tf32_kernel<KT, FLAT, OUT_COMPLEX>;
  const cudaError_t attr_err = prepare_variant<KT, FLAT, OUT_COMPLEX>();
  if (attr_err != cudaSuccess) return cuda_error(attr_err, "cudaFuncSetAttribute(fprop)");
  prm.splits = splits;
  const long long grid = static_cast<long long>(tiles) * splits;
  if (grid > 0x7fffffffLL) return set_error(CCV_ERR_UNSUPPORTED, "problem too large for the grid");
  const cudaError_t le = launch_kernel(kern, dim3(static_cast<unsigned>(grid)), dim3(kThreads),
                                       C::kSmemBytes, stream, splits, prm);
  if (le != cudaSuccess) return cuda_error(le, "fprop kernel launch");
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "fprop kernel launch");
  return CCV_OK;
}

template <bool FLAT, bool OUT_COMPLEX>
int launch_kt(int kt, FpropParams& prm, int tiles, int splits, cudaStream_t stream) {
  switch (kt) {
    case 128: return launch_variant<128, FLAT, OUT_COMPLEX>(prm, tiles, splits, stream);
    case 64: return launch_variant<64, FLAT, OUT_COMPLEX>(prm, tiles, splits, stream);
    default: return launch_variant<32, FLAT, OUT_COMPLEX>(prm, tiles, splits, stream);
  }
}

const int* cluster_capacity_kt(int kt) {
  switch (kt) {
    case 128: return cluster_capacity<128>();
    case 64: return cluster_capacity<64>();
    default: return cluster_capacity<32>();
  }
}

// Plan of the single-CTA kernel: output-channel tile, CTAs per tile (a
// cluster splitting the K loop) and where the split's partial sums meet.
struct SinglePlan {
  int kt = 128;
  int splits = 1;
  bool l2 = false;       // partial sums through L2 (workspace) rather than DSMEM
  size_t ws_bytes = 0;   // workspace the L2 reduction needs
};

size_t single_l2_bytes(int tiles, int splits, int kt) {
  return static_cast<size_t>(tiles) * splits * kBlockM * 2 * kt * sizeof(float);
}

// Picks the channel tile (32, 64 or 128) and the split (1..16 CTAs per tile,
// one cluster) by an estimate of the launch's time on B200:
//   ceil(K steps / split) x step time(tile)          the slowest CTA's loop
// + rows x 2*tile x 4 B / 100 GB/s                    partial (or output) rows out
// + 1.5 us when split                                 cluster barrier + sums
// with step times 0.55 / 0.60 / 0.80 us for tiles of 32 / 64 / 128, rows the
// tile's output rows rounded up to a warp's 32.  Only plans of one wave fit:
// at most one CTA per SM and no more clusters than the device holds at once
// (a second wave of clusters doubled the time).  The constants come from a
// graph-replay sweep of every tile x split on the four batch-1 layers, where
// the estimate ranks the fastest plan first on each: 32->64 @ 56x56 tile 64
// split 5 (10.2 us; split 4: 10.8), 64->128 @ 28x28 64/9 (9.4; 64/8: 9.8),
// 128->256 @ 14x14 64/9 (10.2; 64/8: 10.8), 256->512 @ 7x7 128/16 (10.5;
// 64/8: 12.1) - a split that divides the K steps evenly leaves no CTA a step
// behind the others at the barrier.  With workspace room (`ws_bytes`;
// SIZE_MAX: unbounded) the partial sums meet in L2, else over distributed
// shared memory (~1 us slower on the deep layers).  CCV_KT pins the tile;
// CCV_SPLITK caps the split.
SinglePlan plan_single_cta(const Problem& pb, const Tiling& t, size_t ws_bytes) {
  SinglePlan best;
  double best_us = 1e30;
  const int sms = device_sm_count();
  const int ksteps = ((pb.c + kBlockC - 1) / kBlockC) * pb.r * pb.s;
  const int pin = knobs().kt;
  const int cap = knobs().splitk > 0 ? std::min(knobs().splitk, kMaxSplits) : kMaxSplits;
  const long long m_total = static_cast<long long>(pb.n) * pb.p * pb.q;
  const long long rows_per_tile = (m_total + t.tiles_m - 1) / t.tiles_m;
  const double rows = static_cast<double>(std::min<long long>(kBlockM, (rows_per_tile + 31) / 32 * 32));
  for (int kt = 128; kt >= 32; kt /= 2) {
    if (pin == 32 || pin == 64 || pin == 128) {
      if (kt != pin) continue;
    } else if (kt > t.kt) {
      continue;
    }
    const int tiles_n = (pb.k + kt - 1) / kt;
    const long long tiles = static_cast<long long>(t.tiles_m) * tiles_n;
    const int* caps = cluster_capacity_kt(kt);
    const double step_us = kt == 128 ? 0.80 : (kt == 64 ? 0.60 : 0.55);
    const double out_us = rows * 2.0 * kt * 4.0 / 100e3;
    for (int sp = 1; sp <= cap && sp <= ksteps; ++sp) {
      if (tiles * sp > sms && sp > 1) break;
      if (sp > 1 && caps[sp] < tiles) continue;
      const double us = ((ksteps + sp - 1) / sp) * step_us + out_us + (sp > 1 ? 1.5 : 0.0);
      if (us < best_us - 1e-9) {  // ties keep the wider tile and the smaller split
        best_us = us;
        best.kt = kt;
        best.splits = sp;
        const size_t need = sp > 1 ? single_l2_bytes(static_cast<int>(tiles), sp, kt) : 0;
        best.l2 = sp > 1 && ws_bytes >= need;
        best.ws_bytes = best.l2 ? need : 0;
      }
    }
  }
  return best;
}

}  // namespace

namespace {

enum KernelFamily { kSingleCta = 0, kPairTap = 1, kPairHalo = 2 };

// Kernel family for a problem.  Large problems go to the persistent CTA-pair
// kernels; small ones (fewer pair tiles than half the SMs) to the single-CTA
// kernel.  Among the pair kernels, halo reuse serves stride-1 filters unless
// its one-box tiles compute clearly more rows than the tap kernel's multi-box
// tiles.  3xTF32 runs only on the pair kernels (they take precision passes).
// Testing/benchmarking knobs: CCV_FORCE_KERNEL=1|2 pins single-CTA / pair,
// CCV_HALO=0|1 pins the pair variant.
KernelFamily choose_family(const Problem& pb, bool split, const Tiling& t, Tiling* th) {
  const int forced = knobs().force_kernel;
  const bool use_pair =
      split || forced == 2 || (forced != 1 && pair_tiles(t) * 2 >= device_sm_count());
  if (!use_pair) return kSingleCta;
  const int halo_forced = knobs().halo;
  if (halo_forced != 0 && halo_applicable(pb)) {
    *th = choose_halo_tiling(pb);
    const long long rows_tap = static_cast<long long>(t.tiles_m) * t.tiles_n;
    const long long rows_halo = static_cast<long long>(th->tiles_m) * th->tiles_n;
    if (halo_forced == 1 || rows_halo * 100 <= rows_tap * 115) return kPairHalo;
  }
  return kPairTap;
}

}  // namespace

size_t split_workspace_bytes(const Problem& pb, int precision, bool complex_input) {
  (void)complex_input;
  const bool split = precision == CCV_PRECISION_3XTF32;
  const Tiling t = choose_tiling(pb);
  Tiling th;
  const int passes = split ? 3 : 1;
  switch (choose_family(pb, split, t, &th)) {
    case kPairHalo:
      return pair_split_workspace_bytes(th.kt, pair_tiles(th),
                                        ((pb.c + kBlockC - 1) / kBlockC) * pb.s * passes);
    case kPairTap:
      return pair_split_workspace_bytes(t.kt, pair_tiles(t),
                                        ((pb.c + kBlockC - 1) / kBlockC) * pb.r * pb.s * passes);
    default:
      // Single-CTA kernel: room for its split-K partial sums in L2.
      return plan_single_cta(pb, t, SIZE_MAX).ws_bytes;
  }
}

bool use_layout_warps(const Problem& pb, int precision) { return layout_warps_pay(pb, precision); }

bool layout_warps_pay(const Problem& pb, int precision) {
  // CCV_LW=0: never; CCV_LW=1: wherever a pair kernel runs; unset: when
  //   * the grid runs at least two waves of tiles (below that the first
  //     wave needs most images at once),
  //   * the input is at least 96 MB (below that the layout pass's cost is
  //     small and the layout warps' traffic during the convolution costs as
  //     much or more; at 103 MB - batch 32 of the 56x56 layer - they win
  //     ~4 % once the stream-K split is off, which layout-warp launches now
  //     skip: 226 / 232 / 225 -> 215 / 218 / 222 us in three B200 runs), and
  //   * there are at least 500 flops per input byte, K*R*S*(P*Q)/(H*W) per
  //     pass (the layout warps convert ~1 TB/s; below that - stride 2 at
  //     C = 64 - they hold the MMAs back and a pass at the copy rate wins).
  // Measured on B200 over the BASELINE layers and the batch sweep.
  const int mode = knobs().lw;
  if (mode == 0) return false;
  const Tiling t = choose_tiling(pb);
  Tiling th;
  const int fam = choose_family(pb, precision == CCV_PRECISION_3XTF32, t, &th);
  if (fam != kPairHalo && fam != kPairTap) return false;
  if (pb.n > kSkCounterWords - kLwFlag0) return false;
  if (mode == 1) return true;
  const double in_bytes = 8.0 * pb.n * pb.h * pb.w * pb.c;
  const double flops_per_byte = static_cast<double>(pb.k) * pb.r * pb.s * pb.p * pb.q /
                                (static_cast<double>(pb.h) * pb.w) *
                                (precision == CCV_PRECISION_3XTF32 ? 3 : 1);
  if (in_bytes < 96.0 * 1024 * 1024 || flops_per_byte < 500.0) return false;
  // Pixels per cluster tile: two CTAs of 128 (halo: two sub-boxes each for
  // KT <= 64).
  const int kt = fam == kPairHalo ? th.kt : t.kt;
  const int tiles_n = fam == kPairHalo ? th.tiles_n : t.tiles_n;
  const long long tile_px = 2LL * kBlockM * (fam == kPairHalo && kt <= 64 ? 2 : 1);
  const long long tiles =
      (static_cast<long long>(pb.n) * pb.p * pb.q + tile_px - 1) / tile_px * tiles_n;
  return tiles >= 2LL * (device_sm_count() / 2);
}

bool use_layout_warps_planar(const Problem& pb, int precision) {
  return precision == CCV_PRECISION_3XTF32 && layout_warps_pay(pb, precision);
}

int launch_fprop_planar_lw(const float* x_real, const float* x_imag, float* hr, float* hi,
                           float* lr, float* li, const float* w_packed, float* y_real,
                           float* y_imag, const Problem& pb, const Epilogue& ep, void* ws,
                           size_t ws_bytes, cudaStream_t stream) {
  const Tiling t = choose_tiling(pb);
  Tiling th;
  switch (choose_family(pb, true, t, &th)) {
    case kPairHalo:
      return launch_fprop_pair_halo(hr, hi, lr, li, true, w_packed, y_real, y_imag, pb, th,
                                    OUT_PLANAR_NHWC, ep, ws, ws_bytes, stream, nullptr, x_real,
                                    x_imag);
    case kPairTap:
      return launch_fprop_pair(hr, hi, lr, li, w_packed, y_real, y_imag, pb, t, OUT_PLANAR_NHWC,
                               ep, ws, ws_bytes, stream, nullptr, x_real, x_imag);
    default:
      return set_error(CCV_ERR_UNSUPPORTED, "no layout warps for this problem");
  }
}

int launch_fprop_complex_lw(const float* x, float* xr, float* xi, float* xr_lo, float* xi_lo,
                            const float* w_packed, float* y, const Problem& pb, int precision,
                            const Epilogue& ep, void* ws, size_t ws_bytes, cudaStream_t stream) {
  const bool split = precision == CCV_PRECISION_3XTF32;
  const Tiling t = choose_tiling(pb);
  Tiling th;
  switch (choose_family(pb, split, t, &th)) {
    case kPairHalo:
      return launch_fprop_pair_halo(xr, xi, xr_lo, xi_lo, split, w_packed, y, nullptr, pb, th,
                                    OUT_COMPLEX_NCHW, ep, ws, ws_bytes, stream, x);
    case kPairTap:
      return launch_fprop_pair(xr, xi, split ? xr_lo : nullptr, split ? xi_lo : nullptr, w_packed,
                               y, nullptr, pb, t, OUT_COMPLEX_NCHW, ep, ws, ws_bytes, stream, x);
    default:
      return set_error(CCV_ERR_UNSUPPORTED, "no layout warps for this problem");
  }
}

const char* complex_kernel_name(const Problem& pb, int precision) {
  const bool split = precision == CCV_PRECISION_3XTF32;
  const Tiling t = choose_tiling(pb);
  Tiling th;
  const int fam = choose_family(pb, split, t, &th);
  if (use_layout_warps(pb, precision)) {
    return fam == kPairHalo ? "halo_pair_layout_warps" : "tap_pair_layout_warps";
  }
  switch (fam) {
    case kPairHalo:
      return "layout_pass+halo_pair";
    case kPairTap:
      return "layout_pass+tap_pair";
    default:
      return "layout_pass+single_cta";
  }
}

int launch_fprop(const float* xr, const float* xi, const float* xr_lo, const float* xi_lo,
                 const float* w_packed, float* y0, float* y1, const Problem& pb, int precision,
                 OutLayout out_layout, const Epilogue& ep, void* ws, size_t ws_bytes,
                 cudaStream_t stream) {
  const bool split = precision == CCV_PRECISION_3XTF32;
  if (split && (xr_lo == nullptr || xi_lo == nullptr)) {
    return set_error(CCV_ERR_INVALID_ARGUMENT, "3xTF32 needs the activation remainder planes");
  }
  if (!split) {
    xr_lo = nullptr;
    xi_lo = nullptr;
  }
  Tiling t = choose_tiling(pb);
  Tiling th;
  switch (choose_family(pb, split, t, &th)) {
    case kPairHalo:
      return launch_fprop_pair_halo(xr, xi, xr_lo, xi_lo, split, w_packed, y0, y1, pb, th,
                                    out_layout, ep, ws, ws_bytes, stream);
    case kPairTap:
      return launch_fprop_pair(xr, xi, xr_lo, xi_lo, w_packed, y0, y1, pb, t, out_layout, ep, ws,
                               ws_bytes, stream);
    default:
      break;
  }
  t = choose_tiling(pb, true);  // same tiles, fewer loaded rows (boxes past the end skipped)
  const SinglePlan plan = plan_single_cta(pb, t, ws != nullptr ? ws_bytes : 0);
  t.kt = plan.kt;
  t.tiles_n = (pb.k + t.kt - 1) / t.kt;
  FpropParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.y0 = y0;
  prm.y1 = y1;
  set_epilogue(prm, ep);
  prm.status = device_status_ptr();
  if (prm.status == nullptr) return CCV_ERR_CUDA;
  prm.n = pb.n; prm.h = pb.h; prm.w = pb.w; prm.c = pb.c; prm.k = pb.k;
  prm.r = pb.r; prm.s = pb.s; prm.p = pb.p; prm.q = pb.q;
  prm.sh = pb.sh; prm.sw = pb.sw; prm.ph = pb.ph; prm.pw = pb.pw;
  prm.box_p = t.box_p; prm.box_q = t.box_q;
  prm.box_q_log2 = ilog2(t.box_q);
  prm.box_px_log2 = ilog2(t.box_p * t.box_q);
  prm.nb = t.nb;
  prm.tiles_bp = t.tiles_bp; prm.tiles_bq = t.tiles_bq; prm.total_boxes = t.total_boxes;
  prm.tiles_m = t.tiles_m; prm.tiles_n = t.tiles_n;
  prm.ksteps = ((pb.c + kBlockC - 1) / kBlockC) * pb.r * pb.s;
  prm.m_total = static_cast<long long>(pb.n) * pb.p * pb.q;

  int rc;
  const uint64_t cb = static_cast<uint64_t>(pb.c) * 4;
  if (t.flat) {
    const uint64_t dims[2] = {static_cast<uint64_t>(pb.c),
                              static_cast<uint64_t>(pb.n) * pb.h * pb.w};
    const uint64_t strides[1] = {cb};
    const uint32_t box[2] = {kBlockC, kBlockM};
    const uint32_t es[2] = {1, 1};
    if ((rc = encode_tiled(&prm.tm_xr, xr, 2, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi, xi, 2, dims, strides, box, es, 128)) != CCV_OK) return rc;
  } else {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.w),
                              static_cast<uint64_t>(pb.h), static_cast<uint64_t>(pb.n)};
    const uint64_t strides[3] = {cb, cb * pb.w, cb * pb.w * pb.h};
    const uint32_t box[4] = {kBlockC, static_cast<uint32_t>(t.box_q * pb.sw),
                             static_cast<uint32_t>(t.box_p * pb.sh), 1};
    const uint32_t es[4] = {1, static_cast<uint32_t>(pb.sw), static_cast<uint32_t>(pb.sh), 1};
    if ((rc = encode_tiled(&prm.tm_xr, xr, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi, xi, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.k), 3,
                              static_cast<uint64_t>(pb.r) * pb.s};
    const uint64_t strides[3] = {cb, cb * pb.k, cb * pb.k * 3};
    // Two planes (W_re, W_im) of the packed tap per box (Cfg).
    const uint32_t box[4] = {kBlockC, static_cast<uint32_t>(t.kt), 2, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled(&prm.tm_w, w_packed, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
  }
  const long long grid = static_cast<long long>(t.tiles_m) * t.tiles_n;
  if (grid <= 0 || grid > 0x7fffffffLL) {
    return set_error(CCV_ERR_UNSUPPORTED, "problem too large for the grid");
  }
  // Split-K across a cluster of plan.splits CTAs per tile (plan_single_cta);
  // with workspace room the partial sums meet in L2, else over DSMEM.
  prm.splits = 1;
  prm.split_ws = plan.l2 ? static_cast<float*>(ws) : nullptr;
  const bool cplx = out_layout == OUT_COMPLEX_NCHW;
  const int tiles = static_cast<int>(grid);
  if (t.flat) {
    return cplx ? launch_kt<true, true>(t.kt, prm, tiles, plan.splits, stream)
                : launch_kt<true, false>(t.kt, prm, tiles, plan.splits, stream);
  }
  return cplx ? launch_kt<false, true>(t.kt, prm, tiles, plan.splits, stream)
              : launch_kt<false, false>(t.kt, prm, tiles, plan.splits, stream);
}

// ------------------------------------------------------------------ self-test
namespace {
__global__ void ccv_selftest_wait_kernel(int* status, int mirror) {
  __shared__ uint64_t bar;
  const uint32_t b = ptx::smem_u32(&bar);
  if (threadIdx.x == 0) {
    ptx::mbar_init(b, 1);
    ptx::fence_mbar_init();
  }
  ptx::cta_sync();
  if (threadIdx.x == 0) {
    // Nothing ever arrives on `bar`: the bounded wait must give up.
    const bool ok = mirror ? ptx::mbar_wait_bounded<false, true>(b, 0, status, CCV_ERR_DEVICE_TIMEOUT)
                           : ptx::mbar_wait_bounded<false, false>(b, 0, status, CCV_ERR_DEVICE_TIMEOUT);
    if (ok) atomicExch(status, -1);  // impossible completion is itself an error
  }
}
}  // namespace

int launch_selftest_wait(int* status_dev, bool mirror, cudaStream_t stream) {
  ccv_selftest_wait_kernel<<<1, 32, 0, stream>>>(status_dev, mirror ? 1 : 0);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "selftest kernel launch");
  return CCV_OK;
}

}  // namespace ccv
