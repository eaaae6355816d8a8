// Complex Conv2d forward, CTA-pair kernel family for large problems.
//
// Same implicit planar-complex GEMM as ccv_fprop.cu (M = N*P*Q pixels,
// N = K output channels, reduction R*S*C; the reference's four real products
// of threadblock/implicit_planar_cgemm_multistage.h:251-271), scheduled for
// throughput on B200:
//   * a cluster of two CTAs issues tcgen05.mma.cta_group::2 with M = 256:
//     each CTA holds 128 output pixels of the tile (its A rows) and HALF of
//     each weight operand, so per CTA the weight bytes per K step drop from
//     three planes to two:
//         B_top = [W_re ; W_im]   CTA0 holds W_re, CTA1 holds W_im
//         B_bot = [-W_im ; W_re]  CTA0 holds -W_im, CTA1 holds W_re
//     D[:, 0:2KT] += A_re * B_top^T + A_im * B_bot^T   ([re | im] in TMEM)
//   * 32 input channels per K step: 128-byte TMA rows, 128-byte swizzle;
//   * persistent: each cluster walks tiles cluster_id, + num_clusters, ...;
//   * two TMEM accumulators, so the epilogue of one tile overlaps the
//     mainloop of the next.
// Each CTA TMA-loads only its own half of every operand (no multicast);
// transaction bytes of both CTAs complete on the even CTA's "full" barrier.
//
// Warp roles per CTA (192 threads): warp 0 TMA producer, warp 1 TMEM
// allocation (both CTAs) and MMA issue (even CTA only), warps 2..5 epilogue.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "ccv_epilogue.cuh"
#include "ccv_fprop_common.cuh"
#include "ccv_internal.h"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

constexpr int kThreads2 = 192;
constexpr int kC2 = 32;                 // input channels per K step
constexpr int kRow2 = kC2 * 4;          // 128-byte rows
constexpr int kA2 = kBlockM * kRow2;    // one activation plane of one CTA: 16 KB
constexpr int kTimeout = CCV_ERR_DEVICE_TIMEOUT;

template <int KT>
struct Cfg2 {
  static constexpr int kWSlot = KT * kRow2;              // one weight plane slot
  static constexpr int kStageBytes = 2 * kA2 + 2 * kWSlot;
  static constexpr int kStages = (200 * 1024) / kStageBytes;
  static constexpr int kAccCols = 2 * KT;                // [re | im]
  static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kSmemBytes = kBarOffset + 256 + 1024;
  static_assert(kStages >= 3, "pipeline too shallow");
};

template <int KT, bool FLAT, bool OUT_COMPLEX>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads2, 1)
    ccv_fprop2_tf32_kernel(const __grid_constant__ FpropParams prm) {
  using C = Cfg2<KT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  // full[S] (even CTA), empty[S], tfull[2], tempty[2] (even CTA), done
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 2 * C::kStages + 5);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] skip, [1] abort

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = static_cast<int>(ptx::cluster_id_x());
  const int ncl = static_cast<int>(ptx::nclusters_x());
  const uint32_t smem_base = ptx::smem_u32(smem);
  const uint32_t bar_base = ptx::smem_u32(bars);
  auto full_bar = [&](int i) { return bar_base + 8u * i; };
  auto empty_bar = [&](int i) { return bar_base + 8u * (C::kStages + i); };
  auto tfull_bar = [&](int b) { return bar_base + 8u * (2 * C::kStages + b); };
  auto tempty_bar = [&](int b) { return bar_base + 8u * (2 * C::kStages + 2 + b); };
  const uint32_t done_bar = bar_base + 8u * (2 * C::kStages + 4);

  if (threadIdx.x == 0) {
    flags[0] = *reinterpret_cast<volatile int*>(prm.status) != 0 ? 1 : 0;
    flags[1] = 0;
    for (int i = 0; i < C::kStages; ++i) {
      ptx::mbar_init(full_bar(i), 1);
      ptx::mbar_init(empty_bar(i), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(tfull_bar(b), 1);
      ptx::mbar_init(tempty_bar(b), 8);  // 4 epilogue warps x 2 CTAs
    }
    ptx::mbar_init(done_bar, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&prm.tm_xr);
    ptx::prefetch_tmap(&prm.tm_xi);
    ptx::prefetch_tmap(&prm.tm_w);
    if (prm.passes > 1) {
      ptx::prefetch_tmap(&prm.tm_xr_lo);
      ptx::prefetch_tmap(&prm.tm_xi_lo);
    }
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), C::kTmemCols);
    ptx::tmem_relinquish_pair();
  }
  ptx::tc_fence_before();
  ptx::cluster_sync();
  ptx::tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;
  const bool skip = flags[0] != 0;
  const int rs = prm.r * prm.s;
  const int per_img = prm.tiles_bp * prm.tiles_bq;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip) {
      uint32_t g = 0;
      bool abort = false;
      for (int t = cid; t < prm.num_tiles && !abort; t += ncl) {
        const int n_tile = t % prm.tiles_n;
        const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
        const int k0 = n_tile * KT;
        for (int v = 0; v < prm.ksteps * prm.passes; ++v, ++g) {
          const int ks = v / prm.passes;
          const int pass = v - ks * prm.passes;
          const CUtensorMap* mr = pass == 2 ? &prm.tm_xr_lo : &prm.tm_xr;
          const CUtensorMap* mi = pass == 2 ? &prm.tm_xi_lo : &prm.tm_xi;
          const int stage = static_cast<int>(g % C::kStages);
          const uint32_t phase = (g / C::kStages) & 1u;
          if (!ptx::mbar_wait_bounded(empty_bar(stage), phase ^ 1u, prm.status, kTimeout) ||
              flags[1]) {
            flags[1] = 1;
            abort = true;
            break;
          }
          if (leader) ptx::mbar_arrive_expect_tx(full_bar(stage), 2 * C::kStageBytes);
          const uint32_t fb = ptx::mapa_shared(full_bar(stage), 0);
          const int cb = ks / rs;
          const int tap = ks - cb * rs;
          const int rr = tap / prm.s;
          const int ss = tap - rr * prm.s;
          const int c0 = cb * kC2;
          const uint32_t a_r = smem_base + stage * C::kStageBytes;
          const uint32_t a_i = a_r + kA2;
          const uint32_t w_x = a_i + kA2;
          const uint32_t w_y = w_x + C::kWSlot;
          if constexpr (FLAT) {
            ptx::tma_load_2d_pair(a_r, mr, fb, c0, half * kBlockM);
            ptx::tma_load_2d_pair(a_i, mi, fb, c0, half * kBlockM);
          } else {
            const uint32_t box_bytes = (1u << prm.box_px_log2) * kRow2;
            for (int b = 0; b < prm.nb; ++b) {
              // Boxes past the end repeat the last box; their rows are not stored.
              const int gb = min(half * prm.nb + b, prm.total_boxes - 1);
              const int img = gb / per_img;
              const int rem = gb - img * per_img;
              const int bp = rem / prm.tiles_bq;
              const int bq = rem - bp * prm.tiles_bq;
              const int wc = bq * prm.box_q * prm.sw - prm.pw + ss;
              const int hc = bp * prm.box_p * prm.sh - prm.ph + rr;
              ptx::tma_load_4d_pair(a_r + b * box_bytes, mr, fb, c0, wc, hc, img);
              ptx::tma_load_4d_pair(a_i + b * box_bytes, mi, fb, c0, wc, hc, img);
            }
          }
          // Packed planes per tap: 0 = -W_im, 1 = W_re, 2 = W_im.
          // CTA0: X = W_re, Y = -W_im.  CTA1: X = W_im, Y = W_re.
          // Pass 1 of 3xTF32 reads the weight remainder image.
          const int wtap = pass == 1 ? tap + rs : tap;
          ptx::tma_load_4d_pair(w_x, &prm.tm_w, fb, c0, k0, leader ? 1 : 2, wtap);
          ptx::tma_load_4d_pair(w_y, &prm.tm_w, fb, c0, k0, leader ? 0 : 1, wtap);
        }
      }
      if (leader) {
        // Drain: every issued stage's bytes (both CTAs) have landed.
        for (uint32_t j = 0; j < static_cast<uint32_t>(C::kStages) && j < g; ++j) {
          const uint32_t gg = g - 1 - j;
          ptx::mbar_wait_bounded(full_bar(static_cast<int>(gg % C::kStages)),
                                 (gg / C::kStages) & 1u, prm.status, kTimeout);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0 && !skip) {
      constexpr uint32_t idesc = ptx::idesc_tf32(2 * kBlockM, 2 * KT, false);
      uint32_t g = 0;
      int i = 0;
      bool abort = false;
      for (int t = cid; t < prm.num_tiles && !abort; t += ncl, ++i) {
        const int buf = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        if (!ptx::mbar_wait_bounded(tempty_bar(buf), (use & 1u) ^ 1u, prm.status, kTimeout)) {
          flags[1] = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * C::kAccCols);
        for (int ks = 0; ks < prm.ksteps * prm.passes; ++ks, ++g) {
          const int stage = static_cast<int>(g % C::kStages);
          const uint32_t phase = (g / C::kStages) & 1u;
          if (!ptx::mbar_wait_bounded(full_bar(stage), phase, prm.status, kTimeout)) {
            flags[1] = 1;
            abort = true;
            break;
          }
          ptx::tc_fence_after();
          const uint32_t a_r = smem_base + stage * C::kStageBytes;
          const uint32_t a_i = a_r + kA2;
          const uint32_t w_x = a_i + kA2;
          const uint32_t w_y = w_x + C::kWSlot;
#pragma unroll
          for (int kk = 0; kk < kC2 / 8; ++kk) {
            const uint32_t koff = kk * 32;
            ptx::mma_tf32_pair(d, ptx::desc_kmajor_sw128(a_r + koff),
                               ptx::desc_kmajor_sw128(w_x + koff), idesc,
                               (ks | kk) != 0 ? 1u : 0u);
            ptx::mma_tf32_pair(d, ptx::desc_kmajor_sw128(a_i + koff),
                               ptx::desc_kmajor_sw128(w_y + koff), idesc, 1u);
          }
          ptx::mma_commit_pair(empty_bar(stage));
        }
        ptx::mma_commit_pair(tfull_bar(buf));
      }
      // All issued MMAs complete before teardown.
      ptx::mma_commit_pair(done_bar);
      ptx::mbar_wait_bounded(done_bar, 0, prm.status, kTimeout);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t tempty_leader0 = ptx::mapa_shared(tempty_bar(0), 0);
    const uint32_t tempty_leader1 = ptx::mapa_shared(tempty_bar(1), 0);
    int i = 0;
    for (int t = cid; t < prm.num_tiles && !skip; t += ncl, ++i) {
      const int buf = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      const bool ok = ptx::mbar_wait_bounded_backoff(tfull_bar(buf), use & 1u, prm.status, kTimeout);
      ptx::tc_fence_after();
      if (!ok) flags[1] = 1;
      const int n_tile = t % prm.tiles_n;
      const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
      int img = 0, op = 0, oq = 0;
      const bool valid = tile_row_pixel<FLAT>(prm, half, row, img, op, oq) && ok && !flags[1];
      store_accumulator<KT, OUT_COMPLEX>(prm, t_row + static_cast<uint32_t>(buf * C::kAccCols),
                                         n_tile * KT, valid, img, op, oq);
      // This warp is done with the accumulator buffer: release it to the MMA.
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(buf == 0 ? tempty_leader0 : tempty_leader1);
      if (!ok) break;
    }
  }

  __syncthreads();
  if (flags[1]) ptx::nanosleep(100000);  // let stray copies of an aborted tile land
  ptx::tc_fence_before();
  ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

template <int KT, bool FLAT, bool OUT_COMPLEX>
int launch2_variant(const FpropParams& prm, cudaStream_t stream) {
  using C = Cfg2<KT>;
  auto kern = ccv_fprop2_tf32_kernel<KT, FLAT, OUT_COMPLEX>;
  static std::once_flag once[64];
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t err = cudaSuccess;
  std::call_once(once[dev & 63], [&]() {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (err != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 148, 1, 1);
    cfg.blockDim = dim3(kThreads2, 1, 1);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) {
      max_clusters[dev & 63] = n;
    } else {
      cudaGetLastError();
      max_clusters[dev & 63] = device_sm_count() / 2;
    }
  });
  if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(fprop2)");
  const int clusters = std::max(1, std::min(prm.num_tiles, max_clusters[dev & 63]));
  kern<<<2 * clusters, kThreads2, C::kSmemBytes, stream>>>(prm);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "fprop2 kernel launch");
  return CCV_OK;
}

template <bool FLAT, bool OUT_COMPLEX>
int launch2_kt(int kt, const FpropParams& prm, cudaStream_t stream) {
  switch (kt) {
    case 128: return launch2_variant<128, FLAT, OUT_COMPLEX>(prm, stream);
    case 64: return launch2_variant<64, FLAT, OUT_COMPLEX>(prm, stream);
    default: return launch2_variant<32, FLAT, OUT_COMPLEX>(prm, stream);
  }
}

}  // namespace

int pair_tiles(const Tiling& t) { return ((t.tiles_m + 1) / 2) * t.tiles_n; }

int launch_fprop_pair(const float* xr, const float* xi, const float* xr_lo, const float* xi_lo,
                      const float* w_packed, float* y0, float* y1, const Problem& pb,
                      const Tiling& t, OutLayout out_layout, cudaStream_t stream) {
  FpropParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.y0 = y0;
  prm.y1 = y1;
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
  prm.ksteps = ((pb.c + kC2 - 1) / kC2) * pb.r * pb.s;
  prm.m_total = static_cast<long long>(pb.n) * pb.p * pb.q;
  prm.num_tiles = pair_tiles(t);
  const bool split = xr_lo != nullptr;
  prm.passes = split ? 3 : 1;
  if (!split) {
    xr_lo = xr;
    xi_lo = xi;
  }

  int rc;
  const uint64_t cb = static_cast<uint64_t>(pb.c) * 4;
  if (t.flat) {
    const uint64_t dims[2] = {static_cast<uint64_t>(pb.c),
                              static_cast<uint64_t>(pb.n) * pb.h * pb.w};
    const uint64_t strides[1] = {cb};
    const uint32_t box[2] = {kC2, kBlockM};
    const uint32_t es[2] = {1, 1};
    if ((rc = encode_tiled(&prm.tm_xr, xr, 2, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi, xi, 2, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xr_lo, xr_lo, 2, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi_lo, xi_lo, 2, dims, strides, box, es, 128)) != CCV_OK) return rc;
  } else {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.w),
                              static_cast<uint64_t>(pb.h), static_cast<uint64_t>(pb.n)};
    const uint64_t strides[3] = {cb, cb * pb.w, cb * pb.w * pb.h};
    const uint32_t box[4] = {kC2, static_cast<uint32_t>(t.box_q * pb.sw),
                             static_cast<uint32_t>(t.box_p * pb.sh), 1};
    const uint32_t es[4] = {1, static_cast<uint32_t>(pb.sw), static_cast<uint32_t>(pb.sh), 1};
    if ((rc = encode_tiled(&prm.tm_xr, xr, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi, xi, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xr_lo, xr_lo, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi_lo, xi_lo, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.k), 3,
                              static_cast<uint64_t>(pb.r) * pb.s * (split ? 2 : 1)};
    const uint64_t strides[3] = {cb, cb * pb.k, cb * pb.k * 3};
    const uint32_t box[4] = {kC2, static_cast<uint32_t>(t.kt), 1, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled(&prm.tm_w, w_packed, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
  }
  const bool cplx = out_layout == OUT_COMPLEX_NCHW;
  if (t.flat) {
    return cplx ? launch2_kt<true, true>(t.kt, prm, stream)
                : launch2_kt<true, false>(t.kt, prm, stream);
  }
  return cplx ? launch2_kt<false, true>(t.kt, prm, stream)
              : launch2_kt<false, false>(t.kt, prm, stream);
}

}  // namespace ccv
