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
// allocation (both CTAs) and MMA issue (even CTA only), warps 2..5 epilogue;
// LW: warps 6..7 are layout warps (ccv_layout_role.cuh) converting forward()'s
// complex64 input into the planes the producer reads, in the same launch.
#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

#include "ccv_epilogue.cuh"
#include "ccv_fprop_common.cuh"
#include "ccv_internal.h"
#include "ccv_layout_role.cuh"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

constexpr int kThreads2 = 192;
constexpr int kC2 = 32;                 // input channels per K step
constexpr int kRow2 = kC2 * 4;          // 128-byte rows
constexpr int kA2 = kBlockM * kRow2;    // one activation plane of one CTA: 16 KB
constexpr int kTimeout = CCV_ERR_DEVICE_TIMEOUT;
// Stream-K policy threshold of the tap kernel, % (plan_stream_k): above 100,
// i.e. never by default.  Its split lost wherever it was measured on B200:
// stride 2 batch 32 (model gain 11 %) 121.2 -> 141.5 us, batch 8 (model gain
// 34 %) 47.3 -> 61.7 us; one-tap slots make many short pieces whose partial
// sums cost more than the tail they remove.  CCV_STREAMK=1 still forces it.
constexpr int kTapMinSplitGain = 101;

template <int KT>
struct Cfg2 {
  static constexpr int kWSlot = KT * kRow2;              // one weight plane slot
  static constexpr int kStageBytes = 2 * kA2 + 2 * kWSlot;
  static constexpr int kStages = (200 * 1024) / kStageBytes;
  static constexpr int kAccCols = 2 * KT;                // [re | im]
  static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;
  static constexpr int kBarOffset = kStages * kStageBytes;
  static constexpr int kBarBytes = 1024;
  static constexpr int kOutStageOffset = kBarOffset + kBarBytes;  // TMA-store staging
  // Two staging buffers per epilogue warp where they fit beside the stages.
  static constexpr int kOutBufs =
      kOutStageOffset + 2 * kOutStageBytes + 1024 <= 232448 ? 2 : 1;
  static constexpr int kSmemBytes = kOutStageOffset + kOutBufs * kOutStageBytes + 1024;
  static_assert(kStages >= 3, "pipeline too shallow");
  static_assert((2 * kStages + 8 + 4 * kStageBufs) * 8 <= kBarBytes, "barrier block overflow");
  static_assert(kSmemBytes <= 232448, "shared memory");
};

template <int KT, bool FLAT, bool OUT_COMPLEX, bool LW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads2 + (LW ? 32 * kLwWarps : 0), 1)
    ccv_fprop2_tf32_kernel(const __grid_constant__ FpropParams prm) {
  using C = Cfg2<KT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::kBarOffset);
  // full[S] (even CTA), empty[S], tfull[2], tempty[2] (even CTA), done, the
  // TMEM address and flags, then 4 * kStageBufs staging barriers from slot 2S+8.
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
  // kStageBufs per epilogue warp: staging of a split tile's sum after the
  // last unit.
  const uint32_t stage_bar0 = bar_base + 8u * (2 * C::kStages + 8);

  if (threadIdx.x == 0) {
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
    for (int i = 0; i < 4 * kStageBufs; ++i) ptx::mbar_init(stage_bar0 + 8u * i, 1);
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
  // Everything above may overlap the previous kernel on the stream
  // (programmatic dependent launch); global memory is touched only below.
  ptx::griddep_wait();
  ptx::griddep_launch_dependents();
  if (threadIdx.x == 0) flags[0] = *reinterpret_cast<volatile int*>(prm.status) != 0 ? 1 : 0;
  ptx::cta_sync();
  const uint32_t tmem_base = *tmem_holder;
  const bool skip = flags[0] != 0;
  const int rs = prm.r * prm.s;
  const int per_img = prm.tiles_bp * prm.tiles_bq;

  if constexpr (LW) {
    // Every warp converts the first wave's images first (nothing to do
    // before they are there), then takes up its role.
    if (!skip && prm.lw_prefix > 0) layout_warp(prm, lane, true);
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip) {
      uint32_t g = 0;
      bool abort = false;
      int ready_lo = 0, ready_hi = -1;  // images known converted (layout warps)
      UnitCursor cur = unit_cursor(prm, cid);
      WorkUnit wu;
      while (!abort && next_unit(prm, ncl, cur, wu)) {
        const int t = wu.tile;
        const int n_tile = t % prm.tiles_n;
        const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
        const int k0 = n_tile * KT;
        if constexpr (LW) {
          // Images this CTA's rows read: the planes of each are written
          // before the first load.
          int lo, hi;
          if constexpr (FLAT) {
            // Rows m0 .. m0+127 of N*P*Q (1x1, stride 1: input pixel = output
            // pixel); rows past the end read the fill value.
            const long long pq = static_cast<long long>(prm.p) * prm.q;
            const long long m0 = min(static_cast<long long>(half) * kBlockM, prm.m_total - 1);
            const long long m1 = min(static_cast<long long>(half) * kBlockM + kBlockM, prm.m_total) - 1;
            lo = static_cast<int>(m0 / pq);
            hi = static_cast<int>(max(m0, m1) / pq);
          } else {
            lo = min(half * prm.nb, prm.total_boxes - 1) / per_img;
            hi = min(half * prm.nb + prm.nb - 1, prm.total_boxes - 1) / per_img;
          }
          if (lo < ready_lo || hi > ready_hi) {
            for (int im = lo; im <= hi && !abort; ++im) {
              if (im >= ready_lo && im <= ready_hi) continue;
              if (!lw_wait_image(prm, im)) {
                flags[1] = 1;
                abort = true;
              }
            }
            if (abort) break;
            if (lo > ready_hi + 1 || hi < ready_lo - 1) {
              ready_lo = lo;
              ready_hi = hi;
            } else {
              ready_lo = min(ready_lo, lo);
              ready_hi = max(ready_hi, hi);
            }
          }
        }
        for (int v = wu.jbeg; v < wu.jend; ++v, ++g) {
          int ks;
          const int pass = slot_pass(v, prm.ksteps, prm.passes, &ks);
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
      UnitCursor cur = unit_cursor(prm, cid);
      WorkUnit wu;
      while (!abort && next_unit(prm, ncl, cur, wu)) {
        const int buf = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        ++i;
        if (!ptx::mbar_wait_bounded(tempty_bar(buf), (use & 1u) ^ 1u, prm.status, kTimeout)) {
          flags[1] = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * C::kAccCols);
        for (int ks = wu.jbeg; ks < wu.jend; ++ks, ++g) {
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
                               (ks != wu.jbeg || kk != 0) ? 1u : 0u);
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
  } else if (warp <= 5) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t tempty_leader0 = ptx::mapa_shared(tempty_bar(0), 0);
    const uint32_t tempty_leader1 = ptx::mapa_shared(tempty_bar(1), 0);
    int i = 0;
    uint32_t stores = 0;  // TMA-store chunks this warp has committed
    UnitCursor cur = unit_cursor(prm, cid);
    WorkUnit wu;
    while (!skip && next_unit(prm, ncl, cur, wu)) {
      const int buf = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      ++i;
      const bool ok = ptx::mbar_wait_bounded_backoff(tfull_bar(buf), use & 1u, prm.status, kTimeout);
      ptx::tc_fence_after();
      if (!ok) flags[1] = 1;
      const int t = wu.tile;
      const int n_tile = t % prm.tiles_n;
      const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
      int img = 0, op = 0, oq = 0;
      const bool in_tile = tile_row_pixel<FLAT>(prm, half, row, img, op, oq);
      const uint32_t t_acc = t_row + static_cast<uint32_t>(buf * C::kAccCols);
      const uint32_t t_free = buf == 0 ? tempty_leader0 : tempty_leader1;
      if (wu.split && ok && !flags[1]) {
        // After the cluster's last unit the pipeline stages are idle: they
        // stage the split tile's partial sums.
        const bool final_unit = cursor_done(prm, cur);
        constexpr uint32_t per_warp = (static_cast<uint32_t>(C::kBarOffset) / 4u) & ~127u;
        split_piece_epilogue<KT, OUT_COMPLEX>(
            prm, wu, cid, static_cast<int>(rank), quarter, lane, t_acc, n_tile * KT, in_tile, img,
            op, oq, t_free, final_unit ? smem + quarter * per_warp : nullptr, per_warp,
            stage_bar0 + 8u * kStageBufs * static_cast<uint32_t>(quarter));
      } else {
        bool tma_out = false;
        if constexpr (!OUT_COMPLEX) tma_out = prm.out_tma != 0;
        if (tma_out) {
          int c1 = 0, c2 = 0, c3 = 0;
          const bool wv = warp_box_origin<FLAT>(prm, half, quarter * 32, c1, c2, c3) && ok && !flags[1];
          store_accumulator_tma<KT, FLAT, C::kOutBufs>(
              prm, t_acc, n_tile * KT, wv, c1, c2, c3,
              smem + C::kOutStageOffset + quarter * C::kOutBufs * (kOutStageBytes / 4), lane,
              stores);
        } else {
          store_accumulator<KT, OUT_COMPLEX>(prm, t_acc, n_tile * KT, in_tile && ok && !flags[1],
                                             img, op, oq);
        }
        // This warp is done with the accumulator buffer: release it to the MMA.
        ptx::tc_fence_before();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster_relaxed(t_free);
      }
      if (!ok) break;
    }
    // Output stores still in flight complete before the CTA exits.
    if (lane == 0) ptx::bulk_wait_all();
  }
  if constexpr (LW) {
    if (warp >= kThreads2 / 32 && !skip) {
      // ---------------------------------------------------------- layout warps
      layout_warp(prm, lane, false);
    }
  }

  ptx::cta_sync();
  if constexpr (LW) {
    // The last CTA to finish leaves the conversion counters zero.
    if (threadIdx.x == 0) {
      unsigned old;
      asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], 1;"
                   : "=r"(old)
                   : "l"(prm.lw_ctrs + kLwDone)
                   : "memory");
      if (old == 2u * static_cast<unsigned>(ncl) - 1u) {
        for (int i = 0; i < prm.n; ++i) prm.lw_ctrs[kLwFlag0 + i] = 0u;
        prm.lw_ctrs[kLwTicket] = 0u;
        prm.lw_ctrs[kLwPrefixTicket] = 0u;
        prm.lw_ctrs[kLwDone] = 0u;
        __threadfence();
      }
    }
  }
  if (flags[1]) ptx::nanosleep(100000);  // let stray copies of an aborted tile land
  ptx::tc_fence_before();
  ptx::cluster_sync();
  if (warp == 1) {
    __syncwarp();  // tcgen05.dealloc is warp-collective
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, C::kTmemCols);
  }
}

template <int KT, bool FLAT, bool OUT_COMPLEX, bool LW>
int launch2_variant(FpropParams& prm, void* ws, size_t ws_bytes, cudaStream_t stream) {
  using C = Cfg2<KT>;
  auto kern = ccv_fprop2_tf32_kernel<KT, FLAT, OUT_COMPLEX, LW>;
  constexpr int threads = kThreads2 + (LW ? 32 * kLwWarps : 0);
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
    cfg.blockDim = dim3(threads, 1, 1);
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
  const int clusters = cluster_cap(max_clusters[dev & 63]);
  int rc;
  const int launched = launch_clusters(prm, clusters, prm.ksteps * prm.passes, KT, ws, ws_bytes,
                                       stream, &rc, kTapMinSplitGain);
  if (rc != CCV_OK) return rc;
  if (LW) {
    // The stream-K range runs first: the layout warps start at its first image.
    prm.lw_first_img = 0;
    if (prm.sk_slots > 0) {
      const int half = 2 * (prm.sk_start / prm.tiles_n);
      if (FLAT) {
        prm.lw_first_img = static_cast<int>(
            std::min(static_cast<long long>(half) * kBlockM, prm.m_total - 1) /
            (static_cast<long long>(prm.p) * prm.q));
      } else {
        prm.lw_first_img =
            std::min(half * prm.nb, prm.total_boxes - 1) / (prm.tiles_bp * prm.tiles_bq);
      }
    }
    prm.lw_prefix = lw_prefix_tickets(prm, launched, 2LL * kBlockM);
  }
  cudaError_t e = launch_kernel(kern, dim3(2 * launched), dim3(threads), C::kSmemBytes, stream, 0,
                                prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "fprop2 kernel launch");
  return CCV_OK;
}

template <bool FLAT, bool OUT_COMPLEX, bool LW = false>
int launch2_kt(int kt, FpropParams& prm, void* ws, size_t ws_bytes, cudaStream_t stream) {
  switch (kt) {
    case 128: return launch2_variant<128, FLAT, OUT_COMPLEX, LW>(prm, ws, ws_bytes, stream);
    case 64: return launch2_variant<64, FLAT, OUT_COMPLEX, LW>(prm, ws, ws_bytes, stream);
    default: return launch2_variant<32, FLAT, OUT_COMPLEX, LW>(prm, ws, ws_bytes, stream);
  }
}

}  // namespace

int pair_tiles(const Tiling& t) { return ((t.tiles_m + 1) / 2) * t.tiles_n; }

namespace {
constexpr int kMinSkSlots = 2;  // K slots per stream-K range, at least

size_t partial_bytes(int clusters, int kt) {
  // Two partial buffers per cluster (first and last unit of its range), one
  // per CTA of the pair, 128 rows x 2*KT fp32 each.
  return static_cast<size_t>(clusters) * 2 * 2 * kBlockM * 2 * kt * sizeof(float);
}
}  // namespace

size_t pair_split_workspace_bytes(int kt, int tiles, int slots) {
  const int g = std::max(1, device_sm_count() / 2);
  const long long r = std::min<long long>(tiles, g);  // stream-K tiles, at most
  const long long gs = std::min<long long>(g, r * slots / kMinSkSlots);
  if (gs < 2) return 0;
  return partial_bytes(static_cast<int>(gs), kt);
}

int encode_planar_out_maps(FpropParams& prm, float* y0, float* y1, bool flat) {
  prm.out_tma = 0;
  if (knobs().tma_store == 0) return CCV_OK;
  const uint64_t kb = static_cast<uint64_t>(prm.k) * 4;
  int rc;
  if (flat) {
    const uint64_t dims[2] = {static_cast<uint64_t>(prm.k), static_cast<uint64_t>(prm.m_total)};
    const uint64_t strides[1] = {kb};
    const uint32_t box[2] = {16, 32};
    const uint32_t es[2] = {1, 1};
    if ((rc = encode_tiled_ex(&prm.tm_y0, y0, 2, dims, strides, box, es, kSwizzle64, false)) !=
        CCV_OK) {
      return rc;
    }
    if ((rc = encode_tiled_ex(&prm.tm_y1, y1, 2, dims, strides, box, es, kSwizzle64, false)) !=
        CCV_OK) {
      return rc;
    }
  } else {
    // Each epilogue warp's 32 rows must lie in one box of the tile.
    if ((1 << prm.box_px_log2) < 32) return CCV_OK;
    const uint32_t px = static_cast<uint32_t>(std::min(prm.box_q, 32));
    const uint64_t dims[4] = {static_cast<uint64_t>(prm.k), static_cast<uint64_t>(prm.q),
                              static_cast<uint64_t>(prm.p), static_cast<uint64_t>(prm.n)};
    const uint64_t strides[3] = {kb, kb * prm.q, kb * prm.q * prm.p};
    const uint32_t box[4] = {16, px, 32u / px, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled_ex(&prm.tm_y0, y0, 4, dims, strides, box, es, kSwizzle64, false)) !=
        CCV_OK) {
      return rc;
    }
    if ((rc = encode_tiled_ex(&prm.tm_y1, y1, 4, dims, strides, box, es, kSwizzle64, false)) !=
        CCV_OK) {
      return rc;
    }
  }
  prm.out_tma = 1;
  return CCV_OK;
}

int cluster_cap(int max_clusters) {
  // CCV_MAX_CLUSTERS=n caps the persistent grid (testing knob: exercises the
  // stream-K split on small problems).
  const int cap = knobs().max_clusters;
  return cap > 0 ? std::min(max_clusters, cap) : max_clusters;
}

int plan_stream_k(FpropParams& prm, int clusters, int slots, int kt, void* ws, size_t ws_bytes,
                  cudaStream_t stream, int min_gain_pct) {
  prm.slots_per_tile = slots;
  prm.sk_start = prm.num_tiles;
  prm.sk_slots = 0;
  prm.sk_clusters = 1;
  prm.split_ws = nullptr;
  prm.split_count = nullptr;
  // CCV_STREAMK=0 disables the split, =1 takes it whenever it is possible
  // (testing knob); by default the model below decides.
  const int mode = knobs().streamk;
  if (mode == 0 || ws == nullptr || clusters < 2 || slots < kMinSkSlots) return 0;
  const int T = prm.num_tiles;
  const int r = T % clusters;
  if (r == 0) return 0;
  const long long X = static_cast<long long>(r) * slots;
  if (X > 0x7fffffffLL) return 0;
  const int gs = static_cast<int>(std::min<long long>(clusters, X / kMinSkSlots));
  if (gs < 2) return 0;
  const long long per_range = (X + gs - 1) / gs;
  // Default: split when the slot-count model saves at least min_gain_pct %
  // of the kernel (whole tiles: (q + 1) * L slot times on the busiest
  // cluster; split: q * L + per_range).  The model leaves out the partial
  // sums' traffic, the reduction and the unit switches, which cost B200
  // measurements 10-30 us per launch: the halo kernel (3-tap slots) splits
  // at >= 10 % (batch 8 and 16 of the 56x56 layer gain); the tap kernel
  // (one-tap slots) passes a threshold no model gain reaches.
  const long long q = T / clusters;
  const long long dp_time = (q + 1) * slots;
  const long long sk_time = q * slots + per_range;
  if (mode != 1 && (slots < 4 || (dp_time - sk_time) * 100 < dp_time * min_gain_pct)) return 0;
  const size_t pbytes = partial_bytes(gs, kt);
  if (ws_bytes < pbytes || (reinterpret_cast<uintptr_t>(ws) & 255u) != 0) return 0;
  if (r * 8 > kSkCounterWords) return 0;
  unsigned* counters = acquire_counter_set(stream);
  if (counters == nullptr) return 0;
  prm.sk_start = T - r;
  prm.sk_slots = X;
  prm.sk_clusters = gs;
  prm.split_ws = static_cast<float*>(ws);
  prm.split_count = counters;
  return r * 8;
}

int launch_clusters(FpropParams& prm, int clusters, int slots, int kt, void* ws, size_t ws_bytes,
                    cudaStream_t stream, int* rc, int min_gain_pct) {
  *rc = CCV_OK;
  clusters = std::max(1, clusters);
  // Stream-K counters come zeroed from the library's counter sets (no memset).
  if (plan_stream_k(prm, clusters, slots, kt, ws, ws_bytes, stream, min_gain_pct) > 0) {
    return clusters;
  }
  return std::max(1, std::min(prm.num_tiles, clusters));
}

int launch_fprop_pair(const float* xr, const float* xi, const float* xr_lo, const float* xi_lo,
                      const float* w_packed, float* y0, float* y1, const Problem& pb,
                      const Tiling& t, OutLayout out_layout, const Epilogue& ep, void* ws,
                      size_t ws_bytes, cudaStream_t stream, const float* lw_src,
                      const float* lw_pr, const float* lw_pi) {
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
  if (!cplx && (rc = encode_planar_out_maps(prm, y0, y1, t.flat)) != CCV_OK) return rc;
  if (lw_src != nullptr || lw_pr != nullptr) {
    // Layout warps write xr/xi (and the remainder planes) from lw_src
    // (complex64 NCHW) or from the planes lw_pr/lw_pi (fp32 NHWC).
    if ((lw_pr == nullptr && !cplx) || pb.n > kSkCounterWords - kLwFlag0) {
      return set_error(CCV_ERR_UNSUPPORTED, "no layout warps for this problem");
    }
    prm.xc = lw_src;
    prm.lw_pr = lw_pr;
    prm.lw_pi = lw_pi;
    prm.lw_xr = const_cast<float*>(xr);
    prm.lw_xi = const_cast<float*>(xi);
    prm.lw_xr_lo = const_cast<float*>(xr_lo);
    prm.lw_xi_lo = const_cast<float*>(xi_lo);
    prm.lw_ctrs = acquire_counter_set(stream);
    if (prm.lw_ctrs == nullptr) return kNoCounterSet;
    if (cplx) {
      return t.flat ? launch2_kt<true, true, true>(t.kt, prm, ws, ws_bytes, stream)
                    : launch2_kt<false, true, true>(t.kt, prm, ws, ws_bytes, stream);
    }
    return t.flat ? launch2_kt<true, false, true>(t.kt, prm, ws, ws_bytes, stream)
                  : launch2_kt<false, false, true>(t.kt, prm, ws, ws_bytes, stream);
  }
  if (t.flat) {
    return cplx ? launch2_kt<true, true>(t.kt, prm, ws, ws_bytes, stream)
                : launch2_kt<true, false>(t.kt, prm, ws, ws_bytes, stream);
  }
  return cplx ? launch2_kt<false, true>(t.kt, prm, ws, ws_bytes, stream)
              : launch2_kt<false, false>(t.kt, prm, ws, ws_bytes, stream);
}

}  // namespace ccv
