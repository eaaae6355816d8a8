// Complex Conv2d forward, CTA-pair kernel with halo reuse of the activations.
//
// Same math, pair MMA and epilogue as ccv_fprop2.cu, for stride-1 problems
// with an R x S filter (R*S > 1).  A CTA tile is one box of box_p x box_q
// output pixels (box_q a multiple of 8, 128 pixels).  For input-channel
// block cb (32 channels) and filter column s, one TMA load per plane brings
//     rows p0-pad_h .. p0-pad_h+box_p+R-2,  columns q0-pad_w+s .. +box_q-1
// into an "A slot" laid out as (box_p+R-1)*box_q rows of 128 bytes.  The A
// operand of filter tap (r, s) is that slot starting at row r*box_q: R taps
// read one slot, so activation bytes per K step drop from 128 rows per plane
// to (box_p+R-1)*box_q/R.  Weights stream per tap as in the tap kernel.
// Two rings: A slots (one per (cb, s)) and weight stages (one per tap).
//
// LW (layout warps): two extra warps per CTA convert the whole complex64
// NCHW batch into fp32 NHWC planes in the workspace, image by image, while
// the pair MMA runs; the producer waits for an image's planes before its
// first TMA load from them (ccv_layout_role.cuh).  One launch, TMA-fed MMA.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "ccv_epilogue.cuh"
#include "ccv_fprop_common.cuh"
#include "ccv_internal.h"
#include "ccv_layout_role.cuh"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

constexpr int kThreadsH = 192;
constexpr int kCH = 32;               // input channels per K step
constexpr int kRowH = kCH * 4;        // 128-byte rows
constexpr int kMaxASlots = 4;
constexpr int kMaxWStages = 8;
constexpr int kBarBytes = 1024;       // barrier block at the start of the carve-out
constexpr int kLwTmaBar = 100;        // TMA prefix: kLwBoxBufs barriers, then 20 words
static_assert(8 * (kLwTmaBar + kLwBoxBufs) + 4 * (kLwBoxBufs + kLwTmaMaxImages) <= kBarBytes,
              "barrier block overflow");
static_assert(8 * (32 + 4 * kStageBufs) <= kBarBytes, "barrier block overflow");
constexpr int kSmemDataBudget = 232448 - kBarBytes - 1024;  // minus alignment slack
constexpr int kTimeoutH = CCV_ERR_DEVICE_TIMEOUT;

// NSUB: 128-row sub-boxes per CTA tile (2 for KT <= 64: two accumulators
// share every weight stage, halving weight bytes per MMA).
template <int KT, int NSUB>
struct CfgH {
  static constexpr int kAccCols = 2 * KT;            // one sub-box: [re | im]
  static constexpr int kTileCols = NSUB * kAccCols;  // one tile buffer
  static constexpr int kTmemCols = 2 * kTileCols < 32 ? 32 : 2 * kTileCols;
  static constexpr int kWStageBytes = 2 * KT * kRowH;
  static_assert(2 * kTileCols <= 512, "TMEM");
};

template <bool LW>
constexpr int halo_threads() {
  return kThreadsH + (LW ? 32 * kLwWarps : 0);
}

template <int KT, bool OUT_COMPLEX, int NSUB, bool LW>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(halo_threads<LW>(), 1)
    ccv_fprop2h_tf32_kernel(const __grid_constant__ FpropParams prm) {
  using C = CfgH<KT, NSUB>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base);
  // afull[4], aempty[4], wfull[8], wempty[8], tfull[2], tempty[2], done,
  // then the TMEM address and flags; staging barriers from slot 32.
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 29);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] skip, [1] abort
  uint8_t* data = base + kBarBytes;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = static_cast<int>(ptx::cluster_id_x());
  const int ncl = static_cast<int>(ptx::nclusters_x());
  const uint32_t bar_base = ptx::smem_u32(bars);
  auto afull = [&](int i) { return bar_base + 8u * i; };
  auto aempty = [&](int i) { return bar_base + 8u * (kMaxASlots + i); };
  auto wfull = [&](int i) { return bar_base + 8u * (2 * kMaxASlots + i); };
  auto wempty = [&](int i) { return bar_base + 8u * (2 * kMaxASlots + kMaxWStages + i); };
  auto tfull = [&](int b) { return bar_base + 8u * (2 * kMaxASlots + 2 * kMaxWStages + b); };
  auto tempty = [&](int b) { return bar_base + 8u * (2 * kMaxASlots + 2 * kMaxWStages + 2 + b); };
  const uint32_t done_bar = bar_base + 8u * (2 * kMaxASlots + 2 * kMaxWStages + 4);
  // kStageBufs per epilogue warp: staging of a split tile's sum after the
  // last unit.
  const uint32_t stage_bar0 = bar_base + 8u * 32;

  const int SA = prm.a_slots;
  const int SW = prm.w_stages;
  const uint32_t a_base = ptx::smem_u32(data);
  const uint32_t w_base = a_base + static_cast<uint32_t>(SA * prm.a_slot_bytes);
  const uint32_t a_plane_bytes = static_cast<uint32_t>(prm.a_slot_bytes / 2);
  // TMA-store staging of the planar epilogue, after the weight stages.
  uint8_t* out_stage = data + SA * prm.a_slot_bytes + SW * prm.w_stage_bytes;

  if (threadIdx.x == 0) {
    flags[1] = 0;
    for (int i = 0; i < kMaxASlots; ++i) {
      ptx::mbar_init(afull(i), 1);
      ptx::mbar_init(aempty(i), 1);
    }
    for (int i = 0; i < SW; ++i) {
      ptx::mbar_init(wfull(i), 1);
      ptx::mbar_init(wempty(i), 1);
    }
    for (int b = 0; b < 2; ++b) {
      ptx::mbar_init(tfull(b), 1);
      ptx::mbar_init(tempty(b), 8);  // 4 epilogue warps x 2 CTAs
    }
    ptx::mbar_init(done_bar, 1);
    if (LW) {
      for (int i = 0; i < kLwBoxBufs; ++i) ptx::mbar_init(bar_base + 8u * (kLwTmaBar + i), 1);
    }
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
  const int per_img = prm.tiles_bp * prm.tiles_bq;
  const int per_pass = ((prm.c + kCH - 1) / kCH) * prm.s;  // K slots per precision pass

  const int ucid = cid, uncl = ncl;

  if constexpr (LW) {
    // Every warp converts the first wave's images first (nothing to do
    // before they are there), then takes up its role.
    if (!skip && prm.lw_tma_images > 0) {
      // The operand rings are idle until the producer starts: they hold the
      // TMA prefix's boxes, handed back to TMA by the proxy fence and the
      // barrier below.
      if (!lw_tma_prefix(prm, data, bar_base + 8u * kLwTmaBar,
                         reinterpret_cast<unsigned*>(bars + kLwTmaBar + kLwBoxBufs))) {
        flags[1] = 1;
      }
      ptx::fence_proxy_async_shared();
      ptx::cta_sync();
    } else if (!skip && prm.lw_prefix > 0) {
      layout_warp(prm, lane, true);
    }
  }

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip) {
      uint32_t ga = 0, gw = 0;
      int ready_img = -1;
      bool abort = false;
      UnitCursor cur = unit_cursor(prm, ucid);
      WorkUnit wu;
      while (!abort && next_unit(prm, uncl, cur, wu)) {
        const int t = wu.tile;
        const int n_tile = t % prm.tiles_n;
        const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
        // Boxes past the end repeat the last box; their rows are not stored.
        const int gb = min(half, prm.total_boxes - 1);
        const int img = gb / per_img;
        const int rem = gb - img * per_img;
        const int bp = rem / prm.tiles_bq;
        const int bq = rem - bp * prm.tiles_bq;
        const int h0 = bp * prm.box_p - prm.ph;
        const int w0 = bq * prm.box_q - prm.pw;
        const int k0 = n_tile * KT;
        if constexpr (LW) {
          // This image's planes are written (tiles run in image order).
          if (img != ready_img) {
            if (!lw_wait_image(prm, img)) {
              flags[1] = 1;
              abort = true;
              break;
            }
            ready_img = img;
          }
        }
        for (int j = wu.jbeg; j < wu.jend && !abort; ++j, ++ga) {
          // Slot j: precision pass (slot_pass), channel block cb, filter
          // column ss.
          int rest;
          const int pass = slot_pass(j, per_pass, prm.passes, &rest);
          const int cb = rest / prm.s;
          const int ss = rest - cb * prm.s;
          const int c0 = cb * kCH;
          const CUtensorMap* mr = pass == 2 ? &prm.tm_xr_lo : &prm.tm_xr;
          const CUtensorMap* mi = pass == 2 ? &prm.tm_xi_lo : &prm.tm_xi;
          {
            const int slot = static_cast<int>(ga % SA);
            const uint32_t ph = (ga / SA) & 1u;
            if (!ptx::mbar_wait_bounded(aempty(slot), ph ^ 1u, prm.status, kTimeoutH) ||
                flags[1]) {
              flags[1] = 1;
              abort = true;
              break;
            }
            if (leader) ptx::mbar_arrive_expect_tx(afull(slot), 2u * prm.a_slot_bytes);
            const uint32_t fb = ptx::mapa_shared(afull(slot), 0);
            const uint32_t a_r = a_base + static_cast<uint32_t>(slot * prm.a_slot_bytes);
            ptx::tma_load_4d_pair(a_r, mr, fb, c0, w0 + ss, h0, img);
            ptx::tma_load_4d_pair(a_r + a_plane_bytes, mi, fb, c0, w0 + ss, h0, img);
          }
          for (int rr = 0; rr < prm.r; ++rr, ++gw) {
            const int st = static_cast<int>(gw % SW);
            const uint32_t pw_ = (gw / SW) & 1u;
            if (!ptx::mbar_wait_bounded(wempty(st), pw_ ^ 1u, prm.status, kTimeoutH) ||
                flags[1]) {
              flags[1] = 1;
              abort = true;
              break;
            }
            if (leader) ptx::mbar_arrive_expect_tx(wfull(st), 2u * C::kWStageBytes);
            const uint32_t wb = ptx::mapa_shared(wfull(st), 0);
            const uint32_t w_x = w_base + static_cast<uint32_t>(st * C::kWStageBytes);
            const uint32_t w_y = w_x + C::kWStageBytes / 2;
            const int tap = rr * prm.s + ss + (pass == 1 ? prm.r * prm.s : 0);
            // Packed planes per tap: 0 = -W_im, 1 = W_re, 2 = W_im.
            // CTA0: X = W_re, Y = -W_im.  CTA1: X = W_im, Y = W_re.
            ptx::tma_load_4d_pair(w_x, &prm.tm_w, wb, c0, k0, leader ? 1 : 2, tap);
            ptx::tma_load_4d_pair(w_y, &prm.tm_w, wb, c0, k0, leader ? 0 : 1, tap);
          }
        }
      }
      if (leader) {
        // Drain: every issued slot and stage (both CTAs) has landed.
        for (uint32_t j = 0; j < static_cast<uint32_t>(SA) && j < ga; ++j) {
          const uint32_t g = ga - 1 - j;
          ptx::mbar_wait_bounded(afull(static_cast<int>(g % SA)), (g / SA) & 1u, prm.status,
                                 kTimeoutH);
        }
        for (uint32_t j = 0; j < static_cast<uint32_t>(SW) && j < gw; ++j) {
          const uint32_t g = gw - 1 - j;
          ptx::mbar_wait_bounded(wfull(static_cast<int>(g % SW)), (g / SW) & 1u, prm.status,
                                 kTimeoutH);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0 && !skip) {
      constexpr uint32_t idesc = ptx::idesc_tf32(2 * kBlockM, 2 * KT, false);
      const uint32_t tap_row_bytes = static_cast<uint32_t>(prm.box_q * kRowH);
      uint32_t ga = 0, gw = 0;
      int i = 0;
      bool abort = false;
      UnitCursor cur = unit_cursor(prm, ucid);
      WorkUnit wu;
      while (!abort && next_unit(prm, uncl, cur, wu)) {
        const int buf = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        ++i;
        if (!ptx::mbar_wait_bounded(tempty(buf), (use & 1u) ^ 1u, prm.status, kTimeoutH)) {
          flags[1] = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * C::kTileCols);
        bool first = true;
        for (int j = wu.jbeg; j < wu.jend && !abort; ++j, ++ga) {
          const int slot = static_cast<int>(ga % SA);
          if (!ptx::mbar_wait_bounded(afull(slot), (ga / SA) & 1u, prm.status, kTimeoutH)) {
            flags[1] = 1;
            abort = true;
            break;
          }
          const uint32_t a_r0 = a_base + static_cast<uint32_t>(slot * prm.a_slot_bytes);
          for (int rr = 0; rr < prm.r; ++rr, ++gw) {
            const int st = static_cast<int>(gw % SW);
            if (!ptx::mbar_wait_bounded(wfull(st), (gw / SW) & 1u, prm.status, kTimeoutH)) {
              flags[1] = 1;
              abort = true;
              break;
            }
            ptx::tc_fence_after();
            const uint32_t a_r = a_r0 + static_cast<uint32_t>(rr) * tap_row_bytes;
            const uint32_t a_i = a_r + a_plane_bytes;
            const uint32_t w_x = w_base + static_cast<uint32_t>(st * C::kWStageBytes);
            const uint32_t w_y = w_x + C::kWStageBytes / 2;
#pragma unroll
            for (int kk = 0; kk < kCH / 8; ++kk) {
              const uint32_t koff = kk * 32;
#pragma unroll
              for (int sb = 0; sb < NSUB; ++sb) {
                // Sub-box sb: slot rows from 128*sb on, accumulator columns
                // from sb * 2*KT on.
                const uint32_t aoff = koff + static_cast<uint32_t>(sb) * kBlockM * kRowH;
                const uint32_t dsb = d + static_cast<uint32_t>(sb * C::kAccCols);
                ptx::mma_tf32_pair(dsb, ptx::desc_kmajor_sw128(a_r + aoff),
                                   ptx::desc_kmajor_sw128(w_x + koff), idesc, first ? 0u : 1u);
                ptx::mma_tf32_pair(dsb, ptx::desc_kmajor_sw128(a_i + aoff),
                                   ptx::desc_kmajor_sw128(w_y + koff), idesc, 1u);
              }
              first = false;
            }
            ptx::mma_commit_pair(wempty(st));
          }
          ptx::mma_commit_pair(aempty(slot));
        }
        ptx::mma_commit_pair(tfull(buf));
      }
      // All issued MMAs complete before teardown.
      ptx::mma_commit_pair(done_bar);
      ptx::mbar_wait_bounded(done_bar, 0, prm.status, kTimeoutH);
    }
    __syncwarp();
  } else if (warp <= 5) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t tempty_leader0 = ptx::mapa_shared(tempty(0), 0);
    const uint32_t tempty_leader1 = ptx::mapa_shared(tempty(1), 0);
    int i = 0;
    uint32_t stores = 0;  // TMA-store chunks this warp has committed
    UnitCursor cur = unit_cursor(prm, ucid);
    WorkUnit wu;
    while (!skip && next_unit(prm, uncl, cur, wu)) {
      const int buf = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      ++i;
      const bool ok = ptx::mbar_wait_bounded_backoff(tfull(buf), use & 1u, prm.status, kTimeoutH);
      ptx::tc_fence_after();
      if (!ok) flags[1] = 1;
      const int t = wu.tile;
      const int n_tile = t % prm.tiles_n;
      const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
      const uint32_t t_free = buf == 0 ? tempty_leader0 : tempty_leader1;
      if (NSUB == 1 && wu.split && ok && !flags[1]) {
        int img = 0, op = 0, oq = 0;
        const bool in_tile = tile_row_pixel<false>(prm, half, row, img, op, oq);
        const uint32_t t_acc = t_row + static_cast<uint32_t>(buf * C::kTileCols);
        // After the cluster's last unit the operand buffers are idle: they
        // stage the split tile's partial sums.
        const bool final_unit = cursor_done(prm, cur);
        const uint32_t stage_per_warp =
            (static_cast<uint32_t>(SA * prm.a_slot_bytes + SW * prm.w_stage_bytes) / 4u) & ~127u;
        split_piece_epilogue<KT, OUT_COMPLEX>(
            prm, wu, ucid, static_cast<int>(rank), quarter, lane, t_acc, n_tile * KT, in_tile, img,
            op, oq, t_free, final_unit ? data + quarter * stage_per_warp : nullptr, stage_per_warp,
            stage_bar0 + 8u * kStageBufs * static_cast<uint32_t>(quarter));
      } else {
#pragma unroll 1
        for (int sb = 0; sb < NSUB; ++sb) {
          const int row_sb = sb * kBlockM + row;
          const uint32_t t_acc =
              t_row + static_cast<uint32_t>(buf * C::kTileCols + sb * C::kAccCols);
          bool tma_out = false;
          if constexpr (!OUT_COMPLEX) tma_out = prm.out_tma != 0;
          if (tma_out) {
            int c1 = 0, c2 = 0, c3 = 0;
            const bool wv = warp_box_origin<false>(prm, half, sb * kBlockM + quarter * 32, c1, c2,
                                                   c3) &&
                            ok && !flags[1];
            store_accumulator_tma<KT, false>(prm, t_acc, n_tile * KT, wv, c1, c2, c3,
                                             out_stage + quarter * (kOutStageBytes / 4), lane,
                                             stores);
          } else {
            int img = 0, op = 0, oq = 0;
            const bool in_tile = tile_row_pixel<false>(prm, half, row_sb, img, op, oq);
            store_accumulator<KT, OUT_COMPLEX>(
                prm, t_acc, n_tile * KT, in_tile && ok && !flags[1], img, op, oq);
          }
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
    if (warp >= kThreadsH / 32 && !skip) {
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
        prm.lw_ctrs[kLwTmaTicket] = 0u;
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

template <int KT, bool OUT_COMPLEX, int NSUB = 1, bool LW = false>
int launchh_variant(FpropParams& prm, int smem_bytes, void* ws, size_t ws_bytes,
                    cudaStream_t stream) {
  auto kern = ccv_fprop2h_tf32_kernel<KT, OUT_COMPLEX, NSUB, LW>;
  constexpr int threads = halo_threads<LW>();
  static std::once_flag once[64];
  static int max_clusters[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t err = cudaSuccess;
  std::call_once(once[dev & 63], [&]() {
    err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 232448);
    if (err != cudaSuccess) return;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 148, 1, 1);
    cfg.blockDim = dim3(threads, 1, 1);
    cfg.dynamicSmemBytes = 232448;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) {
      max_clusters[dev & 63] = n;
    } else {
      cudaGetLastError();
      max_clusters[dev & 63] = device_sm_count() / 2;
    }
  });
  if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(fprop2h)");
  const int clusters = cluster_cap(max_clusters[dev & 63]);
  const int slots = ((prm.c + kCH - 1) / kCH) * prm.s * prm.passes;
  int rc;
  int launched = 0;
  if (LW) {
    // Layout warps: no stream-K split by default (CCV_STREAMK=1 forces it).
    // Its partial sums and the split tiles' waits for their images cost the
    // layout-warp launches more than the tail they remove: batch 32 of the
    // 56x56 layer 231 us with the split, 215-222 us without, batch 64 equal
    // within noise (B200).  When forced, the stream-K range runs first, so
    // its first image is converted first.
    launched = launch_clusters(prm, clusters, slots, KT, ws, ws_bytes, stream, &rc, 101);
    if (rc != CCV_OK) return rc;
    prm.lw_first_img = 0;
    if (prm.sk_slots > 0) {
      const int half = 2 * (prm.sk_start / prm.tiles_n);
      prm.lw_first_img = std::min(half, prm.total_boxes - 1) / (prm.tiles_bp * prm.tiles_bq);
    }
    lw_plan_prefix(prm, launched, 2LL * kBlockM * NSUB);
  } else {
    launched = launch_clusters(prm, clusters, slots, KT, ws, ws_bytes, stream, &rc);
    if (rc != CCV_OK) return rc;
  }
  cudaError_t e = launch_kernel(kern, dim3(2 * launched), dim3(threads), smem_bytes, stream, 0,
                                prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "fprop2h kernel launch");
  return CCV_OK;
}

}  // namespace

namespace {
// Two A slots plus three weight stages must fit in shared memory.
bool halo_fits(const Tiling& t, int r) {
  const long long slot = 2LL * (t.box_p + r - 1) * t.box_q * kRowH;
  const long long wst = 2LL * t.kt * kRowH;
  return 2 * slot + 3 * wst <= kSmemDataBudget - kOutStageBytes;
}
}  // namespace

bool halo_applicable(const Problem& pb) {
  if (pb.sh != 1 || pb.sw != 1 || pb.r * pb.s <= 1 || pb.r > 64 || pb.s > 64) return false;
  const Tiling t = choose_halo_tiling(pb);
  return t.total_boxes > 0 && halo_fits(t, pb.r);
}

Tiling choose_halo_tiling(const Problem& pb) { return choose_halo_tiling_px(pb, kBlockM); }

Tiling choose_halo_tiling_px(const Problem& pb, int px) {
  Tiling t;
  t.kt = pb.k > 64 ? 128 : (pb.k > 32 ? 64 : 32);
  t.tiles_n = (pb.k + t.kt - 1) / t.kt;
  t.nb = 1;
  t.total_boxes = 0;
  long long best = -1;
  for (int bq = 8; bq <= 128; bq *= 2) {
    const int bp = px / bq;
    if (bp + pb.r - 1 > 256) continue;
    Tiling cand = t;
    cand.box_p = bp;
    cand.box_q = bq;
    if (!halo_fits(cand, pb.r)) continue;
    const long long tbq = (pb.q + bq - 1) / bq;
    const long long tbp = (pb.p + bp - 1) / bp;
    const long long boxes = static_cast<long long>(pb.n) * tbq * tbp;
    // Rows computed, then halo rows loaded per box (fewer is better).
    const long long cost = boxes * px * 1024 + (bp + pb.r - 1) * bq;
    if (best < 0 || cost < best) {
      best = cost;
      t.box_p = bp;
      t.box_q = bq;
      t.tiles_bp = static_cast<int>(tbp);
      t.tiles_bq = static_cast<int>(tbq);
      t.total_boxes = static_cast<int>(boxes);
      t.tiles_m = static_cast<int>(boxes);
    }
  }
  return t;
}

namespace {
// Tensor maps of the TMA prefix of the layout warps: complex64 NCHW input as 8-byte elements (W, C, H, N), boxes
// of 16 pixels x 32 channels x 8 rows (128-byte rows, 128-byte swizzle), and
// the fp32 NHWC planes (C, W, H, N), boxes of 32 channels x 16 pixels x 8 rows.
int encode_conversion_maps(FpropParams& prm, const float* src, const float* xr, const float* xi,
                           const Problem& pb) {
  const uint64_t hw8 = static_cast<uint64_t>(pb.h) * pb.w * 8;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.w), static_cast<uint64_t>(pb.c),
                              static_cast<uint64_t>(pb.h), static_cast<uint64_t>(pb.n)};
    const uint64_t strides[3] = {hw8, static_cast<uint64_t>(pb.w) * 8, hw8 * pb.c};
    const uint32_t box[4] = {kLwBoxPx, kLwBoxCh, kLwBoxRows, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    const int rc = encode_tiled_ex(&prm.tm_cin, src, 4, dims, strides, box, es, kSwizzle128, true);
    if (rc != CCV_OK) return rc;
  }
  const uint64_t cb4 = static_cast<uint64_t>(pb.c) * 4;
  const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.w),
                            static_cast<uint64_t>(pb.h), static_cast<uint64_t>(pb.n)};
  const uint64_t strides[3] = {cb4, cb4 * pb.w, cb4 * pb.w * pb.h};
  const uint32_t box[4] = {kLwBoxCh, kLwBoxPx, kLwBoxRows, 1};
  const uint32_t es[4] = {1, 1, 1, 1};
  int rc = encode_tiled_ex(&prm.tm_pr, xr, 4, dims, strides, box, es, kSwizzleNone, false);
  if (rc != CCV_OK) return rc;
  return encode_tiled_ex(&prm.tm_pi, xi, 4, dims, strides, box, es, kSwizzleNone, false);
}
}  // namespace

int launch_fprop_pair_halo(const float* xr, const float* xi, const float* xr_lo,
                           const float* xi_lo, bool split, const float* w_packed, float* y0,
                           float* y1, const Problem& pb, const Tiling& t_in, OutLayout out_layout,
                           const Epilogue& ep, void* ws, size_t ws_bytes, cudaStream_t stream,
                           const float* lw_src, const float* lw_pr, const float* lw_pi) {
  // KT <= 64: two 128-pixel sub-boxes per CTA tile when the taller halo slot
  // fits (CCV_SUBBOX=0 turns it off; testing knob).  No stream-K split then.
  Tiling t = t_in;
  int nsub = 1;
  if (knobs().subbox != 0 && t.kt <= 64) {
    const Tiling t2 = choose_halo_tiling_px(pb, 2 * kBlockM);
    if (t2.total_boxes > 0 && halo_fits(t2, pb.r)) {
      t = t2;
      nsub = 2;
      ws = nullptr;
      ws_bytes = 0;
    }
  }
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
  prm.nb = 1;
  prm.tiles_bp = t.tiles_bp; prm.tiles_bq = t.tiles_bq; prm.total_boxes = t.total_boxes;
  prm.tiles_m = t.tiles_m; prm.tiles_n = t.tiles_n;
  prm.ksteps = ((pb.c + kCH - 1) / kCH) * pb.r * pb.s;
  prm.m_total = static_cast<long long>(pb.n) * pb.p * pb.q;
  prm.num_tiles = pair_tiles(t);
  prm.passes = split ? 3 : 1;
  if (!split) {
    xr_lo = xr;
    xi_lo = xi;
  }
  int rc0;
  prm.halo_rows = (t.box_p + pb.r - 1) * t.box_q;
  prm.a_slot_bytes = 2 * prm.halo_rows * kRowH;
  prm.w_stage_bytes = 2 * t.kt * kRowH;
  const bool cplx = out_layout == OUT_COMPLEX_NCHW;
  if (!cplx && (rc0 = encode_planar_out_maps(prm, y0, y1, false)) != CCV_OK) return rc0;
  const bool lw = lw_src != nullptr || lw_pr != nullptr;
  if (lw) {
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
  }
  // Ring depths: at least 2 A slots and 3 weight stages; prefer 4+ weight
  // stages, then a third A slot.
  const int budget = kSmemDataBudget - (prm.out_tma ? kOutStageBytes : 0);
  int sa = 2;
  int sw = (budget - sa * prm.a_slot_bytes) / prm.w_stage_bytes;
  if (sw > 4 && budget - 3 * prm.a_slot_bytes >= 4 * prm.w_stage_bytes) {
    sa = 3;
    sw = (budget - sa * prm.a_slot_bytes) / prm.w_stage_bytes;
  }
  sw = std::min(sw, kMaxWStages);
  if (sw < 3) return set_error(CCV_ERR_UNSUPPORTED, "halo tile does not fit in shared memory");
  prm.a_slots = sa;
  prm.w_stages = sw;
  const int smem_bytes = 1024 + kBarBytes + sa * prm.a_slot_bytes + sw * prm.w_stage_bytes +
                         (prm.out_tma ? kOutStageBytes : 0);
  if (lw && lw_src != nullptr && lw_pr == nullptr && !split && (pb.w & 1) == 0 &&
      (reinterpret_cast<uintptr_t>(lw_src) & 15) == 0 &&
      sa * prm.a_slot_bytes + sw * prm.w_stage_bytes >= static_cast<int>(kLwBoxSmemBytes)) {
    // TMA prefix possible (sized at launch): TF32, even W (8-byte elements,
    // 16-byte row strides), the operand rings can hold its boxes.
    const int rc1 = encode_conversion_maps(prm, lw_src, xr, xi, pb);
    if (rc1 != CCV_OK) return rc1;
    prm.lw_tma_images = -1;
  }

  int rc;
  const uint64_t cb = static_cast<uint64_t>(pb.c) * 4;
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.w),
                              static_cast<uint64_t>(pb.h), static_cast<uint64_t>(pb.n)};
    const uint64_t strides[3] = {cb, cb * pb.w, cb * pb.w * pb.h};
    const uint32_t box[4] = {kCH, static_cast<uint32_t>(t.box_q),
                             static_cast<uint32_t>(t.box_p + pb.r - 1), 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled(&prm.tm_xr, xr, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi, xi, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xr_lo, xr_lo, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
    if ((rc = encode_tiled(&prm.tm_xi_lo, xi_lo, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
  }
  {
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.k), 3,
                              static_cast<uint64_t>(pb.r) * pb.s * (split ? 2 : 1)};
    const uint64_t strides[3] = {cb, cb * pb.k, cb * pb.k * 3};
    const uint32_t box[4] = {kCH, static_cast<uint32_t>(t.kt), 1, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled(&prm.tm_w, w_packed, 4, dims, strides, box, es, 128)) != CCV_OK) return rc;
  }
#define CCV_HALO_LAUNCH(KT_, CPLX_, NSUB_, LW_) \
  launchh_variant<KT_, CPLX_, NSUB_, LW_>(prm, smem_bytes, ws, ws_bytes, stream)
#define CCV_HALO_BY_KT(CPLX_, LW_)                                                   \
  do {                                                                               \
    if (nsub == 2) {                                                                 \
      return t.kt == 64 ? CCV_HALO_LAUNCH(64, CPLX_, 2, LW_)                         \
                        : CCV_HALO_LAUNCH(32, CPLX_, 2, LW_);                        \
    }                                                                                \
    switch (t.kt) {                                                                  \
      case 128: return CCV_HALO_LAUNCH(128, CPLX_, 1, LW_);                          \
      case 64: return CCV_HALO_LAUNCH(64, CPLX_, 1, LW_);                            \
      default: return CCV_HALO_LAUNCH(32, CPLX_, 1, LW_);                            \
    }                                                                                \
  } while (0)
  // Layout warps with planar output: the 3xTF32 split of forward_planar()'s
  // input planes.
  if (lw && cplx) CCV_HALO_BY_KT(true, true);
  if (lw) CCV_HALO_BY_KT(false, true);
  if (cplx) CCV_HALO_BY_KT(true, false);
  CCV_HALO_BY_KT(false, false);
#undef CCV_HALO_BY_KT
#undef CCV_HALO_LAUNCH
}

}  // namespace ccv
