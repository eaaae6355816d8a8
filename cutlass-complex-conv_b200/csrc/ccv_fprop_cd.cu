// Complex Conv2d forward() kernel that reads complex64 NCHW activations
// straight from global memory with TMA ("complex-direct"): no converter
// warps, no layout pass.
//
// Trick: in NCHW complex64, for one channel and one image row, the floats
// along W are re0, im0, re1, im1, ...  Take those floats as the M dimension
// of the GEMM (m' = 2 * pixel + part) and the channels as K: the A tile is
// then an MN-major operand that TMA copies as-is (128-byte rows of 16 pixels
// x (re, im), one row per channel, 32-byte swizzle atoms - the one MN-major
// layout tcgen05 accepts for 32-bit operands).  With B = [W_re ; W_im]
// (N = 2*KT) one MMA gives, per pixel p and output channel k,
//     D[2p  ][k] = xr.Wr   D[2p  ][KT+k] = xr.Wi
//     D[2p+1][k] = xi.Wr   D[2p+1][KT+k] = xi.Wi
// and the epilogue forms y = (xr.Wr - xi.Wi) + i (xr.Wi + xi.Wr) from the
// two TMEM lanes of a pixel (a lane-pair shuffle).  Per pixel this is the
// same MMA work as the planar kernels (64 pixels per 128-row MMA, one MMA
// instead of two per K step).
//
// Geometry: stride-1 problems with an odd filter width S.  A CTA tile is a
// box of 4 output rows x 16 output columns (64 pixels = 128 MMA rows); a
// pair of CTAs (cta_group::2, M = 256) shares each B tile.  Halo reuse as in
// ccv_fprop2h.cu: for channel block cb (32 channels) and filter column s one
// "slot" holds input rows oy0-ph .. oy0-ph+3+R-1 of columns x_s .. x_s+15
// (x_s = ox0 - pw + s), and filter row r reads it from row r on.
//
// TMA can only start a load on a 16-byte (two-pixel) boundary.  Box origins
// are placed so that x_s is even for every even s (ox0 = 16*bq - (pw & 1));
// the slots of odd s are assembled in shared memory by two "shifter" warps:
// slot(s) pixel j = slot(s-1) pixel j+1 (j < 15), pixel 15 = slot(s+1)
// pixel 14.  S odd guarantees s+1 < S for every odd s.
//
// Warp roles (256 threads): warp 0 TMA producer, warp 1 TMEM allocation and
// MMA issue (even CTA), warps 2-5 epilogue, warps 6-7 shifters.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>

#include "ccv_fprop_common.cuh"
#include "ccv_internal.h"
#include "ccv_ptx.cuh"

namespace ccv {

namespace {

constexpr int kThreadsCD = 256;
constexpr int kShiftWarps = 2;
constexpr int kCHc = 32;                       // input channels per K block
constexpr int kBoxRows = 4;                    // output rows per CTA box
constexpr int kBoxCols = 16;                   // output columns per CTA box
constexpr uint32_t kRowBlock = kCHc * 128u;    // one box row of one slot: 32 ch x 128 B
constexpr int kMaxGroups = 8;
constexpr int kMaxWStagesCD = 12;
constexpr int kBarBytesCD = 1024;
constexpr int kBudgetCD = 232448 - kBarBytesCD - 1024;
constexpr int kTimeoutCD = CCV_ERR_DEVICE_TIMEOUT;

template <int KT>
struct CfgCD {
  static constexpr int kAccCols = 2 * KT;
  static constexpr int kTmemCols = 2 * kAccCols < 32 ? 32 : 2 * kAccCols;
  static constexpr uint32_t kWStageBytes = KT * 128u;  // this CTA's half of B: KT rows x 32 ch
};

// MN-major operand descriptor, 128-byte rows with 32-byte swizzle atoms
// (layout type 1): MN blocks of 16 pixels `lbo` bytes apart, 4-row K atoms
// 512 bytes apart.
__device__ __forceinline__ uint64_t desc_mn_atom32(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((512u >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1u) << 46;
  d |= static_cast<uint64_t>(1u) << 61;
  return d;
}

// Filter column of the i-th slot in MMA order: even columns (loaded by TMA)
// first, then odd ones (assembled by the shifters), so the tensor cores start
// on a channel block before its shifted slots are ready.
__device__ __forceinline__ int slot_column(int i, int S) {
  const int neven = (S + 1) / 2;
  return i < neven ? 2 * i : 2 * (i - neven) + 1;
}

// Byte offset of pixel q (0..15) in line `line` (128 bytes) of a slot in the
// 32-byte-atom swizzle: 32-byte chunk index XOR (line mod 4).
__device__ __forceinline__ uint32_t atom32_offset(uint32_t line, uint32_t q) {
  return line * 128u + ((((q >> 2) ^ line) & 3u) << 5) + ((q & 3u) << 3);
}

template <int KT>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreadsCD, 1)
    ccv_fprop_cd_kernel(const __grid_constant__ FpropParams prm) {
  using Cfg = CfgCD<KT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base);
  // a_dfull[8] (TMA bytes, local), a_full_d[8] / a_full_s[8] (direct /
  // shifted slots ready: shifter-warp arrivals, even CTA), a_empty[8],
  // wfull[12] (even CTA), wempty[12], tfull[2], tempty[2] (even CTA), done;
  // then the TMEM address and flags.
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 62);
  volatile int* flags = reinterpret_cast<volatile int*>(tmem_holder + 1);  // [0] skip, [1] abort
  uint8_t* data = base + kBarBytesCD;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = ptx::cluster_ctarank();
  const bool leader = rank == 0;
  const int cid = static_cast<int>(ptx::cluster_id_x());
  const int ncl = static_cast<int>(ptx::nclusters_x());
  const uint32_t bar_base = ptx::smem_u32(bars);
  auto a_dfull = [&](int g) { return bar_base + 8u * g; };
  auto a_full_d = [&](int g) { return bar_base + 8u * (8 + g); };
  auto a_full_s = [&](int g) { return bar_base + 8u * (16 + g); };
  auto a_empty = [&](int g) { return bar_base + 8u * (24 + g); };
  auto wfull = [&](int i) { return bar_base + 8u * (32 + i); };
  auto wempty = [&](int i) { return bar_base + 8u * (44 + i); };
  auto tfull = [&](int b) { return bar_base + 8u * (56 + b); };
  auto tempty = [&](int b) { return bar_base + 8u * (58 + b); };
  const uint32_t done_bar = bar_base + 8u * 60;

  const int G = prm.a_slots;   // slot groups in the ring (one group per channel block)
  const int SW = prm.w_stages;
  const int S = prm.s;
  const int R = prm.r;
  const uint32_t slot_bytes = static_cast<uint32_t>(prm.a_slot_bytes);
  const uint32_t group_bytes = slot_bytes * static_cast<uint32_t>(S);
  const uint32_t a_base = ptx::smem_u32(data);
  const uint32_t w_base = a_base + static_cast<uint32_t>(G) * group_bytes;
  const int ndirect = (S + 1) / 2;   // even s

  if (threadIdx.x == 0) {
    flags[1] = 0;
    for (int g = 0; g < G; ++g) {
      ptx::mbar_init(a_dfull(g), 1);
      ptx::mbar_init(a_full_d(g), 2 * kShiftWarps);  // shifter warps of both CTAs
      ptx::mbar_init(a_full_s(g), 2 * kShiftWarps);
      ptx::mbar_init(a_empty(g), 1);
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
    ptx::fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    ptx::prefetch_tmap(&prm.tm_xr);
    ptx::prefetch_tmap(&prm.tm_w);
  }
  if (warp == 1) {
    ptx::tmem_alloc_pair(ptx::smem_u32(tmem_holder), Cfg::kTmemCols);
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
  __syncthreads();
  const uint32_t tmem_base = *tmem_holder;
  const bool skip = flags[0] != 0;
  const int per_img = prm.tiles_bp * prm.tiles_bq;
  const int col_off = prm.pw & 1;  // box origins: ox0 = 16 * bq - col_off

  // Box of this CTA for pair tile t: (image, first output row, first column).
  auto box_of = [&](int t, int& img, int& oy0, int& ox0) {
    const int half = 2 * (t / prm.tiles_n) + static_cast<int>(rank);
    const int gb = min(half, prm.total_boxes - 1);
    img = gb / per_img;
    const int rem = gb - img * per_img;
    const int bp = rem / prm.tiles_bq;
    const int bq = rem - bp * prm.tiles_bq;
    oy0 = bp * kBoxRows;
    ox0 = bq * kBoxCols - col_off;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && !skip) {
      uint32_t ga = 0, gw = 0;
      bool abort = false;
      UnitCursor cur = unit_cursor(prm, cid);
      WorkUnit wu;
      while (!abort && next_unit(prm, ncl, cur, wu)) {
        int img, oy0, ox0;
        box_of(wu.tile, img, oy0, ox0);
        const int k0 = (wu.tile % prm.tiles_n) * KT;
        for (int cb = wu.jbeg; cb < wu.jend && !abort; ++cb, ++ga) {
          const int c0 = cb * kCHc;
          const int g = static_cast<int>(ga % G);
          if (!ptx::mbar_wait_bounded(a_empty(g), ((ga / G) & 1u) ^ 1u, prm.status, kTimeoutCD) ||
              flags[1]) {
            flags[1] = 1;
            abort = true;
            break;
          }
          ptx::mbar_arrive_expect_tx(a_dfull(g), static_cast<uint32_t>(ndirect) * slot_bytes);
          const uint32_t grp = a_base + static_cast<uint32_t>(g) * group_bytes;
          for (int s = 0; s < S; s += 2) {
            ptx::tma_load_4d(grp + static_cast<uint32_t>(s) * slot_bytes, &prm.tm_xr, a_dfull(g),
                             ox0 - prm.pw + s, c0, oy0 - prm.ph, img);
          }
          for (int si = 0; si < S && !abort; ++si) {
            const int s = slot_column(si, S);
            for (int r = 0; r < R; ++r, ++gw) {
              const int st = static_cast<int>(gw % SW);
              if (!ptx::mbar_wait_bounded(wempty(st), ((gw / SW) & 1u) ^ 1u, prm.status,
                                          kTimeoutCD) ||
                  flags[1]) {
                flags[1] = 1;
                abort = true;
                break;
              }
              if (leader) ptx::mbar_arrive_expect_tx(wfull(st), 2u * Cfg::kWStageBytes);
              // Packed planes per tap: 1 = W_re (even CTA), 2 = W_im (odd CTA).
              ptx::tma_load_4d_pair(w_base + static_cast<uint32_t>(st) * Cfg::kWStageBytes,
                                    &prm.tm_w, ptx::mapa_shared(wfull(st), 0), c0, k0,
                                    leader ? 1 : 2, r * S + s);
            }
          }
        }
      }
      // Drain: this CTA's activation loads and (even CTA) every weight stage.
      for (uint32_t j = 0; j < static_cast<uint32_t>(G) && j < ga; ++j) {
        const uint32_t q = ga - 1 - j;
        ptx::mbar_wait_bounded(a_dfull(static_cast<int>(q % G)), (q / G) & 1u, prm.status,
                               kTimeoutCD);
      }
      if (leader) {
        for (uint32_t j = 0; j < static_cast<uint32_t>(SW) && j < gw; ++j) {
          const uint32_t q = gw - 1 - j;
          ptx::mbar_wait_bounded(wfull(static_cast<int>(q % SW)), (q / SW) & 1u, prm.status,
                                 kTimeoutCD);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (even CTA)
    if (leader && lane == 0 && !skip) {
      // M = 256 (two CTAs x 128 rows), N = 2*KT, A MN-major (bit 15).
      constexpr uint32_t idesc = ptx::idesc_tf32(2 * kBlockM, 2 * KT, false) | (1u << 15);
      uint32_t ga = 0, gw = 0;
      int i = 0;
      bool abort = false;
      UnitCursor cur = unit_cursor(prm, cid);
      WorkUnit wu;
      while (!abort && next_unit(prm, ncl, cur, wu)) {
        const int buf = i & 1;
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        ++i;
        if (!ptx::mbar_wait_bounded(tempty(buf), (use & 1u) ^ 1u, prm.status, kTimeoutCD)) {
          flags[1] = 1;
          break;
        }
        ptx::tc_fence_after();
        const uint32_t d = tmem_base + static_cast<uint32_t>(buf * Cfg::kAccCols);
        bool first = true;
        for (int cb = wu.jbeg; cb < wu.jend && !abort; ++cb, ++ga) {
          const int g = static_cast<int>(ga % G);
          const uint32_t par = (ga / G) & 1u;
          if (!ptx::mbar_wait_bounded<true>(a_full_d(g), par, prm.status, kTimeoutCD)) {
            flags[1] = 1;
            abort = true;
            break;
          }
          const uint32_t grp = a_base + static_cast<uint32_t>(g) * group_bytes;
          for (int si = 0; si < S && !abort; ++si) {
            const int s = slot_column(si, S);
            if (si == ndirect &&
                !ptx::mbar_wait_bounded<true>(a_full_s(g), par, prm.status, kTimeoutCD)) {
              flags[1] = 1;
              abort = true;
              break;
            }
            for (int r = 0; r < R; ++r, ++gw) {
              const int st = static_cast<int>(gw % SW);
              if (!ptx::mbar_wait_bounded(wfull(st), (gw / SW) & 1u, prm.status, kTimeoutCD)) {
                flags[1] = 1;
                abort = true;
                break;
              }
              ptx::tc_fence_after();
              const uint32_t a = grp + static_cast<uint32_t>(s) * slot_bytes +
                                 static_cast<uint32_t>(r) * kRowBlock;
              const uint32_t w = w_base + static_cast<uint32_t>(st) * Cfg::kWStageBytes;
#pragma unroll
              for (int kk = 0; kk < kCHc / 8; ++kk) {
                ptx::mma_tf32_pair(d, desc_mn_atom32(a + kk * 1024u, kRowBlock),
                                   ptx::desc_kmajor_sw128(w + kk * 32u), idesc, first ? 0u : 1u);
                first = false;
              }
              ptx::mma_commit_pair(wempty(st));
            }
          }
          ptx::mma_commit_pair(a_empty(g));
        }
        ptx::mma_commit_pair(tfull(buf));
      }
      ptx::mma_commit_pair(done_bar);
      ptx::mbar_wait_bounded(done_bar, 0, prm.status, kTimeoutCD);
    }
    __syncwarp();
  } else if (warp <= 5) {
    // ------------------------------------------------------------ epilogue
    // Warp q reads TMEM lanes 32q..32q+31 = box row q: lane l holds pixel
    // l/2, part l%2 (0: x_re products, 1: x_im products).
    const int quarter = warp & 3;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16);
    const uint32_t tempty_leader0 = ptx::mapa_shared(tempty(0), 0);
    const uint32_t tempty_leader1 = ptx::mapa_shared(tempty(1), 0);
    const bool odd = (lane & 1) != 0;
    const long long pq = static_cast<long long>(prm.p) * prm.q;
    float2* y = reinterpret_cast<float2*>(prm.y0);
    int i = 0;
    UnitCursor cur = unit_cursor(prm, cid);
    WorkUnit wu;
    while (!skip && next_unit(prm, ncl, cur, wu)) {
      const int buf = i & 1;
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      ++i;
      const bool ok = ptx::mbar_wait_bounded_backoff(tfull(buf), use & 1u, prm.status, kTimeoutCD);
      ptx::tc_fence_after();
      if (!ok) flags[1] = 1;
      int img, oy0, ox0;
      box_of(wu.tile, img, oy0, ox0);
      const int half = 2 * (wu.tile / prm.tiles_n) + static_cast<int>(rank);
      const int oy = oy0 + quarter;
      const int ox = ox0 + (lane >> 1);
      const bool valid = ok && !flags[1] && half < prm.total_boxes && oy < prm.p && ox >= 0 &&
                         ox < prm.q;
      const int k0 = (wu.tile % prm.tiles_n) * KT;
      const uint32_t t_acc = t_row + static_cast<uint32_t>(buf * Cfg::kAccCols);
      const long long pix = static_cast<long long>(img) * prm.k * pq +
                            static_cast<long long>(oy) * prm.q + ox;
#pragma unroll 1
      for (int ch = 0; ch < KT; ch += 32) {
        uint32_t lo[32], hi[32];
        ptx::tmem_ld_32x32b_x32(t_acc + ch, lo);       // . W_re
        ptx::tmem_ld_32x32b_x32(t_acc + KT + ch, hi);  // . W_im
        ptx::tmem_wait_ld();
        // Even lane: channels ch..ch+15; odd lane: ch+16..ch+31.
        const int kb = k0 + ch + (odd ? 16 : 0);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float s_lo = __uint_as_float(odd ? lo[j] : lo[16 + j]);
          const float s_hi = __uint_as_float(odd ? hi[j] : hi[16 + j]);
          const float r_lo = __shfl_xor_sync(0xffffffffu, s_lo, 1);
          const float r_hi = __shfl_xor_sync(0xffffffffu, s_hi, 1);
          float re, im;
          if (!odd) {  // own: xr.Wr, xr.Wi; partner: xi.Wr, xi.Wi
            re = __uint_as_float(lo[j]) - r_hi;
            im = __uint_as_float(hi[j]) + r_lo;
          } else {     // own: xi.Wr, xi.Wi; partner: xr.Wr, xr.Wi
            re = r_lo - __uint_as_float(hi[16 + j]);
            im = r_hi + __uint_as_float(lo[16 + j]);
          }
          if (valid && kb + j < prm.k) {
            y[pix + static_cast<long long>(kb + j) * pq] = make_float2(re, im);
          }
        }
      }
      ptx::tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive_cluster(buf == 0 ? tempty_leader0 : tempty_leader1);
      if (!ok) break;
    }
  } else if (!skip) {
    // ------------------------------------------------------------ shifters
    // Build the slots of odd filter columns from their even neighbours.
    const int sw_id = warp - 6;
    const uint32_t lines = slot_bytes / 128u;  // (4 + R - 1) rows x 32 channels
    uint32_t ga = 0;
    UnitCursor cur = unit_cursor(prm, cid);
    WorkUnit wu;
    bool stop = false;
    while (!stop && next_unit(prm, ncl, cur, wu)) {
      for (int cb = wu.jbeg; cb < wu.jend; ++cb, ++ga) {
        const int g = static_cast<int>(ga % G);
        if (!ptx::mbar_wait_bounded_backoff(a_dfull(g), (ga / G) & 1u, prm.status, kTimeoutCD) ||
            flags[1]) {
          flags[1] = 1;
          stop = true;
          break;
        }
        // The TMA-loaded slots of this CTA are in: tell the MMA issuer.
        ptx::fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(a_full_d(g), 0));
        uint8_t* grp = data + static_cast<uint32_t>(g) * group_bytes;
        for (int s = 1; s < S; s += 2) {
          const uint8_t* src0 = grp + static_cast<uint32_t>(s - 1) * slot_bytes;
          const uint8_t* src1 = grp + static_cast<uint32_t>(s + 1) * slot_bytes;
          uint8_t* dst = grp + static_cast<uint32_t>(s) * slot_bytes;
          // Two lines per warp step: lanes 0-15 line 2i, lanes 16-31 line 2i+1.
          const uint32_t q = static_cast<uint32_t>(lane & 15);
          for (uint32_t l2 = static_cast<uint32_t>(sw_id) * 2u + (lane >> 4); l2 < lines;
               l2 += 2u * kShiftWarps) {
            const float2 v = q < 15u ? *reinterpret_cast<const float2*>(src0 + atom32_offset(l2, q + 1u))
                                     : *reinterpret_cast<const float2*>(src1 + atom32_offset(l2, 14u));
            *reinterpret_cast<float2*>(dst + atom32_offset(l2, q)) = v;
          }
        }
        ptx::fence_proxy_async_shared();
        __syncwarp();
        if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(a_full_s(g), 0));
      }
    }
  }

  __syncthreads();
  if (flags[1]) ptx::nanosleep(100000);  // let stray copies of an aborted tile land
  ptx::tc_fence_before();
  ptx::cluster_sync();
  if (warp == 1) {
    ptx::tc_fence_after();
    ptx::tmem_dealloc_pair(tmem_base, Cfg::kTmemCols);
  }
}

struct CdLayout {
  int groups, w_stages, smem_bytes;
  uint32_t slot_bytes;
};

bool cd_layout(const Problem& pb, int kt, CdLayout* out) {
  const uint32_t slot = static_cast<uint32_t>(kBoxRows + pb.r - 1) * kRowBlock;
  const long long group = static_cast<long long>(slot) * pb.s;
  const long long wst = static_cast<long long>(kt) * 128;
  // Prefer a weight ring of 8 stages (about 2 us of MMAs at N = 256), then as
  // many slot groups as fit (up to 8); at least 2 groups and 3 stages, or one
  // group for wide filters.
  int g = 0, sw = 0;
  for (int cand = kMaxGroups; cand >= 2; --cand) {
    const long long rest = kBudgetCD - cand * group;
    if (rest >= 8 * wst) {
      g = cand;
      sw = static_cast<int>(std::min<long long>(rest / wst, kMaxWStagesCD));
      break;
    }
  }
  if (g == 0) {
    for (int cand = 2; cand >= 1 && g == 0; --cand) {
      const long long rest = kBudgetCD - cand * group;
      if (rest >= 3 * wst) {
        g = cand;
        sw = static_cast<int>(std::min<long long>(rest / wst, kMaxWStagesCD));
      }
    }
  }
  if (g == 0) return false;
  out->groups = g;
  out->w_stages = sw;
  out->slot_bytes = slot;
  out->smem_bytes = 1024 + kBarBytesCD + static_cast<int>(g * group + sw * wst);
  return true;
}

template <int KT>
int launch_cd_variant(FpropParams& prm, int smem_bytes, void* ws, size_t ws_bytes,
                      cudaStream_t stream) {
  auto kern = ccv_fprop_cd_kernel<KT>;
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
    cfg.blockDim = dim3(kThreadsCD, 1, 1);
    cfg.dynamicSmemBytes = 232448;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) {
      max_clusters[dev & 63] = n;
    } else {
      cudaGetLastError();
      max_clusters[dev & 63] = device_sm_count() / 2;
    }
  });
  if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(fprop_cd)");
  (void)ws;
  (void)ws_bytes;
  // Whole tiles only (no stream-K split in this kernel).
  int rc = CCV_OK;
  const int launched =
      launch_clusters(prm, cluster_cap(max_clusters[dev & 63]), prm.slots_per_tile, KT, nullptr,
                      0, stream, &rc);
  if (rc != CCV_OK) return rc;
  cudaError_t e = launch_kernel(kern, dim3(2 * launched), dim3(kThreadsCD), smem_bytes, stream, 0,
                                prm);
  if (e == cudaSuccess) e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_error(e, "fprop_cd kernel launch");
  return CCV_OK;
}

}  // namespace

bool cd_applicable(const Problem& pb) {
  if (pb.sh != 1 || pb.sw != 1 || (pb.s & 1) == 0 || pb.r > 64 || pb.s > 64) return false;
  // TMA strides are multiples of 16 bytes: an even image width.
  if ((pb.w & 1) != 0) return false;
  if (kBoxRows + pb.r - 1 > 256) return false;
  const int kt = pb.k > 64 ? 128 : (pb.k > 32 ? 64 : 32);
  CdLayout lay;
  return cd_layout(pb, kt, &lay);
}

int launch_fprop_cd(const float* xc, const float* w_packed, float* y, const Problem& pb,
                    void* ws, size_t ws_bytes, cudaStream_t stream) {
  if (!cd_applicable(pb)) {
    return set_error(CCV_ERR_UNSUPPORTED, "no complex-direct kernel for this problem");
  }
  FpropParams prm;
  memset(&prm, 0, sizeof(prm));
  prm.xc = xc;
  prm.y0 = y;
  prm.status = device_status_ptr();
  if (prm.status == nullptr) return CCV_ERR_CUDA;
  prm.n = pb.n; prm.h = pb.h; prm.w = pb.w; prm.c = pb.c; prm.k = pb.k;
  prm.r = pb.r; prm.s = pb.s; prm.p = pb.p; prm.q = pb.q;
  prm.sh = pb.sh; prm.sw = pb.sw; prm.ph = pb.ph; prm.pw = pb.pw;
  const int kt = pb.k > 64 ? 128 : (pb.k > 32 ? 64 : 32);
  prm.box_p = kBoxRows;
  prm.box_q = kBoxCols;
  prm.tiles_n = (pb.k + kt - 1) / kt;
  prm.tiles_bp = (pb.p + kBoxRows - 1) / kBoxRows;
  prm.tiles_bq = (pb.q + (pb.pw & 1) + kBoxCols - 1) / kBoxCols;
  const long long boxes = static_cast<long long>(pb.n) * prm.tiles_bp * prm.tiles_bq;
  if (boxes > 0x3fffffffLL) return set_error(CCV_ERR_UNSUPPORTED, "problem too large");
  prm.total_boxes = static_cast<int>(boxes);
  prm.tiles_m = prm.total_boxes;
  prm.num_tiles = ((prm.total_boxes + 1) / 2) * prm.tiles_n;
  prm.passes = 1;
  const int ncb = (pb.c + kCHc - 1) / kCHc;
  prm.ksteps = ncb * pb.r * pb.s;
  prm.m_total = static_cast<long long>(pb.n) * pb.p * pb.q;
  CdLayout lay;
  if (!cd_layout(pb, kt, &lay)) return set_error(CCV_ERR_UNSUPPORTED, "complex-direct tile too large");
  prm.a_slots = lay.groups;
  prm.w_stages = lay.w_stages;
  prm.a_slot_bytes = static_cast<int>(lay.slot_bytes);
  prm.halo_rows = kBoxRows + pb.r - 1;
  prm.slots_per_tile = ncb;  // one unit of K work = one channel block
  int rc;
  {
    // complex64 NCHW as 8-byte elements, dims (W, C, H, N): a box row is 16
    // pixels of one channel, the box holds 32 channels x (4 + R - 1) rows.
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.w), static_cast<uint64_t>(pb.c),
                              static_cast<uint64_t>(pb.h), static_cast<uint64_t>(pb.n)};
    const uint64_t hw8 = static_cast<uint64_t>(pb.h) * pb.w * 8;
    const uint64_t strides[3] = {hw8, static_cast<uint64_t>(pb.w) * 8, hw8 * pb.c};
    const uint32_t box[4] = {kBoxCols, kCHc, static_cast<uint32_t>(kBoxRows + pb.r - 1), 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled_ex(&prm.tm_xr, xc, 4, dims, strides, box, es, kSwizzle128Atom32,
                              true)) != CCV_OK) {
      return rc;
    }
  }
  {
    const uint64_t cb = static_cast<uint64_t>(pb.c) * 4;
    const uint64_t dims[4] = {static_cast<uint64_t>(pb.c), static_cast<uint64_t>(pb.k), 3,
                              static_cast<uint64_t>(pb.r) * pb.s};
    const uint64_t strides[3] = {cb, cb * pb.k, cb * pb.k * 3};
    const uint32_t box[4] = {kCHc, static_cast<uint32_t>(kt), 1, 1};
    const uint32_t es[4] = {1, 1, 1, 1};
    if ((rc = encode_tiled(&prm.tm_w, w_packed, 4, dims, strides, box, es, 128)) != CCV_OK) {
      return rc;
    }
  }
  switch (kt) {
    case 128: return launch_cd_variant<128>(prm, lay.smem_bytes, ws, ws_bytes, stream);
    case 64: return launch_cd_variant<64>(prm, lay.smem_bytes, ws, ws_bytes, stream);
    default: return launch_cd_variant<32>(prm, lay.smem_bytes, ws, ws_bytes, stream);
  }
}

}  // namespace ccv
