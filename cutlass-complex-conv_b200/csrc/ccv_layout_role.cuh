// Layout warps: forward()'s complex64 NCHW -> fp32 NHWC conversion done by
// two extra warps in every CTA of a persistent pair kernel, ahead of (and
// overlapping) the convolution, in the same launch.
//
// Work is handed out by a global counter in chunks of kLwChunk tickets (one
// atomic per chunk, the next chunk's number fetched while the current one
// is converted): one ticket = 32 channels x 32 consecutive pixels of one image (a pixel is h * W + w: both layouts keep an
// image's H x W plane contiguous).  Tickets run image by image, starting at
// image lw_first_img (the first image of a stream-K range, which the kernel
// runs first) and wrapping around; warps count completed tickets per image
// (release), and a producer may load an image's planes once the count
// reaches the image's ticket count (acquire + async-proxy fence).
// A ticket is taken only by a running warp and completed without waiting on
// anything, so a producer waits only for work that is in progress or that any
// running CTA - its own included - will take next: no CTA depends on another
// CTA being resident.
//
// 3xTF32: the warps write tf32(x) into the hi planes and x - tf32(x) into the
// lo planes (the activation split of three-pass TF32).  The same warps also
// take fp32 NHWC planes as the source (lw_pr/lw_pi: forward_planar() at
// 3xTF32, where only the split is needed).
#pragma once

#include <cstdint>

#include "ccv_fprop_common.cuh"
#include "ccv_ptx.cuh"

namespace ccv {

constexpr int kLwWarps = 2;                 // layout warps per CTA
constexpr int kLwPx = 32;                   // pixels per ticket
constexpr int kLwCh = 32;                   // channels per ticket (lane = channel)
constexpr int kLwChunk = 4;                 // tickets per counter increment
// Counter set layout (a zeroed library-owned set; the last CTA resets it).
constexpr int kLwTicket = 0;               // chunks taken past the prefix
constexpr int kLwDone = 1;
constexpr int kLwPrefixTicket = 2;         // chunks taken of the prefix
constexpr int kLwTmaTicket = 3;            // TMA prefix: tiles taken
constexpr int kLwTmaMaxImages = 16;        // TMA prefix: images at most
constexpr int kLwFlag0 = 8;                 // image i: tickets completed
// TMA prefix box: 8 rows x 16 pixels x 32 channels (32 KB of complex64 in,
// two 16 KB fp32 planes out), kLwBoxBufs boxes in flight.
constexpr int kLwBoxRows = 8;
constexpr int kLwBoxPx = 16;
constexpr int kLwBoxCh = 32;
constexpr uint32_t kLwBoxInBytes = kLwBoxRows * kLwBoxCh * kLwBoxPx * 8u;
constexpr uint32_t kLwBoxOutPlane = kLwBoxRows * kLwBoxPx * kLwBoxCh * 4u;
constexpr int kLwBoxBufs = 4;
// Shared memory the TMA prefix needs (input ring + two output buffers).
constexpr uint32_t kLwBoxSmemBytes = kLwBoxBufs * kLwBoxInBytes + 2u * 2u * kLwBoxOutPlane;

__device__ __forceinline__ int lw_tickets_per_image(const FpropParams& prm) {
  return ((prm.h * prm.w + kLwPx - 1) / kLwPx) * ((prm.c + kLwCh - 1) / kLwCh);
}

__device__ __forceinline__ float lw_tf32(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

struct LwTicket {
  long long tk;  // ticket index (>= total: none)
  int img, px0, c0;
};

__device__ __forceinline__ LwTicket lw_decode(const FpropParams& prm, long long tk, int tpx,
                                              int per_img) {
  LwTicket t;
  t.tk = tk;
  const int order = static_cast<int>(tk / per_img);
  const int rem = static_cast<int>(tk - static_cast<long long>(order) * per_img);
  t.img = (order + prm.lw_first_img) % prm.n;
  const int cb = rem / tpx;
  t.px0 = (rem - cb * tpx) * kLwPx;
  t.c0 = cb * kLwCh;
  return t;
}

// Loads of one ticket.  Lane = channel: the lane reads its channel's 32
// pixels (256 contiguous bytes) as 16-byte pieces, so one warp instruction
// touches one 32-byte sector per channel and the next one finds the sector's
// other half in L1.  v[j] = pixels 2j and 2j+1 (re, im, re, im).  `vec`:
// 16-byte loads are aligned (H*W even and a 16-byte-aligned input).
__device__ __forceinline__ void lw_load(const FpropParams& prm, const LwTicket& t, long long total,
                                        int hw, int lane, bool vec, float4 (&v)[kLwPx / 2]) {
  const int c = t.c0 + lane;
  const bool ok = t.tk < total && c < prm.c;
  if (prm.lw_pr != nullptr) {
    // fp32 NHWC planes: for each pixel, lane = channel reads one 128-byte run
    // per plane (already channel-contiguous: no transpose).
    const long long o0 = (static_cast<long long>(t.img) * hw + t.px0) * prm.c + c;
    const int np = min(kLwPx, hw - t.px0);
    const long long cs = prm.c;
#pragma unroll
    for (int j = 0; j < kLwPx / 2; ++j) {
      const bool a = ok && 2 * j < np;
      const bool b = ok && 2 * j + 1 < np;
      const long long o = o0 + 2 * j * cs;
      v[j] = make_float4(a ? __ldg(prm.lw_pr + o) : 0.f, a ? __ldg(prm.lw_pi + o) : 0.f,
                         b ? __ldg(prm.lw_pr + o + cs) : 0.f, b ? __ldg(prm.lw_pi + o + cs) : 0.f);
    }
    return;
  }
  const float2* src = reinterpret_cast<const float2*>(prm.xc) +
                      (static_cast<long long>(t.img) * prm.c + c) * hw + t.px0;
  const int np = min(kLwPx, hw - t.px0);
  if (vec) {
#pragma unroll
    for (int j = 0; j < kLwPx / 2; ++j) {
      v[j] = (ok && 2 * j < np) ? __ldg(reinterpret_cast<const float4*>(src + 2 * j))
                                : make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
#pragma unroll
    for (int j = 0; j < kLwPx / 2; ++j) {
      const float2 a = (ok && 2 * j < np) ? __ldg(src + 2 * j) : make_float2(0.f, 0.f);
      const float2 b = (ok && 2 * j + 1 < np) ? __ldg(src + 2 * j + 1) : make_float2(0.f, 0.f);
      v[j] = make_float4(a.x, a.y, b.x, b.y);
    }
  }
}

// Stores of one ticket: for each pixel, lane = channel gives one 128-byte
// run per plane (fp32 NHWC).
__device__ __forceinline__ void lw_store(const FpropParams& prm, const LwTicket& t, int hw,
                                         int lane, const float4 (&v)[kLwPx / 2]) {
  const int c = t.c0 + lane;
  if (c >= prm.c) return;
  const long long o0 = (static_cast<long long>(t.img) * hw + t.px0) * prm.c + c;
  const int np = min(kLwPx, hw - t.px0);
  const long long cs = prm.c;
  if (prm.passes > 1) {
#pragma unroll
    for (int p = 0; p < kLwPx; ++p) {
      if (p < np) {
        const float a = (p & 1) ? v[p / 2].z : v[p / 2].x;
        const float b = (p & 1) ? v[p / 2].w : v[p / 2].y;
        const float ah = lw_tf32(a);
        const float bh = lw_tf32(b);
        prm.lw_xr[o0 + p * cs] = ah;
        prm.lw_xi[o0 + p * cs] = bh;
        prm.lw_xr_lo[o0 + p * cs] = a - ah;
        prm.lw_xi_lo[o0 + p * cs] = b - bh;
      }
    }
  } else {
#pragma unroll
    for (int p = 0; p < kLwPx; ++p) {
      if (p < np) {
        prm.lw_xr[o0 + p * cs] = (p & 1) ? v[p / 2].z : v[p / 2].x;
        prm.lw_xi[o0 + p * cs] = (p & 1) ? v[p / 2].w : v[p / 2].y;
      }
    }
  }
}

// One layout warp: takes chunks of tickets, two tickets in flight (the
// loads of one overlap the stores of the other), until its range runs out.
// prefix: the range is tickets [0, lw_prefix), counted by their own word, so
// the phase ends exactly there; otherwise [lw_prefix, total).  Every chunk a
// warp takes inside its range is converted by that warp.
// Completed tickets are counted per image and published in batches: after a
// warp barrier, lane 0 fences (cumulative over the warp's stores) and adds
// the count with release semantics.
__device__ __forceinline__ void layout_warp(const FpropParams& prm, int lane, bool prefix) {
  const int hw = prm.h * prm.w;
  const int tpx = (hw + kLwPx - 1) / kLwPx;
  const int per_img = tpx * ((prm.c + kLwCh - 1) / kLwCh);
  const long long total = static_cast<long long>(per_img) * prm.n;
  const bool vec = (hw & 1) == 0 && (reinterpret_cast<uintptr_t>(prm.xc) & 15) == 0;
  unsigned* ctrs = prm.lw_ctrs;
  const long long first = prefix ? 0 : prm.lw_prefix;
  const long long end = prefix ? (prm.lw_prefix < total ? prm.lw_prefix : total) : total;
  unsigned* counter = ctrs + (prefix ? kLwPrefixTicket : kLwTicket);
  // Lane 0 holds the prefetched chunk number; it is read (shuffled) only
  // when the current chunk is used up.
  unsigned pre = lane == 0 ? atomicAdd(counter, 1u) : 0u;
  long long base = 0;
  int idx = kLwChunk;
  bool out = false;  // the range is used up
  auto grab = [&]() -> long long {
    if (idx == kLwChunk) {
      if (out) return total;
      base = first + static_cast<long long>(__shfl_sync(0xffffffffu, pre, 0)) * kLwChunk;
      idx = 0;
      if (base >= end) {
        out = true;
        return total;
      }
      pre = lane == 0 ? atomicAdd(counter, 1u) : 0u;
    }
    return base + idx < end ? base + idx++ : total;
  };
  int pend_img = -1;
  unsigned pend = 0;
  auto publish = [&]() {
    if (pend == 0) return;
    __syncwarp();
    if (lane == 0) {
      __threadfence();
      asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(ctrs + kLwFlag0 + pend_img),
                   "r"(pend)
                   : "memory");
    }
    pend = 0;
  };
  auto done = [&](const LwTicket& t) {
    if (t.img != pend_img || pend >= 8) {
      publish();
      pend_img = t.img;
    }
    ++pend;
  };
  float4 va[kLwPx / 2], vb[kLwPx / 2];
  LwTicket ta = lw_decode(prm, grab(), tpx, per_img);
  lw_load(prm, ta, total, hw, lane, vec, va);
  LwTicket tb = lw_decode(prm, grab(), tpx, per_img);
  lw_load(prm, tb, total, hw, lane, vec, vb);
#pragma unroll 1
  while (ta.tk < total) {
    const long long na = grab();
    lw_store(prm, ta, hw, lane, va);
    done(ta);
    ta = lw_decode(prm, na, tpx, per_img);
    lw_load(prm, ta, total, hw, lane, vec, va);
    if (tb.tk >= total) break;
    const long long nb = grab();
    lw_store(prm, tb, hw, lane, vb);
    done(tb);
    tb = lw_decode(prm, nb, tpx, per_img);
    lw_load(prm, tb, total, hw, lane, vec, vb);
  }
  publish();
}

// Tickets every warp of a CTA converts before taking up its role: the
// images the first unit of every cluster reads (the stream-K range's images,
// when there is one, then the first wave of whole tiles), which no MMA can
// start without (a multiple of kLwChunk).  `tile_px`: output pixels per
// cluster tile (one m-tile); CCV_LW_PREFIX=0 turns the phase off (timing
// knob).
inline long long lw_prefix_images(const FpropParams& prm, int launched, long long tile_px) {
  if (knobs().lw_prefix == 0) return 0;
  const long long pq = static_cast<long long>(prm.p) * prm.q;
  const long long mtiles = (launched + prm.tiles_n - 1) / prm.tiles_n;
  long long images = (mtiles * tile_px + pq - 1) / pq;
  if (prm.sk_slots > 0) images += prm.n - prm.lw_first_img;
  return images < prm.n ? images : prm.n;
}

inline long long lw_prefix_tickets(const FpropParams& prm, int launched, long long tile_px) {
  const long long per_img = ((static_cast<long long>(prm.h) * prm.w + kLwPx - 1) / kLwPx) *
                            ((prm.c + kLwCh - 1) / kLwCh);
  return (lw_prefix_images(prm, launched, tile_px) * per_img + kLwChunk - 1) / kLwChunk * kLwChunk;
}

// Sets the prefix of a layout-warp launch: the TMA prefix when the host
// prepared it (lw_tma_images < 0: eligible) and the first wave's images
// number 1..kLwTmaMaxImages, else the all-warp ticket prefix.
inline void lw_plan_prefix(FpropParams& prm, int launched, long long tile_px) {
  long long images = lw_prefix_images(prm, launched, tile_px);
  const bool tma_on = knobs().lw_tma != 0;
  if (prm.lw_tma_images < 0 && tma_on && images >= 1) {
    // The TMA prefix converts at ~3 TB/s with every warp, the layout warps
    // at ~0.85 TB/s of input beside the MMAs (B200): take so many images
    // into the prefix that the rest converts within the convolution's time
    // (~600 TFLOP/s), when that is more than the first wave's.
    const double img_bytes = 8.0 * prm.h * prm.w * prm.c;
    const double t_conv = 8.0 * prm.n * prm.p * prm.q * static_cast<double>(prm.k) * prm.c *
                          prm.r * prm.s / 600e12;
    const long long fit = static_cast<long long>(t_conv * 0.85e12 / img_bytes);
    const long long balance = prm.n - fit;
    if (balance > images) images = balance;
    if (knobs().lw_tma_images > 0) images = knobs().lw_tma_images;
    images = images < prm.n ? images : prm.n;
  }
  if (prm.lw_tma_images < 0 && tma_on && images >= 1 && images <= kLwTmaMaxImages) {
    const long long per_img = ((static_cast<long long>(prm.h) * prm.w + kLwPx - 1) / kLwPx) *
                              ((prm.c + kLwCh - 1) / kLwCh);
    const int bufs = knobs().lw_tma_bufs;  // boxes in flight (timing knob)
    prm.lw_tma_bufs = bufs >= 2 && bufs <= kLwBoxBufs ? bufs : kLwBoxBufs;
    prm.lw_tma_images = static_cast<int>(images);
    prm.lw_prefix = images * per_img;
    return;
  }
  prm.lw_tma_images = 0;
  prm.lw_prefix = lw_prefix_tickets(prm, launched, tile_px);
}

// TMA prefix: before taking up their roles, every thread of the CTA converts
// tiles of the first lw_tma_images images (conversion order) through the
// idle operand rings: complex64 boxes of 8 rows x 16 pixels x 32 channels
// loaded by TMA (kLwBoxBufs in flight), transposed in shared memory, the
// two fp32 planes stored by TMA.  Tiles are handed out by a counter, so any
// running CTA can finish them; each CTA adds its tile count per image once
// its stores have landed.  `buf`: kLwBoxSmemBytes at a 1024-byte boundary;
// `full0`: kLwBoxBufs mbarriers (count 1); `sm`: kLwBoxBufs + kLwTmaMaxImages
// words of shared memory.  Returns false if a wait ran out (status set).
__device__ __forceinline__ bool lw_tma_prefix(const FpropParams& prm, uint8_t* buf, uint32_t full0,
                                              unsigned* sm) {
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int nwarps = blockDim.x >> 5;
  const int th = (prm.h + kLwBoxRows - 1) / kLwBoxRows;
  const int tw = (prm.w + kLwBoxPx - 1) / kLwBoxPx;
  const int tc = (prm.c + kLwBoxCh - 1) / kLwBoxCh;
  const int per_img = th * tw * tc;
  const unsigned total = static_cast<unsigned>(per_img * prm.lw_tma_images);
  const int nbuf = prm.lw_tma_bufs;  // boxes in flight (<= kLwBoxBufs)
  unsigned* ctr = prm.lw_ctrs + kLwTmaTicket;
  volatile unsigned* tks = sm;                   // ticket of each input buffer
  volatile unsigned* cnt = sm + kLwBoxBufs;      // this CTA's tiles per image (order)
  uint8_t* in = buf;
  uint8_t* out = buf + nbuf * kLwBoxInBytes;
  const uint32_t in_u = ptx::smem_u32(in);
  const uint32_t out_u = ptx::smem_u32(out);
  auto coords = [&](unsigned tk, int& order, int& img, int& c0, int& w0, int& h0) {
    order = static_cast<int>(tk / per_img);
    const int j = static_cast<int>(tk - static_cast<unsigned>(order) * per_img);
    img = (order + prm.lw_first_img) % prm.n;
    const int cb = j % tc;
    const int rest = j / tc;
    c0 = cb * kLwBoxCh;
    w0 = (rest % tw) * kLwBoxPx;
    h0 = (rest / tw) * kLwBoxRows;
  };
  auto load = [&](int b, unsigned tk) {  // thread 0
    tks[b] = tk;
    if (tk < total) {
      int order, img, c0, w0, h0;
      coords(tk, order, img, c0, w0, h0);
      const uint32_t bar = full0 + 8u * static_cast<uint32_t>(b);
      ptx::mbar_arrive_expect_tx(bar, kLwBoxInBytes);
      ptx::tma_load_4d(in_u + static_cast<uint32_t>(b) * kLwBoxInBytes, &prm.tm_cin, bar, w0, c0, h0,
                       img);
    }
  };
  if (tid == 0) {
    for (int i = 0; i < kLwTmaMaxImages; ++i) cnt[i] = 0u;
    for (int b = 0; b < nbuf; ++b) load(b, atomicAdd(ctr, 1u));
  }
  ptx::cta_sync();
  bool ok = true;
#pragma unroll 1
  for (int k = 0;; ++k) {
    const int b = k % nbuf;
    const unsigned tk = tks[b];
    if (tk >= total) break;  // tickets grow: the later buffers are past the end too
    int order, img, c0, w0, h0;
    coords(tk, order, img, c0, w0, h0);
    // The ticket for this buffer's next box: taken now, used after the
    // transpose, so the atomic's round trip overlaps the wait and the copy.
    unsigned nxt = 0;
    if (tid == 0) nxt = atomicAdd(ctr, 1u);
    const bool got = ptx::mbar_wait_bounded_backoff(full0 + 8u * static_cast<uint32_t>(b),
                                                    static_cast<uint32_t>(k / nbuf) & 1u,
                                                    prm.status, CCV_ERR_DEVICE_TIMEOUT);
    const int ob = k & 1;
    if (tid == 0 && k >= 2) ptx::bulk_wait_read_le1();  // the store of k-2 has read its buffer
    if (ptx::cta_sync_or(!got)) {
      ok = false;
      break;
    }
    // Transpose: lane = channel, (row, pixel pair) spread over the warps.
    const uint8_t* src = in + static_cast<uint32_t>(b) * kLwBoxInBytes;
    float* orr = reinterpret_cast<float*>(out + static_cast<uint32_t>(ob) * 2u * kLwBoxOutPlane);
    float* oii = orr + kLwBoxOutPlane / 4;
    for (int idx = warp; idx < kLwBoxRows * (kLwBoxPx / 2); idx += nwarps) {
      const int r = idx / (kLwBoxPx / 2);
      const int q = idx % (kLwBoxPx / 2);
      const int line = r * kLwBoxCh + lane;
      // 128-byte swizzle: 16-byte chunk q of line `line` is at chunk q ^ (line & 7).
      const float4 v = *reinterpret_cast<const float4*>(
          src + static_cast<uint32_t>(line) * 128u + (static_cast<uint32_t>(q ^ (line & 7)) << 4));
      const int p0 = (r * kLwBoxPx + 2 * q) * kLwBoxCh + lane;
      orr[p0] = v.x;
      oii[p0] = v.y;
      orr[p0 + kLwBoxCh] = v.z;
      oii[p0 + kLwBoxCh] = v.w;
    }
    ptx::fence_proxy_async_shared();
    ptx::cta_sync();
    if (tid == 0) {
      const uint32_t o = out_u + static_cast<uint32_t>(ob) * 2u * kLwBoxOutPlane;
      ptx::tma_store_4d(&prm.tm_pr, o, c0, w0, h0, img);
      ptx::tma_store_4d(&prm.tm_pi, o + kLwBoxOutPlane, c0, w0, h0, img);
      ptx::bulk_commit_group();
      cnt[order] = cnt[order] + 1u;
      load(b, nxt);  // buffer b was read by the transpose above
    }
  }
  if (tid == 0) {
    // Every store has landed: publish this CTA's tiles per image.
    ptx::bulk_wait_all();
    ptx::fence_proxy_async_all();
    __threadfence();
    for (int o = 0; o < prm.lw_tma_images; ++o) {
      const unsigned c = cnt[o];
      if (c != 0u) {
        const int img = (o + prm.lw_first_img) % prm.n;
        asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(prm.lw_ctrs + kLwFlag0 + img),
                     "r"(c)
                     : "memory");
      }
    }
  }
  ptx::cta_sync();
  return ok;
}

// Waits (bounded) until image `img`'s planes are written; then orders the
// caller's later TMA (async-proxy) reads after those generic-proxy stores.
__device__ __forceinline__ int lw_tma_tiles_per_image(const FpropParams& prm) {
  return ((prm.h + kLwBoxRows - 1) / kLwBoxRows) * ((prm.w + kLwBoxPx - 1) / kLwBoxPx) *
         ((prm.c + kLwBoxCh - 1) / kLwBoxCh);
}

__device__ __forceinline__ bool lw_wait_image(const FpropParams& prm, int img) {
  const unsigned* f = prm.lw_ctrs + kLwFlag0 + img;
  // Images the TMA prefix converted count tiles, the others tickets.
  const int order = (img - prm.lw_first_img + prm.n) % prm.n;
  const unsigned need = static_cast<unsigned>(order < prm.lw_tma_images
                                                  ? lw_tma_tiles_per_image(prm)
                                                  : lw_tickets_per_image(prm));
  const uint64_t t0 = ptx::globaltimer();
  uint32_t ns = 64;
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
    if (v >= need) break;
    if (ptx::globaltimer() - t0 > CCV_WAIT_TIMEOUT_NS) {
      ptx::report_status(prm.status, CCV_ERR_DEVICE_TIMEOUT);
      return false;
    }
    ptx::nanosleep(ns);
    if (ns < 512) ns <<= 1;
  }
  ptx::fence_proxy_async_all();
  return true;
}

}  // namespace ccv
