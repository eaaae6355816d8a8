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

// Stores channels [kb, kb + W) of pixel (img, op, oq) from vr (real) and
// vi (imaginary), final sums, as fp32 NPQK planes or complex64 NKPQ
// (W % 4 == 0), adding the launch's complex bias if it has one.
template <bool OUT_COMPLEX, int W>
__device__ __forceinline__ void store_chunk(const FpropParams& prm, int kb, int img, int op,
                                            int oq, uint32_t (&vr)[W], uint32_t (&vi)[W]) {
  add_bias<W>(prm, kb, vr, vi);
  if constexpr (!OUT_COMPLEX) {
    const long long pix = (static_cast<long long>(img) * prm.p + op) * prm.q + oq;
    float* dr = prm.y0 + pix * prm.k + kb;
    float* di = prm.y1 + pix * prm.k + kb;
#pragma unroll
    for (int j = 0; j < W; j += 4) {
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
    for (int j = 0; j < W; ++j) {
      if (kb + j < prm.k) {
        y[base + static_cast<long long>(kb + j) * pq] =
            make_float2(__uint_as_float(vr[j]), __uint_as_float(vi[j]));
      }
    }
  }
}

// Reads the accumulator row of this thread (TMEM address `t_acc`: lane of
// the thread, column 0 of the [re | im] block) in CW-column chunks (16 or 32;
// 16 halves the registers it holds) and stores output channels [k0, k0 + KT)
// of pixel (img, op, oq).  Every thread of the warp must call this
// (tcgen05.ld is warp-collective); `valid` masks stores.
template <int KT, bool OUT_COMPLEX, int CW = 32>
__device__ __forceinline__ void store_accumulator(const FpropParams& prm, uint32_t t_acc, int k0,
                                                  bool valid, int img, int op, int oq) {
#pragma unroll 1
  for (int ch = 0; ch < KT; ch += CW) {
    uint32_t vr[CW], vi[CW];
    ptx::tmem_ld_32x32b<CW>(t_acc + ch, vr);
    ptx::tmem_ld_32x32b<CW>(t_acc + KT + ch, vi);
    ptx::tmem_wait_ld();
    const int kb = k0 + ch;
    if (!valid || kb >= prm.k) continue;
    store_chunk<OUT_COMPLEX, CW>(prm, kb, img, op, oq, vr, vi);
  }
}

// Planar output through TMA stores.  The warp's 32 rows (TMEM lanes) are one
// box of the output: a 4 KB buffer of `stage` (32 rows x 16 channels for each
// plane) is filled from TMEM 16 channels at a time and lane 0 issues the two
// tensor stores.  With NBUF = 2 the warp's chunks alternate between two
// buffers, so filling one overlaps the stores still reading the other;
// `seq` counts this warp's committed chunks across calls (the buffer of the
// next one) and must start at 0.  (c1, c2, c3) are the box's pixel
// coordinates in the output tensor map (q, p, n; or m, -, - for flat tiles).
// `valid`: the box holds real pixels.
template <int KT, bool FLAT, int NBUF = 1>
__device__ __forceinline__ void store_accumulator_tma(const FpropParams& prm, uint32_t t_acc,
                                                      int k0, bool valid, int c1, int c2, int c3,
                                                      uint8_t* stage, int lane, uint32_t& seq) {
  static_assert(NBUF == 1 || NBUF == 2, "one or two staging buffers");
  static_assert(KT % 32 == 0, "chunks are processed in pairs");
  // TMEM reads run one chunk ahead: chunk ch+16's loads are issued before
  // chunk ch is staged and stored, so their latency overlaps that work.
  uint32_t nr[16], ni[16];
  ptx::tmem_ld_32x32b_x16(t_acc, nr);
  ptx::tmem_ld_32x32b_x16(t_acc + KT, ni);
  ptx::tmem_wait_ld();
  ptx::reg_fence(nr);
  ptx::reg_fence(ni);
#pragma unroll 2
  for (int ch = 0; ch < KT; ch += 16) {
    uint32_t vr[16], vi[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      vr[j] = nr[j];
      vi[j] = ni[j];
    }
    if (ch + 16 < KT) {
      ptx::tmem_ld_32x32b_x16(t_acc + ch + 16, nr);
      ptx::tmem_ld_32x32b_x16(t_acc + KT + ch + 16, ni);
    }
    const bool go = valid && k0 + ch < prm.k;
    if (!go) {
      ptx::tmem_wait_ld();
      ptx::reg_fence(nr);
      ptx::reg_fence(ni);
      continue;
    }
    add_bias<16>(prm, k0 + ch, vr, vi);
    float* sr = reinterpret_cast<float*>(stage + (NBUF == 2 ? (seq & 1u) * 4096u : 0u));
    float* si = sr + 32 * 16;
    ++seq;
    // The stores that last read this buffer are done with it: with two
    // buffers that is every group but the most recent one.
    if (lane == 0) {
      if constexpr (NBUF == 2) {
        ptx::bulk_wait_read_le1();
      } else {
        ptx::bulk_wait_read_all();
      }
    }
    __syncwarp();
    // Row `lane`: 16 channels (64 B) in the 64-byte swizzle of the output
    // tensor maps - 16-byte chunk j of row r sits at chunk j ^ ((r >> 1) & 3)
    // (the buffers are 512-byte aligned) - so the lanes of each store below
    // cover all banks with static register indices.
    const int rot = (lane >> 1) & 3;
    float4* rr = reinterpret_cast<float4*>(sr + lane * 16);
    float4* ri = reinterpret_cast<float4*>(si + lane * 16);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      rr[j ^ rot] = make_float4(__uint_as_float(vr[4 * j]), __uint_as_float(vr[4 * j + 1]),
                                __uint_as_float(vr[4 * j + 2]), __uint_as_float(vr[4 * j + 3]));
      ri[j ^ rot] = make_float4(__uint_as_float(vi[4 * j]), __uint_as_float(vi[4 * j + 1]),
                                __uint_as_float(vi[4 * j + 2]), __uint_as_float(vi[4 * j + 3]));
    }
    ptx::fence_proxy_async_shared();
    __syncwarp();
    if (lane == 0) {
      const uint32_t ur = ptx::smem_u32(sr);
      const uint32_t ui = ptx::smem_u32(si);
      if constexpr (FLAT) {
        ptx::tma_store_2d(&prm.tm_y0, ur, k0 + ch, c1);
        ptx::tma_store_2d(&prm.tm_y1, ui, k0 + ch, c1);
      } else {
        ptx::tma_store_4d(&prm.tm_y0, ur, k0 + ch, c1, c2, c3);
        ptx::tma_store_4d(&prm.tm_y1, ui, k0 + ch, c1, c2, c3);
      }
      ptx::bulk_commit_group();
    }
    ptx::tmem_wait_ld();
    ptx::reg_fence(nr);
    ptx::reg_fence(ni);
  }
}

// Output pixel of tile row `row0` (the first of an epilogue warp's 32 rows)
// of tile half `half` in the coordinates of the planar output maps; false
// when it holds no output.
template <bool FLAT>
__device__ __forceinline__ bool warp_box_origin(const FpropParams& prm, int half, int row0,
                                                int& c1, int& c2, int& c3) {
  if constexpr (FLAT) {
    const long long m = static_cast<long long>(half) * kBlockM + row0;
    c1 = static_cast<int>(m);
    c2 = c3 = 0;
    return m < prm.m_total;
  } else {
    int img = 0, op = 0, oq = 0;
    const bool ok = tile_row_pixel<false>(prm, half, row0, img, op, oq);
    c1 = oq;
    c2 = op;
    c3 = img;
    return ok;
  }
}

// Epilogue of one piece of a split (stream-K) tile, for the 32 rows of one
// warp (`quarter`) of CTA `rank`.  The warp writes its TMEM accumulator rows
// to this piece's partial buffer and adds the piece's slot count to the
// tile's counter.  The warp that completes the count (all L slots summed;
// nobody waits for anybody) adds every piece's rows in cluster order - its
// own taken from TMEM, the others from the partial buffers; the same order
// whichever piece finishes last, so results are deterministic - and stores
// the output rows.  Then TMEM is released by an arrival on the MMA CTA's
// barrier `tempty_remote` (cluster address).  Returns whether this warp
// stored the tile.
//
// Partial buffer layout (per CTA: 128 rows x 2*KT fp32): four 32-row blocks,
// one per epilogue warp.  A block is a sequence of 8-channel granules; a
// granule holds four float4 "columns" (re 0-3, re 4-7, im 0-3, im 4-7) and
// column j of row `lane` sits at float4 index j * 32 + lane.  So a warp
// moves 512 contiguous bytes per access and any run of granules is one
// contiguous range (2 KB per granule).
//
// The sum is staged through shared memory when the caller hands this warp a
// free region (`stage`, `stage_bytes`; the kernel's operand buffers after its
// last unit) and kStageBufs mbarriers from `stage_bar` (8 bytes apart): one
// bulk copy per other piece brings a run of granules in (as long a run as
// the region allows, so the copies are large), into a ring of up to
// kStageBufs buffers.  Otherwise the partial rows are read into registers,
// two granules per step.
constexpr int kStageBufs = 16;  // staging ring depth (mbarriers per epilogue warp)

template <int KT, bool OUT_COMPLEX>
__device__ __noinline__ bool split_piece_epilogue(const FpropParams& prm, WorkUnit w, int cid,
                                                  int rank, int quarter, int lane, uint32_t t_acc,
                                                  int k0, bool valid, int img, int op, int oq,
                                                  uint32_t tempty_remote, uint8_t* stage,
                                                  uint32_t stage_bytes, uint32_t stage_bar) {
  static_assert(KT % 16 == 0, "KT");
  constexpr int kRowF4 = 2 * KT / 4;       // float4 per row
  constexpr uint32_t kGranBytes = 2048u;   // one granule of a 32-row block
  float4* ws4 = reinterpret_cast<float4*>(prm.split_ws);
  // float4 index of column 0 of granule 0, row 0 of cluster g's block.
  auto block0 = [&](int g) {
    return sk_partial_index(prm, g, w.sk, rank) * (static_cast<long long>(kBlockM) * kRowF4) +
           static_cast<long long>(quarter) * 32 * kRowF4;
  };
  {
    float4* dst = ws4 + block0(cid) + lane;
    // TMEM reads one chunk ahead of the stores (as in store_accumulator_tma).
    uint32_t nr[16], ni[16];
    ptx::tmem_ld_32x32b_x16(t_acc, nr);
    ptx::tmem_ld_32x32b_x16(t_acc + KT, ni);
    ptx::tmem_wait_ld();
    ptx::reg_fence(nr);
    ptx::reg_fence(ni);
#pragma unroll 2
    for (int ch = 0; ch < KT; ch += 16) {
      uint32_t vr[16], vi[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        vr[j] = nr[j];
        vi[j] = ni[j];
      }
      if (ch + 16 < KT) {
        ptx::tmem_ld_32x32b_x16(t_acc + ch + 16, nr);
        ptx::tmem_ld_32x32b_x16(t_acc + KT + ch + 16, ni);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float4* gd = dst + ((ch / 8 + h) * 4) * 32;
        const uint32_t* r = vr + 8 * h;
        const uint32_t* m = vi + 8 * h;
        __stcg(gd, make_float4(__uint_as_float(r[0]), __uint_as_float(r[1]),
                               __uint_as_float(r[2]), __uint_as_float(r[3])));
        __stcg(gd + 32, make_float4(__uint_as_float(r[4]), __uint_as_float(r[5]),
                                    __uint_as_float(r[6]), __uint_as_float(r[7])));
        __stcg(gd + 64, make_float4(__uint_as_float(m[0]), __uint_as_float(m[1]),
                                    __uint_as_float(m[2]), __uint_as_float(m[3])));
        __stcg(gd + 96, make_float4(__uint_as_float(m[4]), __uint_as_float(m[5]),
                                    __uint_as_float(m[6]), __uint_as_float(m[7])));
      }
      ptx::tmem_wait_ld();
      ptx::reg_fence(nr);
      ptx::reg_fence(ni);
    }
  }
  // Publish this warp's rows, then count its slots.
  __threadfence();
  __syncwarp();
  unsigned old = 0;
  unsigned* cnt = prm.split_count + (static_cast<long long>(w.sk) * 2 + rank) * 4 + quarter;
  if (lane == 0) {
    asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
                 : "=r"(old)
                 : "l"(cnt), "r"(static_cast<unsigned>(w.jend - w.jbeg))
                 : "memory");
  }
  old = __shfl_sync(0xffffffffu, old, 0);
  const bool last =
      old + static_cast<unsigned>(w.jend - w.jbeg) == static_cast<unsigned>(prm.slots_per_tile);
  // Every piece has counted: leave the counter zero for the next launch
  // that uses this counter set.
  if (last && lane == 0) {
    asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(cnt), "r"(0u) : "memory");
  }
  if (last) {
    __threadfence();
    int g0 = 0, g1 = 0;
    sk_tile_clusters(prm, w.sk, g0, g1);
    const int ng = g1 - g0 + 1;
    const int ngran = min(KT / 8, (prm.k - k0 + 7) / 8);  // granules with output channels
    // Largest run of granules per copy with at least two buffers in the
    // region (or one buffer holding every granule).
    int run = 0, nbuf = 0;
    if (stage != nullptr && ng > 1) {
      for (int cand = ngran; cand >= 1; cand = cand > 1 ? (cand + 1) / 2 : 0) {
        const uint32_t per_buf = static_cast<uint32_t>(ng - 1) * cand * kGranBytes;
        const int nchunk = (ngran + cand - 1) / cand;
        const int fit = min(kStageBufs, static_cast<int>(stage_bytes / per_buf));
        if (fit >= min(nchunk, 2)) {
          run = cand;
          nbuf = min(fit, nchunk);
          break;
        }
        if (cand == 1) break;
      }
    }
    if (run > 0) {
      const uint32_t per_buf = static_cast<uint32_t>(ng - 1) * run * kGranBytes;
      const int nchunk = (ngran + run - 1) / run;
      const uint32_t s_base = ptx::smem_u32(stage);
      // Chunk k (granules k*run ..) goes to buffer k % nbuf.
      auto issue = [&](int k) {
        if (lane == 0) {
          const int b = k % nbuf;
          const uint32_t bar = stage_bar + 8u * static_cast<uint32_t>(b);
          // First fill: order the counter acquire (generic proxy) before the
          // copies' global reads.  Refills: order this warp's shared reads of
          // the buffer before the copies' writes (shared only: a global
          // proxy fence would also wait for the output stores in flight).
          if (k < nbuf) {
            if (k == 0) ptx::fence_proxy_async_all();
          } else {
            ptx::fence_proxy_async_shared();
          }
          const int q0 = k * run;
          const int nq = min(run, ngran - q0);
          const uint32_t bytes = static_cast<uint32_t>(nq) * kGranBytes;
          ptx::mbar_arrive_expect_tx(bar, static_cast<uint32_t>(ng - 1) * bytes);
          uint32_t dst = s_base + static_cast<uint32_t>(b) * per_buf;
          for (int g = g0; g <= g1; ++g) {
            if (g == cid) continue;
            ptx::bulk_load(dst, ws4 + block0(g) + q0 * 128, bytes, bar);
            dst += static_cast<uint32_t>(run) * kGranBytes;
          }
        }
      };
      for (int k = 0; k < nbuf; ++k) issue(k);
#pragma unroll 1
      for (int k = 0; k < nchunk; ++k) {
        const int b = k % nbuf;
        if (!ptx::mbar_wait_bounded_backoff(stage_bar + 8u * static_cast<uint32_t>(b),
                                            static_cast<uint32_t>(k / nbuf) & 1u, prm.status,
                                            CCV_ERR_DEVICE_TIMEOUT)) {
          break;
        }
        const int q0 = k * run;
        const int nq = min(run, ngran - q0);
        const uint8_t* bufp = stage + static_cast<uint32_t>(b) * per_buf;
#pragma unroll 1
        for (int q = 0; q < nq; ++q) {
          const int ch = 8 * (q0 + q);
          uint32_t vr[8], vi[8];
          int o = 0;
#pragma unroll 1
          for (int g = g0; g <= g1; ++g) {
            uint32_t ar[8], ai[8];
            if (g == cid) {
              ptx::tmem_ld_32x32b_x8(t_acc + ch, ar);
              ptx::tmem_ld_32x32b_x8(t_acc + KT + ch, ai);
              ptx::tmem_wait_ld();
            } else {
              const float4* sp = reinterpret_cast<const float4*>(
                  bufp + static_cast<uint32_t>(o) * run * kGranBytes + q * kGranBytes);
              ++o;
              const float4 a0 = sp[lane], a1 = sp[32 + lane], b0 = sp[64 + lane],
                           b1 = sp[96 + lane];
              const float fa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
              const float fb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
              for (int e = 0; e < 8; ++e) {
                ar[e] = __float_as_uint(fa[e]);
                ai[e] = __float_as_uint(fb[e]);
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              vr[e] = g == g0 ? ar[e]
                              : __float_as_uint(__uint_as_float(vr[e]) + __uint_as_float(ar[e]));
              vi[e] = g == g0 ? ai[e]
                              : __float_as_uint(__uint_as_float(vi[e]) + __uint_as_float(ai[e]));
            }
          }
          if (valid) store_chunk<OUT_COMPLEX, 8>(prm, k0 + ch, img, op, oq, vr, vi);
        }
        // Every lane is done with this buffer before it is refilled.
        __syncwarp();
        if (k + nbuf < nchunk) issue(k + nbuf);
      }
    } else {
      // Register path: two granules (16 channels) per step.  The other
      // pieces' rows are "items" (step, piece) read in summation order; two
      // items are in flight at a time, so the L2 round trip of the next item
      // overlaps the sums of the current one instead of every step waiting
      // for its own loads (this path runs while the cluster's MMAs stream
      // operands, which makes each round trip long).
      const int npo = ng - 1;                        // other pieces
      const int nsteps = (8 * ngran + 15) / 16;
      const int nitems = nsteps * npo;
      auto load_item = [&](int it, float4 (&v)[8]) {
        const int step = it / npo;
        const int po = it - step * npo;
        const int g = g0 + po + (g0 + po >= cid ? 1 : 0);  // po-th piece other than cid
        const float4* src = ws4 + block0(g) + lane + (2 * step) * 128;
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = __ldcg(src + j * 32);
      };
      float4 bufa[8], bufb[8];
      if (nitems > 0) load_item(0, bufa);
      if (nitems > 1) load_item(1, bufb);
      uint32_t vr[16], vi[16];
      bool first = true, own_done = false;
      // Adds one piece's 16 channels (in cluster order) to the step's sums.
      auto add16 = [&](const uint32_t (&ar)[16], const uint32_t (&ai)[16]) {
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          vr[e] = first ? ar[e] : __float_as_uint(__uint_as_float(vr[e]) + __uint_as_float(ar[e]));
          vi[e] = first ? ai[e] : __float_as_uint(__uint_as_float(vi[e]) + __uint_as_float(ai[e]));
        }
        first = false;
      };
      // This CTA's own partial of the step, read from TMEM where it joins.
      auto add_own = [&](int step) {
        uint32_t ar[16], ai[16];
        ptx::tmem_ld_32x32b_x16(t_acc + 16 * step, ar);
        ptx::tmem_ld_32x32b_x16(t_acc + KT + 16 * step, ai);
        ptx::tmem_wait_ld();
        add16(ar, ai);
        own_done = true;
      };
      auto begin_step = [&](int) {
        first = true;
        own_done = false;
      };
      auto end_step = [&](int step) {
        if (!own_done) add_own(step);
        if (valid) store_chunk<OUT_COMPLEX, 16>(prm, k0 + 16 * step, img, op, oq, vr, vi);
      };
      // Consumes item `it` from v: the piece's value joins the sums after
      // this CTA's own partial when the piece comes later in cluster order.
      auto consume = [&](int it, const float4 (&v)[8]) {
        const int step = it / npo;
        const int po = it - step * npo;
        if (po == 0) begin_step(step);
        const int g = g0 + po + (g0 + po >= cid ? 1 : 0);
        if (!own_done && g > cid) add_own(step);
        uint32_t ar[16], ai[16];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float4 a0 = v[4 * h], a1 = v[4 * h + 1], b0 = v[4 * h + 2], b1 = v[4 * h + 3];
          const float fa[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
          const float fb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            ar[8 * h + e] = __float_as_uint(fa[e]);
            ai[8 * h + e] = __float_as_uint(fb[e]);
          }
        }
        add16(ar, ai);
        if (po == npo - 1) end_step(step);
      };
      if (npo == 0) {
#pragma unroll 1
        for (int step = 0; step < nsteps; ++step) {
          begin_step(step);
          end_step(step);
        }
      }
#pragma unroll 1
      for (int it = 0; it < nitems; it += 2) {
        consume(it, bufa);
        if (it + 2 < nitems) load_item(it + 2, bufa);
        if (it + 1 < nitems) {
          consume(it + 1, bufb);
          if (it + 3 < nitems) load_item(it + 3, bufb);
        }
      }
    }
  }
  ptx::tc_fence_before();
  __syncwarp();
  if (lane == 0) ptx::mbar_arrive_cluster_relaxed(tempty_remote);
  return last;
}

}  // namespace ccv
