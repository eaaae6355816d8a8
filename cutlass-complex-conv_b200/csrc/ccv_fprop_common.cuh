// Shared by the fprop kernel families: kernel parameters and the spatial
// tiling of the GEMM M dimension (output pixels) into TMA boxes.
#pragma once

#include <cuda.h>

#include "ccv_internal.h"

namespace ccv {

constexpr int kBlockM = 128;  // GEMM rows (output pixels) per CTA tile

struct alignas(64) FpropParams {
  CUtensorMap tm_xr;  // activation real plane
  CUtensorMap tm_xi;  // activation imaginary plane
  CUtensorMap tm_w;   // packed weights [image][R*S][3][K][C] (image 1 = 3xTF32 remainders)
  CUtensorMap tm_xr_lo;  // 3xTF32: activation remainder planes (x - tf32(x))
  CUtensorMap tm_xi_lo;
  // Planar output through TMA stores (out_tma != 0): y_real / y_imag as
  // (K, Q, P, N) boxes of 16 channels x out_px pixels x out_rows rows, or
  // (K, N*P*Q) boxes of 16 channels x 32 pixels for flat tiles.
  CUtensorMap tm_y0;
  CUtensorMap tm_y1;
  // TMA prefix of the layout warps: complex64 NCHW input as 8-byte elements
  // (W, C, H, N), and the fp32 NHWC planes it fills (C, W, H, N) - the
  // planes tm_xr / tm_xi read.
  CUtensorMap tm_cin;
  CUtensorMap tm_pr;
  CUtensorMap tm_pi;
  unsigned* lw_ctrs;  // layout-warp counter set
  const float* xc;    // layout warps: complex64 NCHW input (interleaved)
  // Layout warps: the fp32 NHWC planes they write from xc (the planes tm_xr,
  // tm_xi, tm_xr_lo, tm_xi_lo read).
  float* lw_xr;
  float* lw_xi;
  float* lw_xr_lo;
  float* lw_xi_lo;
  // Planar source of the layout warps (3xTF32 forward_planar: fp32 NHWC
  // planes split into hi/remainder planes); null: complex64 NCHW from xc.
  const float* lw_pr;
  const float* lw_pi;
  int lw_first_img;  // image the layout warps convert first
  long long lw_prefix;  // tickets every warp converts before its role (first wave's images)
  int lw_tma_images;    // images the TMA prefix converts instead (0: warp prefix)
  int lw_tma_bufs;      // TMA prefix: boxes in flight
  float* y0;          // planar: y_real (NPQK); complex: interleaved NKPQ
  float* y1;          // planar: y_imag (NPQK); complex: unused
  // Complex bias per output channel (K fp32 each), added in the epilogue;
  // null: none.  Either both are set or neither.
  const float* bias_r;
  const float* bias_i;
  int* status;        // device status word
  int n, h, w, c, k, r, s, p, q;
  int sh, sw, ph, pw;
  int box_p, box_q, box_q_log2, box_px_log2, nb;  // spatial box tiling
  int tiles_bp, tiles_bq, total_boxes;
  int tiles_m, tiles_n;
  int ksteps;         // ceil(C/16) * R * S
  long long m_total;  // N*P*Q (flat mode)
  int num_tiles;      // work units of the persistent kernel
  // halo kernel: rows of one shifted activation copy, ring depths and sizes
  int halo_rows, a_slots, w_stages, a_slot_bytes, w_stage_bytes;
  // precision passes per K step: 1 (TF32) or 3 (3xTF32: hi*hi, hi*lo, lo*hi;
  // see slot_pass for their order)
  int passes;
  // single-CTA kernel: CTAs per output tile (a cluster splitting the K loop)
  int splits;
  // Pair kernels, stream-K tail.  Tiles [0, sk_start) run whole, tile t on
  // cluster t mod G.  The K slots (A-operand loads; slots_per_tile per tile)
  // of the tiles from sk_start on are numbered s = (t - sk_start) * L + j and
  // cut into sk_clusters contiguous ranges, range g going to cluster g before
  // its whole tiles.  A tile covered by several ranges is "split": each piece
  // writes fp32 partial rows to split_ws and adds its slot count to a counter
  // in split_count (a zeroed library-owned set); the piece that brings the
  // count to L (the last to finish; nobody waits) sums all pieces' partials in
  // cluster order, stores the output and zeroes the counter.  sk_slots == 0:
  // no tail split (split_ws unused).
  int out_tma;
  int sk_start, sk_clusters, slots_per_tile;
  long long sk_slots;  // < 2^31 (checked on the host)
  float* split_ws;
  unsigned* split_count;
};

inline void set_epilogue(FpropParams& prm, const Epilogue& ep) {
  prm.bias_r = ep.bias_r;
  prm.bias_i = ep.bias_i;
}

#ifdef __CUDACC__
// Adds the complex bias of output channels [kb, kb + W) to a row's real and
// imaginary accumulator values (fp32 bits), once per output element: callers
// apply it to final sums only, never to split-K partials.  K % 4 == 0, so a
// group of four channels is either wholly inside K or wholly outside.
template <int W>
__device__ __forceinline__ void add_bias(const FpropParams& prm, int kb, uint32_t (&vr)[W],
                                         uint32_t (&vi)[W]) {
  if (prm.bias_r == nullptr) return;
#pragma unroll
  for (int j = 0; j < W; j += 4) {
    if (kb + j < prm.k) {
      const float4 br = __ldg(reinterpret_cast<const float4*>(prm.bias_r + kb + j));
      const float4 bi = __ldg(reinterpret_cast<const float4*>(prm.bias_i + kb + j));
      vr[j] = __float_as_uint(__uint_as_float(vr[j]) + br.x);
      vr[j + 1] = __float_as_uint(__uint_as_float(vr[j + 1]) + br.y);
      vr[j + 2] = __float_as_uint(__uint_as_float(vr[j + 2]) + br.z);
      vr[j + 3] = __float_as_uint(__uint_as_float(vr[j + 3]) + br.w);
      vi[j] = __float_as_uint(__uint_as_float(vi[j]) + bi.x);
      vi[j + 1] = __float_as_uint(__uint_as_float(vi[j + 1]) + bi.y);
      vi[j + 2] = __float_as_uint(__uint_as_float(vi[j + 2]) + bi.z);
      vi[j + 3] = __float_as_uint(__uint_as_float(vi[j + 3]) + bi.w);
    }
  }
}
#endif

// Work of one persistent cluster: its stream-K range, then whole tiles.
// K slot order of the pair kernels: the precision pass is outermost, and
// 3xTF32 runs its two correction passes (pass 1: hi(x)*lo(w), pass 2:
// lo(x)*hi(w)) before the main pass 0 (hi*hi).  The tensor cores' fp32
// accumulation loses a fraction of the accumulator's magnitude per MMA, so
// the correction MMAs run while the accumulator is still small and only the
// main pass's MMAs see the full magnitude.  Returns the pass of slot j;
// *rest = the slot's index inside its pass (per_pass slots per pass).
__device__ __forceinline__ int slot_pass(int j, int per_pass, int passes, int* rest) {
  const int pidx = j / per_pass;
  *rest = j - pidx * per_pass;
  return passes == 1 ? 0 : (pidx == 2 ? 0 : pidx + 1);
}

struct UnitCursor {
  int dp;       // next whole tile
  int s, s1;    // remaining stream-K slot range
};

// One unit: slots [jbeg, jend) of tile `tile`; `split` when the unit is a
// piece of a split tile (sk = the tile's index among stream-K tiles).
struct WorkUnit {
  int tile, jbeg, jend, sk;
  bool split;
};

__host__ __device__ inline long long sk_range_begin(const FpropParams& prm, int g) {
  return static_cast<long long>(g) * prm.sk_slots / prm.sk_clusters;
}

__host__ __device__ inline UnitCursor unit_cursor(const FpropParams& prm, int cid) {
  UnitCursor c;
  c.dp = cid;
  c.s = c.s1 = 0;
  if (prm.sk_slots > 0 && cid < prm.sk_clusters) {
    c.s = static_cast<int>(sk_range_begin(prm, cid));
    c.s1 = static_cast<int>(sk_range_begin(prm, cid + 1));
  }
  return c;
}

__host__ __device__ inline bool next_unit(const FpropParams& prm, int ncl, UnitCursor& c,
                                          WorkUnit& w) {
  const int L = prm.slots_per_tile;
  // The stream-K range first: a split tile's sum is then finished by
  // whichever piece ends last while its cluster goes on with whole tiles.
  // (Measured: whole tiles first, split pieces last, ran the batch-8 share
  // of the 56x56 layer in 73 us instead of 56 us - the last pieces then
  // wait for each other at the end of the launch.)
  if (c.s < c.s1) {
    const int a = c.s / L;
    const int end = c.s1 < (a + 1) * L ? c.s1 : (a + 1) * L;
    w.sk = a;
    w.tile = prm.sk_start + a;
    w.jbeg = c.s - a * L;
    w.jend = end - a * L;
    w.split = !(w.jbeg == 0 && w.jend == L);
    c.s = end;
    return true;
  }
  if (c.dp < prm.sk_start) {
    w.tile = c.dp;
    w.jbeg = 0;
    w.jend = L;
    w.sk = -1;
    w.split = false;
    c.dp += ncl;
    return true;
  }
  return false;
}

// True when the cursor has no unit left.
__host__ __device__ inline bool cursor_done(const FpropParams& prm, const UnitCursor& c) {
  return c.dp >= prm.sk_start && c.s >= c.s1;
}

// Clusters whose stream-K ranges cover parts of stream-K tile `a`: g_first
// .. g_last (every range holds at least one slot).
__host__ __device__ inline void sk_tile_clusters(const FpropParams& prm, int a, int& g_first,
                                                 int& g_last) {
  const long long L = prm.slots_per_tile;
  const long long G = prm.sk_clusters;
  const long long X = prm.sk_slots;
  long long f = ((a * L + 1) * G + X - 1) / X - 1;
  long long l = (((a + 1) * L) * G + X - 1) / X - 1;
  g_first = static_cast<int>(f < G - 1 ? f : G - 1);
  g_last = static_cast<int>(l < G - 1 ? l : G - 1);
}

// Partial buffer of cluster g's piece of stream-K tile a: index 0 when g's
// range starts inside the tile, 1 when it started in an earlier tile (then
// the piece is the range's last unit).  Buffers hold 128 rows x 2*KT fp32
// per CTA of the pair.
__host__ __device__ inline long long sk_partial_index(const FpropParams& prm, int g, int a,
                                                      int rank) {
  const int idx = sk_range_begin(prm, g) >= static_cast<long long>(a) * prm.slots_per_tile ? 0 : 1;
  return (static_cast<long long>(g) * 2 + idx) * 2 + rank;
}

// Tiling of the output pixels: 128-row tiles made of NB boxes of
// box_p x box_q output pixels (powers of two), or flat 128-pixel runs for
// 1x1 / stride-1 / pad-0 problems.
struct Tiling {
  bool flat = false;
  int kt = 128;
  int box_p = 1, box_q = 1, nb = 1;
  int tiles_bp = 1, tiles_bq = 1, total_boxes = 1;
  int tiles_m = 1, tiles_n = 1;
};

inline int ilog2(int v) {
  int l = 0;
  while ((1 << l) < v) ++l;
  return l;
}

// fewest_loaded: among tilings computing the same rows prefer the one that
// loads the fewest activation rows when boxes past the problem's last box are
// skipped (the single-CTA kernel skips them; the pair kernels repeat the last
// box), then the fewest boxes per tile; boxes of at least 64 pixels (smaller
// TMA boxes load slower).  A 7x7 image is then one 8x8 box of a two-box tile
// (64 loaded rows) rather than one 8x16 box (128).
inline Tiling choose_tiling(const Problem& pb, bool fewest_loaded = false) {
  Tiling t;
  t.kt = pb.k > 64 ? 128 : (pb.k > 32 ? 64 : 32);
  t.tiles_n = (pb.k + t.kt - 1) / t.kt;
  t.flat = (pb.r == 1 && pb.s == 1 && pb.sh == 1 && pb.sw == 1 && pb.ph == 0 && pb.pw == 0);
  if (t.flat) {
    const long long m = static_cast<long long>(pb.n) * pb.p * pb.q;
    t.tiles_m = static_cast<int>((m + kBlockM - 1) / kBlockM);
    return t;
  }
  // Spatial boxes: box_p x box_q (powers of two, product 8..128, at most 4
  // boxes per tile), chosen to cover P x Q with the fewest computed rows.
  long long best_cost = -1;
  for (int px = fewest_loaded ? 64 : 32; px <= 128; px *= 2) {
    const int nb = kBlockM / px;
    for (int bq = 1; bq <= px; bq *= 2) {
      const int bp = px / bq;
      if (bq * pb.sw > 256 || bp * pb.sh > 256) continue;
      const long long tbq = (pb.q + bq - 1) / bq;
      const long long tbp = (pb.p + bp - 1) / bp;
      const long long boxes = static_cast<long long>(pb.n) * tbq * tbp;
      const long long tiles = (boxes + nb - 1) / nb;
      // Rows computed, then (fewest_loaded) rows loaded, then fewer boxes.
      const long long cost = fewest_loaded ? (tiles * kBlockM * 4096 + boxes * px * 4 + nb)
                                           : (tiles * kBlockM * 4 + nb);
      if (best_cost < 0 || cost < best_cost) {
        best_cost = cost;
        t.box_p = bp;
        t.box_q = bq;
        t.nb = nb;
        t.tiles_bp = static_cast<int>(tbp);
        t.tiles_bq = static_cast<int>(tbq);
        t.total_boxes = static_cast<int>(boxes);
        t.tiles_m = static_cast<int>(tiles);
      }
    }
  }
  return t;
}

// CTA-pair kernel family (ccv_fprop2.cu): work units are pairs of 128-row
// tiles; returns the number of such units.
int pair_tiles(const Tiling& t);
// xr_lo/xi_lo: 3xTF32 remainder planes (nullptr for TF32); xr/xi then hold
// the TF32-rounded parts.
// lw_src (complex64 NCHW) or lw_pr/lw_pi (fp32 NHWC planes): layout warps
// fill xr/xi (and the remainder planes) from that source in the same launch.
int launch_fprop_pair(const float* xr, const float* xi, const float* xr_lo, const float* xi_lo,
                      const float* w_packed, float* y0, float* y1, const Problem& pb,
                      const Tiling& t, OutLayout out_layout, const Epilogue& ep, void* ws,
                      size_t ws_bytes, cudaStream_t stream, const float* lw_src = nullptr,
                      const float* lw_pr = nullptr, const float* lw_pi = nullptr);

// Halo variant of the pair kernel (ccv_fprop2h.cu): stride-1 problems with a
// filter wider than 1x1.  Each CTA tile is one box of box_p x box_q pixels
// (box_q a multiple of 8); per 32-channel block the S column-shifted halo
// copies of the box are loaded once and reused by the R filter rows.
bool halo_applicable(const Problem& pb);
// Scratch bytes that let a pair kernel with KT-wide tiles, `tiles` pair
// tiles and `slots` K slots per tile split its last partial wave stream-K
// style (partials and counters; an upper bound for the current device).
size_t pair_split_workspace_bytes(int kt, int tiles, int slots);
// Stream-K plan for a persistent pair kernel: sets prm.sk_* / slots_per_tile
// for `clusters` co-resident clusters and `slots` K slots per tile, using ws
// (at least pair_split_workspace_bytes(kt)) when given and worthwhile.
// Returns the number of counters to zero before the launch (0: no split).
int plan_stream_k(FpropParams& prm, int clusters, int slots, int kt, void* ws, size_t ws_bytes,
                  cudaStream_t stream, int min_gain_pct = 10);
// Persistent-grid size after the CCV_MAX_CLUSTERS testing cap.
int cluster_cap(int max_clusters);
// Plans the stream-K split and returns the number of clusters to launch;
// *rc receives the status.
int launch_clusters(FpropParams& prm, int clusters, int slots, int kt, void* ws, size_t ws_bytes,
                    cudaStream_t stream, int* rc, int min_gain_pct = 10);
Tiling choose_halo_tiling(const Problem& pb);
// Same for tiles of `px` output pixels per CTA (128 or 256).
Tiling choose_halo_tiling_px(const Problem& pb, int px);
// Bytes of shared memory a pair kernel sets aside for the TMA-store epilogue
// (4 warps x 32 rows x 16 channels x 2 planes).
constexpr int kOutStageBytes = 4 * 32 * 16 * 4 * 2;
// Encodes prm.tm_y0 / tm_y1 for planar output (16-channel x 32-pixel boxes,
// 64-byte swizzle: the layout store_accumulator_tma stages) and sets
// prm.out_tma when the tiling lets each epilogue warp's 32 rows form one box.
int encode_planar_out_maps(FpropParams& prm, float* y0, float* y1, bool flat);

// ws/ws_bytes: optional scratch for the tail split (pair_split_workspace_bytes);
// without it every tile runs whole.  lw_src / lw_pr, lw_pi: as for
// launch_fprop_pair (layout warps in the same launch).
int launch_fprop_pair_halo(const float* xr, const float* xi, const float* xr_lo,
                           const float* xi_lo, bool split, const float* w_packed, float* y0,
                           float* y1, const Problem& pb, const Tiling& t, OutLayout out_layout,
                           const Epilogue& ep, void* ws, size_t ws_bytes, cudaStream_t stream,
                           const float* lw_src = nullptr, const float* lw_pr = nullptr,
                           const float* lw_pi = nullptr);

}  // namespace ccv
