// Multilevel DWT synthesis (the exact transpose of the analysis) by independent output tiles,
// for sm_100a.  Included by dwt_impl.cuh; instantiated per element type with the analysis.
//
// A CTA produces T consecutive samples of one output row.  Going from the coarsest level to
// the finest, level i turns coefficients (a_i, d_i) into a_{i-1} (y for i = 0):
//   z[p] = sum_{2o + off - j = p} h0[j] a_i[o] + h1[j] d_i[o]  on  [off - L + 1, 2(nc-1) + off],
//   a_{i-1}[q] = sum_{p : ext(p) = q} z[p]                       (fdwt/kernels/dwt.py:101-175)
// The tile needs, at every level, only the dependency cone of its outputs -- a "main" range
// that halves from level to level plus L/2 coefficients -- and, where the cone reaches a row
// end, the extended positions that fold back onto it.  Those come from two fixed windows of W
// coefficients at the two row ends of every level: a window's outputs need only the windows
// of the next coarser level (W >= L + off), so {left window, main range, right window} is
// closed under the recursion for every boundary mode.  Levels whose whole row is about as
// short as that are simply computed whole ("full" levels, which also handle rows shorter than
// the filter, where the extension wraps several times).
//
// Every coefficient the tile reads (its d ranges at all levels and its part of the coarsest
// approximation) is staged into shared memory once, up front, with cp.async; after that each
// level works from shared memory only and costs one barrier (three for a tile that computes
// outputs onto which exterior positions fold).  There are no clusters and no inter-CTA
// dependencies, so the grid is rows x tiles independent CTAs.  A CTA is small (128 threads)
// so that several tiles, each a chain of dependent levels, are in flight on every SM.
//
// Inner loop: a work item is 8 consecutive outputs starting at a multiple of 8.  Output pairs
// (p, p+1) share their coefficient window, so each coefficient o of the window feeds the pair
// through the packed taps (h[m], h[m-1]) with m = 2o - p + off: in fp32 one fma.rn.f32x2 per
// pair, tap and filter.  Because items start at multiples of 8, their windows start at o
// congruent to a launch-wide constant mod 4; segments are stored from an origin with that
// residue and one pad element per 4, so window loads are bank-conflict free and use a base
// plus immediates.
#pragma once

namespace fdwt {
namespace dwtk {

constexpr int TNT = 128;     // threads per CTA
constexpr int TQ = 4;        // output pairs per work item
constexpr int TPS = 2;       // one pad element per 4 stored coefficients
constexpr int kTileSegs = 3;

// Outputs per tile of rows longer than about one tile (shorter rows are one tile).
template <typename A>
constexpr int tile_outputs() { return sizeof(A) == 8 ? 2048 : 4096; }

// The streaming one-level synthesis (dwt_stream.cuh): filters up to kStreamMaxLM taps; a level
// of a shape for which stream_fills() holds streams every tile down to kStreamMinOut outputs.
constexpr int kStreamMaxLM = 24;
constexpr int kStreamMinOut = 512;

// One-level synthesis of this shape streams every tile: periodization over exactly one period
// (n = 2 nc: a circular convolution of the coefficients) or zero mode (nothing folds back).
inline bool stream_fills(const Level& l) {
  return (l.mode == FDWT_MODE_PERIODIZATION && l.n_in == 2 * l.n_coef && l.P == l.n_in) ||
         l.mode == FDWT_MODE_ZERO;
}

struct TileLevel {     // level i (0 = finest)
  int32_t n_out;       // output length (before the next level's trim)
  int32_t nc;          // coefficients
  int32_t mode;        // normalized boundary mode of the output length
  int32_t P;           // its period
  int32_t full;        // computed over the whole row
  int32_t d_base;      // element offset of the level's d staging
  int32_t cap[kTileSegs];  // stored elements (unpadded, multiple of 4) of each segment slot
  int32_t slot[kTileSegs]; // padded element offset of each slot within its region / buffer
  const void* d;       // (rows, nc) details, or null for zeros
};

template <typename A, int LM>
struct TileParams {
  int64_t rows;
  const void* a;       // coarsest approximation (rows, a_stride)
  int64_t a_stride;
  void* y;             // (rows, lv[0].n_out)
  int32_t J, off, T, W, tiles, ML;
  int32_t run_tiles;    // tiles per row this launch runs: k < t_split is tile k, the others
  int32_t t_split;      // tile k + t_skip (tiles [t_split, t_split + t_skip) run elsewhere)
  int32_t t_skip;
  int32_t abuf_len[2]; // padded elements of the approximation buffers of even / odd levels
  int32_t d_len;       // padded elements of the d staging area
  int32_t origin_res;  // residue mod 4 of every segment origin
  alignas(16) A hp[2 * (LM + 1) * 2];  // (h0[m], h0[m-1]) then (h1[m], h1[m-1]), m = 0..LM
  A h0[LM], h1[LM];
  TileLevel lv[kMaxLevels];
};

struct TileGeo {              // coefficient segments of one level (a and d share them)
  int32_t start[kTileSegs];   // first coefficient
  int32_t len[kTileSegs];     // coefficients (0: unused)
  int32_t origin[kTileSegs];  // coefficient stored at padded index 0
};

// Everything one level of a tile needs, precomputed by the plan (one shared-memory record per
// level, so that a level starts with independent loads rather than a chain of dependent ones).
struct LevelInfo {
  int32_t n_out, nc, mode, P;
  int32_t nleft, nright, edge, d_base;   // edge: the tile has outputs onto which exterior
                                          // positions fold
  int32_t ext_slot[2], ext_org[2], ext_len[2];  // segments read by the left / right exterior
  int32_t js[kTileSegs], je[kTileSegs];          // output ranges
  int32_t src_slot[kTileSegs], src_org[kTileSegs];  // coefficient segment feeding each range
  int32_t dst_slot[kTileSegs], dst_org[kTileSegs];  // where level i-1 keeps each range
  int32_t zl_end[kTileSegs];                    // margin cells to zero: [0, zl_end) and
  int32_t zr_beg[kTileSegs], zr_end[kTileSegs]; // [zr_beg, zr_end) of each output segment
                                                // (all of its storage outside the outputs)
};

// ------------------------------------------------------------------------------ planning

// Output range p in [ms, me) of a level needs coefficients [lo, hi) (clipped to [0, nc)).
// (>> 1 is floor division by 2 for the signed 32-bit values involved.)
__host__ __device__ __forceinline__ void cone(int ms, int me, int off, int LM, int nc, int& lo,
                                              int& hi) {
  lo = (ms - off + 1) >> 1;
  hi = ((me + LM - 2 - off) >> 1) + 1;
  lo = lo < 0 ? 0 : lo;
  hi = hi > nc ? nc : hi;
  if (hi < lo) hi = lo;
}

// Segment geometry of every level for tile t, computed by warp 0 (lane i = level i; results
// in shared memory).  Every lane runs the short cone recursion over the levels (uniform
// parameter loads), keeps its own level's main range and writes its level's geometry; the
// finest level near a row end comes from a ballot.
template <typename A, int LM>
__device__ void plan_tile(const TileParams<A, LM>& p, int t, TileGeo* geo, LevelInfo* info) {
  const int J = p.J;
  const int lane = threadIdx.x & 31;
  int my_nc = 0, my_full = 0, my_nout = 0, my_mode = 0, my_P = 0, my_dbase = 0;
  int my_slot[kTileSegs] = {0, 0, 0};
  int f_nc = 0, f_slot[kTileSegs] = {0, 0, 0}, f_cap[kTileSegs] = {0, 0, 0};  // level lane-1
  int ms = t * p.T;
  int me = min(p.lv[0].n_out, ms + p.T);
  int my_ms = 0, my_me = 0;
  bool my_edge = false;
  for (int i = 0; i < J; ++i) {
    // same address in every lane: broadcast constant loads
    const TileLevel& L = p.lv[i];
    const int n_out = L.n_out;
    const int nc = L.nc;
    if (lane == i) {
      my_nc = nc;
      my_full = L.full;
      my_nout = n_out;
      my_mode = L.mode;
      my_P = L.P;
      my_dbase = L.d_base;
#pragma unroll
      for (int s = 0; s < kTileSegs; ++s) my_slot[s] = L.slot[s];
      my_ms = ms;
      my_me = me;
      my_edge = ms < LM || me > n_out - LM;
    }
    if (lane == i + 1) {
      f_nc = nc;
#pragma unroll
      for (int s = 0; s < kTileSegs; ++s) {
        f_slot[s] = L.slot[s];
        f_cap[s] = L.cap[s];
      }
    }
    int lo, hi;
    cone(ms, me, p.off, LM, nc, lo, hi);
    ms = lo;
    me = hi;
  }
  const unsigned edges = __ballot_sync(0xffffffffu, lane < J && my_edge);
  const int first_edge = edges ? __ffs(edges) - 1 : J;
  int st[kTileSegs] = {0, 0, 0}, ln[kTileSegs] = {0, 0, 0}, org[kTileSegs];
  if (lane < J) {
    if (my_full) {
      ln[0] = my_nc;
    } else {
      int lo, hi;
      cone(my_ms, my_me, p.off, LM, my_nc, lo, hi);
      const bool win = lane >= first_edge;
      ln[0] = win ? min(p.W, my_nc) : 0;
      st[1] = lo;
      ln[1] = hi - lo;
      st[2] = max(0, my_nc - p.W);
      ln[2] = win ? my_nc - st[2] : 0;
    }
  }
#pragma unroll
  for (int s = 0; s < kTileSegs; ++s) {
    // origin: at least ML below the segment start, with the launch-wide residue mod 4
    const int lo = st[s] - p.ML;
    org[s] = lo - ((lo - p.origin_res) & 3);
  }
  if (lane < J) {
    TileGeo& G = geo[lane];
#pragma unroll
    for (int s = 0; s < kTileSegs; ++s) {
      G.start[s] = st[s];
      G.len[s] = ln[s];
      G.origin[s] = org[s];
    }
  }
  // the output segments of level i are the coefficient segments of level i-1
  int ps[kTileSegs], pl[kTileSegs], porg[kTileSegs];
#pragma unroll
  for (int s = 0; s < kTileSegs; ++s) {
    ps[s] = __shfl_up_sync(0xffffffffu, st[s], 1);
    pl[s] = __shfl_up_sync(0xffffffffu, ln[s], 1);
    porg[s] = __shfl_up_sync(0xffffffffu, org[s], 1);
  }
  if (lane < J) {
    LevelInfo& I = info[lane];
    I.n_out = my_nout;
    I.nc = my_nc;
    I.mode = my_mode;
    I.P = my_P;
    I.d_base = my_dbase;
    const int pmin = p.off - (LM - 1);
    const int pmax = 2 * (my_nc - 1) + p.off;
    I.nleft = max(0, min(-1, pmax) - pmin + 1);
    I.nright = max(0, pmax - max(my_nout, pmin) + 1);
    const bool folds = my_mode != FDWT_MODE_ZERO && I.nleft + I.nright > 0;
    const int rs = my_full ? 0 : 2;
    I.ext_slot[0] = my_slot[0];
    I.ext_org[0] = org[0];
    I.ext_len[0] = ln[0];
    I.ext_slot[1] = my_slot[rs];
    I.ext_org[1] = org[rs];
    I.ext_len[1] = ln[rs];
    bool edge = false;
#pragma unroll
    for (int s = 0; s < kTileSegs; ++s) {
      int js, je;
      if (lane == 0) {  // y: the main range only, fed by the main (or full) segment
        const bool mine = my_full ? s == 0 : s == 1;
        js = mine ? my_ms : 0;
        je = mine ? my_me : 0;
      } else {
        js = ps[s];
        je = ps[s] + pl[s];
      }
      I.js[s] = js;
      I.je[s] = je;
      edge |= je > js && (js < LM || je > my_nout - LM);
      const int ss = my_full ? 0 : s;
      I.src_slot[s] = my_slot[ss];
      I.src_org[s] = org[ss];
      I.dst_slot[s] = f_slot[s];
      I.dst_org[s] = porg[s];
      // every margin cell of the output segment is zeroed (see the kernel)
      const int s0 = ps[s] - porg[s];
      const bool live = lane > 0 && pl[s] > 0;
      I.zl_end[s] = live ? s0 : 0;
      I.zr_beg[s] = s0 + pl[s];
      I.zr_end[s] = live ? f_cap[s] : 0;
    }
    I.edge = edge && folds;
  }
}

// ext_index in 32-bit arithmetic (one wrap unless the level is full).
__device__ __forceinline__ int ext32(int p, int n, int mode, int P) {
  if (p >= 0 && p < n) return p;
  if (mode == FDWT_MODE_ZERO) return -1;
  int q = p < 0 ? p + P : (p >= P ? p - P : p);
  if (q < 0 || q >= P) {
    q = p % P;
    q = q < 0 ? q + P : q;
  }
  switch (mode) {
    case FDWT_MODE_PERIODIC: return q;
    case FDWT_MODE_SYMMETRIC: return q < n ? q : P - 1 - q;
    case FDWT_MODE_REFLECT: return q < n ? q : P - q;
    default: return q < n - 1 ? q : n - 1;
  }
}

// Slot of output q in the edge-zone table: [0, LM) for the left zone, LM + offset for the
// right zone [n - LM, n) (the left zone wins where they overlap); -1 elsewhere.
__device__ __forceinline__ int zone_index(int q, int n, int LM) {
  if (q < 0 || q >= n) return -1;
  if (q < LM) return q;
  if (q >= n - LM) return LM + q - (n - LM);
  return -1;
}

// ------------------------------------------------------------------------------ kernel

template <typename A>
__device__ __forceinline__ void cp_async_zfill(A* smem_dst, const A* gsrc, bool valid) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  const int src_bytes = valid ? static_cast<int>(sizeof(A)) : 0;
  if (sizeof(A) == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;\n" ::"r"(s), "l"(gsrc),
                 "r"(src_bytes) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;\n" ::"r"(s), "l"(gsrc),
                 "r"(src_bytes) : "memory");
}

// Stage segment storage [origin, origin + cap) of a global row (zero outside [0, nc) or when
// the row pointer is null); the 32 lanes of a warp share the segment.
template <typename T, typename A>
__device__ __forceinline__ void stage_segment(A* dst, const T* row, int origin, int cap, int nc,
                                              int lane) {
  if (row == nullptr) {
    for (int i = lane; i < cap; i += 32) dst[sidx<TPS>(i)] = A(0);
    return;
  }
  // groups of 4 stored elements are contiguous in the padded layout (cap is a multiple of 4)
  for (int g = lane; 4 * g < cap; g += 32) {
    const int o = origin + 4 * g;
    A* d = dst + 5 * g;
    if (o >= 0 && o + 4 <= nc) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if constexpr (std::is_same<T, A>::value) cp_async_zfill<A>(d + k, row + o + k, true);
        else d[k] = to_acc<T>(row[o + k]);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const bool valid = o + k >= 0 && o + k < nc;
        if constexpr (std::is_same<T, A>::value)
          cp_async_zfill<A>(d + k, valid ? row + o + k : row, valid);
        else d[k] = valid ? to_acc<T>(row[o + k]) : A(0);
      }
    }
  }
}

// z at one extended position p (any p), straight from a coefficient segment.
template <typename A, int LM>
__device__ __forceinline__ A z_at(const TileParams<A, LM>& p, int pos, const A* abase,
                                  const A* dbase, int origin, int nc) {
  A z = A(0);
#pragma unroll
  for (int j = 0; j < LM; ++j) {
    const int u = pos + j - p.off;
    if ((u & 1) == 0) {
      const int o = u >> 1;
      if (o >= 0 && o < nc) {
        const int q = sidx<TPS>(o - origin);
        z = fma(p.h0[j], abase[q], z);
        z = fma(p.h1[j], dbase[q], z);
      }
    }
  }
  return z;
}

// Packed pairs: fp32 pairs in one 64-bit register (fma.rn.f32x2), fp64 as two doubles.
template <typename A>
struct Pair;
template <>
struct Pair<float> {
  unsigned long long v;
  __device__ __forceinline__ void zero() { v = 0ull; }
  __device__ __forceinline__ void dup(float x) { v = pair(x, x); }
  __device__ __forceinline__ void load(const float* h) {
    v = *reinterpret_cast<const unsigned long long*>(h);
  }
  __device__ __forceinline__ void fma(const Pair& h, const Pair& x) { ffma2(v, h.v, x.v); }
  __device__ __forceinline__ float even() const { return lo32(v); }
  __device__ __forceinline__ float odd() const { return hi32(v); }
};
template <>
struct Pair<double> {
  double e, o;
  __device__ __forceinline__ void zero() { e = 0.0; o = 0.0; }
  __device__ __forceinline__ void dup(double x) { e = x; o = x; }
  __device__ __forceinline__ void load(const double* h) { e = h[0]; o = h[1]; }
  __device__ __forceinline__ void fma(const Pair& h, const Pair& x) {
    e = ::fma(h.e, x.e, e);
    o = ::fma(h.o, x.o, o);
  }
  __device__ __forceinline__ double even() const { return e; }
  __device__ __forceinline__ double odd() const { return o; }
};

// Outputs [p0, p0 + 8) from the window of coefficients starting at o0 = (p0 - off - C0) / 2:
// pair q (outputs p0 + 2q, p0 + 2q + 1) takes coefficient o0 + q + v through the packed taps
// hp[2v - C0] (v = 0..LM/2).  The window is loaded (and duplicated into pairs) once; each tap
// pair is loaded once and feeds the four output pairs.
template <typename A, int LM, int C0>
__device__ __forceinline__ void tile_item(const TileParams<A, LM>& p, const A* aw, const A* dw,
                                          A (&z)[2 * TQ]) {
  constexpr int NV = LM / 2 + 1;
  constexpr int NWIN = TQ + NV - 1;
  Pair<A> xa[NWIN], xd[NWIN];
#pragma unroll
  for (int u = 0; u < NWIN; ++u) {
    xa[u].dup(aw[u + (u >> TPS)]);
    xd[u].dup(dw[u + (u >> TPS)]);
  }
  Pair<A> acc[TQ];
#pragma unroll
  for (int q = 0; q < TQ; ++q) acc[q].zero();
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int m = 2 * v - C0;
    if (m < 0 || m > LM) continue;  // resolved at compile time
    Pair<A> ha, hd;
    ha.load(&p.hp[2 * m]);
    hd.load(&p.hp[2 * (LM + 1) + 2 * m]);
#pragma unroll
    for (int q = 0; q < TQ; ++q) {
      acc[q].fma(ha, xa[q + v]);
      acc[q].fma(hd, xd[q + v]);
    }
  }
#pragma unroll
  for (int q = 0; q < TQ; ++q) {
    z[2 * q] = acc[q].even();
    z[2 * q + 1] = acc[q].odd();
  }
}

template <typename T, int LM, int C0>
__global__ void __launch_bounds__(TNT)
dwt_syn_tile_kernel(const __grid_constant__ TileParams<typename AccOf<T>::type, LM> p) {
  using A = typename AccOf<T>::type;
  extern __shared__ __align__(16) unsigned char smem[];
  A* dreg = reinterpret_cast<A*>(smem);
  A* abufs[2] = {dreg + p.d_len, dreg + p.d_len + p.abuf_len[0]};  // a_i lives in abufs[i & 1]
  __shared__ TileGeo geo[kMaxLevels];
  __shared__ LevelInfo info[kMaxLevels];
  __shared__ A zl[2 * LM + 8], zr[2 * LM + 8];
  __shared__ A zadd[2 * LM];  // folded exterior values per edge-zone output (see zone_index)

  const int64_t row = blockIdx.x / p.run_tiles;
  const int tk = static_cast<int>(blockIdx.x % p.run_tiles);
  const int t = tk < p.t_split ? tk : tk + p.t_skip;
  const int J = p.J;
  if (threadIdx.x < 32) plan_tile<A, LM>(p, t, geo, info);
  __syncthreads();

  // stage every level's details and the coarsest approximation: one warp per segment
  {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int k = warp; k < 3 * (J + 1); k += TNT / 32) {
      const int i = k / 3, s = k % 3;
      const bool approx = i == J;
      const int li = approx ? J - 1 : i;
      if (geo[li].len[s] == 0) continue;
      const TileLevel& L = p.lv[li];
      const T* row_ptr;
      A* dst;
      if (approx) {
        row_ptr = static_cast<const T*>(p.a) + row * p.a_stride;
        dst = abufs[li & 1] + L.slot[s];
      } else {
        row_ptr = L.d ? static_cast<const T*>(L.d) + row * L.nc : nullptr;
        dst = dreg + L.d_base + L.slot[s];
      }
      stage_segment<T, A>(dst, row_ptr, geo[li].origin[s], L.cap[s], L.nc, lane);
    }
  }
  cp_async_commit();
  cp_async_wait<0>();
  __syncthreads();

  // padded offsets of the 8 outputs of an item relative to its first (items start at the
  // same residue mod 4 in every output segment)
  int soff[2 * TQ];
  {
    const int r = (8 - p.origin_res) & 3;
#pragma unroll
    for (int k = 0; k < 2 * TQ; ++k) soff[k] = k + ((r + k) >> TPS);
  }
  T* yrow = static_cast<T*>(p.y) + row * p.lv[0].n_out;
  const int pmin = p.off - (LM - 1);
  for (int i = J - 1; i >= 0; --i) {
    const LevelInfo& I = info[i];
    const A* acur = abufs[i & 1];
    A* anext = abufs[(i + 1) & 1];
    const A* dcur = dreg + I.d_base;
    const int n_out = I.n_out, nc = I.nc;
    const int nleft = I.nleft, nright = I.nright;
    const bool edge = I.edge != 0;
    if (edge) {
      // exterior positions that fold back into the row
      for (int k = threadIdx.x; k < nleft + nright; k += TNT) {
        const int side = k < nleft ? 0 : 1;
        const int pos = side == 0 ? pmin + k : max(n_out, pmin) + (k - nleft);
        const A z = I.ext_len[side] > 0
                        ? z_at<A, LM>(p, pos, acur + I.ext_slot[side], dcur + I.ext_slot[side],
                                      I.ext_org[side], nc)
                        : A(0);
        if (side == 0) zl[k] = z;
        else zr[k - nleft] = z;
      }
      for (int k = threadIdx.x; k < 2 * LM; k += TNT) zadd[k] = A(0);
    }
    // in the next level's buffer, every margin cell around the segments this level writes is
    // zeroed: cells that stand for coefficients outside [0, nc) must read as zero, and the
    // others are read through the zero taps (h[-1], h[LM]) of output pairs with one kept and one
    // discarded output, so they must hold a finite value (0 * inf or 0 * nan left in shared
    // memory by an earlier kernel would be nan); they are disjoint from the cells this level's
    // items write
#pragma unroll
    for (int s = 0; s < kTileSegs; ++s) {
      A* b = anext + I.dst_slot[s];
      for (int k = threadIdx.x; k < I.zl_end[s]; k += TNT) b[sidx<TPS>(k)] = A(0);
      for (int k = I.zr_beg[s] + threadIdx.x; k < I.zr_end[s]; k += TNT) b[sidx<TPS>(k)] = A(0);
    }
    if (edge) {
      __syncthreads();
      // one thread sums the exterior values onto their targets, in a fixed order
      if (threadIdx.x == 0) {
        for (int e = 0; e < nleft + nright; ++e) {
          const int pe = e < nleft ? pmin + e : max(n_out, pmin) + (e - nleft);
          const int q = ext32(pe, n_out, I.mode, I.P);
          const int zi = zone_index(q, n_out, LM);
          if (zi >= 0) zadd[zi] += e < nleft ? zl[e] : zr[e - nleft];
        }
      }
      __syncthreads();
    }

#pragma unroll 1
    for (int s = 0; s < kTileSegs; ++s) {
      const int js = I.js[s], je = I.je[s];
      if (je <= js) continue;
      const A* ab = acur + I.src_slot[s];
      const A* db = dcur + I.src_slot[s];
      const int origin = I.src_org[s];
      const int i0 = js >> 3, i1 = (je + 7) >> 3;
      A* dst = anext + I.dst_slot[s];  // level i > 0: the next level's coefficients
      const int dorigin = I.dst_org[s];
      for (int it = i0 + static_cast<int>(threadIdx.x); it < i1; it += TNT) {
        const int p0 = it * 8;
        const int o0 = (p0 - p.off - C0) >> 1;  // exact: p0 - off - C0 is even
        const int w = sidx<TPS>(o0 - origin);
        A z[2 * TQ];
        tile_item<A, LM, C0>(p, ab + w, db + w, z);
        if (edge && (p0 < LM || p0 + 8 > n_out - LM)) {
#pragma unroll
          for (int k = 0; k < 2 * TQ; ++k) {
            const int zi = zone_index(p0 + k, n_out, LM);
            if (zi >= 0) z[k] += zadd[zi];
          }
        }
        if (i > 0) {
          const int b = p0 - dorigin;  // b = -origin_res (mod 4) for every item
          A* d0 = dst + sidx<TPS>(b);
          if (p0 >= js && p0 + 8 <= je) {
#pragma unroll
            for (int k = 0; k < 2 * TQ; ++k) d0[soff[k]] = z[k];
          } else {
#pragma unroll
            for (int k = 0; k < 2 * TQ; ++k) {
              const int q = p0 + k;
              if (q >= js && q < je) d0[soff[k]] = z[k];
            }
          }
        } else {
          T* yd = yrow + p0;
          const bool whole = p0 >= js && p0 + 8 <= je;
          if (whole && (reinterpret_cast<uintptr_t>(yd) & 15) == 0) {
            T v[2 * TQ];
#pragma unroll
            for (int k = 0; k < 2 * TQ; ++k) v[k] = from_acc<T>(z[k]);
            store_vec<T, 2 * TQ>(yd, v);
          } else {
#pragma unroll
            for (int k = 0; k < 2 * TQ; ++k) {
              const int q = p0 + k;
              if (q >= js && q < je) yd[k] = from_acc<T>(z[k]);
            }
          }
        }
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------ host

// Plans and launches the tile synthesis of the levels lv (processing order, coarsest first);
// FDWT_ERR_UNSUPPORTED when it does not apply (the caller then uses the cluster kernel).
// Tiles [skip_lo, skip_hi) of every row are left out (another kernel computes them).
template <typename T, int LM>
int run_syn_tile_launch(int64_t rows, const void* a, const std::vector<Level>& lv, void* y,
                        const double* h0, const double* h1, int L, int off, cudaStream_t stream,
                        bool dry_run, int skip_lo = 0, int skip_hi = 0) {
  using A = typename AccOf<T>::type;
  const int J = static_cast<int>(lv.size());
  if (J < 1 || J > kMaxLevels) return FDWT_ERR_UNSUPPORTED;
  TileParams<A, LM> p{};
  p.rows = rows;
  p.a = a;
  p.a_stride = lv[0].a_len;
  p.y = y;
  p.J = J;
  p.off = off;
  p.W = ((2 * LM + 8) + 3) / 4 * 4;
  p.ML = ((LM / 2 + 12) + 3) / 4 * 4;
  const int MR = ((TQ + LM / 2 + 12) + 3) / 4 * 4;
  p.origin_res = static_cast<int>(((floor_div(-off - (off & 1), 2)) % 4 + 4) % 4);
  const int64_t n0 = lv[J - 1].n_in;
  for (const auto& l : lv)
    if (l.n_in > 0x3fffffffLL || l.a_len > 0x3fffffffLL) return FDWT_ERR_UNSUPPORTED;
  int T_tile = tile_outputs<A>();
  const int F0 = 4 * LM + 2 * p.W + 64;
  if (n0 <= T_tile + 2 * p.W) T_tile = static_cast<int>(n0);
  p.T = T_tile;
  p.tiles = static_cast<int>(cdiv(n0, T_tile));
  if (skip_hi > skip_lo && (skip_lo < 0 || skip_hi > p.tiles)) return FDWT_ERR_INVALID;
  p.t_split = skip_hi > skip_lo ? skip_lo : p.tiles;
  p.t_skip = skip_hi > skip_lo ? skip_hi - skip_lo : 0;
  p.run_tiles = p.tiles - p.t_skip;
  // bounds of the main ranges, fine to coarse, and the full / partial split
  std::vector<int64_t> mbound(J), cbound(J);
  int64_t mb = T_tile;
  for (int i = 0; i < J; ++i) {
    mbound[i] = mb;
    cbound[i] = (mb + LM) / 2 + 2;
    mb = cbound[i];
  }
  // level i (0 = finest) corresponds to lv[J - 1 - i]
  int first_full = J;
  for (int i = J - 1; i >= 0; --i) {
    const Level& l = lv[J - 1 - i];
    const bool full = p.tiles == 1 || l.n_in <= std::max<int64_t>(F0, mbound[i] + 2 * p.W + LM);
    if (!full) break;
    first_full = i;
  }
  int d_len = 0, abuf[2] = {0, 0};
  for (int i = 0; i < J; ++i) {
    const Level& l = lv[J - 1 - i];
    TileLevel& t = p.lv[i];
    t.n_out = static_cast<int>(l.n_in);
    t.nc = static_cast<int>(l.n_coef);
    t.mode = l.mode;
    t.P = static_cast<int>(l.P);
    t.full = i >= first_full;
    t.d = l.detail;
    int caps[kTileSegs];
    if (t.full) {
      caps[0] = t.nc + p.ML + MR + 8;
      caps[1] = caps[2] = 0;
    } else {
      caps[0] = caps[2] = p.W + p.ML + MR + 8;
      caps[1] = static_cast<int>(cbound[i]) + p.ML + MR + 8;
    }
    int off_e = 0;
    for (int s = 0; s < kTileSegs; ++s) {
      caps[s] = (caps[s] + 3) / 4 * 4;  // staging writes whole groups of 4
      t.cap[s] = caps[s];
      t.slot[s] = off_e;
      off_e += static_cast<int>((padded_len<TPS>(caps[s]) + 3) / 4 * 4);
    }
    t.d_base = d_len;
    d_len += off_e;
    abuf[i & 1] = std::max(abuf[i & 1], off_e);
  }
  p.d_len = d_len;
  p.abuf_len[0] = abuf[0];
  p.abuf_len[1] = abuf[1];
  for (int j = 0; j < LM; ++j) {
    p.h0[j] = (j < L && !dry_run) ? static_cast<A>(h0[j]) : A(0);
    p.h1[j] = (j < L && !dry_run) ? static_cast<A>(h1[j]) : A(0);
  }
  for (int m = 0; m <= LM; ++m) {
    p.hp[2 * m] = m < LM ? p.h0[m] : A(0);
    p.hp[2 * m + 1] = m >= 1 ? p.h0[m - 1] : A(0);
    p.hp[2 * (LM + 1) + 2 * m] = m < LM ? p.h1[m] : A(0);
    p.hp[2 * (LM + 1) + 2 * m + 1] = m >= 1 ? p.h1[m - 1] : A(0);
  }
  const size_t smem = static_cast<size_t>(d_len + abuf[0] + abuf[1]) * sizeof(A) + 16;
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 2048 -
                        sizeof(TileGeo) * kMaxLevels - sizeof(LevelInfo) * kMaxLevels -
                        2 * (2 * LM + 8) * sizeof(A) - 2 * LM * sizeof(A);
  if (smem > budget) return FDWT_ERR_UNSUPPORTED;
  if (rows * p.tiles > 0x7fffffffLL) return FDWT_ERR_UNSUPPORTED;
  if (p.run_tiles == 0) return FDWT_OK;
  if (dry_run || rows == 0) return FDWT_OK;
  const bool c0 = (off & 1) != 0;
  auto kern = c0 ? dwt_syn_tile_kernel<T, LM, 1> : dwt_syn_tile_kernel<T, LM, 0>;
  int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
  if (st != FDWT_OK) return st;
  if ((st = pre_launch(stream)) != FDWT_OK) return st;
  kern<<<static_cast<unsigned>(rows * p.run_tiles), TNT, smem, stream>>>(p);
  return launch_status();
}

}  // namespace dwtk
}  // namespace fdwt

namespace fdwt {
namespace dwtk {

// Every tile recomputes the cone of every level, so a deep transform of a long row pays the
// per-level cost tiles x levels times, and every level of a tile is a barrier-separated step
// with few warps per SM (the staging of all its levels limits the CTAs per SM).  Deep fp32 /
// fp64 syntheses are therefore split into stages: the coarse levels run first as their own
// (shorter-row, fewer-tile) synthesis that writes its approximation to the workspace, and the
// finer levels run one per stage, reading the approximation of the stage before.  A level that
// the streaming kernel (dwt_stream.cuh) can take whole -- periodization or zero mode, rows of a
// multiple of 16 bytes, at least kStreamMinOut outputs -- runs alone; it then moves its bytes
// near the copy bandwidth, which outweighs the extra write and read of the handed-over
// approximation.  Other levels run alone while their rows are long (one-level tile launches
// were 3-15% faster than two or three levels per launch on B200).  Returns the workspace it
// needs through ws_needed when asked.
constexpr int kSplitLevels = 1;

template <typename T, int LM>
int run_syn_stream(int64_t rows, const void* a, const Level& L0, void* y, const double* h0,
                   const double* h1, int L, int off, cudaStream_t stream);

// One stage: a one-level stage tries the streaming kernel (dwt_stream.cuh) first.
template <typename T, int LM>
int run_syn_stage(int64_t rows, const void* a, const std::vector<Level>& lv, void* y,
                  const double* h0, const double* h1, int L, int off, cudaStream_t stream) {
  if (lv.size() == 1) {
    const int st = run_syn_stream<T, LM>(rows, a, lv[0], y, h0, h1, L, off, stream);
    if (st != FDWT_ERR_UNSUPPORTED) return st;
  }
  return run_syn_tile_launch<T, LM>(rows, a, lv, y, h0, h1, L, off, stream, false);
}

template <typename T, int LM>
int run_syn2_stream(int64_t rows, const void* a2, const Level& Lc, const Level& Lf, void* y,
                    const double* h0, const double* h1, int L, int off, cudaStream_t stream);
template <typename T, int LM>
bool syn2_fuses(int64_t rows, const Level& Lc, const Level& Lf, int off);

template <typename T, int LM>
int run_syn_tiles(int64_t rows, const void* a, const std::vector<Level>& lv, void* y,
                  const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
                  cudaStream_t stream, size_t* ws_needed) {
  using A = typename AccOf<T>::type;
  const int J = static_cast<int>(lv.size());
  const int64_t T_tile = tile_outputs<A>();
  // stages in processing order: the coarse levels [0, c) together (if any), then the finer
  // levels one or two per stage; each stage but the last hands its approximation to the next
  // through the workspace
  std::vector<std::pair<int, int>> fine;  // (first level, levels), finest first
  int c = J;
  while (std::is_same<T, A>::value && c > 0) {
    if (c >= 2 && syn2_fuses<T, LM>(std::max<int64_t>(rows, 1), lv[c - 2], lv[c - 1], off)) {
      fine.emplace_back(c - 2, 2);  // two levels per streaming pass (dwt_stream2.cuh)
      c -= 2;
      continue;
    }
    // a level that streams every tile (dwt_stream.cuh) runs alone down to short rows; the
    // others while their rows are long
    const Level& f = lv[c - 1];
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    const bool streams = stream_fills(f) && LM <= kStreamMaxLM && f.n_in >= kStreamMinOut &&
                         f.n_in % VW == 0 && f.n_coef % VW == 0 && f.a_len % VW == 0;
    const bool alone = streams || (c > kSplitLevels + 1 && f.n_in >= 2 * T_tile);
    if (!alone || c == 1) break;
    fine.emplace_back(c - 1, 1);
    c -= 1;
  }
  std::vector<std::pair<int, int>> stages;
  if (c > 0) stages.emplace_back(0, c);
  for (auto it = fine.rbegin(); it != fine.rend(); ++it) stages.push_back(*it);
  const int ns = static_cast<int>(stages.size());
  if (ns == 1) {
    if (ws_needed == nullptr && rows > 0) {
      if (c == 0 && J == 2) {  // the whole synthesis is one fused pair
        const int st = run_syn2_stream<T, LM>(rows, a, lv[0], lv[1], y, h0, h1, L, off, stream);
        if (st != FDWT_ERR_UNSUPPORTED) return st;
      }
      return run_syn_stage<T, LM>(rows, a, lv, y, h0, h1, L, off, stream);
    }
    const int st = run_syn_tile_launch<T, LM>(rows, a, lv, y, h0, h1, L, off, stream,
                                              ws_needed != nullptr);
    if (st == FDWT_OK && ws_needed) *ws_needed = 0;
    return st;
  }
  auto stage = [&](int s) {
    return std::vector<Level>(lv.begin() + stages[s].first,
                              lv.begin() + stages[s].first + stages[s].second);
  };
  // stage s (but the last) outputs the n_in samples per row of its finest level; the outputs
  // alternate between two regions, the last-but-one in region 0
  size_t region[2] = {0, 0};
  for (int s = 0; s + 1 < ns; ++s) {
    const int last = stages[s].first + stages[s].second - 1;
    const size_t bytes = (static_cast<size_t>(rows) * lv[last].n_in * sizeof(T) + 255) &
                         ~size_t(255);
    size_t& r = region[(ns - 2 - s) & 1];
    r = std::max(r, bytes);
  }
  for (int s = 0; s < ns; ++s) {  // every stage must be plannable before anything launches
    const int st = run_syn_tile_launch<T, LM>(rows, nullptr, stage(s), nullptr, h0, h1, L, off,
                                              stream, true);
    if (st != FDWT_OK) return st;
  }
  if (ws_needed) {
    *ws_needed = region[0] + region[1];
    return FDWT_OK;
  }
  if (rows == 0) return FDWT_OK;
  if (ws == nullptr || ws_bytes < region[0] + region[1]) return FDWT_ERR_WORKSPACE;
  unsigned char* base[2] = {static_cast<unsigned char*>(ws),
                            static_cast<unsigned char*>(ws) + region[0]};
  const void* src = a;
  for (int s = 0; s < ns; ++s) {
    void* dst = s + 1 < ns ? static_cast<void*>(base[(ns - 2 - s) & 1]) : y;
    const auto lvs = stage(s);
    int st = FDWT_ERR_UNSUPPORTED;
    const bool pair = stages[s].second == 2 && (s > 0 || c == 0);  // a fused pair, not the coarse part
    if (pair) st = run_syn2_stream<T, LM>(rows, src, lvs[0], lvs[1], dst, h0, h1, L, off, stream);
    if (st == FDWT_ERR_UNSUPPORTED)
      st = run_syn_stage<T, LM>(rows, src, lvs, dst, h0, h1, L, off, stream);
    if (st != FDWT_OK) return st;
    src = dst;
  }
  return FDWT_OK;
}

}  // namespace dwtk
}  // namespace fdwt
