// Two analysis levels per streaming pass, for sm_100a.  Included by dwt_impl.cuh after
// dwt_stream.cuh, whose ring, copies, bounded waits and window items it uses.
//
// Levels k and k+1 of a multilevel analysis in one pass over x: a tile owns T2 outputs of level
// k+1 (cA2, cD2) and the 2 T2 level-k details under them (cD1).  Level k+1 reads the level-k
// approximation cA1 over 2 T2 + LM - 2 positions (its tile plus a halo of LM - 2): the CTA
// computes those from its x slot into a shared buffer (the halo is recomputed by both tiles
// that need it, about 1% more level-k arithmetic), stores the details it owns, and after a
// barrier computes level k+1 from the buffer.  cA1 never touches HBM: the pass reads x once
// and writes cD1, cA2 and cD2 once -- a third less traffic than two one-level passes.
//
// Level k+1 extends cA1 past its ends with its own boundary mode:
// - periodization (x of an even length, one period): cA1 is itself periodic with period nc1,
//   and the positions outside [0, nc1) computed from the periodically continued x are exactly
//   its continuation;
// - zero: those positions are set to 0;
// - symmetric, reflect: they are copied from their mirror images, which lie in the same tile
//   (the host checks the tiles at both row ends);
// - periodic (period nc1 != n / 2) needs the other row end and is not fused.
//
// Items are those of the one-level kernel (V outputs, windows 48 bytes apart).  Level-k items
// start V kh outputs before the tile's first owned detail, so that the owned details are whole
// items, and the buffer starts B cells in, so that every level-(k+1) window has the same
// 16-byte shift R as the level-k windows.
#pragma once

namespace fdwt {
namespace dwtk {

// Ring slots of the fused analysis: fp32 needs three tiles in flight; fp64 tiles are as large
// in bytes and run faster at three CTAs per SM with two slots (measured on B200).
template <typename A>
constexpr int ana2_stages() { return sizeof(A) == 8 ? 2 : 3; }

template <typename A, int LM>
struct Ana2Params {
  const A* x;        // (rows, xs)
  A* d1;             // (rows, nc1) level-k details
  A* a2;             // (rows, as) level-(k+1) approximation
  A* d2;             // (rows, nc2) level-(k+1) details
  int* err;          // device error word
  uint32_t dbg_tx;   // test hook: extra expected bytes of global tile 0's copy
  long long tries;   // poll limit of the main mbarrier waits
  int64_t ntile;     // rows * tiles
  int64_t P;         // period of level k's boundary mode on n
  int64_t P2;        // period of level k+1's boundary mode on n1
  int32_t n, nc1, n1, nc2, a_len2, off, mode, mode2, tiles;
  int32_t xs, as;    // row strides of x and of cA2 (xs a multiple of 16 bytes)
  int32_t n_al;      // n rounded down to 16 bytes: the bulk copies end there
  int32_t span;      // x elements per ring slot
  int32_t T2;        // level-(k+1) outputs per tile (V q, with K1 = kh + 2q + kr <= 2 SNT)
  int32_t K1, kh;    // level-k items per tile, of which kh before the first owned detail
  int32_t B, S2;     // buffer offset of the first level-k output; level-(k+1) window base
  int32_t abuf;      // buffer elements
  int32_t x_hi;      // x positions past the row end up to x_hi are gathered
  alignas(16) A taps[2 * LM];  // (h0[j], h1[j]) interleaved
};

template <typename A, int LM, int R>
__device__ void ana2_tiles(const Ana2Params<A, LM>& p, A* ring, A* abuf, uint64_t* bar) {
  constexpr int V = ana_stream_v<A>();
  const int T2 = p.T2;
  const int T1 = 2 * T2;
  const int tid = threadIdx.x;
  const int64_t G = gridDim.x;
  const int span = p.span, n = p.n;
  const int pmin = p.off - (LM - 1);
  auto slot = [&](int s) { return ring + static_cast<size_t>(s) * span; };
  auto first_o1 = [&](int t) { return t * T1 - V * p.kh; };
  auto slot_lo = [&](int t) { return 2 * first_o1(t) + pmin - R; };  // a multiple of 16 bytes
  // all threads: extended x positions of tile g outside [0, n), gathered with cp.async
  auto ext_fill = [&](int64_t g, int s) {
    const int64_t row = g / p.tiles;
    const int xlo = slot_lo(static_cast<int>(g % p.tiles));
    const A* xr = p.x + row * p.xs;
    A* sl = slot(s);
    auto one = [&](int q) {
      const int64_t e = ext_index(q, n, p.mode, p.P);
      if (e < 0) sl[q - xlo] = A(0);
      else cp_async(sl + (q - xlo), xr + e, sizeof(A));
    };
    const int l1 = min(xlo + span, 0), r1 = min(xlo + span, p.x_hi);
    for (int q = xlo + tid; q < l1; q += SNT) one(q);
    for (int q = max(xlo, p.n_al) + tid; q < r1; q += SNT) one(q);
    cp_async_commit();
  };
  auto issue = [&](int64_t g, int s) {
    const int64_t row = g / p.tiles;
    const int xlo = slot_lo(static_cast<int>(g % p.tiles));
    const int lo = max(xlo, 0), hi = min(xlo + span, p.n_al);
    const unsigned bytes = static_cast<unsigned>(max(hi - lo, 0)) * sizeof(A);
    mbar_expect_tx(&bar[s], bytes + (g == 0 ? p.dbg_tx : 0u));
    if (bytes) bulk_g2s(slot(s) + (lo - xlo), p.x + row * p.xs + lo, bytes, &bar[s]);
  };
#pragma unroll 1
  for (int s = 0; s < ana2_stages<A>(); ++s) {
    const int64_t g = blockIdx.x + s * G;
    if (g < p.ntile) ext_fill(g, s);
    else cp_async_commit();
  }
  cp_async_wait<ana2_stages<A>() - 1>();
  __syncthreads();
  if (tid == 0) {
#pragma unroll 1
    for (int s = 0; s < ana2_stages<A>(); ++s) {
      const int64_t g = blockIdx.x + s * G;
      if (g < p.ntile) issue(g, s);
    }
  }
  int k = 0;
#pragma unroll 1
  for (int64_t g = blockIdx.x; g < p.ntile; g += G, ++k) {
    const int s = k % ana2_stages<A>();
    const unsigned par = static_cast<unsigned>(k / ana2_stages<A>()) & 1u;
    const bool ok = mbar_wait_bounded(&bar[s], par, p.tries);
    const int64_t row = g / p.tiles;
    const int t = static_cast<int>(g % p.tiles);
    const int o1_0 = first_o1(t);
    if (ok) {  // level k: cA1 into the buffer, the owned cD1 to HBM
      const A* sl = slot(s);
      A* d1row = p.d1 + row * p.nc1;
#pragma unroll 1
      for (int it = tid; it < p.K1; it += SNT) {
        A ra[V], rd[V];
        ana_window_item<A, LM, R>(p.taps, sl + 2 * V * it, ra, rd);
        A* b = abuf + p.B + V * it;
#pragma unroll
        for (int v = 0; v < V; ++v) b[v] = ra[v];
        const int o1 = o1_0 + V * it;
        if (it >= p.kh && it < p.kh + T1 / V && o1 < p.nc1)
          store_run<A, V>(d1row + o1, rd, min(V, p.nc1 - o1));
      }
    }
    __syncthreads();
    // level k+1's extension of cA1 (tiles at the row ends; periodization needs none)
    const int nb = V * p.K1;
    if (p.mode2 != FDWT_MODE_PERIODIZATION && (o1_0 < 0 || o1_0 + nb > p.nc1)) {
      if (ok) {
        const int l_end = min(nb, -o1_0), r_beg = max(0, p.nc1 - o1_0);
        // cells outside [0, nc1) take their image under the boundary map; the images lie in
        // [0, nc1) (or are 0), which this step never writes, so the loops need no ordering
        auto fix = [&](int i) {
          const int64_t q = ext_index(o1_0 + i, p.n1, p.mode2, p.P2);
          return q >= 0 && q < p.nc1 ? abuf[p.B + static_cast<int>(q) - o1_0] : A(0);
        };
        for (int i = tid; i < l_end; i += SNT) abuf[p.B + i] = fix(i);
        for (int i = r_beg + tid; i < nb; i += SNT) abuf[p.B + i] = fix(i);
      }
      __syncthreads();
    }
    if (ok) {  // level k+1 from the buffer
      A* a2row = p.a2 + row * p.as;
      A* d2row = p.d2 + row * p.nc2;
#pragma unroll 1
      for (int m = tid; m < T2 / V; m += SNT) {
        const int o2 = t * T2 + V * m;
        if (o2 >= p.nc2) break;
        A ra[V], rd[V];
        ana_window_item<A, LM, R>(p.taps, abuf + 2 * V * m + p.S2 - R, ra, rd);
        const int cnt = min(V, p.nc2 - o2);
        store_run<A, V>(d2row + o2, rd, cnt);
        store_run<A, V>(a2row + o2, ra, cnt);
      }
      if (t == p.tiles - 1 && tid == 0)
        for (int q = p.nc2; q < p.a_len2; ++q) a2row[q] = A(0);  // transpose of waverec's trim
    }
    cp_async_wait<ana2_stages<A>() - 2>();  // this thread's gathers of tile k + 1
    if (__syncthreads_or(!ok)) {
      cp_async_wait<0>();
      if (tid == 0) {
        atomicExch(p.err, kErrCopyTimeout);
#pragma unroll 1
        for (int j = 0; j < ana2_stages<A>(); ++j) {
          const int64_t gj = g + j * G;
          if (gj >= p.ntile) break;
          const int kj = k + j;
          mbar_wait_bounded(&bar[kj % ana2_stages<A>()],
                            static_cast<unsigned>(kj / ana2_stages<A>()) & 1u,
                            cleanup_tries(p.tries));
        }
      }
      return;
    }
    const int64_t gn = g + ana2_stages<A>() * G;
    if (gn < p.ntile) {
      ext_fill(gn, s);
      if (tid == 0) issue(gn, s);
    } else {
      cp_async_commit();
    }
  }
}

template <typename A, int LM>
__global__ void __launch_bounds__(SNT, 2)
dwt_ana2_stream_kernel(const __grid_constant__ Ana2Params<A, LM> p, int r) {
  extern __shared__ __align__(16) unsigned char ring_smem[];
  __shared__ __align__(8) uint64_t bar[ana2_stages<A>()];
  A* ring = reinterpret_cast<A*>(ring_smem);
  A* abuf = ring + static_cast<size_t>(ana2_stages<A>()) * p.span;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < ana2_stages<A>(); ++s) mbar_init(&bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if constexpr (sizeof(A) == 4) {
    switch (r) {
      case 0: ana2_tiles<A, LM, 0>(p, ring, abuf, bar); break;
      case 1: ana2_tiles<A, LM, 1>(p, ring, abuf, bar); break;
      case 2: ana2_tiles<A, LM, 2>(p, ring, abuf, bar); break;
      default: ana2_tiles<A, LM, 3>(p, ring, abuf, bar); break;
    }
  } else {
    if (r == 0) ana2_tiles<A, LM, 0>(p, ring, abuf, bar);
    else ana2_tiles<A, LM, 1>(p, ring, abuf, bar);
  }
}

// ------------------------------------------------------------------------------ host

// Geometry of a fused pair (levels L1, L2 of one analysis with offset off); ok = false when the
// pair does not fuse.  Shape-only: the input pointer's alignment is the caller's check.
template <typename T, int LM>
struct Ana2Plan {
  bool ok = false;
  int R = 0;
  Ana2Params<typename AccOf<T>::type, LM> p{};
  size_t smem = 0;
};

template <typename T, int LM>
Ana2Plan<T, LM> plan_ana2(int64_t rows, const Level& L1, const Level& L2, int off,
                          int64_t xs) {
  using A = typename AccOf<T>::type;
  Ana2Plan<T, LM> pl;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return pl;
  } else {
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    constexpr int V = ana_stream_v<A>();
    const int64_t n = L1.n_in, nc1 = L1.n_coef, n1 = L2.n_in, nc2 = L2.n_coef;
    if (n < 1024 || xs % VW || xs < n || xs > 0x3fffffffLL || nc2 < 1 || L1.a_len != n1 ||
        L2.a_len > nc2 + 1 || rows <= 0)
      return pl;
    const int mode = L1.mode, mode2 = L2.mode;
    if (mode == FDWT_MODE_PERIODIC || mode2 != mode) return pl;
    if (mode == FDWT_MODE_PERIODIZATION &&
        !(n == 2 * nc1 && n1 == nc1 && nc1 % 2 == 0 && nc2 == nc1 / 2 && L1.P == n &&
          L2.P == n1))
      return pl;
    const int pmin = off - (LM - 1);
    const int R = ((pmin % VW) + VW) % VW;
    constexpr int W = 2 * V + LM - 2;
    const int NL = (R + W + VW - 1) / VW;
    const int kh = (-pmin + V - 1) / V;
    const int kr = (std::max(off - 1, 0) + V - 1) / V;
    // two level-k items per thread: K1 = kh + T1 / V + kr <= 2 SNT; then tiles of equal size
    const int q_max = (2 * SNT - kh - kr) / 2;
    const int64_t n_tiles = cdiv(nc2, static_cast<int64_t>(V) * q_max);
    const int T2 = V * static_cast<int>(cdiv(cdiv(nc2, n_tiles), V));
    const int T1 = 2 * T2;
    const int K1 = kh + T1 / V + kr;
    const int span = 2 * V * K1 - 2 * V + NL * VW;
    const int B = (((R - pmin - V * kh) % VW) + VW) % VW;
    const int S2 = pmin + V * kh + B;
    int abuf = std::max(B + V * K1, 2 * V * (T2 / V - 1) + S2 - R + NL * VW);
    abuf = (abuf + VW - 1) / VW * VW;
    const int64_t tiles = cdiv(nc2, T2);
    const int64_t max_o1 = std::max<int64_t>(2 * (nc2 - 1) + off, nc1 - 1);
    // mirror sources of the extension must lie in the tile (first and last two tiles)
    if (mode == FDWT_MODE_SYMMETRIC || mode == FDWT_MODE_REFLECT) {
      for (int64_t t : {int64_t(0), tiles - 2, tiles - 1}) {
        if (t < 0) continue;
        const int64_t o1_0 = t * T1 - V * kh;
        for (int64_t i = 0; i < V * K1; ++i) {
          const int64_t o1 = o1_0 + i;
          if (o1 >= 0 && o1 < nc1) continue;
          const int64_t q = ext_index(o1, n1, mode2, L2.P);
          if (q >= 0 && q < nc1 && (q - o1_0 < 0 || q - o1_0 >= V * K1)) return pl;
        }
      }
    }
    if (rows * tiles > (1LL << 40)) return pl;
    auto& p = pl.p;
    p.ntile = rows * tiles;
    p.P = L1.P;
    p.P2 = L2.P;
    p.n = static_cast<int>(n);
    p.nc1 = static_cast<int>(nc1);
    p.n1 = static_cast<int>(n1);
    p.nc2 = static_cast<int>(nc2);
    p.a_len2 = static_cast<int>(L2.a_len);
    p.xs = static_cast<int>(xs);
    p.n_al = static_cast<int>(n / VW * VW);
    p.off = off;
    p.mode = mode;
    p.mode2 = mode2;
    p.tiles = static_cast<int>(tiles);
    p.span = span;
    p.T2 = T2;
    p.K1 = K1;
    p.kh = kh;
    p.B = B;
    p.S2 = S2;
    p.abuf = abuf;
    p.x_hi = static_cast<int>(std::min<int64_t>(2 * max_o1 + off + 1, 0x3fffffffLL));
    pl.R = R;
    pl.smem = (static_cast<size_t>(ana2_stages<A>()) * span + abuf) * sizeof(A);
    pl.ok = pl.smem <= static_cast<size_t>(max_smem_optin()) - 2048;
    return pl;
  }
}

// Runs levels L1, L2 of an analysis in one streaming pass: x (rows of L1.n_in samples, xs apart)
// -> details of both levels (L1.detail, L2.detail) and the level-2 approximation a2_out (rows
// of L2.a_len, as apart).  FDWT_ERR_UNSUPPORTED when the pair does not fuse.
template <typename T, int LM>
int run_ana2_stream(int64_t rows, const void* x, const Level& L1, const Level& L2, int64_t xs,
                    void* a2_out, int64_t as, const double* h0, const double* h1, int L, int off,
                    cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return FDWT_ERR_UNSUPPORTED;
  } else {
    Ana2Plan<T, LM> pl = plan_ana2<T, LM>(rows, L1, L2, off, xs);
    if (!pl.ok || as < L2.a_len || as > 0x3fffffffLL || x == nullptr || a2_out == nullptr || L1.detail == nullptr ||
        L2.detail == nullptr || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
      return FDWT_ERR_UNSUPPORTED;
    auto& p = pl.p;
    p.x = static_cast<const A*>(x);
    p.d1 = static_cast<A*>(L1.detail);
    p.a2 = static_cast<A*>(a2_out);
    p.as = static_cast<int>(as);
    p.d2 = static_cast<A*>(L2.detail);
    p.err = device_error_flag();
    if (p.err == nullptr) return FDWT_ERR_CUDA;
    {
      const CopyWaitTest wt = copy_wait_test();
      p.dbg_tx = wt.extra_tx;
      p.tries = wt.tries;
    }
    for (int j = 0; j < LM; ++j) {
      p.taps[2 * j] = j < L ? static_cast<A>(h0[j]) : A(0);
      p.taps[2 * j + 1] = j < L ? static_cast<A>(h1[j]) : A(0);
    }
    auto kern = dwt_ana2_stream_kernel<A, LM>;
    int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (st != FDWT_OK) return st;
    int occ = 0;
    if ((st = occupancy(reinterpret_cast<const void*>(kern), SNT, pl.smem, &occ)) != FDWT_OK) return st;
    if (occ < 1) return FDWT_ERR_UNSUPPORTED;
    const int64_t grid = std::min<int64_t>(p.ntile, static_cast<int64_t>(occ) * sm_count());
    if ((st = pre_launch(stream)) != FDWT_OK) return st;
    kern<<<static_cast<unsigned>(grid), SNT, pl.smem, stream>>>(p, pl.R);
    return launch_status();
  }
}

// ------------------------------------------------------------------------------ synthesis
//
// Levels k+1 and k of a multilevel synthesis in one pass (periodization or zero mode, the two
// that stream every tile): a tile owns T outputs of y (level k).  Their windows read the
// level-k approximation a1 and the details d1 over one slot range [glo, glo + span), exactly
// as the one-level kernel.  a1 there is computed from a slot of a2 and d2 into a shared buffer
// (items of 8 a1 values; the buffer range is recomputed by both tiles that overlap in it), d1
// arrives by bulk copy with the slot, and after a barrier the y items run.  a1 never touches
// HBM.  In zero mode the buffer cells outside [0, nc1) are set to 0 (the coefficients that
// level k reads there are zero); in periodization the values computed from the periodically
// continued a2, d2 are already a1's continuation.  The a1 items start delta - 8 cells before
// glo (delta even, < 2 VW, one per launch), which gives their a2/d2 windows the same 16-byte
// shift R as the y windows.

template <typename A, int LM>
struct Syn2Params {
  const A* a2;       // (rows, a2_stride) level-(k+1) approximation
  const A* d2;       // (rows, nc2)
  const A* d1;       // (rows, nc1)
  A* y;              // (rows, n_out)
  int* err;          // device error word
  uint32_t dbg_tx;   // test hook: extra expected bytes of global tile 0's copy
  long long tries;   // poll limit of the main mbarrier waits
  int64_t a2_stride;
  int64_t ntile;     // rows * tiles
  int32_t nc2, nc1, n_out, off, fill, tiles, T;
  int32_t span;      // d1 (and buffer) cells per tile
  int32_t span2;     // a2 / d2 cells per tile
  int32_t M1, delta; // a1 items per tile and their start (see above)
  int32_t abuf;      // buffer elements
  alignas(16) A hp[2 * (LM + 1) * 2];
};

template <typename A, int LM, int C0, int R>
__device__ void syn2_tiles(const Syn2Params<A, LM>& p, A* ring, A* abuf, uint64_t* bar) {
  const int T = p.T;
  const int tid = threadIdx.x;
  const int64_t G = gridDim.x;
  const int span = p.span, span2 = p.span2;
  const int slot_elems = span + 2 * span2;
  auto slot = [&](int s) { return ring + static_cast<size_t>(s) * slot_elems; };
  auto glo_of = [&](int t) { return ((t * T - p.off - C0) >> 1) - R; };
  auto g2lo_of = [&](int t) { return ((glo_of(t) - p.off - C0 + p.delta - 8) >> 1) - R; };
  // zero mode: slot cells outside [0, nc) of the arrays of tile g (all threads)
  auto zero_fill = [&](int64_t g, int s) {
    if (p.fill != kFillZero) return;
    const int t = static_cast<int>(g % p.tiles);
    const int gl = glo_of(t), g2 = g2lo_of(t);
    A* d1s = slot(s);
    A* a2s = d1s + span;
    A* d2s = a2s + span2;
    for (int i = tid; i < -gl && i < span; i += SNT) d1s[i] = A(0);
    for (int i = max(p.nc1 - gl, 0) + tid; i < span; i += SNT) d1s[i] = A(0);
    for (int i = tid; i < -g2 && i < span2; i += SNT) a2s[i] = d2s[i] = A(0);
    for (int i = max(p.nc2 - g2, 0) + tid; i < span2; i += SNT) a2s[i] = d2s[i] = A(0);
  };
  // one array's cells [lo_el, lo_el + cnt) of a row of length nc into dst: the in-range part by
  // bulk copy, and in periodic mode the continuation past either end from the other end
  auto copy_range = [&](A* dst, const A* row, int lo_el, int cnt, int nc, int s) {
    const int lo = max(lo_el, 0), hi = min(lo_el + cnt, nc);
    unsigned tx = 0;
    if (hi > lo) {
      bulk_g2s(dst + (lo - lo_el), row + lo, (hi - lo) * sizeof(A), &bar[s]);
      tx += (hi - lo) * sizeof(A);
    }
    if (p.fill == kFillPeriodic) {
      const int pre = max(0, -lo_el), suf = max(0, lo_el + cnt - nc);
      if (pre) {
        bulk_g2s(dst, row + (nc - pre), pre * sizeof(A), &bar[s]);
        tx += pre * sizeof(A);
      }
      if (suf) {
        bulk_g2s(dst + (nc - lo_el), row, suf * sizeof(A), &bar[s]);
        tx += suf * sizeof(A);
      }
    }
    return tx;
  };
  auto tx_range = [&](int lo_el, int cnt, int nc) {
    const int lo = max(lo_el, 0), hi = min(lo_el + cnt, nc);
    unsigned tx = hi > lo ? (hi - lo) * sizeof(A) : 0;
    if (p.fill == kFillPeriodic)
      tx += (max(0, -lo_el) + max(0, lo_el + cnt - nc)) * sizeof(A);
    return tx;
  };
  auto issue = [&](int64_t g, int s) {
    const int64_t row = g / p.tiles;
    const int t = static_cast<int>(g % p.tiles);
    const int gl = glo_of(t), g2 = g2lo_of(t);
    mbar_expect_tx(&bar[s], tx_range(gl, span, p.nc1) + 2 * tx_range(g2, span2, p.nc2) +
                                (g == 0 ? p.dbg_tx : 0u));
    A* d1s = slot(s);
    copy_range(d1s, p.d1 + row * p.nc1, gl, span, p.nc1, s);
    copy_range(d1s + span, p.a2 + row * p.a2_stride, g2, span2, p.nc2, s);
    copy_range(d1s + span + span2, p.d2 + row * p.nc2, g2, span2, p.nc2, s);
  };
#pragma unroll 1
  for (int s = 0; s < kStreamStages; ++s) {
    const int64_t g = blockIdx.x + s * G;
    if (g < p.ntile) zero_fill(g, s);
  }
  __syncthreads();
  if (tid == 0) {
#pragma unroll 1
    for (int s = 0; s < kStreamStages; ++s) {
      const int64_t g = blockIdx.x + s * G;
      if (g < p.ntile) issue(g, s);
    }
  }
  int k = 0;
#pragma unroll 1
  for (int64_t g = blockIdx.x; g < p.ntile; g += G, ++k) {
    const int s = k % kStreamStages;
    const unsigned par = static_cast<unsigned>(k / kStreamStages) & 1u;
    const bool ok = mbar_wait_bounded(&bar[s], par, p.tries);
    const int64_t row = g / p.tiles;
    const int t = static_cast<int>(g % p.tiles);
    const int gl = glo_of(t);
    const A* d1s = slot(s);
    const A* a2s = d1s + span;
    const A* d2s = a2s + span2;
    if (ok) {  // level k+1: a1 over the slot range (buffer cell q - glo + 8)
#pragma unroll 1
      for (int m = tid; m < p.M1; m += SNT) {
        A z[2 * TQ];
        syn_window_item<A, LM, C0, R>(p.hp, a2s + 4 * m, d2s + 4 * m, z);
        A* b = abuf + p.delta + 8 * m;  // vector stores (delta is even; the buffer is aligned)
        if constexpr (sizeof(A) == 4) {
          if ((p.delta & 3) == 0) {
            reinterpret_cast<float4*>(b)[0] = make_float4(z[0], z[1], z[2], z[3]);
            reinterpret_cast<float4*>(b)[1] = make_float4(z[4], z[5], z[6], z[7]);
          } else {
#pragma unroll
            for (int q = 0; q < 2 * TQ; q += 2)
              *reinterpret_cast<float2*>(b + q) = make_float2(z[q], z[q + 1]);
          }
        } else {
#pragma unroll
          for (int q = 0; q < 2 * TQ; q += 2)
            *reinterpret_cast<double2*>(b + q) = make_double2(z[q], z[q + 1]);
        }
      }
    }
    __syncthreads();
    const int c_lo = p.delta, c_hi = p.delta + 8 * p.M1;  // computed buffer cells
    if (p.fill == kFillZero && (gl + c_lo - 8 < 0 || gl + c_hi - 8 > p.nc1)) {
      if (ok) {
        for (int i = c_lo + tid; i < min(c_hi, 8 - gl); i += SNT) abuf[i] = A(0);
        for (int i = max(c_lo, p.nc1 - gl + 8) + tid; i < c_hi; i += SNT) abuf[i] = A(0);
      }
      __syncthreads();
    }
    if (ok) {  // level k: y
      A* yrow = p.y + row * p.n_out;
      const int ms = t * T;
#pragma unroll 1
      for (int it = tid; it < T / 8; it += SNT) {
        const int p0 = ms + 8 * it;
        if (p0 >= p.n_out) break;
        A z[2 * TQ];
        syn_window_item<A, LM, C0, R>(p.hp, abuf + 8 + 4 * it, d1s + 4 * it, z);
        if (p0 + 8 <= p.n_out) {
          store_vec<A, 2 * TQ>(yrow + p0, z);
        } else {
#pragma unroll
          for (int q = 0; q < 2 * TQ; ++q)
            if (p0 + q < p.n_out) yrow[p0 + q] = z[q];
        }
      }
    }
    if (__syncthreads_or(!ok)) {
      if (tid == 0) {
        atomicExch(p.err, kErrCopyTimeout);
#pragma unroll 1
        for (int j = 0; j < kStreamStages; ++j) {
          const int64_t gj = g + j * G;
          if (gj >= p.ntile) break;
          const int kj = k + j;
          mbar_wait_bounded(&bar[kj % kStreamStages],
                            static_cast<unsigned>(kj / kStreamStages) & 1u,
                            cleanup_tries(p.tries));
        }
      }
      return;
    }
    const int64_t gn = g + kStreamStages * G;
    if (gn < p.ntile) {
      zero_fill(gn, s);
      if (tid == 0) issue(gn, s);
    }
  }
}

template <typename A, int LM, int C0>
__global__ void __launch_bounds__(SNT, 2)
dwt_syn2_stream_kernel(const __grid_constant__ Syn2Params<A, LM> p, int r) {
  extern __shared__ __align__(16) unsigned char ring_smem[];
  __shared__ __align__(8) uint64_t bar[kStreamStages];
  A* ring = reinterpret_cast<A*>(ring_smem);
  A* abuf = ring + static_cast<size_t>(kStreamStages) * (p.span + 2 * p.span2);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStreamStages; ++s) mbar_init(&bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if constexpr (sizeof(A) == 4) {
    switch (r) {
      case 0: syn2_tiles<A, LM, C0, 0>(p, ring, abuf, bar); break;
      case 1: syn2_tiles<A, LM, C0, 1>(p, ring, abuf, bar); break;
      case 2: syn2_tiles<A, LM, C0, 2>(p, ring, abuf, bar); break;
      default: syn2_tiles<A, LM, C0, 3>(p, ring, abuf, bar); break;
    }
  } else {
    if (r == 0) syn2_tiles<A, LM, C0, 0>(p, ring, abuf, bar);
    else syn2_tiles<A, LM, C0, 1>(p, ring, abuf, bar);
  }
}

// Geometry of a fused synthesis pair: Lc (level k+1, processing order) then Lf (level k).
template <typename T, int LM>
struct Syn2Plan {
  bool ok = false;
  int R = 0;
  Syn2Params<typename AccOf<T>::type, LM> p{};
  size_t smem = 0;
};

template <typename T, int LM>
Syn2Plan<T, LM> plan_syn2(int64_t rows, const Level& Lc, const Level& Lf, int off) {
  using A = typename AccOf<T>::type;
  Syn2Plan<T, LM> pl;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return pl;
  } else {
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    const int64_t nc2 = Lc.n_coef, a2_stride = Lc.a_len, n1 = Lc.n_in;
    const int64_t nc1 = Lf.n_coef, n_out = Lf.n_in;
    if (!stream_fills(Lc) || !stream_fills(Lf) || Lc.mode != Lf.mode || rows <= 0) return pl;
    if (Lf.a_len != n1 || nc1 > n1 || n_out < kStreamMinOut || n_out > 0x3fffffffLL) return pl;
    if (nc2 % VW || a2_stride % VW || nc1 % VW || n_out % VW) return pl;
    if (Lc.mode == FDWT_MODE_PERIODIZATION && nc1 != n1) return pl;
    const int fill = Lf.mode == FDWT_MODE_ZERO ? kFillZero : kFillPeriodic;
    const int C0 = off & 1;
    const int half = (off + C0) / 2;
    const int R = ((-half) % VW + VW) % VW;
    constexpr int NWIN = TQ + LM / 2;
    const int NL = (R + NWIN + VW - 1) / VW;
    const int Mmax = sizeof(A) == 8 ? SNT / 2 : SNT;  // a1 items per tile
    // the largest tile whose a1 items fit one per thread, then tiles of equal size
    const int T_max = 16 * VW * ((2 * (8 * Mmax - 4 - NL * VW)) / (16 * VW));
    const int64_t n_tiles = cdiv(n_out, T_max);
    const int Tt = static_cast<int>(cdiv(cdiv(n_out, n_tiles), 16 * VW) * 16 * VW);
    const int span = Tt / 2 - 4 + NL * VW;
    auto glo = [&](int64_t t) { return ((t * Tt - off - C0) >> 1) - R; };
    const int64_t c0 = glo(0) - off - C0;
    const int delta = static_cast<int>(((2 * R - c0) % (2 * VW) + 2 * VW) % (2 * VW));
    const int M1 = (span + 8 - delta + 7) / 8;
    const int span2 = 4 * (M1 - 1) + NL * VW;
    int abuf = std::max(8 + span, delta + 8 * M1);
    abuf = (abuf + VW - 1) / VW * VW;
    const int64_t tiles = cdiv(n_out, Tt);
    if (fill == kFillPeriodic) {  // one period at most on either side
      auto g2lo = [&](int64_t t) { return ((glo(t) - off - C0 + delta - 8) >> 1) - R; };
      if (-glo(0) > nc1 || glo(tiles - 1) + span - nc1 > nc1 || -g2lo(0) > nc2 ||
          g2lo(tiles - 1) + span2 - nc2 > nc2)
        return pl;
    }
    if (rows * tiles > (1LL << 40)) return pl;
    auto& p = pl.p;
    p.a2_stride = a2_stride;
    p.ntile = rows * tiles;
    p.nc2 = static_cast<int>(nc2);
    p.nc1 = static_cast<int>(nc1);
    p.n_out = static_cast<int>(n_out);
    p.off = off;
    p.fill = fill;
    p.tiles = static_cast<int>(tiles);
    p.T = Tt;
    p.span = span;
    p.span2 = span2;
    p.M1 = M1;
    p.delta = delta;
    p.abuf = abuf;
    pl.R = R;
    pl.smem = (static_cast<size_t>(kStreamStages) * (span + 2 * span2) + abuf) * sizeof(A);
    pl.ok = pl.smem <= static_cast<size_t>(max_smem_optin()) - 2048;
    return pl;
  }
}

template <typename T, int LM>
bool syn2_fuses(int64_t rows, const Level& Lc, const Level& Lf, int off) {
  return plan_syn2<T, LM>(rows, Lc, Lf, off).ok;
}

// Runs the synthesis levels Lc (coarser) and Lf (finer) in one streaming pass: a2 (rows x
// Lc.a_len), Lc.detail and Lf.detail -> y (rows x Lf.n_in).  FDWT_ERR_UNSUPPORTED when the pair
// does not fuse.
template <typename T, int LM>
int run_syn2_stream(int64_t rows, const void* a2, const Level& Lc, const Level& Lf, void* y,
                    const double* h0, const double* h1, int L, int off, cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return FDWT_ERR_UNSUPPORTED;
  } else {
    Syn2Plan<T, LM> pl = plan_syn2<T, LM>(rows, Lc, Lf, off);
    auto aligned = [](const void* q) { return q && (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (!pl.ok || !aligned(a2) || !aligned(Lc.detail) || !aligned(Lf.detail) || !aligned(y))
      return FDWT_ERR_UNSUPPORTED;
    auto& p = pl.p;
    p.a2 = static_cast<const A*>(a2);
    p.d2 = static_cast<const A*>(Lc.detail);
    p.d1 = static_cast<const A*>(Lf.detail);
    p.y = static_cast<A*>(y);
    p.err = device_error_flag();
    if (p.err == nullptr) return FDWT_ERR_CUDA;
    {
      const CopyWaitTest wt = copy_wait_test();
      p.dbg_tx = wt.extra_tx;
      p.tries = wt.tries;
    }
    A hh0[LM], hh1[LM];
    for (int j = 0; j < LM; ++j) {
      hh0[j] = j < L ? static_cast<A>(h0[j]) : A(0);
      hh1[j] = j < L ? static_cast<A>(h1[j]) : A(0);
    }
    for (int m = 0; m <= LM; ++m) {
      p.hp[2 * m] = m < LM ? hh0[m] : A(0);
      p.hp[2 * m + 1] = m >= 1 ? hh0[m - 1] : A(0);
      p.hp[2 * (LM + 1) + 2 * m] = m < LM ? hh1[m] : A(0);
      p.hp[2 * (LM + 1) + 2 * m + 1] = m >= 1 ? hh1[m - 1] : A(0);
    }
    auto kern = (off & 1) ? dwt_syn2_stream_kernel<A, LM, 1> : dwt_syn2_stream_kernel<A, LM, 0>;
    int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (st != FDWT_OK) return st;
    int occ = 0;
    if ((st = occupancy(reinterpret_cast<const void*>(kern), SNT, pl.smem, &occ)) != FDWT_OK) return st;
    if (occ < 1) return FDWT_ERR_UNSUPPORTED;
    const int64_t grid = std::min<int64_t>(p.ntile, static_cast<int64_t>(occ) * sm_count());
    if ((st = pre_launch(stream)) != FDWT_OK) return st;
    kern<<<static_cast<unsigned>(grid), SNT, pl.smem, stream>>>(p, pl.R);
    return launch_status();
  }
}

}  // namespace dwtk
}  // namespace fdwt
