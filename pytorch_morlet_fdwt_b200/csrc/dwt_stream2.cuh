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

template <typename A, int LM>
struct Ana2Params {
  const A* x;        // (rows, n)
  A* d1;             // (rows, nc1) level-k details
  A* a2;             // (rows, a_len2) level-(k+1) approximation
  A* d2;             // (rows, nc2) level-(k+1) details
  int* err;          // device error word
  int64_t ntile;     // rows * tiles
  int64_t P;         // period of level k's boundary mode on n
  int64_t P2;        // period of level k+1's boundary mode on n1
  int32_t n, nc1, n1, nc2, a_len2, off, mode, mode2, tiles;
  int32_t span;      // x elements per ring slot
  int32_t T2;        // level-(k+1) outputs per tile (V q, with K1 = kh + 2q + kr <= SNT)
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
    const A* xr = p.x + row * n;
    A* sl = slot(s);
    auto one = [&](int q) {
      const int64_t e = ext_index(q, n, p.mode, p.P);
      if (e < 0) sl[q - xlo] = A(0);
      else cp_async(sl + (q - xlo), xr + e, sizeof(A));
    };
    const int l1 = min(xlo + span, 0), r1 = min(xlo + span, p.x_hi);
    for (int q = xlo + tid; q < l1; q += SNT) one(q);
    for (int q = max(xlo, n) + tid; q < r1; q += SNT) one(q);
    cp_async_commit();
  };
  auto issue = [&](int64_t g, int s) {
    const int64_t row = g / p.tiles;
    const int xlo = slot_lo(static_cast<int>(g % p.tiles));
    const int lo = max(xlo, 0), hi = min(xlo + span, n);
    const unsigned bytes = static_cast<unsigned>(max(hi - lo, 0)) * sizeof(A);
    mbar_expect_tx(&bar[s], bytes);
    if (bytes) bulk_g2s(slot(s) + (lo - xlo), p.x + row * n + lo, bytes, &bar[s]);
  };
#pragma unroll 1
  for (int s = 0; s < kStreamStages; ++s) {
    const int64_t g = blockIdx.x + s * G;
    if (g < p.ntile) ext_fill(g, s);
    else cp_async_commit();
  }
  cp_async_wait<kStreamStages - 1>();
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
    const bool ok = mbar_wait_bounded(&bar[s], par);
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
      A* a2row = p.a2 + row * p.a_len2;
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
    cp_async_wait<kStreamStages - 2>();  // this thread's gathers of tile k + 1
    if (__syncthreads_or(!ok)) {
      cp_async_wait<0>();
      if (tid == 0) {
        atomicExch(p.err, kErrCopyTimeout);
#pragma unroll 1
        for (int j = 0; j < kStreamStages; ++j) {
          const int64_t gj = g + j * G;
          if (gj >= p.ntile) break;
          const int kj = k + j;
          mbar_wait_bounded(&bar[kj % kStreamStages],
                            static_cast<unsigned>(kj / kStreamStages) & 1u);
        }
      }
      return;
    }
    const int64_t gn = g + kStreamStages * G;
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
  __shared__ __align__(8) uint64_t bar[kStreamStages];
  A* ring = reinterpret_cast<A*>(ring_smem);
  A* abuf = ring + static_cast<size_t>(kStreamStages) * p.span;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStreamStages; ++s) mbar_init(&bar[s], 1);
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
Ana2Plan<T, LM> plan_ana2(int64_t rows, const Level& L1, const Level& L2, int off) {
  using A = typename AccOf<T>::type;
  Ana2Plan<T, LM> pl;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return pl;
  } else {
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    constexpr int V = ana_stream_v<A>();
    const int64_t n = L1.n_in, nc1 = L1.n_coef, n1 = L2.n_in, nc2 = L2.n_coef;
    if (n < 1024 || n % VW || n > 0x3fffffffLL || nc2 < 1 || L1.a_len != n1 ||
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
    // one level-k item per thread: K1 = kh + T1 / V + kr <= SNT
    const int T2 = V * ((SNT - kh - kr) / 2);
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
    pl.smem = (static_cast<size_t>(kStreamStages) * span + abuf) * sizeof(A);
    pl.ok = pl.smem <= static_cast<size_t>(max_smem_optin()) - 2048;
    return pl;
  }
}

// Runs levels L1, L2 of an analysis in one streaming pass: x (rows x L1.n_in) -> details of both
// levels (L1.detail, L2.detail) and the level-2 approximation a2_out (rows x L2.a_len).
// FDWT_ERR_UNSUPPORTED when the pair does not fuse.
template <typename T, int LM>
int run_ana2_stream(int64_t rows, const void* x, const Level& L1, const Level& L2, void* a2_out,
                    const double* h0, const double* h1, int L, int off, cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return FDWT_ERR_UNSUPPORTED;
  } else {
    Ana2Plan<T, LM> pl = plan_ana2<T, LM>(rows, L1, L2, off);
    if (!pl.ok || x == nullptr || a2_out == nullptr || L1.detail == nullptr ||
        L2.detail == nullptr || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
      return FDWT_ERR_UNSUPPORTED;
    auto& p = pl.p;
    p.x = static_cast<const A*>(x);
    p.d1 = static_cast<A*>(L1.detail);
    p.a2 = static_cast<A*>(a2_out);
    p.d2 = static_cast<A*>(L2.detail);
    p.err = device_error_flag();
    if (p.err == nullptr) return FDWT_ERR_CUDA;
    for (int j = 0; j < LM; ++j) {
      p.taps[2 * j] = j < L ? static_cast<A>(h0[j]) : A(0);
      p.taps[2 * j + 1] = j < L ? static_cast<A>(h1[j]) : A(0);
    }
    auto kern = dwt_ana2_stream_kernel<A, LM>;
    int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (st != FDWT_OK) return st;
    int occ = 0;
    FDWT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, SNT, pl.smem));
    if (occ < 1) return FDWT_ERR_UNSUPPORTED;
    const int64_t grid = std::min<int64_t>(p.ntile, static_cast<int64_t>(occ) * sm_count());
    if ((st = pre_launch(stream)) != FDWT_OK) return st;
    kern<<<static_cast<unsigned>(grid), SNT, pl.smem, stream>>>(p, pl.R);
    return launch_status();
  }
}

}  // namespace dwtk
}  // namespace fdwt
