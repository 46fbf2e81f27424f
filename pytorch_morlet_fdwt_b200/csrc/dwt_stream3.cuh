// Three analysis levels per streaming pass, for sm_100a.  Included by dwt_impl.cuh after
// dwt_stream2.cuh, whose ring, copies, bounded waits and window items it uses.
//
// Levels k, k+1 and k+2 of a multilevel analysis in one pass over x, for the periodization and
// zero modes: a tile owns T3 outputs of level k+2 (cA3, cD3), the 2 T3 level-(k+1) details and
// the 4 T3 level-k details under them.  Level k+1 reads cA1 and level k+2 reads cA2, each over
// its tile plus a halo of LM - 2 positions; the CTA computes cA1 from its x slot into a first
// shared buffer and cA2 from that into a second (the halos are recomputed by both tiles that
// need them, a few percent more arithmetic), storing the details it owns on the way.  Neither
// cA1 nor cA2 touches HBM: the pass reads x once and writes cD1, cD2, cD3 and cA3 once -- the
// handover of cA2 between two passes (written, then read back) disappears.
//
// Boundary modes: in periodization (x of a length divisible by 8, one period) cA1 and cA2 are
// periodic with periods n / 2 and n / 4, and the positions outside a row computed from the
// periodically continued x are exactly their continuation; in zero mode the cells outside
// [0, nc) of each buffer are set to 0 (the next level's zero extension).  Other modes run as
// pairs and single levels.
//
// Items are those of the one-level kernel (V outputs, windows 48 bytes apart).  Level j's items
// start V kh_j outputs before the tile's first owned detail of that level, and each buffer
// starts B_j cells in, so that the next level's windows keep the 16-byte shift R of the level-k
// windows.
#pragma once

namespace fdwt {
namespace dwtk {

template <typename A, int LM>
struct Ana3Params {
  const A* x;        // (rows, xs)
  A* d1;             // (rows, nc1) level-k details
  A* d2;             // (rows, nc2) level-(k+1) details
  A* d3;             // (rows, nc3) level-(k+2) details
  A* a3;             // (rows, as) level-(k+2) approximation
  int* err;          // device error word
  uint32_t dbg_tx;   // test hook: extra expected bytes of global tile 0's copy
  long long tries;   // poll limit of the main mbarrier waits
  int64_t ntile;     // rows * tiles
  int64_t P;         // period of level k's boundary mode on n
  int32_t n, nc1, nc2, nc3, a_len3, off, mode, tiles;
  int32_t xs, as;    // row strides of x and of cA3 (xs a multiple of 16 bytes)
  int32_t n_al;      // n rounded down to 16 bytes: the bulk copies end there
  int32_t span;      // x elements per ring slot
  int32_t T3;        // level-(k+2) outputs per tile (a multiple of V)
  int32_t K1, kh1;   // level-k items per tile, of which kh1 before the first owned detail
  int32_t K2, kh2;   // level-(k+1) items per tile, of which kh2 before the first owned detail
  int32_t B1, S2;    // first cA1 cell in buffer 1; level-(k+1) window base (S2 - R aligned)
  int32_t B2, S3;    // first cA2 cell in buffer 2; level-(k+2) window base (S3 - R aligned)
  int32_t abuf1, abuf2;  // buffer elements
  int32_t x_hi;      // x positions past the row end up to x_hi are gathered
  alignas(16) A taps[2 * LM];  // (h0[j], h1[j]) interleaved
};

template <typename A, int LM, int R>
__device__ void ana3_tiles(const Ana3Params<A, LM>& p, A* ring, A* buf1, A* buf2,
                           uint64_t* bar) {
  constexpr int V = ana_stream_v<A>();
  const int T3 = p.T3;
  const int T2 = 2 * T3, T1 = 4 * T3;
  const int tid = threadIdx.x;
  const int64_t G = gridDim.x;
  const int span = p.span, n = p.n;
  const int pmin = p.off - (LM - 1);
  auto slot = [&](int s) { return ring + static_cast<size_t>(s) * span; };
  auto first_o1 = [&](int t) { return t * T1 - V * p.kh1; };
  auto first_o2 = [&](int t) { return t * T2 - V * p.kh2; };
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
  // zero mode: buffer cells of positions outside [0, nc) are the next level's zero extension
  auto zero_outside = [&](A* b, int cell0, int first, int cnt, int nc) {
    const int l_end = min(cnt, -first), r_beg = max(0, nc - first);
    for (int i = tid; i < l_end; i += SNT) b[cell0 + i] = A(0);
    for (int i = r_beg + tid; i < cnt; i += SNT) b[cell0 + i] = A(0);
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
  const bool zero = p.mode == FDWT_MODE_ZERO;
  int k = 0;
#pragma unroll 1
  for (int64_t g = blockIdx.x; g < p.ntile; g += G, ++k) {
    const int s = k % ana2_stages<A>();
    const unsigned par = static_cast<unsigned>(k / ana2_stages<A>()) & 1u;
    const bool ok = mbar_wait_bounded(&bar[s], par, p.tries);
    const int64_t row = g / p.tiles;
    const int t = static_cast<int>(g % p.tiles);
    const int o1_0 = first_o1(t), o2_0 = first_o2(t);
    if (ok) {  // level k: cA1 into buffer 1, the owned cD1 to HBM
      const A* sl = slot(s);
      A* d1row = p.d1 + row * p.nc1;
#pragma unroll 1
      for (int it = tid; it < p.K1; it += SNT) {
        A ra[V], rd[V];
        ana_window_item<A, LM, R>(p.taps, sl + 2 * V * it, ra, rd);
        A* b = buf1 + p.B1 + V * it;
#pragma unroll
        for (int v = 0; v < V; ++v) b[v] = ra[v];
        const int o1 = o1_0 + V * it;
        if (it >= p.kh1 && it < p.kh1 + T1 / V && o1 < p.nc1)
          store_run<A, V>(d1row + o1, rd, min(V, p.nc1 - o1));
      }
    }
    __syncthreads();
    if (zero && (o1_0 < 0 || o1_0 + V * p.K1 > p.nc1)) {
      if (ok) zero_outside(buf1, p.B1, o1_0, V * p.K1, p.nc1);
      __syncthreads();
    }
    if (ok) {  // level k+1: cA2 into buffer 2, the owned cD2 to HBM
      A* d2row = p.d2 + row * p.nc2;
#pragma unroll 1
      for (int it = tid; it < p.K2; it += SNT) {
        A ra[V], rd[V];
        ana_window_item<A, LM, R>(p.taps, buf1 + 2 * V * it + p.S2 - R, ra, rd);
        A* b = buf2 + p.B2 + V * it;
#pragma unroll
        for (int v = 0; v < V; ++v) b[v] = ra[v];
        const int o2 = o2_0 + V * it;
        if (it >= p.kh2 && it < p.kh2 + T2 / V && o2 < p.nc2)
          store_run<A, V>(d2row + o2, rd, min(V, p.nc2 - o2));
      }
    }
    __syncthreads();
    if (zero && (o2_0 < 0 || o2_0 + V * p.K2 > p.nc2)) {
      if (ok) zero_outside(buf2, p.B2, o2_0, V * p.K2, p.nc2);
      __syncthreads();
    }
    if (ok) {  // level k+2 from buffer 2
      A* a3row = p.a3 + row * p.as;
      A* d3row = p.d3 + row * p.nc3;
#pragma unroll 1
      for (int m = tid; m < T3 / V; m += SNT) {
        const int o3 = t * T3 + V * m;
        if (o3 >= p.nc3) break;
        A ra[V], rd[V];
        ana_window_item<A, LM, R>(p.taps, buf2 + 2 * V * m + p.S3 - R, ra, rd);
        const int cnt = min(V, p.nc3 - o3);
        store_run<A, V>(d3row + o3, rd, cnt);
        store_run<A, V>(a3row + o3, ra, cnt);
      }
      if (t == p.tiles - 1 && tid == 0)
        for (int q = p.nc3; q < p.a_len3; ++q) a3row[q] = A(0);  // transpose of waverec's trim
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
dwt_ana3_stream_kernel(const __grid_constant__ Ana3Params<A, LM> p, int r) {
  extern __shared__ __align__(16) unsigned char ring_smem[];
  __shared__ __align__(8) uint64_t bar[ana2_stages<A>()];
  A* ring = reinterpret_cast<A*>(ring_smem);
  A* buf1 = ring + static_cast<size_t>(ana2_stages<A>()) * p.span;
  A* buf2 = buf1 + p.abuf1;
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < ana2_stages<A>(); ++s) mbar_init(&bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if constexpr (sizeof(A) == 4) {
    switch (r) {
      case 0: ana3_tiles<A, LM, 0>(p, ring, buf1, buf2, bar); break;
      case 1: ana3_tiles<A, LM, 1>(p, ring, buf1, buf2, bar); break;
      case 2: ana3_tiles<A, LM, 2>(p, ring, buf1, buf2, bar); break;
      default: ana3_tiles<A, LM, 3>(p, ring, buf1, buf2, bar); break;
    }
  } else {
    if (r == 0) ana3_tiles<A, LM, 0>(p, ring, buf1, buf2, bar);
    else ana3_tiles<A, LM, 1>(p, ring, buf1, buf2, bar);
  }
}

// ------------------------------------------------------------------------------ host

template <typename T, int LM>
struct Ana3Plan {
  bool ok = false;
  int R = 0;
  Ana3Params<typename AccOf<T>::type, LM> p{};
  size_t smem = 0;
};

// Geometry of a fused triple (levels L1, L2, L3 of one analysis with offset off); ok = false
// when the triple does not fuse.  Shape-only: the input pointer's alignment is the caller's check.
template <typename T, int LM>
Ana3Plan<T, LM> plan_ana3(int64_t rows, const Level& L1, const Level& L2, const Level& L3,
                          int off, int64_t xs) {
  using A = typename AccOf<T>::type;
  Ana3Plan<T, LM> pl;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return pl;
  } else {
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    constexpr int V = ana_stream_v<A>();
    const int64_t n = L1.n_in, nc1 = L1.n_coef, nc2 = L2.n_coef, nc3 = L3.n_coef;
    if (n < 4096 || xs % VW || xs < n || xs > 0x3fffffffLL || nc3 < 1 || rows <= 0) return pl;
    if (L1.a_len != L2.n_in || L2.a_len != L3.n_in || L3.a_len > nc3 + 1) return pl;
    const int mode = L1.mode;
    if (L2.mode != mode || L3.mode != mode) return pl;
    if (mode == FDWT_MODE_PERIODIZATION) {
      if (!(n % 8 == 0 && nc1 == n / 2 && L2.n_in == nc1 && nc2 == nc1 / 2 &&
            L3.n_in == nc2 && nc3 == nc2 / 2 && L1.P == n && L2.P == nc1 && L3.P == nc2))
        return pl;
    } else if (mode != FDWT_MODE_ZERO) {
      return pl;
    }
    const int pmin = off - (LM - 1);
    const int R = ((pmin % VW) + VW) % VW;
    constexpr int W = 2 * V + LM - 2;
    const int NL = (R + W + VW - 1) / VW;
    const int hl = (std::max(-pmin, 0) + V - 1) / V;        // left halo items of one level
    const int hr = (std::max(off - 1, 0) + V - 1) / V;      // right halo items of one level
    const int kh2 = hl, kh1 = 2 * kh2 + hl;
    // two level-k items per thread: K1 = kh1 + 4 T3 / V + 3 hr <= 2 SNT
    const int q_max = (2 * SNT - kh1 - 3 * hr) / 4;
    if (q_max < 1) return pl;
    const int64_t n_tiles = cdiv(nc3, static_cast<int64_t>(V) * q_max);
    const int T3 = V * static_cast<int>(cdiv(cdiv(nc3, n_tiles), V));
    const int T2 = 2 * T3, T1 = 4 * T3;
    const int K2 = kh2 + T2 / V + hr;
    const int K1 = kh1 + T1 / V + 3 * hr;
    const int span = 2 * V * K1 - 2 * V + NL * VW;
    const int B1 = (((R - pmin - V * (kh1 - 2 * kh2)) % VW) + VW) % VW;
    const int S2 = B1 + pmin + V * (kh1 - 2 * kh2);
    const int B2 = (((R - pmin - V * kh2) % VW) + VW) % VW;
    const int S3 = B2 + pmin + V * kh2;
    int abuf1 = std::max(B1 + V * K1, 2 * V * (K2 - 1) + S2 - R + NL * VW);
    abuf1 = (abuf1 + VW - 1) / VW * VW;
    int abuf2 = std::max(B2 + V * K2, 2 * V * (T3 / V - 1) + S3 - R + NL * VW);
    abuf2 = (abuf2 + VW - 1) / VW * VW;
    const int64_t tiles = cdiv(nc3, T3);
    if (rows * tiles > (1LL << 40)) return pl;
    // every level-(k+1) window of a tile lies inside the cA1 cells it computed, and every
    // level-(k+2) window inside its cA2 cells
    if (S2 - R < 0 || S3 - R < 0 || 2 * V * (K2 - 1) + S2 + W > B1 + V * K1 ||
        2 * V * (T3 / V - 1) + S3 + W > B2 + V * K2)
      return pl;
    const int64_t max_o1 = std::max<int64_t>(tiles * T1 - V * kh1 + V * K1 - 1, nc1 - 1);
    auto& p = pl.p;
    p.ntile = rows * tiles;
    p.P = L1.P;
    p.n = static_cast<int>(n);
    p.nc1 = static_cast<int>(nc1);
    p.nc2 = static_cast<int>(nc2);
    p.nc3 = static_cast<int>(nc3);
    p.a_len3 = static_cast<int>(L3.a_len);
    p.xs = static_cast<int>(xs);
    p.n_al = static_cast<int>(n / VW * VW);
    p.off = off;
    p.mode = mode;
    p.tiles = static_cast<int>(tiles);
    p.span = span;
    p.T3 = T3;
    p.K1 = K1;
    p.kh1 = kh1;
    p.K2 = K2;
    p.kh2 = kh2;
    p.B1 = B1;
    p.S2 = S2;
    p.B2 = B2;
    p.S3 = S3;
    p.abuf1 = abuf1;
    p.abuf2 = abuf2;
    p.x_hi = static_cast<int>(std::min<int64_t>(2 * max_o1 + off + 1, 0x3fffffffLL));
    pl.R = R;
    pl.smem = (static_cast<size_t>(ana2_stages<A>()) * span + abuf1 + abuf2) * sizeof(A);
    pl.ok = pl.smem <= static_cast<size_t>(max_smem_optin()) - 2048;
    return pl;
  }
}

// Runs levels L1, L2, L3 of an analysis in one streaming pass: x (rows of L1.n_in samples, xs
// apart) -> the details of all three levels and the level-3 approximation a3_out (rows of
// L3.a_len, as apart).  FDWT_ERR_UNSUPPORTED when the triple does not fuse.
template <typename T, int LM>
int run_ana3_stream(int64_t rows, const void* x, const Level& L1, const Level& L2,
                    const Level& L3, int64_t xs, void* a3_out, int64_t as, const double* h0,
                    const double* h1, int L, int off, cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return FDWT_ERR_UNSUPPORTED;
  } else {
    Ana3Plan<T, LM> pl = plan_ana3<T, LM>(rows, L1, L2, L3, off, xs);
    if (!pl.ok || as < L3.a_len || as > 0x3fffffffLL || x == nullptr || a3_out == nullptr || L1.detail == nullptr ||
        L2.detail == nullptr || L3.detail == nullptr ||
        (reinterpret_cast<uintptr_t>(x) & 15) != 0)
      return FDWT_ERR_UNSUPPORTED;
    auto& p = pl.p;
    p.x = static_cast<const A*>(x);
    p.d1 = static_cast<A*>(L1.detail);
    p.d2 = static_cast<A*>(L2.detail);
    p.d3 = static_cast<A*>(L3.detail);
    p.a3 = static_cast<A*>(a3_out);
    p.as = static_cast<int>(as);
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
    auto kern = dwt_ana3_stream_kernel<A, LM>;
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
