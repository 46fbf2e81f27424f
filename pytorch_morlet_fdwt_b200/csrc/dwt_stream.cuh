// One-level DWT synthesis of the interior output tiles of long rows by persistent CTAs that
// stream their coefficients through a ring of bulk asynchronous copies, for sm_100a.  Included
// by dwt_impl.cuh after dwt_syn_tile.cuh, whose tile geometry and inner loop it shares.
//
// Away from the row ends (no boundary folds, the whole dependency cone inside the row) the
// one-level synthesis y = S(a, d) is a plain stencil: a tile of T outputs [t T, t T + T) reads
// T/2 + L/2 + O(1) consecutive coefficients of a and of d -- two contiguous ranges which, for
// rows whose lengths are multiples of 16 bytes, start on a 16-byte boundary at a launch-wide
// offset R before the first window.  One thread copies both ranges of a tile into a ring slot
// with cp.async.bulk, completing on the slot's mbarrier.  The CTA is persistent: it walks a
// strided list of interior tiles with kStreamStages tiles in flight, so the copies of the next
// tiles overlap the arithmetic and stores of the current one, and one CTA barrier per tile
// releases its slot.  The few tiles near the row ends (and rows that do not meet the alignment
// conditions) run on the tile kernel.
//
// Every wait on an mbarrier is bounded (kStreamWaitTries polls): a copy that never completes
// makes the CTA record kErrCopyTimeout in the device error word, wait (bounded again) for the
// rest of its copies, and return.
//
// Inner loop: items of 8 outputs as in the tile kernel; item i of a tile takes the window
// slot[4 i + R, 4 i + R + TQ + LM/2) of both arrays, read as whole 16-byte words from the dense
// slot (the lanes of a warp read consecutive 16-byte words: no bank conflicts).
#pragma once

namespace fdwt {
namespace dwtk {

constexpr int SNT = 256;             // threads per streaming CTA
constexpr int kStreamStages = 3;     // ring slots (tiles in flight per CTA)
constexpr long long kStreamWaitTries = kCopyWaitTries;
constexpr int kFillNone = 0, kFillZero = 1, kFillPeriodic = 2;

template <typename A, int LM>
struct StreamParams {
  const A* a;        // (rows, a_stride) approximation
  const A* d;        // (rows, nc) details
  A* y;              // (rows, n_out)
  int* err;          // device error word
  uint32_t dbg_tx;   // test hook: extra expected bytes of global tile 0's copy
  long long tries;   // poll limit of the main mbarrier waits
  int64_t a_stride;
  int64_t ntile;     // rows * ni interior tiles
  int32_t nc, n_out, off, ni, t_lo;
  int32_t T;         // outputs per tile (a multiple of 64)
  int32_t span;      // elements per slot array (multiple of 16 bytes)
  int32_t fill;      // kFillNone: interior tiles only; kFillZero / kFillPeriodic: every tile,
                     // the slot outside [0, nc) holds zeros / the periodic continuation
  alignas(16) A hp[2 * (LM + 1) * 2];  // (h0[m], h0[m-1]) then (h1[m], h1[m-1]), m = 0..LM
};

__device__ __forceinline__ unsigned smem_u32(const void* p) {
  return static_cast<unsigned>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, unsigned parity,
                                                  long long tries) {
  for (long long i = 0; i < tries; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// Poll limit of the wait for a CTA's copies still in flight after a timeout: never shorter than
// 2^20 polls, so that a shortened test limit cannot end a CTA while its copies still land.
__device__ __forceinline__ long long cleanup_tries(long long tries) {
  return tries > (1LL << 20) ? tries : (1LL << 20);
}
// global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned)
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, unsigned bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <typename A>
__device__ __forceinline__ void load16(const A* s, A* r) {
  if constexpr (sizeof(A) == 4) {
    const float4 v = *reinterpret_cast<const float4*>(s);
    r[0] = v.x;
    r[1] = v.y;
    r[2] = v.z;
    r[3] = v.w;
  } else {
    const double2 v = *reinterpret_cast<const double2*>(s);
    r[0] = v.x;
    r[1] = v.y;
  }
}

// Outputs [p0, p0 + 8) from the windows aw[R .. R + NWIN), dw[R .. R + NWIN) (aw, dw 16-byte
// aligned): the packed-tap recursion of tile_item on a dense window; hp = the packed taps
// (h0[m], h0[m-1]) for m = 0..LM followed by those of h1.
template <typename A, int LM, int C0, int R>
__device__ __forceinline__ void syn_window_item(const A* hp, const A* aw, const A* dw,
                                                A (&z)[2 * TQ]) {
  constexpr int NV = LM / 2 + 1;
  constexpr int NWIN = TQ + NV - 1;
  constexpr int VW = 16 / static_cast<int>(sizeof(A));
  constexpr int NL = (R + NWIN + VW - 1) / VW;
  A wa[NL * VW], wd[NL * VW];
#pragma unroll
  for (int k = 0; k < NL; ++k) {
    load16<A>(aw + k * VW, wa + k * VW);
    load16<A>(dw + k * VW, wd + k * VW);
  }
  Pair<A> xa[NWIN], xd[NWIN];
#pragma unroll
  for (int u = 0; u < NWIN; ++u) {
    xa[u].dup(wa[R + u]);
    xd[u].dup(wd[R + u]);
  }
  Pair<A> acc[TQ];
#pragma unroll
  for (int q = 0; q < TQ; ++q) acc[q].zero();
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int m = 2 * v - C0;
    if (m < 0 || m > LM) continue;  // resolved at compile time
    Pair<A> ha, hd;
    ha.load(&hp[2 * m]);
    hd.load(&hp[2 * (LM + 1) + 2 * m]);
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

template <typename A, int LM, int C0, int R>
__device__ void stream_tiles(const StreamParams<A, LM>& p, A* ring, uint64_t* bar) {
  const int T = p.T;
  const int tid = threadIdx.x;
  const int64_t G = gridDim.x;
  const int span = p.span, nc = p.nc;
  auto slot = [&](int s) { return ring + static_cast<size_t>(s) * 2 * span; };
  // first coefficient of the slot of tile t (a multiple of 16 bytes)
  auto slot_lo = [&](int t) { return ((t * T - p.off - C0) >> 1) - R; };
  // zero the slot cells outside [0, nc) of the tile about to be copied into slot s (all threads)
  auto zero_fill = [&](int64_t g, int s) {
    if (p.fill != kFillZero) return;
    const int glo = slot_lo(p.t_lo + static_cast<int>(g % p.ni));
    const int pre = max(0, -glo), suf0 = max(0, nc - glo);
    A* sa = slot(s);
    A* sd = sa + span;
    for (int i = tid; i < pre; i += SNT) sa[i] = sd[i] = A(0);
    for (int i = suf0 + tid; i < span; i += SNT) sa[i] = sd[i] = A(0);
  };
  // one thread: the bulk copies of tile g's coefficients into slot s, completing on bar[s]
  auto issue = [&](int64_t g, int s) {
    const int64_t row = g / p.ni;
    const int glo = slot_lo(p.t_lo + static_cast<int>(g % p.ni));
    const int lo = max(glo, 0), hi = min(glo + span, nc);
    const int pre = p.fill == kFillPeriodic ? max(0, -glo) : 0;
    const int suf = p.fill == kFillPeriodic ? max(0, glo + span - nc) : 0;
    const unsigned tx = static_cast<unsigned>(max(hi - lo, 0) + pre + suf) * sizeof(A);
    mbar_expect_tx(&bar[s], 2 * tx + (g == 0 ? p.dbg_tx : 0u));
    const A* src[2] = {p.a + row * p.a_stride, p.d + row * nc};
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      A* dst = slot(s) + c * span;
      if (hi > lo) bulk_g2s(dst + (lo - glo), src[c] + lo, (hi - lo) * sizeof(A), &bar[s]);
      if (pre) bulk_g2s(dst, src[c] + (nc - pre), pre * sizeof(A), &bar[s]);
      if (suf) bulk_g2s(dst + (nc - glo), src[c], suf * sizeof(A), &bar[s]);
    }
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
    if (ok) {
      const int64_t row = g / p.ni;
      const int t = p.t_lo + static_cast<int>(g % p.ni);
      const int ms = t * T;
      A* yrow = p.y + row * p.n_out;
      const A* as = slot(s);
      const A* ds = as + span;
#pragma unroll 1
      for (int it = tid; it < T / 8; it += SNT) {
        const int p0 = ms + 8 * it;
        if (p0 >= p.n_out) break;
        A z[2 * TQ];
        syn_window_item<A, LM, C0, R>(p.hp, as + 4 * it, ds + 4 * it, z);
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
      // a copy never completed: record it, wait (bounded) for this CTA's copies still in
      // flight -- this tile's and the ones issued after it -- and stop
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
__global__ void __launch_bounds__(SNT, 3)
dwt_syn_stream_kernel(const __grid_constant__ StreamParams<A, LM> p, int r) {
  extern __shared__ __align__(16) unsigned char ring_smem[];
  __shared__ __align__(8) uint64_t bar[kStreamStages];
  A* ring = reinterpret_cast<A*>(ring_smem);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStreamStages; ++s) mbar_init(&bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if constexpr (sizeof(A) == 4) {
    switch (r) {
      case 0: stream_tiles<A, LM, C0, 0>(p, ring, bar); break;
      case 1: stream_tiles<A, LM, C0, 1>(p, ring, bar); break;
      case 2: stream_tiles<A, LM, C0, 2>(p, ring, bar); break;
      default: stream_tiles<A, LM, C0, 3>(p, ring, bar); break;
    }
  } else {
    if (r == 0) stream_tiles<A, LM, C0, 0>(p, ring, bar);
    else stream_tiles<A, LM, C0, 1>(p, ring, bar);
  }
}

// ------------------------------------------------------------------------------ host

// Runs the one-level synthesis of level L0 (output y, rows x L0.n_in) as the streaming kernel
// over the interior tiles plus the tile kernel over the others.  FDWT_ERR_UNSUPPORTED when the
// streaming kernel does not apply (element type, filter length, alignment, short rows); the
// caller then runs the tile kernel over every tile.
template <typename T, int LM>
int run_syn_stream(int64_t rows, const void* a, const Level& L0, void* y, const double* h0,
                   const double* h1, int L, int off, cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return FDWT_ERR_UNSUPPORTED;
  } else {
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    constexpr int T_full = tile_outputs<A>();
    const int64_t n_out = L0.n_in, nc = L0.n_coef, a_stride = L0.a_len;
    if (L0.detail == nullptr || a == nullptr || y == nullptr || rows <= 0) return FDWT_ERR_UNSUPPORTED;
    if (n_out > 0x3fffffffLL || a_stride > 0x3fffffffLL) return FDWT_ERR_UNSUPPORTED;
    auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
    if (!aligned(a) || !aligned(L0.detail) || !aligned(y) || a_stride % VW || nc % VW ||
        n_out % VW)
      return FDWT_ERR_UNSUPPORTED;
    const int C0 = off & 1;
    const int half = (off + C0) / 2;  // off + C0 is even
    const int R = ((-half) % VW + VW) % VW;
    constexpr int NWIN = TQ + LM / 2;
    const int NL = (R + NWIN + VW - 1) / VW;
    int fill = stream_fills(L0) ? (L0.mode == FDWT_MODE_ZERO ? kFillZero : kFillPeriodic)
                                : kFillNone;
    // filling stages take every tile (rows of one short tile included); the others leave the
    // tiles near the row ends to the tile kernel, whose tiles then must be the same
    const int64_t T_s = fill != kFillNone  // tiles of equal size, at most T_full outputs
                            ? cdiv(cdiv(n_out, cdiv(n_out, T_full)), 64) * 64
                            : T_full;
    const int span = static_cast<int>(T_s / 2 - 4 + NL * VW);  // a multiple of VW
    const int64_t tiles = cdiv(n_out, T_s);
    auto slot_lo = [&](int64_t t) { return ((t * T_s - off - C0) >> 1) - R; };
    if (fill == kFillPeriodic &&
        (-slot_lo(0) > nc || slot_lo(tiles - 1) + span - nc > nc))  // more than one period
      fill = kFillNone;
    if (fill == kFillNone && (T_s != T_full || n_out < 3 * T_full)) return FDWT_ERR_UNSUPPORTED;
    if (fill != kFillNone && n_out < kStreamMinOut) return FDWT_ERR_UNSUPPORTED;
    auto interior = [&](int64_t t) {
      if (fill != kFillNone) return true;
      const int64_t ms = t * T_s, me = ms + T_s;
      if (ms < LM || me > n_out - LM) return false;
      const int64_t glo = slot_lo(t);
      return glo >= 0 && glo + span <= nc;
    };
    int64_t t_lo = 0;
    while (t_lo < tiles && !interior(t_lo)) ++t_lo;
    int64_t t_hi = t_lo;
    while (t_hi < tiles && interior(t_hi)) ++t_hi;
    const int64_t ni = t_hi - t_lo;
    if (ni < 1 || rows * ni > (1LL << 40)) return FDWT_ERR_UNSUPPORTED;

    StreamParams<A, LM> p{};
    p.a = static_cast<const A*>(a);
    p.d = static_cast<const A*>(L0.detail);
    p.y = static_cast<A*>(y);
    p.err = device_error_flag();
    if (p.err == nullptr) return FDWT_ERR_CUDA;
    {
      const CopyWaitTest wt = copy_wait_test();
      p.dbg_tx = wt.extra_tx;
      p.tries = wt.tries;
    }
    p.a_stride = a_stride;
    p.ntile = rows * ni;
    p.nc = static_cast<int>(nc);
    p.n_out = static_cast<int>(n_out);
    p.off = off;
    p.ni = static_cast<int>(ni);
    p.t_lo = static_cast<int>(t_lo);
    p.T = static_cast<int>(T_s);
    p.span = span;
    p.fill = fill;
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
    const size_t smem = static_cast<size_t>(kStreamStages) * 2 * span * sizeof(A);
    auto kern = C0 ? dwt_syn_stream_kernel<A, LM, 1> : dwt_syn_stream_kernel<A, LM, 0>;
    int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (st != FDWT_OK) return st;
    int occ = 0;
    if ((st = occupancy(reinterpret_cast<const void*>(kern), SNT, smem, &occ)) != FDWT_OK) return st;
    if (occ < 1) return FDWT_ERR_UNSUPPORTED;
    const int64_t grid = std::min<int64_t>(p.ntile, static_cast<int64_t>(occ) * sm_count());
    if (fill == kFillNone) {  // the tiles near the row ends on the tile kernel (same tile size)
      std::vector<Level> one(1, L0);
      st = run_syn_tile_launch<T, LM>(rows, a, one, y, h0, h1, L, off, stream, false,
                                      static_cast<int>(t_lo), static_cast<int>(t_hi));
      if (st != FDWT_OK) return st;
    }
    if ((st = pre_launch(stream)) != FDWT_OK) return st;
    kern<<<static_cast<unsigned>(grid), SNT, smem, stream>>>(p, R);
    return launch_status();
  }
}

// ------------------------------------------------------------------------------ analysis
//
// One-level analysis (a, d) = A(x) of rows whose length is a multiple of 16 bytes, every tile
// of every row on the same persistent, bulk-copy-fed ring: tile t computes the outputs
// [t T, t T + T) from the input positions [2 t T + off - (LM - 1), 2 t T + 2 T + off - 1] of the
// extended signal.  The in-range part arrives by one cp.async.bulk; the few extended positions
// outside [0, n) that the tile's outputs read (at most LM - 1 at each row end) are gathered by
// the threads through the boundary map (ext_index) into the slot before its copy is issued.
// An item is V = 48 bytes / 2 element sizes of consecutive outputs (6 in fp32, 3 in fp64), so
// the windows of consecutive lanes start 48 bytes apart: their 128-bit loads hit distinct bank
// groups in every quarter warp.

template <typename A>
constexpr int ana_stream_v() { return sizeof(A) == 8 ? 3 : 6; }
template <typename A>
constexpr int ana_stream_tile() { return 2 * SNT * ana_stream_v<A>(); }

template <typename A, int LM>
struct AnaStreamParams {
  const A* x;        // (rows, xs) input
  A* ap;             // (rows, as) approximation (a_len = nc or nc + 1: trailing zero)
  A* dp;             // (rows, nc) details
  int* err;          // device error word
  uint32_t dbg_tx;   // test hook: extra expected bytes of global tile 0's copy
  long long tries;   // poll limit of the main mbarrier waits
  int64_t ntile;     // rows * tiles
  int64_t P;         // period of the boundary mode
  int32_t n, nc, a_len, off, mode, tiles, span;
  int32_t xs, as;    // row strides of x and of the approximation (xs a multiple of 16 bytes)
  int32_t n_al;      // n rounded down to 16 bytes: the bulk copies end there
  int32_t T;         // outputs per tile (a multiple of 2 V)
  alignas(16) A taps[2 * LM];  // (h0[j], h1[j]) interleaved
};

// V outputs (a, d) from the window xw[R .. R + 2V + LM - 2) (xw 16-byte aligned): output v is
// sum_j h[j] w[2v + LM - 1 - j], the recursion of ana_compute; taps = (h0[j], h1[j]) pairs.
template <typename A, int LM, int R>
__device__ __forceinline__ void ana_window_item(const A* taps, const A* xw, A* ra, A* rd) {
  constexpr int V = ana_stream_v<A>();
  constexpr int W = 2 * V + LM - 2;
  constexpr int VW = 16 / static_cast<int>(sizeof(A));
  constexpr int NL = (R + W + VW - 1) / VW;
  A w[NL * VW];
#pragma unroll
  for (int k = 0; k < NL; ++k) load16<A>(xw + k * VW, w + k * VW);
  if constexpr (sizeof(A) == 4) {
    unsigned long long acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0ull;
#pragma unroll
    for (int i = W - 1; i >= 0; --i) {
      const unsigned long long xx = pair(w[R + i], w[R + i]);
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const int j = 2 * v + LM - 1 - i;
        if (j >= 0 && j < LM)
          ffma2(acc[v], *reinterpret_cast<const unsigned long long*>(&taps[2 * j]), xx);
      }
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      ra[v] = lo32(acc[v]);
      rd[v] = hi32(acc[v]);
    }
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v) {
      A a = A(0), d = A(0);
#pragma unroll
      for (int j = 0; j < LM; ++j) {
        const A xv = w[R + 2 * v + LM - 1 - j];
        a = fma(taps[2 * j], xv, a);
        d = fma(taps[2 * j + 1], xv, d);
      }
      ra[v] = a;
      rd[v] = d;
    }
  }
}

// Store the first `count` of V values at dst (8-byte stores of pairs when dst is 8-byte aligned).
template <typename A, int V>
__device__ __forceinline__ void store_run(A* dst, const A* v, int count) {
  if constexpr (sizeof(A) == 4 && V % 2 == 0) {
    if (count == V && (reinterpret_cast<uintptr_t>(dst) & 7) == 0) {
#pragma unroll
      for (int k = 0; k < V; k += 2) *reinterpret_cast<float2*>(dst + k) = make_float2(v[k], v[k + 1]);
      return;
    }
  }
#pragma unroll
  for (int k = 0; k < V; ++k)
    if (k < count) dst[k] = v[k];
}

template <typename A, int LM, int R>
__device__ void ana_stream_tiles(const AnaStreamParams<A, LM>& p, A* ring, uint64_t* bar) {
  constexpr int V = ana_stream_v<A>();
  const int T = p.T;
  const int tid = threadIdx.x;
  const int64_t G = gridDim.x;
  const int span = p.span, n = p.n;
  const int pmin = p.off - (LM - 1);       // first extended position an output reads
  const int pmax = 2 * (p.nc - 1) + p.off;  // last
  auto slot = [&](int s) { return ring + static_cast<size_t>(s) * span; };
  auto slot_lo = [&](int t) { return 2 * t * T + pmin - R; };  // a multiple of 16 bytes
  // all threads: the extended positions outside [0, n) that tile g's outputs read, gathered
  // through the boundary map with element-wise cp.async (one commit group per call, so that
  // a thread's group count advances by one per tile)
  auto ext_fill = [&](int64_t g, int s) {
    const int64_t row = g / p.tiles;
    const int xlo = slot_lo(static_cast<int>(g % p.tiles));
    const A* xr = p.x + row * p.xs;
    A* sl = slot(s);
    const int l1 = min(xlo + span, 0), r1 = min(xlo + span, pmax + 1);
    auto one = [&](int q) {
      const int64_t e = ext_index(q, n, p.mode, p.P);
      if (e < 0) sl[q - xlo] = A(0);
      else cp_async(sl + (q - xlo), xr + e, sizeof(A));
    };
    for (int q = max(xlo, pmin) + tid; q < l1; q += SNT) one(q);
    for (int q = max(xlo, p.n_al) + tid; q < r1; q += SNT) one(q);
    cp_async_commit();
  };
  // one thread: the bulk copy of tile g's in-range input into slot s
  auto issue = [&](int64_t g, int s) {
    const int64_t row = g / p.tiles;
    const int xlo = slot_lo(static_cast<int>(g % p.tiles));
    const int lo = max(xlo, 0), hi = min(xlo + span, p.n_al);
    const unsigned bytes = static_cast<unsigned>(max(hi - lo, 0)) * sizeof(A);
    mbar_expect_tx(&bar[s], bytes + (g == 0 ? p.dbg_tx : 0u));
    if (bytes) bulk_g2s(slot(s) + (lo - xlo), p.x + row * p.xs + lo, bytes, &bar[s]);
  };
  // the gathers of tile k form the k-th commit group of every thread; the group of tile k + 1
  // is waited for before the barrier that ends tile k
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
    const bool ok = mbar_wait_bounded(&bar[s], par, p.tries);
    if (ok) {
      const int64_t row = g / p.tiles;
      const int t = static_cast<int>(g % p.tiles);
      A* arow = p.ap + row * p.as;
      A* drow = p.dp + row * p.nc;
      const A* sl = slot(s);
#pragma unroll 1
      for (int it = tid; it < T / V; it += SNT) {
        const int o0 = t * T + V * it;
        if (o0 >= p.nc) break;
        A ra[V], rd[V];
        ana_window_item<A, LM, R>(p.taps, sl + 2 * V * it, ra, rd);
        const int cnt = min(V, p.nc - o0);
        store_run<A, V>(drow + o0, rd, cnt);
        store_run<A, V>(arow + o0, ra, cnt);
      }
      if (t == p.tiles - 1 && tid == 0)
        for (int q = p.nc; q < p.a_len; ++q) arow[q] = A(0);  // transpose of waverec's trim
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
                            static_cast<unsigned>(kj / kStreamStages) & 1u,
                            cleanup_tries(p.tries));
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
__global__ void __launch_bounds__(SNT, 3)
dwt_ana_stream_kernel(const __grid_constant__ AnaStreamParams<A, LM> p, int r) {
  extern __shared__ __align__(16) unsigned char ring_smem[];
  __shared__ __align__(8) uint64_t bar[kStreamStages];
  A* ring = reinterpret_cast<A*>(ring_smem);
  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < kStreamStages; ++s) mbar_init(&bar[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
  }
  __syncthreads();
  if constexpr (sizeof(A) == 4) {
    switch (r) {
      case 0: ana_stream_tiles<A, LM, 0>(p, ring, bar); break;
      case 1: ana_stream_tiles<A, LM, 1>(p, ring, bar); break;
      case 2: ana_stream_tiles<A, LM, 2>(p, ring, bar); break;
      default: ana_stream_tiles<A, LM, 3>(p, ring, bar); break;
    }
  } else {
    if (r == 0) ana_stream_tiles<A, LM, 0>(p, ring, bar);
    else ana_stream_tiles<A, LM, 1>(p, ring, bar);
  }
}

// The analysis of level L0 as the streaming kernel when the shape allows it: element type with
// fp32 / fp64 accumulation, LM <= kStreamMaxLM, input rows at least kStreamMinOut samples long
// and xs apart, xs a multiple of 16 bytes.  Shape-only test (pointers are checked at launch).
template <typename T, int LM>
bool ana_streams(const Level& L0, int64_t xs) {
  using A = typename AccOf<T>::type;
  constexpr int VW = 16 / static_cast<int>(sizeof(A));
  return std::is_same<T, A>::value && LM <= kStreamMaxLM && L0.n_in >= kStreamMinOut &&
         xs % VW == 0 && xs >= L0.n_in && xs <= 0x3fffffffLL && L0.a_len <= L0.n_coef + 1;
}

// Runs the one-level analysis of L0 (x: rows of L0.n_in samples, xs apart; approximation to
// a_out, rows of a_len, as apart; details to L0.detail) on the streaming kernel;
// FDWT_ERR_UNSUPPORTED when it does not apply.
template <typename T, int LM>
int run_ana_stream(int64_t rows, const void* x, const Level& L0, int64_t xs, void* a_out,
                   int64_t as, const double* h0, const double* h1, int L, int off,
                   cudaStream_t stream) {
  using A = typename AccOf<T>::type;
  if constexpr (!std::is_same<T, A>::value || LM > kStreamMaxLM) {
    return FDWT_ERR_UNSUPPORTED;
  } else {
    constexpr int VW = 16 / static_cast<int>(sizeof(A));
    constexpr int V = ana_stream_v<A>();
    if (!ana_streams<T, LM>(L0, xs) || as < L0.a_len || as > 0x3fffffffLL || x == nullptr || a_out == nullptr || L0.detail == nullptr ||
        rows <= 0 || (reinterpret_cast<uintptr_t>(x) & 15) != 0)
      return FDWT_ERR_UNSUPPORTED;
    const int64_t nc = L0.n_coef;
    if (nc < 1) return FDWT_ERR_UNSUPPORTED;
    // tiles of equal size, at most ana_stream_tile outputs (a multiple of 2V)
    const int64_t T_s = cdiv(cdiv(nc, cdiv(nc, ana_stream_tile<A>())), 2 * V) * 2 * V;
    const int pmin = off - (LM - 1);
    const int R = ((pmin % VW) + VW) % VW;
    constexpr int W = 2 * V + LM - 2;
    const int NL = (R + W + VW - 1) / VW;
    const int span = static_cast<int>(2 * T_s - 2 * V + NL * VW);
    const int64_t tiles = cdiv(nc, T_s);
    if (rows * tiles > (1LL << 40)) return FDWT_ERR_UNSUPPORTED;
    AnaStreamParams<A, LM> p{};
    p.x = static_cast<const A*>(x);
    p.ap = static_cast<A*>(a_out);
    p.dp = static_cast<A*>(L0.detail);
    p.err = device_error_flag();
    if (p.err == nullptr) return FDWT_ERR_CUDA;
    {
      const CopyWaitTest wt = copy_wait_test();
      p.dbg_tx = wt.extra_tx;
      p.tries = wt.tries;
    }
    p.ntile = rows * tiles;
    p.P = L0.P;
    p.n = static_cast<int>(L0.n_in);
    p.nc = static_cast<int>(nc);
    p.a_len = static_cast<int>(L0.a_len);
    p.xs = static_cast<int>(xs);
    p.as = static_cast<int>(as);
    p.n_al = static_cast<int>(L0.n_in / VW * VW);
    p.off = off;
    p.mode = L0.mode;
    p.tiles = static_cast<int>(tiles);
    p.span = span;
    p.T = static_cast<int>(T_s);
    for (int j = 0; j < LM; ++j) {
      p.taps[2 * j] = j < L ? static_cast<A>(h0[j]) : A(0);
      p.taps[2 * j + 1] = j < L ? static_cast<A>(h1[j]) : A(0);
    }
    const size_t smem = static_cast<size_t>(kStreamStages) * span * sizeof(A);
    auto kern = dwt_ana_stream_kernel<A, LM>;
    int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
    if (st != FDWT_OK) return st;
    int occ = 0;
    if ((st = occupancy(reinterpret_cast<const void*>(kern), SNT, smem, &occ)) != FDWT_OK) return st;
    if (occ < 1) return FDWT_ERR_UNSUPPORTED;
    const int64_t grid = std::min<int64_t>(p.ntile, static_cast<int64_t>(occ) * sm_count());
    if ((st = pre_launch(stream)) != FDWT_OK) return st;
    kern<<<static_cast<unsigned>(grid), SNT, smem, stream>>>(p, R);
    return launch_status();
  }
}

}  // namespace dwtk
}  // namespace fdwt
