// Backward of the Morlet CWT pyramid for rows too long for the row-resident kernel
// (cwt_bwd.cuh): one launch per octave, coarse to fine, over time tiles.
//
// The chain dL/dx_j = M_j^T dL/dW_j + LP_j^T dL/dx_{j+1} (G_j) is cut at every octave: launch j
// reads G_{j+1} from global memory, adds the adjoint of its own scales and writes G_j (G_0 is
// dL/dx).  G_j lives on [-live_j, n + live_j) and is stored on [-e, n + e) (e the largest live
// extent, zero outside live_j), so the tiles of every launch cover [-e, n + e).  x_j (j >= 1) is
// read from a global pyramid written before by the half-band chain of the forward kernel
// (run_pyramid, the PYR mode).
//
// A tile of launch j owns the positions [t0, t0 + tk).  Its shared windows hold:
//   X  = x_j on [t0 - XH, t0 + tk + XH)      (filter gradient; recomputation of W)
//   gW = dL/dW_s on [t0 - H, t0 + tk + H)    (H = the octave's filter reach half_j 2^j, rounded
//                                             up to 8; zero outside [0, n))
//   Gp = G_{j+1} on [t0 - c_lp 2^j, t0 + tk + c_lp 2^j)
//   Go = G_j on [t0, t0 + tk)
// with XH = H when only the filter gradient reads X, 2H when W is recomputed (the mix and the
// spectral softmax: dL/dW at t0 - H needs W there, which reads x_j down to t0 - 2H).  Every
// owned output is then exact; sums over positions (filter gradient, mix weights, per-channel V)
// take the owned positions inside [0, n) only, into per-(tile, row) partials reduced after the
// last launch.
#pragma once

#include "cwt_bwd.cuh"

namespace fdwt {
namespace cwtk {

template <typename A>
struct OctParams {
  BwdParams<A> b;       // plan, caller arrays, partial arrays (row index tile * rows + row)
  int64_t rows;
  int32_t j;            // octave of this launch
  int32_t ntile, t_len, t_base;  // tiles [t_base + t t_len, +t_len), t < ntile, cover [-e, n + e)
  int32_t e;            // G arrays hold [-e, n + e) per row
  int64_t g_stride;     // n + 2 e
  const A* g_in;        // G_{j+1}, or null (coarsest octave)
  A* g_out;             // G_j, or null: j == 0 writes dL/dx
  int32_t H, XH, R;     // reaches of gW, X, Gp past the owned range
  int32_t x_off, gw_off, gp_off, go_off, tab_off, red_off;  // byte offsets in shared memory
  int32_t gw_len;       // elements of the gW window
};

// dL/dH partial of one scale over the owned positions [lo, hi) (absolute):
// part[c * hcols + center + k] = sum_a gW_c(a) x_j(a - dil k), |k| <= K, zero elsewhere.  Same
// reduction as gradh_scale (runs of RL positions of a phase per lane, 8 taps per warp pass); gW
// is read from its window (origin o, virtual length nv) and counts only inside [lo, hi).
template <typename A, int C>
__device__ void gradh_tile(const Oct& O, int center, const A* X, int xorg, int xlen,
                           const A* gw, int o, int nv, int lo, int hi, A* part) {
  const int dil = O.dil, K = O.half;
  const int lg = __ffs(dil) - 1;
  const int hcols = 2 * center + 1;
  const int nkb = static_cast<int>(cdiv(2 * K + 1, KT));
  const int len = max(hi - lo, 0);
  const int U = static_cast<int>(cdiv(len, dil));
  const int runs = dil * ((U + RL - 1) / RL);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  using V2 = typename Cplx<A>::type;
  for (int c = threadIdx.x; c < C * hcols; c += nthreads()) {
    const int k = c % hcols - center;
    if (k < -K || k > K) part[c] = A(0);
  }
  for (int kb = w; kb < nkb; kb += nwarps()) {
    const int k0 = -K + kb * KT;
    Acc2<A> acc[KT];
#pragma unroll
    for (int i = 0; i < KT; ++i) acc[i].zero();
    for (int r = lane; r < runs; r += 32) {
      const int nn = lo + (r & (dil - 1)) + (r >> lg) * (RL << lg);  // phase + dil RL run
      if (nn >= hi) continue;
      const int base = nn - dil * k0;
      A xw[RL + KT - 1];  // x_j(base + dil (m - 7)); taps past K read clamped cells (discarded)
#pragma unroll
      for (int m = 0; m < RL + KT - 1; ++m) {
        const int i = min(max(base + dil * (m - (KT - 1)) - xorg, 0), xlen - 1);
        xw[m] = X[bix(i)];
      }
#pragma unroll
      for (int t = 0; t < RL; ++t) {
        const int a = nn + dil * t;
        V2 gv = ld_gw<A, C>(gw, nv, a - o);
        if (a >= hi) {
          gv.x = A(0);
          gv.y = A(0);
        }
#pragma unroll
        for (int i = 0; i < KT; ++i) {
          const A xv = xw[t - i + KT - 1];
          acc[i].fmav(gv.x, gv.y, xv, xv);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < KT; ++i) {
      A re = acc[i].re(), im = acc[i].im();
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) {
        re += __shfl_xor_sync(0xffffffffu, re, s);
        if (C == 2) im += __shfl_xor_sync(0xffffffffu, im, s);
      }
      const int k = k0 + i;
      if (lane == 0 && k <= K) {
        part[center + k] = re;
        if (C == 2) part[hcols + center + k] = im;
      }
    }
  }
}

// dL/dW of scale gs on the gW window (virtual positions v in [0, nv), absolute o + v), zero
// outside [0, n).  STORE: the caller's gradient.  MIX / SOFTMAX: W recomputed from the X window
// (wx) and the consumer's derivative applied; the parameter sums and per-position V gradients
// take the owned positions [lo, hi) only.
template <typename A, int EPI, int C, bool SYM>
__device__ void make_gw_tile(const BwdParams<A>& p, const Oct& O, int gs, const A* X,
                             const Win& wx, const A* tab, A* gw, int64_t row, int o, int nv,
                             int lo, int hi, A& sa, A& sb) {
  const FwdParams<A>& f = p.f;
  const int n = static_cast<int>(f.n);
  if (EPI == EPI_STORE) {
    const A* g = p.g + (row * f.n_scales + gs) * f.n * C;
    for (int v = threadIdx.x; v < nv; v += nthreads()) {
      const int a = o + v;
      A re = A(0), im = A(0);
      if (a >= 0 && a < n) {
        re = g[static_cast<int64_t>(a) * C];
        if (C == 2) im = g[static_cast<int64_t>(a) * C + 1];
      }
      st_gw<A, C>(gw, v, re, im);
    }
    return;
  }
  const int dil = O.dil;
  const int runs = static_cast<int>(cdiv(cdiv(nv, dil), P));
  const int items = dil * runs;
  const A* gy = p.g + row * f.n;
  A av = A(0), bv = A(0), vconst = A(0);
  int64_t grp = 0;
  if (EPI == EPI_MIX) {
    const int64_t d = row % f.dim;
    av = static_cast<const A*>(f.a)[d * f.n_scales + gs];
    bv = static_cast<const A*>(f.b)[d * f.n_scales + gs];
  } else {
    grp = row / f.dim;
    if (!f.v_pos) vconst = static_cast<const A*>(f.a)[(row % f.dim) * f.n_scales + gs];
  }
  const int lg = __ffs(dil) - 1;  // dil = 2^lg
  for (int it = threadIdx.x; it < items; it += nthreads()) {
    const int phi = it & (dil - 1), u0 = (it >> lg) * P;
    if (phi >= nv) continue;
    const int base = phi + dil * u0;
    Acc2<A> acc[P];
    conv_one<A, SYM>(wx, X, tab, O.half, dil, base, acc);
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int v = base + dil * i;
      if (v >= nv) continue;
      const int a = o + v;
      if (a < 0 || a >= n) {
        st_gw<A, C>(gw, v, A(0), A(0));
        continue;
      }
      const bool own = a >= lo && a < hi;
      const A re = acc[i].re(), im = C == 2 ? acc[i].im() : A(0);
      A vv = vconst;
      A* vpos = nullptr;
      if (EPI == EPI_SOFTMAX && f.v_pos) {
        const int64_t vq = (grp * f.n_scales + gs) * f.n + a;
        vv = static_cast<const A*>(f.a)[vq];
        vpos = p.v_part + vq;
      }
      A gre, gim;
      consumer_grad<A, EPI, C>(p, re, im, gy[a], av, bv, vv, row * f.n + a, vpos, own, sa, sb,
                               gre, gim);
      st_gw<A, C>(gw, v, gre, gim);
    }
  }
}

template <typename A, int EPI, int C>
__device__ void octave_tile_scales(const OctParams<A>& q, const Oct& O, const A* X, A* gw, A* Go,
                                   const A* tab, const int* sym, const int* klast, A* red,
                                   int64_t row, int tile, int t0, int tk) {
  const BwdParams<A>& p = q.b;
  const FwdParams<A>& f = p.f;
  const int n = static_cast<int>(f.n);
  const int o = t0 - q.H;               // origin of the gW window
  const int nv = tk + 2 * q.H;          // its length
  const Win wx{nv, q.XH - q.H};         // X seen from the gW window
  const Win wg{nv, -q.H};               // Go seen from the gW window
  const int lo = max(t0, 0), hi = min(t0 + tk, n);
  const int64_t prow = static_cast<int64_t>(tile) * q.rows + row;  // partial row
  const int K1 = O.half + 1;
  const int hcols = 2 * f.center + 1;
  for (int s = 0; s < O.count; ++s) {
    const A* ts = tab + 4 * K1 * s;
    const bool sy = sym[s] != 0;
    const int ks = klast[s];
    const int gs = f.order[O.begin + s];
    A sa = A(0), sb = A(0);
    if (sy) make_gw_tile<A, EPI, C, true>(p, O, gs, X, wx, ts, gw, row, o, nv, lo, hi, sa, sb);
    else make_gw_tile<A, EPI, C, false>(p, O, gs, X, wx, ts, gw, row, o, nv, lo, hi, sa, sb);
    if (EPI == EPI_MIX) {
      const A ta = block_sum(sa, red);
      const A tb = block_sum(sb, red);
      if (threadIdx.x == 0) {
        p.a_part[prow * f.n_scales + gs] = ta;
        p.b_part[prow * f.n_scales + gs] = tb;
      }
    } else if (EPI == EPI_SOFTMAX && !f.v_pos) {
      const A ta = block_sum(sa, red);
      if (threadIdx.x == 0) p.v_part[prow * f.n_scales + gs] = ta;
    }
    __syncthreads();
    if (p.need_gx) {  // the adjoint into the owned positions within the scale's reach
      const int reach = min(O.live, ks * O.dil);
      const int pa = max(t0, -reach) - o, pb = min(t0 + tk, n + reach) - o;
      if (pa < pb) {
        if (sy) adjoint_scale<A, C, true>(wg, O, ts, gw, Go, pa, pb, ks);
        else adjoint_scale<A, C, false>(wg, O, ts, gw, Go, pa, pb, ks);
      }
    }
    if (p.gh_part)
      gradh_tile<A, C>(O, f.center, X, t0 - q.XH, tk + 2 * q.XH, gw, o, nv, lo, hi,
                       p.gh_part + (prow * f.n_scales + gs) * C * hcols);
    __syncthreads();
  }
}

template <typename A, int EPI>
__global__ void __launch_bounds__(NT) cwt_octave_bwd_kernel(const __grid_constant__ OctParams<A> q) {
  extern __shared__ __align__(16) unsigned char smem[];
  const BwdParams<A>& p = q.b;
  const FwdParams<A>& f = p.f;
  const Oct& O = f.oct[q.j];
  A* X = reinterpret_cast<A*>(smem + q.x_off);
  A* gw = reinterpret_cast<A*>(smem + q.gw_off);
  A* Gp = reinterpret_cast<A*>(smem + q.gp_off);
  A* Go = reinterpret_cast<A*>(smem + q.go_off);
  A* tab = reinterpret_cast<A*>(smem + q.tab_off);
  A* red = reinterpret_cast<A*>(smem + q.red_off);
  __shared__ int sym[kMaxScales];
  __shared__ int klast[kMaxScales];
  const int64_t row = blockIdx.x / q.ntile;
  const int tile = static_cast<int>(blockIdx.x - row * q.ntile);
  const int n = static_cast<int>(f.n);
  const int t0 = q.t_base + tile * q.t_len;
  const int tk = q.t_len;  // the last tile may pass n + e: those positions are outside every
                           // live extent (zero) and are not stored
  const int live = O.live;
  const int dil = O.dil;
  const int tid = threadIdx.x;
  const bool has_in = p.need_gx && q.g_in != nullptr;

  if (p.need_x && O.count > 0) {  // X = x_j, zero outside [-live_j, n + live_j)
    const RowRef<const A> src =
        q.j == 0 ? row_ref(static_cast<const A*>(f.x), f, row)
                 : RowRef<const A>{p.pyr + row * p.pyr_len + p.pyr_off[q.j] + live, 1};
    for (int i = tid; i < tk + 2 * q.XH; i += nthreads()) {
      const int a = t0 - q.XH + i;
      X[bix(i)] = (a >= -live && a < n + live) ? src[a] : A(0);
    }
  }
  if (has_in) {
    const A* gi = q.g_in + row * q.g_stride + q.e;
    for (int i = tid; i < tk + 2 * q.R; i += nthreads()) {
      const int a = t0 - q.R + i;
      Gp[bix(i)] = (a >= -q.e && a < n + q.e) ? gi[a] : A(0);
    }
  }
  for (int i = tid; i < q.gw_len; i += nthreads()) gw[i] = A(0);  // the window's end cells stay zero
  __syncthreads();
  if (p.need_gx) {  // Go = LP_j^T G_{j+1} on the owned positions inside live_j
    for (int i = tid; i < tk; i += nthreads()) {
      const int a = t0 + i;
      A v = A(0);
      if (has_in && a >= -live && a < n + live) {
        const int c = i + q.R;
        v = f.lpp[0] * Gp[bix(c)];
        for (int k = 0; k < f.n_lp; ++k) {
          const int t = f.lp_t[k];
          v = fma(f.lp_p[k], Gp[bix(c + dil * t)], v);
          v = fma(f.lp_m[k], Gp[bix(c - dil * t)], v);
        }
      }
      Go[bix(i)] = v;
    }
  }
  if (O.count > 0) {
    build_octave_taps<A>(f, O, tab, sym, klast);  // ends with a barrier
    if (f.channels == 2)
      octave_tile_scales<A, EPI, 2>(q, O, X, gw, Go, tab, sym, klast, red, row, tile, t0, tk);
    else
      octave_tile_scales<A, EPI, 1>(q, O, X, gw, Go, tab, sym, klast, red, row, tile, t0, tk);
  } else {
    __syncthreads();
  }
  if (p.need_gx) {
    if (q.g_out) {
      A* go = q.g_out + row * q.g_stride + q.e;
      for (int i = tid; i < tk; i += nthreads()) {
        const int a = t0 + i;
        if (a < n + q.e) go[a] = Go[bix(i)];
      }
    } else {
      const RowRef<A> gx = row_ref(p.gx, f, row);
      for (int i = tid; i < tk; i += nthreads()) {
        const int a = t0 + i;
        if (a >= 0 && a < n) gx[a] = Go[bix(i)];
      }
    }
  }
}

// ------------------------------------------------------------------------------ host

// Per-octave reaches and shared layout of one octave launch for tiles of t_len positions;
// returns the bytes (0: does not fit the budget).
template <typename A, int EPI>
size_t oct_layout(OctParams<A>& q, const fdwt_morlet_plan* pl, int j, int t_len, bool need_x,
                  bool need_gx, size_t budget) {
  const int dil = 1 << j;
  const int cnt = pl->oct_count[j];
  q.H = cnt > 0 ? static_cast<int>((static_cast<int64_t>(pl->oct_half[j]) * dil + 7) / 8 * 8) : 0;
  q.XH = (need_x && cnt > 0) ? (EPI == EPI_STORE ? q.H : 2 * q.H) : 0;
  q.R = (need_gx && j + 1 < pl->n_octaves) ? pl->c_lp * dil : 0;
  const int64_t nv = static_cast<int64_t>(t_len) + 2 * q.H;
  if (nv + 2 * static_cast<int64_t>(q.XH) > 0x3fffffffLL) return 0;
  const int C = pl->channels;
  size_t off = 0;
  auto region = [&](size_t elems) {
    const size_t at = off;
    off = (off + elems * sizeof(A) + 15) / 16 * 16;
    return static_cast<int32_t>(at);
  };
  q.x_off = region(q.XH > 0 || (need_x && cnt > 0)
                       ? static_cast<size_t>((t_len + 2 * q.XH)) + 8 : 0);
  q.gw_len = cnt > 0 ? static_cast<int32_t>(C * (nv + 2) + 8) : 0;
  q.gw_off = region(q.gw_len);
  q.gp_off = region(q.R > 0 ? static_cast<size_t>((t_len + 2 * q.R)) + 8 : 0);
  q.go_off = region(need_gx ? static_cast<size_t>((t_len)) + 8 : 0);
  q.tab_off = region(4 * static_cast<size_t>(cnt) * (pl->oct_half[j] + 1));
  q.red_off = region(NW_MAX);
  const size_t smem = off + 16;
  return smem > budget ? 0 : smem;
}

// Backward over time tiles (see the notes at the top of this file).  Same contract as
// run_backward, whose whole-row kernel does not fit these rows (or a test forced tiles).
template <typename A, int EPI>
int run_backward_tiled(int64_t rows, int64_t n, const void* x, const void* h,
                       const fdwt_morlet_plan* pl, const Geometry& geo, const void* a,
                       const void* b, int64_t dim, int v_pos, double inv_tau, const void* g,
                       const void* sm_m, const void* sm_l, const void* sm_out, void* gx, void* gh,
                       void* ga, void* gb, void* gv, bool need_h, void* ws, size_t ws_bytes,
                       cudaStream_t stream, size_t* ws_needed, int tok) {
  const int J = pl->n_octaves;
  const bool need_gx = ws_needed ? true : gx != nullptr;
  const bool need_x = need_h || EPI != EPI_STORE;
  int e = 0;
  for (int j = 0; j < J; ++j) e = std::max(e, geo.live[j]);
  const int64_t ext_len = n + 2 * static_cast<int64_t>(e);
  // one tile length for every octave launch (the partial rows are tile * rows + row)
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 2048;
  OctParams<A> q{};
  auto fits = [&](int tl, size_t cap) {
    for (int j = 0; j < J; ++j)
      if (!oct_layout<A, EPI>(q, pl, j, tl, need_x, need_gx, cap)) return false;
    return true;
  };
  int t_len = 0;
  const int forced = cwt_tile_test();
  if (forced > 0) {
    t_len = fits(forced, budget) ? forced : 0;
  } else {
    const size_t two_per_sm = std::min(budget, static_cast<size_t>(113) << 10);
    for (const size_t cap : {two_per_sm, budget}) {
      for (int tl = 1 << 14; tl >= 256 && !t_len; tl >>= 1)
        if (fits(std::min<int64_t>(tl, ext_len), cap)) t_len = static_cast<int>(std::min<int64_t>(tl, ext_len));
      if (t_len) break;
    }
  }
  if (t_len == 0) return FDWT_ERR_UNSUPPORTED;
  const int64_t ntile = cdiv(ext_len, t_len);
  if (rows * ntile > 0x7fffffffLL) return FDWT_ERR_UNSUPPORTED;
  const int64_t prows = rows * ntile;  // partial rows
  const int64_t S = pl->n_scales;
  const int64_t hcols = 2 * static_cast<int64_t>(pl->center) + 1;
  const int64_t ghcols = S * pl->channels * hcols;
  if ((EPI == EPI_MIX || (EPI == EPI_SOFTMAX && !v_pos)) && ntile > 1 && rows % dim != 0)
    return FDWT_ERR_UNSUPPORTED;  // the partial rows keep the residue row % dim only then

  // workspace: pyramid, two G arrays, partials, reduction scratch
  BwdLayout lay = bwd_layout<A>(EPI, rows, n, pl, geo, need_h, dim, v_pos != 0);  // pyramid
  const size_t g_bytes = (need_gx && J > 1)
      ? align256(static_cast<size_t>(rows) * ext_len * sizeof(A)) : 0;
  const size_t gh_bytes = need_h ? align256(static_cast<size_t>(prows) * ghcols * sizeof(A)) : 0;
  const size_t pab = EPI == EPI_MIX ? align256(static_cast<size_t>(prows) * S * sizeof(A)) : 0;
  const size_t pv = (EPI == EPI_SOFTMAX && !v_pos)
      ? align256(static_cast<size_t>(prows) * S * sizeof(A)) : 0;
  size_t tmp = 0;
  if (need_h) tmp = std::max(tmp, reduce_tmp_elems(prows, ghcols, 1));
  if (EPI == EPI_MIX) tmp = std::max(tmp, reduce_tmp_elems(prows, S, dim));
  if (EPI == EPI_SOFTMAX && !v_pos) tmp = std::max(tmp, reduce_tmp_elems(prows, S, dim));
  const size_t tmp_bytes = align256(tmp * sizeof(A));
  const size_t total = lay.pyr + 2 * g_bytes + gh_bytes + 2 * pab + pv + tmp_bytes;
  if (ws_needed) {
    *ws_needed = total;
    return FDWT_OK;
  }
  if (total > 0 && (ws == nullptr || ws_bytes < total)) return FDWT_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  A* pyr = reinterpret_cast<A*>(w);
  A* gbuf[2] = {reinterpret_cast<A*>(w + lay.pyr), reinterpret_cast<A*>(w + lay.pyr + g_bytes)};
  A* ghp = reinterpret_cast<A*>(w + lay.pyr + 2 * g_bytes);
  A* pa = reinterpret_cast<A*>(w + lay.pyr + 2 * g_bytes + gh_bytes);
  A* pb = reinterpret_cast<A*>(w + lay.pyr + 2 * g_bytes + gh_bytes + pab);
  A* pvp = reinterpret_cast<A*>(w + lay.pyr + 2 * g_bytes + gh_bytes + 2 * pab);
  A* tmpp = reinterpret_cast<A*>(w + lay.pyr + 2 * g_bytes + gh_bytes + 2 * pab + pv);

  int st;
  if (need_x && J > 1 && lay.pyr_len > 0 &&
      (st = run_pyramid<A>(rows, n, x, pl, geo, pyr, lay.pyr_len, lay.pyr_off, stream, tok,
                           dim)) != FDWT_OK)
    return st;

  BwdParams<A>& p = q.b;
  fill_common(p.f, pl, geo, n);
  p.f.rows = rows;
  p.f.x = x;
  p.f.h = h;
  p.f.a = a;
  p.f.b = b;
  p.f.dim = dim;
  p.f.v_pos = v_pos;
  p.f.inv_tau = static_cast<A>(inv_tau);
  p.f.tok = tok;
  p.g = static_cast<const A*>(g);
  p.sm_m = static_cast<const A*>(sm_m);
  p.sm_l = static_cast<const A*>(sm_l);
  p.sm_out = static_cast<const A*>(sm_out);
  p.gx = static_cast<A*>(gx);
  p.gh_part = gh ? ghp : nullptr;
  p.a_part = pa;
  p.b_part = pb;
  p.v_part = EPI == EPI_SOFTMAX ? (v_pos ? static_cast<A*>(gv) : pvp) : nullptr;
  p.pyr = lay.pyr_len > 0 ? pyr : nullptr;
  p.pyr_len = lay.pyr_len;
  for (int j = 0; j < kMaxOct; ++j) p.pyr_off[j] = lay.pyr_off[j];
  p.need_gx = gx != nullptr;
  p.need_x = need_x ? 1 : 0;
  q.rows = rows;
  q.ntile = static_cast<int32_t>(ntile);
  q.t_len = t_len;
  q.t_base = -e;
  q.e = e;
  q.g_stride = ext_len;
  auto kern = cwt_octave_bwd_kernel<A, EPI>;
  if ((st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern))) != FDWT_OK) return st;
  for (int j = J - 1; j >= 0; --j) {
    q.j = j;
    q.g_in = (p.need_gx && j + 1 < J) ? gbuf[(j + 1) & 1] : nullptr;
    q.g_out = (p.need_gx && j > 0) ? gbuf[j & 1] : nullptr;
    if (!p.need_gx && pl->oct_count[j] == 0) continue;
    const size_t smem = oct_layout<A, EPI>(q, pl, j, t_len, need_x, p.need_gx != 0, budget);
    if (!smem) return FDWT_ERR_UNSUPPORTED;
    if ((st = pre_launch(stream)) != FDWT_OK) return st;
    kern<<<static_cast<unsigned>(rows * ntile), NT, smem, stream>>>(q);
    if ((st = launch_status()) != FDWT_OK) return st;
  }
  if (gh && (st = reduce_rows<A>(ghp, prows, ghcols, 1, static_cast<A*>(gh), tmpp, stream)) != FDWT_OK)
    return st;
  if (EPI == EPI_MIX) {
    if (ga && (st = reduce_rows<A>(pa, prows, S, dim, static_cast<A*>(ga), tmpp, stream)) != FDWT_OK)
      return st;
    if (gb && (st = reduce_rows<A>(pb, prows, S, dim, static_cast<A*>(gb), tmpp, stream)) != FDWT_OK)
      return st;
  }
  if (EPI == EPI_SOFTMAX && !v_pos && gv &&
      (st = reduce_rows<A>(pvp, prows, S, dim, static_cast<A*>(gv), tmpp, stream)) != FDWT_OK)
    return st;
  return FDWT_OK;
}

}  // namespace cwtk
}  // namespace fdwt
