// Backward of the Morlet CWT pyramid for sm_100a: the adjoint of the transform (dL/dx), the
// filter gradient (dL/dH) and the fused epilogues of the two scalogram consumers (mix and
// spectral softmax), which recompute W instead of storing it.  Included by cwt.cu after
// cwt_impl.cuh.
//
// One CTA owns one row.  The forward pyramid is x_{j+1} = LP_j x_j and W_j = M_j x_j, so
//   dL/dx_j = M_j^T dL/dW_j + LP_j^T dL/dx_{j+1},
// a chain that runs from the coarsest octave to the finest (fdwt/cwt.py:248-281), while the
// filter gradient of octave j needs x_j, which is built from the finest octave up.  The kernel
// therefore runs two passes over a row:
//   1. fine -> coarse: rebuild x_1 .. x_{J-1} (the half-band chain of the forward) and store
//      each on its live extent in a per-row global scratch (only when a pass-2 consumer needs
//      x_j: the filter gradient, or the recomputation of W for mix / softmax);
//   2. coarse -> fine: G_j = LP_j^T G_{j+1}; then, scale by scale, stage dL/dW_s in shared
//      memory (read from the caller, or formed from the recomputed W_s and the epilogue's
//      saved state), add M_s^T dL/dW_s into G_j, and reduce dL/dH_s = sum_n dL/dW_s(n) x_j(n-dk)
//      into a per-row partial.  dL/dx = G_0.
// x_j is zero outside [-live_j, n + live_j) (live_j as in the forward), and so is any gradient
// that can reach x_0 through it: every shared buffer covers [-E, n + E) with E = max live + 1,
// reads are clamped into that range, and the two end cells are always zero.
//
// Reductions over rows (dL/dH, the mix weights, per-channel V) are written as per-row partials
// and summed by reduce_rows_kernel in a fixed order, so results are deterministic.  The
// per-position V gradient of the spectral softmax (V of shape (G, S, n), shared by the nch rows
// of a group) is accumulated with atomic adds.
#pragma once

#include "cwt_impl.cuh"

namespace fdwt {
namespace cwtk {

// Threads of a backward CTA: NT, or NTB_MAX when the row's buffers leave room for one CTA per
// SM only (more warps to cover the latencies of that CTA).  Device code reads the launched
// size (nthreads(), nwarps()).
constexpr int NTB_MAX = 512;
constexpr int NW_MAX = NTB_MAX / 32;
__device__ __forceinline__ int nthreads() { return static_cast<int>(blockDim.x); }
__device__ __forceinline__ int nwarps() { return static_cast<int>(blockDim.x) >> 5; }
constexpr int KT = 8;        // taps per thread in the filter-gradient reduction
constexpr int RL = 7;        // positions per lane run of the filter-gradient reduction

// The backward's shared buffers are linear (position q of a buffer reaching e past the row at
// index q + e).  Work items of P (7) outputs and filter-gradient runs of RL (7) positions are odd
// in length, so the 32 lanes of a warp, which start P 2^j (or RL 2^j) apart, read distinct banks
// at every power-of-two dilation 2^j.
__host__ __device__ __forceinline__ int bix(int e) { return e; }

template <typename A>
struct BwdParams {
  FwdParams<A> f;     // plan, filters f.h, input f.x, MIX a/b or SOFTMAX V in f.a/f.b, f.dim,
                      // f.v_pos, f.inv_tau; f.ext = E (buffer reach), f.buf_len
  const A* g;         // STORE: dL/dW (rows, S, n, C); MIX: dL/dy (rows, n); SOFTMAX: dL/dout
  const A* sm_m;      // SOFTMAX saved state (rows, n): running max, denominator, output
  const A* sm_l;
  const A* sm_out;
  A* gx;              // (rows, n) or null
  A* gh_part;         // (rows, S*C*hcols) per-row filter gradient or null
  A* a_part;          // MIX: (rows, S) partials of dL/da and dL/db
  A* b_part;
  A* v_part;          // SOFTMAX: per-channel V: (rows, S) partials; per-position V: dL/dV (G, S, n)
  A* pyr;             // (rows, pyr_len) pyramid scratch or null
  int64_t pyr_len;
  int32_t pyr_off[kMaxOct];  // start of x_j in a row's scratch (-1: not stored)
  int32_t need_gx;    // build G (dL/dx) at all
  int32_t need_x;     // pass 2 reads x_j (filter gradient, or recomputation of W)
  int32_t gw_len;     // elements of the dL/dW buffer
  int32_t gw_off, tab_off, red_off;  // byte offsets of the dL/dW buffer, tap table, reduce slots
  int32_t pipe;       // MIX / SOFTMAX: scales pipelined over two dL/dW buffers (octave_pass)
};

template <typename A>
struct Cplx;
template <>
struct Cplx<float> {
  using type = float2;
};
template <>
struct Cplx<double> {
  using type = double2;
};

// ------------------------------------------------------------------------------ buffers

// A shared buffer holding positions [-ext, n + ext) of a row (or of a tile's window): position
// q at index q + ext.  Reads through ldE are clamped into that range.
struct Win {
  int n, ext;
};
template <typename A>
__device__ __forceinline__ Win win(const FwdParams<A>& f) {
  return Win{static_cast<int>(f.n), f.ext};
}
__device__ __forceinline__ int clampE(const Win& w, int pos) {
  return min(max(pos, -w.ext), w.n + w.ext - 1);
}
template <typename A>
__device__ __forceinline__ A ldE(const Win& w, const A* buf, int pos) {
  return buf[bix(clampE(w, pos) + w.ext)];
}
template <typename A>
__device__ __forceinline__ A& atE(const Win& w, A* buf, int pos) {
  return buf[bix(pos + w.ext)];
}
template <typename A>
__device__ __forceinline__ A ldE(const FwdParams<A>& f, const A* buf, int pos) {
  return ldE(win(f), buf, pos);
}
template <typename A>
__device__ __forceinline__ A& atE(const FwdParams<A>& f, A* buf, int pos) {
  return atE(win(f), buf, pos);
}

// dL/dW buffer: positions [-1, n] (the two ends stay zero), complex values interleaved.
template <typename A, int C>
__device__ __forceinline__ typename Cplx<A>::type ld_gw(const A* gw, int n, int pos) {
  const int q = bix(min(max(pos, -1), n) + 1);
  typename Cplx<A>::type v;
  if (C == 2) {
    v = *reinterpret_cast<const typename Cplx<A>::type*>(gw + 2 * q);
  } else {
    v.x = gw[q];
    v.y = A(0);
  }
  return v;
}
// The same without the clamp, for positions known to lie in [-1, n].
template <typename A, int C>
__device__ __forceinline__ typename Cplx<A>::type ld_gw_in(const A* gw, int pos) {
  const int q = bix(pos + 1);
  typename Cplx<A>::type v;
  if (C == 2) {
    v = *reinterpret_cast<const typename Cplx<A>::type*>(gw + 2 * q);
  } else {
    v.x = gw[q];
    v.y = A(0);
  }
  return v;
}
template <typename A, int C, bool CLAMP>
__device__ __forceinline__ typename Cplx<A>::type ld_gw_sel(const A* gw, int n, int pos) {
  return CLAMP ? ld_gw<A, C>(gw, n, pos) : ld_gw_in<A, C>(gw, pos);
}
template <typename A, bool CLAMP>
__device__ __forceinline__ A ldE_sel(const FwdParams<A>& f, const A* buf, int pos) {
  return CLAMP ? ldE(f, buf, pos) : buf[bix(pos + f.ext)];
}

template <typename A, int C>
__device__ __forceinline__ void st_gw(A* gw, int pos, A re, A im) {
  const int q = bix(pos + 1);
  if (C == 2) {
    gw[2 * q] = re;
    gw[2 * q + 1] = im;
  } else {
    gw[q] = re;
  }
}

// Deterministic CTA sum of one value per thread (all threads must call it).
template <typename A>
__device__ __forceinline__ A block_sum(A v, A* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  A s = A(0);
  if (threadIdx.x == 0)
    for (int i = 0; i < nwarps(); ++i) s += red[i];
  return s;  // valid in thread 0
}

// Folded taps of every scale of an octave (k = 0..K), as in the forward's coefficient table:
// tab[(s * (K + 1) + k) * 4 + c]; sym[s] = 1 when the scale's antisymmetric-real /
// symmetric-imaginary halves are all zero (exactly symmetric filter); klast[s] = the last tap k
// of the scale with a nonzero coefficient (the octave's table spans its widest filter; past
// klast[s] the scale's taps are zero, so its adjoint stops there).  Ends with a barrier.
template <typename A>
__device__ void build_octave_taps(const FwdParams<A>& f, const Oct& O, A* tab, int* sym,
                                  int* klast) {
  const int K1 = O.half + 1;
  for (int s = threadIdx.x; s < O.count; s += nthreads()) {
    sym[s] = 1;
    klast[s] = 0;
  }
  __syncthreads();
  for (int w = threadIdx.x; w < O.count * K1; w += nthreads()) {
    const int s = w / K1, k = w - s * K1;
    A t[4];
    fold_coef<A>(f, O, s, k, t);
    A* d = tab + 4 * w;
    d[0] = t[0];
    d[1] = t[1];
    d[2] = t[2];
    d[3] = t[3];
    if (t[2] != A(0) || t[3] != A(0)) sym[s] = 0;
    if (k > 0 && (t[0] != A(0) || t[1] != A(0) || t[2] != A(0) || t[3] != A(0)))
      atomicMax(&klast[s], k);
  }
  __syncthreads();
}

// dL/dW of scale gs of the row (caller's gradient, (rows, S, n, C)) into a dL/dW buffer,
// asynchronously (cp.async; the caller commits and waits).
template <typename A, int C>
__device__ __forceinline__ void stage_gw(const BwdParams<A>& p, int gs, int64_t row, A* gw) {
  const int n = static_cast<int>(p.f.n);
  const A* g = p.g + (row * p.f.n_scales + gs) * p.f.n * C;
  constexpr int bytes = static_cast<int>(sizeof(A)) * C;
  for (int q = threadIdx.x; q < n; q += nthreads()) {
    A* d = C == 2 ? gw + 2 * bix(q + 1) : gw + bix(q + 1);
    const unsigned sa = static_cast<unsigned>(__cvta_generic_to_shared(d));
    const A* src = g + static_cast<int64_t>(q) * C;
    if (bytes == 16)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 16;\n" ::"r"(sa), "l"(src) : "memory");
    else if (bytes == 8)
      asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(sa), "l"(src) : "memory");
    else
      asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(sa), "l"(src) : "memory");
  }
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

// ------------------------------------------------------------------------------ pyramid

// x_{j+1} = LP_j x_j on the whole buffer (zero outside live_{j+1}), reads clamped.
template <typename A>
__device__ void bwd_lowpass(const FwdParams<A>& f, const A* cur, A* nxt, int dil, int live) {
  const int n = static_cast<int>(f.n);
  for (int q = static_cast<int>(threadIdx.x) - f.ext; q < n + f.ext; q += nthreads()) {
    A v = A(0);
    if (q >= -live && q < n + live) {
      v = f.lpp[0] * ldE(f, cur, q);
      for (int i = 0; i < f.n_lp; ++i) {
        const int t = f.lp_t[i];
        v = fma(f.lp_p[i], ldE(f, cur, q - dil * t), v);
        v = fma(f.lp_m[i], ldE(f, cur, q + dil * t), v);
      }
    }
    atE(f, nxt, q) = v;
  }
}

// G_j = LP_j^T G_{j+1} on the whole buffer (zero outside live_j):
//   G_j(p) = lpp[0] G(p) + sum_t lpp[t] G(p + dil t) + lpm[t] G(p - dil t).
template <typename A>
__device__ void bwd_lowpass_adjoint(const FwdParams<A>& f, const A* src, A* dst, int dil,
                                    int live) {
  const int n = static_cast<int>(f.n);
  for (int q = static_cast<int>(threadIdx.x) - f.ext; q < n + f.ext; q += nthreads()) {
    A v = A(0);
    if (q >= -live && q < n + live) {
      v = f.lpp[0] * ldE(f, src, q);
      for (int i = 0; i < f.n_lp; ++i) {
        const int t = f.lp_t[i];
        v = fma(f.lp_p[i], ldE(f, src, q + dil * t), v);
        v = fma(f.lp_m[i], ldE(f, src, q - dil * t), v);
      }
    }
    atE(f, dst, q) = v;
  }
}

// ------------------------------------------------------------------------------ per scale

// (re, im) of one scale at the P outputs n_i = base + dil i, windows read from X: clamped
// (CLAMP) or, for items whose windows lie inside the buffer, straight.
template <typename A, bool SYM, bool CLAMP = true>
__device__ __forceinline__ void conv_one(const Win& f, const A* X, const A* tab, int K,
                                         int dil, int base, Acc2<A> (&acc)[P]) {
  auto ld = [&](int pos) { return CLAMP ? ldE(f, X, pos) : X[bix(pos + f.ext)]; };
  A L[P], R[P];
#pragma unroll
  for (int i = 0; i < P; ++i) L[i] = R[i] = ld(base + dil * i);
  {
    alignas(16) A t0[2] = {tab[0], tab[3]};
#pragma unroll
    for (int i = 0; i < P; ++i) {
      acc[i].zero();
      acc[i].fma(t0, L[i], L[i]);
    }
  }
  int pl = base - dil, pr = base + dil * P;
#pragma unroll 8
  for (int k = 1; k <= K; ++k, pl -= dil, pr += dil) {
#pragma unroll
    for (int i = P - 1; i > 0; --i) L[i] = L[i - 1];
#pragma unroll
    for (int i = 0; i < P - 1; ++i) R[i] = R[i + 1];
    L[0] = ld(pl);
    R[P - 1] = ld(pr);
    alignas(16) A t[4] = {tab[4 * k], tab[4 * k + 1], tab[4 * k + 2], tab[4 * k + 3]};
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const A sum = L[i] + R[i], dif = L[i] - R[i];
      acc[i].fma(t, sum, dif);
      if (!SYM) acc[i].fma(t + 2, dif, sum);
    }
  }
}

// Tap loop of one adjoint item: acc_i += sum_k (taps of k) . (R_i(k) +- conj L_i(k)), where
// L_i(k) = gW(p_i - dk), R_i(k) = gW(p_i + dk).  In fp32 the complex sum and difference are one
// packed FMA each: R + conj(L) = L * (1, -1) + R and R - conj(L) = L * (-1, 1) + R.
template <typename A, int C, bool SYM, bool CLAMP>
__device__ __forceinline__ void adjoint_taps(const A* tab, const A* gw, int n, int K, int dil,
                                             int base, typename Cplx<A>::type (&L)[P],
                                             typename Cplx<A>::type (&R)[P], Acc2<A> (&acc)[P]) {
  int pl = base - dil, pr = base + dil * P;
#pragma unroll 8
  for (int k = 1; k <= K; ++k, pl -= dil, pr += dil) {
#pragma unroll
    for (int i = P - 1; i > 0; --i) L[i] = L[i - 1];
#pragma unroll
    for (int i = 0; i < P - 1; ++i) R[i] = R[i + 1];
    L[0] = ld_gw_sel<A, C, CLAMP>(gw, n, pl);
    R[P - 1] = ld_gw_sel<A, C, CLAMP>(gw, n, pr);
    const A t[4] = {tab[4 * k], tab[4 * k + 1], tab[4 * k + 2], tab[4 * k + 3]};
    if constexpr (std::is_same<A, float>::value) {
      const unsigned long long pm = pk(1.0f, -1.0f), mp = pk(-1.0f, 1.0f);
      const unsigned long long t01 = pk(t[0], t[1]), t23 = pk(t[2], t[3]);
#pragma unroll
      for (int i = 0; i < P; ++i) {
        const unsigned long long l = pk(L[i].x, L[i].y);
        unsigned long long sd = pk(R[i].x, R[i].y);
        ffma2(sd, l, pm);  // (Rre + Lre, Rim - Lim)
        ffma2(acc[i].v, t01, sd);
        if (!SYM) {
          unsigned long long ds = pk(R[i].x, R[i].y);
          ffma2(ds, l, mp);  // (Rre - Lre, Rim + Lim)
          ffma2(acc[i].v, t23, ds);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < P; ++i) {
        acc[i].fmav(t[0], t[1], R[i].x + L[i].x, R[i].y - L[i].y);
        if (!SYM) acc[i].fmav(t[2], t[3], R[i].x - L[i].x, R[i].y + L[i].y);
      }
    }
  }
}

// G(p) += sum_k h_re(k) gWre(p + dk) + h_im(k) gWim(p + dk) for p in [pa, pb).  Items whose
// whole window lies in [-1, n] skip the per-load clamp.
template <typename A, int C, bool SYM>
__device__ void adjoint_scale(const Win& f, const Oct& O, const A* tab, const A* gw,
                              A* G, int pa, int pb, int K) {
  const int n = f.n;
  const int dil = O.dil;
  const int len = pb - pa;
  if (len <= 0) return;
  const int runs = static_cast<int>(cdiv(cdiv(len, dil), P));
  const int items = dil * runs;
  using V2 = typename Cplx<A>::type;
  const int lg = __ffs(dil) - 1;  // dil = 2^lg
  for (int it = threadIdx.x; it < items; it += nthreads()) {
    const int phi = it & (dil - 1), u0 = (it >> lg) * P;
    if (phi >= len) continue;
    const int base = pa + phi + dil * u0;
    V2 L[P], R[P];
    Acc2<A> acc[P];
#pragma unroll
    for (int i = 0; i < P; ++i) L[i] = R[i] = ld_gw<A, C>(gw, n, base + dil * i);
    {
      const A t0 = tab[0], t3 = tab[3];
#pragma unroll
      for (int i = 0; i < P; ++i) {
        acc[i].zero();
        acc[i].fmav(t0, t3, L[i].x, L[i].y);
      }
    }
    if (base - dil * K >= -1 && base + dil * (P - 1 + K) <= n)
      adjoint_taps<A, C, SYM, false>(tab, gw, n, K, dil, base, L, R, acc);
    else
      adjoint_taps<A, C, SYM, true>(tab, gw, n, K, dil, base, L, R, acc);
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int q = base + dil * i;
      if (q < pb) atE(f, G, q) += acc[i].re() + acc[i].im();
    }
  }
}

// One run of gradh_scale: RL positions nn + dil*t against the taps k0 .. k0 + 7 (base = nn - dil k0).
template <typename A, int C, bool CLAMP>
__device__ __forceinline__ void gradh_run(const FwdParams<A>& f, const A* X, const A* gw, int n,
                                          int dil, int nn, int base, Acc2<A> (&acc)[KT]) {
  using V2 = typename Cplx<A>::type;
  A xw[RL + KT - 1];  // x_j(base + dil*(m - 7)), m = 0..13
#pragma unroll
  for (int m = 0; m < RL + KT - 1; ++m)
    xw[m] = ldE_sel<A, CLAMP>(f, X, base + dil * (m - (KT - 1)));
#pragma unroll
  for (int t = 0; t < RL; ++t) {
    const V2 gv = ld_gw_sel<A, C, CLAMP>(gw, n, nn + dil * t);
#pragma unroll
    for (int i = 0; i < KT; ++i) {
      const A xv = xw[t - i + KT - 1];  // x_j(nn + dil*t - dil*(k0 + i))
      acc[i].fmav(gv.x, gv.y, xv, xv);
    }
  }
}

// Per-row dL/dH of one scale: part[c*hcols + center + k] = sum_n gW_c(n) x_j(n - dil k) for
// |k| <= K (zero elsewhere).  Warp w reduces taps [k0, k0 + KT) for kb = w, w + NW, ...; its lanes
// take runs of RL positions n = nn + dil*t of one phase (runs ordered phase-minor, so that the
// lanes of a warp read distinct banks), load the run's 14-value window of x_j and its 7 dL/dW
// pairs once, and accumulate 7 x 8 packed products.  Positions past the row end read the zero
// cells of the dL/dW buffer.  Lane partials are summed with shuffles.
template <typename A, int C>
__device__ void gradh_scale(const FwdParams<A>& f, const Oct& O, const A* X, const A* gw,
                            A* part) {

  const int n = static_cast<int>(f.n);
  const int dil = O.dil, K = O.half;
  const int lg = __ffs(dil) - 1;  // dil = 2^lg
  const int hcols = 2 * f.center + 1;
  const int ntap = 2 * K + 1;
  const int nkb = static_cast<int>(cdiv(ntap, KT));
  const int U = static_cast<int>(cdiv(n, dil));
  const int runs = dil * ((U + RL - 1) / RL);
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  using V2 = typename Cplx<A>::type;
  for (int c = threadIdx.x; c < C * hcols; c += nthreads()) {
    const int k = c % hcols - f.center;
    if (k < -K || k > K) part[c] = A(0);
  }
  for (int kb = w; kb < nkb; kb += nwarps()) {
    const int k0 = -K + kb * KT;
    Acc2<A> acc[KT];
#pragma unroll
    for (int i = 0; i < KT; ++i) acc[i].zero();
    for (int r = lane; r < runs; r += 32) {
      const int nn = (r & (dil - 1)) + (r >> lg) * (RL << lg);  // phase + dil * RL * run
      if (nn >= n) continue;
      const int base = nn - dil * k0;
      const bool inside = base - dil * (KT - 1) >= -f.ext &&
                          base + dil * (RL - 1) <= n + f.ext - 1 && nn + dil * (RL - 1) <= n;
      if (inside) gradh_run<A, C, false>(f, X, gw, n, dil, nn, base, acc);
      else gradh_run<A, C, true>(f, X, gw, n, dil, nn, base, acc);
    }
#pragma unroll
    for (int i = 0; i < KT; ++i) {
      A re = acc[i].re(), im = acc[i].im();
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        re += __shfl_xor_sync(0xffffffffu, re, o);
        if (C == 2) im += __shfl_xor_sync(0xffffffffu, im, o);
      }
      const int k = k0 + i;
      if (lane == 0 && k <= K) {
        part[f.center + k] = re;
        if (C == 2) part[hcols + f.center + k] = im;
      }
    }
  }
}

// dL/dW at one position from the recomputed W = (re, im) and the upstream gradient go of the
// consumer (MIX: y = sum a |W| + b Re W; SOFTMAX: out = sum pr V, pr = softmax(|W| tau^-1)
// with the forward's running max m and denominator l at rq).  The parameter sums go to sa / sb
// (or, for a per-position V, to *vpos) when `own`.  fp32 takes |W| and 1/|W| from one
// reciprocal square root and the softmax weight from the fast exponential and division
// (rsqrtf, __expf, __fdividef: a few ulp, l >= 1); fp64 uses exact operations.
template <typename A, int EPI, int C>
__device__ __forceinline__ void consumer_grad(const BwdParams<A>& p, A re, A im, A go, A av,
                                              A bv, A vv, int64_t rq, A* vpos, bool own,
                                              A& sa, A& sb, A& gre, A& gim) {
  constexpr bool F32 = std::is_same<A, float>::value;
  A mag, rs = A(0);
  if (C == 2) {
    if constexpr (F32) {
      const float s2 = fmaf(re, re, im * im);
      rs = s2 > 0.0f ? rsqrtf(s2) : 0.0f;
      mag = s2 * rs;
    } else {
      mag = sqrt(re * re + im * im);
      rs = mag > A(0) ? A(1) / mag : A(0);
    }
  } else {
    mag = fabs(re);
  }
  if (EPI == EPI_MIX) {
    if (own) {
      sa += go * mag;
      sb += go * re;
    }
    if (C == 2) {
      const A r = av * go * rs;
      gre = r * re + bv * go;
      gim = r * im;
    } else {
      const A sg = re > A(0) ? A(1) : (re < A(0) ? A(-1) : A(0));
      gre = go * (av * sg + bv);
      gim = A(0);
    }
  } else {
    const A inv_tau = p.f.inv_tau;
    A w;  // pr * go
    if constexpr (F32)
      w = __fdividef(__expf(fmaf(mag, inv_tau, -p.sm_m[rq])) * go, p.sm_l[rq]);
    else
      w = exp(mag * inv_tau - p.sm_m[rq]) / p.sm_l[rq] * go;
    const A gmag = w * (vv - p.sm_out[rq]) * inv_tau;
    if (own) {
      if (vpos) atomicAdd(vpos, w);
      else sa += w;
    }
    const A r = gmag * rs;
    gre = r * re;
    gim = r * im;
  }
}

// dL/dW_s on [0, n) into the gW buffer.  STORE: copied from the caller's gradient.  MIX /
// SOFTMAX: W_s is recomputed from x_j and the epilogue's derivative applied; the per-row
// parameter partials are returned through *pa_sum, *pb_sum (thread-local, summed by caller).
template <typename A, int EPI, int C, bool SYM>
__device__ void make_gw(const BwdParams<A>& p, const Oct& O, int s, int gs, const A* X,
                        const A* tab, int ks, A* gw, int64_t row, A& sa, A& sb) {
  const FwdParams<A>& f = p.f;
  const int n = static_cast<int>(f.n);
  if (EPI == EPI_STORE) {
    const A* g = p.g + (row * f.n_scales + gs) * f.n * C;
    for (int q = threadIdx.x; q < n; q += nthreads()) {
      if (C == 2) {
        const typename Cplx<A>::type v = reinterpret_cast<const typename Cplx<A>::type*>(g)[q];
        st_gw<A, C>(gw, q, v.x, v.y);
      } else {
        st_gw<A, C>(gw, q, g[q], A(0));
      }
    }
    return;
  }
  const int dil = O.dil;
  const int runs = static_cast<int>(cdiv(cdiv(n, dil), P));
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
  const Win wf = win(f);
  for (int it = threadIdx.x; it < items; it += nthreads()) {
    const int phi = it & (dil - 1), u0 = (it >> lg) * P;
    if (phi >= n) continue;
    const int base = phi + dil * u0;
    Acc2<A> acc[P];
    // W of the scale up to its last nonzero tap (ks): the taps past it are zero
    if (base - dil * ks >= -wf.ext && base + dil * (P - 1 + ks) <= n + wf.ext - 1)
      conv_one<A, SYM, false>(wf, X, tab, ks, dil, base, acc);
    else
      conv_one<A, SYM, true>(wf, X, tab, ks, dil, base, acc);
#pragma unroll
    for (int i = 0; i < P; ++i) {
      const int q = base + dil * i;
      if (q >= n) continue;
      const A re = acc[i].re(), im = C == 2 ? acc[i].im() : A(0);
      A vv = vconst;
      A* vpos = nullptr;
      if (EPI == EPI_SOFTMAX && f.v_pos) {
        const int64_t vq = (grp * f.n_scales + gs) * f.n + q;
        vv = static_cast<const A*>(f.a)[vq];
        vpos = p.v_part + vq;
      }
      A gre, gim;
      consumer_grad<A, EPI, C>(p, re, im, gy[q], av, bv, vv, row * f.n + q, vpos, true, sa, sb,
                               gre, gim);
      st_gw<A, C>(gw, q, gre, gim);
    }
  }
}

// The gradient work of one scale whose dL/dW is in gw (barrier-separated from the producer):
// its adjoint into G and its filter-gradient partial.
template <typename A, int C, bool SYM>
__device__ __forceinline__ void scale_grads(const BwdParams<A>& p, const Oct& O, int live, int gs,
                                            A* G, const A* X, const A* gw, const A* tab,
                                            int64_t row, int ks) {
  const FwdParams<A>& f = p.f;
  if (p.need_gx) {  // the adjoint over the scale's nonzero taps (ks <= O.half) and their reach
    const int reach = min(live, ks * O.dil);
    adjoint_scale<A, C, SYM>(win(f), O, tab, gw, G, -reach, static_cast<int>(f.n) + reach, ks);
  }
  if (p.gh_part) {
    const int hcols = 2 * f.center + 1;
    gradh_scale<A, C>(f, O, X, gw, p.gh_part + (row * f.n_scales + gs) * C * hcols);
  }
}

// MIX / SOFTMAX: dL/dW of each scale is formed from the recomputed W (make_gw) into one buffer.
template <typename A, int EPI, int C, bool SYM>
__device__ void scale_pass(const BwdParams<A>& p, const Oct& O, int live, int s, A* G,
                           const A* X, A* gw, const A* tab, A* red, int64_t row, int ks) {
  const FwdParams<A>& f = p.f;
  const int gs = f.order[O.begin + s];
  A sa = A(0), sb = A(0);
  make_gw<A, EPI, C, SYM>(p, O, s, gs, X, tab, ks, gw, row, sa, sb);
  if (EPI == EPI_MIX) {
    const A ta = block_sum(sa, red);
    const A tb = block_sum(sb, red);
    if (threadIdx.x == 0) {
      p.a_part[row * f.n_scales + gs] = ta;
      p.b_part[row * f.n_scales + gs] = tb;
    }
  } else if (EPI == EPI_SOFTMAX && !f.v_pos) {
    const A ta = block_sum(sa, red);
    if (threadIdx.x == 0) p.v_part[row * f.n_scales + gs] = ta;
  }
  __syncthreads();
  scale_grads<A, C, SYM>(p, O, live, gs, G, X, gw, tab, row, ks);
  __syncthreads();
}

// One octave.  STORE: the caller's dL/dW rows are double-buffered with cp.async, scale s + 1
// loading while scale s is processed (the first one was issued by the caller).
template <typename A, int EPI, int C>
__device__ void octave_pass(const BwdParams<A>& p, const Oct& O, int live, A* G, const A* X,
                            A* const* gws, const A* tab, const int* sym, const int* klast,
                            A* red, int64_t row) {
  const int K1 = O.half + 1;
  for (int s = 0; s < O.count; ++s) {
    const A* ts = tab + 4 * K1 * s;
    const bool sy = sym[s] != 0;
    const int ks = klast[s];
    if (EPI == EPI_STORE) {
      if (s + 1 < O.count) {
        stage_gw<A, C>(p, p.f.order[O.begin + s + 1], row, gws[(s + 1) & 1]);
        cp_commit();
        cp_wait<1>();
      } else {
        cp_wait<0>();
      }
      __syncthreads();
      const int gs = p.f.order[O.begin + s];
      if (sy) scale_grads<A, C, true>(p, O, live, gs, G, X, gws[s & 1], ts, row, ks);
      else scale_grads<A, C, false>(p, O, live, gs, G, X, gws[s & 1], ts, row, ks);
      __syncthreads();
    } else if (!p.pipe) {
      if (sy) scale_pass<A, EPI, C, true>(p, O, live, s, G, X, gws[0], ts, red, row, ks);
      else scale_pass<A, EPI, C, false>(p, O, live, s, G, X, gws[0], ts, red, row, ks);
    }
  }
  if (EPI == EPI_STORE || !p.pipe) return;
  // MIX / SOFTMAX, pipelined: step t recomputes scale t and forms its dL/dW in gws[t & 1] while
  // the adjoint and filter gradient of scale t - 1 run from gws[(t - 1) & 1], with one barrier
  // per step.  The parameter sums of scale t go per warp into slot t & 1 of red + NW_MAX (two
  // sums x NW_MAX warps) and thread 0 adds them up in warp order at the next step.
  const FwdParams<A>& f = p.f;
  A* wsum = red + NW_MAX;
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = 0; t <= O.count; ++t) {
    if (t > 0 && threadIdx.x == 0 && (EPI == EPI_MIX || !f.v_pos)) {
      const A* ws = wsum + ((t - 1) & 1) * 2 * NW_MAX;
      A ta = A(0), tb = A(0);
      for (int i = 0; i < nwarps(); ++i) {
        ta += ws[i];
        tb += ws[NW_MAX + i];
      }
      const int64_t at = row * f.n_scales + f.order[O.begin + t - 1];
      if (EPI == EPI_MIX) {
        p.a_part[at] = ta;
        p.b_part[at] = tb;
      } else {
        p.v_part[at] = ta;
      }
    }
    if (t < O.count) {
      const int gs = f.order[O.begin + t];
      const A* ts = tab + 4 * K1 * t;
      A sa = A(0), sb = A(0);
      if (sym[t]) make_gw<A, EPI, C, true>(p, O, t, gs, X, ts, klast[t], gws[t & 1], row, sa, sb);
      else make_gw<A, EPI, C, false>(p, O, t, gs, X, ts, klast[t], gws[t & 1], row, sa, sb);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sa += __shfl_xor_sync(0xffffffffu, sa, o);
        sb += __shfl_xor_sync(0xffffffffu, sb, o);
      }
      if (lane == 0) {
        wsum[(t & 1) * 2 * NW_MAX + w] = sa;
        wsum[(t & 1) * 2 * NW_MAX + NW_MAX + w] = sb;
      }
    }
    if (t > 0) {
      const int s = t - 1;
      const int gs = f.order[O.begin + s];
      const A* ts = tab + 4 * K1 * s;
      if (sym[s]) scale_grads<A, C, true>(p, O, live, gs, G, X, gws[s & 1], ts, row, klast[s]);
      else scale_grads<A, C, false>(p, O, live, gs, G, X, gws[s & 1], ts, row, klast[s]);
    }
    __syncthreads();
  }
}

template <typename A, int EPI>
__global__ void __launch_bounds__(NTB_MAX) cwt_backward_kernel(const __grid_constant__ BwdParams<A> p) {
  extern __shared__ __align__(16) unsigned char smem[];
  const FwdParams<A>& f = p.f;
  A* bufs[3] = {reinterpret_cast<A*>(smem), reinterpret_cast<A*>(smem) + f.buf_len,
                reinterpret_cast<A*>(smem) + 2 * f.buf_len};
  A* gws[2] = {reinterpret_cast<A*>(smem + p.gw_off),
               reinterpret_cast<A*>(smem + p.gw_off) + p.gw_len};
  A* tab = reinterpret_cast<A*>(smem + p.tab_off);
  A* red = reinterpret_cast<A*>(smem + p.red_off);
  __shared__ int sym[kMaxScales];
  __shared__ int klast[kMaxScales];  // per scale of the octave: last nonzero tap
  const int64_t row = blockIdx.x;
  const int n = static_cast<int>(f.n);
  const int E = f.ext;
  const int J = f.n_oct;
  const RowRef<const A> xr = row_ref(static_cast<const A*>(f.x), f, row);

  // the end cells of the dL/dW buffers (positions -1 and n) are never written again
  for (int q = threadIdx.x; q < (EPI == EPI_STORE || p.pipe ? 2 : 1) * p.gw_len; q += nthreads())
    gws[0][q] = A(0);
  __syncthreads();

  // pass 1: x_1 .. x_{J-1} into the row's scratch
  if (p.need_x && J > 1) {
    A* cur = bufs[0];
    A* nxt = bufs[1];
    for (int q = static_cast<int>(threadIdx.x) - E; q < n + E; q += nthreads())
      atE(f, cur, q) = (q >= 0 && q < n) ? xr[q] : A(0);
    __syncthreads();
    for (int j = 0; j + 1 < J; ++j) {
      bwd_lowpass<A>(f, cur, nxt, f.oct[j].dil, f.oct[j + 1].live);
      __syncthreads();
      if (p.pyr_off[j + 1] >= 0) {
        const int lv = f.oct[j + 1].live;
        A* dst = p.pyr + row * p.pyr_len + p.pyr_off[j + 1];
        for (int q = static_cast<int>(threadIdx.x) - lv; q < n + lv; q += nthreads())
          dst[q + lv] = atE(f, nxt, q);
      }
      A* t = cur;
      cur = nxt;
      nxt = t;
    }
    __syncthreads();
  }

  // pass 2: coarse -> fine
  A* G = bufs[0];
  A* Gn = bufs[1];
  A* X = bufs[2];
  for (int q = static_cast<int>(threadIdx.x) - E; q < n + E; q += nthreads()) atE(f, G, q) = A(0);
  for (int j = J - 1; j >= 0; --j) {
    const Oct& O = f.oct[j];
    if (j + 1 < J && p.need_gx) {
      __syncthreads();
      bwd_lowpass_adjoint<A>(f, G, Gn, O.dil, O.live);
      A* t = G;
      G = Gn;
      Gn = t;
    }
    if (O.count > 0 && EPI == EPI_STORE) {
      // the octave's first dL/dW row loads while x_j and the taps are prepared
      if (f.channels == 2) stage_gw<A, 2>(p, f.order[O.begin], row, gws[0]);
      else stage_gw<A, 1>(p, f.order[O.begin], row, gws[0]);
      cp_commit();
    }
    if (O.count > 0) {
      if (p.need_x && j == 0) {  // x_0 = x on [0, n)
        for (int q = static_cast<int>(threadIdx.x) - E; q < n + E; q += nthreads())
          atE(f, X, q) = (q >= 0 && q < n) ? xr[q] : A(0);
      } else if (p.need_x) {
        const int lv = O.live;
        const A* srcp = p.pyr + row * p.pyr_len + p.pyr_off[j];
        for (int q = static_cast<int>(threadIdx.x) - E; q < n + E; q += nthreads())
          atE(f, X, q) = (q >= -lv && q < n + lv) ? srcp[q + lv] : A(0);
      }
      __syncthreads();
      build_octave_taps<A>(f, O, tab, sym, klast);
      if (f.channels == 2)
        octave_pass<A, EPI, 2>(p, O, O.live, G, X, gws, tab, sym, klast, red, row);
      else
        octave_pass<A, EPI, 1>(p, O, O.live, G, X, gws, tab, sym, klast, red, row);
    }
  }
  __syncthreads();
  if (p.need_gx) {
    const RowRef<A> gx = row_ref(p.gx, f, row);
    for (int q = threadIdx.x; q < n; q += nthreads()) gx[q] = atE(f, G, q);
  }
}

// out[d, e] = sum_{i} part[(d + i D), e] over the rows r = d + i D < rows, in order of i.
// Two stages for parallelism: stage 1 sums row chunks into tmp, stage 2 sums the chunks.
template <typename A>
__global__ void reduce_rows_kernel(const A* __restrict__ part, int64_t rows, int64_t cols,
                                   int64_t D, int64_t per_chunk, int64_t nchunk, A* __restrict__ out) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t d = blockIdx.y;
  const int64_t ch = blockIdx.z;
  if (e >= cols) return;
  const int64_t per_d = cdiv(rows - d, D);  // rows of residue d
  const int64_t i0 = ch * per_chunk, i1 = imin(per_d, i0 + per_chunk);
  A s = A(0);
  for (int64_t i = i0; i < i1; ++i) s += part[(d + i * D) * cols + e];
  out[(ch * D + d) * cols + e] = s;
}

// ------------------------------------------------------------------------------ host

// Two-stage reduction plan of reduce_rows: chunks per residue so that stage 1 fills the GPU.
inline int64_t reduce_chunks(int64_t rows, int64_t cols, int64_t D) {
  const int64_t per_d = cdiv(rows, D);
  const int64_t blocks = cdiv(cols, 256) * D;
  int64_t nch = cdiv(2 * static_cast<int64_t>(sm_count()), blocks);
  nch = imin(nch, imax(1, per_d / 16));
  return imax(1, nch);
}
inline size_t reduce_tmp_elems(int64_t rows, int64_t cols, int64_t D) {
  const int64_t nch = reduce_chunks(rows, cols, D);
  return nch > 1 ? static_cast<size_t>(nch * D * cols) : 0;
}

template <typename A>
int reduce_rows(const A* part, int64_t rows, int64_t cols, int64_t D, A* out, A* tmp,
                cudaStream_t stream) {
  if (cols == 0 || D == 0) return FDWT_OK;
  if (D > 65535) return FDWT_ERR_UNSUPPORTED;
  const int64_t nch = reduce_chunks(rows, cols, D);
  const int64_t per_d = cdiv(rows, D);
  const dim3 block(256);
  int st = pre_launch(stream);
  if (st != FDWT_OK) return st;
  if (nch == 1) {
    reduce_rows_kernel<A><<<dim3(static_cast<unsigned>(cdiv(cols, 256)), static_cast<unsigned>(D), 1),
                            block, 0, stream>>>(part, rows, cols, D, per_d, 1, out);
    return launch_status();
  }
  const int64_t per_chunk = cdiv(per_d, nch);
  reduce_rows_kernel<A><<<dim3(static_cast<unsigned>(cdiv(cols, 256)), static_cast<unsigned>(D),
                               static_cast<unsigned>(nch)),
                          block, 0, stream>>>(part, rows, cols, D, per_chunk, nch, tmp);
  st = launch_status();
  if (st != FDWT_OK) return st;
  if ((st = pre_launch(stream)) != FDWT_OK) return st;
  reduce_rows_kernel<A><<<dim3(static_cast<unsigned>(cdiv(cols, 256)), static_cast<unsigned>(D), 1),
                          block, 0, stream>>>(tmp, nch * D, cols, D, nch, 1, out);
  return launch_status();
}

// Workspace regions of one backward call (bytes, each 256-aligned).
struct BwdLayout {
  int64_t pyr_len = 0;
  int32_t pyr_off[kMaxOct];
  size_t pyr = 0, gh = 0, pa = 0, pb = 0, pv = 0, tmp = 0, total = 0;
};

inline size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

template <typename A>
BwdLayout bwd_layout(int EPI, int64_t rows, int64_t n, const fdwt_morlet_plan* pl,
                     const Geometry& g, bool need_h, int64_t dim, bool v_pos) {
  BwdLayout L;
  const int J = pl->n_octaves;
  const bool need_x = need_h || EPI != EPI_STORE;
  for (int j = 0; j < kMaxOct; ++j) L.pyr_off[j] = -1;
  if (need_x)
    for (int j = 1; j < J; ++j)
      if (pl->oct_count[j] > 0) {
        L.pyr_off[j] = static_cast<int32_t>(L.pyr_len);
        L.pyr_len += n + 2 * static_cast<int64_t>(g.live[j]);
      }
  const int64_t S = pl->n_scales;
  const int64_t hcols = 2 * static_cast<int64_t>(pl->center) + 1;
  const int64_t ghcols = S * pl->channels * hcols;
  L.pyr = align256(static_cast<size_t>(rows) * L.pyr_len * sizeof(A));
  L.gh = need_h ? align256(static_cast<size_t>(rows) * ghcols * sizeof(A)) : 0;
  L.pa = EPI == EPI_MIX ? align256(static_cast<size_t>(rows) * S * sizeof(A)) : 0;
  L.pb = L.pa;
  L.pv = (EPI == EPI_SOFTMAX && !v_pos) ? align256(static_cast<size_t>(rows) * S * sizeof(A)) : 0;
  size_t tmp = 0;
  if (need_h) tmp = std::max(tmp, reduce_tmp_elems(rows, ghcols, 1));
  if (EPI == EPI_MIX) tmp = std::max(tmp, reduce_tmp_elems(rows, S, dim));
  if (EPI == EPI_SOFTMAX && !v_pos) tmp = std::max(tmp, reduce_tmp_elems(rows, S, dim));
  L.tmp = align256(tmp * sizeof(A));
  L.total = L.pyr + L.gh + L.pa + L.pb + L.pv + L.tmp;
  return L;
}

// Shared bytes of the row-resident backward kernel for rows of n samples (the buffer offsets go
// into p when it is given).
template <typename A, int EPI>
size_t row_bwd_smem(int64_t n, const fdwt_morlet_plan* pl, int ext, BwdParams<A>* p,
                    bool pipe = false) {
  const int64_t buf_len = (n + 2 * static_cast<int64_t>(ext)) + 8;
  const int64_t gw_len = 2 * (n + 2) + 8;
  if (buf_len > 0x3fffffffLL) return ~size_t(0);
  size_t off = 3 * static_cast<size_t>(buf_len) * sizeof(A);
  off = (off + 15) / 16 * 16;
  const size_t gw_off = off;
  off += (EPI == EPI_STORE || pipe ? 2 : 1) * static_cast<size_t>(gw_len) * sizeof(A);
  off = (off + 15) / 16 * 16;
  const size_t tab_off = off;
  size_t tab = 0;  // the largest octave's tap tables
  for (int j = 0; j < pl->n_octaves; ++j)
    tab = std::max(tab, 4 * static_cast<size_t>(pl->oct_count[j]) * (pl->oct_half[j] + 1));
  off += tab * sizeof(A);
  off = (off + 15) / 16 * 16;
  const size_t red_off = off;
  off += 5 * NW_MAX * sizeof(A);  // block sums, then the pipelined steps' per-warp sums
  if (p) {
    p->f.buf_len = static_cast<int>(buf_len);
    p->gw_len = static_cast<int>(gw_len);
    p->gw_off = static_cast<int>(gw_off);
    p->tab_off = static_cast<int>(tab_off);
    p->red_off = static_cast<int>(red_off);
    p->pipe = pipe ? 1 : 0;
  }
  return off + 16;
}

template <typename A, int EPI>
int run_backward_tiled(int64_t rows, int64_t n, const void* x, const void* h,
                       const fdwt_morlet_plan* pl, const Geometry& geo, const void* a,
                       const void* b, int64_t dim, int v_pos, double inv_tau, const void* g,
                       const void* sm_m, const void* sm_l, const void* sm_out, void* gx, void* gh,
                       void* ga, void* gb, void* gv, bool need_h, void* ws, size_t ws_bytes,
                       cudaStream_t stream, size_t* ws_needed, int tok);

// Backward of the transform (EPI_STORE), of the mix (EPI_MIX) or of the spectral softmax
// (EPI_SOFTMAX).  Rows whose buffers do not fit one CTA's shared memory take the octave-tiled
// launches of cwt_bwd_tiled.cuh.  Outputs gx (rows, n), gh (S*C, 2*center+1), ga/gb (dim, S), gv (nch, S) or
// (G, S, n); null outputs are skipped.  ws_needed != null: only report the workspace size (for
// a call with or without gh, as need_h says).
template <typename A, int EPI>
int run_backward(int64_t rows, int64_t n, const void* x, const void* h,
                 const fdwt_morlet_plan* pl, const void* a, const void* b, int64_t dim,
                 int v_pos, double inv_tau, const void* g, const void* sm_m, const void* sm_l,
                 const void* sm_out, void* gx, void* gh, void* ga, void* gb, void* gv, bool need_h,
                 void* ws, size_t ws_bytes, cudaStream_t stream, size_t* ws_needed,
                 int tok = 0) {
  int st = check_plan(pl, n);
  if (st != FDWT_OK) return st;
  if (EPI == EPI_SOFTMAX && pl->channels != 2) return FDWT_ERR_INVALID;
  if (rows > 0x7fffffffLL || n > 0x3fffffffLL) return FDWT_ERR_UNSUPPORTED;
  const Geometry geo = geometry(pl);
  if (ws_needed == nullptr) need_h = gh != nullptr;
  if (v_pos && (dim < 1 || rows % dim != 0)) return FDWT_ERR_INVALID;
  int E = 0;
  for (int j = 0; j < pl->n_octaves; ++j) E = std::max(E, geo.live[j]);
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 2048;
  const bool tiled = cwt_tile_test() > 0 || row_bwd_smem<A, EPI>(n, pl, E + 1, nullptr) > budget;
  const BwdLayout lay = bwd_layout<A>(EPI, rows, n, pl, geo, need_h, dim, v_pos != 0);
  if (ws_needed) {
    if (tiled)
      return run_backward_tiled<A, EPI>(rows, n, x, h, pl, geo, a, b, dim, v_pos, inv_tau, g,
                                        sm_m, sm_l, sm_out, gx, gh, ga, gb, gv, need_h, ws,
                                        ws_bytes, stream, ws_needed, tok);
    *ws_needed = lay.total;
    return FDWT_OK;
  }
  const int64_t S = pl->n_scales;
  const int64_t hcols = 2 * static_cast<int64_t>(pl->center) + 1;
  const int64_t ghcols = S * pl->channels * hcols;
  // outputs that are sums over rows start from zero when there are no rows
  if (rows == 0 || EPI == EPI_SOFTMAX) {
    auto zero = [&](void* ptr, size_t bytes) -> int {
      if (ptr == nullptr || bytes == 0) return FDWT_OK;
      cudaError_t e = cudaMemsetAsync(ptr, 0, bytes, stream);
      if (e != cudaSuccess) {
        set_cuda_error(e);
        return FDWT_ERR_CUDA;
      }
      return FDWT_OK;
    };
    if (rows == 0) {
      if ((st = zero(gh, ghcols * sizeof(A))) != FDWT_OK) return st;
      if (EPI == EPI_MIX) {
        if ((st = zero(ga, dim * S * sizeof(A))) != FDWT_OK) return st;
        if ((st = zero(gb, dim * S * sizeof(A))) != FDWT_OK) return st;
      }
      if (EPI == EPI_SOFTMAX && !v_pos && (st = zero(gv, dim * S * sizeof(A))) != FDWT_OK)
        return st;
      return FDWT_OK;
    }
    if (v_pos && (st = zero(gv, static_cast<size_t>(rows / dim) * S * n * sizeof(A))) != FDWT_OK)
      return st;
  }
  if (tiled)
    return run_backward_tiled<A, EPI>(rows, n, x, h, pl, geo, a, b, dim, v_pos, inv_tau, g, sm_m,
                                      sm_l, sm_out, gx, gh, ga, gb, gv, need_h, ws, ws_bytes,
                                      stream, nullptr, tok);
  if (lay.total > 0 && (ws == nullptr || ws_bytes < lay.total)) return FDWT_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  A* pyr = reinterpret_cast<A*>(w);
  A* ghp = reinterpret_cast<A*>(w + lay.pyr);
  A* pa = reinterpret_cast<A*>(w + lay.pyr + lay.gh);
  A* pb = reinterpret_cast<A*>(w + lay.pyr + lay.gh + lay.pa);
  A* pv = reinterpret_cast<A*>(w + lay.pyr + lay.gh + lay.pa + lay.pb);
  A* tmp = reinterpret_cast<A*>(w + lay.pyr + lay.gh + lay.pa + lay.pb + lay.pv);

  BwdParams<A> p{};
  fill_common(p.f, pl, geo, n);
  p.f.ext = E + 1;
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
  p.v_part = EPI == EPI_SOFTMAX ? (v_pos ? static_cast<A*>(gv) : pv) : nullptr;
  p.pyr = lay.pyr_len > 0 ? pyr : nullptr;
  p.pyr_len = lay.pyr_len;
  for (int j = 0; j < kMaxOct; ++j) p.pyr_off[j] = lay.pyr_off[j];
  p.need_gx = gx != nullptr;
  p.need_x = (gh != nullptr || EPI != EPI_STORE) ? 1 : 0;
  size_t smem = row_bwd_smem<A, EPI>(n, pl, p.f.ext, &p);
  // rows that already take one CTA per SM pipeline their scales when a second dL/dW buffer fits
  if (EPI != EPI_STORE && smem > budget / 2 &&
      row_bwd_smem<A, EPI>(n, pl, p.f.ext, nullptr, true) <= budget)
    smem = row_bwd_smem<A, EPI>(n, pl, p.f.ext, &p, true);
  if (smem > budget) return FDWT_ERR_UNSUPPORTED;
  if (!p.need_gx && gh == nullptr && EPI == EPI_STORE) return FDWT_OK;
  auto kern = cwt_backward_kernel<A, EPI>;
  st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
  if (st != FDWT_OK) return st;
  if ((st = pre_launch(stream)) != FDWT_OK) return st;
  // one CTA per SM when the row needs more than half the shared memory: give it NTB_MAX threads
  const int threads = smem > budget / 2 ? NTB_MAX : NT;
  kern<<<static_cast<unsigned>(rows), threads, smem, stream>>>(p);
  if ((st = launch_status()) != FDWT_OK) return st;
  if (gh && (st = reduce_rows<A>(ghp, rows, ghcols, 1, static_cast<A*>(gh), tmp, stream)) != FDWT_OK)
    return st;
  if (EPI == EPI_MIX) {
    if (ga && (st = reduce_rows<A>(pa, rows, S, dim, static_cast<A*>(ga), tmp, stream)) != FDWT_OK)
      return st;
    if (gb && (st = reduce_rows<A>(pb, rows, S, dim, static_cast<A*>(gb), tmp, stream)) != FDWT_OK)
      return st;
  }
  if (EPI == EPI_SOFTMAX && !v_pos && gv &&
      (st = reduce_rows<A>(pv, rows, S, dim, static_cast<A*>(gv), tmp, stream)) != FDWT_OK)
    return st;
  return FDWT_OK;
}

// ------------------------------------------------------------------------------ token layout

// dL/dy of MorletTokenMixer's (B, n, dim) output into the (B dim, n) rows the backward reads
// once per scale, and the column sums of each (b, 32-position) tile for dL/dbias: 32 x 32
// tiles through shared memory (coalesced on both sides), 32 x 8 threads.
template <typename A>
__global__ void __launch_bounds__(256) tokens_to_rows_kernel(const A* __restrict__ in, int64_t B,
                                                             int64_t n, int64_t dim,
                                                             A* __restrict__ out,
                                                             A* __restrict__ colsum) {
  __shared__ A t[32][33];
  const int64_t q0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t d0 = static_cast<int64_t>(blockIdx.y) * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;
  for (int64_t b = blockIdx.z; b < B; b += gridDim.z) {
    for (int i = ty; i < 32; i += 8) {
      const int64_t q = q0 + i, d = d0 + tx;
      t[i][tx] = (q < n && d < dim) ? in[(b * n + q) * dim + d] : A(0);
    }
    __syncthreads();
    if (ty == 0 && d0 + tx < dim) {
      A v = A(0);
      for (int i = 0; i < 32; ++i) v += t[i][tx];
      colsum[(b * gridDim.x + blockIdx.x) * dim + d0 + tx] = v;
    }
    for (int i = ty; i < 32; i += 8) {
      const int64_t d = d0 + i, q = q0 + tx;
      if (d < dim && q < n) out[(b * dim + d) * n + q] = t[tx][i];
    }
    __syncthreads();
  }
}

// Workspace of the token-layout mix backward: dL/dy rows, tile column sums, their reduction
// scratch, then the mix backward's own regions.
struct TokLayout {
  size_t rows_bytes = 0, colsum = 0, tmp = 0, head = 0;
};
template <typename A>
TokLayout tok_layout(int64_t B, int64_t n, int64_t dim) {
  TokLayout L;
  const int64_t ntq = cdiv(n, 32);
  L.rows_bytes = align256(static_cast<size_t>(B * dim) * n * sizeof(A));
  L.colsum = align256(static_cast<size_t>(B * ntq) * dim * sizeof(A));
  L.tmp = align256(reduce_tmp_elems(B * ntq, dim, 1) * sizeof(A));
  L.head = L.rows_bytes + L.colsum + L.tmp;
  return L;
}

// Backward of the mix on MorletTokenMixer's layout: x, dL/dy, dL/dx are (B, n, dim); dL/dbias
// (dim) is the sum of dL/dy over (B, n).  ws_needed != null: only report the workspace size.
template <typename A>
int run_mix_tokens_backward(int64_t B, int64_t n, int64_t dim, const void* x, const void* h,
                            const fdwt_morlet_plan* pl, const void* a, const void* b,
                            const void* gy, void* gx, void* gh, void* ga, void* gb, void* gbias,
                            bool need_h, void* ws, size_t ws_bytes, cudaStream_t stream,
                            size_t* ws_needed) {
  if (B < 0 || n < 1 || dim < 1 || B > 0x7fffffffLL / dim) return FDWT_ERR_INVALID;
  const int64_t rows = B * dim;
  const TokLayout T = tok_layout<A>(B, n, dim);
  size_t inner = 0;
  int st = run_backward<A, EPI_MIX>(rows, n, nullptr, nullptr, pl, nullptr, nullptr, dim, 0, 1.0,
                                    nullptr, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                                    nullptr, nullptr, need_h, nullptr, 0, nullptr, &inner, 1);
  if (st != FDWT_OK) return st;
  if (ws_needed) {
    *ws_needed = T.head + inner;
    return FDWT_OK;
  }
  if (B == 0) {
    if (gbias) {
      const cudaError_t e = cudaMemsetAsync(gbias, 0, dim * sizeof(A), stream);
      if (e != cudaSuccess) {
        set_cuda_error(e);
        return FDWT_ERR_CUDA;
      }
    }
    return run_backward<A, EPI_MIX>(0, n, x, h, pl, a, b, dim, 0, 1.0, gy, nullptr, nullptr,
                                    nullptr, gx, gh, ga, gb, nullptr, need_h, nullptr, 0, stream,
                                    nullptr, 1);
  }
  if (ws == nullptr || ws_bytes < T.head + inner) return FDWT_ERR_WORKSPACE;
  unsigned char* w = static_cast<unsigned char*>(ws);
  A* gy_rows = reinterpret_cast<A*>(w);
  A* colsum = reinterpret_cast<A*>(w + T.rows_bytes);
  A* tmp = reinterpret_cast<A*>(w + T.rows_bytes + T.colsum);
  const int64_t ntq = cdiv(n, 32), ntd = cdiv(dim, 32);
  if (ntq > 0x7fffffffLL || ntd > 65535) return FDWT_ERR_UNSUPPORTED;
  if ((st = pre_launch(stream)) != FDWT_OK) return st;
  tokens_to_rows_kernel<A><<<dim3(static_cast<unsigned>(ntq), static_cast<unsigned>(ntd),
                                  static_cast<unsigned>(imin(B, 65535))),
                             dim3(32, 8), 0, stream>>>(static_cast<const A*>(gy), B, n, dim,
                                                       gy_rows, colsum);
  if ((st = launch_status()) != FDWT_OK) return st;
  if (gbias && (st = reduce_rows<A>(colsum, B * ntq, dim, 1, static_cast<A*>(gbias), tmp,
                                    stream)) != FDWT_OK)
    return st;
  return run_backward<A, EPI_MIX>(rows, n, x, h, pl, a, b, dim, 0, 1.0, gy_rows, nullptr, nullptr,
                                  nullptr, gx, gh, ga, gb, nullptr, need_h, w + T.head, inner,
                                  stream, nullptr, 1);
}

}  // namespace cwtk
}  // namespace fdwt
