// Morlet CWT octave pyramid for sm_100a: forward transform and the two fused scalogram
// consumers (magnitude/phase mix, online spectral softmax).  Templates; instantiated per
// element type and epilogue in cwt_<type>_<epilogue>.cu (cwt_entry.cuh).
//
// One CTA owns one signal row, or one time tile of a row too long for one CTA's shared memory.
// The pyramid x_0, x_1, ... lives in two ping-pong shared buffers that cover every position a
// later octave reads; x_j is exactly the reference's zero-padded, margin-truncated signal
// (fdwt/cwt.py:130-138, 512-519): it is nonzero only on [-e_j, n + e_j) with e_0 = 0 and
// e_{j+1} = min(margin_{j+1}, e_j + c_lp 2^j), and is stored as zeros elsewhere.
//
// Time tiles.  A tile owns the outputs [t0, t0 + tk) and its buffers cover [t0 - H, t0 + tk + H)
// with H the reach of the pyramid: H_J-1 = half_J-1 2^(J-1), H_j = max(half_j 2^j,
// H_j+1 + c_lp 2^j), H = H_0.  x_j is then exact on [t0 - H_j, t0 + tk + H_j), which holds
// every position the tile's outputs of octave j read; positions further out are computed from
// an incomplete window (or set to zero where the window leaves the buffer) and never read by a
// kept output.  A whole row is the tile t0 = 0, tk = n with H the row's reach (positions past
// the live extents are zero).  The PYR mode runs the half-band chain alone over tiles of
// [-e, n + e) and writes x_1 .. x_J-1 to global memory for the backward pass.
//
// Octave j applies the Morlet filters of its scales at spacing 2^j (fdwt/kernels/conv.py:38-134)
// and then the dilated half-band step produces x_{j+1} (fdwt/kernels/conv.py:251-279).
//
// Filter stage.  A work item is PF = 5 consecutive polyphase outputs n_i = phi + 2^j (u0 + i) of
// one phase; the thread keeps a left window x[n_i - 2^j k] and a right window x[n_i + 2^j k] in
// registers, each advancing with one shared load per tap through a pointer that moves by 2^j
// (the pyramid buffers are linear; the lanes of a warp start their windows 5 2^j apart, on
// distinct banks for every power-of-two 2^j, so no padding is needed).  Items whose windows stay
// inside the buffer skip the per-load clamp.  A block of up to 5 scales shares the window sums;
// the scales (sorted by support) leave the tap loop one by one at their own last nonzero tap,
// so the packed FMAs are exactly the filters' nonzero taps.  The Morlet filters are even (real
// part) and odd (imaginary part) in k (fdwt/cwt.py:192-203), so a tap pair costs one packed
// fp32 FMA per scale: (re, im) += (h_re[k], h_im[k]) * (x_l + x_r, x_l - x_r).  The symmetric
// and antisymmetric halves of every filter are separated exactly when its coefficient table is
// built; filters that are not exactly symmetric (never the case for MorletPlan.filters) take a
// second packed FMA per tap with the antisymmetric halves, so any filter is computed exactly.
//
// Epilogues.  STORE writes W (rows, S, n, C) in the user's scale order.  MIX reduces each tile
// to sum_s a[d,s] |W_s| + b[d,s] Re W_s in registers and accumulates a per-row shared
// accumulator (no atomics: an item owns its outputs for the whole octave).  SOFTMAX folds
// |W| / tau into a per-position online softmax (max, denominator, numerator) kept in shared
// memory across octaves (fdwt/kernels/softmax.py:133-139, 242-247).  Neither writes W.
#pragma once

#include <algorithm>
#include <cmath>
#include <type_traits>
#include <vector>

#include "common.cuh"

namespace fdwt {
namespace cwtk {

constexpr int NT = 256;           // threads per CTA
constexpr int P = 7;              // consecutive polyphase outputs per work item (backward):
                                  // odd, like PF below, for the backward's linear buffers
constexpr int PF = 5;             // the same in the forward: an odd run length keeps the
                                  // windows of a warp's lanes on distinct banks of the linear
                                  // (unpadded) buffers for every power-of-two dilation
constexpr int SBMAX = 5;          // scales per block of the forward's tap loop
constexpr int PS = 3;             // pyramid buffers: one pad element per 8
constexpr int kMaxOct = FDWT_MAX_OCTAVES;
constexpr int kMaxScales = FDWT_MAX_SCALES;
constexpr int kMaxC = (FDWT_MAX_LOWPASS - 1) / 2;

enum Epi { EPI_STORE = 0, EPI_MIX = 1, EPI_SOFTMAX = 2, EPI_PYR = 3 };

struct Oct {
  int32_t dil, half, begin, count;
  int32_t live;  // x_j may be nonzero on [-live, n + live)
};

template <typename A>
struct FwdParams {
  int64_t rows, n;
  const void* x;    // (rows, n)
  const void* h;    // filters (S*C, 2*center+1)
  void* y;          // STORE: (rows, S, n, C); MIX / SOFTMAX: (rows, n)
  const void* a;    // MIX: (dim, S)        SOFTMAX: V
  const void* b;    // MIX: (dim, S)
  void* m_out;      // SOFTMAX: (rows, n)
  void* l_out;
  int64_t dim;      // MIX: channels of the a/b tables; SOFTMAX: nch
  int32_t v_pos;    // SOFTMAX: V per position
  int32_t n_oct, n_scales, channels, center, c_lp;
  int32_t ext;      // the pyramid buffers hold positions [-ext, n + ext)
  int32_t buf_len;  // padded elements of one pyramid buffer
  int32_t coef_off, extra_off;  // byte offsets of the coefficient table and epilogue state
  int32_t coef_cap;             // elements of the shared coefficient table (0: taps read from
                                // global memory, for octaves whose table does not fit)
  A inv_tau;
  A lpp[kMaxC + 1];  // lowpass[c_lp + t]
  A lpm[kMaxC + 1];  // lowpass[c_lp - t]
  // the half-band taps that matter: offsets t >= 1 whose coefficient is not negligible (the
  // even-offset taps of a half-band filter are zero up to rounding, ~1e-17 of the centre), with
  // (lpp, lpm) for each; lp_sym when every kept pair is equal (x(q-dt) + x(q+dt) once)
  int32_t n_lp, lp_sym;
  int32_t lp_t[kMaxC];
  A lp_p[kMaxC], lp_m[kMaxC];
  Oct oct[kMaxOct];
  int32_t order[kMaxScales];
  int32_t support[kMaxScales];
  // time tiles: CTA b owns [t_base + (b % ntile) t_len, ...) up to t_end, buffers reach `halo`
  // past both ends of the owned range (a whole row: ntile 1, t_len = t_end = n, halo = ext)
  int32_t ntile, t_len, t_base, t_end, halo;
  // PYR: x_j (j >= 1, pyr_off[j] >= 0) into pyr + row * pyr_len + pyr_off[j] on [-live_j, n + live_j)
  A* pyr;
  int64_t pyr_len;
  int32_t pyr_off[kMaxOct];
  // token layout (MorletTokenMixer's (B, n, dim) input): x, and MIX's y, hold row b dim + d at
  // element stride dim (element q at (b n + q) dim + d); MIX adds bias[d] to y when non-null
  int32_t tok;
  const void* bias;
};

// Row `row` of a signal argument: (rows, n) row-major, or the token layout of FwdParams::tok.
template <typename T>
struct RowRef {
  T* p;
  int64_t step;
  __device__ __forceinline__ T& operator[](int64_t q) const { return p[q * step]; }
};
template <typename T, typename Prm>
__device__ __forceinline__ RowRef<T> row_ref(T* base, const Prm& f, int64_t row) {
  if (f.tok) return RowRef<T>{base + (row / f.dim) * f.n * f.dim + row % f.dim, f.dim};
  return RowRef<T>{base + row * f.n, 1};
}

// The part of a row a CTA computes: buffers cover [org, org + span); kept outputs [t0, tend).
struct Span {
  int org, limit, t0, tend;
};

// ------------------------------------------------------------------------------ helpers

__device__ __forceinline__ unsigned long long pk(float lo, float hi) {
  return static_cast<unsigned long long>(__float_as_uint(lo)) |
         (static_cast<unsigned long long>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float lo_f(unsigned long long v) {
  return __uint_as_float(static_cast<unsigned>(v));
}
__device__ __forceinline__ float hi_f(unsigned long long v) {
  return __uint_as_float(static_cast<unsigned>(v >> 32));
}
__device__ __forceinline__ void ffma2(unsigned long long& acc, unsigned long long a,
                                      unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

// Accumulator pair (re, im) of one scale and output: packed fp32 or two fp64.
template <typename A>
struct Acc2;
template <>
struct Acc2<float> {
  unsigned long long v;
  __device__ __forceinline__ void zero() { v = 0ull; }
  // (re, im) += (c0, c1) * (s0, s1), c from a 16-byte aligned float pair
  __device__ __forceinline__ void fma(const float* c, float s0, float s1) {
    ffma2(v, *reinterpret_cast<const unsigned long long*>(c), pk(s0, s1));
  }
  // the same with the coefficient pair by value (no addressable temporary)
  __device__ __forceinline__ void fmav(float c0, float c1, float s0, float s1) {
    ffma2(v, pk(c0, c1), pk(s0, s1));
  }
  __device__ __forceinline__ float re() const { return lo_f(v); }
  __device__ __forceinline__ float im() const { return hi_f(v); }
};
template <>
struct Acc2<double> {
  double r, i;
  __device__ __forceinline__ void zero() { r = 0.0; i = 0.0; }
  __device__ __forceinline__ void fma(const double* c, double s0, double s1) {
    r = ::fma(c[0], s0, r);
    i = ::fma(c[1], s1, i);
  }
  __device__ __forceinline__ void fmav(double c0, double c1, double s0, double s1) {
    r = ::fma(c0, s0, r);
    i = ::fma(c1, s1, i);
  }
  __device__ __forceinline__ double re() const { return r; }
  __device__ __forceinline__ double im() const { return i; }
};

// |W| of a complex value: fp32 through one reciprocal square root (rsqrtf, a few ulp), fp64
// exact.
__device__ __forceinline__ float cabs_w(float re, float im) {
  const float s2 = fmaf(re, re, im * im);
  return s2 > 0.0f ? s2 * rsqrtf(s2) : 0.0f;
}
__device__ __forceinline__ double cabs_w(double re, double im) { return sqrt(re * re + im * im); }
// exp(x) for the softmax weights (x <= 0): fp32 the fast exponential, fp64 exact.
__device__ __forceinline__ float exp_w(float x) { return __expf(x); }
__device__ __forceinline__ double exp_w(double x) { return exp(x); }

// Partition of an octave's `count` scales into blocks of 1..4 (each block shares the pair
// sums of its tap loop).
__device__ __forceinline__ int block_size(int rem) {
  if (rem <= SBMAX) return rem;
  if (rem <= 2 * SBMAX) return (rem + 1) / 2;
  return SBMAX;
}

// Coefficient table of an octave, per tap k in [0, half] and scale slot s:
//   [0] sym(re)  = (h_re[c+k] + h_re[c-k]) / 2   (k = 0: h_re[c])
//   [1] anti(im) = (h_im[c+k] - h_im[c-k]) / 2   (k = 0: 0)
//   [2] anti(re) = (h_re[c+k] - h_re[c-k]) / 2   (k = 0: 0)
//   [3] sym(im)  = (h_im[c+k] + h_im[c-k]) / 2   (k = 0: h_im[c])
// so that  re += [0] (xl + xr) + [2] (xl - xr),  im += [1] (xl - xr) + [3] (xl + xr)  exactly
// reproduces sum_k h[c+k] x[n - dk] over k = -half..half of the octave.
// build_coef records per scale slot s whether its [2]/[3] halves are nonzero (anti[s]) and the
// last tap k with a nonzero coefficient (klast[s]): the taps past it are zero (a scale's filter
// is shorter than the octave's widest), so the scale leaves the tap loop there -- exact for any
// filter tensor.
// fold_coef: folded coefficients of tap k of scale slot s, straight from the filter tensor.
template <typename A>
__device__ __forceinline__ void fold_coef(const FwdParams<A>& p, const Oct& O, int s, int k,
                                          A (&t)[4]) {
  const A* H = static_cast<const A*>(p.h);
  const int C = p.channels;
  const int hcols = 2 * p.center + 1;
  const int gs = p.order[O.begin + s];
  A ip = 0, im = 0;
  // every tap of the octave's window is used (fdwt/cwt.py:566-578 slices the columns
  // center-half .. center+half for all scales of the stage), so filters that are nonzero past a
  // scale's support give the reference's results too
  const A* hr = H + static_cast<int64_t>(gs * C) * hcols + p.center;
  const A rp = __ldg(hr + k);
  const A rm = __ldg(hr - k);
  if (C == 2) {
    ip = __ldg(hr + hcols + k);
    im = __ldg(hr + hcols - k);
  }
  if (k == 0) {
    t[0] = rp;
    t[1] = 0;
    t[2] = 0;
    t[3] = ip;
  } else {
    t[0] = (rp + rm) * A(0.5);
    t[1] = (ip - im) * A(0.5);
    t[2] = (rp - rm) * A(0.5);
    t[3] = (ip + im) * A(0.5);
  }
}

template <typename A>
__device__ void build_coef(const FwdParams<A>& p, const Oct& O, A* tab, int* anti, int* klast) {
  const int cnt = O.count, K = O.half;
  const int tid = threadIdx.x;
  for (int s = tid; s < cnt; s += NT) {
    anti[s] = 0;
    klast[s] = 0;
  }
  __syncthreads();
  const bool in_smem = cnt * (K + 1) * 4 <= p.coef_cap;
  for (int w = tid; w < cnt * (K + 1); w += NT) {
    const int s = w % cnt, k = w / cnt;
    A t[4];
    fold_coef<A>(p, O, s, k, t);
    if (in_smem) {
      A* d = tab + (k * cnt + s) * 4;
      d[0] = t[0];
      d[1] = t[1];
      d[2] = t[2];
      d[3] = t[3];
    }
    const bool an = t[2] != A(0) || t[3] != A(0);
    if (an) atomicOr(&anti[s], 1);
    if (k > 0 && (an || t[0] != A(0) || t[1] != A(0))) atomicMax(&klast[s], k);
  }
}

// The window state of an item's tap loop: the two register windows, the next load pointers
// (or index, when clamped) and the block's coefficients of the current tap.
template <typename A>
struct TapState {
  A L[PF], R[PF];
  const A* pl;
  const A* pr;
  int qr;
  const A* tk;
  int k;
};

// Taps state.k .. kend for the scales M .. SB-1 of the block (the earlier ones have left).
template <typename A, int SB, int M, bool SYM, bool GTAB, bool CLAMP>
__device__ __forceinline__ void conv_seg(const FwdParams<A>& p, const Oct& O,
                                         const A* __restrict__ xb, int lim, int s0, int kend,
                                         TapState<A>& st, Acc2<A> (&acc)[SB][PF]) {
  const int dil = O.dil, cnt = O.count;
#pragma unroll 5
  for (; st.k <= kend; ++st.k) {
    st.tk += 4 * cnt;
#pragma unroll
    for (int i = PF - 1; i > 0; --i) st.L[i] = st.L[i - 1];
#pragma unroll
    for (int i = 0; i < PF - 1; ++i) st.R[i] = st.R[i + 1];
    st.L[0] = *st.pl;
    st.pl -= dil;
    if (CLAMP) {
      st.R[PF - 1] = xb[min(st.qr, lim)];
      st.qr += dil;
    } else {
      st.R[PF - 1] = *st.pr;
      st.pr += dil;
    }
    alignas(16) A t[SB][4];
#pragma unroll
    for (int s = M; s < SB; ++s) {
      if (GTAB) {
        fold_coef<A>(p, O, s0 + s, st.k, t[s]);
      } else {
        const A* c = st.tk + 4 * s;
        t[s][0] = c[0];
        t[s][1] = c[1];
        if (!SYM) {
          t[s][2] = c[2];
          t[s][3] = c[3];
        }
      }
    }
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      const A sum = st.L[i] + st.R[i], dif = st.L[i] - st.R[i];
#pragma unroll
      for (int s = M; s < SB; ++s) {
        acc[s][i].fma(t[s], sum, dif);
        if (!SYM) acc[s][i].fma(t[s] + 2, dif, sum);
      }
    }
  }
}

// The segments of a block: scale m is the first active one on the taps past the prefix maximum
// of the earlier scales' last taps, up to its own (prefix maximum) last tap.
template <typename A, int SB, int M, bool SYM, bool GTAB, bool CLAMP>
__device__ __forceinline__ void conv_segs(const FwdParams<A>& p, const Oct& O,
                                          const A* __restrict__ xb, int lim, int s0,
                                          const int* klast, int e, TapState<A>& st,
                                          Acc2<A> (&acc)[SB][PF]) {
  if constexpr (M < SB) {
    e = max(e, klast[s0 + M]);
    conv_seg<A, SB, M, SYM, GTAB, CLAMP>(p, O, xb, lim, s0, e, st, acc);
    conv_segs<A, SB, M + 1, SYM, GTAB, CLAMP>(p, O, xb, lim, s0, klast, e, st, acc);
  }
}

// (re, im) of the SB scales of a block for the item's PF outputs.  Coefficients come from the
// shared table (GTAB = false) or are folded from the global filter tensor per tap (GTAB).
// CLAMP: some right-window position passes the buffer's last index (items past the kept range).
template <typename A, int SB, bool SYM, bool GTAB, bool CLAMP>
__device__ __forceinline__ void conv_block(const FwdParams<A>& p, const Oct& O,
                                           const A* __restrict__ xb, int phi, int u0, int limit,
                                           int org, const A* __restrict__ tab, int s0,
                                           const int* klast, Acc2<A> (&acc)[SB][PF]) {
  const int dil = O.dil;
  const int c0 = phi + dil * u0 - org;  // buffer index of the item's first output
  const int lim = limit - org;          // last buffer index
  TapState<A> st;
#pragma unroll
  for (int i = 0; i < PF; ++i) {
    const int q = CLAMP ? min(c0 + dil * i, lim) : c0 + dil * i;
    st.L[i] = st.R[i] = xb[q];
  }
  st.tk = tab + 4 * s0;  // the block's coefficients of tap 0
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    alignas(16) A t[4];
    if (GTAB) {
      fold_coef<A>(p, O, s0 + s, 0, t);
    } else {
      const A* c = st.tk + 4 * s;
      t[0] = c[0];
      t[1] = c[1];
      t[2] = c[2];
      t[3] = c[3];
    }
#pragma unroll
    for (int i = 0; i < PF; ++i) {
      acc[s][i].zero();
      acc[s][i].fma(t, st.L[i], A(0));        // re += h_re[c] x
      acc[s][i].fma(t + 2, A(0), st.L[i]);    // im += h_im[c] x
    }
  }
  st.pl = xb + (c0 - dil);         // next left load
  st.pr = xb + (c0 + dil * PF);    // next right load (no clamp)
  st.qr = c0 + dil * PF;           // next right load index (clamp)
  st.k = 1;
  conv_segs<A, SB, 0, SYM, GTAB, CLAMP>(p, O, xb, lim, s0, klast, 0, st, acc);
}

// One block for one item, then its epilogue.
template <typename T, typename A, int EPI, bool GT, int SB, bool SYM>
__device__ __forceinline__ void do_block(const FwdParams<A>& p, const Oct& O, const A* xb,
                                         const A* tab, int s0, const int* klast, int phi, int u0,
                                         int64_t row, const Span& sp, A (&mix)[PF], A (&sm_m)[PF],
                                         A (&sm_l)[PF], A (&sm_num)[PF]) {
  const int64_t n = p.n;
  const int64_t tend = sp.tend;  // outputs past the kept range read clamped windows (limit =
                                 // the last buffer position) and are not stored
  const int dil = O.dil;
  Acc2<A> acc[SB][PF];
  int K = 0;  // the block's last nonzero tap
#pragma unroll
  for (int s = 0; s < SB; ++s) K = max(K, klast[s0 + s]);
  const bool clamp = phi + dil * (u0 + PF - 1 + K) > sp.limit;
  if (clamp) conv_block<A, SB, SYM, GT, true>(p, O, xb, phi, u0, sp.limit, sp.org, tab, s0, klast, acc);
  else conv_block<A, SB, SYM, GT, false>(p, O, xb, phi, u0, sp.limit, sp.org, tab, s0, klast, acc);
  const int C = p.channels;
#pragma unroll
  for (int s = 0; s < SB; ++s) {
    const int gs = p.order[O.begin + s0 + s];
    if (EPI == EPI_STORE) {
      A* yb = static_cast<A*>(p.y) + ((row * p.n_scales + gs) * n) * C;
      {
#pragma unroll
        for (int i = 0; i < PF; ++i) {
          const int64_t ni = phi + static_cast<int64_t>(dil) * (u0 + i);
          if (ni < tend) {
            if (C == 2) {
              typename std::conditional<std::is_same<A, float>::value, float2, double2>::type v;
              v.x = acc[s][i].re();
              v.y = acc[s][i].im();
              *reinterpret_cast<decltype(v)*>(yb + 2 * ni) = v;
            } else {
              yb[ni] = acc[s][i].re();
            }
          }
        }
      }
    } else if (EPI == EPI_MIX) {
      const int64_t d = row % p.dim;
      const A av = static_cast<const A*>(p.a)[d * p.n_scales + gs];
      const A bv = static_cast<const A*>(p.b)[d * p.n_scales + gs];
#pragma unroll
      for (int i = 0; i < PF; ++i) {
        const A re = acc[s][i].re(), im = acc[s][i].im();
        const A mag = C == 2 ? cabs_w(re, im) : fabs(re);
        mix[i] += av * mag + bv * re;
      }
    } else {
      const A* V = static_cast<const A*>(p.a);
      const int64_t g = row / p.dim, c = row % p.dim;
#pragma unroll
      for (int i = 0; i < PF; ++i) {
        const int64_t ni = phi + static_cast<int64_t>(dil) * (u0 + i);
        const A re = acc[s][i].re(), im = acc[s][i].im();
        const A a = cabs_w(re, im) * p.inv_tau;
        A v;
        if (p.v_pos) v = ni < tend ? V[(g * p.n_scales + gs) * n + ni] : A(0);
        else v = V[c * p.n_scales + gs];
        // online softmax: one exponential, of -|a - m| (the larger side's weight is exactly 1)
        const A dlt = a - sm_m[i];
        const A ex = exp_w(-fabs(dlt));
        if (dlt > A(0)) {
          sm_l[i] = sm_l[i] * ex + A(1);
          sm_num[i] = sm_num[i] * ex + v;
          sm_m[i] = a;
        } else {
          sm_l[i] = sm_l[i] + ex;
          sm_num[i] = sm_num[i] + ex * v;
        }
      }
    }
  }
}

template <typename T, typename A, int EPI, bool GT, int SB>
__device__ __forceinline__ void do_block_sym(const FwdParams<A>& p, const Oct& O, const A* xb,
                                             const A* tab, int s0, const int* K, bool sym, int phi, int u0,
                                             int64_t row, const Span& sp, A (&mix)[PF],
                                             A (&sm_m)[PF], A (&sm_l)[PF], A (&sm_num)[PF]) {
  if (sym) do_block<T, A, EPI, GT, SB, true>(p, O, xb, tab, s0, K, phi, u0, row, sp, mix, sm_m, sm_l, sm_num);
  else do_block<T, A, EPI, GT, SB, false>(p, O, xb, tab, s0, K, phi, u0, row, sp, mix, sm_m, sm_l, sm_num);
}

// Dispatch a block of runtime size 1..4.
template <typename T, typename A, int EPI, bool GT>
__device__ __forceinline__ void run_block(const FwdParams<A>& p, const Oct& O, const A* xb,
                                          const A* tab, int s0, int sb, const int* K, bool sym,
                                          int phi, int u0, int64_t row, const Span& sp,
                                          A (&mix)[PF], A (&sm_m)[PF], A (&sm_l)[PF],
                                          A (&sm_num)[PF]) {
  switch (sb) {
    case 1: do_block_sym<T, A, EPI, GT, 1>(p, O, xb, tab, s0, K, sym, phi, u0, row, sp, mix, sm_m, sm_l, sm_num); break;
    case 2: do_block_sym<T, A, EPI, GT, 2>(p, O, xb, tab, s0, K, sym, phi, u0, row, sp, mix, sm_m, sm_l, sm_num); break;
    case 3: do_block_sym<T, A, EPI, GT, 3>(p, O, xb, tab, s0, K, sym, phi, u0, row, sp, mix, sm_m, sm_l, sm_num); break;
    case 4: do_block_sym<T, A, EPI, GT, 4>(p, O, xb, tab, s0, K, sym, phi, u0, row, sp, mix, sm_m, sm_l, sm_num); break;
    default: do_block_sym<T, A, EPI, GT, SBMAX>(p, O, xb, tab, s0, K, sym, phi, u0, row, sp, mix, sm_m, sm_l, sm_num); break;
  }
}

// x_{j+1} from x_j (dilation dil) over the buffer [org, org + span): zero outside live and where
// the window leaves the buffer (positions no kept output reads, see the tile notes above).
template <typename A>
__device__ void lowpass_step(const FwdParams<A>& p, const A* cur, A* nxt, int dil, int live,
                             int org, int span) {
  const int n = static_cast<int>(p.n);
  const int ext = -org;
  const int reach = p.n_lp > 0 ? p.lp_t[p.n_lp - 1] * dil : 0;
  for (int q = static_cast<int>(threadIdx.x) + org; q < org + span; q += NT) {
    A v = A(0);
    if (q >= -live && q < n + live && q - reach >= org && q + reach < org + span) {
      v = p.lpp[0] * cur[(q + ext)];
      if (p.lp_sym) {
        for (int i = 0; i < p.n_lp; ++i) {
          const int t = p.lp_t[i];
          v = fma(p.lp_p[i], cur[(q - dil * t + ext)] + cur[(q + dil * t + ext)],
                  v);
        }
      } else {
        for (int i = 0; i < p.n_lp; ++i) {
          const int t = p.lp_t[i];
          v = fma(p.lp_p[i], cur[(q - dil * t + ext)], v);
          v = fma(p.lp_m[i], cur[(q + dil * t + ext)], v);
        }
      }
    }
    nxt[(q + ext)] = v;
  }
}

// GT: the octaves' coefficient tables do not fit the shared budget (read from the filters).
template <typename T, typename A, int EPI, bool GT>
__global__ void __launch_bounds__(NT, (sizeof(A) == 4 && EPI == EPI_STORE) ? 2 : 1)
cwt_forward_kernel(const __grid_constant__ FwdParams<A> p) {
  extern __shared__ __align__(16) unsigned char smem[];
  A* buf0 = reinterpret_cast<A*>(smem);
  A* buf1 = buf0 + p.buf_len;
  A* tab = reinterpret_cast<A*>(smem + p.coef_off);
  A* extra = reinterpret_cast<A*>(smem + p.extra_off);
  __shared__ int anti[kMaxScales];   // per scale slot of the octave: antisymmetric halves
  __shared__ int klast[kMaxScales];  // per scale slot: last tap with a nonzero coefficient
  const int64_t row = blockIdx.x / p.ntile;
  const int tile = static_cast<int>(blockIdx.x - row * p.ntile);
  const int n = static_cast<int>(p.n);
  const int tid = threadIdx.x;
  Span sp;
  sp.t0 = p.t_base + tile * p.t_len;
  const int tk = min(p.t_len, p.t_end - sp.t0);  // owned (kept) positions [t0, t0 + tk)
  sp.tend = sp.t0 + tk;
  sp.org = sp.t0 - p.halo;
  const int span = tk + 2 * p.halo;
  sp.limit = sp.org + span - 1;

  const RowRef<const T> xr = row_ref(static_cast<const T*>(p.x), p, row);
  for (int i = tid; i < span; i += NT) {
    const int q = sp.org + i;
    buf0[(i)] = (q >= 0 && q < n) ? to_acc<T>(xr[q]) : A(0);
  }
  if (EPI == EPI_MIX) {
    for (int i = tid; i < tk; i += NT) extra[i] = A(0);
  } else if (EPI == EPI_SOFTMAX) {
    for (int i = tid; i < tk; i += NT) {
      extra[i] = -INFINITY;
      extra[tk + i] = A(0);
      extra[2 * tk + i] = A(0);
    }
  }
  __syncthreads();

  A* cur = buf0;
  A* nxt = buf1;
  for (int j = 0; j < p.n_oct; ++j) {
    const Oct& O = p.oct[j];
    if (O.count > 0 && EPI != EPI_PYR) {
      build_coef<A>(p, O, tab, anti, klast);
      __syncthreads();
      const int dil = O.dil;
      const int runs = (static_cast<int>((tk + dil - 1) / dil) + PF - 1) / PF;
      const int items = dil * runs;
      int nblk = 0;
      for (int s0 = 0; s0 < O.count; s0 += block_size(O.count - s0)) ++nblk;
      const int lg = __ffs(dil) - 1;  // dil = 2^lg
      if (EPI == EPI_STORE) {
        // spread (block, item) pairs over the threads: work unit w = (block, item), walked
        // incrementally (no divisions)
        int blk = 0, s0 = 0, it = tid;
        while (blk < nblk && it >= items) {
          it -= items;
          s0 += block_size(O.count - s0);
          ++blk;
        }
        for (; blk < nblk;) {
          const int sb = block_size(O.count - s0);
          const int phi = it & (dil - 1), u0 = (it >> lg) * PF;
          if (phi < tk) {
            bool sym = true;
            for (int s = 0; s < sb; ++s) sym = sym && anti[s0 + s] == 0;
            A mix[PF], m_[PF], l_[PF], num_[PF];
            run_block<T, A, EPI, GT>(p, O, cur, tab, s0, sb, klast, sym, sp.t0 + phi, u0, row, sp,
                                     mix, m_, l_, num_);
          }
          it += NT;
          while (blk < nblk && it >= items) {
            it -= items;
            s0 += block_size(O.count - s0);
            ++blk;
          }
        }
      } else {
        for (int it = tid; it < items; it += NT) {
          const int phi = it & (dil - 1), u0 = (it >> lg) * PF;
          if (phi >= tk) continue;
          A mix[PF], sm_m[PF], sm_l[PF], sm_num[PF];
#pragma unroll
          for (int i = 0; i < PF; ++i) {
            const int li = phi + dil * (u0 + i);  // tile-local output index
            mix[i] = A(0);
            if (EPI == EPI_SOFTMAX && li < tk) {
              sm_m[i] = extra[li];
              sm_l[i] = extra[tk + li];
              sm_num[i] = extra[2 * tk + li];
            } else {
              sm_m[i] = -INFINITY;
              sm_l[i] = A(0);
              sm_num[i] = A(0);
            }
          }
          int s0 = 0;
          for (int b = 0; b < nblk; ++b) {
            const int sb = block_size(O.count - s0);
            bool sym = true;
            for (int s = 0; s < sb; ++s) sym = sym && anti[s0 + s] == 0;
            run_block<T, A, EPI, GT>(p, O, cur, tab, s0, sb, klast, sym, sp.t0 + phi, u0, row, sp,
                                     mix, sm_m, sm_l, sm_num);
            s0 += sb;
          }
#pragma unroll
          for (int i = 0; i < PF; ++i) {
            const int li = phi + dil * (u0 + i);
            if (li < tk) {
              if (EPI == EPI_MIX) {
                extra[li] += mix[i];
              } else {
                extra[li] = sm_m[i];
                extra[tk + li] = sm_l[i];
                extra[2 * tk + li] = sm_num[i];
              }
            }
          }
        }
      }
      __syncthreads();
    }
    if (j + 1 < p.n_oct) {
      lowpass_step<A>(p, cur, nxt, O.dil, p.oct[j + 1].live, sp.org, span);
      __syncthreads();
      if (EPI == EPI_PYR && p.pyr_off[j + 1] >= 0) {
        // x_{j+1} on the owned positions inside its live extent
        const int lv = p.oct[j + 1].live;
        A* dst = p.pyr + row * p.pyr_len + p.pyr_off[j + 1] + lv;
        const int lo = max(sp.t0, -lv), hi = min(sp.tend, n + lv);
        for (int q = lo + tid; q < hi; q += NT) dst[q] = nxt[(q - sp.org)];
      }
      A* t = cur;
      cur = nxt;
      nxt = t;
    }
  }

  if (EPI == EPI_MIX) {
    const RowRef<A> yr = row_ref(static_cast<A*>(p.y), p, row);
    const A bias = p.bias ? static_cast<const A*>(p.bias)[row % p.dim] : A(0);
    for (int i = tid; i < tk; i += NT) yr[sp.t0 + i] = extra[i] + bias;
  } else if (EPI == EPI_SOFTMAX) {
    A* o = static_cast<A*>(p.y) + row * p.n + sp.t0;
    A* mo = static_cast<A*>(p.m_out) + row * p.n + sp.t0;
    A* lo = static_cast<A*>(p.l_out) + row * p.n + sp.t0;
    for (int i = tid; i < tk; i += NT) {
      const A l = extra[tk + i];
      o[i] = extra[2 * tk + i] / l;
      mo[i] = extra[i];
      lo[i] = l;
    }
  }
}

// ------------------------------------------------------------------------------ host

struct Geometry {
  int ext;            // buffer reach
  std::vector<int> live;
};

inline int check_plan(const fdwt_morlet_plan* pl, int64_t n) {
  if (pl == nullptr) return FDWT_ERR_INVALID;
  if (pl->n_octaves < 1 || pl->n_octaves > kMaxOct) return FDWT_ERR_INVALID;
  if (pl->n_scales < 1 || pl->n_scales > kMaxScales) return FDWT_ERR_INVALID;
  if (pl->channels != 1 && pl->channels != 2) return FDWT_ERR_INVALID;
  if (pl->c_lp < 0 || pl->c_lp > kMaxC) return FDWT_ERR_UNSUPPORTED;
  if (pl->n_octaves > 1 && pl->c_lp < 1) return FDWT_ERR_INVALID;
  if (n < 1) return FDWT_ERR_INVALID;
  int total = 0;
  for (int j = 0; j < pl->n_octaves; ++j) {
    if (pl->oct_count[j] < 0 || pl->oct_half[j] < 0 || pl->oct_half[j] > pl->center)
      return FDWT_ERR_INVALID;
    if (pl->oct_count[j] > 0 && pl->oct_begin[j] + pl->oct_count[j] > pl->n_scales)
      return FDWT_ERR_INVALID;
    total += pl->oct_count[j];
    for (int s = 0; s < pl->oct_count[j]; ++s) {
      const int k = pl->oct_begin[j] + s;
      if (pl->order[k] < 0 || pl->order[k] >= pl->n_scales) return FDWT_ERR_INVALID;
      if (pl->support[k] < 0 || pl->support[k] > pl->oct_half[j]) return FDWT_ERR_INVALID;
    }
  }
  if (total != pl->n_scales) return FDWT_ERR_INVALID;
  return FDWT_OK;
}

inline Geometry geometry(const fdwt_morlet_plan* pl) {
  Geometry g;
  const int J = pl->n_octaves;
  g.live.assign(J, 0);
  for (int j = 0; j + 1 < J; ++j)
    g.live[j + 1] = std::min(pl->margins[j + 1], g.live[j] + pl->c_lp * (1 << j));
  int ext = 0;
  for (int j = 0; j < J; ++j) {
    const int dil = 1 << j;
    if (pl->oct_count[j] > 0) ext = std::max(ext, pl->oct_half[j] * dil);
    ext = std::max(ext, g.live[j]);
    if (j + 1 < J) ext = std::max(ext, g.live[j + 1] + pl->c_lp * dil);
  }
  g.ext = ext + 8;
  return g;
}

template <typename A>
void fill_common(FwdParams<A>& p, const fdwt_morlet_plan* pl, const Geometry& g, int64_t n) {
  p.n = n;
  p.n_oct = pl->n_octaves;
  p.n_scales = pl->n_scales;
  p.channels = pl->channels;
  p.center = pl->center;
  p.c_lp = pl->c_lp;
  p.ext = g.ext;
  double lp_max = 0.0;
  for (int t = 0; t <= 2 * pl->c_lp; ++t) lp_max = std::max(lp_max, std::fabs(pl->lowpass[t]));
  p.n_lp = 0;
  p.lp_sym = 1;
  for (int t = 0; t <= kMaxC; ++t) {
    p.lpp[t] = t <= pl->c_lp ? static_cast<A>(pl->lowpass[pl->c_lp + t]) : A(0);
    p.lpm[t] = t <= pl->c_lp ? static_cast<A>(pl->lowpass[pl->c_lp - t]) : A(0);
    if (t >= 1 && t <= pl->c_lp) {
      const double a = pl->lowpass[pl->c_lp + t], b = pl->lowpass[pl->c_lp - t];
      if (std::fabs(a) > 1e-13 * lp_max || std::fabs(b) > 1e-13 * lp_max) {
        p.lp_t[p.n_lp] = t;
        p.lp_p[p.n_lp] = static_cast<A>(a);
        p.lp_m[p.n_lp] = static_cast<A>(b);
        if (a != b) p.lp_sym = 0;
        ++p.n_lp;
      }
    }
  }
  for (int j = 0; j < pl->n_octaves; ++j) {
    p.oct[j].dil = 1 << j;
    p.oct[j].half = pl->oct_half[j];
    p.oct[j].begin = pl->oct_begin[j];
    p.oct[j].count = pl->oct_count[j];
    p.oct[j].live = g.live[j];
  }
  for (int k = 0; k < pl->n_scales; ++k) {
    p.order[k] = pl->order[k];
    p.support[k] = pl->support[k];
  }
}

// Reach of a tile's pyramid buffers past both ends of its owned range (the H of the tile
// notes): the filter reach of each octave and the half-band chain below it.  pyr_only: the
// half-band chain alone (x_1 .. x_J-1 on the owned range).
inline int tile_halo(const fdwt_morlet_plan* pl, bool pyr_only) {
  int H = 0;
  for (int j = pl->n_octaves - 1; j >= 0; --j) {
    const int dil = 1 << j;
    const int own = (!pyr_only && pl->oct_count[j] > 0) ? pl->oct_half[j] * dil : 0;
    const int chain = j + 1 < pl->n_octaves ? H + pl->c_lp * dil : 0;
    H = std::max(own, chain);
  }
  return H + 8;
}

// Shared-memory layout of a forward launch whose CTAs own t_len positions and whose buffers
// reach `halo` past both ends: fills the offsets of p, returns the bytes (0: does not fit).
template <typename A, int EPI>
size_t fwd_layout(FwdParams<A>& p, const fdwt_morlet_plan* pl, int64_t t_len, int halo,
                  size_t budget) {
  const int64_t span = t_len + 2 * static_cast<int64_t>(halo);
  if (span > 0x3fffffffLL) return 0;
  p.buf_len = static_cast<int>(span + 8);  // linear buffers (no padding)
  // the coefficient table takes what is left of the shared budget (up to the largest octave)
  int coef = 0;
  if (EPI != EPI_PYR)
    for (int j = 0; j < pl->n_octaves; ++j)
      coef = std::max(coef, pl->oct_count[j] * (pl->oct_half[j] + 1) * 4);
  const size_t nextra = (EPI == EPI_MIX ? 1 : EPI == EPI_SOFTMAX ? 3 : 0) *
                        static_cast<size_t>(t_len);
  const size_t fixed = 2 * static_cast<size_t>(p.buf_len) * sizeof(A) + 64 + nextra * sizeof(A);
  if (fixed > budget) return 0;
  const size_t room = (budget - fixed) / sizeof(A);
  if (static_cast<size_t>(coef) > room) coef = static_cast<int>(room / 4 * 4);
  coef = std::min(coef, 24 * 1024 / static_cast<int>(sizeof(A)) * 4);  // keep occupancy
  p.coef_cap = coef;
  size_t off = 2 * static_cast<size_t>(p.buf_len) * sizeof(A);
  off = (off + 15) / 16 * 16;
  p.coef_off = static_cast<int>(off);
  off += static_cast<size_t>(coef) * sizeof(A);
  off = (off + 15) / 16 * 16;
  p.extra_off = static_cast<int>(off);
  off += nextra * sizeof(A);
  const size_t smem = off + 16;
  return smem > budget ? 0 : smem;
}

// Tiles of the range [t_base, t_end) for a forward launch: the longest tile (a power of two,
// at least 256) whose layout keeps two CTAs per SM, else the longest that fits at all; a test
// may force the tile length (fdwt_set_cwt_tile_test).  Returns the shared bytes (0: none fits).
template <typename A, int EPI>
size_t plan_fwd_tiles(FwdParams<A>& p, const fdwt_morlet_plan* pl, int64_t t_base,
                      int64_t t_end, int halo, size_t budget) {
  const int64_t range = t_end - t_base;
  p.t_base = static_cast<int32_t>(t_base);
  p.t_end = static_cast<int32_t>(t_end);
  p.halo = halo;
  auto take = [&](int64_t tl) -> size_t {
    const size_t sm = fwd_layout<A, EPI>(p, pl, tl, halo, budget);
    if (sm) {
      p.t_len = static_cast<int32_t>(tl);
      p.ntile = static_cast<int32_t>(cdiv(range, tl));
    }
    return sm;
  };
  const int forced = cwt_tile_test();
  if (forced > 0) return take(std::min<int64_t>(forced, range));
  const size_t two_per_sm = std::min(budget, static_cast<size_t>(113) << 10);
  for (const size_t cap : {two_per_sm, budget})
    for (int64_t tl = int64_t(1) << 16; tl >= 256; tl >>= 1) {
      const size_t sm = fwd_layout<A, EPI>(p, pl, std::min(tl, range), halo, cap);
      if (sm) return take(std::min(tl, range));
    }
  return 0;
}

template <typename T, typename A, int EPI>
int launch_forward(FwdParams<A>& p, int64_t rows, size_t smem, cudaStream_t stream) {
  if (rows * p.ntile > 0x7fffffffLL) return FDWT_ERR_UNSUPPORTED;
  bool gt = false;  // some octave's coefficient table does not fit the shared table
  if (EPI != EPI_PYR)
    for (int j = 0; j < p.n_oct; ++j)
      if (p.oct[j].count * (p.oct[j].half + 1) * 4 > p.coef_cap) gt = true;
  auto kern = gt ? cwt_forward_kernel<T, A, EPI, true> : cwt_forward_kernel<T, A, EPI, false>;
  int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
  if (st != FDWT_OK) return st;
  if ((st = pre_launch(stream)) != FDWT_OK) return st;
  kern<<<static_cast<unsigned>(rows * p.ntile), NT, smem, stream>>>(p);
  return launch_status();
}

template <typename T, typename A, int EPI>
int run_forward(int64_t rows, int64_t n, const void* x, const void* h,
                const fdwt_morlet_plan* pl, void* y, const void* a, const void* b,
                void* m_out, void* l_out, int64_t dim, int v_pos, double inv_tau,
                cudaStream_t stream, int tok = 0, const void* bias = nullptr) {
  int st = check_plan(pl, n);
  if (st != FDWT_OK) return st;
  if (rows == 0) return FDWT_OK;
  if (rows > 0x7fffffffLL || n > 0x3fffffffLL) return FDWT_ERR_UNSUPPORTED;
  const Geometry g = geometry(pl);
  FwdParams<A> p{};
  fill_common(p, pl, g, n);
  p.rows = rows;
  p.x = x;
  p.h = h;
  p.y = y;
  p.a = a;
  p.b = b;
  p.m_out = m_out;
  p.l_out = l_out;
  p.dim = dim;
  p.v_pos = v_pos;
  p.inv_tau = static_cast<A>(inv_tau);
  p.tok = tok;
  p.bias = bias;
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 2048;
  // a whole row per CTA when it fits (buffers over the row's own reach); time tiles otherwise
  size_t smem = 0;
  if (cwt_tile_test() <= 0) {
    smem = fwd_layout<A, EPI>(p, pl, n, g.ext, budget);
    if (smem) {
      p.ntile = 1;
      p.t_len = static_cast<int32_t>(n);
      p.t_base = 0;
      p.t_end = static_cast<int32_t>(n);
      p.halo = g.ext;
    }
  }
  if (!smem) smem = plan_fwd_tiles<A, EPI>(p, pl, 0, n, tile_halo(pl, false), budget);
  if (!smem) return FDWT_ERR_UNSUPPORTED;
  return launch_forward<T, A, EPI>(p, rows, smem, stream);
}

// x_1 .. x_J-1 of every row into pyr (row stride pyr_len; level j at pyr_off[j] >= 0, stored on
// [-live_j, n + live_j)): the half-band chain of the forward over tiles of [-e, n + e), e the
// largest live extent.
template <typename A>
int run_pyramid(int64_t rows, int64_t n, const void* x, const fdwt_morlet_plan* pl,
                const Geometry& g, A* pyr, int64_t pyr_len, const int32_t* pyr_off,
                cudaStream_t stream, int tok = 0, int64_t dim = 1) {
  if (rows == 0 || pl->n_octaves < 2) return FDWT_OK;
  FwdParams<A> p{};
  fill_common(p, pl, g, n);
  p.rows = rows;
  p.tok = tok;
  p.dim = dim;
  p.x = x;
  p.pyr = pyr;
  p.pyr_len = pyr_len;
  for (int j = 0; j < kMaxOct; ++j) p.pyr_off[j] = pyr_off[j];
  int e = 0;
  for (int j = 0; j < pl->n_octaves; ++j) e = std::max(e, g.live[j]);
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 2048;
  const size_t smem = plan_fwd_tiles<A, EPI_PYR>(p, pl, -e, n + e, tile_halo(pl, true), budget);
  if (!smem) return FDWT_ERR_UNSUPPORTED;
  return launch_forward<A, A, EPI_PYR>(p, rows, smem, stream);
}

}  // namespace cwtk
}  // namespace fdwt
