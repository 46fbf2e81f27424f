// Fused multilevel DWT analysis and its exact transpose for sm_100a.
//
// One CTA owns one signal row and runs every level of a multilevel transform in a single
// launch: the input row is streamed from HBM in tiles (boundary extension applied while
// staging), every intermediate approximation stays resident in shared memory, and only the
// details and the final approximation are written.  When the resident approximations of a
// long row do not fit in shared memory the host splits the levels into consecutive launches
// ("segments") that hand the approximation over through a caller-provided workspace.
//
// The taps live in the kernel's parameter block (constant bank), so every tap product is one
// FMA with a constant operand.  Each thread computes V consecutive outputs from a register
// window of its inputs; shared-memory arrays use a padded layout so that the windows of a
// warp's 32 lanes fall into distinct banks.
//
// Semantics follow the reference's Triton kernels fdwt/kernels/dwt.py:73-98 (analysis,
// index-arithmetic boundary extension _ext_index 52-70) and 101-175 (exact transpose).  The
// transpose is evaluated as y = Fold(z): z[p] = sum_{2o+off-j = p} h0[j] a[o] + h1[j] d[o] on
// the extended range [off-L+1, 2(nc-1)+off], polyphase-split so each output visits only the
// taps of its parity, and every extended position outside [0, n) is folded back onto
// ext(p) (periodic wrap, symmetric / reflect mirror, periodization's repeated last sample);
// zero mode drops them.
#pragma once
#include <algorithm>
#include <vector>

#include "common.cuh"

namespace fdwt {
namespace dwtk {

constexpr int kThreads = 256;
constexpr int kMaxLevels = 40;

struct Level {
  int64_t n_in;    // analysis: input length;  synthesis: output length
  int64_t n_coef;  // coefficient length
  int64_t a_len;   // analysis: stored approximation length (n_coef + pad);
                   // synthesis: length of the incoming approximation (>= n_coef)
  int64_t P;       // period of the (normalized) boundary mode for the signal length
  void* detail;    // analysis: detail output; synthesis: detail input (nullptr = zeros)
  int32_t mode;    // normalized boundary mode
  int32_t fold_n;  // synthesis: number of exterior positions folded back (0 in zero mode)
};

template <typename A, int LM>
struct Params {
  int64_t rows;
  const void* src;  // analysis: (rows, lv[0].n_in); synthesis: (rows, lv[0].a_len)
  void* dst;        // analysis: (rows, lv[nlev-1].a_len); synthesis: (rows, lv[nlev-1].n_in)
  int32_t nlev;
  int32_t off;
  int32_t buf_len[2];  // element offsets of the resident buffers
  int32_t stage_len;   // element count of one stage buffer (synthesis uses two)
  A h0[LM];
  A h1[LM];
  Level lv[kMaxLevels];
};

template <typename T, int LM>
struct Cfg {
  static constexpr int V = sizeof(T) == 8 ? (LM >= 32 ? 2 : 4) : (LM >= 32 ? 4 : 8);
  static constexpr int PS_ANA = V == 8 ? 4 : (V == 4 ? 3 : 2);  // pad period = 2V
  static constexpr int PS_SYN = V == 8 ? 3 : (V == 4 ? 2 : 1);  // pad period = V
  static constexpr int ANA_TILE = kThreads * V;                 // outputs per staged tile
  static constexpr int ANA_SPAN = 2 * ANA_TILE + LM - 2;        // inputs per staged tile
  static constexpr int SYN_TILE = kThreads * V;                 // u-positions per tile
  static constexpr int SYN_SPAN = SYN_TILE + LM / 2 - 1;
  static constexpr int FOLD_MAX = 2 * LM + 8;
};

// ------------------------------------------------------------------------------------ analysis

template <typename T, typename A, int LM, int V, int PS>
__device__ __forceinline__ void ana_outputs(const Params<A, LM>& p, const A (&w)[2 * V + LM - 2],
                                            int64_t o0, int64_t n_coef, T* gdet, T* sdst,
                                            T* gdst) {
#pragma unroll
  for (int v = 0; v < V; ++v) {
    A a = A(0), d = A(0);
#pragma unroll
    for (int j = 0; j < LM; ++j) {
      const A xv = w[2 * v + LM - 1 - j];
      a = fma(p.h0[j], xv, a);
      d = fma(p.h1[j], xv, d);
    }
    const int64_t o = o0 + v;
    if (o < n_coef) {
      gdet[o] = from_acc<T>(d);
      if (sdst) {
        sdst[sidx<PS>(static_cast<int>(o))] = from_acc<T>(a);
      } else {
        gdst[o] = from_acc<T>(a);
      }
    }
  }
}

template <typename T, int LM>
__global__ void __launch_bounds__(kThreads)
dwt_analysis_kernel(const __grid_constant__ Params<typename AccOf<T>::type, LM> p) {
  using A = typename AccOf<T>::type;
  using C = Cfg<T, LM>;
  constexpr int V = C::V;
  constexpr int PS = C::PS_ANA;
  constexpr int W = 2 * V + LM - 2;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* buf0 = reinterpret_cast<T*>(smem_raw);
  T* buf1 = buf0 + p.buf_len[0];
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;

  for (int l = 0; l < p.nlev; ++l) {
    const Level& L = p.lv[l];
    const bool last = (l == p.nlev - 1);
    T* sdst = last ? nullptr : ((l & 1) ? buf1 : buf0);
    T* gdst = last ? static_cast<T*>(p.dst) + row * L.a_len : nullptr;
    T* gdet = static_cast<T*>(L.detail) + row * L.n_coef;
    const int64_t n_in = L.n_in, n_coef = L.n_coef;

    if (l == 0) {
      // input row in HBM: stream it through buf1 in tiles, extension applied while staging
      const T* src = static_cast<const T*>(p.src) + row * n_in;
      T* stage = buf1;
      constexpr int IT = (C::ANA_SPAN + kThreads - 1) / kThreads;
      for (int64_t t0 = 0; t0 < n_coef; t0 += C::ANA_TILE) {
        const int64_t s0 = 2 * t0 + p.off - (LM - 1);
        const int cnt = static_cast<int>(imin(C::ANA_TILE, n_coef - t0));
        const int span = 2 * cnt + LM - 2;
        T r[IT];
        if (s0 >= 0 && s0 + span <= n_in) {
#pragma unroll
          for (int k = 0; k < IT; ++k) {
            const int i = tid + k * kThreads;
            r[k] = i < span ? src[s0 + i] : T(0);
          }
        } else {
#pragma unroll
          for (int k = 0; k < IT; ++k) {
            const int i = tid + k * kThreads;
            const int64_t q = i < span ? ext_index(s0 + i, n_in, L.mode, L.P) : -1;
            r[k] = q >= 0 ? src[q] : T(0);
          }
        }
#pragma unroll
        for (int k = 0; k < IT; ++k) {
          const int i = tid + k * kThreads;
          if (i < span) stage[sidx<PS>(i)] = r[k];
        }
        __syncthreads();
        const int ol = tid * V;
        if (ol < cnt) {
          A w[W];
#pragma unroll
          for (int i = 0; i < W; ++i) w[i] = to_acc<T>(stage[sidx<PS>(2 * ol + i)]);
          ana_outputs<T, A, LM, V, PS>(p, w, t0 + ol, n_coef, gdet, sdst, gdst);
        }
        __syncthreads();
      }
    } else {
      // input resident in shared memory (the previous level's approximation)
      const T* src = (l & 1) ? buf0 : buf1;
      for (int64_t o0 = static_cast<int64_t>(tid) * V; o0 < n_coef; o0 += kThreads * V) {
        const int64_t e0 = 2 * o0 + p.off - (LM - 1);
        A w[W];
        if (e0 >= 0 && e0 + W <= n_in) {
          const int e = static_cast<int>(e0);
#pragma unroll
          for (int i = 0; i < W; ++i) w[i] = to_acc<T>(src[sidx<PS>(e + i)]);
        } else {
#pragma unroll
          for (int i = 0; i < W; ++i) {
            const int64_t q = ext_index(e0 + i, n_in, L.mode, L.P);
            w[i] = q >= 0 ? to_acc<T>(src[sidx<PS>(static_cast<int>(q))]) : A(0);
          }
        }
        ana_outputs<T, A, LM, V, PS>(p, w, o0, n_coef, gdet, sdst, gdst);
      }
    }
    if (L.a_len > n_coef && tid == 0) {  // transpose of waverec's trim: a trailing zero
      if (sdst) sdst[sidx<PS>(static_cast<int>(n_coef))] = T(0);
      else gdst[n_coef] = T(0);
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------------------------ synthesis

template <typename T, int LM>
__global__ void __launch_bounds__(kThreads)
dwt_synthesis_kernel(const __grid_constant__ Params<typename AccOf<T>::type, LM> p) {
  using A = typename AccOf<T>::type;
  using C = Cfg<T, LM>;
  constexpr int V = C::V;
  constexpr int PS = C::PS_SYN;
  constexpr int H = LM / 2;
  constexpr int W = V + H - 1;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* buf0 = reinterpret_cast<T*>(smem_raw);
  T* buf1 = buf0 + p.buf_len[0];
  T* stage_a = buf1 + p.buf_len[1];
  T* stage_d = stage_a + p.stage_len;
  const size_t zoff =
      ((static_cast<size_t>(p.buf_len[0] + p.buf_len[1] + 2 * p.stage_len) * sizeof(T)) + 15) &
      ~size_t(15);
  A* zext = reinterpret_cast<A*>(smem_raw + zoff);
  int* ztg = reinterpret_cast<int*>(zext + C::FOLD_MAX);
  const int64_t row = blockIdx.x;
  const int tid = threadIdx.x;
  const int off = p.off;

  for (int l = 0; l < p.nlev; ++l) {
    const Level& L = p.lv[l];
    const bool first = (l == 0), last = (l == p.nlev - 1);
    const int64_t n = L.n_in, nc = L.n_coef;
    const T* ga = first ? static_cast<const T*>(p.src) + row * L.a_len : nullptr;
    const T* sa = first ? nullptr : ((l & 1) ? buf0 : buf1);
    const T* gd = L.detail ? static_cast<const T*>(L.detail) + row * nc : nullptr;
    T* sdst = last ? nullptr : ((l & 1) ? buf1 : buf0);
    T* gdst = last ? static_cast<T*>(p.dst) + row * n : nullptr;

    auto a_at = [&](int64_t o) -> A {  // approximation sample o in [0, nc)
      return first ? to_acc<T>(ga[o]) : to_acc<T>(sa[sidx<PS>(static_cast<int>(o))]);
    };

    // 1. exterior positions of the extended range, evaluated once and folded below
    const int64_t pmin = off - (LM - 1), pmax = 2 * (nc - 1) + off;
    const int E = L.fold_n;
    const int64_t nleft = imax(0, imin(-1, pmax) - pmin + 1);
    const int64_t rstart = imax(n, pmin);
    for (int e = tid; e < E; e += kThreads) {
      const int64_t pp = e < nleft ? pmin + e : rstart + (e - nleft);
      A z = A(0);
#pragma unroll
      for (int j = 0; j < LM; ++j) {
        const int64_t q = pp - off + j;
        if ((q & 1) == 0) {
          const int64_t o = q >> 1;
          if (o >= 0 && o < nc) {
            z = fma(p.h0[j], a_at(o), z);
            if (gd) z = fma(p.h1[j], to_acc<T>(gd[o]), z);
          }
        }
      }
      zext[e] = z;
      ztg[e] = static_cast<int>(ext_index(pp, n, L.mode, L.P));
    }
    __syncthreads();
    const int64_t zedge = imax(1 - pmin, pmax - n + 2);
    const bool fold_all = 2 * zedge >= n;

    // 2. direct pass, polyphase: u -> outputs off+2u-1 (odd taps) and off+2u (even taps)
    const int64_t u_min = floor_div(1 - off, 2), u_max = floor_div(n - off, 2);
    for (int64_t ut0 = u_min; ut0 <= u_max; ut0 += C::SYN_TILE) {
      const int cnt = static_cast<int>(imin(C::SYN_TILE, u_max - ut0 + 1));
      const int span = cnt + H - 1;
      for (int i = tid; i < span; i += kThreads) {
        const int64_t o = ut0 + i;
        const bool in = o >= 0 && o < nc;
        stage_d[sidx<PS>(i)] = (in && gd) ? gd[o] : T(0);
        if (first) stage_a[sidx<PS>(i)] = in ? ga[o] : T(0);
      }
      __syncthreads();
      const int ul = tid * V;
      if (ul < cnt) {
        A wa[W], wd[W];
        const int64_t ob = ut0 + ul;
        if (first || (ob >= 0 && ob + W <= nc)) {
#pragma unroll
          for (int i = 0; i < W; ++i) {
            wd[i] = to_acc<T>(stage_d[sidx<PS>(ul + i)]);
            wa[i] = first ? to_acc<T>(stage_a[sidx<PS>(ul + i)])
                          : to_acc<T>(sa[sidx<PS>(static_cast<int>(ob + i))]);
          }
        } else {
#pragma unroll
          for (int i = 0; i < W; ++i) {
            wd[i] = to_acc<T>(stage_d[sidx<PS>(ul + i)]);
            const int64_t o = ob + i;
            wa[i] = (o >= 0 && o < nc) ? to_acc<T>(sa[sidx<PS>(static_cast<int>(o))]) : A(0);
          }
        }
#pragma unroll
        for (int v = 0; v < V; ++v) {
          A ze = A(0), zo = A(0);
#pragma unroll
          for (int t = 0; t < H; ++t) {
            ze = fma(p.h0[2 * t], wa[v + t], ze);
            ze = fma(p.h1[2 * t], wd[v + t], ze);
            zo = fma(p.h0[2 * t + 1], wa[v + t], zo);
            zo = fma(p.h1[2 * t + 1], wd[v + t], zo);
          }
          const int64_t iodd = off + 2 * (ob + v) - 1;
#pragma unroll
          for (int ph = 0; ph < 2; ++ph) {
            const int64_t i = iodd + ph;
            A val = ph ? ze : zo;
            if (i >= 0 && i < n) {
              if (E > 0 && (fold_all || i < zedge || i >= n - zedge)) {
                for (int e = 0; e < E; ++e)
                  if (ztg[e] == i) val += zext[e];
              }
              if (sdst) sdst[sidx<PS>(static_cast<int>(i))] = from_acc<T>(val);
              else gdst[i] = from_acc<T>(val);
            }
          }
        }
      }
      __syncthreads();
    }
  }
}

// ------------------------------------------------------------------------------------ host

constexpr int kLM[] = {2, 4, 6, 8, 10, 12, 16, 20, 24, 32, 40, 64};

inline int pick_lm(int L) {
  for (int lm : kLM)
    if (L <= lm) return lm;
  return -1;
}

// Opt a kernel into the device's full dynamic shared memory (once per kernel and device).
inline int smem_budget_set(const void* fn) { return allow_max_dynamic_smem(fn); }

// analysis: segment planning over the level list (finest first)
struct Seg {
  int l0, l1;  // inclusive level range
  size_t smem;
  int buf0, buf1;
};

template <typename T, int LM>
std::vector<Seg> plan_analysis(const std::vector<Level>& lv, size_t budget) {
  using C = Cfg<T, LM>;
  std::vector<Seg> segs;
  const int nl = static_cast<int>(lv.size());
  int l0 = 0;
  while (l0 < nl) {
    int64_t b0 = 0, b1 = padded_len<C::PS_ANA>(C::ANA_SPAN);
    Seg best{l0, l0, 0, 0, 0};
    for (int l1 = l0; l1 < nl; ++l1) {
      // level l1 is the last of the segment; levels l0..l1-1 keep their approximation resident
      if (l1 > l0) {
        const int r = l1 - 1 - l0;
        const int64_t need = padded_len<C::PS_ANA>(lv[l1 - 1].a_len);
        if (r % 2 == 0) b0 = std::max(b0, need);
        else b1 = std::max(b1, need);
      }
      const size_t bytes = static_cast<size_t>(b0 + b1) * sizeof(T) + 16;
      if (bytes > budget || l1 - l0 + 1 > kMaxLevels) break;
      best = Seg{l0, l1, bytes, static_cast<int>(b0), static_cast<int>(b1)};
    }
    segs.push_back(best);
    l0 = best.l1 + 1;
  }
  return segs;
}

template <typename T, int LM>
std::vector<Seg> plan_synthesis(const std::vector<Level>& lv, size_t budget) {
  using C = Cfg<T, LM>;
  using A = typename AccOf<T>::type;
  std::vector<Seg> segs;
  const int nl = static_cast<int>(lv.size());
  const int64_t stage = padded_len<C::PS_SYN>(C::SYN_SPAN);
  const size_t fold_bytes = C::FOLD_MAX * (sizeof(A) + sizeof(int)) + 32;
  int l0 = 0;
  while (l0 < nl) {
    int64_t b0 = 0, b1 = 0;
    Seg best{l0, l0, 0, 0, 0};
    for (int l1 = l0; l1 < nl; ++l1) {
      if (l1 > l0) {
        const int r = l1 - 1 - l0;
        const int64_t need = padded_len<C::PS_SYN>(lv[l1 - 1].n_in);
        if (r % 2 == 0) b0 = std::max(b0, need);
        else b1 = std::max(b1, need);
      }
      const size_t bytes = static_cast<size_t>(b0 + b1 + 2 * stage) * sizeof(T) + fold_bytes;
      if (bytes > budget || l1 - l0 + 1 > kMaxLevels) break;
      best = Seg{l0, l1, bytes, static_cast<int>(b0), static_cast<int>(b1)};
    }
    segs.push_back(best);
    l0 = best.l1 + 1;
  }
  return segs;
}

// Workspace: two ping-pong regions, each big enough for any approximation handed over
// between consecutive segments.
inline size_t handover_bytes(const std::vector<Level>& lv, const std::vector<Seg>& segs, int64_t rows,
                      size_t esize, bool analysis) {
  size_t mx = 0;
  for (size_t s = 0; s + 1 < segs.size(); ++s) {
    const Level& L = lv[segs[s].l1];
    const int64_t len = analysis ? L.a_len : L.n_in;
    mx = std::max(mx, static_cast<size_t>(rows) * static_cast<size_t>(len) * esize);
  }
  mx = (mx + 255) & ~size_t(255);
  return segs.size() > 1 ? (segs.size() > 2 ? 2 * mx : mx) : 0;
}

inline int fold_count(int64_t n, int64_t nc, int off, int LM, int mode) {
  if (mode == FDWT_MODE_ZERO) return 0;
  const int64_t pmin = off - (LM - 1), pmax = 2 * (nc - 1) + off;
  const int64_t nleft = std::max<int64_t>(0, std::min<int64_t>(-1, pmax) - pmin + 1);
  const int64_t nright = std::max<int64_t>(0, pmax - std::max<int64_t>(n, pmin) + 1);
  return static_cast<int>(nleft + nright);
}

template <typename T, int LM>
int run_analysis(int64_t rows, const void* x, std::vector<Level> lv, void* approx_out,
                 const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
                 cudaStream_t stream, size_t* ws_needed) {
  using A = typename AccOf<T>::type;
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 1024;
  auto segs = plan_analysis<T, LM>(lv, budget);
  const size_t need = handover_bytes(lv, segs, rows, sizeof(T), true);
  if (ws_needed) {
    *ws_needed = need;
    return FDWT_OK;
  }
  if (rows == 0) return FDWT_OK;
  if (need > 0 && (ws == nullptr || ws_bytes < need)) return FDWT_ERR_WORKSPACE;
  if (rows > 0x7fffffffLL) return FDWT_ERR_UNSUPPORTED;
  auto kern = dwt_analysis_kernel<T, LM>;
  int st = smem_budget_set(reinterpret_cast<const void*>(kern));
  if (st != FDWT_OK) return st;
  const size_t half = segs.size() > 2 ? need / 2 : need;
  const void* src = x;
  for (size_t s = 0; s < segs.size(); ++s) {
    Params<A, LM> p{};
    p.rows = rows;
    p.src = src;
    const bool final_seg = (s + 1 == segs.size());
    p.dst = final_seg ? approx_out : static_cast<unsigned char*>(ws) + (s % 2) * half;
    p.nlev = segs[s].l1 - segs[s].l0 + 1;
    p.off = off;
    p.buf_len[0] = segs[s].buf0;
    p.buf_len[1] = segs[s].buf1;
    for (int j = 0; j < LM; ++j) {
      p.h0[j] = j < L ? static_cast<A>(h0[j]) : A(0);
      p.h1[j] = j < L ? static_cast<A>(h1[j]) : A(0);
    }
    for (int k = 0; k < p.nlev; ++k) p.lv[k] = lv[segs[s].l0 + k];
    kern<<<static_cast<unsigned>(rows), kThreads, segs[s].smem, stream>>>(p);
    st = launch_status();
    if (st != FDWT_OK) return st;
    src = p.dst;
  }
  return FDWT_OK;
}

template <typename T, int LM>
int run_synthesis(int64_t rows, const void* approx_in, std::vector<Level> lv, void* y,
                  const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
                  cudaStream_t stream, size_t* ws_needed) {
  using A = typename AccOf<T>::type;
  using C = Cfg<T, LM>;
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 1024;
  for (auto& l : lv) {
    l.fold_n = fold_count(l.n_in, l.n_coef, off, LM, l.mode);
    if (l.fold_n > C::FOLD_MAX) return FDWT_ERR_UNSUPPORTED;
  }
  auto segs = plan_synthesis<T, LM>(lv, budget);
  const size_t need = handover_bytes(lv, segs, rows, sizeof(T), false);
  if (ws_needed) {
    *ws_needed = need;
    return FDWT_OK;
  }
  if (rows == 0) return FDWT_OK;
  if (need > 0 && (ws == nullptr || ws_bytes < need)) return FDWT_ERR_WORKSPACE;
  if (rows > 0x7fffffffLL) return FDWT_ERR_UNSUPPORTED;
  auto kern = dwt_synthesis_kernel<T, LM>;
  int st = smem_budget_set(reinterpret_cast<const void*>(kern));
  if (st != FDWT_OK) return st;
  const size_t half = segs.size() > 2 ? need / 2 : need;
  const void* src = approx_in;
  for (size_t s = 0; s < segs.size(); ++s) {
    Params<A, LM> p{};
    p.rows = rows;
    p.src = src;
    const bool final_seg = (s + 1 == segs.size());
    p.dst = final_seg ? y : static_cast<unsigned char*>(ws) + (s % 2) * half;
    p.nlev = segs[s].l1 - segs[s].l0 + 1;
    p.off = off;
    p.buf_len[0] = segs[s].buf0;
    p.buf_len[1] = segs[s].buf1;
    p.stage_len = static_cast<int>(padded_len<C::PS_SYN>(C::SYN_SPAN));
    for (int j = 0; j < LM; ++j) {
      p.h0[j] = j < L ? static_cast<A>(h0[j]) : A(0);
      p.h1[j] = j < L ? static_cast<A>(h1[j]) : A(0);
    }
    for (int k = 0; k < p.nlev; ++k) p.lv[k] = lv[segs[s].l0 + k];
    kern<<<static_cast<unsigned>(rows), kThreads, segs[s].smem, stream>>>(p);
    st = launch_status();
    if (st != FDWT_OK) return st;
    src = p.dst;
  }
  return FDWT_OK;
}

// Per-dtype entry points (one translation unit per dtype instantiates every LM).
template <typename T>
int analysis_dtype(int LM, int64_t rows, const void* x, std::vector<Level> lv, void* approx_out,
                   const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
                   cudaStream_t stream, size_t* ws_needed);
template <typename T>
int synthesis_dtype(int LM, int64_t rows, const void* approx_in, std::vector<Level> lv, void* y,
                    const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
                    cudaStream_t stream, size_t* ws_needed);

#define FDWT_DWT_INSTANTIATE(T)                                                              \
  template <>                                                                                \
  int analysis_dtype<T>(int LM, int64_t rows, const void* x, std::vector<Level> lv,          \
                        void* approx_out, const double* h0, const double* h1, int L, int off,\
                        void* ws, size_t ws_bytes, cudaStream_t stream, size_t* ws_needed) { \
    switch (LM) {                                                                            \
      case 2: return run_analysis<T, 2>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 4: return run_analysis<T, 4>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 6: return run_analysis<T, 6>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 8: return run_analysis<T, 8>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 10: return run_analysis<T, 10>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 12: return run_analysis<T, 12>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 16: return run_analysis<T, 16>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 20: return run_analysis<T, 20>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 24: return run_analysis<T, 24>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 32: return run_analysis<T, 32>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 40: return run_analysis<T, 40>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 64: return run_analysis<T, 64>(rows, x, lv, approx_out, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      default: return FDWT_ERR_UNSUPPORTED;                                                  \
    }                                                                                        \
  }                                                                                          \
  template <>                                                                                \
  int synthesis_dtype<T>(int LM, int64_t rows, const void* a, std::vector<Level> lv, void* y, \
                         const double* h0, const double* h1, int L, int off, void* ws,       \
                         size_t ws_bytes, cudaStream_t stream, size_t* ws_needed) {          \
    switch (LM) {                                                                            \
      case 2: return run_synthesis<T, 2>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 4: return run_synthesis<T, 4>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 6: return run_synthesis<T, 6>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 8: return run_synthesis<T, 8>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);   \
      case 10: return run_synthesis<T, 10>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 12: return run_synthesis<T, 12>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 16: return run_synthesis<T, 16>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 20: return run_synthesis<T, 20>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 24: return run_synthesis<T, 24>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 32: return run_synthesis<T, 32>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 40: return run_synthesis<T, 40>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      case 64: return run_synthesis<T, 64>(rows, a, lv, y, h0, h1, L, off, ws, ws_bytes, stream, ws_needed); \
      default: return FDWT_ERR_UNSUPPORTED;                                                  \
    }                                                                                        \
  }

}  // namespace dwtk
}  // namespace fdwt
