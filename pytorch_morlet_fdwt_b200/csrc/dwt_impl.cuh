// Fused multilevel DWT analysis and its exact transpose for sm_100a (templates; instantiated
// per element type in dwt_f32.cu / dwt_f64.cu / dwt_f16.cu / dwt_bf16.cu).
//
// Work decomposition.  A signal row is owned by a thread-block cluster of C CTAs (C = 1 for
// short rows).  Every level of a multilevel transform runs inside one launch.  A level's
// output array (the next approximation) is partitioned among the C CTAs so that each CTA's
// outputs need input windows that start inside the CTA's own part of the previous array; the
// arrays stay resident in shared memory.  Before a level is computed, each CTA fills a small
// halo around its part -- neighbours' samples through distributed shared memory (DSMEM), the
// boundary extension of the row ends (periodic wrap, symmetric/reflect mirror, zero) by index
// arithmetic -- so that every thread then reads one contiguous local window.  Only details and
// the last approximation are written to HBM.  Rows that live in HBM (the signal of the
// analysis; details and the coarsest approximation of the synthesis) stream through a
// double-buffered cp.async pipeline in tiles.  A cluster barrier separates levels.  When even
// a cluster of 8 cannot hold the resident approximations, the host splits the levels into
// consecutive launches ("segments") that hand the approximation over through a caller-provided
// workspace.
//
// Inner loops.  Taps live in the kernel parameter block (constant bank).  A thread computes V
// consecutive outputs from a register window of its inputs; in fp32 the two filters advance
// together with Blackwell's packed FMA (fma.rn.f32x2: (cA, cD) += (h0[j], h1[j]) * (x, x)).
// Thread output chunks start on a 16-byte boundary of the destination row so that details
// leave as 128-bit stores, and every resident array is stored with a per-CTA origin that puts
// each thread window at a multiple of the shared-memory padding period (one pad element per
// 2V (analysis) or V (synthesis) elements): window loads are bank-conflict free and address
// with a per-thread base plus immediates.
//
// Semantics follow the reference's Triton kernels fdwt/kernels/dwt.py:73-98 (analysis with the
// index-arithmetic extension _ext_index, 52-70) and 101-175 (exact transpose).  The transpose
// is evaluated as y = Fold(z) with z[p] = sum_{2o+off-j = p} h0[j] a[o] + h1[j] d[o] on the
// extended range [off-L+1, 2(nc-1)+off]; per output only the L/2 taps of its parity are
// visited, and extended positions outside [0, n) are folded onto ext(p) (zero mode drops them).
#pragma once

#include <cooperative_groups.h>

#include <algorithm>
#include <type_traits>
#include <vector>

#include "common.cuh"

namespace fdwt {
namespace dwtk {

namespace cg = cooperative_groups;

constexpr int NT = 256;          // threads per CTA
constexpr int kMaxLevels = 24;   // levels per launch
constexpr int kMaxCluster = 8;   // portable cluster size
constexpr int kMargin = 16;      // local slots before a resident array's first window

struct Level {
  int64_t n_in;    // analysis: input length;  synthesis: output length
  int64_t n_coef;  // coefficient length
  int64_t a_len;   // analysis: stored approximation length (n_coef + pad);
                   // synthesis: length of the incoming approximation (>= n_coef)
  int64_t P;       // period of the (normalized) boundary mode for the signal length
  void* detail;    // analysis: detail output; synthesis: detail input (nullptr = zeros)
  int32_t mode;    // normalized boundary mode
  int32_t fold_n;  // synthesis: exterior positions folded back (0 in zero mode)
  int32_t bnd[kMaxCluster + 1];  // partition of the level's output array among the CTAs
};

template <typename A, int LM>
struct Params {
  int64_t rows;
  const void* src;      // analysis: (rows, lv[0].n_in); synthesis: (rows, lv[0].a_len)
  void* dst;            // analysis: (rows, lv[nlev-1].a_len); synthesis: (rows, lv[nlev-1].n_in)
  int32_t nlev;
  int32_t off;
  int32_t csize;        // CTAs per row (cluster size)
  int32_t buf_len[2];   // padded elements of the two resident buffers
  int32_t stage_off;    // element offset of the stage area
  int32_t stage_len;    // padded elements of one stage buffer (buffer stride)
  int32_t stage_span;   // elements staged per tile
  int32_t nstage;       // stage buffers per staged stream (1 or 2)
  int32_t fold_off;     // byte offset of the fold arrays (synthesis)
  // analysis: (h0[j], h1[j]) interleaved;  synthesis: h0[0..LM) followed by h1[0..LM)
  alignas(16) A taps[2 * LM];
  Level lv[kMaxLevels];
};

template <typename T, int LM>
struct Cfg {
  static constexpr int V = sizeof(T) == 8 ? 4 : 8;  // outputs (analysis) / u-values (synthesis)
  static constexpr int VW = 16 / sizeof(T);         // elements per 128-bit store
  static constexpr int PSA = sizeof(T) == 8 ? 3 : 4;  // pad period 2V (analysis windows)
  static constexpr int PSS = sizeof(T) == 8 ? 2 : 3;  // pad period V (synthesis windows)
  static constexpr int H = LM / 2;
  static constexpr int WA = 2 * V + LM - 2;  // analysis window
  static constexpr int WS = V + H + 1;       // synthesis window (V+1 u-pairs read V+H samples)
  static constexpr int FOLD_MAX = 2 * LM + 8;
  static constexpr int ZONE_MAX = 4 * LM + 16;  // edge outputs that can receive folds
};

// ------------------------------------------------------------------------------ primitives

__device__ __forceinline__ void cp_async(void* smem_dst, const void* gsrc, int bytes) {
  const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem_dst));
  if (bytes == 8)
    asm volatile("cp.async.ca.shared.global [%0], [%1], 8;\n" ::"r"(s), "l"(gsrc) : "memory");
  else
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(s), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;\n" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

// wait until at most n-1 committed groups are pending (n = ring depth, 1..4)
__device__ __forceinline__ void cp_async_wait_ring(int n) {
  if (n <= 1) cp_async_wait<0>();
  else if (n == 2) cp_async_wait<1>();
  else if (n == 3) cp_async_wait<2>();
  else cp_async_wait<3>();
}

__device__ __forceinline__ void group_sync(int csize) {
  if (csize > 1) cg::this_cluster().sync();
  else __syncthreads();
}

__device__ __forceinline__ unsigned long long pair(float lo, float hi) {
  return static_cast<unsigned long long>(__float_as_uint(lo)) |
         (static_cast<unsigned long long>(__float_as_uint(hi)) << 32);
}
__device__ __forceinline__ float lo32(unsigned long long v) {
  return __uint_as_float(static_cast<unsigned>(v));
}
__device__ __forceinline__ float hi32(unsigned long long v) {
  return __uint_as_float(static_cast<unsigned>(v >> 32));
}
// acc += a * b on both fp32 halves (one packed FMA instruction on sm_100)
__device__ __forceinline__ void ffma2(unsigned long long& acc, unsigned long long a,
                                      unsigned long long b) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(a), "l"(b));
}

template <typename T>
__device__ __forceinline__ int elem_misalign(const T* p) {
  constexpr int VW = 16 / sizeof(T);
  return static_cast<int>((reinterpret_cast<uintptr_t>(p) / sizeof(T)) & (VW - 1));
}

__device__ __forceinline__ unsigned bits32(float a) { return __float_as_uint(a); }
__device__ __forceinline__ unsigned bits32(__half a, __half b) {
  return static_cast<unsigned>(__half_as_ushort(a)) |
         (static_cast<unsigned>(__half_as_ushort(b)) << 16);
}
__device__ __forceinline__ unsigned bits32(__nv_bfloat16 a, __nv_bfloat16 b) {
  return static_cast<unsigned>(__bfloat16_as_ushort(a)) |
         (static_cast<unsigned>(__bfloat16_as_ushort(b)) << 16);
}
template <typename T>
__device__ __forceinline__ uint4 pack16(const T* v) {
  if constexpr (sizeof(T) == 4) {
    return make_uint4(bits32(v[0]), bits32(v[1]), bits32(v[2]), bits32(v[3]));
  } else if constexpr (sizeof(T) == 8) {
    const unsigned long long a = __double_as_longlong(v[0]), b = __double_as_longlong(v[1]);
    return make_uint4(static_cast<unsigned>(a), static_cast<unsigned>(a >> 32),
                      static_cast<unsigned>(b), static_cast<unsigned>(b >> 32));
  } else {
    return make_uint4(bits32(v[0], v[1]), bits32(v[2], v[3]), bits32(v[4], v[5]),
                      bits32(v[6], v[7]));
  }
}

// Store N consecutive values starting at an element whose address is 16-byte aligned.
template <typename T, int N>
__device__ __forceinline__ void store_vec(T* dst, const T (&v)[N]) {
  constexpr int VW = 16 / sizeof(T);
#pragma unroll
  for (int k = 0; k < N / VW; ++k) reinterpret_cast<uint4*>(dst)[k] = pack16<T>(&v[k * VW]);
}

// Owner rank of element e of an array partitioned by bnd[0..cs].
__device__ __forceinline__ int owner_of(const int32_t* bnd, int cs, int64_t e) {
  int r = 0;
  while (r + 1 < cs && e >= bnd[r + 1]) ++r;
  return r;
}

template <typename T>
__device__ __forceinline__ T peer_load(T* local_buf, int rank, int owner, int loc) {
  if (owner == rank) return local_buf[loc];
  const T* peer = cg::this_cluster().map_shared_rank(local_buf, owner);
  return peer[loc];
}

// Stage `span` elements of a global row from extended position s0 into a padded shared buffer
// (pad period 2^PS): positions inside [0, n) are copied, the others through the boundary map
// (or zero).  4- and 8-byte elements use cp.async; narrower ones a synchronous copy.
template <typename T, int PS>
__device__ __forceinline__ void stage_ext(T* stage, const T* row, int64_t s0, int span,
                                          int64_t n, int mode, int64_t P) {
  const int tid = threadIdx.x;
  if (s0 >= 0 && s0 + span <= n) {
    const T* g = row + s0 + tid;
    int si = sidx<PS>(tid);
    for (int i = tid; i < span; i += NT, g += NT, si += NT + (NT >> PS)) {
      if constexpr (sizeof(T) >= 4) cp_async(stage + si, g, sizeof(T));
      else stage[si] = *g;
    }
  } else {
    for (int i = tid; i < span; i += NT) {
      const int64_t q = ext_index(s0 + i, n, mode, P);
      T* d = stage + sidx<PS>(i);
      if (q < 0) *d = T(0);
      else if constexpr (sizeof(T) >= 4) cp_async(d, row + q, sizeof(T));
      else *d = row[q];
    }
  }
}

// Stage coefficients c[u0 .. u0+span) (zero outside [0, nc) or for a null row).
template <typename T, int PS>
__device__ __forceinline__ void stage_coef(T* stage, const T* row, int64_t u0, int span,
                                           int64_t nc) {
  const int tid = threadIdx.x;
  if (row != nullptr && u0 >= 0 && u0 + span <= nc) {
    const T* g = row + u0 + tid;
    int si = sidx<PS>(tid);
    for (int i = tid; i < span; i += NT, g += NT, si += NT + (NT >> PS)) {
      if constexpr (sizeof(T) >= 4) cp_async(stage + si, g, sizeof(T));
      else stage[si] = *g;
    }
    return;
  }
  for (int i = tid; i < span; i += NT) {
    const int64_t u = u0 + i;
    T* d = stage + sidx<PS>(i);
    if (row == nullptr || u < 0 || u >= nc) *d = T(0);
    else if constexpr (sizeof(T) >= 4) cp_async(d, row + u, sizeof(T));
    else *d = row[u];
  }
}

// ------------------------------------------------------------------------------ analysis

// First output chunk and window origin of CTA r at a level whose details are misaligned by ad.
template <int V, int LM>
__device__ __forceinline__ int64_t ana_cb(const Level& L, int r, int ad) {
  return floor_div(static_cast<int64_t>(L.bnd[r]) + ad, V);
}
template <int V, int LM>
__device__ __forceinline__ int64_t ana_org(const Level& L, int r, int ad, int off) {
  return 2 * (ana_cb<V, LM>(L, r, ad) * V - ad) + off - (LM - 1);
}

// V outputs from the window w (w[i] = in_ext[2 o_c + off - (LM-1) + i]).
template <typename T, typename A, int LM>
__device__ __forceinline__ void ana_compute(const A* taps, const A* w, A* ra, A* rd) {
  constexpr int V = Cfg<T, LM>::V;
  constexpr int W = Cfg<T, LM>::WA;
  if constexpr (std::is_same<A, float>::value) {
    unsigned long long acc[V];
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = 0ull;
#pragma unroll
    for (int i = W - 1; i >= 0; --i) {  // descending window index = ascending tap index
      const unsigned long long xx = pair(w[i], w[i]);
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
        const A xv = w[2 * v + LM - 1 - j];
        a = fma(taps[2 * j], xv, a);
        d = fma(taps[2 * j + 1], xv, d);
      }
      ra[v] = a;
      rd[v] = d;
    }
  }
}

template <typename T, typename A, int LM>
__device__ __forceinline__ void ana_store(const A* ra, const A* rd, int64_t o_c, int64_t o_b,
                                          int64_t o_end, T* gdet, T* sdst, int64_t sorg,
                                          T* gdst, bool vec_a) {
  constexpr int V = Cfg<T, LM>::V;
  constexpr int PS = Cfg<T, LM>::PSA;
  T va[V], vd[V];
#pragma unroll
  for (int v = 0; v < V; ++v) {
    va[v] = from_acc<T>(ra[v]);
    vd[v] = from_acc<T>(rd[v]);
  }
  const bool full = o_c >= o_b && o_c + V <= o_end;
  if (full) {
    store_vec<T, V>(gdet + o_c, vd);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (o_c + v >= o_b && o_c + v < o_end) gdet[o_c + v] = vd[v];
  }
  if (sdst) {
    const int base = static_cast<int>(o_c - sorg);
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (o_c + v >= o_b && o_c + v < o_end) sdst[sidx<PS>(base + v)] = va[v];
  } else if (full && vec_a) {
    store_vec<T, V>(gdst + o_c, va);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v)
      if (o_c + v >= o_b && o_c + v < o_end) gdst[o_c + v] = va[v];
  }
}

template <typename T, int LM>
__global__ void __launch_bounds__(NT, 2)
dwt_analysis_kernel(const __grid_constant__ Params<typename AccOf<T>::type, LM> p) {
  using A = typename AccOf<T>::type;
  using C = Cfg<T, LM>;
  constexpr int V = C::V;
  constexpr int W = C::WA;
  constexpr int PS = C::PSA;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sbase = reinterpret_cast<T*>(smem_raw);
  T* const bufs[2] = {sbase, sbase + p.buf_len[0]};
  T* const stage0 = sbase + p.stage_off;
  const int cs = p.csize;
  const int rank = cs > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
  const int64_t row = blockIdx.x / cs;
  const int tid = threadIdx.x;
  const int off = p.off;

  for (int l = 0; l < p.nlev; ++l) {
    const Level& L = p.lv[l];
    const bool last = (l == p.nlev - 1);
    T* gdet = static_cast<T*>(L.detail) + row * L.n_coef;
    T* gdst = last ? static_cast<T*>(p.dst) + row * L.a_len : nullptr;
    const int64_t n_in = L.n_in, nc = L.n_coef;
    const int64_t o_b = L.bnd[rank], o_e = L.bnd[rank + 1];
    const int64_t o_end = imin(o_e, nc);
    const int ad = elem_misalign(gdet);
    const bool vec_a = gdst != nullptr && elem_misalign(gdst) == ad;
    const int64_t c_b = ana_cb<V, LM>(L, rank, ad);
    const int64_t c_e = o_end > o_b ? floor_div(o_end + ad + V - 1, V) : c_b;
    // where this level's outputs go when resident: the next level's window origin
    T* sdst = nullptr;
    int64_t sorg = 0;
    if (!last) {
      const Level& N = p.lv[l + 1];
      const int adn = elem_misalign(static_cast<T*>(N.detail) + row * N.n_coef);
      sdst = bufs[l & 1];
      sorg = ana_org<V, LM>(N, rank, adn, off) - kMargin;
    }

    if (l == 0) {
      const T* src = static_cast<const T*>(p.src) + row * n_in;
      const int64_t ntiles = (c_e - c_b + NT - 1) / NT;
      const int ns = p.nstage;
      auto tile_s0 = [&](int64_t t) { return 2 * ((c_b + t * NT) * V - ad) + off - (LM - 1); };
      auto slot = [&](int64_t t) { return stage0 + static_cast<int>(t % ns) * p.stage_len; };
      auto tile_span = [&](int64_t t) {
        return static_cast<int>(imin(p.stage_span, 2 * V * imin(NT, c_e - c_b - t * NT) + LM - 2));
      };
      // ring prologue: exactly ns-1 groups (empty when the row has fewer tiles), so that the
      // wait in iteration t always leaves tile t complete
      for (int64_t k = 0; k < ns - 1; ++k) {
        if (k < ntiles)
          stage_ext<T, PS>(slot(k), src, tile_s0(k), tile_span(k), n_in, L.mode, L.P);
        cp_async_commit();
      }
      for (int64_t t = 0; t < ntiles; ++t) {
        if (t + ns - 1 < ntiles)
          stage_ext<T, PS>(slot(t + ns - 1), src, tile_s0(t + ns - 1), tile_span(t + ns - 1),
                           n_in, L.mode, L.P);
        cp_async_commit();  // possibly empty: keeps one group per tile
        cp_async_wait_ring(ns);
        __syncthreads();
        const int64_t c = c_b + t * NT + tid;
        if (c < c_e) {
          A w[W], ra[V], rd[V];
          const T* sw = slot(t) + (2 * V + 1) * tid;  // = &stage[sidx(2V tid)] (pad period 2V)
#pragma unroll
          for (int i = 0; i < W; ++i) w[i] = to_acc<T>(sw[i + (i >> PS)]);
          ana_compute<T, A, LM>(p.taps, w, ra, rd);
          ana_store<T, A, LM>(ra, rd, c * V - ad, o_b, o_end, gdet, sdst, sorg, gdst, vec_a);
        }
        __syncthreads();
      }
    } else if (c_e > c_b) {
      // resident input: the previous level's outputs, stored from local slot kMargin at org
      const Level& Pv = p.lv[l - 1];
      T* src = bufs[(l - 1) & 1];
      const int64_t org = ana_org<V, LM>(L, rank, ad, off);
      const int64_t in_b = Pv.bnd[rank], in_e = Pv.bnd[rank + 1];
      const int64_t need_hi = org + 2 * V * (c_e - c_b) + LM - 2;
      // halo: window samples outside this CTA's part (neighbours via DSMEM, row-end extension)
      const int64_t nl = imax(0, imin(in_b, need_hi) - org);
      const int64_t r0 = imax(in_e, org);
      const int64_t nr = imax(0, need_hi - r0);
      // issue the halo loads first (at most one per thread in practice), keep them in
      // registers while the interior chunks -- windows inside this CTA's own part -- compute
      constexpr int kHaloRegs = 2;
      T hv[kHaloRegs];
      int hloc[kHaloRegs];
#pragma unroll
      for (int h = 0; h < kHaloRegs; ++h) {
        const int64_t k = tid + static_cast<int64_t>(h) * NT;
        hloc[h] = -1;
        hv[h] = T(0);
        if (k < nl + nr) {
          const int64_t e = k < nl ? org + k : r0 + (k - nl);
          const int64_t q = ext_index(e, n_in, L.mode, L.P);
          if (q >= 0) {
            const int ow = owner_of(Pv.bnd, cs, q);
            const int64_t org_ow = ana_org<V, LM>(L, ow, ad, off);
            hv[h] = peer_load(src, rank, ow, sidx<PS>(static_cast<int>(q - org_ow + kMargin)));
          }
          hloc[h] = sidx<PS>(static_cast<int>(e - org + kMargin));
        }
      }
      for (int64_t k = tid + kHaloRegs * NT; k < nl + nr; k += NT) {  // very short rows only
        const int64_t e = k < nl ? org + k : r0 + (k - nl);
        const int64_t q = ext_index(e, n_in, L.mode, L.P);
        T v = T(0);
        if (q >= 0) {
          const int ow = owner_of(Pv.bnd, cs, q);
          const int64_t org_ow = ana_org<V, LM>(L, ow, ad, off);
          v = peer_load(src, rank, ow, sidx<PS>(static_cast<int>(q - org_ow + kMargin)));
        }
        src[sidx<PS>(static_cast<int>(e - org + kMargin))] = v;
      }
      auto chunk = [&](int64_t c) {
        const int rel = static_cast<int>(c - c_b);
        A w[W], ra[V], rd[V];
        const T* sw = src + (2 * V + 1) * rel + sidx<PS>(kMargin);
#pragma unroll
        for (int i = 0; i < W; ++i) w[i] = to_acc<T>(sw[i + (i >> PS)]);
        ana_compute<T, A, LM>(p.taps, w, ra, rd);
        ana_store<T, A, LM>(ra, rd, c * V - ad, o_b, o_end, gdet, sdst, sorg, gdst, vec_a);
      };
      auto interior = [&](int64_t c) {
        const int64_t e0 = org + 2 * V * (c - c_b);
        return e0 >= in_b && e0 + W <= in_e;
      };
      for (int64_t c = c_b + tid; c < c_e; c += NT)
        if (interior(c)) chunk(c);
#pragma unroll
      for (int h = 0; h < kHaloRegs; ++h)
        if (hloc[h] >= 0) src[hloc[h]] = hv[h];
      __syncthreads();
      for (int64_t c = c_b + tid; c < c_e; c += NT)
        if (!interior(c)) chunk(c);
    }
    // transpose of waverec's trim: the approximation carries a trailing zero
    if (L.a_len > nc && nc >= o_b && nc < o_e && tid == 0) {
      if (sdst) sdst[sidx<PS>(static_cast<int>(nc - sorg))] = T(0);
      else gdst[nc] = T(0);
    }
    group_sync(cs);
  }
}

// ------------------------------------------------------------------------------ synthesis

template <int V>
__device__ __forceinline__ int64_t syn_cb(const Level& L, int r, int ay) {
  return floor_div(static_cast<int64_t>(L.bnd[r]) + ay, 2 * V);
}
// first u of the window of output chunk c (chunk c starts at output 2Vc - ay)
__device__ __forceinline__ int64_t syn_ufirst(int64_t c, int V, int ay, int off) {
  return floor_div(c * 2 * V - ay - off + 1, 2);
}

// Output pairs at V+1 consecutive u: ze(u) = output off+2u (even taps), zo(u) = off+2u-1.
template <typename T, typename A, int LM>
__device__ __forceinline__ void syn_compute(const A* taps, const A* wa, const A* wd,
                                            A (&zo)[Cfg<T, LM>::V + 1],
                                            A (&ze)[Cfg<T, LM>::V + 1]) {
  constexpr int V = Cfg<T, LM>::V;
  constexpr int H = LM / 2;
  const A* h0 = taps;
  const A* h1 = taps + LM;
  if constexpr (std::is_same<A, float>::value) {
    unsigned long long acc[V + 1];  // (even-phase, odd-phase) at u
#pragma unroll
    for (int u = 0; u <= V; ++u) acc[u] = 0ull;
#pragma unroll
    for (int i = 0; i < V + H; ++i) {
      const unsigned long long aa = pair(wa[i], wa[i]);
      const unsigned long long dd = pair(wd[i], wd[i]);
#pragma unroll
      for (int u = 0; u <= V; ++u) {
        const int t = i - u;
        if (t >= 0 && t < H) {
          ffma2(acc[u], *reinterpret_cast<const unsigned long long*>(&h0[2 * t]), aa);
          ffma2(acc[u], *reinterpret_cast<const unsigned long long*>(&h1[2 * t]), dd);
        }
      }
    }
#pragma unroll
    for (int u = 0; u <= V; ++u) {
      ze[u] = lo32(acc[u]);
      zo[u] = hi32(acc[u]);
    }
  } else {
#pragma unroll
    for (int u = 0; u <= V; ++u) {
      A e = A(0), o = A(0);
#pragma unroll
      for (int t = 0; t < H; ++t) {
        e = fma(h0[2 * t], wa[u + t], e);
        e = fma(h1[2 * t], wd[u + t], e);
        o = fma(h0[2 * t + 1], wa[u + t], o);
        o = fma(h1[2 * t + 1], wd[u + t], o);
      }
      ze[u] = e;
      zo[u] = o;
    }
  }
}

template <typename T, int LM>
__global__ void __launch_bounds__(NT, 2)
dwt_synthesis_kernel(const __grid_constant__ Params<typename AccOf<T>::type, LM> p) {
  using A = typename AccOf<T>::type;
  using C = Cfg<T, LM>;
  constexpr int V = C::V;
  constexpr int W = C::WS;
  constexpr int PS = C::PSS;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  T* sbase = reinterpret_cast<T*>(smem_raw);
  T* const bufs[2] = {sbase, sbase + p.buf_len[0]};
  const int ns = p.nstage;
  T* const sa0 = sbase + p.stage_off;    // approximation ring (first level only)
  T* const sd0 = sa0 + ns * p.stage_len;  // detail ring
  A* const zext = reinterpret_cast<A*>(smem_raw + p.fold_off);
  A* const ztab = zext + C::FOLD_MAX;  // per edge output: sum of the folds it receives
  int* const ztg = reinterpret_cast<int*>(ztab + C::ZONE_MAX);
  const int cs = p.csize;
  const int rank = cs > 1 ? static_cast<int>(cg::this_cluster().block_rank()) : 0;
  const int64_t row = blockIdx.x / cs;
  const int tid = threadIdx.x;
  const int off = p.off;
  const A* h0 = p.taps;
  const A* h1 = p.taps + LM;

  for (int l = 0; l < p.nlev; ++l) {
    const Level& L = p.lv[l];
    const bool first = (l == 0), last = (l == p.nlev - 1);
    const int64_t n = L.n_in, nc = L.n_coef;
    const T* ga = first ? static_cast<const T*>(p.src) + row * L.a_len : nullptr;
    const T* gd = L.detail ? static_cast<const T*>(L.detail) + row * nc : nullptr;
    T* gdst = last ? static_cast<T*>(p.dst) + row * n : nullptr;
    const int64_t o_b = L.bnd[rank], o_e = L.bnd[rank + 1];
    const int ay = gdst ? elem_misalign(gdst) : 0;
    const int64_t c_b = syn_cb<V>(L, rank, ay);
    const int64_t c_e = o_e > o_b ? floor_div(o_e + ay + 2 * V - 1, 2 * V) : c_b;
    const bool odd = ((-(int64_t)ay - off) & 1) != 0;  // parity of (i_c - off), uniform
    const int64_t uorg = syn_ufirst(c_b, V, ay, off);
    // resident destination: the next level's window origin
    T* sdst = nullptr;
    int64_t sorg = 0;
    if (!last) {
      const Level& N = p.lv[l + 1];
      const bool nlast = (l + 1 == p.nlev - 1);
      const int ayn = nlast ? elem_misalign(static_cast<T*>(p.dst) + row * N.n_in) : 0;
      sdst = bufs[l & 1];
      sorg = syn_ufirst(syn_cb<V>(N, rank, ayn), V, ayn, off) - kMargin;
    }
    T* sa = first ? nullptr : bufs[(l - 1) & 1];
    const Level* Pv = first ? nullptr : &p.lv[l - 1];

    // 0. tiles 0 .. ns-2 of the detail (and, first level, approximation) rows: issued first so
    //    that their latency overlaps the halo and fold work; every later level had them
    //    prefetched at the end of the previous level.
    const int64_t ntiles = (c_e - c_b + NT - 1) / NT;
    auto stage_tile = [&](int64_t t) {
      const int64_t u0 = syn_ufirst(c_b + t * NT, V, ay, off);
      const int k = static_cast<int>(t % ns) * p.stage_len;
      const int span = static_cast<int>(imin(p.stage_span, V * imin(NT, c_e - c_b - t * NT) + W));
      stage_coef<T, PS>(sd0 + k, gd, u0, span, nc);
      if (first) stage_coef<T, PS>(sa0 + k, ga, u0, span, nc);
    };
    if (first) {  // ring prologue: exactly ns-1 groups (see the analysis kernel)
      for (int64_t k = 0; k < ns - 1; ++k) {
        if (k < ntiles) stage_tile(k);
        cp_async_commit();
      }
    }
    // 1. halo of the resident approximation (neighbours via DSMEM; zero outside [0, nc))
    if (!first && c_e > c_b) {
      // samples at or past nc are pywt's trimmed tail: they read as zero like the exterior
      const int64_t in_b = imin(Pv->bnd[rank], nc), in_e = imin(Pv->bnd[rank + 1], nc);
      const int64_t need_hi = uorg + V * (c_e - c_b) + W;
      const int64_t nl = imax(0, imin(in_b, need_hi) - uorg);
      const int64_t r0 = imax(in_e, uorg);
      const int64_t nr = imax(0, need_hi - r0);
      for (int64_t k = tid; k < nl + nr; k += NT) {
        const int64_t e = k < nl ? uorg + k : r0 + (k - nl);
        T v = T(0);
        if (e >= 0 && e < nc) {
          const int ow = owner_of(Pv->bnd, cs, e);
          const int64_t org_ow = syn_ufirst(syn_cb<V>(L, ow, ay), V, ay, off);
          v = peer_load(sa, rank, ow, sidx<PS>(static_cast<int>(e - org_ow + kMargin)));
        }
        sa[sidx<PS>(static_cast<int>(e - uorg + kMargin))] = v;
      }
    }

    // 2. exterior positions of the extended range, folded back onto ext(p); only CTAs whose
    //    outputs reach an end of the row need them
    const int64_t pmin = off - (LM - 1), pmax = 2 * (nc - 1) + off;
    const int E = L.fold_n;
    const int64_t nleft = imax(0, imin(-1, pmax) - pmin + 1);
    const int64_t rstart = imax(n, pmin);
    const int64_t zedge0 = imax(1 - pmin, pmax - n + 2);
    const bool fold_here = E > 0 && (2 * zedge0 >= n || o_b < zedge0 || o_e > n - zedge0);
    for (int e = tid; fold_here && e < E; e += NT) {
      const int64_t pp = e < nleft ? pmin + e : rstart + (e - nleft);
      A av[LM], dv[LM];
#pragma unroll
      for (int j = 0; j < LM; ++j) {  // gather first: independent (possibly remote) loads
        const int64_t q = pp - off + j;
        const int64_t o = q >> 1;
        av[j] = A(0);
        dv[j] = A(0);
        if ((q & 1) == 0 && o >= 0 && o < nc) {
          if (first) {
            av[j] = to_acc<T>(ga[o]);
          } else {
            const int ow = owner_of(Pv->bnd, cs, o);
            const int64_t org_ow = syn_ufirst(syn_cb<V>(L, ow, ay), V, ay, off);
            av[j] = to_acc<T>(
                peer_load(sa, rank, ow, sidx<PS>(static_cast<int>(o - org_ow + kMargin))));
          }
          if (gd) dv[j] = to_acc<T>(gd[o]);
        }
      }
      A z = A(0);
#pragma unroll
      for (int j = 0; j < LM; ++j) {
        z = fma(h0[j], av[j], z);
        z = fma(h1[j], dv[j], z);
      }
      zext[e] = z;
      ztg[e] = static_cast<int>(ext_index(pp, n, L.mode, L.P));
    }
    // fold table: edge output i (i < zedge, or i >= n - zedge, or every i of a short row)
    // collects the folds mapped onto it, so the direct pass adds one value per edge output
    const int64_t zedge_t = imax(1 - pmin, pmax - n + 2);
    const bool zall = 2 * zedge_t >= n;
    const int zcount = fold_here ? static_cast<int>(zall ? n : 2 * zedge_t) : 0;
    if (fold_here) {
      __syncthreads();
      for (int t = tid; t < zcount; t += NT) {
        const int64_t i = zall ? t : (t < zedge_t ? t : n - 2 * zedge_t + t);
        A acc = A(0);
        for (int e = 0; e < E; ++e)
          if (ztg[e] == i) acc += zext[e];
        ztab[t] = acc;
      }
    }
    const int64_t zedge = imax(1 - pmin, pmax - n + 2);
    const bool fold_all = 2 * zedge >= n;

    // 3. direct pass over thread chunks of 2V outputs (16-byte aligned in the output row); a
    //    chunk needs the fold check only when it touches either end of the output row
    const int64_t fold_lo = E > 0 ? (fold_all ? n : zedge) : 0;
    const int64_t fold_hi = E > 0 ? (fold_all ? 0 : n - zedge) : n;
    for (int64_t t = 0; t < ntiles; ++t) {
      if (t + ns - 1 < ntiles) stage_tile(t + ns - 1);
      cp_async_commit();
      cp_async_wait_ring(ns);
      __syncthreads();  // stage t, the halo and the fold arrays visible to every thread
      const int64_t c = c_b + t * NT + tid;
      if (c < c_e) {
        const int64_t i_c = c * 2 * V - ay;
        const int k0 = static_cast<int>(t % ns) * p.stage_len;
        A wa[W], wd[W];
        const T* sdc = sd0 + k0 + (V + 1) * tid;
#pragma unroll
        for (int i = 0; i < W; ++i) wd[i] = to_acc<T>(sdc[i + (i >> PS)]);
        if (first) {
          const T* sac = sa0 + k0 + (V + 1) * tid;
#pragma unroll
          for (int i = 0; i < W; ++i) wa[i] = to_acc<T>(sac[i + (i >> PS)]);
        } else {
          const int rel = static_cast<int>(c - c_b);
          const T* sw = sa + (V + 1) * rel + sidx<PS>(kMargin);
#pragma unroll
          for (int i = 0; i < W; ++i) wa[i] = to_acc<T>(sw[i + (i >> PS)]);
        }
        A zo[V + 1], ze[V + 1];
        syn_compute<T, A, LM>(p.taps, wa, wd, zo, ze);
        const bool edge = i_c < fold_lo || i_c + 2 * V > fold_hi;
        T out[2 * V];
#pragma unroll
        for (int k = 0; k < 2 * V; ++k) {
          // even start: ze(0), zo(1), ze(1), zo(2), ...;  odd start: zo(0), ze(0), zo(1), ...
          A val = odd ? ((k & 1) ? ze[k >> 1] : zo[k >> 1])
                      : ((k & 1) ? zo[(k + 1) >> 1] : ze[k >> 1]);
          if (edge) {
            const int64_t i = i_c + k;
            if (i >= 0 && i < n && (i < fold_lo || i >= fold_hi))
              val += ztab[zall ? i : (i < zedge_t ? i : i - n + 2 * zedge_t)];
          }
          out[k] = from_acc<T>(val);
        }
        const bool full = i_c >= o_b && i_c + 2 * V <= o_e;
        if (sdst) {
          const int base = static_cast<int>(i_c - sorg);
#pragma unroll
          for (int k = 0; k < 2 * V; ++k)
            if (i_c + k >= o_b && i_c + k < o_e) sdst[sidx<PS>(base + k)] = out[k];
        } else if (full) {
          store_vec<T, 2 * V>(gdst + i_c, out);
        } else {
#pragma unroll
          for (int k = 0; k < 2 * V; ++k)
            if (i_c + k >= o_b && i_c + k < o_e) gdst[i_c + k] = out[k];
        }
      }
      __syncthreads();  // stage slot free for refill
    }
    if (!last) {  // prefetch the next level's first tiles (its ring prologue)
      const Level& N = p.lv[l + 1];
      const bool nlast = (l + 1 == p.nlev - 1);
      const int ayn = nlast ? elem_misalign(static_cast<T*>(p.dst) + row * N.n_in) : 0;
      const int64_t cbn = syn_cb<V>(N, rank, ayn);
      const int64_t ob = N.bnd[rank], oe = N.bnd[rank + 1];
      const int64_t cen = oe > ob ? floor_div(oe + ayn + 2 * V - 1, 2 * V) : cbn;
      const int64_t ntn = (cen - cbn + NT - 1) / NT;
      const T* gdn = N.detail ? static_cast<const T*>(N.detail) + row * N.n_coef : nullptr;
      for (int64_t k = 0; k < ns - 1; ++k) {
        if (k < ntn) {
          const int span =
              static_cast<int>(imin(p.stage_span, V * imin(NT, cen - cbn - k * NT) + W));
          stage_coef<T, PS>(sd0 + static_cast<int>(k % ns) * p.stage_len, gdn,
                            syn_ufirst(cbn + k * NT, V, ayn, off), span, N.n_coef);
        }
        cp_async_commit();
      }
    }
    group_sync(cs);
  }
}

// ------------------------------------------------------------------------------ host

constexpr int kLM[] = {2, 4, 6, 8, 10, 12, 16, 20, 24, 32, 40, 64};

}  // namespace dwtk
}  // namespace fdwt

#include "dwt_syn_tile.cuh"
#include "dwt_stream.cuh"
#include "dwt_stream2.cuh"
#include "dwt_stream3.cuh"

namespace fdwt {
namespace dwtk {

inline int pick_lm(int L) {
  for (int lm : kLM)
    if (L <= lm) return lm;
  return -1;
}

struct Seg {
  int l0, l1;  // inclusive level range
  int csize;
  size_t smem;
  int buf_len[2];
  int stage_span, stage_len, nstage;
  int fold_off;
  std::vector<std::vector<int32_t>> bnd;  // per level of the segment: cs+1 boundaries
};

// Output partitions of the levels [l0, l1] for cluster size cs (see the kernel header).
inline std::vector<std::vector<int32_t>> partitions(const std::vector<Level>& lv, int l0, int l1,
                                                    int cs, int off, int LM, int V,
                                                    bool analysis) {
  std::vector<std::vector<int32_t>> out;
  for (int l = l0; l <= l1; ++l) {
    const int64_t len = analysis ? lv[l].a_len : lv[l].n_in;
    std::vector<int32_t> b(cs + 1);
    b[0] = 0;
    b[cs] = static_cast<int32_t>(len);
    for (int k = 1; k < cs; ++k) {
      int64_t v;
      if (l == l0) {
        const int64_t q = analysis ? V : 2 * V;
        v = (len * k / cs) / q * q;
      } else if (analysis) {
        v = floor_div(out.back()[k] - off + LM, 2);  // ceil((B - off + LM - 1) / 2)
      } else {
        v = 2 * static_cast<int64_t>(out.back()[k]) + off - 1;
      }
      v = std::max<int64_t>(v, b[k - 1]);
      v = std::min<int64_t>(v, len);
      b[k] = static_cast<int32_t>(v);
    }
    out.push_back(b);
  }
  return out;
}

// Shared memory of one launch covering levels [l0, l1] with cluster size cs.
template <typename T, int LM>
Seg plan_one(const std::vector<Level>& lv, int l0, int l1, int cs, int off, bool analysis,
             int nstage_max) {
  using C = Cfg<T, LM>;
  using A = typename AccOf<T>::type;
  constexpr int V = C::V;
  Seg s{l0, l1, cs, 0, {0, 0}, 0, 0, 1, 0, {}};
  s.bnd = partitions(lv, l0, l1, cs, off, LM, V, analysis);
  // resident buffers per CTA: level l's outputs live in buffer (l - l0) & 1 and must hold the
  // next level's input window span (which contains the CTA's part of those outputs, give or
  // take one chunk of alignment slack), plus margins
  int64_t buf[2] = {0, 0};
  for (int l = l0 + 1; l <= l1; ++l) {
    const auto& bi = s.bnd[l - l0 - 1];
    const auto& bo = s.bnd[l - l0];
    for (int k = 0; k < cs; ++k) {
      const int64_t outs = bo[k + 1] - bo[k];
      const int64_t ins = bi[k + 1] - bi[k];
      const int64_t span = analysis ? 2 * (outs + 2 * V) + LM + 4 * V : outs / 2 + 4 * V + LM;
      int64_t& b = buf[(l - 1 - l0) & 1];
      b = std::max(b, kMargin + std::max(span, ins + 4 * V + LM) + 8);
    }
  }
  const int PS = analysis ? C::PSA : C::PSS;
  for (int i = 0; i < 2; ++i)
    s.buf_len[i] = static_cast<int>(buf[i] == 0 ? 0 : buf[i] + (buf[i] >> PS) + 16);
  int64_t maxchunks = 0;
  for (int l = l0; l <= l1; ++l) {
    const auto& b = s.bnd[l - l0];
    for (int k = 0; k < cs; ++k)
      maxchunks = std::max<int64_t>(maxchunks, (b[k + 1] - b[k]) / (analysis ? V : 2 * V) + 2);
  }
  const int64_t per_tile = std::min<int64_t>(maxchunks, NT);
  const int64_t tiles = (maxchunks + NT - 1) / NT;
  s.nstage = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(nstage_max, tiles)));
  if (analysis) {
    s.stage_span = static_cast<int>(2 * V * per_tile + LM - 2);
    s.stage_len = static_cast<int>(s.stage_span + (s.stage_span >> PS) + 16);
    const int64_t stage = int64_t(s.stage_len) * s.nstage;
    // the stages are used by the first level only, while buffer 1 is still free
    const int64_t total = s.buf_len[0] + std::max<int64_t>(s.buf_len[1], stage);
    s.smem = static_cast<size_t>(total) * sizeof(T) + 16;
  } else {
    s.stage_span = static_cast<int>(V * per_tile + LM / 2 + 2);
    s.stage_len = static_cast<int>(s.stage_span + (s.stage_span >> PS) + 16);
    const int64_t elems =
        int64_t(s.buf_len[0]) + s.buf_len[1] + 2 * int64_t(s.nstage) * s.stage_len;
    s.fold_off = static_cast<int>((elems * sizeof(T) + 15) / 16 * 16);
    s.smem = s.fold_off + C::FOLD_MAX * (sizeof(A) + sizeof(int)) + C::ZONE_MAX * sizeof(A) + 16;
  }
  return s;
}

// Greedy segmentation: each launch takes as many levels as fit.  The budget first leaves room
// for two CTAs per SM, then one.  Among the fitting (cluster size, ring depth) choices the one
// reaching the farthest level wins, then the smaller cluster (every level of a cluster pays a
// cluster barrier and DSMEM halo traffic), then the deeper staging ring.
//
// An analysis whose first segment needs a cluster (rows too long for one CTA to keep a level
// resident) ends that segment after kClusterLevels levels: the deeper levels of a cluster run
// with few outputs per CTA between cluster barriers and leave the SMs idle, while the next
// segment's rows, 2^kClusterLevels times shorter, fit one CTA per row.  The extra write and
// read of the handed-over approximation costs less than that (measured on B200, db8 fp32 and
// fp64 at 16K..64K samples per row: 10-25% faster analyses).
constexpr int kClusterLevels = 2;

template <typename T, int LM>
std::vector<Seg> plan_segments(const std::vector<Level>& lv, size_t budget, int off,
                               bool analysis) {
  std::vector<Seg> segs;
  const int nl = static_cast<int>(lv.size());
  int l0 = 0;
  int lmax = nl - 1;  // last level the segment being planned may take
  while (l0 < nl) {
    Seg best{};
    bool have = false;
    for (int pass = 0; pass < 2 && !have; ++pass) {
      const size_t lim = pass == 0 ? budget / 2 : budget;
      for (int cs = 1; cs <= kMaxCluster; cs *= 2) {
        for (int ns = 3; ns >= 1; --ns) {
          Seg s = plan_one<T, LM>(lv, l0, l0, cs, off, analysis, ns);
          if (s.smem > lim) continue;
          while (s.l1 + 1 <= lmax && s.l1 + 1 - l0 + 1 <= kMaxLevels) {
            Seg t = plan_one<T, LM>(lv, l0, s.l1 + 1, cs, off, analysis, ns);
            if (t.smem > lim) break;
            s = t;
          }
          if (!have || s.l1 > best.l1) {
            best = s;
            have = true;
          }
        }
      }
    }
    if (!have) best = plan_one<T, LM>(lv, l0, l0, kMaxCluster, off, analysis, 1);
    if (analysis && segs.empty() && lmax == nl - 1 && best.csize > 1 &&
        best.l1 - l0 + 1 > kClusterLevels) {
      lmax = l0 + kClusterLevels - 1;  // replan the first segment with fewer levels
      continue;
    }
    lmax = nl - 1;
    segs.push_back(best);
    l0 = best.l1 + 1;
  }
  return segs;
}

// Workspace: two ping-pong regions, each big enough for any approximation handed over
// between consecutive segments.
inline size_t handover_bytes(const std::vector<Level>& lv, const std::vector<Seg>& segs,
                             int64_t rows, size_t esize, bool analysis) {
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

template <typename K, typename P>
int launch(K kern, const P& p, int64_t rows, int cs, size_t smem, cudaStream_t stream) {
  int st = allow_max_dynamic_smem(reinterpret_cast<const void*>(kern));
  if (st != FDWT_OK) return st;
  if ((st = pre_launch(stream)) != FDWT_OK) return st;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(rows * cs));
  cfg.blockDim = dim3(NT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = cs;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = cs > 1 ? 1 : 0;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  if (e != cudaSuccess) {
    set_cuda_error(e);
    return FDWT_ERR_CUDA;
  }
  return launch_status();
}

template <typename T, int LM, bool ANALYSIS>
int run(int64_t rows, const void* src0, std::vector<Level> lv, void* dst_final,
        const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
        cudaStream_t stream, size_t* ws_needed, bool allow_stream = true);

// Analysis whose finest levels stream (dwt_stream.cuh, dwt_stream2.cuh, dwt_stream3.cuh): from
// the finest level on, each triple of levels that fuses runs as one three-level pass, else each
// pair that fuses as a two-level pass, else each level that streams as a one-level pass; the
// approximations are handed over through two alternating workspace regions; the remaining
// (short-row) levels run on the cluster kernel after them.  A handover between two streaming
// stages stores its rows 16 bytes apart (length rounded up), so that the next stage's bulk
// copies start on 16-byte boundaries whatever the coefficient lengths (odd in every mode but
// periodization); the handover into the cluster kernel stays unpadded.
// FDWT_ERR_UNSUPPORTED when the finest level does not stream (or x is not 16-byte aligned).
template <typename T, int LM>
int run_ana_stages(int64_t rows, const void* src0, const std::vector<Level>& lv, void* dst_final,
                   const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
                   cudaStream_t stream, size_t* ws_needed) {
  using A = typename AccOf<T>::type;
  constexpr int64_t VW = 16 / static_cast<int64_t>(sizeof(A));
  const int nl = static_cast<int>(lv.size());
  if (ws_needed == nullptr && (reinterpret_cast<uintptr_t>(src0) & 15) != 0)
    return FDWT_ERR_UNSUPPORTED;
  // input row stride of level c when a streaming stage feeds it (x itself for c = 0)
  auto pitch = [&](int c) { return c == 0 ? lv[0].n_in : (lv[c].n_in + VW - 1) / VW * VW; };
  const int64_t r1 = std::max<int64_t>(rows, 1);
  std::vector<std::pair<int, int>> stages;  // (first level, levels)
  int c = 0;
  while (c < nl) {
    const int64_t xs = pitch(c);
    if (c + 2 < nl && plan_ana3<T, LM>(r1, lv[c], lv[c + 1], lv[c + 2], off, xs).ok) {
      stages.emplace_back(c, 3);
      c += 3;
    } else if (c + 1 < nl && plan_ana2<T, LM>(r1, lv[c], lv[c + 1], off, xs).ok) {
      stages.emplace_back(c, 2);
      c += 2;
    } else if (ana_streams<T, LM>(lv[c], xs)) {
      stages.emplace_back(c, 1);
      c += 1;
    } else {
      break;
    }
  }
  if (stages.empty()) return FDWT_ERR_UNSUPPORTED;
  const int ns = static_cast<int>(stages.size());
  // approximation row stride of stage i: padded when the next stage streams
  auto out_pitch = [&](int i) {
    const int last = stages[i].first + stages[i].second - 1;
    return i + 1 < ns ? pitch(last + 1) : lv[last].a_len;
  };
  size_t region[2] = {0, 0};
  for (int i = 0; i < ns; ++i) {
    const int last = stages[i].first + stages[i].second - 1;
    if (last == nl - 1) continue;
    const size_t b = (static_cast<size_t>(rows) * out_pitch(i) * sizeof(T) + 255) & ~size_t(255);
    region[i & 1] = std::max(region[i & 1], b);
  }
  const std::vector<Level> rest(lv.begin() + c, lv.end());
  size_t rest_ws = 0;
  if (!rest.empty()) {
    const int st = run<T, LM, true>(rows, nullptr, rest, nullptr, h0, h1, L, off, nullptr, 0,
                                    stream, &rest_ws, false);
    if (st != FDWT_OK) return st;
  }
  const size_t need = region[0] + region[1] + rest_ws;
  if (ws_needed) {
    *ws_needed = need;
    return FDWT_OK;
  }
  if (rows == 0) return FDWT_OK;
  if (need > 0 && (ws == nullptr || ws_bytes < need)) return FDWT_ERR_WORKSPACE;
  unsigned char* base = static_cast<unsigned char*>(ws);
  unsigned char* reg[2] = {base, base + region[0]};
  const void* src = src0;
  for (int i = 0; i < ns; ++i) {
    const int k = stages[i].first, m = stages[i].second;
    void* a_out = k + m - 1 == nl - 1 ? dst_final : static_cast<void*>(reg[i & 1]);
    const int64_t xs = pitch(k), as = out_pitch(i);
    int st = m == 3 ? run_ana3_stream<T, LM>(rows, src, lv[k], lv[k + 1], lv[k + 2], xs, a_out,
                                             as, h0, h1, L, off, stream)
             : m == 2 ? run_ana2_stream<T, LM>(rows, src, lv[k], lv[k + 1], xs, a_out, as, h0,
                                               h1, L, off, stream)
                      : run_ana_stream<T, LM>(rows, src, lv[k], xs, a_out, as, h0, h1, L, off,
                                              stream);
    // a one-level stage with unpadded rows on both sides can run on the cluster kernel; any
    // other refusal sends the whole call to the cluster plan
    if (st == FDWT_ERR_UNSUPPORTED && m == 1 && xs == lv[k].n_in && as == lv[k].a_len)
      st = run<T, LM, true>(rows, src, std::vector<Level>(1, lv[k]), a_out, h0, h1, L, off,
                            nullptr, 0, stream, nullptr, false);
    if (st != FDWT_OK) return st;
    src = a_out;
  }
  if (rest.empty()) return FDWT_OK;
  return run<T, LM, true>(rows, src, rest, dst_final, h0, h1, L, off,
                          rest_ws ? base + region[0] + region[1] : nullptr, rest_ws, stream,
                          nullptr, false);
}

template <typename T, int LM, bool ANALYSIS>
int run(int64_t rows, const void* src0, std::vector<Level> lv, void* dst_final,
        const double* h0, const double* h1, int L, int off, void* ws, size_t ws_bytes,
        cudaStream_t stream, size_t* ws_needed, bool allow_stream) {
  using A = typename AccOf<T>::type;
  using C = Cfg<T, LM>;
  const size_t budget = static_cast<size_t>(max_smem_optin()) - 2048;
  if (ANALYSIS && allow_stream) {
    size_t stream_need = 0;
    const int sa = run_ana_stages<T, LM>(rows, src0, lv, dst_final, h0, h1, L, off, ws, ws_bytes,
                                         stream, ws_needed ? &stream_need : nullptr);
    if (ws_needed != nullptr && sa == FDWT_OK) {
      // At run time an x that is not 16-byte aligned does not stream: the call then takes the
      // cluster plan below, so the query covers both plans.
      size_t cluster_need = 0;
      if (run<T, LM, true>(rows, src0, lv, dst_final, h0, h1, L, off, nullptr, 0, stream,
                           &cluster_need, false) != FDWT_OK)
        cluster_need = 0;
      *ws_needed = std::max(stream_need, cluster_need);
      return FDWT_OK;
    }
    if (sa != FDWT_ERR_UNSUPPORTED) return sa;
  }
  if (!ANALYSIS) {
    // independent output tiles when their staging fits; the cluster kernel otherwise
    const int ts = run_syn_tiles<T, LM>(rows, src0, lv, dst_final, h0, h1, L, off, ws,
                                        ws_bytes, stream, ws_needed);
    if (ts != FDWT_ERR_UNSUPPORTED) return ts;
  }
  if (!ANALYSIS) {
    for (auto& l : lv) {
      l.fold_n = fold_count(l.n_in, l.n_coef, off, LM, l.mode);
      if (l.fold_n > C::FOLD_MAX) return FDWT_ERR_UNSUPPORTED;
      const int64_t pmin = off - (LM - 1), pmax = 2 * (l.n_coef - 1) + off;
      const int64_t ze = std::max<int64_t>(1 - pmin, pmax - l.n_in + 2);
      if (l.fold_n > 0 && std::min<int64_t>(l.n_in, 2 * ze) > C::ZONE_MAX) return FDWT_ERR_UNSUPPORTED;
    }
  }
  for (const auto& l : lv)
    if (l.n_in > 0x3fffffffLL || l.a_len > 0x3fffffffLL) return FDWT_ERR_UNSUPPORTED;
  auto segs = plan_segments<T, LM>(lv, budget, off, ANALYSIS);
  const size_t need = handover_bytes(lv, segs, rows, sizeof(T), ANALYSIS);
  if (ws_needed) {
    *ws_needed = need;
    return FDWT_OK;
  }
  if (rows == 0) return FDWT_OK;
  if (need > 0 && (ws == nullptr || ws_bytes < need)) return FDWT_ERR_WORKSPACE;
  if (rows * kMaxCluster > 0x7fffffffLL) return FDWT_ERR_UNSUPPORTED;
  const size_t half = segs.size() > 2 ? need / 2 : need;
  const void* src = src0;
  for (size_t s = 0; s < segs.size(); ++s) {
    const Seg& g = segs[s];
    if (g.smem > budget) return FDWT_ERR_UNSUPPORTED;
    Params<A, LM> p{};
    p.rows = rows;
    p.src = src;
    p.dst = (s + 1 == segs.size()) ? dst_final : static_cast<unsigned char*>(ws) + (s % 2) * half;
    p.nlev = g.l1 - g.l0 + 1;
    p.off = off;
    p.csize = g.csize;
    p.buf_len[0] = g.buf_len[0];
    p.buf_len[1] = g.buf_len[1];
    p.stage_off = ANALYSIS ? g.buf_len[0] : g.buf_len[0] + g.buf_len[1];
    p.stage_len = g.stage_len;
    p.stage_span = g.stage_span;
    p.nstage = g.nstage;
    p.fold_off = g.fold_off;
    for (int j = 0; j < LM; ++j) {
      const A a = j < L ? static_cast<A>(h0[j]) : A(0);
      const A d = j < L ? static_cast<A>(h1[j]) : A(0);
      if (ANALYSIS) {
        p.taps[2 * j] = a;
        p.taps[2 * j + 1] = d;
      } else {
        p.taps[j] = a;
        p.taps[LM + j] = d;
      }
    }
    for (int k = 0; k < p.nlev; ++k) {
      Level v = lv[g.l0 + k];
      for (int r = 0; r <= kMaxCluster; ++r)
        v.bnd[r] = r <= g.csize ? g.bnd[k][r] : g.bnd[k][g.csize];
      p.lv[k] = v;
    }
    const int st = ANALYSIS
        ? launch(dwt_analysis_kernel<T, LM>, p, rows, g.csize, g.smem, stream)
        : launch(dwt_synthesis_kernel<T, LM>, p, rows, g.csize, g.smem, stream);
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

#define FDWT_DWT_CASE(T, M, AN)                                                              \
  case M:                                                                                    \
    return run<T, M, AN>(rows, src, lv, dst, h0, h1, L, off, ws, ws_bytes, stream, ws_needed);

#define FDWT_DWT_SWITCH(T, AN)                                                                \
  switch (LM) {                                                                               \
    FDWT_DWT_CASE(T, 2, AN) FDWT_DWT_CASE(T, 4, AN) FDWT_DWT_CASE(T, 6, AN)                   \
    FDWT_DWT_CASE(T, 8, AN) FDWT_DWT_CASE(T, 10, AN) FDWT_DWT_CASE(T, 12, AN)                 \
    FDWT_DWT_CASE(T, 16, AN) FDWT_DWT_CASE(T, 20, AN) FDWT_DWT_CASE(T, 24, AN)                \
    FDWT_DWT_CASE(T, 32, AN) FDWT_DWT_CASE(T, 40, AN) FDWT_DWT_CASE(T, 64, AN)                \
    default: return FDWT_ERR_UNSUPPORTED;                                                     \
  }

#define FDWT_DWT_INSTANTIATE(T)                                                               \
  template <>                                                                                 \
  int analysis_dtype<T>(int LM, int64_t rows, const void* src, std::vector<Level> lv,         \
                        void* dst, const double* h0, const double* h1, int L, int off,        \
                        void* ws, size_t ws_bytes, cudaStream_t stream, size_t* ws_needed) {  \
    FDWT_DWT_SWITCH(T, true)                                                                  \
  }                                                                                           \
  template <>                                                                                 \
  int synthesis_dtype<T>(int LM, int64_t rows, const void* src, std::vector<Level> lv,        \
                         void* dst, const double* h0, const double* h1, int L, int off,       \
                         void* ws, size_t ws_bytes, cudaStream_t stream, size_t* ws_needed) { \
    FDWT_DWT_SWITCH(T, false)                                                                 \
  }

}  // namespace dwtk
}  // namespace fdwt
