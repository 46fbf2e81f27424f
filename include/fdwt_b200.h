/*
 * fdwt_b200.h -- C ABI of the sm_100a wavelet filter-bank kernels (libfdwt_b200.so).
 *
 * Every entry point takes raw device pointers to contiguous row-major arrays, host arrays for
 * small descriptors (filter taps, level lengths, the Morlet plan), a dtype code and a CUDA
 * stream (a cudaStream_t passed as void*; NULL = the legacy default stream).  Outputs and
 * workspaces are allocated by the caller; nothing here allocates device memory or
 * synchronises the host.  Each call returns FDWT_OK (0) or an error code; the launch is
 * asynchronous on `stream`.
 *
 * The reference (Mousakaa/pytorch_morlet_fdwt, package `fdwt`) has no C interface: its
 * autograd Functions call Python launchers of Triton kernels.  Each entry point below names
 * the launcher(s) it replaces (path:line in the reference tree).
 */
#ifndef FDWT_B200_H
#define FDWT_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* element types: the storage type of the row arrays */
enum { FDWT_F32 = 0, FDWT_F64 = 1, FDWT_F16 = 2, FDWT_BF16 = 3 };

/* boundary modes, numbered like the reference's MODES (fdwt/kernels/dwt.py:30) */
enum {
  FDWT_MODE_ZERO = 0,
  FDWT_MODE_PERIODIC = 1,
  FDWT_MODE_SYMMETRIC = 2,
  FDWT_MODE_REFLECT = 3,
  FDWT_MODE_PERIODIZATION = 4
};

/* status codes */
enum {
  FDWT_OK = 0,
  FDWT_ERR_INVALID = 1,     /* bad argument: null pointer, negative or inconsistent size  */
  FDWT_ERR_UNSUPPORTED = 2, /* valid but outside what the kernels implement (e.g. L > 64)  */
  FDWT_ERR_WORKSPACE = 3,   /* workspace missing or smaller than the matching *_workspace() */
  FDWT_ERR_CUDA = 4,        /* a CUDA runtime call failed; see fdwt_last_cuda_error()      */
  FDWT_ERR_SCRATCH_LIMIT = 5 /* the call needs more than FDWT_NOALLOC_SCRATCH_BYTES        */
};

/* Human-readable name of a status code (static storage). */
const char* fdwt_status_string(int status);
/* The cudaError_t of the last FDWT_ERR_CUDA on the calling thread (0 if none). */
int fdwt_last_cuda_error(void);
/* ABI version of this library: major * 100 + minor. */
int fdwt_version(void);
/* Number of kernels this library has launched in the process (all threads, all devices). */
unsigned long long fdwt_launch_count(void);
/* Test hook.  While enabled (enable != 0), every kernel launch of this library is preceded,
 * on the same stream, by a kernel that sets every shared-memory word of every SM to the 32-bit
 * pattern `word` (e.g. a NaN or infinity bit pattern).  Shared memory is not cleared between
 * kernels, so a kernel that reads a cell it has not written then sees that pattern: tests use
 * this to check that no output depends on uninitialised shared memory.  Process-wide; the fill
 * kernels are not counted by fdwt_launch_count(). */
void fdwt_set_shared_memory_fill(int enable, unsigned int word);
/* Device-side error word of the current device: kernels that wait on asynchronous copies give
 * up after a bounded number of tries, store a nonzero code there (1: a copy never completed)
 * and return without finishing their work.  Synchronises the device, writes the code to
 * *code (0: none since the last call) and clears it. */
int fdwt_device_error(int* code);
/* Test hook of the bounded copy waits above (no counterpart in the reference).  While
 * extra_tx_bytes > 0, the streaming DWT kernels expect that many bytes more than they copy for
 * global tile 0, so its wait runs out without any fault (every issued copy still lands); the
 * kernel then stores 1 in the error word, waits for its copies still in flight and returns.
 * `tries` replaces the poll limit of the main waits (<= 0: the default 2^22); the wait for
 * copies in flight after a timeout polls at least 2^20 times.  Process-wide; (0, 0) restores
 * the defaults.  The per-device caches of this library (error word, device attributes,
 * allocation-free scratch) assume each device's primary context lives as long as the process
 * (no cudaDeviceReset between calls). */
void fdwt_set_copy_wait_test(unsigned int extra_tx_bytes, long long tries);
/* Test hook of the Morlet kernels (no counterpart in the reference).  While t_len > 0 every
 * Morlet forward and backward call runs on time tiles of t_len positions, the path rows too
 * long for one CTA's shared memory take, even where whole rows would fit (tests compare the
 * two paths).  Process-wide; 0 restores the automatic choice. */
void fdwt_set_cwt_tile_test(int t_len);

/* ------------------------------------------------------------------------------------------
 * Discrete wavelet transform.  One call runs every level of a multilevel transform (the
 * reference launches one Triton kernel per level from a Python loop).  Filter taps are host
 * arrays of `filter_len` doubles (even length, as FilterBank pads them); they are passed to
 * the kernels by value.
 * ---------------------------------------------------------------------------------------- */

/* Multilevel analysis: level l (1-based) maps its input (length n_l-1; n_0 = n) to
 *   cA_l[o] = sum_j h0[j] in_ext[2o + off - j],  cD_l[o] = sum_j h1[j] in_ext[2o + off - j]
 * for o < coef_len[l-1], `in_ext` being the input extended by `mode`.  The approximation that
 * feeds level l+1 is cA_l followed by pad_last[l-1] (0 or 1) zero samples.
 *   x      : (rows, n)
 *   out[0] : (rows, coef_len[levels-1] + pad_last[levels-1])    final approximation
 *   out[k] : (rows, coef_len[levels-k])  for k = 1..levels       details, coarsest first
 * pad_last may be NULL (no padding).  Replaces the analysis launcher
 * fdwt/kernels/dwt.py:191-206 as called by _Analysis.forward (fdwt/dwt.py:36-49) once per level
 * from wavedec (fdwt/dwt.py:146-158) and by _Synthesis.backward (fdwt/dwt.py:75-82). */
int fdwt_dwt_analysis(int dtype, int64_t rows, const void* x, int64_t n, int levels,
                      const int64_t* coef_len, const int64_t* pad_last, void* const* out,
                      const double* h0, const double* h1, int filter_len, int mode, int off,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Device workspace (bytes) fdwt_dwt_analysis needs for the same arguments (0 when every
 * level fits in one launch's shared memory). */
size_t fdwt_dwt_analysis_workspace(int dtype, int64_t rows, int64_t n, int levels,
                                   const int64_t* coef_len, const int64_t* pad_last,
                                   int filter_len, int mode, int off);

/* Multilevel synthesis: the exact transpose of fdwt_dwt_analysis, level by level from the
 * coarsest.  Level l maps (a, d) -- a = the first coef_len[l-1] samples of the incoming
 * approximation, d = the level's detail -- to the signal of length out_len[l-1]:
 *   y[i] = sum over extended positions p with ext(p) == i of
 *          sum_{j, o : 2o + off - j == p} h0[j] a[o] + h1[j] d[o]
 * (`ext` = the boundary map of `mode` for a signal of length out_len[l-1]).
 *   in[0]  : (rows, approx_len)  approximation entering the coarsest level; approx_len is
 *            coef_len[levels-1] or coef_len[levels-1] + 1 (the trailing sample is dropped)
 *   in[k]  : (rows, coef_len[levels-k]) details, coarsest first; NULL reads as zeros
 *   y      : (rows, out_len[0])
 * out_len[l] must be coef_len[l-1] or coef_len[l-1] + 1 for l >= 1 (pywt's trim rule).
 * Replaces the synthesis launcher fdwt/kernels/dwt.py:209-228 as called by
 * _Synthesis.forward (fdwt/dwt.py:59-73) from idwt / waverec (fdwt/dwt.py:114-135, 161-171)
 * and by _Analysis.backward (fdwt/dwt.py:51-56). */
int fdwt_dwt_synthesis(int dtype, int64_t rows, int levels, const void* const* in,
                       int64_t approx_len, const int64_t* coef_len, const int64_t* out_len,
                       void* y, const double* h0, const double* h1, int filter_len, int mode,
                       int off, void* workspace, size_t workspace_bytes, void* stream);

/* Device workspace (bytes) fdwt_dwt_synthesis needs for the same arguments. */
size_t fdwt_dwt_synthesis_workspace(int dtype, int64_t rows, int levels, int64_t approx_len,
                                    const int64_t* coef_len, const int64_t* out_len,
                                    int filter_len, int mode, int off);

/* Size of the static device array behind fdwt_dwt_analysis_noalloc (16 MiB). */
#define FDWT_NOALLOC_SCRATCH_BYTES ((size_t)16 << 20)

/* fdwt_dwt_analysis for callers that cannot allocate device memory while they run (a real-time
 * loop where cudaMalloc/cudaFree would synchronise the device, or a host whose own allocator
 * owns the GPU and cannot pass a workspace through its FFI).  No counterpart in the reference:
 * it has no C interface and allocates through torch.
 *
 * Same arguments and results as fdwt_dwt_analysis without the workspace pair.  The workspace
 * that long rows need is a file-scope device array of FDWT_NOALLOC_SCRATCH_BYTES compiled into
 * the library; every GPU that loads the library holds it until the process exits.  The call
 * allocates nothing.
 *  - Sizes whose fdwt_dwt_analysis_workspace() exceeds FDWT_NOALLOC_SCRATCH_BYTES return
 *    FDWT_ERR_SCRATCH_LIMIT without launching anything.
 *  - The first call on a device that needs the array (multi-launch rows) looks up the array's
 *    device address with that device current (cudaGetSymbolAddress) and caches it; make that
 *    first call before any stream capture.
 *  - Every call on a device shares the one array and leaves its contents behind.  Nothing in it
 *    needs to start at zero, but calls that overlap on the GPU (different streams, or different
 *    host threads, without ordering between them) race on it: serialise them. */
int fdwt_dwt_analysis_noalloc(int dtype, int64_t rows, const void* x, int64_t n, int levels,
                              const int64_t* coef_len, const int64_t* pad_last, void* const* out,
                              const double* h0, const double* h1, int filter_len, int mode,
                              int off, void* stream);

/* ------------------------------------------------------------------------------------------
 * Morlet continuous wavelet transform (the a-trous octave pyramid of MorletPlan).
 *
 * A plan describes the octaves exactly as the reference's MorletPlan computes them
 * (fdwt/cwt.py:80-139): octave j holds the scales order[oct_begin[j] .. +oct_count[j]) (global
 * scale indices, sorted by support) whose filters have 2*oct_half[j]+1 taps at spacing 2^j;
 * x_j (j >= 1) is the dilated half-band low-pass of x_{j-1} materialised on
 * [-margins[j], n + margins[j]).  Filters are the (n_scales*channels, 2*center+1) tensor of
 * MorletPlan.filters (row i*channels + c), read from device memory; every scale of octave j
 * uses the taps center-oct_half[j] .. center+oct_half[j], as the reference's CPU path does
 * (MorletPlan.filters makes the taps past a scale's support zero).
 * ---------------------------------------------------------------------------------------- */
#define FDWT_MAX_OCTAVES 24
#define FDWT_MAX_SCALES 256
#define FDWT_MAX_LOWPASS 49

typedef struct {
  int32_t n_octaves;  /* J + 1 */
  int32_t n_scales;   /* S */
  int32_t channels;   /* 2: complex Morlet, 1: its real part */
  int32_t center;     /* filters have 2*center+1 columns */
  int32_t c_lp;       /* the half-band filter has 2*c_lp+1 taps (0 for a single octave) */
  int32_t margins[FDWT_MAX_OCTAVES];
  int32_t oct_half[FDWT_MAX_OCTAVES];   /* 0 when the octave holds no scale */
  int32_t oct_begin[FDWT_MAX_OCTAVES];
  int32_t oct_count[FDWT_MAX_OCTAVES];
  int32_t order[FDWT_MAX_SCALES];
  int32_t support[FDWT_MAX_SCALES];     /* half-support (taps) of order[k] */
  double lowpass[FDWT_MAX_LOWPASS];     /* the full half-band filter, 2*c_lp+1 taps */
} fdwt_morlet_plan;

/* Row length.  A row whose pyramid buffers fit one CTA's shared memory is computed by one CTA;
 * longer rows run on time tiles whose buffers reach the pyramid's dependency cone past both ends
 * of the tile (forward), or as one launch per octave over tiles with the half-band chain's
 * gradient handed between octaves through the workspace (backward).  Any n up to 2^30 - 1 is
 * accepted; the workspace queries size both cases. */

/* Forward transform: y (rows, n_scales, n, channels) from x (rows, n).  Replaces the
 * per-octave launches of the forward and half-band launchers (fdwt/kernels/conv.py:306-329,
 * 411-430) issued by _MorletCWTFunction.forward (fdwt/cwt.py:217-244). */
int fdwt_cwt_forward(int dtype, int64_t rows, int64_t n, const void* x, const void* filters,
                     const fdwt_morlet_plan* plan, void* y, void* stream);

/* Fused scalogram mix: y[r, t] = sum_s a[d, s] |W_s[r, t]| + b[d, s] Re W_s[r, t], d = r % dim,
 * a and b (dim, n_scales); the scalogram is never written.  Replaces mix_forward
 * (fdwt/kernels/mix.py:74-89) and the half-band chain of _MorletMixFunction.forward
 * (fdwt/cwt.py:294-320). */
int fdwt_mix_forward(int dtype, int64_t rows, int64_t n, const void* x, const void* filters,
                     const fdwt_morlet_plan* plan, const void* a, const void* b, int64_t dim,
                     void* y, void* stream);

/* Fused spectral softmax: out[r, t] = sum_f softmax_f(|W_f[r, t]| * inv_tau) V_f[r, t] with
 * V (nch, n_scales) (row r uses V[r % nch]) or, when v_per_position, (rows / nch, n_scales, n)
 * (row r uses V[r / nch]).  Also writes the softmax max m and denominator l per (r, t) for
 * the backward pass.  Replaces forward_stage (fdwt/kernels/softmax.py:195-203) and the
 * octave loop of _SpectralSoftmaxFunction.forward (fdwt/cwt.py:417-450). */
int fdwt_specsoftmax_forward(int dtype, int64_t rows, int64_t n, const void* x,
                             const void* filters, const fdwt_morlet_plan* plan, const void* v,
                             int v_per_position, int64_t nch, double inv_tau, void* out, void* m,
                             void* l, void* stream);

/* Backward passes.  One kernel per call runs a row's whole adjoint chain (coarsest octave
 * first) and, when requested, the filter gradient; per-row partial sums are then reduced over
 * rows in a fixed order, so results are deterministic (except dL/dV of a per-position V, which
 * is accumulated with atomic adds).  Gradients are in the computation type (fp32 or fp64).
 * Null output pointers skip that output.  The workspace holds the rebuilt pyramid and the
 * per-row partials; query its size with the matching *_workspace function (need_gh says
 * whether gh will be requested). */

/* dL/dx (rows, n) and dL/dH (n_scales*channels, 2*center+1) from dL/dW (rows, n_scales, n,
 * channels).  x is only read when gh is requested.  Replaces backward_x, backward_h and the
 * transposed half-band (fdwt/kernels/conv.py:345-430) as issued by
 * _MorletCWTFunction.backward (fdwt/cwt.py:246-281). */
size_t fdwt_cwt_backward_workspace(int dtype, int64_t rows, int64_t n,
                                   const fdwt_morlet_plan* plan, int need_gh);
int fdwt_cwt_backward(int dtype, int64_t rows, int64_t n, const void* x, const void* filters,
                      const fdwt_morlet_plan* plan, const void* gy, void* gx, void* gh,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Backward of fdwt_mix_forward from dL/dy (rows, n): dL/dx, dL/dH, dL/da and dL/db (dim,
 * n_scales).  W is recomputed, never stored.  Replaces mix_backward (fdwt/kernels/mix.py:92-108)
 * and the backward_x / backward_h calls of _MorletMixFunction.backward (fdwt/cwt.py:322-376). */
size_t fdwt_mix_backward_workspace(int dtype, int64_t rows, int64_t n,
                                   const fdwt_morlet_plan* plan, int64_t dim, int need_gh);
int fdwt_mix_backward(int dtype, int64_t rows, int64_t n, const void* x, const void* filters,
                      const fdwt_morlet_plan* plan, const void* a, const void* b, int64_t dim,
                      const void* gy, void* gx, void* gh, void* ga, void* gb, void* workspace,
                      size_t workspace_bytes, void* stream);

/* MorletTokenMixer's layout.  x and y are (batch, n, dim) tensors, channel d of token q of item
 * b at (b*n + q)*dim + d, and y gets bias[d] added (bias may be null).  The reference
 * transposes x to (batch, dim, n) rows, calls morlet_mix, transposes back and adds the bias in
 * separate torch kernels (fdwt/layers.py:49-55); here the kernels read and write the token
 * layout themselves.  The backward takes dL/dy (batch, n, dim) and returns dL/dx in the same
 * layout, dL/dH, dL/da, dL/db (dim, n_scales) and dL/dbias (dim; null skips it). */
int fdwt_mix_tokens_forward(int dtype, int64_t batch, int64_t n, int64_t dim, const void* x,
                            const void* filters, const fdwt_morlet_plan* plan, const void* a,
                            const void* b, const void* bias, void* y, void* stream);
size_t fdwt_mix_tokens_backward_workspace(int dtype, int64_t batch, int64_t n, int64_t dim,
                                          const fdwt_morlet_plan* plan, int need_gh);
int fdwt_mix_tokens_backward(int dtype, int64_t batch, int64_t n, int64_t dim, const void* x,
                             const void* filters, const fdwt_morlet_plan* plan, const void* a,
                             const void* b, const void* gy, void* gx, void* gh, void* ga,
                             void* gb, void* gbias, void* workspace, size_t workspace_bytes,
                             void* stream);

/* Backward of fdwt_specsoftmax_forward from dL/dout (rows, n), given the forward's out, m and
 * l: dL/dx, dL/dH and dL/dV (the shape of V).  Replaces backward_stage
 * (fdwt/kernels/softmax.py:206-210) and the octave loop of _SpectralSoftmaxFunction.backward
 * (fdwt/cwt.py:452-509). */
size_t fdwt_specsoftmax_backward_workspace(int dtype, int64_t rows, int64_t n,
                                           const fdwt_morlet_plan* plan, int v_per_position,
                                           int64_t nch, int need_gh);
int fdwt_specsoftmax_backward(int dtype, int64_t rows, int64_t n, const void* x,
                              const void* filters, const fdwt_morlet_plan* plan, const void* v,
                              int v_per_position, int64_t nch, double inv_tau, const void* m,
                              const void* l, const void* out, const void* gout, void* gx,
                              void* gh, void* gv, void* workspace, size_t workspace_bytes,
                              void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FDWT_B200_H */
