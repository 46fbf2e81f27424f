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
  FDWT_ERR_CUDA = 4         /* a CUDA runtime call failed; see fdwt_last_cuda_error()      */
};

/* Human-readable name of a status code (static storage). */
const char* fdwt_status_string(int status);
/* The cudaError_t of the last FDWT_ERR_CUDA on the calling thread (0 if none). */
int fdwt_last_cuda_error(void);
/* ABI version of this library: major * 100 + minor. */
int fdwt_version(void);
/* Number of kernels this library has launched in the process (all threads, all devices). */
unsigned long long fdwt_launch_count(void);

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

#ifdef __cplusplus
}
#endif

#endif /* FDWT_B200_H */
