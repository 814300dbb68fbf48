// Shared host/device helpers for the msa_b200 CUDA library (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <string>

#include "../../include/msa_b200.h"

namespace msa {

// ------------------------------------------------------------------ errors
int set_error(int code, const char* fmt, ...);

#define MSA_CHECK_ARG(cond, ...)                                                 \
  do {                                                                          \
    if (!(cond)) return ::msa::set_error(MSA_ERR_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

#define MSA_CUDA_RETURN(expr)                                                            \
  do {                                                                                  \
    cudaError_t err__ = (expr);                                                         \
    if (err__ != cudaSuccess)                                                           \
      return ::msa::set_error(MSA_ERR_CUDA, "%s: %s (%s:%d)", #expr,                   \
                              cudaGetErrorString(err__), __FILE__, __LINE__);           \
  } while (0)

// Count `n` kernel launches for msa_kernel_launches().
void count_launches(int n);

// Per-kernel device timing (msa_timing_enable / msa_timing_read): while enabled,
// timing_begin records a start event on `st` and returns its slot (-1 when off);
// timing_end records the matching end event under `name`.
int timing_begin(cudaStream_t st);
void timing_end(const char* name, int slot, cudaStream_t st);

// Status of the kernels just launched on the stream (launch-time errors only).
inline int launch_status(const char* what) {
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return set_error(MSA_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(err));
  return MSA_OK;
}

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline bool valid_dtype(int d) { return d == MSA_F32 || d == MSA_F16 || d == MSA_BF16; }

// ------------------------------------------------------------------ device
__device__ __forceinline__ double load_f64(const void* p, int64_t i, int dtype) {
  if (dtype == MSA_BF16) return (double)__bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
  if (dtype == MSA_F16) return (double)__half2float(reinterpret_cast<const __half*>(p)[i]);
  return (double)reinterpret_cast<const float*>(p)[i];
}

// float64 result -> public dtype the way the reference produces it: its kernels
// write float32 and the host casts to the input dtype (sparse_attention.py:359,
// index_score.py:291-295), i.e. round to float32 first, then to bf16/f16
// (round to nearest even at each step). The float64 oracle's expected values
// are cast by torch the same way, so bf16 outputs that sit within a float32
// ulp of a bf16 rounding midpoint agree with the reference's tests.
__device__ __forceinline__ void store_from_f64(void* p, int64_t i, int dtype, double x) {
  const float f = __double2float_rn(x);
  if (dtype == MSA_BF16) {
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(f);
  } else if (dtype == MSA_F16) {
    reinterpret_cast<__half*>(p)[i] = __float2half_rn(f);
  } else {
    reinterpret_cast<float*>(p)[i] = f;
  }
}

// Sequence containing packed token t: the largest s with cu[s] <= t. Because
// cu[nseq] = T > t, cu[s+1] > t, so empty sequences are never returned.
__device__ __forceinline__ int find_sequence(const int32_t* cu, int nseq, int64_t t) {
  int lo = 0, hi = nseq - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if ((int64_t)__ldg(cu + mid) <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Deterministic float64 dot product: fixed left-to-right order with explicit
// round-to-nearest products and sums so every call site produces identical bits
// (winner tests in the score backward compare recomputed values for equality).
__device__ __forceinline__ double dot_f64(const double* __restrict__ a, const void* b, int64_t b_off,
                                          int dtype, int n) {
  double s = 0.0;
  for (int i = 0; i < n; ++i) s = __dadd_rn(s, __dmul_rn(a[i], load_f64(b, b_off + i, dtype)));
  return s;
}

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_max(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

inline int ceil_div(int64_t a, int64_t b) { return (int)((a + b - 1) / b); }

}  // namespace msa
