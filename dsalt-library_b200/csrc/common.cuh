// Shared device helpers for the DSALT B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>

#include "dsalt_b200.h"

namespace dsalt {

// ---------------------------------------------------------------- dtypes
template <typename T> __device__ __forceinline__ float to_f32(T x);
template <> __device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ float to_f32<__half>(__half x) { return __half2float(x); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) {
  return __bfloat162float(x);
}

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// value of x after a round trip through T (the rounding torch applies when it
// stores a result in T)
template <typename T> __device__ __forceinline__ float round_to(float x) {
  return to_f32<T>(from_f32<T>(x));
}

// ---------------------------------------------------------------- warps
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ void flag_status(int32_t* status, int bit) {
  if (status) atomicOr(status, bit);
}

// Largest b in [0, S) with cu[b] <= t (sequence of packed token t).
__device__ __forceinline__ int find_seq(const int32_t* __restrict__ cu, int S, int64_t t) {
  int lo = 0, hi = S - 1;
  while (lo < hi) {
    int mid = (lo + hi + 1) >> 1;
    if ((int64_t)__ldg(cu + mid) <= t) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// ---------------------------------------------------------------- windows
// Per-query window under either semantics, reduced to the training form:
//   band     : 0 <= d <= wt            (d = i - j, integer)  -> W = floor(wt)
//   core     : d <= wt - edge           (soft-edge bias 0)
//   landmark : p <= i  and  float(p) < float(i) - wt
// Inference (integer w, dsalt_triton_attn.py:102-105,133-135) maps exactly to
// wt = max(trunc(w), 1) - 1 with edge = 0.
struct RowWindow {
  float wt;      // effective continuous window
  float core;    // wt - edge (float32, as the reference computes it)
  float win_lo;  // float(i) - wt (float32)
  int W;         // number of band keys before the diagonal (-1: empty band)
};

__device__ __forceinline__ RowWindow row_window(float w_raw, int i, int semantics, float win_edge) {
  RowWindow r;
  if (semantics == DSALT_INFER) {
    float tw = truncf(w_raw);
    tw = fminf(fmaxf(tw, 1.0f), 1073741824.0f);
    r.wt = tw - 1.0f;
    r.core = r.wt;
  } else {
    r.wt = w_raw;
    r.core = __fsub_rn(w_raw, win_edge);
  }
  r.win_lo = __fsub_rn((float)i, r.wt);
  if (!(r.wt >= 0.0f)) {
    r.W = -1;  // d = 0 is already outside the band (also catches NaN)
  } else {
    float f = floorf(fminf(r.wt, 1073741824.0f));
    r.W = (int)f;
  }
  return r;
}

// Soft-edge log-bias log σ((wt − d)/τ) for a band key at distance d
// (dsalt_triton_train.py:151-156): 0 in the core.
__device__ __forceinline__ float edge_bias(const RowWindow& r, float d, float inv_tau) {
  if (d <= r.core) return 0.0f;
  float z = (r.wt - d) * inv_tau;
  return -log1pf(expf(-z));
}
// d(bias)/d(wt) = (1 − σ(z))/τ on the edge, 0 in the core (dsalt_triton_train.py:371)
__device__ __forceinline__ float edge_dbias(const RowWindow& r, float d, float inv_tau) {
  if (d <= r.core) return 0.0f;
  float z = (r.wt - d) * inv_tau;
  float sig = 1.0f / (1.0f + expf(-z));
  return (1.0f - sig) * inv_tau;
}

}  // namespace dsalt
