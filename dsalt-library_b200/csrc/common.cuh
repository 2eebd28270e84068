// Shared device helpers for the DSALT B200 kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <math.h>
#include <climits>
#include <mutex>

#include "dsalt_b200.h"

namespace dsalt {

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) once per (kernel, device,
// size): the attribute persists, so repeated launches skip the driver call.
inline cudaError_t ensure_smem(const void* kernel, size_t bytes) {
  struct Entry { const void* k; int dev; size_t bytes; };
  static Entry done[256];
  static int n_done = 0;
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_done; ++i)
    if (done[i].k == kernel && done[i].dev == dev && done[i].bytes >= bytes) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e == cudaSuccess && n_done < 256) done[n_done++] = Entry{kernel, dev, bytes};
  return e;
}

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

// Grouped kv heads: the kv heads of k and v (0 in the params means H) and the kv
// head that query head h reads.
__host__ __device__ __forceinline__ int attn_kv_heads(const DsaltAttnParams& p) { return p.H_kv > 0 ? p.H_kv : p.H; }
__host__ __device__ __forceinline__ int attn_kv_head(const DsaltAttnParams& p, int h) {
  return h / (p.H / attn_kv_heads(p));
}

// ------------------------------------------------------ backward query records
// One record per (head, query token) of the backward, written by the preprocess
// stage next to Delta and read by the tensor-core dK/dV and dQ stages, so that
// the per-query window / soft-edge work is done once instead of once per tile.
constexpr int kQRecEdge = 8;  // soft-edge factors stored per record
struct alignas(16) QRec {
  float nlse2;  // −LSE·log2(e) (0 for a row without keys)
  float delta;  // Δ = Σ_d O·dO
  int lo;       // first band key (INT_MAX: none)
  int qi;       // query position in its sequence (INT_MIN: row without keys)
  int ehi;      // last soft-edge key (INT_MIN: none)
  int elo;      // first soft-edge key (INT_MAX: none); the edge keys are elo … ehi
  float wlo;    // float(i) − w̃ (landmark rule)
  float wt;     // w̃
  float eg[kQRecEdge];  // σ((w̃ − d)/τ) of edge key ehi − e (d = i − ehi + e), e < kQRecEdge
};
static_assert(sizeof(QRec) == DSALT_QREC_FLOATS * 4, "record size");
__device__ __forceinline__ int qrec_ne(const QRec& r) { return r.elo <= r.ehi ? r.ehi - r.elo + 1 : 0; }

// Record fields of query token t (global index), head h, given its Δ; the
// soft-edge factors are left to qrec_edge_factor (d_e0: first edge distance).
__device__ __forceinline__ QRec qrec_fields(const DsaltAttnParams& p, int64_t t, int h, float delta, int* d_e0) {
  QRec rec;
  rec.nlse2 = 0.f; rec.delta = 0.f; rec.lo = INT_MAX; rec.qi = INT_MIN;
  rec.wlo = -INFINITY; rec.wt = 0.f; rec.ehi = INT_MIN; rec.elo = INT_MAX;
  *d_e0 = 0;
  const float lse = p.lse[t * p.H + h];
  if (lse != -INFINITY) {
    const int s = find_seq(p.cu_seqlens, p.S, t);
    const int i = (int)(t - __ldg(p.cu_seqlens + s));
    const RowWindow rw = row_window(__ldg(p.w + t), i, p.semantics, p.win_edge);
    rec.nlse2 = -lse * 1.4426950408889634f;
    rec.delta = delta;
    rec.qi = i;
    rec.wlo = rw.win_lo;
    rec.wt = rw.wt;
    if (rw.W >= 0) {
      rec.lo = i - min(rw.W, i);
      const int de = max((int)floorf(rw.core) + 1, 0);
      if (de <= rw.W) {
        rec.ehi = i - de;
        rec.elo = rec.lo;  // the edge runs down to the band start (d = min(W, i))
        *d_e0 = de;
      }
    }
  }
  return rec;
}
// σ((w̃ − d)/τ) of the soft-edge key at distance d
__device__ __forceinline__ float qrec_edge_factor(float wt, int d, float inv_tau) {
  return 1.0f / (1.0f + expf(-((wt - (float)d) * inv_tau)));
}
__device__ __forceinline__ float4* qrec_ptr(const DsaltAttnParams& p, int64_t t, int h) {
  return reinterpret_cast<float4*>(p.qrec + ((int64_t)h * p.T + t) * DSALT_QREC_FLOATS);
}

// The whole record of one (token, head) from one thread.
__device__ __forceinline__ void write_qrec(const DsaltAttnParams& p, int64_t t, int h, float delta) {
  int d_e0;
  QRec rec = qrec_fields(p, t, h, delta, &d_e0);
  const float inv_tau = 1.0f / p.tau_win;
  const int ne = qrec_ne(rec);
#pragma unroll
  for (int e = 0; e < kQRecEdge; ++e) rec.eg[e] = e < ne ? qrec_edge_factor(rec.wt, d_e0 + e, inv_tau) : 1.0f;
  float4* dst = qrec_ptr(p, t, h);
  const float4* src = reinterpret_cast<const float4*>(&rec);
#pragma unroll
  for (int k = 0; k < DSALT_QREC_FLOATS / 4; ++k) dst[k] = src[k];
}

// Bit c (0 ≤ c < 32) set iff lo ≤ c ≤ hi: a per-thread column mask, so that an
// unrolled loop tests one bit per element instead of two compares.
__device__ __forceinline__ uint32_t range_mask32(int lo, int hi) {
  lo = max(lo, 0);
  hi = min(hi, 31);
  if (lo > hi) return 0u;
  const uint32_t up = hi >= 31 ? 0xffffffffu : ((1u << (hi + 1)) - 1u);
  return up & ~((1u << lo) - 1u);
}

}  // namespace dsalt
