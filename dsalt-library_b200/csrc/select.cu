// Selection and gating kernels: window gate, hybrid landmark score, top-k.
//
// These replace the torch code of the reference's selectors:
//   win_gate        DSALTAttention._window_continuous   (dsalt/modules/dsalt_attention.py:270-284)
//   hybrid scores   hybrid_scores_per_head              (dsalt/kernels/landmark_tokens_ker.py:19-61)
//   top-k           _compute_landmark_indices           (dsalt/kernels/selectors.py:75-134)
// All three are HBM/latency-bound byte work: coalesced 16-byte loads, one warp
// per token for the row reductions, shared-memory radix select for top-k.
#include <mutex>

#include "common.cuh"

namespace dsalt {

// ------------------------------------------------------------------ win_gate
// logit = x·W + b accumulated in fp32; under autocast (dtype f16/bf16) torch
// rounds the Linear output, the sigmoid, the product with (n_max - n_min) and
// the sum with n_min to the dtype, each once; fp32 rounds each op to fp32.
template <typename T>
__global__ void __launch_bounds__(256) win_gate_kernel(DsaltWinGateParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const T* x = reinterpret_cast<const T*>(p.x) + t * p.d_model;
  const T* w = reinterpret_cast<const T*>(p.weight);
  float acc = 0.f;
  if (sizeof(T) == 2 && p.d_model % 8 == 0 && ((uintptr_t)p.x & 15u) == 0 && ((uintptr_t)p.weight & 15u) == 0) {
    // 16-byte pieces (uniform over the launch)
    for (int j = lane; j < p.d_model / 8; j += 32) {
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x) + j);
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + j);
      const T* xe = reinterpret_cast<const T*>(&xv);
      const T* we = reinterpret_cast<const T*>(&wv);
#pragma unroll
      for (int k = 0; k < 8; ++k) acc = fmaf(to_f32<T>(xe[k]), to_f32<T>(we[k]), acc);
    }
  } else {
    for (int d = lane; d < p.d_model; d += 32) acc = fmaf(to_f32<T>(x[d]), to_f32<T>(w[d]), acc);
  }
  acc = warp_sum(acc);
  if (lane != 0) return;
  const float b = to_f32<T>(reinterpret_cast<const T*>(p.bias)[0]);
  const float logit = __fadd_rn(acc, b);
  const float span = p.n_max - p.n_min;
  float wv;
  if (sizeof(T) == 4) {
    const float sg = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-logit)));
    wv = __fadd_rn(p.n_min, __fmul_rn(sg, span));
  } else {
    const float lg = round_to<T>(logit);
    const float sg = round_to<T>(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-lg))));
    const float pr = round_to<T>(__fmul_rn(sg, span));
    wv = round_to<T>(__fadd_rn(p.n_min, pr));
  }
  reinterpret_cast<T*>(p.w_cont)[t] = from_f32<T>(wv);
  if (p.w_f32) p.w_f32[t] = wv;
  if (p.w_disc) p.w_disc[t] = fmaxf(floorf(wv), 1.0f);
  if (p.logits) p.logits[t] = logit;
}

cudaError_t launch_win_gate(const DsaltWinGateParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((p.T + 7) / 8);
  switch (p.dtype) {
    case DSALT_F16: win_gate_kernel<__half><<<grid, 256, 0, st>>>(p); break;
    case DSALT_BF16: win_gate_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p); break;
    case DSALT_F32: win_gate_kernel<float><<<grid, 256, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// Backward of the window gate's Linear (a rank-one product): dx[t, j] =
// R(dl[t]·w[j]) (the fp32 product rounded once to the dtype) and the weight
// gradient Σ_t dl[t]·x[t, j] as fp32 partials of DSALT_WIN_GATE_ROWS_PER_PART
// rows each, accumulated in row order; the caller adds the partials.  A thread
// owns 8 adjacent columns (16-byte pieces).
constexpr int kWgRows = DSALT_WIN_GATE_ROWS_PER_PART;

template <typename T>
__global__ void __launch_bounds__(128) win_gate_bwd_kernel(const DsaltWinGateBwdParams p) {
  const int64_t r0 = (int64_t)blockIdx.x * kWgRows;
  const int nrow = (int)(p.T - r0 < kWgRows ? p.T - r0 : kWgRows);
  const int pieces = p.d_model / 8;
  for (int c = threadIdx.x; c < pieces; c += blockDim.x) {
    float wv[8], acc[8];
    {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(p.weight) + c);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < 8; ++k) { wv[k] = to_f32<T>(e[k]); acc[k] = 0.f; }
    }
#pragma unroll 4
    for (int r = 0; r < nrow; ++r) {
      const int64_t t = r0 + r;
      const float dl = __ldg(p.dl + t);
      if (p.dw_part) {
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.x) + t * p.d_model) + c);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int k = 0; k < 8; ++k) acc[k] = fmaf(dl, to_f32<T>(e[k]), acc[k]);
      }
      if (p.dx) {
        uint4 o;
        T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
        for (int k = 0; k < 8; ++k) oe[k] = from_f32<T>(__fmul_rn(dl, wv[k]));
        reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.dx) + t * p.d_model)[c] = o;
      }
    }
    if (p.dw_part) {
      float4* dst = reinterpret_cast<float4*>(p.dw_part + (int64_t)blockIdx.x * p.d_model + 8 * c);
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

cudaError_t launch_win_gate_bwd(const DsaltWinGateBwdParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((p.T + kWgRows - 1) / kWgRows);
  switch (p.dtype) {
    case DSALT_F16: win_gate_bwd_kernel<__half><<<grid, 128, 0, st>>>(p); break;
    case DSALT_BF16: win_gate_bwd_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// ------------------------------------------------------------- hybrid score
// Pass 1: per token ‖x‖ and per kv-head ‖x W_Vᵀ‖, rounded to the dtype as
// torch's norm on a dtype tensor is, then widened (landmark_tokens_ker.py:47,52).
// The norms are stored column-major, [1 + n_kv][T], so that the statistics of a
// column read contiguous memory.
template <typename T>
__global__ void __launch_bounds__(256) score_norms_kernel(DsaltScoreParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const T* x = reinterpret_cast<const T*>(p.x) + t * p.d_model;
  float a = 0.f;
  for (int d = lane; d < p.d_model; d += 32) { const float v = to_f32<T>(x[d]); a = fmaf(v, v, a); }
  a = warp_sum(a);
  if (lane == 0) p.norms[t] = round_to<T>(sqrtf(a));
  const T* xv = reinterpret_cast<const T*>(p.xwv) + t * (int64_t)p.n_kv * p.dh;
  for (int g = 0; g < p.n_kv; ++g) {
    float b = 0.f;
    for (int d = lane; d < p.dh; d += 32) { const float v = to_f32<T>(xv[g * p.dh + d]); b = fmaf(v, v, b); }
    b = warp_sum(b);
    if (lane == 0) p.norms[(1 + g) * p.T + t] = round_to<T>(sqrtf(b));
  }
}

template <typename T>
__device__ __forceinline__ float sumsq8(const uint4 u) {
  const T* e = reinterpret_cast<const T*>(&u);
  float a = 0.f;
#pragma unroll
  for (int k = 0; k < 8; ++k) { const float v = to_f32<T>(e[k]); a = fmaf(v, v, a); }
  return a;
}

// Pass 1 for 16-bit rows in 16-byte pieces (d_model and dh multiples of 8, dh / 8
// a power of two up to 32): a value head spans dh / 8 adjacent lanes, reduced by
// an xor-shuffle tree inside the lane group.
template <typename T>
__global__ void __launch_bounds__(256) score_norms_vec_kernel(DsaltScoreParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= p.T) return;  // warp-uniform
  const uint4* x = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.x) + t * p.d_model);
  float a = 0.f;
  for (int j = lane; j < p.d_model / 8; j += 32) a += sumsq8<T>(__ldg(x + j));
  a = warp_sum(a);
  if (lane == 0) p.norms[t] = round_to<T>(sqrtf(a));
  const int hv = p.dh / 8, nv = p.n_kv * hv;
  const uint4* xv = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.xwv) + t * (int64_t)p.n_kv * p.dh);
  for (int j0 = 0; j0 < nv; j0 += 32) {
    const int j = j0 + lane;
    float b = j < nv ? sumsq8<T>(__ldg(xv + j)) : 0.f;
    for (int off = hv / 2; off > 0; off >>= 1) b += __shfl_xor_sync(0xffffffffu, b, off);
    if (j < nv && (lane & (hv - 1)) == 0) p.norms[(int64_t)(1 + j / hv) * p.T + t] = round_to<T>(sqrtf(b));
  }
}

static bool score_norms_vectorizable(const DsaltScoreParams& p) {
  const int hv = p.dh / 8;
  return p.dtype != DSALT_F32 && p.d_model % 8 == 0 && p.dh % 8 == 0 && hv >= 1 && hv <= 32 &&
         (hv & (hv - 1)) == 0 && ((uintptr_t)p.x & 15u) == 0 && ((uintptr_t)p.xwv & 15u) == 0;
}

// Pass 2 (one CTA per norm column): mean and unbiased std of the column over
// all T packed tokens, accumulated in fp64 (landmark_tokens_ker.py:48, 53-54):
// thread i sums tokens i, i + 1024, … of the (contiguous) column, then a fixed
// shuffle tree and a fixed sum over the warps: one sweep for the mean, one for
// the centred squares.
__global__ void __launch_bounds__(1024) score_stats_kernel(DsaltScoreParams p) {
  __shared__ double red[32];
  {
    const int c = blockIdx.x;
    const float* col = p.norms + (int64_t)c * p.T;
    double acc = 0.0;
    for (int64_t t = threadIdx.x; t < p.T; t += blockDim.x) acc += col[t];
    acc = warp_sum_d(acc);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < 32; ++w) tot += red[w];
    __syncthreads();
    const double mean = tot / (double)p.T;
    double sq = 0.0;
    for (int64_t t = threadIdx.x; t < p.T; t += blockDim.x) {
      const double d = col[t] - mean;
      sq += d * d;
    }
    sq = warp_sum_d(sq);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = sq;
    __syncthreads();
    double sqt = 0.0;
    for (int w = 0; w < 32; ++w) sqt += red[w];
    __syncthreads();
    if (threadIdx.x == 0) {
      const float mu = (float)mean;
      const float sd = p.T > 1 ? (float)sqrt(sqt / (double)(p.T - 1)) : NAN;
      p.stats[2 * c] = mu;
      // clamp(min=1e-6) keeps a NaN (torch.clamp propagates it): one token gives NaN z-scores
      p.stats[2 * c + 1] = p.T > 1 ? fmaxf(sd, 1e-6f) : NAN;
    }
  }
}

// Pass 3: z-scores and the per-head mix s = α·z_v + (1−α)·z_x (:49,55,60),
// each op rounded to fp32 like the eager torch expression.
__global__ void score_mix_kernel(DsaltScoreParams p) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= p.T * p.H) return;
  const int64_t t = e / p.H;
  const int h = (int)(e % p.H);
  const int g = h / (p.H / p.n_kv);
  const float zx = __fdiv_rn(__fsub_rn(p.norms[t], p.stats[0]), p.stats[1]);
  const float zv = __fdiv_rn(__fsub_rn(p.norms[(1 + g) * p.T + t], p.stats[2 + 2 * g]), p.stats[3 + 2 * g]);
  const float a = p.alpha[h];
  p.scores[e] = __fadd_rn(__fmul_rn(a, zv), __fmul_rn(__fsub_rn(1.0f, a), zx));
  if (p.z_v) p.z_v[e] = zv;
  if (h == 0 && p.z_x) p.z_x[t] = zx;
}

cudaError_t launch_hybrid_scores(const DsaltScoreParams& p, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  const unsigned g1 = (unsigned)((p.T + 7) / 8);
  const bool vec = score_norms_vectorizable(p);
  switch (p.dtype) {
    case DSALT_F16:
      if (vec) score_norms_vec_kernel<__half><<<g1, 256, 0, st>>>(p);
      else score_norms_kernel<__half><<<g1, 256, 0, st>>>(p);
      break;
    case DSALT_BF16:
      if (vec) score_norms_vec_kernel<__nv_bfloat16><<<g1, 256, 0, st>>>(p);
      else score_norms_kernel<__nv_bfloat16><<<g1, 256, 0, st>>>(p);
      break;
    case DSALT_F32: score_norms_kernel<float><<<g1, 256, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  score_stats_kernel<<<(unsigned)(1 + p.n_kv), 1024, 0, st>>>(p);
  score_mix_kernel<<<(unsigned)((p.T * p.H + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError();
}

// --------------------------------------------------------- hybrid score backward
// The gradient of s = α·z_v + (1−α)·z_x through the z-scores to the norms, as the
// reference's autograd computes it: per token t and norm column c (c = 0: ‖x‖,
// c = 1 + g: value head group g)
//   dz[t,0] = Σ_h g[t,h]·(1 − α_h),  dz[t,1+g] = Σ_{h ∈ g} g[t,h]·α_h,
//   dn[t,c] = (dz[t,c] − mean_t dz[·,c]) / sd_c
//             − [sd_c unclamped]·z[t,c]·Σ_t dz[·,c]·z[·,c] / ((T − 1)·sd_c),
//   coef[t,c] = dn[t,c] / ‖·‖[t,c] (1 where the norm is 0),
// and d α_h = Σ_t g[t,h]·(z_v[t,h] − z_x[t]).  Pass 1: the column sums (Σ dz,
// Σ dz·z per column, d α per head) as per-128-token partials and a block-order
// total (fixed-order reductions); pass 2: one thread per token writes its
// coefficients.
__device__ __forceinline__ float score_dz(const DsaltScoreBwdParams& p, int64_t t, int c) {
  const float* g = p.g_s + t * p.H;
  const int rep = p.H / p.n_kv;
  float acc = 0.f;
  if (c == 0) {
    for (int h = 0; h < p.H; ++h) acc = fmaf(g[h], 1.0f - p.alpha[h], acc);
  } else {
    const int h0 = (c - 1) * rep;
    for (int r = 0; r < rep; ++r) acc = fmaf(g[h0 + r], p.alpha[h0 + r], acc);
  }
  return acc;
}

__device__ __forceinline__ float score_z(const DsaltScoreBwdParams& p, int64_t t, int c) {
  return c == 0 ? p.z_x[t] : p.z_v[t * p.H + (c - 1) * (p.H / p.n_kv)];
}

// Pass 1a: CTA b takes tokens [128·b, 128·b + 128): each thread writes its token's
// contributions to every sum (Σ dz, Σ dz·z per column, d α per head) into shared
// memory, then one thread per sum adds the 128 in token order.
constexpr int kSbTok = DSALT_SCORE_BWD_TOKENS;
__global__ void __launch_bounds__(kSbTok) score_bwd_partial_kernel(DsaltScoreBwdParams p) {
  extern __shared__ float contrib[];  // [kSbTok][jobs]
  const int ncol = 1 + p.n_kv, jobs = 2 * ncol + p.H;
  const int rep = p.H / p.n_kv;
  const int64_t t = (int64_t)blockIdx.x * kSbTok + threadIdx.x;
  float* row = contrib + threadIdx.x * jobs;
  if (t < p.T) {
    const float zx = p.z_x[t];
    for (int c = 0; c < ncol; ++c) {
      const float dz = score_dz(p, t, c);
      row[c] = dz;
      row[ncol + c] = dz * score_z(p, t, c);
    }
    for (int h = 0; h < p.H; ++h) row[2 * ncol + h] = p.g_s[t * p.H + h] * (p.z_v[t * p.H + h] - zx);
  } else {
    for (int j = 0; j < jobs; ++j) row[j] = 0.f;
  }
  (void)rep;
  __syncthreads();
  for (int j = threadIdx.x; j < jobs; j += kSbTok) {
    float acc = 0.f;
    for (int k = 0; k < kSbTok; ++k) acc += contrib[k * jobs + j];
    p.partials[(int64_t)blockIdx.x * jobs + j] = acc;
  }
}

// Pass 1b: one thread per sum adds the per-block partials in block order.
__global__ void __launch_bounds__(128) score_bwd_final_kernel(DsaltScoreBwdParams p, int nblk) {
  const int ncol = 1 + p.n_kv, jobs = 2 * ncol + p.H;
  const int j = blockIdx.x * blockDim.x + threadIdx.x;
  if (j >= jobs) return;
  float acc = 0.f;
  for (int b = 0; b < nblk; ++b) acc += p.partials[(int64_t)b * jobs + j];
  if (j < 2 * ncol) p.sums[j] = acc;
  else p.d_alpha[j - 2 * ncol] = acc;
}

__global__ void __launch_bounds__(256) score_bwd_coef_kernel(DsaltScoreBwdParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= p.T) return;
  const int ncol = 1 + p.n_kv;
  const float inv_t = 1.0f / (float)p.T;
  for (int c = 0; c < ncol; ++c) {
    const float sd = p.stats[2 * c + 1];
    const float dz = score_dz(p, t, c);
    float dn = (dz - p.sums[c] * inv_t) / sd;
    if (p.T > 1 && sd > 1e-6f) dn -= score_z(p, t, c) * p.sums[ncol + c] / ((float)(p.T - 1) * sd);
    const float nrm = p.norms[(int64_t)c * p.T + t];
    const float coef = dn / (nrm > 0.f ? nrm : 1.0f);
    if (c == 0) p.coef_x[t] = coef;
    else p.coef_v[t * p.n_kv + (c - 1)] = coef;
  }
}

cudaError_t launch_hybrid_scores_bwd(const DsaltScoreBwdParams& p, cudaStream_t st) {
  const int jobs = 2 * (1 + p.n_kv) + p.H;
  const int nblk = (int)((p.T + kSbTok - 1) / kSbTok);
  if (nblk > 0) {
    const size_t smem = sizeof(float) * (size_t)kSbTok * jobs;
    cudaError_t e = ensure_smem((const void*)score_bwd_partial_kernel, smem);
    if (e != cudaSuccess) return e;
    score_bwd_partial_kernel<<<(unsigned)nblk, kSbTok, smem, st>>>(p);
  }
  score_bwd_final_kernel<<<(unsigned)((jobs + 127) / 128), 128, 0, st>>>(p, nblk);
  if (p.T > 0) score_bwd_coef_kernel<<<(unsigned)((p.T + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError();
}

// Backward of the norms (landmark_tokens_ker.py:47,52 through the z-scores):
// out[t, g·width + j] = round(coef[t·groups + g] · x[t, g·width + j]), the fp32
// product rounded once to the dtype, as (coef · x.float()).to(dtype) computes it.
template <typename T>
__global__ void __launch_bounds__(256) scale_rows_kernel(DsaltScaleRowsParams p) {
  const int64_t n8 = p.T * p.groups * (p.width / 8);
  const int64_t i = (int64_t)blockIdx.x * 256 + threadIdx.x;
  if (i >= n8) return;
  const int64_t tg = i / (p.width / 8);  // t·groups + g
  const float c = __ldg(p.coef + tg);
  if constexpr (sizeof(T) == 2) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p.x) + i);
    const T* e = reinterpret_cast<const T*>(&u);
    uint4 o;
    T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < 8; ++k) oe[k] = from_f32<T>(__fmul_rn(c, to_f32<T>(e[k])));
    reinterpret_cast<uint4*>(p.out)[i] = o;
  } else {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float4 v = __ldg(reinterpret_cast<const float4*>(p.x) + 2 * i + h);
      v.x = __fmul_rn(c, v.x); v.y = __fmul_rn(c, v.y); v.z = __fmul_rn(c, v.z); v.w = __fmul_rn(c, v.w);
      reinterpret_cast<float4*>(p.out)[2 * i + h] = v;
    }
  }
}

cudaError_t launch_scale_rows(const DsaltScaleRowsParams& p, cudaStream_t st) {
  const int64_t n8 = p.T * p.groups * (p.width / 8);
  if (n8 == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n8 + 255) / 256);
  switch (p.dtype) {
    case DSALT_F16: scale_rows_kernel<__half><<<grid, 256, 0, st>>>(p); break;
    case DSALT_BF16: scale_rows_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p); break;
    case DSALT_F32: scale_rows_kernel<float><<<grid, 256, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

// -------------------------------------------------------------------- top-k
// Orderable key: larger float -> larger unsigned; excluded / -inf -> 0.  torch.topk
// ranks NaN above +inf above every finite score, and the reference then turns the
// non-finite winners into -1 slots (selectors.py:117-133): NaN maps to the largest
// key, +inf to the next one, and both are written out as -1.
constexpr uint32_t kKeyPosInf = 0xFF800000u;
__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xFFFFFFFFu;
  if (f == -INFINITY) return 0u;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxLen = 49152;  // keys held in shared memory
constexpr int kTopkMaxK = 1024;

// Warp-collective: add one count per active key to hist[bin], one shared-memory
// atomic per distinct bin of the warp (keys of a radix round crowd into few bins).
__device__ __forceinline__ void hist_add(uint32_t* hist, bool in, uint32_t bin) {
  const uint32_t act = __ballot_sync(0xffffffffu, in);
  if (in) {
    const uint32_t peers = __match_any_sync(act, bin);
    if ((int)(threadIdx.x & 31) == __ffs(peers) - 1) atomicAdd(&hist[bin], (uint32_t)__popc(peers));
  }
}

// One CTA per (head, sequence): 4 rounds of 8-bit radix select find the k-th
// largest key; the keys above it and the lowest-position ties fill the k slots.
__global__ void __launch_bounds__(kTopkThreads) topk_kernel(DsaltTopkParams p) {
  extern __shared__ uint32_t sm[];
  uint32_t* keys = sm;                       // [max_len]
  __shared__ uint32_t hist[256];
  __shared__ uint32_t sel_prefix, sel_mask;
  __shared__ int need, n_above, n_ties, n_tie_taken;
  __shared__ uint32_t out_key[kTopkMaxK];
  __shared__ int out_pos[kTopkMaxK];

  const int h = blockIdx.x / p.S;
  const int s = blockIdx.x % p.S;
  const int64_t s0 = p.cu_seqlens[s];
  const int L = min((int)(p.cu_seqlens[s + 1] - s0), p.max_len);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int i = tid; i < L; i += kTopkThreads) {
    const float ws = p.w_sizes[s0 + i];
    // covered = seq_off < w_sizes.long()  (selectors.py:105) -> excluded
    const bool covered = (float)i < truncf(ws);
    keys[i] = covered ? 0u : order_key(p.scores[(s0 + i) * p.H + h]);
  }
  if (tid == 0) { sel_prefix = 0; sel_mask = 0; need = p.k; n_above = 0; n_ties = 0; n_tie_taken = 0; }
  __syncthreads();

  const int k_eff = min(p.k, L);
  if (k_eff > 0) {
    for (int shift = 24; shift >= 0; shift -= 8) {
      for (int b = tid; b < 256; b += kTopkThreads) hist[b] = 0;
      __syncthreads();
      const uint32_t pre = sel_prefix, msk = sel_mask;
      for (int i0 = tid & ~31; i0 < L; i0 += kTopkThreads) {  // warp-uniform trip count
        const int i = i0 + lane;
        const uint32_t kk = i < L ? keys[i] : 0u;
        hist_add(hist, i < L && (kk & msk) == pre, (kk >> shift) & 255u);
      }
      __syncthreads();
      if (warp == 0) {
        // the bin holding the rem-th largest key: lane l owns bins 255 − 8l … 248 − 8l
        const int rem0 = (shift == 24) ? k_eff : need;
        uint32_t c[8];
        uint32_t tot = 0;
#pragma unroll
        for (int q = 0; q < 8; ++q) { c[q] = hist[255 - 8 * lane - q]; tot += c[q]; }
        uint32_t incl = tot;  // inclusive scan from the top bins down
#pragma unroll
        for (int off = 1; off < 32; off <<= 1) {
          const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
          if (lane >= off) incl += y;
        }
        const uint32_t excl = incl - tot;
        // the first lane whose cumulative count reaches rem0 (the last lane if none does)
        const uint32_t hit = __ballot_sync(0xffffffffu, incl >= (uint32_t)rem0);
        const int owner = hit ? __ffs(hit) - 1 : 31;
        if (lane == owner) {
          int rem = rem0 - (int)excl;
          int b = 255 - 8 * lane;
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            if (b == 0 || (int)c[q] >= rem) break;
            rem -= (int)c[q];
            --b;
          }
          sel_prefix = pre | ((uint32_t)b << shift);
          sel_mask = msk | (255u << shift);
          need = rem;  // how many keys equal to the final threshold are still needed
        }
      }
      __syncthreads();
    }
  }
  // threshold = sel_prefix (the k-th largest key); take all above, then `need` ties by position
  const uint32_t thr = sel_prefix;
  if (k_eff > 0) {
    for (int i0 = tid & ~31; i0 < L; i0 += kTopkThreads) {
      const int i = i0 + lane;
      const uint32_t kk = i < L ? keys[i] : 0u;
      const bool above = i < L && kk > thr, tie = i < L && kk == thr;
      const uint32_t ba = __ballot_sync(0xffffffffu, above), bt = __ballot_sync(0xffffffffu, tie);
      int base_a = 0;
      if (lane == 0 && ba) base_a = atomicAdd(&n_above, __popc(ba));
      if (lane == 0 && bt) atomicAdd(&n_ties, __popc(bt));
      base_a = __shfl_sync(0xffffffffu, base_a, 0);
      if (above) {
        const int slot = base_a + __popc(ba & ((1u << lane) - 1u));
        if (slot < kTopkMaxK) { out_key[slot] = kk; out_pos[slot] = i; }
      }
    }
    __syncthreads();
    if (n_ties == need) {
      // every key equal to the threshold is taken (the usual case): any order
      for (int i0 = tid & ~31; i0 < L; i0 += kTopkThreads) {
        const int i = i0 + lane;
        const bool tie = i < L && keys[i] == thr;
        const uint32_t bt = __ballot_sync(0xffffffffu, tie);
        int base_t = 0;
        if (lane == 0 && bt) base_t = atomicAdd(&n_tie_taken, __popc(bt));
        base_t = __shfl_sync(0xffffffffu, base_t, 0);
        if (tie) {
          const int slot = n_above + base_t + __popc(bt & ((1u << lane) - 1u));
          if (slot < kTopkMaxK) { out_key[slot] = thr; out_pos[slot] = i; }
        }
      }
    } else if (tid < 32) {
      // more ties than slots: the lowest positions, a single warp scanning with ballots
      int taken = 0;
      const int base = n_above;
      for (int i0 = 0; i0 < L && taken < need; i0 += 32) {
        const int i = i0 + tid;
        const bool tie = i < L && keys[i] == thr;
        const uint32_t bal = __ballot_sync(0xffffffffu, tie);
        const int before = __popc(bal & ((1u << tid) - 1u));
        if (tie && taken + before < need) {
          const int slot = base + taken + before;
          if (slot < kTopkMaxK) { out_key[slot] = thr; out_pos[slot] = i; }
        }
        taken += __popc(bal);
      }
      if (tid == 0) n_tie_taken = min(taken, need);
    }
  }
  __syncthreads();
  const int n_sel = k_eff > 0 ? min(n_above + n_tie_taken, k_eff) : 0;
  // order the selection: key descending, position ascending
  int64_t* out = p.idx + ((int64_t)h * p.S + s) * p.k;
  for (int r = tid; r < p.k; r += kTopkThreads) out[r] = -1;
  __syncthreads();
  for (int a = tid; a < n_sel; a += kTopkThreads) {
    const uint32_t ka = out_key[a];
    const int pa = out_pos[a];
    int rank = 0;
    for (int b = 0; b < n_sel; ++b) {
      const uint32_t kb = out_key[b];
      rank += (kb > ka) || (kb == ka && out_pos[b] < pa);
    }
    out[rank] = (ka == 0u || ka >= kKeyPosInf) ? -1 : (int64_t)pa;  // non-finite: -1 (selectors.py:131-132)
  }
}

cudaError_t launch_topk(const DsaltTopkParams& p, cudaStream_t st) {
  if (p.H * p.S == 0) return cudaSuccess;
  if (p.max_len > kTopkMaxLen || p.k > kTopkMaxK) return cudaErrorInvalidValue;  // checked by the entry point
  const size_t smem = sizeof(uint32_t) * (size_t)max(p.max_len, 1);
  cudaError_t e = ensure_smem((const void*)topk_kernel, smem);
  if (e != cudaSuccess) return e;
  topk_kernel<<<p.H * p.S, kTopkThreads, smem, st>>>(p);
  return cudaGetLastError();
}

// ------------------------------------------------ no-allocation score variant
// dsalt_hybrid_scores_noalloc runs the same three kernels as
// dsalt_hybrid_scores, but keeps their scratch (the per-token norms and the
// mean/std statistics) in the fixed array below instead of in buffers the
// caller allocates.  It is meant for callers that are not allowed to allocate
// device memory themselves: for example a host application that plans and
// owns every device buffer and gives plugins only their inputs and outputs.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds DSALT_NOALLOC_SCORE_MAX_FLOATS floats (8 MiB) of it until the
// process exits.  All calls on a device share it and it keeps the previous
// call's contents; the kernels overwrite every element they read, so nothing
// has to be cleared between calls.  Two calls that overlap on the GPU (on
// different streams, or from different host threads) race on the array.
static __device__ __align__(256) float g_score_scratch[DSALT_NOALLOC_SCORE_MAX_FLOATS];

// Device address of g_score_scratch on the current device.  In host code the
// symbol names a host-side stand-in, never the device array, so the address is
// fetched with cudaGetSymbolAddress once per device (with that device
// current) and cached.
cudaError_t noalloc_score_scratch(float** out) {
  constexpr int kMaxDevices = 64;
  static float* cache[kMaxDevices] = {};
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_score_scratch);
    if (e != cudaSuccess) return e;
    cache[dev] = static_cast<float*>(ptr);
  }
  *out = cache[dev];
  return cudaSuccess;
}

}  // namespace dsalt
