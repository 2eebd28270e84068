// RMSNorm of the model blocks (reference dsalt/kernels/RMSENorm.py, F.rms_norm
// in fp32 under autocast) as one forward and one backward kernel:
//   y = round(x·r·w),  r = 1/sqrt(mean(x²) + eps)   (x·r and ·w rounded to fp32
//   separately, the result once to the input dtype),
//   dx = r·(g − x·r²·mean(g·x)),  g = dy·w,  dw = Σ_t dy·x·r.
// Optionally with the residual add before it (the block's x + attn(x)): the
// forward normalises x_sum = round(x + res) and writes x_sum, the backward adds
// the gradient reaching x_sum from elsewhere (dres): dx = round(round(dx) + dres),
// as torch's two ops and autograd's sum round them.
// One warp per token row (d = 256, 512, 768 or 1024), d/32 elements per lane in
// 16-byte pieces; the weight row is read as float4s.  dw: each CTA sums its 64
// rows in a fixed order into one fp32 partial row, and a second kernel adds the
// partials column by column in a fixed order (deterministic).
#include "common.cuh"

namespace dsalt {
namespace {

constexpr int kWarps = 8, kRowsPerWarp = 8, kRowsPerCta = kWarps * kRowsPerWarp;
static_assert(kRowsPerCta == DSALT_RMSNORM_ROWS_PER_PART, "dw partial rows");

template <typename T, int V>  // V = elements per lane = d / 32
__device__ __forceinline__ void load_row(const T* src, int lane, float* x) {
#pragma unroll
  for (int c = 0; c < V / 8; ++c) {
    if constexpr (sizeof(T) == 2) {
      const uint4 u = __ldg(reinterpret_cast<const uint4*>(src) + c * 32 + lane);
      const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) x[8 * c + i] = to_f32<T>(e[i]);
    } else {
      const float4 a = __ldg(reinterpret_cast<const float4*>(src) + (c * 32 + lane) * 2);
      const float4 b = __ldg(reinterpret_cast<const float4*>(src) + (c * 32 + lane) * 2 + 1);
      x[8 * c + 0] = a.x; x[8 * c + 1] = a.y; x[8 * c + 2] = a.z; x[8 * c + 3] = a.w;
      x[8 * c + 4] = b.x; x[8 * c + 5] = b.y; x[8 * c + 6] = b.z; x[8 * c + 7] = b.w;
    }
  }
}

template <typename T, int V>
__device__ __forceinline__ void store_row(T* dst, int lane, const float* y) {
#pragma unroll
  for (int c = 0; c < V / 8; ++c) {
    if constexpr (sizeof(T) == 2) {
      uint4 u;
      T* e = reinterpret_cast<T*>(&u);
#pragma unroll
      for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(y[8 * c + i]);
      reinterpret_cast<uint4*>(dst)[c * 32 + lane] = u;
    } else {
      reinterpret_cast<float4*>(dst)[(c * 32 + lane) * 2] = make_float4(y[8 * c], y[8 * c + 1], y[8 * c + 2], y[8 * c + 3]);
      reinterpret_cast<float4*>(dst)[(c * 32 + lane) * 2 + 1] =
          make_float4(y[8 * c + 4], y[8 * c + 5], y[8 * c + 6], y[8 * c + 7]);
    }
  }
}

// element j of a lane's registers is column (j / 8)·256 + 8·lane + j % 8
__device__ __forceinline__ int col_of(int j, int lane) { return (j >> 3) * 256 + 8 * lane + (j & 7); }

template <int V>
__device__ __forceinline__ void load_w(const float* w, int lane, float* wv) {
#pragma unroll
  for (int c = 0; c < V / 8; ++c) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(w) + c * 64 + 2 * lane);
    const float4 b = __ldg(reinterpret_cast<const float4*>(w) + c * 64 + 2 * lane + 1);
    wv[8 * c + 0] = a.x; wv[8 * c + 1] = a.y; wv[8 * c + 2] = a.z; wv[8 * c + 3] = a.w;
    wv[8 * c + 4] = b.x; wv[8 * c + 5] = b.y; wv[8 * c + 6] = b.z; wv[8 * c + 7] = b.w;
  }
}

template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32) rmsnorm_fwd_kernel(const DsaltRmsNormParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (row >= p.T) return;
  float x[V];
  load_row<T, V>(reinterpret_cast<const T*>(p.x) + row * p.d, lane, x);
  if (p.res) {
    float r[V];
    load_row<T, V>(reinterpret_cast<const T*>(p.res) + row * p.d, lane, r);
#pragma unroll
    for (int j = 0; j < V; ++j) x[j] = round_to<T>(__fadd_rn(x[j], r[j]));
    store_row<T, V>(reinterpret_cast<T*>(p.x_sum) + row * p.d, lane, x);
  }
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < V; ++j) ss = fmaf(x[j], x[j], ss);
  ss = warp_sum(ss);
  const float r = rsqrtf(__fadd_rn(__fdiv_rn(ss, (float)p.d), p.eps));
  if (lane == 0 && p.rstd) p.rstd[row] = r;
  float w[V];
  load_w<V>(p.w, lane, w);
#pragma unroll
  for (int j = 0; j < V; ++j) x[j] = __fmul_rn(__fmul_rn(x[j], r), w[j]);
  store_row<T, V>(reinterpret_cast<T*>(p.y) + row * p.d, lane, x);
}

// Backward: one warp per row, kRowsPerWarp rows per warp in turn, the weight row
// and the dw accumulators in registers (two CTAs per SM).
template <typename T, int V>
__global__ void __launch_bounds__(kWarps * 32, 2) rmsnorm_bwd_kernel(const DsaltRmsNormParams p) {
  __shared__ float part[kWarps][V * 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float w[V], dw[V];
  load_w<V>(p.w, lane, w);
#pragma unroll
  for (int j = 0; j < V; ++j) dw[j] = 0.f;
  for (int k = 0; k < kRowsPerWarp; ++k) {
    const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + warp * kRowsPerWarp + k;
    if (row >= p.T) break;
    float x[V], g[V];
    load_row<T, V>(reinterpret_cast<const T*>(p.x) + row * p.d, lane, x);
    load_row<T, V>(reinterpret_cast<const T*>(p.dy) + row * p.d, lane, g);
    const float r = __ldg(p.rstd + row);
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < V; ++j) {
      const float xr = x[j] * r;
      dw[j] = fmaf(g[j], xr, dw[j]);
      g[j] *= w[j];
      dot = fmaf(g[j], x[j], dot);
    }
    dot = warp_sum(dot);
    const float c = r * r * dot / (float)p.d;
#pragma unroll
    for (int j = 0; j < V; ++j) g[j] = r * fmaf(-x[j], c, g[j]);
    if (p.dres) {
      load_row<T, V>(reinterpret_cast<const T*>(p.dres) + row * p.d, lane, x);
#pragma unroll
      for (int j = 0; j < V; ++j) g[j] = __fadd_rn(round_to<T>(g[j]), x[j]);
    }
    store_row<T, V>(reinterpret_cast<T*>(p.dx) + row * p.d, lane, g);
  }
  // the CTA's partial of dw: warps added in order
#pragma unroll
  for (int j = 0; j < V; ++j) part[warp][col_of(j, lane)] = dw[j];
  __syncthreads();
  for (int cidx = threadIdx.x; cidx < p.d; cidx += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w8 = 0; w8 < kWarps; ++w8) s += part[w8][cidx];
    p.dw_part[(int64_t)blockIdx.x * p.d + cidx] = s;
  }
}

// dw[c] = Σ_i part[i][c] over the partial rows in a fixed order: a CTA owns 32
// columns; warp g sums rows g, g + 32, …, then the 32 warp sums are added in order.
constexpr int kColsumWarps = 32;

__global__ void __launch_bounds__(kColsumWarps * 32) colsum_kernel(const float* __restrict__ part, int nparts, int d,
                                                                   float* __restrict__ out) {
  __shared__ float s[kColsumWarps][33];
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + lane;
  float acc = 0.f;
  if (col < d) {
#pragma unroll 8
    for (int i = grp; i < nparts; i += kColsumWarps) acc += __ldg(part + (int64_t)i * d + col);
  }
  s[grp][lane] = acc;
  __syncthreads();
  if (grp == 0 && col < d) {
    float t = 0.f;
#pragma unroll
    for (int g = 0; g < kColsumWarps; ++g) t += s[g][lane];
    out[col] = t;
  }
}

template <typename T, int V>
cudaError_t launch_v(const DsaltRmsNormParams& p, bool bwd, cudaStream_t st) {
  if (bwd) {
    const unsigned grid = (unsigned)((p.T + kRowsPerCta - 1) / kRowsPerCta);
    rmsnorm_bwd_kernel<T, V><<<grid, kWarps * 32, 0, st>>>(p);
    if (p.dw) colsum_kernel<<<(unsigned)((p.d + 31) / 32), kColsumWarps * 32, 0, st>>>(p.dw_part, (int)grid, p.d, p.dw);
  } else {
    const unsigned grid = (unsigned)((p.T + kWarps - 1) / kWarps);
    rmsnorm_fwd_kernel<T, V><<<grid, kWarps * 32, 0, st>>>(p);
  }
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_t(const DsaltRmsNormParams& p, bool bwd, cudaStream_t st) {
  switch (p.d) {
    case 256: return launch_v<T, 8>(p, bwd, st);
    case 512: return launch_v<T, 16>(p, bwd, st);
    case 768: return launch_v<T, 24>(p, bwd, st);
    case 1024: return launch_v<T, 32>(p, bwd, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

bool rmsnorm_supported(int d) { return d == 256 || d == 512 || d == 768 || d == 1024; }


cudaError_t launch_rmsnorm(const DsaltRmsNormParams& p, bool bwd, cudaStream_t st) {
  switch (p.dtype) {
    case DSALT_BF16: return launch_t<__nv_bfloat16>(p, bwd, st);
    case DSALT_F16: return launch_t<__half>(p, bwd, st);
    case DSALT_F32: return launch_t<float>(p, bwd, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace dsalt
