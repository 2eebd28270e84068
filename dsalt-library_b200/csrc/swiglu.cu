// SwiGLU activation of the feed-forward blocks (reference
// dsalt/modules/dsalt_transformer.py:10-21: down(silu(gate(x)) * up(x))) in one
// pass each way, with torch's rounding under autocast (16-bit tensors, fp32 math):
//   forward   s = R(g / (1 + exp(−g))),  h = R(s·u)
//   backward  ds = R(dh·u),  du = R(dh·s),
//             dg = R(ds·σ·(1 + g·(1 − σ))),  σ = 1 / (1 + exp(−g))
// where R rounds to the tensor dtype; s is recomputed in the backward (one exp
// serves s and σ).  g and u are read with a row stride, so they can be the two
// halves of one [T, 2F] GEMM output; dg and du are written the same way.  One
// warp per row, 8 elements per lane in 16-byte pieces.
#include "common.cuh"

namespace dsalt {
namespace {

constexpr int kThreads = 256, kRowsPerCta = kThreads / 32;

// 1 + exp(−g): the denominator of both silu(g) = g / den and σ(g) = 1 / den
__device__ __forceinline__ float silu_den(float g) { return __fadd_rn(1.f, expf(-g)); }

// One warp per token row; lane l takes the 8-element pieces l, l + 32, … of the row.
template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_fwd_kernel(const DsaltSwigluParams p) {
  const int64_t t = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const int lane = threadIdx.x & 31, pieces = (int)(p.F / 8);
  const uint4* gr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.g) + t * p.ld_in);
  const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.u) + t * p.ld_in);
  uint4* hr = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.h) + t * p.F);
#pragma unroll 2
  for (int c = lane; c < pieces; c += 32) {
    const uint4 gv = __ldg(gr + c), uv = __ldg(ur + c);
    const T* ge = reinterpret_cast<const T*>(&gv);
    const T* ue = reinterpret_cast<const T*>(&uv);
    uint4 hv;
    T* he = reinterpret_cast<T*>(&hv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float g = to_f32<T>(ge[k]);
      const float s = round_to<T>(__fdiv_rn(g, silu_den(g)));
      he[k] = from_f32<T>(__fmul_rn(s, to_f32<T>(ue[k])));
    }
    hr[c] = hv;
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) swiglu_bwd_kernel(const DsaltSwigluParams p) {
  const int64_t t = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  if (t >= p.T) return;
  const int lane = threadIdx.x & 31, pieces = (int)(p.F / 8);
  const uint4* gr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.g) + t * p.ld_in);
  const uint4* ur = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.u) + t * p.ld_in);
  const uint4* dr = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.dh) + t * p.F);
  uint4* dgr = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.dg) + t * p.ld_out);
  uint4* dur = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.du) + t * p.ld_out);
#pragma unroll 2
  for (int c = lane; c < pieces; c += 32) {
    const uint4 gv = __ldg(gr + c), uv = __ldg(ur + c), dv = __ldg(dr + c);
    const T* ge = reinterpret_cast<const T*>(&gv);
    const T* ue = reinterpret_cast<const T*>(&uv);
    const T* de = reinterpret_cast<const T*>(&dv);
    uint4 dgv, duv;
    T* dge = reinterpret_cast<T*>(&dgv);
    T* due = reinterpret_cast<T*>(&duv);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const float g = to_f32<T>(ge[k]), dh = to_f32<T>(de[k]);
      const float den = silu_den(g);
      const float s = round_to<T>(__fdiv_rn(g, den));
      const float ds = round_to<T>(__fmul_rn(dh, to_f32<T>(ue[k])));
      due[k] = from_f32<T>(__fmul_rn(dh, s));
      const float sig = __fdiv_rn(1.f, den);
      const float tail = fmaf(g, __fsub_rn(1.f, sig), 1.f);
      dge[k] = from_f32<T>(__fmul_rn(__fmul_rn(ds, sig), tail));
    }
    dgr[c] = dgv;
    dur[c] = duv;
  }
}

}  // namespace

cudaError_t launch_swiglu(const DsaltSwigluParams& p, bool bwd, cudaStream_t st) {
  if (p.T == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((p.T + kRowsPerCta - 1) / kRowsPerCta);
  switch (p.dtype) {
    case DSALT_BF16:
      if (bwd) swiglu_bwd_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
      else swiglu_fwd_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>(p);
      break;
    case DSALT_F16:
      if (bwd) swiglu_bwd_kernel<__half><<<grid, kThreads, 0, st>>>(p);
      else swiglu_fwd_kernel<__half><<<grid, kThreads, 0, st>>>(p);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace dsalt
