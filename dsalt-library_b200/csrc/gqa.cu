// Grouped kv heads: the sum of the per-query-head K/V gradients of each group.
//
// With H_kv < H the attention kernels read kv head h / (H / H_kv) in place, and
// the backward writes dk, dv per query head: the gradients of the expanded K/V
// of the reference's _repeat_kv (dsalt/modules/dsalt_attention.py:254-268).
// Their sum over each group of H / H_kv query heads is the gradient of the
// [T, H_kv, D] K/V: summed here in fp32 and rounded once, as the autograd of the
// expansion does.  One thread per 16-byte piece of an output row.
#include "common.cuh"

namespace dsalt {

template <typename T>
__global__ void __launch_bounds__(256) gqa_reduce_kernel(const T* __restrict__ x, T* __restrict__ y, int64_t T_,
                                                         int H, int H_kv, int D) {
  constexpr int kVec = 16 / (int)sizeof(T);
  const int pieces = D / kVec;
  const int64_t n = T_ * H_kv * pieces;
  const int rep = H / H_kv;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)(e % pieces);
    const int64_t tg = e / pieces;  // t * H_kv + g
    const int g = (int)(tg % H_kv);
    const int64_t t = tg / H_kv;
    float acc[kVec];
#pragma unroll
    for (int k = 0; k < kVec; ++k) acc[k] = 0.f;
    for (int r = 0; r < rep; ++r) {
      const uint4 u = reinterpret_cast<const uint4*>(x + (t * H + (int64_t)g * rep + r) * D)[c];
      const T* v = reinterpret_cast<const T*>(&u);
#pragma unroll
      for (int k = 0; k < kVec; ++k) acc[k] += to_f32<T>(v[k]);
    }
    uint4 o;
    T* ov = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int k = 0; k < kVec; ++k) ov[k] = from_f32<T>(acc[k]);
    reinterpret_cast<uint4*>(y + tg * D)[c] = o;
  }
}

cudaError_t launch_gqa_reduce(const DsaltGqaReduceParams& p, cudaStream_t st) {
  const int esz = p.dtype == DSALT_F32 ? 4 : 2;
  const int64_t n = p.T * p.H_kv * (p.D * esz / 16);
  if (n == 0) return cudaSuccess;
  const unsigned grid = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
  switch (p.dtype) {
    case DSALT_BF16:
      gqa_reduce_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(p.x),
                                                             static_cast<__nv_bfloat16*>(p.y), p.T, p.H, p.H_kv, p.D);
      break;
    case DSALT_F16:
      gqa_reduce_kernel<__half><<<grid, 256, 0, st>>>(static_cast<const __half*>(p.x), static_cast<__half*>(p.y),
                                                      p.T, p.H, p.H_kv, p.D);
      break;
    case DSALT_F32:
      gqa_reduce_kernel<float><<<grid, 256, 0, st>>>(static_cast<const float*>(p.x), static_cast<float*>(p.y), p.T,
                                                     p.H, p.H_kv, p.D);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace dsalt
