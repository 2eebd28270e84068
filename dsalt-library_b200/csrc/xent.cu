// Cross-entropy of one chunk of LM-head logits with its gradient, in place (the
// chunked loss of dsalt/model/dsalt_lm.py:19-39: F.cross_entropy on the chunk's
// logits, fp32 under autocast, sum reduction, divided by the valid-label count).
// One CTA per row: an online max / sum of exp over the row in fp32, lse = m +
// log(s), loss = lse − logit[y] (0 for ignore_index), then the row is overwritten
// with d loss / d logit = (exp(l − lse) − [j = y]) · scale, rounded to the dtype,
// where scale = *p.scale (1 / #valid labels of the whole batch) and 0 for an
// ignored row.
#include "common.cuh"

namespace dsalt {
namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ void online_merge(float& m, float& s, float m2, float s2) {
  if (m2 == -INFINITY) return;
  if (m == -INFINITY) { m = m2; s = s2; return; }
  const float mm = fmaxf(m, m2);
  s = s * expf(m - mm) + s2 * expf(m2 - mm);
  m = mm;
}

template <typename T>
__global__ void __launch_bounds__(kThreads) xent_kernel(const DsaltXentParams p) {
  __shared__ float red_m[kThreads / 32], red_s[kThreads / 32];
  __shared__ float row_lse;
  const int64_t row = blockIdx.x;
  T* lg = reinterpret_cast<T*>(p.logits) + row * p.vocab;
  const int V = p.vocab, V8 = V % 8 == 0 ? V / 8 : 0;  // 16-byte rows only when V is a multiple of 8
  // pass 1: running max and sum of exp (8 elements per 16-byte load)
  float m = -INFINITY, s = 0.f;
  for (int i = threadIdx.x; i < V8; i += kThreads) {
    const uint4 u = reinterpret_cast<const uint4*>(lg)[i];
    const T* e = reinterpret_cast<const T*>(&u);
    float x[8], mx = -INFINITY;
#pragma unroll
    for (int k = 0; k < 8; ++k) { x[k] = to_f32<T>(e[k]); mx = fmaxf(mx, x[k]); }
    float sx = 0.f;
#pragma unroll
    for (int k = 0; k < 8; ++k) sx += expf(x[k] - mx);
    online_merge(m, s, mx, sx);
  }
  for (int i = V8 * 8 + threadIdx.x; i < V; i += kThreads) online_merge(m, s, to_f32<T>(lg[i]), 1.f);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off), s2 = __shfl_xor_sync(0xffffffffu, s, off);
    online_merge(m, s, m2, s2);
  }
  if ((threadIdx.x & 31) == 0) { red_m[threadIdx.x >> 5] = m; red_s[threadIdx.x >> 5] = s; }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red_m[0], ss = red_s[0];
    for (int w = 1; w < kThreads / 32; ++w) online_merge(mm, ss, red_m[w], red_s[w]);
    const float lse = mm + logf(ss);
    row_lse = lse;
    const int64_t y = p.labels[row];
    const bool valid = y != p.ignore_index && y >= 0 && y < V;
    p.row_loss[row] = valid ? lse - to_f32<T>(lg[y]) : 0.f;
  }
  __syncthreads();
  const float lse = row_lse;
  const int64_t y = p.labels[row];
  const bool valid = y != p.ignore_index && y >= 0 && y < V;
  const float sc = valid ? __ldg(p.scale) : 0.f;
  // pass 2: the gradient, in place
  for (int i = threadIdx.x; i < V8; i += kThreads) {
    uint4 u = reinterpret_cast<const uint4*>(lg)[i];
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int j = 8 * i + k;
      const float g = expf(to_f32<T>(e[k]) - lse) - (j == y ? 1.f : 0.f);
      e[k] = from_f32<T>(g * sc);
    }
    reinterpret_cast<uint4*>(lg)[i] = u;
  }
  for (int j = V8 * 8 + threadIdx.x; j < V; j += kThreads) {
    const float g = expf(to_f32<T>(lg[j]) - lse) - (j == y ? 1.f : 0.f);
    lg[j] = from_f32<T>(g * sc);
  }
}

}  // namespace

cudaError_t launch_xent(const DsaltXentParams& p, cudaStream_t st) {
  if (p.rows == 0) return cudaSuccess;
  switch (p.dtype) {
    case DSALT_BF16: xent_kernel<__nv_bfloat16><<<(unsigned)p.rows, kThreads, 0, st>>>(p); break;
    case DSALT_F16: xent_kernel<__half><<<(unsigned)p.rows, kThreads, 0, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace dsalt
