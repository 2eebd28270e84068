// The attention prologue of DSALTAttention._packed in one HBM-bound pass: RoPE on
// q and k (reference apply_rotary_emb, dsalt/kernels/window_utils.py:73-88) and
// the GQA expansion of k and v to the query heads (_repeat_kv,
// dsalt/modules/dsalt_attention.py:254-268), plus the backward of both.
//
// Layout: q [T, H, D], k and v [T, Hkv, D], cos and sin [T, D] (each token's
// position row, input dtype), outputs [T, H, D].  With ld set, q, k and v (and in
// the backward dq, dk and dv) are column blocks of one [T, ld] buffer, the output
// of a single q|k|v projection GEMM.  One thread handles the 8
// elements j0 … j0+7 of the first half of a row and their partners j0+D/2 …,
// with 16-byte (fp32: 32-byte) loads and stores.
//
// Rounding follows the reference's tensor ops exactly: out = R(R(x·c) + R(rot(x)·s))
// with R the rounding to the input dtype (fp32: products and the sum kept apart,
// never contracted into an FMA); the backward rounds g·c, g·s and their sum, and
// the sum over the n_rep copies of a kv head once (the expand's reduction).
#include "common.cuh"

namespace dsalt {
namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ void load8(const T* src, float* x) {
  if constexpr (sizeof(T) == 2) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(src));
    const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[i] = to_f32<T>(e[i]);
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(src));
    const float4 b = __ldg(reinterpret_cast<const float4*>(src) + 1);
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
}

template <typename T>
__device__ __forceinline__ void store8(T* dst, const float* x) {
  if constexpr (sizeof(T) == 2) {
    uint4 u;
    T* e = reinterpret_cast<T*>(&u);
#pragma unroll
    for (int i = 0; i < 8; ++i) e[i] = from_f32<T>(x[i]);
    *reinterpret_cast<uint4*>(dst) = u;
  } else {
    reinterpret_cast<float4*>(dst)[0] = make_float4(x[0], x[1], x[2], x[3]);
    reinterpret_cast<float4*>(dst)[1] = make_float4(x[4], x[5], x[6], x[7]);
  }
}

// products and sums rounded to T one by one (fp32: no FMA contraction)
template <typename T> __device__ __forceinline__ float mul_r(float a, float b) { return round_to<T>(__fmul_rn(a, b)); }
template <typename T> __device__ __forceinline__ float add_r(float a, float b) { return round_to<T>(__fadd_rn(a, b)); }

// forward rotation of a row's element pairs, in place (a = x[j], b = x[j + D/2]):
//   out[j] = x[j]·c[j] − x[j+D/2]·s[j],  out[j+D/2] = x[j+D/2]·c[j+D/2] + x[j]·s[j+D/2]
template <typename T>
__device__ __forceinline__ void rope8(float* a, float* b, const float* c1, const float* c2, const float* s1,
                                      const float* s2) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float o1 = add_r<T>(mul_r<T>(a[i], c1[i]), -mul_r<T>(b[i], s1[i]));
    const float o2 = add_r<T>(mul_r<T>(b[i], c2[i]), mul_r<T>(a[i], s2[i]));
    a[i] = o1;
    b[i] = o2;
  }
}

// transposed rotation of the gradient pairs, in place (g1 = g[j], g2 = g[j + D/2]):
//   dx[j] = g[j]·c[j] + g[j+D/2]·s[j+D/2],  dx[j+D/2] = g[j+D/2]·c[j+D/2] − g[j]·s[j]
template <typename T>
__device__ __forceinline__ void rope8_t(float* g1, float* g2, const float* c1, const float* c2, const float* s1,
                                        const float* s2) {
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float d1 = add_r<T>(mul_r<T>(g1[i], c1[i]), mul_r<T>(g2[i], s2[i]));
    const float d2 = add_r<T>(mul_r<T>(g2[i], c2[i]), -mul_r<T>(g1[i], s1[i]));
    g1[i] = d1;
    g2[i] = d2;
  }
}

template <typename T>
__device__ __forceinline__ void load_cs(const DsaltRopeParams& p, uint32_t t, int j0, int half, float* c1, float* c2,
                                        float* s1, float* s2) {
  const T* cs = reinterpret_cast<const T*>(p.cos) + (int64_t)t * p.D + j0;
  const T* sn = reinterpret_cast<const T*>(p.sin) + (int64_t)t * p.D + j0;
  load8<T>(cs, c1);
  load8<T>(cs + half, c2);
  load8<T>(sn, s1);
  load8<T>(sn + half, s2);
}

// One thread per (token, query head, 8-element group of the first half); the
// thread counts stay below 2^31 (checked by the host), so the index arithmetic is
// 32-bit (lg = log2(D / 16)).
template <typename T>
__global__ void __launch_bounds__(kThreads, 4) rope_gqa_fwd_kernel(const DsaltRopeParams p, int lg) {
  const int half = p.D / 2, n_rep = p.H / p.Hkv;
  const uint32_t idx = blockIdx.x * kThreads + threadIdx.x;
  if (idx >= (uint32_t)p.T * p.H << lg) return;
  const int j0 = 8 * (int)(idx & ((1u << lg) - 1));
  const uint32_t row = idx >> lg;  // t·H + h
  const uint32_t t = row / (uint32_t)p.H;
  const uint32_t h = row - t * (uint32_t)p.H;
  const int64_t ldq = p.ld ? p.ld : (int64_t)p.H * p.D, ldk = p.ld ? p.ld : (int64_t)p.Hkv * p.D;
  const int64_t kofs = (int64_t)t * ldk + (int64_t)(h / (uint32_t)n_rep) * p.D + j0;
  float c1[8], c2[8], s1[8], s2[8], a[8], b[8];
  load_cs<T>(p, t, j0, half, c1, c2, s1, s2);
  const T* q = reinterpret_cast<const T*>(p.q) + (int64_t)t * ldq + (int64_t)h * p.D + j0;
  load8<T>(q, a);
  load8<T>(q + half, b);
  rope8<T>(a, b, c1, c2, s1, s2);
  T* qo = reinterpret_cast<T*>(p.q_out) + (int64_t)row * p.D + j0;
  store8<T>(qo, a);
  store8<T>(qo + half, b);
  // k_out expanded to the query heads, or (kv_out_heads = Hkv) once per kv head
  const bool expand = p.kv_out_heads <= 0 || p.kv_out_heads == p.H;
  if (!expand && h % (uint32_t)n_rep != 0) return;
  const int64_t orow = expand ? (int64_t)row : (int64_t)t * p.Hkv + h / (uint32_t)n_rep;
  const T* k = reinterpret_cast<const T*>(p.k) + kofs;
  load8<T>(k, a);
  load8<T>(k + half, b);
  rope8<T>(a, b, c1, c2, s1, s2);
  T* ko = reinterpret_cast<T*>(p.k_out) + orow * p.D + j0;
  store8<T>(ko, a);
  store8<T>(ko + half, b);
  if (p.v_out) {
    const T* v = reinterpret_cast<const T*>(p.v) + kofs;
    T* vo = reinterpret_cast<T*>(p.v_out) + orow * p.D + j0;
    load8<T>(v, a);
    load8<T>(v + half, b);
    store8<T>(vo, a);
    store8<T>(vo + half, b);
  }
}

// threads [0, T·H·G): dq rows; then [T·H·G, T·(H + Hkv)·G): dk / dv rows of the kv heads
template <typename T>
__global__ void __launch_bounds__(kThreads, 4) rope_gqa_bwd_kernel(const DsaltRopeParams p, int lg) {
  const int half = p.D / 2, n_rep = p.H / p.Hkv;
  const uint32_t nq = (uint32_t)p.T * p.H << lg;
  uint32_t idx = blockIdx.x * kThreads + threadIdx.x;
  if (idx >= nq + ((uint32_t)p.T * p.Hkv << lg)) return;
  float c1[8], c2[8], s1[8], s2[8], g1[8], g2[8];
  if (idx < nq) {
    const int j0 = 8 * (int)(idx & ((1u << lg) - 1));
    const uint32_t row = idx >> lg;
    const uint32_t t = row / (uint32_t)p.H;
    const uint32_t h = row - t * (uint32_t)p.H;
    load_cs<T>(p, t, j0, half, c1, c2, s1, s2);
    const T* g = reinterpret_cast<const T*>(p.dq_out) + (int64_t)row * p.D + j0;
    load8<T>(g, g1);
    load8<T>(g + half, g2);
    rope8_t<T>(g1, g2, c1, c2, s1, s2);
    const int64_t ldq = p.ld ? p.ld : (int64_t)p.H * p.D;
    T* dq = reinterpret_cast<T*>(p.dq) + (int64_t)t * ldq + (int64_t)h * p.D + j0;
    store8<T>(dq, g1);
    store8<T>(dq + half, g2);
    return;
  }
  idx -= nq;
  const int j0 = 8 * (int)(idx & ((1u << lg) - 1));
  const uint32_t krow = idx >> lg;  // t·Hkv + hk
  const uint32_t t = krow / (uint32_t)p.Hkv;
  const uint32_t hk = krow - t * (uint32_t)p.Hkv;
  // the copies of this kv head in dk_out: n_rep query-head rows (expanded), or
  // its own row (kv_out_heads = Hkv)
  const bool expand = p.kv_out_heads <= 0 || p.kv_out_heads == p.H;
  const int copies = expand ? n_rep : 1;
  const int64_t row0 = expand ? (int64_t)t * p.H + (int64_t)hk * n_rep : (int64_t)t * p.Hkv + hk;
  // the sum over the copies (fp32, rounded once), then the transposed rotation
  float x[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) { g1[i] = 0.f; g2[i] = 0.f; }
  for (int r = 0; r < copies; ++r) {
    const T* g = reinterpret_cast<const T*>(p.dk_out) + (row0 + r) * p.D + j0;
    load8<T>(g, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) g1[i] += x[i];
    load8<T>(g + half, x);
#pragma unroll
    for (int i = 0; i < 8; ++i) g2[i] += x[i];
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) { g1[i] = round_to<T>(g1[i]); g2[i] = round_to<T>(g2[i]); }
  load_cs<T>(p, t, j0, half, c1, c2, s1, s2);
  rope8_t<T>(g1, g2, c1, c2, s1, s2);
  const int64_t kofs = (int64_t)t * (p.ld ? p.ld : (int64_t)p.Hkv * p.D) + (int64_t)hk * p.D + j0;
  T* dk = reinterpret_cast<T*>(p.dk) + kofs;
  store8<T>(dk, g1);
  store8<T>(dk + half, g2);
  if (p.dv_out && p.dv) {
#pragma unroll
    for (int i = 0; i < 8; ++i) { g1[i] = 0.f; g2[i] = 0.f; }
    for (int r = 0; r < copies; ++r) {
      const T* g = reinterpret_cast<const T*>(p.dv_out) + (row0 + r) * p.D + j0;
      load8<T>(g, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) g1[i] += x[i];
      load8<T>(g + half, x);
#pragma unroll
      for (int i = 0; i < 8; ++i) g2[i] += x[i];
    }
    T* dv = reinterpret_cast<T*>(p.dv) + kofs;
    store8<T>(dv, g1);
    store8<T>(dv + half, g2);
  }
}

template <typename T>
cudaError_t launch(const DsaltRopeParams& p, bool bwd, cudaStream_t st) {
  const int G = p.D / 16;
  int lg = 0;
  while ((1 << lg) < G) ++lg;
  const int64_t n = bwd ? p.T * (p.H + p.Hkv) * G : p.T * p.H * G;
  if (n == 0) return cudaSuccess;
  const unsigned grid = (unsigned)((n + kThreads - 1) / kThreads);
  if (bwd) rope_gqa_bwd_kernel<T><<<grid, kThreads, 0, st>>>(p, lg);
  else rope_gqa_fwd_kernel<T><<<grid, kThreads, 0, st>>>(p, lg);
  return cudaGetLastError();
}

}  // namespace

// thread count of the larger (backward) launch: the kernels index in 32 bits
bool rope_gqa_fits(const DsaltRopeParams& p) { return p.T * (int64_t)(p.H + p.Hkv) * (p.D / 16) < (1ll << 31); }

namespace {

}  // namespace

cudaError_t launch_rope_gqa(const DsaltRopeParams& p, bool bwd, cudaStream_t st) {
  switch (p.dtype) {
    case DSALT_BF16: return launch<__nv_bfloat16>(p, bwd, st);
    case DSALT_F16: return launch<__half>(p, bwd, st);
    case DSALT_F32: return launch<float>(p, bwd, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace dsalt
