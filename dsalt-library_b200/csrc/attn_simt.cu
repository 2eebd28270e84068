// Exact-arithmetic SIMT kernels for the DSALT attention (fp32 math for every
// input dtype).  These are the fp32 path (fp32 inputs keep fp32 precision,
// unlike the reference, which casts them to fp16 at
// dsalt/kernels/dsalt_triton_train.py:601-604) and the cross-check for the
// tcgen05 kernels.  One warp owns one (token, head) row and walks the row's
// attended set explicitly, so no masked work is done.
//
// Attended set of query i (training semantics; inference is mapped onto it by
// row_window()):
//   band      j in [i - min(W, i), i],  W = floor(w̃)      (dsalt_triton_train.py:147-150)
//   landmarks the sorted landmark prefix with p <= i and float(p) < float(i) - w̃
//                                                            (dsalt_triton_train.py:182-185)
#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {

constexpr int kSimtWarps = 8;  // warps per CTA

// Lane `lane` holds elements lane + 32 r (r < R = ceil(D/32)) of a head row;
// elements past the runtime head dim D read as zero.
template <typename T, int R>
struct RowVec {
  float x[R];
  __device__ __forceinline__ void load(const T* __restrict__ p, int lane, int D) {
#pragma unroll
    for (int r = 0; r < R; ++r) x[r] = (lane + 32 * r < D) ? to_f32<T>(p[lane + 32 * r]) : 0.f;
  }
  __device__ __forceinline__ float dot(const T* __restrict__ p, int lane, int D) const {
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (lane + 32 * r < D) s = fmaf(x[r], to_f32<T>(p[lane + 32 * r]), s);
    return warp_sum(s);
  }
};

// ------------------------------------------------------------------ forward
template <typename T, int R>
__global__ void __launch_bounds__(kSimtWarps * 32)
simt_fwd_kernel(const DsaltAttnParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kSimtWarps + (threadIdx.x >> 5);
  if (row >= p.T * p.H) return;
  const int64_t t = row / p.H;
  const int h = (int)(row % p.H);
  const int s = find_seq(p.cu_seqlens, p.S, t);
  const int64_t s0 = p.cu_seqlens[s];
  const int i = (int)(t - s0);
  const RowWindow rw = row_window(p.w[t], i, p.semantics, p.win_edge);
  const float inv_tau = 1.0f / p.tau_win;
  const int D = p.D;
  const int64_t HD = (int64_t)p.H * D;
  const int64_t KHD = (int64_t)attn_kv_heads(p) * D;  // k, v row stride (grouped kv heads)

  const T* q = reinterpret_cast<const T*>(p.q) + t * HD + (int64_t)h * D;
  const T* kb = reinterpret_cast<const T*>(p.k) + (int64_t)attn_kv_head(p, h) * D;
  const T* vb = reinterpret_cast<const T*>(p.v) + (int64_t)attn_kv_head(p, h) * D;
  RowVec<T, R> qv;
  qv.load(q, lane, D);

  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  float m = -INFINITY, l = 0.f;

  auto visit = [&](const T* kp, const T* vp, float bias) {
    const float sc = fmaf(qv.dot(kp, lane, D), p.scale, bias);
    if (sc > m) {
      const float corr = (m == -INFINITY) ? 0.f : expf(m - sc);
      l *= corr;
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] *= corr;
      m = sc;
    }
    const float pr = expf(sc - m);
    l += pr;
#pragma unroll
    for (int r = 0; r < R; ++r)
      if (lane + 32 * r < D) acc[r] = fmaf(pr, to_f32<T>(vp[lane + 32 * r]), acc[r]);
  };

  if (rw.W >= 0) {
    const int jlo = i - min(rw.W, i);
    for (int j = jlo; j <= i; ++j) {
      const float d = (float)(i - j);
      const int64_t kt = s0 + j;
      visit(kb + kt * KHD, vb + kt * KHD, edge_bias(rw, d, inv_tau));
    }
  }
  const int64_t lbase = ((int64_t)h * p.S + s) * p.kp;
  for (int c = 0; c < p.kp; ++c) {
    const int ps = p.pos_sorted[lbase + c];
    if (ps < 0 || ps > i || !((float)ps < rw.win_lo)) break;  // valid set is a sorted prefix
    const T* lk = reinterpret_cast<const T*>(p.lmk_k) + (lbase + c) * D;
    const T* lv = reinterpret_cast<const T*>(p.lmk_v) + (lbase + c) * D;
    visit(lk, lv, p.w_sorted[lbase + c]);
  }

  const bool nonempty = l > 1e-9f;
  const float inv_l = nonempty ? 1.0f / l : 0.f;
  T* o = reinterpret_cast<T*>(p.o) + t * HD + (int64_t)h * D;
  float* of = p.o_f32 ? p.o_f32 + t * HD + (int64_t)h * D : nullptr;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (lane + 32 * r >= D) continue;
    const T ov = from_f32<T>(acc[r] * inv_l);
    if (p.o) o[lane + 32 * r] = ov;
    if (of) of[lane + 32 * r] = to_f32<T>(ov);
  }
  if (lane == 0) p.lse[t * p.H + h] = nonempty ? m + logf(l) : -INFINITY;
}

// ------------------------------------------------------------- preprocess
// Delta[t,h] = Σ_d O·dO with O the stored (input-dtype) output and dO rounded to
// the input dtype (dsalt_triton_train.py:220-237, 673-674).  When the caller
// passes the fp32 upstream gradient (dout_f32), this kernel also writes its
// input-dtype copy to dout for the tensor-core stages.
template <typename T, int R>
__global__ void __launch_bounds__(kSimtWarps * 32)
bwd_preprocess_kernel(const DsaltAttnParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kSimtWarps + (threadIdx.x >> 5);
  if (row >= p.T * p.H) return;
  const int D = p.D;
  // the stored O: the input-dtype copy, or the fp32 copy (same values) when only that was written
  const T* o = p.o ? reinterpret_cast<const T*>(p.o) + row * D : nullptr;
  const float* of = p.o ? nullptr : p.o_f32 + row * D;
  const T* g = reinterpret_cast<const T*>(p.dout) + row * D;
  const float* gf = p.dout_f32 ? p.dout_f32 + row * D : nullptr;
  T* gw = const_cast<T*>(g);
  float s = 0.f;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int e = lane + 32 * r;
    if (e >= D) continue;
    float gv;
    if (gf) {
      const T gt = from_f32<T>(gf[e]);
      gw[e] = gt;
      gv = to_f32<T>(gt);
    } else {
      gv = to_f32<T>(g[e]);
    }
    s = fmaf(o ? to_f32<T>(o[e]) : of[e], gv, s);
  }
  s = warp_sum(s);
  if (lane == 0) {
    p.delta[row] = s;
    if (p.qrec && p.dw_head) p.dw_head[row] = 0.f;  // the tensor-core dK/dV stage adds into it
    if (p.qrec) write_qrec(p, row / p.H, (int)(row % p.H), s);
  }
}

// ---------------------------------------------------------------- dQ, d_w̃
template <typename T, int R>
__global__ void __launch_bounds__(kSimtWarps * 32)
simt_bwd_dq_kernel(const DsaltAttnParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kSimtWarps + (threadIdx.x >> 5);
  if (row >= p.T * p.H) return;
  const int64_t t = row / p.H;
  const int h = (int)(row % p.H);
  const int s = find_seq(p.cu_seqlens, p.S, t);
  const int64_t s0 = p.cu_seqlens[s];
  const int i = (int)(t - s0);
  const RowWindow rw = row_window(p.w[t], i, p.semantics, p.win_edge);
  const float inv_tau = 1.0f / p.tau_win;
  const int D = p.D;
  const int64_t HD = (int64_t)p.H * D;

  const float lse = p.lse[row];
  const float delta = p.delta[row];
  float dq[R];
#pragma unroll
  for (int r = 0; r < R; ++r) dq[r] = 0.f;
  float dw = 0.f;

  if (lse != -INFINITY) {
    RowVec<T, R> qv, gv;
    qv.load(reinterpret_cast<const T*>(p.q) + t * HD + (int64_t)h * D, lane, D);
    gv.load(reinterpret_cast<const T*>(p.dout) + t * HD + (int64_t)h * D, lane, D);
    const int64_t KHD = (int64_t)attn_kv_heads(p) * D;  // k, v row stride (grouped kv heads)
    const T* kb = reinterpret_cast<const T*>(p.k) + (int64_t)attn_kv_head(p, h) * D;
    const T* vb = reinterpret_cast<const T*>(p.v) + (int64_t)attn_kv_head(p, h) * D;
    auto visit = [&](const T* kp, const T* vp, float bias, float dbias) {
      const float sc = fmaf(qv.dot(kp, lane, D), p.scale, bias);
      const float pr = expf(sc - lse);
      const float dp = gv.dot(vp, lane, D);
      const float ds = pr * (dp - delta);
      dw = fmaf(ds, dbias, dw);
      const float dss = ds * p.scale;
#pragma unroll
      for (int r = 0; r < R; ++r)
        if (lane + 32 * r < D) dq[r] = fmaf(dss, to_f32<T>(kp[lane + 32 * r]), dq[r]);
    };
    if (rw.W >= 0) {
      const int jlo = i - min(rw.W, i);
      for (int j = jlo; j <= i; ++j) {
        const float d = (float)(i - j);
        const int64_t kt = s0 + j;
        visit(kb + kt * KHD, vb + kt * KHD, edge_bias(rw, d, inv_tau), edge_dbias(rw, d, inv_tau));
      }
    }
    const int64_t lbase = ((int64_t)h * p.S + s) * p.kp;
    for (int c = 0; c < p.kp; ++c) {
      const int ps = p.pos_sorted[lbase + c];
      if (ps < 0 || ps > i || !((float)ps < rw.win_lo)) break;
      visit(reinterpret_cast<const T*>(p.lmk_k) + (lbase + c) * D,
            reinterpret_cast<const T*>(p.lmk_v) + (lbase + c) * D, p.w_sorted[lbase + c], 0.f);
    }
  }
  T* out = reinterpret_cast<T*>(p.dq) + t * HD + (int64_t)h * D;
#pragma unroll
  for (int r = 0; r < R; ++r)
    if (lane + 32 * r < D) out[lane + 32 * r] = from_f32<T>(dq[r]);
  if (lane == 0 && p.dw_head) p.dw_head[row] = dw;
}

// ---------------------------------------------------------- dK, dV, d_lw
// Key-parallel and atomic-free: one warp owns key j of head h and visits every
// query that attends it, through the band (i in [j, j + wmax]) and, when j is
// a landmark of (h, seq), through the landmark rule (all later queries whose
// window no longer covers j).  d_lw of that landmark is a plain warp sum.
template <typename T, int R>
__global__ void __launch_bounds__(kSimtWarps * 32)
simt_bwd_dkdv_kernel(const DsaltAttnParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kSimtWarps + (threadIdx.x >> 5);
  if (row >= p.T * p.H) return;
  const int64_t t = row / p.H;
  const int h = (int)(row % p.H);
  const int s = find_seq(p.cu_seqlens, p.S, t);
  const int64_t s0 = p.cu_seqlens[s];
  const int L = (int)(p.cu_seqlens[s + 1] - s0);
  const int j = (int)(t - s0);
  const float inv_tau = 1.0f / p.tau_win;
  const int D = p.D;
  const int64_t HD = (int64_t)p.H * D;

  RowVec<T, R> kv, vv;
  // the kv head of query head h; dk, dv are written per query head
  const int64_t KHD = (int64_t)attn_kv_heads(p) * D;
  kv.load(reinterpret_cast<const T*>(p.k) + t * KHD + (int64_t)attn_kv_head(p, h) * D, lane, D);
  vv.load(reinterpret_cast<const T*>(p.v) + t * KHD + (int64_t)attn_kv_head(p, h) * D, lane, D);
  const T* qb = reinterpret_cast<const T*>(p.q) + (int64_t)h * D;
  const T* gb = reinterpret_cast<const T*>(p.dout) + (int64_t)h * D;
  float dk[R], dv[R];
#pragma unroll
  for (int r = 0; r < R; ++r) { dk[r] = 0.f; dv[r] = 0.f; }

  auto visit = [&](int64_t qt, float bias) -> float {
    const float lse = p.lse[qt * p.H + h];
    if (lse == -INFINITY) return 0.f;
    const T* qp = qb + qt * HD;
    const T* gp = gb + qt * HD;
    const float sc = fmaf(kv.dot(qp, lane, D), p.scale, bias);
    const float pr = expf(sc - lse);
    const float dp = vv.dot(gp, lane, D);
    const float ds = pr * (dp - p.delta[qt * p.H + h]);
    const float dss = ds * p.scale;
#pragma unroll
    for (int r = 0; r < R; ++r) {
      if (lane + 32 * r >= D) continue;
      dv[r] = fmaf(pr, to_f32<T>(gp[lane + 32 * r]), dv[r]);
      dk[r] = fmaf(dss, to_f32<T>(qp[lane + 32 * r]), dk[r]);
    }
    return ds;
  };

  // band: query i attends j iff 0 <= i - j <= W_i
  const int ihi = min(L - 1, j + max(p.seq_wmax[s], 0));
  for (int i = j; i <= ihi; ++i) {
    const RowWindow rw = row_window(p.w[s0 + i], i, p.semantics, p.win_edge);
    const int d = i - j;
    if (d > rw.W) continue;
    visit(s0 + i, edge_bias(rw, (float)d, inv_tau));
  }
  // landmark slots at this token (sorted, duplicates adjacent)
  const int64_t lbase = ((int64_t)h * p.S + s) * p.kp;
  int c = p.lmk_slot ? p.lmk_slot[t * p.H + h] : -1;
  for (; c >= 0 && c < p.kp && p.pos_sorted[lbase + c] == j; ++c) {
    const float bias = p.w_sorted[lbase + c];
    float dlw = 0.f;
    for (int i = j; i < L; ++i) {
      const RowWindow rw = row_window(p.w[s0 + i], i, p.semantics, p.win_edge);
      if (!((float)j < rw.win_lo)) continue;  // (p <= i holds: i >= j)
      dlw += visit(s0 + i, bias);
    }
    const int slot = p.perm[lbase + c];
    if (lane == 0 && slot >= 0 && p.d_lw)
      p.d_lw[((int64_t)h * p.S + s) * p.k_lmk + slot] = p.grad_round ? round_to<T>(dlw) : dlw;
  }
  T* dko = reinterpret_cast<T*>(p.dk) + t * HD + (int64_t)h * D;
  T* dvo = reinterpret_cast<T*>(p.dv) + t * HD + (int64_t)h * D;
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (lane + 32 * r >= D) continue;
    dko[lane + 32 * r] = from_f32<T>(dk[r]);
    dvo[lane + 32 * r] = from_f32<T>(dv[r]);
  }
}

// The same Delta with 16-byte accesses: one thread per 8 consecutive elements
// (bf16/fp16 inputs), G = D/8 lanes per (t, h) row, G a power of two ≤ 32, so a
// row's lanes are an aligned group of one warp.  The fp32 dO is read with
// streaming loads (it is not read again).
template <typename T, int G>
__global__ void __launch_bounds__(256)
bwd_preprocess_vec_kernel(const DsaltAttnParams p) {
  static_assert(sizeof(T) == 2, "16-bit inputs only");
  const int64_t chunk = (int64_t)blockIdx.x * 256 + threadIdx.x;
  const int64_t n_chunks = p.T * p.H * G;
  float s = 0.f;
  if (chunk < n_chunks) {
    // the stored O: the input-dtype copy, or the fp32 copy (same values) when only that was written
    float of[8];
    if (p.o) {
      const uint4 ov = __ldg(reinterpret_cast<const uint4*>(p.o) + chunk);
      const T* o8 = reinterpret_cast<const T*>(&ov);
#pragma unroll
      for (int e = 0; e < 8; ++e) of[e] = to_f32<T>(o8[e]);
    } else {
      const float4 a = __ldg(reinterpret_cast<const float4*>(p.o_f32) + 2 * chunk);
      const float4 b = __ldg(reinterpret_cast<const float4*>(p.o_f32) + 2 * chunk + 1);
      of[0] = a.x; of[1] = a.y; of[2] = a.z; of[3] = a.w; of[4] = b.x; of[5] = b.y; of[6] = b.z; of[7] = b.w;
    }
    uint4 gv;
    if (p.dout_f32) {
      const float4 a = __ldcs(reinterpret_cast<const float4*>(p.dout_f32) + 2 * chunk);
      const float4 b = __ldcs(reinterpret_cast<const float4*>(p.dout_f32) + 2 * chunk + 1);
      constexpr bool kBF16 = !std::is_same<T, __half>::value;
      gv.x = sm100::pack2(a.x, a.y, kBF16);
      gv.y = sm100::pack2(a.z, a.w, kBF16);
      gv.z = sm100::pack2(b.x, b.y, kBF16);
      gv.w = sm100::pack2(b.z, b.w, kBF16);
      reinterpret_cast<uint4*>(const_cast<void*>(p.dout))[chunk] = gv;
    } else {
      gv = __ldg(reinterpret_cast<const uint4*>(p.dout) + chunk);
    }
    const T* g8 = reinterpret_cast<const T*>(&gv);
#pragma unroll
    for (int e = 0; e < 8; ++e) s = fmaf(of[e], to_f32<T>(g8[e]), s);
  }
#pragma unroll
  for (int off = G / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  const int gl = threadIdx.x & (G - 1);  // lane within the row's group
  const int64_t row = chunk / G;
  if (chunk < n_chunks && gl == 0) {
    p.delta[row] = s;
    if (p.dw_head) p.dw_head[row] = 0.f;  // the tensor-core dK/dV stage adds ∂loss/∂w̃ into it
  }
  if (!p.qrec) return;  // uniform over the grid
  if constexpr (G >= 8) {
    // the row's record: lane gl < 8 computes edge factor gl, lanes 0-3 write its four 16-byte parts
    const bool in = chunk < n_chunks;
    const int64_t t = in ? row / p.H : 0;
    const int h = in ? (int)(row % p.H) : 0;
    int d_e0 = 0;
    QRec rec;
    if (in) rec = qrec_fields(p, t, h, s, &d_e0);
    const float eg = (in && gl < qrec_ne(rec) && gl < kQRecEdge) ? qrec_edge_factor(rec.wt, d_e0 + gl, 1.0f / p.tau_win)
                                                           : 1.0f;
    const int base = threadIdx.x & 31 & ~(G - 1);
    const int src = base + (gl == 3 ? 4 : 0);
    float4 egv;
    egv.x = __shfl_sync(0xffffffffu, eg, src + 0);
    egv.y = __shfl_sync(0xffffffffu, eg, src + 1);
    egv.z = __shfl_sync(0xffffffffu, eg, src + 2);
    egv.w = __shfl_sync(0xffffffffu, eg, src + 3);
    if (in && gl < 4) {
      const float4 h0 = make_float4(rec.nlse2, rec.delta, __int_as_float(rec.lo), __int_as_float(rec.qi));
      const float4 h1 = make_float4(__int_as_float(rec.ehi), __int_as_float(rec.elo), rec.wlo, rec.wt);
      qrec_ptr(p, t, h)[gl] = gl == 0 ? h0 : gl == 1 ? h1 : egv;
    }
  } else {
    if (chunk < n_chunks && gl == 0) write_qrec(p, row / p.H, (int)(row % p.H), s);
  }
}

template <typename T>
static bool launch_preprocess_vec(const DsaltAttnParams& p, cudaStream_t st) {
  if constexpr (sizeof(T) != 2) {
    return false;
  } else {
  const auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15u) == 0; };
  if (!aligned(p.o ? p.o : p.o_f32) || !aligned(p.dout) || (p.dout_f32 && !aligned(p.dout_f32))) return false;
  const int G = p.D / 8;
  const int64_t n_chunks = p.T * p.H * G;
  const dim3 grid((unsigned)((n_chunks + 255) / 256));
  switch (G) {
    case 4: bwd_preprocess_vec_kernel<T, 4><<<grid, 256, 0, st>>>(p); return true;
    case 8: bwd_preprocess_vec_kernel<T, 8><<<grid, 256, 0, st>>>(p); return true;
    case 16: bwd_preprocess_vec_kernel<T, 16><<<grid, 256, 0, st>>>(p); return true;
    case 32: bwd_preprocess_vec_kernel<T, 32><<<grid, 256, 0, st>>>(p); return true;
    default: return false;
  }
  }
}

// d_w̃[t] = Σ_h dw_head[t,h] in fp32; with round set, the value after the cast to
// the input dtype (dsalt_triton_train.py:748,756), kept in fp32
template <typename T>
__global__ void dw_reduce_kernel(const float* __restrict__ dw_head, float* __restrict__ dw, int64_t T_, int H,
                                 int round) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T_) return;
  float s = 0.f;
  for (int h = 0; h < H; ++h) s += dw_head[t * H + h];
  dw[t] = round ? round_to<T>(s) : s;
}

// ------------------------------------------------------------------ launchers
template <typename T, int R>
static cudaError_t launch_simt(int stage, const DsaltAttnParams& p, cudaStream_t st) {
  const int64_t rows = p.T * p.H;
  if (rows == 0) return cudaSuccess;
  const dim3 grid((unsigned)((rows + kSimtWarps - 1) / kSimtWarps));
  const dim3 block(kSimtWarps * 32);
  switch (stage) {
    case 0: simt_fwd_kernel<T, R><<<grid, block, 0, st>>>(p); break;
    case 1:
      if (!launch_preprocess_vec<T>(p, st)) bwd_preprocess_kernel<T, R><<<grid, block, 0, st>>>(p);
      break;
    case 2: {
      // the kernel visits keys that hold a landmark: empty slots get their zero here
      const size_t n_lw = (size_t)p.H * p.S * p.k_lmk;
      if (p.d_lw && n_lw) {
        const cudaError_t e = cudaMemsetAsync(p.d_lw, 0, n_lw * sizeof(float), st);
        if (e != cudaSuccess) return e;
      }
      simt_bwd_dkdv_kernel<T, R><<<grid, block, 0, st>>>(p);
      break;
    }
    case 3:
      simt_bwd_dq_kernel<T, R><<<grid, block, 0, st>>>(p);
      if (p.dw && p.dw_head)
        dw_reduce_kernel<T><<<(unsigned)((p.T + 255) / 256), 256, 0, st>>>(p.dw_head, p.dw, p.T, p.H, p.grad_round);
      break;
    case 4:  // d_w̃ head reduction only (after the tensor-core dQ kernel)
      dw_reduce_kernel<T><<<(unsigned)((p.T + 255) / 256), 256, 0, st>>>(p.dw_head, p.dw, p.T, p.H, p.grad_round);
      break;
  }
  return cudaGetLastError();
}

// R = ceil(D/32) values per lane; any head dim that is a multiple of 8 up to 256
template <typename T>
static cudaError_t launch_simt_d(int stage, const DsaltAttnParams& p, cudaStream_t st) {
  if (p.D <= 0 || p.D > 256 || p.D % 8 != 0) return cudaErrorInvalidValue;
  switch ((p.D + 31) / 32) {
    case 1: return launch_simt<T, 1>(stage, p, st);
    case 2: return launch_simt<T, 2>(stage, p, st);
    case 3: return launch_simt<T, 3>(stage, p, st);
    case 4: return launch_simt<T, 4>(stage, p, st);
    case 5: return launch_simt<T, 5>(stage, p, st);
    case 6: return launch_simt<T, 6>(stage, p, st);
    case 7: return launch_simt<T, 7>(stage, p, st);
    case 8: return launch_simt<T, 8>(stage, p, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t simt_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st) {
  switch (p.dtype) {
    case DSALT_F16: return launch_simt_d<__half>(stage, p, st);
    case DSALT_BF16: return launch_simt_d<__nv_bfloat16>(stage, p, st);
    case DSALT_F32: return launch_simt_d<float>(stage, p, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace dsalt
