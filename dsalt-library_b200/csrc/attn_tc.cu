// tcgen05 / TMEM / TMA forward kernel of the DSALT attention for sm_100a.
//
// One CTA computes 128 query rows of one (sequence, head): the rows' landmark
// tile(s) and their band of keys [min_i(i − W_i), max_i i], in 128-key tiles.
//
//   warp 4      TMA producer: Q once, then K/V tiles into a 2-stage ring
//   warp 5      TMEM allocator + single-thread tcgen05.mma issuer:
//                 S[t%2] = Q·K_tᵀ (TMEM, fp32), then O += P_{t−1}·V_{t−1} (TMEM)
//   warps 0-3   softmax: thread r owns query row r (TMEM lane r): masks its row,
//               online softmax in the exp2 domain with a lazy rescale (the
//               running max only moves when it grows by more than 2^8), writes
//               P (bf16/fp16, 128B-swizzled K-major) to shared memory, applies
//               the soft window edge to its ≤ ceil(win_edge)+1 edge keys in place,
//               and finally normalises O and writes O, O(fp32) and LSE.
//
// Semantics follow the reference's _train_fwd_kernel
// (dsalt/kernels/dsalt_triton_train.py:116-214): band 0 ≤ d ≤ w̃, edge bias
// log σ((w̃ − d)/τ) outside the core d ≤ w̃ − win_edge, landmarks p ≤ i and
// float(p) < float(i) − w̃ with bias lmk_logw.  Inference is the same kernel with
// w̃ = w − 1 and no edge (row_window()).
//
// Every mbarrier wait is bounded (sm100::mbar_wait): a wait that runs out sets
// DSALT_DEV_WAIT_TIMEOUT in the status word and the CTA drains and exits.
#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {

cudaError_t simt_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st);
cudaError_t tc_bwd_stage(int stage, const DsaltAttnParams& p, float* lmk_scratch, cudaStream_t st);

namespace {

constexpr int BM = 128;              // query rows per CTA
constexpr int BN = 128;              // keys per tile
constexpr int kMaxLmk = 512;         // landmark slots held in shared memory
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

enum Bar {
  Q_FULL = 0, K_FULL = 1, V_FULL = 3, K_EMPTY = 5, V_EMPTY = 7, S_FULL = 9, S_EMPTY = 11, P_FULL = 13,
  O_DONE = 14, FINAL = 15, NUM_BARS = 16
};

template <int D>
struct alignas(1024) FwdSmem {
  uint8_t q[BM * D * 2];
  uint8_t k[2][BN * D * 2];
  uint8_t v[2][BN * D * 2];
  uint8_t p[BM * BN * 2];
  uint64_t bars[NUM_BARS];
  uint32_t tmem_base;
  int abort_flag;
  int band_lo, band_hi, cnt_max, n_valid;
  int lmk_pos[kMaxLmk];
  float lmk_lw2[kMaxLmk];
};

struct alignas(64) FwdArgs {
  CUtensorMap tm_q, tm_k, tm_v, tm_lk, tm_lv;
  DsaltAttnParams p;
  int lmk_box;  // rows of one landmark TMA box
};

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) tc_fwd_kernel(const __grid_constant__ FwdArgs a) {
  using namespace sm100;
  const DsaltAttnParams& p = a.p;
  const int blk = blockIdx.x;
  const int h = blockIdx.y;
  if (blk >= __ldg(p.num_blocks)) return;  // CTA-uniform, before any barrier or TMEM use
  const int s = __ldg(p.block_map + 2 * blk);
  const int mb = __ldg(p.block_map + 2 * blk + 1);
  const int64_t s0 = __ldg(p.cu_seqlens + s);
  const int L = (int)(__ldg(p.cu_seqlens + s + 1) - s0);
  const int m0 = mb * BM;

  extern __shared__ uint8_t smem_raw[];
  FwdSmem<D>& sm = *reinterpret_cast<FwdSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  constexpr bool kBF16 = sizeof(T) == 2 && !std::is_same<T, __half>::value;
  const BarArray bar{smem_u32(&sm.bars[0])};

  if (tid == 0) {
    mbar_init(bar[Q_FULL], 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar[K_FULL + st], 1);
      mbar_init(bar[V_FULL + st], 1);
      mbar_init(bar[K_EMPTY + st], 1);
      mbar_init(bar[V_EMPTY + st], 1);
      mbar_init(bar[S_FULL + st], 1);
      mbar_init(bar[S_EMPTY + st], BM);
    }
    mbar_init(bar[P_FULL], BM);
    mbar_init(bar[O_DONE], 1);
    mbar_init(bar[FINAL], 1);
    fence_mbar_init();
    sm.abort_flag = 0;
    sm.band_lo = INT_MAX;
    sm.band_hi = -1;
    sm.cnt_max = 0;
    sm.n_valid = 0;
  }
  if (warp == 4 && lane == 0) {
    prefetch_tmap(&a.tm_q);
    prefetch_tmap(&a.tm_k);
    prefetch_tmap(&a.tm_v);
  }
  if (warp == 5) tmem_alloc(smem_u32(&sm.tmem_base), 512);
  const int kp = p.kp;
  const int64_t lbase = ((int64_t)h * p.S + s) * kp;
  for (int c = tid; c < kp; c += kThreads) {
    const int ps = __ldg(p.pos_sorted + lbase + c);
    sm.lmk_pos[c] = ps;
    sm.lmk_lw2[c] = __ldg(p.w_sorted + lbase + c) * kLog2e;
    if (ps >= 0) atomicAdd(&sm.n_valid, 1);
  }
  __syncthreads();

  // ---- per-row window (threads 0..127 own rows m0 + tid)
  const int i = m0 + tid;
  const bool row_ok = tid < BM && i < L;
  RowWindow rw = {};
  int lo = INT_MAX, hi = -1, cnt = 0;
  if (row_ok) {
    rw = row_window(__ldg(p.w + s0 + i), i, p.semantics, p.win_edge);
    if (rw.W >= 0) {
      lo = i - min(rw.W, i);
      hi = i;
    }
    // landmarks valid for row i form a prefix of the sorted positions
    int a0 = 0, a1 = sm.n_valid;  // first index failing the predicate
    while (a0 < a1) {
      const int mid = (a0 + a1) >> 1;
      const int ps = sm.lmk_pos[mid];
      if (ps <= i && (float)ps < rw.win_lo) a0 = mid + 1; else a1 = mid;
    }
    cnt = a0;
    if (lo <= hi) {
      atomicMin(&sm.band_lo, lo);
      atomicMax(&sm.band_hi, hi);
    }
    if (cnt > 0) atomicMax(&sm.cnt_max, cnt);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int cnt_max = sm.cnt_max;
  const int band_lo = sm.band_lo, band_hi = sm.band_hi;
  const int n_lt = (cnt_max + BN - 1) / BN;
  const int n_bt = band_hi >= band_lo ? (band_hi - band_lo + BN) / BN : 0;
  const int n_tiles = n_lt + n_bt;
  volatile int* abort_flag = &sm.abort_flag;
  // tile t: landmark tile (t < n_lt) or band tile starting at key band_lo + BN*(t - n_lt)
  auto tile_n = [&](int t) -> int {
    if (t < n_lt) return round16(min(BN, cnt_max - BN * t));
    return round16(min(BN, band_hi - (band_lo + BN * (t - n_lt)) + 1));
  };
  const uint32_t tS = tmem;            // S buffers: columns [0,128) and [128,256)
  const uint32_t tO = tmem + 2 * BN;   // O: columns [256, 256 + D)

  if (warp == 4) {
    // ------------------------------------------------------------ producers
    // lane 0: Q, then K tiles (a K stage frees as soon as its S = Q·Kᵀ is done);
    // lane 1: V tiles (a V stage frees when its P·V is done).
    if (lane < 2 && n_tiles > 0) {
      const bool is_k = lane == 0;
      if (is_k) {
        mbar_expect_tx(bar[Q_FULL], BM * D * 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(smem_u32(sm.q + c * (BM * 128)), &a.tm_q, bar[Q_FULL], c * 64, h, (int)(s0 + m0));
      }
      const int FULL = is_k ? K_FULL : V_FULL, EMPTY = is_k ? K_EMPTY : V_EMPTY;
      int issued = 0;
      for (int t = 0; t < n_tiles; ++t) {
        const int st = t & 1;
        if (t >= 2 && !mbar_wait(bar[EMPTY + st], ((t >> 1) - 1) & 1, abort_flag, p.status)) break;
        const bool lmk = t < n_lt;
        mbar_expect_tx(bar[FULL + st], (lmk ? a.lmk_box : BN) * D * 2);
        uint8_t* dst = is_k ? sm.k[st] : sm.v[st];
        const CUtensorMap* map = lmk ? (is_k ? &a.tm_lk : &a.tm_lv) : (is_k ? &a.tm_k : &a.tm_v);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          if (lmk) tma_load_3d(smem_u32(dst + c * (BN * 128)), map, bar[FULL + st], c * 64, BN * t, h * p.S + s);
          else tma_load_3d(smem_u32(dst + c * (BN * 128)), map, bar[FULL + st], c * 64, h,
                           (int)(s0 + band_lo + BN * (t - n_lt)));
        }
        issued = t + 1;
      }
      // drain: never leave a TMA write in flight into shared memory
      for (int t = max(0, issued - 2); t < issued; ++t) mbar_drain(bar[FULL + (t & 1)], (t >> 1) & 1);
      if (is_k) mbar_drain(bar[Q_FULL], 0);
    }
  } else if (warp == 5) {
    // ------------------------------------------------------------ MMA issuer
    // order: S_0, S_1, then for every t: P_t·V_t as soon as P_t is ready, then S_{t+2}
    if (lane == 0 && n_tiles > 0) {
      const uint32_t id_o = idesc_f16(kBF16, BM, D, false, true);
      const uint32_t q_addr = smem_u32(sm.q);
      const uint32_t p_addr = smem_u32(sm.p);
      bool ok = mbar_wait(bar[Q_FULL], 0, abort_flag, p.status);
      auto issue_s = [&](int t) -> bool {
        const int st = t & 1;
        if (!mbar_wait(bar[K_FULL + st], (t >> 1) & 1, abort_flag, p.status)) return false;
        if (t >= 2 && !mbar_wait(bar[S_EMPTY + st], ((t >> 1) - 1) & 1, abort_flag, p.status)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_u32(sm.k[st]);
        const uint32_t id_s = idesc_f16(kBF16, BM, tile_n(t), false, false);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(q_addr + off, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
          mma_f16(tS + st * BN, ad, bd, id_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(bar[S_FULL + st]);
        mma_commit(bar[K_EMPTY + st]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n_tiles > 1) ok = issue_s(1);
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int st = t & 1;
        if (!mbar_wait(bar[P_FULL], t & 1, abort_flag, p.status)) { ok = false; break; }
        if (!mbar_wait(bar[V_FULL + st], (t >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sm.v[st]);
        const int nk = tile_n(t) / 16;
        for (int kk = 0; kk < nk; ++kk) {
          const uint64_t ad = sdesc_sw128(p_addr + (kk >> 2) * (BM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, BN * 128, 1024);
          mma_f16(tO, ad, bd, id_o, (t > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar[O_DONE]);
        mma_commit(bar[V_EMPTY + st]);
        if (t + 2 < n_tiles && !issue_s(t + 2)) { ok = false; break; }
      }
      // drain: every issued MMA completes before TMEM is released
      mma_commit(bar[FINAL]);
      mbar_drain(bar[FINAL], 0);
    }
  } else {
    // ------------------------------------------------------------ softmax (rows)
    const int r = tid;
    const uint32_t lane_addr = ((uint32_t)(warp * 32) << 16);
    const float sl2 = p.scale * kLog2e;
    const float inv_tau = 1.0f / p.tau_win;
    // edge keys of this row: d in [d_e0, min(W, i)] (soft-edge bias), empty when d_e0 > W
    int d_e0 = INT_MAX;
    if (row_ok && rw.W >= 0) d_e0 = max((int)floorf(rw.core) + 1, 0);
    float m = -INFINITY, l = 0.f;
    bool ok = true;
    uint8_t* sp = sm.p;
    for (int t = 0; t < n_tiles; ++t) {
      const int st = t & 1;
      ok = mbar_wait(bar[S_FULL + st], (t >> 1) & 1, abort_flag, p.status);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const int N = tile_n(t);
      // all 128 columns are read: columns past N hold stale values and are masked below
      float x[BN];
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch) tmem_ld32(tS + lane_addr + st * BN + ch * 32, x + ch * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar[S_EMPTY + st]);

      const bool lmk = t < n_lt;
      float xs;  // multiplier applied inside exp2
      int n0 = 0;
      float mx[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) mx[g] = -INFINITY;
      if (lmk) {
        const int climit = cnt - BN * t;
        const float* lw2 = sm.lmk_lw2 + BN * t;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          x[c] = (c < climit) ? fmaf(x[c], sl2, lw2[c]) : -INFINITY;
          mx[c & 7] = fmaxf(mx[c & 7], x[c]);
        }
        xs = 1.0f;
      } else {
        n0 = band_lo + BN * (t - n_lt);
        const int clo = lo - n0, chi = hi - n0;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          x[c] = (c >= clo && c <= chi) ? x[c] : -INFINITY;
          mx[c & 7] = fmaxf(mx[c & 7], x[c]);
        }
        xs = sl2;
      }
      float mt = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])), fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7])));
      if (!lmk) mt *= sl2;
      const float m_new = fmaxf(m, mt);
      bool rescale = false;
      float factor = 1.0f;
      if (m == -INFINITY) {
        m = m_new;
      } else if (m_new > m + kRescaleThreshold) {
        factor = exp2f(m - m_new);
        m = m_new;
        rescale = true;
      }
      const float ms = (m == -INFINITY) ? 0.f : m;
      float sm8[8];
#pragma unroll
      for (int g = 0; g < 8; ++g) sm8[g] = 0.f;
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        x[c] = fast_exp2(fmaf(x[c], xs, -ms));
        sm8[c & 7] += x[c];
      }
      const float sum = ((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7]));
      l = l * factor + sum;

      // P buffer and O are free once the previous P·V has completed
      if (t >= 1) {
        ok = mbar_wait(bar[O_DONE], (t - 1) & 1, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
      }
      if (__any_sync(0xffffffffu, rescale && t >= 1)) {
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch) {
          float o[32];
          tmem_ld32(tO + lane_addr + ch * 32, o);
          tmem_wait_ld();
          const float f = (rescale && t >= 1) ? factor : 1.0f;
#pragma unroll
          for (int j = 0; j < 32; ++j) o[j] *= f;
          tmem_st32(tO + lane_addr + ch * 32, o);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c8 = 0; c8 < BN / 8; ++c8) {
        const int c = c8 * 8;
        uint4 u;
        u.x = pack2(x[c + 0], x[c + 1], kBF16);
        u.y = pack2(x[c + 2], x[c + 3], kBF16);
        u.z = pack2(x[c + 4], x[c + 5], kBF16);
        u.w = pack2(x[c + 6], x[c + 7], kBF16);
        *reinterpret_cast<uint4*>(sp + (c >> 6) * (BM * 128) + sw128_offset(r, c & 63)) = u;
      }
      if (!lmk && row_ok && d_e0 <= rw.W) {
        // soft window edge on this row's edge keys inside the tile: p *= σ((w̃ − d)/τ)
        const int d_hi = min(min(rw.W, i), i - n0);
        const int d_lo = max(d_e0, i - (n0 + N - 1));
        for (int d = d_lo; d <= d_hi; ++d) {
          const int c = i - d - n0;
          T* e = reinterpret_cast<T*>(sp + (c >> 6) * (BM * 128) + sw128_offset(r, c & 63));
          const float pv = to_f32<T>(*e);
          const float z = (rw.wt - (float)d) * inv_tau;
          const float sg = 1.0f / (1.0f + expf(-z));
          *e = from_f32<T>(pv * sg);
          l -= pv * (1.0f - sg);
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(bar[P_FULL]);
    }
    // ---- epilogue: O / l, LSE
    if (ok && n_tiles > 0) {
      ok = mbar_wait(bar[O_DONE], (n_tiles - 1) & 1, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
    }
    const bool nonempty = ok && l > 1e-9f && n_tiles > 0;
    const float inv_l = nonempty ? 1.0f / l : 0.f;
    const int64_t row_off = (s0 + i) * (int64_t)p.H * D + (int64_t)h * D;
    T* og = reinterpret_cast<T*>(p.o) + row_off;
    float* of = p.o_f32 ? p.o_f32 + row_off : nullptr;
#pragma unroll
    for (int ch = 0; ch < D / 32; ++ch) {
      float o[32];
      if (ok && n_tiles > 0) {
        tmem_ld32(tO + lane_addr + ch * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0.f;
      }
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float rv[8];
#pragma unroll
          for (int e = 0; e < 8; ++e) rv[e] = round_to<T>(o[j + e] * inv_l);
          uint4 u;
          u.x = pack2(rv[0], rv[1], kBF16);
          u.y = pack2(rv[2], rv[3], kBF16);
          u.z = pack2(rv[4], rv[5], kBF16);
          u.w = pack2(rv[6], rv[7], kBF16);
          *reinterpret_cast<uint4*>(og + ch * 32 + j) = u;
          if (of) {
            *reinterpret_cast<float4*>(of + ch * 32 + j) = make_float4(rv[0], rv[1], rv[2], rv[3]);
            *reinterpret_cast<float4*>(of + ch * 32 + j + 4) = make_float4(rv[4], rv[5], rv[6], rv[7]);
          }
        }
      }
    }
    if (row_ok) p.lse[(s0 + i) * p.H + h] = nonempty ? (m + log2f(l)) * kLn2 : -INFINITY;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 512);
}

// ---------------------------------------------------------------- host side
CUresult encode_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                   uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2) {
  return encode_tensor_map_3d(m, dt, base, d0, d1, d2, stride1_bytes, stride2_bytes, box0, box1, box2);
}

template <typename T, int D>
cudaError_t launch_tc_fwd(const DsaltAttnParams& p, cudaStream_t stream) {
  FwdArgs a;
  memset(&a, 0, sizeof(a));
  a.p = p;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t row = (uint64_t)D * 2;
  const uint64_t trow = (uint64_t)p.H * D * 2;
  if (encode_3d(&a.tm_q, dt, p.q, D, p.H, p.T, row, trow, 64, 1, BM) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_3d(&a.tm_k, dt, p.k, D, p.H, p.T, row, trow, 64, 1, BN) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_3d(&a.tm_v, dt, p.v, D, p.H, p.T, row, trow, 64, 1, BN) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const int kp = p.kp > 0 ? p.kp : 16;
  a.lmk_box = kp < BN ? kp : BN;
  const void* lk = p.kp > 0 ? p.lmk_k : p.k;  // any valid address when there are no landmarks
  const void* lv = p.kp > 0 ? p.lmk_v : p.v;
  const uint64_t hs = p.kp > 0 ? (uint64_t)p.H * p.S : 1;
  if (encode_3d(&a.tm_lk, dt, lk, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  if (encode_3d(&a.tm_lv, dt, lv, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const size_t smem = sizeof(FwdSmem<D>) + 1024;
  cudaError_t e = cudaFuncSetAttribute(tc_fwd_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)p.max_blocks, (unsigned)p.H);
  tc_fwd_kernel<T, D><<<grid, kThreads, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool tc_supported(const DsaltAttnParams& p) {
  return (p.dtype == DSALT_BF16 || p.dtype == DSALT_F16) && (p.D == 64 || p.D == 128) && p.kp <= kMaxLmk &&
         p.T < (1ll << 31) && p.max_blocks > 0;
}

// stage 0 forward, 1 Delta (bandwidth-bound, SIMT), 2 dK/dV, 3 dQ (+ d_w̃)
cudaError_t tc_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st) {
  if (stage == 1) return simt_attention_stage(stage, p, st);
  if (stage != 0) return tc_bwd_stage(stage, p, p.lmk_grad, st);
  if (p.dtype == DSALT_BF16) {
    if (p.D == 64) return launch_tc_fwd<__nv_bfloat16, 64>(p, st);
    return launch_tc_fwd<__nv_bfloat16, 128>(p, st);
  }
  if (p.D == 64) return launch_tc_fwd<__half, 64>(p, st);
  return launch_tc_fwd<__half, 128>(p, st);
}

}  // namespace dsalt
