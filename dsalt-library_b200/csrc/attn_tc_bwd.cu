// tcgen05 / TMEM / TMA backward kernels of the DSALT attention for sm_100a.
//
// dQ (query-parallel, reference _train_bwd_kernel dsalt_triton_train.py:240-383):
//   one CTA = 128 query rows of one (sequence, head); 64-key tiles (landmark
//   tiles first, then the rows' band).  Per tile the MMA warp computes
//   S = Q·Kᵀ and dP = dO·Vᵀ into TMEM (double buffered); the softmax warps form
//   P = exp(S·scale + bias − LSE) and dS = P·(dP − Δ) row by row, apply the soft
//   window edge to their ≤ ceil(win_edge)+1 edge keys (and accumulate
//   ∂loss/∂w̃ from them), and write dS to shared memory; the MMA warp then adds
//   dQ += dS·K in TMEM.
//
// dK/dV (key-parallel, atomic-free; reference _train_bwd_dkdv_kernel :386-481 and
//   the landmark atomics of :302-333):
//   one CTA = 128 keys and the 64-query tiles that can attend them.  Per tile:
//   Sᵀ = K·Qᵀ, dPᵀ = V·dOᵀ (TMEM), then Pᵀ, dSᵀ (shared memory) and
//   dV += Pᵀ·dO, dK += dSᵀ·Q (TMEM).  Two passes: landmark items (the sorted
//   landmark slots of one (head, sequence) as the 128 "keys", every later query
//   as columns) write fp32 dK/dV per slot and d_lw (a row sum, no atomics);
//   band items (128 consecutive keys) then add those slot rows into their
//   own dK/dV before the single store.  The backward is therefore deterministic.
//
// All waits are bounded (sm100::mbar_wait); see attn_tc.cu.
#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {

cudaError_t simt_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st);

namespace bwd {

constexpr int kThreads = 192;
constexpr int kMaxLmk = 512;
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

struct alignas(64) BwdArgs {
  CUtensorMap tm_q, tm_do, tm_k, tm_v, tm_lk, tm_lv;
  DsaltAttnParams p;
  float* dk_lmk;  // [H,S,kp,D] fp32 scratch: landmark-slot dK / dV
  float* dv_lmk;
  int lmk_box;    // rows of one landmark TMA box
};

// ======================================================================= dQ
namespace dq {
constexpr int BM = 128, BN = 64;
enum { QD_FULL = 0, K_FULL = 1, V_FULL = 3, KV_EMPTY = 5, SD_FULL = 7, SD_EMPTY = 9, DS_FULL = 11, DS_EMPTY = 13,
       DQ_DONE = 15, FINAL = 16, NB = 17 };

template <int D>
struct alignas(1024) Smem {
  uint8_t q[BM * D * 2];
  uint8_t dO[BM * D * 2];
  uint8_t k[2][BN * D * 2];
  uint8_t v[2][BN * D * 2];
  uint8_t ds[2][BM * BN * 2];
  uint64_t bars[NB];
  uint32_t tmem_base;
  int abort_flag, band_lo, band_hi, cnt_max, n_valid;
  int lmk_pos[kMaxLmk];
  float lmk_lw2[kMaxLmk];
};

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) tc_bwd_dq_kernel(const __grid_constant__ BwdArgs a) {
  using namespace sm100;
  const DsaltAttnParams& p = a.p;
  const int blk = blockIdx.x, h = blockIdx.y;
  if (blk >= __ldg(p.num_blocks)) return;
  const int s = __ldg(p.block_map + 2 * blk);
  const int64_t s0 = __ldg(p.cu_seqlens + s);
  const int L = (int)(__ldg(p.cu_seqlens + s + 1) - s0);
  const int m0 = __ldg(p.block_map + 2 * blk + 1) * BM;
  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBF16 = !std::is_same<T, __half>::value;
  const BarArray bar{smem_u32(&sm.bars[0])};
  if (tid == 0) {
    mbar_init(bar[QD_FULL], 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar[K_FULL + st], 1);
      mbar_init(bar[V_FULL + st], 1);
      mbar_init(bar[KV_EMPTY + st], 1);
      mbar_init(bar[SD_FULL + st], 1);
      mbar_init(bar[SD_EMPTY + st], BM);
      mbar_init(bar[DS_FULL + st], BM);
      mbar_init(bar[DS_EMPTY + st], 1);
    }
    mbar_init(bar[DQ_DONE], 1);
    mbar_init(bar[FINAL], 1);
    fence_mbar_init();
    sm.abort_flag = 0;
    sm.band_lo = INT_MAX;
    sm.band_hi = -1;
    sm.cnt_max = 0;
    sm.n_valid = 0;
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
  const int i = m0 + tid;
  const bool row_ok = tid < BM && i < L;
  RowWindow rw = {};
  int lo = INT_MAX, hi = -1, cnt = 0;
  float lse2 = -INFINITY, delta = 0.f;
  if (row_ok) {
    const int64_t row = (s0 + i) * p.H + h;
    lse2 = __ldg(p.lse + row) * kLog2e;
    delta = __ldg(p.delta + row);
    rw = row_window(__ldg(p.w + s0 + i), i, p.semantics, p.win_edge);
    if (rw.W >= 0) { lo = i - min(rw.W, i); hi = i; }
    int a0 = 0, a1 = sm.n_valid;
    while (a0 < a1) {
      const int mid = (a0 + a1) >> 1;
      const int ps = sm.lmk_pos[mid];
      if (ps <= i && (float)ps < rw.win_lo) a0 = mid + 1; else a1 = mid;
    }
    cnt = a0;
    if (lse2 == -INFINITY) { lo = INT_MAX; hi = -1; cnt = 0; }  // empty row: no gradient
    if (lo <= hi) { atomicMin(&sm.band_lo, lo); atomicMax(&sm.band_hi, hi); }
    if (cnt > 0) atomicMax(&sm.cnt_max, cnt);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  const int cnt_max = sm.cnt_max, band_lo = sm.band_lo, band_hi = sm.band_hi;
  const int n_lt = (cnt_max + BN - 1) / BN;
  const int n_bt = band_hi >= band_lo ? (band_hi - band_lo + BN) / BN : 0;
  const int n_tiles = n_lt + n_bt;
  volatile int* abort_flag = &sm.abort_flag;
  auto tile_n = [&](int t) -> int {
    if (t < n_lt) return round16(min(BN, cnt_max - BN * t));
    return round16(min(BN, band_hi - (band_lo + BN * (t - n_lt)) + 1));
  };
  const uint32_t tS = tmem, tdP = tmem + 2 * BN, tdQ = tmem + 4 * BN;

  if (warp == 4) {
    if (lane == 0 && n_tiles > 0) {
      mbar_expect_tx(bar[QD_FULL], 2 * BM * D * 2);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        tma_load_3d(smem_u32(sm.q + c * (BM * 128)), &a.tm_q, bar[QD_FULL], c * 64, h, (int)(s0 + m0));
        tma_load_3d(smem_u32(sm.dO + c * (BM * 128)), &a.tm_do, bar[QD_FULL], c * 64, h, (int)(s0 + m0));
      }
      int issued = 0;
      for (int t = 0; t < n_tiles; ++t) {
        const int st = t & 1;
        if (t >= 2 && !mbar_wait(bar[KV_EMPTY + st], ((t >> 1) - 1) & 1, abort_flag, p.status)) break;
        const bool lmk = t < n_lt;
        const uint32_t bytes = (lmk ? a.lmk_box : BN) * D * 2;
        const int z = (int)(s0 + band_lo + BN * (t - n_lt));
        mbar_expect_tx(bar[K_FULL + st], bytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          if (lmk) tma_load_3d(smem_u32(sm.k[st] + c * (BN * 128)), &a.tm_lk, bar[K_FULL + st], c * 64, BN * t, h * p.S + s);
          else tma_load_3d(smem_u32(sm.k[st] + c * (BN * 128)), &a.tm_k, bar[K_FULL + st], c * 64, h, z);
        }
        mbar_expect_tx(bar[V_FULL + st], bytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          if (lmk) tma_load_3d(smem_u32(sm.v[st] + c * (BN * 128)), &a.tm_lv, bar[V_FULL + st], c * 64, BN * t, h * p.S + s);
          else tma_load_3d(smem_u32(sm.v[st] + c * (BN * 128)), &a.tm_v, bar[V_FULL + st], c * 64, h, z);
        }
        issued = t + 1;
      }
      for (int t = max(0, issued - 2); t < issued; ++t) {
        mbar_drain(bar[K_FULL + (t & 1)], (t >> 1) & 1);
        mbar_drain(bar[V_FULL + (t & 1)], (t >> 1) & 1);
      }
      mbar_drain(bar[QD_FULL], 0);
    }
  } else if (warp == 5) {
    if (lane == 0 && n_tiles > 0) {
      const uint32_t id_dq = idesc_f16(kBF16, BM, D, false, true);
      const uint32_t q_addr = smem_u32(sm.q), do_addr = smem_u32(sm.dO);
      bool ok = mbar_wait(bar[QD_FULL], 0, abort_flag, p.status);
      auto issue_dq = [&](int tp) -> bool {
        const int st = tp & 1;
        if (!mbar_wait(bar[DS_FULL + st], (tp >> 1) & 1, abort_flag, p.status)) return false;
        tc_fence_after();
        const uint32_t ds_addr = smem_u32(sm.ds[st]), k_addr = smem_u32(sm.k[st]);
        const int nk = tile_n(tp) / 16;
        for (int kk = 0; kk < nk; ++kk) {
          const uint64_t ad = sdesc_sw128(ds_addr + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(k_addr + kk * 2048, BN * 128, 1024);
          mma_f16(tdQ, ad, bd, id_dq, (tp > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar[DS_EMPTY + st]);
        mma_commit(bar[KV_EMPTY + st]);
        return true;
      };
      for (int t = 0; ok && t < n_tiles; ++t) {
        const int st = t & 1;
        if (!mbar_wait(bar[K_FULL + st], (t >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        if (!mbar_wait(bar[V_FULL + st], (t >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        if (t >= 2 && !mbar_wait(bar[SD_EMPTY + st], ((t >> 1) - 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t id_s = idesc_f16(kBF16, BM, tile_n(t), false, false);
        const uint32_t k_addr = smem_u32(sm.k[st]), v_addr = smem_u32(sm.v[st]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t boff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_f16(tS + st * BN, sdesc_sw128(q_addr + aoff, 16, 1024), sdesc_sw128(k_addr + boff, 16, 1024), id_s,
                  kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t boff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_f16(tdP + st * BN, sdesc_sw128(do_addr + aoff, 16, 1024), sdesc_sw128(v_addr + boff, 16, 1024), id_s,
                  kk > 0 ? 1u : 0u);
        }
        mma_commit(bar[SD_FULL + st]);
        if (t >= 1 && !issue_dq(t - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_dq(n_tiles - 1);
      mma_commit(bar[DQ_DONE]);
      mma_commit(bar[FINAL]);
      mbar_drain(bar[FINAL], 0);
    }
  } else {
    const int r = tid;
    const uint32_t lane_addr = ((uint32_t)(warp * 32) << 16);
    const float sl2 = p.scale * kLog2e;
    const float inv_tau = 1.0f / p.tau_win;
    int d_e0 = INT_MAX;
    if (row_ok && rw.W >= 0) d_e0 = max((int)floorf(rw.core) + 1, 0);
    float dw = 0.f;
    bool ok = true;
    for (int t = 0; t < n_tiles; ++t) {
      const int st = t & 1;
      ok = mbar_wait(bar[SD_FULL + st], (t >> 1) & 1, abort_flag, p.status);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      const int N = tile_n(t);
      float sv[BN], dpv[BN];
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch) {
        if (ch * 32 < N) {
          tmem_ld32(tS + lane_addr + st * BN + ch * 32, sv + ch * 32);
          tmem_ld32(tdP + lane_addr + st * BN + ch * 32, dpv + ch * 32);
        }
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar[SD_EMPTY + st]);
      const bool lmk = t < n_lt;
      const int n0 = lmk ? 0 : band_lo + BN * (t - n_lt);
      if (lmk) {
        const int climit = cnt - BN * t;
        const float* lw2 = sm.lmk_lw2 + BN * t;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          if (c < N) {
            const float pr = (c < climit) ? fast_exp2(fmaf(sv[c], sl2, lw2[c] - lse2)) : 0.f;
            sv[c] = pr * (dpv[c] - delta);
          }
        }
      } else {
        const int clo = lo - n0, chi = hi - n0;
#pragma unroll
        for (int c = 0; c < BN; ++c) {
          if (c < N) {
            const float pr = (c >= clo && c <= chi) ? fast_exp2(fmaf(sv[c], sl2, -lse2)) : 0.f;
            sv[c] = pr * (dpv[c] - delta);
          }
        }
      }
      if (t >= 2) {
        ok = mbar_wait(bar[DS_EMPTY + st], ((t >> 1) - 1) & 1, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      }
      uint8_t* dsb = sm.ds[st];
#pragma unroll
      for (int c8 = 0; c8 < BN / 8; ++c8) {
        if (c8 * 8 < N) {
          const int c = c8 * 8;
          uint4 u;
          u.x = pack2(sv[c + 0], sv[c + 1], kBF16);
          u.y = pack2(sv[c + 2], sv[c + 3], kBF16);
          u.z = pack2(sv[c + 4], sv[c + 5], kBF16);
          u.w = pack2(sv[c + 6], sv[c + 7], kBF16);
          *reinterpret_cast<uint4*>(dsb + sw128_offset(r, c)) = u;
        }
      }
      if (!lmk && row_ok && lo <= hi && d_e0 <= rw.W) {
        // soft window edge: P and dS scale by σ((w̃ − d)/τ); ∂loss/∂w̃ += dS·(1 − σ)/τ
        const int d_hi = min(min(rw.W, i), i - n0);
        const int d_lo = max(d_e0, i - (n0 + N - 1));
        for (int d = d_lo; d <= d_hi; ++d) {
          const int c = i - d - n0;
          T* e = reinterpret_cast<T*>(dsb + sw128_offset(r, c));
          const float z = (rw.wt - (float)d) * inv_tau;
          const float sg = 1.0f / (1.0f + expf(-z));
          const float dsb_v = to_f32<T>(*e) * sg;
          *e = from_f32<T>(dsb_v);
          dw = fmaf(dsb_v, (1.0f - sg) * inv_tau, dw);
        }
      }
      fence_async_smem();
      mbar_arrive(bar[DS_FULL + st]);
    }
    if (ok && n_tiles > 0) {
      ok = mbar_wait(bar[DQ_DONE], 0, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
    }
    const int64_t row_off = (s0 + i) * (int64_t)p.H * D + (int64_t)h * D;
    T* dq = reinterpret_cast<T*>(p.dq) + row_off;
#pragma unroll
    for (int ch = 0; ch < D / 32; ++ch) {
      float o[32];
      if (ok && n_tiles > 0) {
        tmem_ld32(tdQ + lane_addr + ch * 32, o);
        tmem_wait_ld();
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 0.f;
      }
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 u;
          u.x = pack2(o[j + 0] * p.scale, o[j + 1] * p.scale, kBF16);
          u.y = pack2(o[j + 2] * p.scale, o[j + 3] * p.scale, kBF16);
          u.z = pack2(o[j + 4] * p.scale, o[j + 5] * p.scale, kBF16);
          u.w = pack2(o[j + 6] * p.scale, o[j + 7] * p.scale, kBF16);
          *reinterpret_cast<uint4*>(dq + ch * 32 + j) = u;
        }
      }
    }
    if (row_ok && p.dw_head) p.dw_head[(s0 + i) * p.H + h] = ok ? dw : 0.f;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 512);
}
}  // namespace dq

// ==================================================================== dK / dV
namespace dkv {
constexpr int BM = 128, BN = 64;  // BM keys (TMEM lanes), BN queries per tile
enum { KV_FULL = 0, Q_FULL = 1, DO_FULL = 3, QDO_EMPTY = 5, SD_FULL = 7, SD_EMPTY = 9, PDS_FULL = 11,
       PDS_EMPTY = 13, KV_DONE = 15, FINAL = 16, ROWS_DONE = 17, NB = 18 };

template <int D>
struct alignas(1024) Smem {
  uint8_t k[BM * D * 2];
  uint8_t v[BM * D * 2];
  uint8_t q[2][BN * D * 2];
  uint8_t dO[2][BN * D * 2];
  uint8_t pt[2][BM * BN * 2];
  uint8_t dst[2][BM * BN * 2];
  uint64_t bars[NB];
  uint32_t tmem_base;
  int abort_flag;
  // per query column of the current / next tile
  float c_lse2[2][BN], c_delta[2][BN], c_wt[2][BN], c_wlo[2][BN];
  int c_lo[2][BN], c_i[2][BN], c_ehi[2][BN];
};

// Column data of query q (sequence position) for head h.
struct ColInfo {
  float lse2, delta, wt, wlo;
  int lo, i, ehi;  // band start of the query, its position, last edge key (< lo: no edge)
};

template <bool LMK, typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) tc_bwd_dkdv_kernel(const __grid_constant__ BwdArgs a) {
  using namespace sm100;
  const DsaltAttnParams& p = a.p;
  const int h = blockIdx.y;
  int s, key0, nkeys, q_start;
  int64_t s0;
  int L;
  int64_t lbase = 0;
  if (LMK) {
    // item = (h, s, chunk of 128 sorted landmark slots)
    const int nch = (p.kp + BM - 1) / BM;
    s = blockIdx.x / nch;
    const int chunk = blockIdx.x % nch;
    s0 = __ldg(p.cu_seqlens + s);
    L = (int)(__ldg(p.cu_seqlens + s + 1) - s0);
    lbase = ((int64_t)h * p.S + s) * p.kp;
    key0 = chunk * BM;
    int nv = 0;  // valid slots of this chunk
    while (key0 + nv < p.kp && nv < BM && __ldg(p.pos_sorted + lbase + key0 + nv) >= 0) ++nv;
    nkeys = nv;
    if (nkeys == 0) return;
    q_start = __ldg(p.pos_sorted + lbase + key0);
  } else {
    if ((int)blockIdx.x >= __ldg(p.num_blocks)) return;
    s = __ldg(p.block_map + 2 * blockIdx.x);
    s0 = __ldg(p.cu_seqlens + s);
    L = (int)(__ldg(p.cu_seqlens + s + 1) - s0);
    key0 = __ldg(p.block_map + 2 * blockIdx.x + 1) * BM;
    nkeys = min(BM, L - key0);
    q_start = key0;
    lbase = ((int64_t)h * p.S + s) * p.kp;
  }
  const int q_end = LMK ? L - 1 : min(L - 1, key0 + BM - 1 + max(__ldg(p.seq_wmax + s), 0));
  const int n_tiles = q_end >= q_start ? (q_end - q_start + BN) / BN : 0;

  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBF16 = !std::is_same<T, __half>::value;
  const BarArray bar{smem_u32(&sm.bars[0])};
  if (tid == 0) {
    mbar_init(bar[KV_FULL], 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar[Q_FULL + st], 1);
      mbar_init(bar[DO_FULL + st], 1);
      mbar_init(bar[QDO_EMPTY + st], 1);
      mbar_init(bar[SD_FULL + st], 1);
      mbar_init(bar[SD_EMPTY + st], BM);
      mbar_init(bar[PDS_FULL + st], BM);
      mbar_init(bar[PDS_EMPTY + st], 1);
    }
    mbar_init(bar[KV_DONE], 1);
    mbar_init(bar[FINAL], 1);
    mbar_init(bar[ROWS_DONE], BM);
    fence_mbar_init();
    sm.abort_flag = 0;
  }
  if (warp == 5) tmem_alloc(smem_u32(&sm.tmem_base), 512);
  const float inv_tau = 1.0f / p.tau_win;
  auto col_info = [&](int q) -> ColInfo {
    ColInfo ci;
    ci.i = q;
    ci.lse2 = -INFINITY; ci.delta = 0.f; ci.wt = 0.f; ci.wlo = -INFINITY; ci.lo = INT_MAX; ci.ehi = INT_MIN;
    if (q >= 0 && q < L) {
      const int64_t row = (s0 + q) * p.H + h;
      ci.lse2 = __ldg(p.lse + row) * kLog2e;
      ci.delta = __ldg(p.delta + row);
      const RowWindow rw = row_window(__ldg(p.w + s0 + q), q, p.semantics, p.win_edge);
      ci.wt = rw.wt;
      ci.wlo = rw.win_lo;
      if (rw.W >= 0 && ci.lse2 != -INFINITY) {
        ci.lo = q - min(rw.W, q);
        const int d_e0 = max((int)floorf(rw.core) + 1, 0);
        ci.ehi = d_e0 <= rw.W ? q - d_e0 : INT_MIN;
      }
      if (ci.lse2 == -INFINITY) ci.wlo = -INFINITY;  // empty rows take no landmark gradient either
    }
    return ci;
  };
  auto store_col = [&](int buf, int c, const ColInfo& ci) {
    sm.c_lse2[buf][c] = ci.lse2; sm.c_delta[buf][c] = ci.delta; sm.c_wt[buf][c] = ci.wt; sm.c_wlo[buf][c] = ci.wlo;
    sm.c_lo[buf][c] = ci.lo; sm.c_i[buf][c] = ci.i; sm.c_ehi[buf][c] = ci.ehi;
  };
  if (tid < BN && n_tiles > 0) store_col(0, tid, col_info(q_start + tid));
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  const uint32_t tS = tmem, tdP = tmem + 2 * BN, tdK = tmem + 4 * BN, tdV = tmem + 4 * BN + D;
  auto tile_n = [&](int u) -> int { return round16(min(BN, q_end - (q_start + BN * u) + 1)); };

  if (warp == 4) {
    if (lane == 0 && n_tiles > 0) {
      const uint32_t kv_bytes = (LMK ? a.lmk_box : BM) * D * 2;
      mbar_expect_tx(bar[KV_FULL], 2 * kv_bytes);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {
        if (LMK) {
          tma_load_3d(smem_u32(sm.k + c * (BM * 128)), &a.tm_lk, bar[KV_FULL], c * 64, key0, h * p.S + s);
          tma_load_3d(smem_u32(sm.v + c * (BM * 128)), &a.tm_lv, bar[KV_FULL], c * 64, key0, h * p.S + s);
        } else {
          tma_load_3d(smem_u32(sm.k + c * (BM * 128)), &a.tm_k, bar[KV_FULL], c * 64, h, (int)(s0 + key0));
          tma_load_3d(smem_u32(sm.v + c * (BM * 128)), &a.tm_v, bar[KV_FULL], c * 64, h, (int)(s0 + key0));
        }
      }
      int issued = 0;
      for (int u = 0; u < n_tiles; ++u) {
        const int st = u & 1;
        if (u >= 2 && !mbar_wait(bar[QDO_EMPTY + st], ((u >> 1) - 1) & 1, abort_flag, p.status)) break;
        const int z = (int)(s0 + q_start + BN * u);
        mbar_expect_tx(bar[Q_FULL + st], BN * D * 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(smem_u32(sm.q[st] + c * (BN * 128)), &a.tm_q, bar[Q_FULL + st], c * 64, h, z);
        mbar_expect_tx(bar[DO_FULL + st], BN * D * 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(smem_u32(sm.dO[st] + c * (BN * 128)), &a.tm_do, bar[DO_FULL + st], c * 64, h, z);
        issued = u + 1;
      }
      for (int u = max(0, issued - 2); u < issued; ++u) {
        mbar_drain(bar[Q_FULL + (u & 1)], (u >> 1) & 1);
        mbar_drain(bar[DO_FULL + (u & 1)], (u >> 1) & 1);
      }
      mbar_drain(bar[KV_FULL], 0);
    }
  } else if (warp == 5) {
    if (lane == 0 && n_tiles > 0) {
      const uint32_t id_s = idesc_f16(kBF16, BM, BN, false, false);
      const uint32_t id_kv = idesc_f16(kBF16, BM, D, false, true);
      const uint32_t k_addr = smem_u32(sm.k), v_addr = smem_u32(sm.v);
      bool ok = mbar_wait(bar[KV_FULL], 0, abort_flag, p.status);
      auto issue_kv = [&](int up) -> bool {
        const int st = up & 1;
        if (!mbar_wait(bar[PDS_FULL + st], (up >> 1) & 1, abort_flag, p.status)) return false;
        tc_fence_after();
        const uint32_t pt = smem_u32(sm.pt[st]), dst = smem_u32(sm.dst[st]);
        const uint32_t qa = smem_u32(sm.q[st]), da = smem_u32(sm.dO[st]);
        const int nk = tile_n(up) / 16;
        for (int kk = 0; kk < nk; ++kk) {
          mma_f16(tdV, sdesc_sw128(pt + kk * 32, 16, 1024), sdesc_sw128(da + kk * 2048, BN * 128, 1024), id_kv,
                  (up > 0 || kk > 0) ? 1u : 0u);
          mma_f16(tdK, sdesc_sw128(dst + kk * 32, 16, 1024), sdesc_sw128(qa + kk * 2048, BN * 128, 1024), id_kv,
                  (up > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(bar[PDS_EMPTY + st]);
        mma_commit(bar[QDO_EMPTY + st]);
        return true;
      };
      for (int u = 0; ok && u < n_tiles; ++u) {
        const int st = u & 1;
        if (!mbar_wait(bar[Q_FULL + st], (u >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        if (!mbar_wait(bar[DO_FULL + st], (u >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
        if (u >= 2 && !mbar_wait(bar[SD_EMPTY + st], ((u >> 1) - 1) & 1, abort_flag, p.status)) { ok = false; break; }
        tc_fence_after();
        const uint32_t qa = smem_u32(sm.q[st]), da = smem_u32(sm.dO[st]);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t boff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_f16(tS + st * BN, sdesc_sw128(k_addr + aoff, 16, 1024), sdesc_sw128(qa + boff, 16, 1024), id_s,
                  kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t aoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
          const uint32_t boff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
          mma_f16(tdP + st * BN, sdesc_sw128(v_addr + aoff, 16, 1024), sdesc_sw128(da + boff, 16, 1024), id_s,
                  kk > 0 ? 1u : 0u);
        }
        mma_commit(bar[SD_FULL + st]);
        if (u >= 1 && !issue_kv(u - 1)) { ok = false; break; }
      }
      if (ok) ok = issue_kv(n_tiles - 1);
      mma_commit(bar[KV_DONE]);
      mma_commit(bar[FINAL]);
      mbar_drain(bar[FINAL], 0);
    }
  } else {
    // --------------------------------------------------- key rows (Pᵀ, dSᵀ)
    const int r = tid;
    const uint32_t lane_addr = ((uint32_t)(warp * 32) << 16);
    const float sl2 = p.scale * kLog2e;
    const bool key_ok = r < nkeys;
    const int j = LMK ? (key_ok ? p.pos_sorted[lbase + key0 + r] : INT_MAX) : key0 + r;  // key position
    const float lw2 = (LMK && key_ok) ? __ldg(p.w_sorted + lbase + key0 + r) * kLog2e : 0.f;
    float dlw = 0.f;
    bool ok = true;
    ColInfo nxt;
    for (int u = 0; u < n_tiles; ++u) {
      const int st = u & 1;
      ok = mbar_wait(bar[SD_FULL + st], (u >> 1) & 1, abort_flag, p.status);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      if (r < BN && u + 1 < n_tiles) nxt = col_info(q_start + BN * (u + 1) + r);  // prefetch next columns
      const int N = tile_n(u);
      float sv[BN], dpv[BN];
#pragma unroll
      for (int ch = 0; ch < BN / 32; ++ch) {
        if (ch * 32 < N) {
          tmem_ld32(tS + lane_addr + st * BN + ch * 32, sv + ch * 32);
          tmem_ld32(tdP + lane_addr + st * BN + ch * 32, dpv + ch * 32);
        }
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(bar[SD_EMPTY + st]);
#pragma unroll
      for (int c = 0; c < BN; ++c) {
        if (c < N) {
          const float l2 = sm.c_lse2[st][c];
          bool valid;
          if (LMK) valid = key_ok && j <= sm.c_i[st][c] && (float)j < sm.c_wlo[st][c];
          else valid = key_ok && j >= sm.c_lo[st][c] && j <= sm.c_i[st][c];
          const float pr = valid ? fast_exp2(fmaf(sv[c], sl2, lw2 - l2)) : 0.f;
          const float dsv = pr * (dpv[c] - sm.c_delta[st][c]);
          sv[c] = pr;
          dpv[c] = dsv;
          if (LMK) dlw += dsv;
        }
      }
      if (u >= 2) {
        ok = mbar_wait(bar[PDS_EMPTY + st], ((u >> 1) - 1) & 1, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      }
      uint8_t* ptb = sm.pt[st];
      uint8_t* dsb = sm.dst[st];
#pragma unroll
      for (int c8 = 0; c8 < BN / 8; ++c8) {
        if (c8 * 8 < N) {
          const int c = c8 * 8;
          uint4 u0, u1;
          u0.x = pack2(sv[c + 0], sv[c + 1], kBF16); u0.y = pack2(sv[c + 2], sv[c + 3], kBF16);
          u0.z = pack2(sv[c + 4], sv[c + 5], kBF16); u0.w = pack2(sv[c + 6], sv[c + 7], kBF16);
          u1.x = pack2(dpv[c + 0], dpv[c + 1], kBF16); u1.y = pack2(dpv[c + 2], dpv[c + 3], kBF16);
          u1.z = pack2(dpv[c + 4], dpv[c + 5], kBF16); u1.w = pack2(dpv[c + 6], dpv[c + 7], kBF16);
          *reinterpret_cast<uint4*>(ptb + sw128_offset(r, c)) = u0;
          *reinterpret_cast<uint4*>(dsb + sw128_offset(r, c)) = u1;
        }
      }
      if (r < BN && u + 1 < n_tiles) store_col(st ^ 1, r, nxt);
      // all rows written and next columns stored (bounded mbarrier sync of the 128 row threads)
      mbar_arrive(bar[ROWS_DONE]);
      ok = mbar_wait(bar[ROWS_DONE], u & 1, abort_flag, p.status);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      if (!LMK && r < N) {
        // soft window edge of query column r: its edge keys [lo, ehi] inside this key block
        const int ehi = sm.c_ehi[st][r];
        const int jlo = max(sm.c_lo[st][r], key0);
        const int jhi = min(ehi, key0 + nkeys - 1);
        const float wt = sm.c_wt[st][r];
        const int qi = sm.c_i[st][r];
        for (int jj = jlo; jj <= jhi; ++jj) {
          const int rr = jj - key0;
          const float z = (wt - (float)(qi - jj)) * inv_tau;
          const float sg = 1.0f / (1.0f + expf(-z));
          T* e1 = reinterpret_cast<T*>(ptb + sw128_offset(rr, r));
          T* e2 = reinterpret_cast<T*>(dsb + sw128_offset(rr, r));
          *e1 = from_f32<T>(to_f32<T>(*e1) * sg);
          *e2 = from_f32<T>(to_f32<T>(*e2) * sg);
        }
      }
      fence_async_smem();
      mbar_arrive(bar[PDS_FULL + st]);
    }
    if (ok && n_tiles > 0) {
      ok = mbar_wait(bar[KV_DONE], 0, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
    }
    const bool have = ok && n_tiles > 0;
    if (LMK) {
      const int64_t slot = lbase + key0 + r;
      float* dkl = a.dk_lmk + slot * D;
      float* dvl = a.dv_lmk + slot * D;
#pragma unroll
      for (int ch = 0; ch < D / 32; ++ch) {
        float ok_[32], ov[32];
        if (have) {
          tmem_ld32(tdK + lane_addr + ch * 32, ok_);
          tmem_ld32(tdV + lane_addr + ch * 32, ov);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) { ok_[e] = 0.f; ov[e] = 0.f; }
        }
        if (key_ok) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            *reinterpret_cast<float4*>(dkl + ch * 32 + e) =
                make_float4(ok_[e] * p.scale, ok_[e + 1] * p.scale, ok_[e + 2] * p.scale, ok_[e + 3] * p.scale);
            *reinterpret_cast<float4*>(dvl + ch * 32 + e) = make_float4(ov[e], ov[e + 1], ov[e + 2], ov[e + 3]);
          }
        }
      }
      if (key_ok && p.d_lw) {
        const int slot_c = __ldg(p.perm + lbase + key0 + r);
        if (slot_c >= 0) p.d_lw[((int64_t)h * p.S + s) * p.k_lmk + slot_c] = have ? dlw : 0.f;
      }
    } else {
      // landmark slots at this key (sorted, duplicates adjacent) add their fp32 rows
      int c0 = -1;
      if (key_ok && p.lmk_slot) c0 = __ldg(p.lmk_slot + (s0 + j) * p.H + h);
      const int64_t row_off = (s0 + j) * (int64_t)p.H * D + (int64_t)h * D;
      T* dko = reinterpret_cast<T*>(p.dk) + row_off;
      T* dvo = reinterpret_cast<T*>(p.dv) + row_off;
#pragma unroll
      for (int ch = 0; ch < D / 32; ++ch) {
        float kk_[32], vv[32];
        if (have) {
          tmem_ld32(tdK + lane_addr + ch * 32, kk_);
          tmem_ld32(tdV + lane_addr + ch * 32, vv);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) { kk_[e] = 0.f; vv[e] = 0.f; }
        }
        if (key_ok) {
#pragma unroll
          for (int e = 0; e < 32; ++e) kk_[e] *= p.scale;
          for (int c = c0; c >= 0 && c < p.kp && __ldg(p.pos_sorted + lbase + c) == j; ++c) {
            const float* lk = a.dk_lmk + (lbase + c) * D + ch * 32;
            const float* lv = a.dv_lmk + (lbase + c) * D + ch * 32;
#pragma unroll
            for (int e = 0; e < 32; ++e) { kk_[e] += __ldg(lk + e); vv[e] += __ldg(lv + e); }
          }
#pragma unroll
          for (int e = 0; e < 32; e += 8) {
            uint4 u0, u1;
            u0.x = pack2(kk_[e], kk_[e + 1], kBF16); u0.y = pack2(kk_[e + 2], kk_[e + 3], kBF16);
            u0.z = pack2(kk_[e + 4], kk_[e + 5], kBF16); u0.w = pack2(kk_[e + 6], kk_[e + 7], kBF16);
            u1.x = pack2(vv[e], vv[e + 1], kBF16); u1.y = pack2(vv[e + 2], vv[e + 3], kBF16);
            u1.z = pack2(vv[e + 4], vv[e + 5], kBF16); u1.w = pack2(vv[e + 6], vv[e + 7], kBF16);
            *reinterpret_cast<uint4*>(dko + ch * 32 + e) = u0;
            *reinterpret_cast<uint4*>(dvo + ch * 32 + e) = u1;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) tmem_dealloc(tmem, 512);
}
}  // namespace dkv

// ---------------------------------------------------------------- host side
CUresult encode_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                   uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2) {
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t es[3] = {1, 1, 1};
  return cuTensorMapEncodeTiled(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                                CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// q/do boxes: rows_q; k/v boxes: rows_k; landmark boxes: min(kp, rows_l)
template <typename T, int D>
static bool make_args(BwdArgs& a, const DsaltAttnParams& p, int rows_q, int rows_k, int rows_l) {
  memset(&a, 0, sizeof(a));
  a.p = p;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t row = (uint64_t)D * 2, trow = (uint64_t)p.H * D * 2;
  if (encode_3d(&a.tm_q, dt, p.q, D, p.H, p.T, row, trow, 64, 1, rows_q) != CUDA_SUCCESS) return false;
  if (encode_3d(&a.tm_do, dt, p.dout, D, p.H, p.T, row, trow, 64, 1, rows_q) != CUDA_SUCCESS) return false;
  if (encode_3d(&a.tm_k, dt, p.k, D, p.H, p.T, row, trow, 64, 1, rows_k) != CUDA_SUCCESS) return false;
  if (encode_3d(&a.tm_v, dt, p.v, D, p.H, p.T, row, trow, 64, 1, rows_k) != CUDA_SUCCESS) return false;
  const int kp = p.kp > 0 ? p.kp : 16;
  a.lmk_box = kp < rows_l ? kp : rows_l;
  const void* lk = p.kp > 0 ? p.lmk_k : p.k;
  const void* lv = p.kp > 0 ? p.lmk_v : p.v;
  const uint64_t hs = p.kp > 0 ? (uint64_t)p.H * p.S : 1;
  if (encode_3d(&a.tm_lk, dt, lk, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS) return false;
  if (encode_3d(&a.tm_lv, dt, lv, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS) return false;
  return true;
}

template <typename T, int D>
cudaError_t launch_dq(const DsaltAttnParams& p, cudaStream_t st) {
  BwdArgs a;
  if (!make_args<T, D>(a, p, dq::BM, dq::BN, dq::BN)) return cudaErrorInvalidValue;
  // at least ~116 KB so that one CTA (and its 512 TMEM columns) owns the SM
  const size_t smem = std::max(sizeof(dq::Smem<D>) + 1024, (size_t)(116 * 1024));
  cudaError_t e = cudaFuncSetAttribute(dq::tc_bwd_dq_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dq::tc_bwd_dq_kernel<T, D><<<dim3((unsigned)p.max_blocks, (unsigned)p.H), kThreads, smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.dw && p.dw_head) return simt_attention_stage(4, p, st);  // dw = Σ_h dw_head
  return cudaSuccess;
}

template <typename T, int D>
cudaError_t launch_dkdv(const DsaltAttnParams& p, float* dk_lmk, float* dv_lmk, cudaStream_t st) {
  BwdArgs a;
  if (!make_args<T, D>(a, p, dkv::BN, dkv::BM, dkv::BM)) return cudaErrorInvalidValue;
  a.dk_lmk = dk_lmk;
  a.dv_lmk = dv_lmk;
  const size_t smem = std::max(sizeof(dkv::Smem<D>) + 1024, (size_t)(116 * 1024));
  cudaError_t e;
  if (p.kp > 0 && p.S > 0) {
    e = cudaFuncSetAttribute(dkv::tc_bwd_dkdv_kernel<true, T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    const int nch = (p.kp + dkv::BM - 1) / dkv::BM;
    dkv::tc_bwd_dkdv_kernel<true, T, D><<<dim3((unsigned)(p.S * nch), (unsigned)p.H), kThreads, smem, st>>>(a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  e = cudaFuncSetAttribute(dkv::tc_bwd_dkdv_kernel<false, T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dkv::tc_bwd_dkdv_kernel<false, T, D><<<dim3((unsigned)p.max_blocks, (unsigned)p.H), kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

}  // namespace bwd

// lmk_scratch: the caller's [2,H,S,kp,D] fp32 buffer for the landmark-slot dK / dV
// that the landmark items of the key-parallel pass hand to the band items.
cudaError_t tc_bwd_stage(int stage, const DsaltAttnParams& p, float* lmk_scratch, cudaStream_t st) {
  const bool bf = p.dtype == DSALT_BF16;
  const size_t half = (size_t)p.H * p.S * p.kp * p.D;
  if (stage == 3) {
    if (bf) return p.D == 64 ? bwd::launch_dq<__nv_bfloat16, 64>(p, st) : bwd::launch_dq<__nv_bfloat16, 128>(p, st);
    return p.D == 64 ? bwd::launch_dq<__half, 64>(p, st) : bwd::launch_dq<__half, 128>(p, st);
  }
  if (stage == 2) {
    float* dk = lmk_scratch;
    float* dv = lmk_scratch ? lmk_scratch + half : nullptr;
    if (p.kp > 0 && !lmk_scratch) return cudaErrorInvalidValue;
    if (bf) return p.D == 64 ? bwd::launch_dkdv<__nv_bfloat16, 64>(p, dk, dv, st)
                             : bwd::launch_dkdv<__nv_bfloat16, 128>(p, dk, dv, st);
    return p.D == 64 ? bwd::launch_dkdv<__half, 64>(p, dk, dv, st) : bwd::launch_dkdv<__half, 128>(p, dk, dv, st);
  }
  return simt_attention_stage(stage, p, st);
}

}  // namespace dsalt
