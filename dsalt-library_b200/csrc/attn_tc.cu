// tcgen05 / TMEM / TMA forward kernel of the DSALT attention for sm_100a.
//
// Persistent: one CTA per SM walks the work items (128 query rows of one
// (sequence, head)) round-robin.  For each item it scans the rows' landmark
// tile(s) and their band of keys [min_i(i − W_i), max_i i], in 128-key tiles;
// tile stages, TMEM buffers and barrier phases run on across items, so the next
// item's loads and first MMAs overlap the current item's last tiles and epilogue.
// 384 threads:
//   warps 0-7   softmax: TMEM lane r = 32·(warp % 4) + lane is query row r;
//               warps 0-3 own key columns 0-63 of every tile, warps 4-7 columns
//               64-127.  Each half keeps its own running max / sum and its own
//               O accumulator in TMEM, so the two halves of a row exchange
//               nothing until the epilogue merges them.  Online softmax in the
//               exp2 domain with a lazy rescale (the running max only moves when
//               it grows by more than 2^8); P (bf16/fp16) goes to a 128B-swizzled
//               K-major smem tile (chunk h = half h), where each thread applies
//               the soft window edge to its row's ≤ ceil(win_edge)+1 edge keys in
//               place, walking only those entries.
//               The epilogue stages O in the P buffer: the input-dtype O is stored
//               row-contiguously by the threads; the op's fp32 output (o_f32: then
//               the only O written) in rounds of 64 columns, both halves merging 32
//               columns each into two 32-column boxes that thread 0 stores with
//               TMA without waiting (plain stores for a block cut by its sequence
//               end); the next round's columns come out of TMEM meanwhile, and the
//               next item's first P waits for the last round's read (STAGE_FREE).
//   warp 8      TMA producers: lane 0 loads Q (once the previous item's last S has
//               read it) and the K tiles, lane 1 the V tiles.
//   warp 9      TMEM allocator + single-thread tcgen05.mma issuer:
//               S[t%2] = Q·K_tᵀ two tiles ahead.
//   warp 10     O_h += P_t,h·V_t,h for each half h as soon as that half's P is
//               written (an item's first one once the previous epilogue read O).
//   warp 11     scheduler: resolves each item's row windows, landmark slots,
//               band and soft-edge factors one or two items ahead into a
//               double-buffered info block.
//
// TMEM (512 columns): S double buffer [0, 256), O_0 [256, 256 + D), O_1 after it.
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

constexpr int BM = 128;              // query rows per item
constexpr int BN = 128;              // keys per tile
constexpr int HALF = BN / 2;         // key columns per softmax thread
constexpr int kMaxLmk = 512;         // landmark slots held in shared memory
constexpr int kThreads = 384;
constexpr int kRowThreads = 256;
constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;    // TMEM owner; issues S = Q·Kᵀ
constexpr int kMmaWarpB = 10;  // issues O_h += P_h·V_h
constexpr int kSchedWarp = 11; // resolves the next items' windows and landmarks
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
constexpr int kMaxEdge = 8;                // soft-edge keys per row handled with precomputed factors
// arrivals that release an item's info block: the eight softmax warps, the
// producer, the two MMA warps (one elected lane each)
constexpr int kInfoConsumers = 11;

enum Bar {
  Q_FULL = 0, Q_EMPTY = 1, K_FULL = 2, V_FULL = 4, K_EMPTY = 6, V_EMPTY = 8, S_FULL = 10, S_EMPTY = 12,
  P_FULL = 14, O_DONE = 16, O_FREE = 18, INFO_FULL = 19, INFO_EMPTY = 21, EPI = 23, FINAL = 24, STAGE_FREE = 26,
  NUM_BARS = 27
};

// Everything the roles need about one item (128 query rows of one (sequence,
// head)), resolved by the scheduler warp one or two items ahead.
struct ItemInfo {
  int h, s, m0, L;
  int64_t s0;
  int band_lo, band_hi, n_valid, n_lt, n_tiles;
  int row_lo[BM], row_hi[BM], row_cnt[BM], row_de0[BM], row_ne[BM];
  float row_wt[BM];
  float row_eg[kMaxEdge][BM];  // σ((w̃ − d)/τ) of each row's first kMaxEdge edge keys (1 past ne)
  int lmk_pos[kMaxLmk];
  float lmk_lw2[kMaxLmk];
};

template <int D>
struct alignas(1024) FwdSmem {
  uint8_t q[BM * D * 2];
  uint8_t k[2][BN * D * 2];
  uint8_t v[2][BN * D * 2];
  uint8_t p[BM * BN * 2];       // chunk h (64 keys) is written by softmax half h
  ItemInfo info[2];
  float m_half[2][2][BM];       // epilogue [item parity][half]: running max (log2) and sum
  float l_half[2][2][BM];
  uint64_t bars[NUM_BARS];
  uint32_t tmem_base;
  int abort_flag;
};

struct alignas(64) FwdArgs {
  CUtensorMap tm_q, tm_k, tm_v, tm_lk, tm_lv;
  CUtensorMap tm_o;  // fp32 O [T, H, D], 32-column x 128-row boxes (valid when o_tma)
  DsaltAttnParams p;
  int lmk_box;  // rows of one landmark TMA box
  int o_tma;    // 1: full blocks of the fp32 O are stored with TMA
};

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

// MMA N extent of tile t of an item: landmark tiles first, then the band tiles
__device__ __forceinline__ int tile_cols(const ItemInfo& in, int t) {
  if (t < in.n_lt) return round16(min(BN, in.n_valid - BN * t));
  return round16(min(BN, in.band_hi - (in.band_lo + BN * (t - in.n_lt)) + 1));
}

// Scheduler warp: resolve item idx into `in` (every row's window, the landmark
// slots of its (head, sequence), the band of key tiles).  An item always has at
// least one tile: a block whose rows attend nothing scans one masked tile.
__device__ __forceinline__ void resolve_item(const DsaltAttnParams& p, int idx, int nb, ItemInfo& in) {
  const int lane = threadIdx.x & 31;
  const int blk = idx % nb, h = idx / nb;
  const int s = __ldg(p.block_map + 2 * blk);
  const int m0 = __ldg(p.block_map + 2 * blk + 1) * BM;
  const int64_t s0 = __ldg(p.cu_seqlens + s);
  const int L = (int)(__ldg(p.cu_seqlens + s + 1) - s0);
  const int kp = p.kp;
  const int64_t lbase = ((int64_t)h * p.S + s) * kp;
  const float inv_tau = 1.0f / p.tau_win;
  int nv = 0;
  for (int c0 = 0; c0 < kp; c0 += 32) {
    const int c = c0 + lane;
    const int ps = c < kp ? __ldg(p.pos_sorted + lbase + c) : -1;
    if (c < kp) {
      in.lmk_pos[c] = ps;
      in.lmk_lw2[c] = __ldg(p.w_sorted + lbase + c) * kLog2e;
    }
    nv += __popc(__ballot_sync(0xffffffffu, ps >= 0));
  }
  __syncwarp();
  int blo = INT_MAX, bhi = -1;
  for (int r = lane; r < BM; r += 32) {
    const int i = m0 + r;
    int lo = INT_MAX, hi = -1, cnt = 0, d_e0 = INT_MAX, ne = 0;
    float wt = 0.f;
    if (i < L) {
      const RowWindow rw = row_window(__ldg(p.w + s0 + i), i, p.semantics, p.win_edge);
      wt = rw.wt;
      if (rw.W >= 0) {
        lo = i - min(rw.W, i);
        hi = i;
        d_e0 = max((int)floorf(rw.core) + 1, 0);
        ne = max(min(rw.W, i) - d_e0 + 1, 0);
      }
      // landmarks valid for row i form a prefix of the sorted positions
      int a0 = 0, a1 = nv;
      while (a0 < a1) {
        const int mid = (a0 + a1) >> 1;
        const int ps = in.lmk_pos[mid];
        if (ps <= i && (float)ps < rw.win_lo) a0 = mid + 1; else a1 = mid;
      }
      cnt = a0;
    }
    in.row_lo[r] = lo; in.row_hi[r] = hi; in.row_cnt[r] = cnt;
    in.row_de0[r] = d_e0; in.row_ne[r] = ne; in.row_wt[r] = wt;
    // soft-edge factors σ((w̃ − d)/τ) of the row's first edge keys (d ≤ w̃: the
    // exponent is ≤ 0), with the fast intrinsics: they scale 16-bit P values
#pragma unroll
    for (int e = 0; e < kMaxEdge; ++e) {
      float f = 1.0f;
      if (e < ne) f = __fdividef(1.0f, 1.0f + __expf(-((wt - (float)(d_e0 + e)) * inv_tau)));
      in.row_eg[e][r] = f;
    }
    if (lo <= hi) { blo = min(blo, lo); bhi = max(bhi, hi); }
  }
  blo = __reduce_min_sync(0xffffffffu, blo);
  bhi = __reduce_max_sync(0xffffffffu, bhi);
  if (lane == 0) {
    const int n_lt = (nv + BN - 1) / BN;
    int n_bt = bhi >= blo ? (bhi - blo + BN) / BN : 0;
    if (n_lt + n_bt == 0) { blo = 0; bhi = 0; n_bt = 1; }  // one fully masked tile
    in.h = h; in.s = s; in.m0 = m0; in.L = L; in.s0 = s0;
    in.band_lo = blo; in.band_hi = bhi; in.n_valid = nv; in.n_lt = n_lt; in.n_tiles = n_lt + n_bt;
  }
  __syncwarp();
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) tc_fwd_kernel(const __grid_constant__ FwdArgs a) {
  using namespace sm100;
  const DsaltAttnParams& p = a.p;
  const int nb = __ldg(p.num_blocks);
  const int n_items = nb * p.H;
  if ((int)blockIdx.x >= n_items) return;  // CTA-uniform, before any barrier or TMEM use

  extern __shared__ uint8_t smem_raw[];
  FwdSmem<D>& sm = *reinterpret_cast<FwdSmem<D>*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  constexpr bool kBF16 = !std::is_same<T, __half>::value;
  const BarArray bar{smem_u32(&sm.bars[0])};

  if (tid == 0) {
    mbar_init(bar[Q_FULL], 1);
    mbar_init(bar[Q_EMPTY], 1);
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar[K_FULL + st], 1);
      mbar_init(bar[V_FULL + st], 1);
      mbar_init(bar[K_EMPTY + st], 1);
      mbar_init(bar[V_EMPTY + st], 1);
      mbar_init(bar[S_FULL + st], 1);
      mbar_init(bar[S_EMPTY + st], kRowThreads);
      mbar_init(bar[P_FULL + st], kRowThreads / 2);  // index = softmax half
      mbar_init(bar[O_DONE + st], 1);                // index = softmax half
      mbar_init(bar[INFO_FULL + st], 32);
      mbar_init(bar[INFO_EMPTY + st], kInfoConsumers);
    }
    mbar_init(bar[O_FREE], kRowThreads);
    mbar_init(bar[EPI], kRowThreads);
    mbar_init(bar[STAGE_FREE], 1);
    mbar_init(bar[FINAL], 1);
    mbar_init(bar[FINAL + 1], 1);
    fence_mbar_init();
    sm.abort_flag = 0;
  }
  if (warp == kProducerWarp && lane == 0) {
    prefetch_tmap(&a.tm_q);
    prefetch_tmap(&a.tm_k);
    prefetch_tmap(&a.tm_v);
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&sm.tmem_base), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  const int stride = gridDim.x;
  const uint32_t tS = tmem;            // S buffers: columns [0,128) and [128,256)
  const uint32_t tO = tmem + 2 * BN;   // O_h: columns [256 + h·D, 256 + (h+1)·D)

  if (warp == kSchedWarp) {
    // ------------------------------------------------------------ scheduler
    int li = 0;
    for (int idx = blockIdx.x; idx < n_items; idx += stride, ++li) {
      const int ib = li & 1;
      if (li >= 2 &&
          !__all_sync(0xffffffffu, mbar_wait(bar[INFO_EMPTY + ib], ((li >> 1) - 1) & 1, abort_flag, p.status)))
        break;
      resolve_item(p, idx, nb, sm.info[ib]);
      mbar_arrive(bar[INFO_FULL + ib]);
    }
  } else if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producers
    // lane 0: Q (once the previous item's last S is issued) and the K tiles;
    // lane 1: the V tiles.  Tile stages follow a tile counter that runs across items.
    int gk = 0, li = 0, issued_k = 0, issued_q = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride, ++li) {
      const int ib = li & 1;
      ok = mbar_wait(bar[INFO_FULL + ib], (li >> 1) & 1, abort_flag, p.status);
      const ItemInfo& in = sm.info[ib];
      const int n_tiles = in.n_tiles, n_lt = in.n_lt;
      if (ok && lane < 2) {
        const bool is_k = lane == 0;
        if (is_k) {
          if (li >= 1) ok = mbar_wait(bar[Q_EMPTY], (li - 1) & 1, abort_flag, p.status);
          if (ok) {
            mbar_expect_tx(bar[Q_FULL], BM * D * 2);
#pragma unroll
            for (int c = 0; c < D / 64; ++c)
              tma_load_3d(smem_u32(sm.q + c * (BM * 128)), &a.tm_q, bar[Q_FULL], c * 64, in.h, (int)(in.s0 + in.m0));
            issued_q = li + 1;
          }
        }
        const int FULL = is_k ? K_FULL : V_FULL, EMPTY = is_k ? K_EMPTY : V_EMPTY;
        for (int t = 0; ok && t < n_tiles; ++t) {
          const int g = gk + t, st = g & 1;
          if (g >= 2 && !mbar_wait(bar[EMPTY + st], ((g >> 1) - 1) & 1, abort_flag, p.status)) { ok = false; break; }
          const bool lmk = t < n_lt;
          mbar_expect_tx(bar[FULL + st], (lmk ? a.lmk_box : BN) * D * 2);
          uint8_t* dst = is_k ? sm.k[st] : sm.v[st];
          const CUtensorMap* map = lmk ? (is_k ? &a.tm_lk : &a.tm_lv) : (is_k ? &a.tm_k : &a.tm_v);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            if (lmk) tma_load_3d(smem_u32(dst + c * (BN * 128)), map, bar[FULL + st], c * 64, BN * t, in.h * p.S + in.s);
            else tma_load_3d(smem_u32(dst + c * (BN * 128)), map, bar[FULL + st], c * 64, attn_kv_head(p, in.h),
                             (int)(in.s0 + in.band_lo + BN * (t - n_lt)));
          }
          issued_k = g + 1;
        }
      }
      ok = __all_sync(0xffffffffu, ok);
      gk += n_tiles;
      if (lane == 0) mbar_arrive(bar[INFO_EMPTY + ib]);
    }
    // drain: never leave a TMA write in flight into shared memory
    if (lane < 2) {
      const int FULL = lane == 0 ? K_FULL : V_FULL;
      for (int g = max(0, issued_k - 2); g < issued_k; ++g) mbar_drain(bar[FULL + (g & 1)], (g >> 1) & 1);
    }
    if (lane == 0 && issued_q > 0) mbar_drain(bar[Q_FULL], (issued_q - 1) & 1);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ S issuer
    // S_t = Q·K_tᵀ as soon as K_t is in and the softmax has read S_{t−2}.  The
    // P·V products come from warp 10: one issuing thread sustains only about
    // one MMA per 110 cycles, two overlap.
    int gs = 0, li = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride, ++li) {
      const int ib = li & 1;
      ok = mbar_wait(bar[INFO_FULL + ib], (li >> 1) & 1, abort_flag, p.status);
      const ItemInfo& in = sm.info[ib];
      const int n_tiles = in.n_tiles;
      if (ok && lane == 0) {
        const uint32_t q_addr = smem_u32(sm.q);
        ok = mbar_wait(bar[Q_FULL], li & 1, abort_flag, p.status);
        for (int t = 0; ok && t < n_tiles; ++t) {
          const int g = gs + t, st = g & 1;
          if (!mbar_wait(bar[K_FULL + st], (g >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
          if (g >= 2 && !mbar_wait(bar[S_EMPTY + st], ((g >> 1) - 1) & 1, abort_flag, p.status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sm.k[st]);
          const uint32_t id_s = idesc_f16(kBF16, BM, tile_cols(in, t), false, false);
#pragma unroll
          for (int kk = 0; kk < D / 16; ++kk) {
            const uint32_t off = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
            const uint64_t ad = sdesc_sw128(q_addr + off, 16, 1024);
            const uint64_t bd = sdesc_sw128(k_addr + (kk >> 2) * (BN * 128) + (kk & 3) * 32, 16, 1024);
            mma_f16(tS + st * BN, ad, bd, id_s, kk > 0 ? 1u : 0u);
          }
          mma_commit(bar[S_FULL + st]);
          mma_commit(bar[K_EMPTY + st]);
        }
        if (ok) mma_commit(bar[Q_EMPTY]);  // the item's last S has read Q
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      gs += n_tiles;
      if (lane == 0) mbar_arrive(bar[INFO_EMPTY + ib]);
    }
    if (lane == 0) {
      // drain: every issued MMA completes before TMEM is released
      mma_commit(bar[FINAL]);
      mbar_drain(bar[FINAL], 0);
    }
  } else if (warp == kMmaWarpB) {
    // ------------------------------------------------------------ P·V issuer
    // O_h += P_t,h·V_t,h for each half h as soon as that half of P is written.
    // O_DONE[h] is committed once per tile and half, also when the half had no
    // valid key (its P·V is skipped).  An item's first P·V waits until the
    // previous item's epilogue has read O (O_FREE).
    int gv = 0, li = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride, ++li) {
      const int ib = li & 1;
      ok = mbar_wait(bar[INFO_FULL + ib], (li >> 1) & 1, abort_flag, p.status);
      const ItemInfo& in = sm.info[ib];
      const int n_tiles = in.n_tiles;
      if (ok && lane == 0) {
        const uint32_t id_o = idesc_f16(kBF16, BM, D, false, true);
        const uint32_t p_addr = smem_u32(sm.p);
        if (li >= 1) ok = mbar_wait(bar[O_FREE], (li - 1) & 1, abort_flag, p.status);
        bool o_written0 = false, o_written1 = false;
        for (int t = 0; ok && t < n_tiles; ++t) {
          const int g = gv + t, st = g & 1;
          const int nvalid = tile_cols(in, t);
          if (!mbar_wait(bar[V_FULL + st], (g >> 1) & 1, abort_flag, p.status)) { ok = false; break; }
          const uint32_t v_addr = smem_u32(sm.v[st]);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            if (!mbar_wait(bar[P_FULL + hh], g & 1, abort_flag, p.status)) { ok = false; break; }
            tc_fence_after();
            const int nk = min(max(nvalid - HALF * hh, 0), HALF) / 16;  // valid 16-key steps of this half
            bool& written = hh == 0 ? o_written0 : o_written1;
            for (int kk = 0; kk < nk; ++kk) {
              const uint64_t ad = sdesc_sw128(p_addr + hh * (BM * 128) + kk * 32, 16, 1024);
              const uint64_t bd = sdesc_sw128(v_addr + (HALF / 16 * hh + kk) * 2048, BN * 128, 1024);
              mma_f16(tO + hh * D, ad, bd, id_o, (written || kk > 0) ? 1u : 0u);
            }
            if (nk > 0) written = true;
            mma_commit(bar[O_DONE + hh]);
          }
          if (!ok) break;
          mma_commit(bar[V_EMPTY + st]);
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      gv += n_tiles;
      if (lane == 0) mbar_arrive(bar[INFO_EMPTY + ib]);
    }
    if (lane == 0) {
      mma_commit(bar[FINAL + 1]);
      mbar_drain(bar[FINAL + 1], 0);
    }
  } else {
    // ------------------------------------------------------------ softmax (row halves)
    // row r = 32·(warp % 4) + lane, key-column half = warp / 4
    const int r = 32 * (warp & 3) + lane;
    const int half = (warp >> 2) & 1;
    const uint32_t lane_addr = ((uint32_t)(32 * (warp & 3)) << 16);
    const int c0 = HALF * half;          // first tile column owned by this thread
    const uint32_t tOh = tO + half * D;  // this half's O accumulator
    const float sl2 = p.scale * kLog2e;
    const float inv_tau = 1.0f / p.tau_win;
    uint8_t* sp = sm.p + half * (BM * 128);  // this half's P chunk: 128 rows x 64 keys
    int gt = 0, li = 0, epi_phase = 0;
    bool ok = true;
    // all softmax threads meet (bounded wait on the EPI barrier)
    auto epi_sync = [&]() -> bool {
      mbar_arrive(bar[EPI]);
      const bool w = mbar_wait(bar[EPI], epi_phase & 1, abort_flag, p.status);
      ++epi_phase;
      return __all_sync(0xffffffffu, w);
    };
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride, ++li) {
      const int ib = li & 1;
      ok = __all_sync(0xffffffffu, mbar_wait(bar[INFO_FULL + ib], (li >> 1) & 1, abort_flag, p.status));
      if (!ok) break;
      const ItemInfo& in = sm.info[ib];
      const int n_tiles = in.n_tiles, n_lt = in.n_lt, band_lo = in.band_lo;
      const int m0 = in.m0, L = in.L, h = in.h;
      const int64_t s0 = in.s0;
      const int i = m0 + r;
      const bool row_ok = i < L;
      const int lo = in.row_lo[r], hi = in.row_hi[r], cnt = in.row_cnt[r];
      const int d_e0 = in.row_de0[r], ne = in.row_ne[r];
      const float wt = in.row_wt[r];
      float m = -INFINITY, l = 0.f;  // this half's running max (log2 units) and sum
      for (int t = 0; t < n_tiles; ++t) {
        const int g = gt + t, st = g & 1;
        ok = mbar_wait(bar[S_FULL + st], (g >> 1) & 1, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        // columns past the tile's valid keys hold stale values and are masked below
        float x[HALF];
        tmem_ld32(tS + lane_addr + st * BN + c0, x);
        tmem_ld32(tS + lane_addr + st * BN + c0 + 32, x + 32);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(bar[S_EMPTY + st]);

        const bool lmk = t < n_lt;
        const int n0 = lmk ? 0 : band_lo + BN * (t - n_lt);
        // valid columns of this thread: [vlo, vhi] (band) or [0, vhi] (landmarks)
        int vlo, vhi;
        if (lmk) {
          vlo = 0;
          vhi = cnt - BN * t - c0 - 1;
        } else {
          vlo = lo - n0 - c0;  // lo = INT_MAX for a row without band: stays positive
          vhi = hi - n0 - c0;
        }
        const bool all_in = __all_sync(0xffffffffu, vlo <= 0 && vhi >= HALF - 1);
        const bool all_out = __all_sync(0xffffffffu, vhi < 0 || vlo > HALF - 1 || vlo > vhi);
        float xs = lmk ? 1.0f : sl2;  // multiplier applied inside exp2
        if (lmk) {
          const float* lw2 = in.lmk_lw2 + BN * t + c0;
#pragma unroll
          for (int c = 0; c < HALF; ++c) x[c] = fmaf(x[c], sl2, lw2[c]);
        }
        float mt = -INFINITY;
        if (!all_out) {
          if (!all_in) {
            const uint32_t m_lo = range_mask32(vlo, vhi), m_hi = range_mask32(vlo - 32, vhi - 32);
#pragma unroll
            for (int c = 0; c < 32; ++c) x[c] = (m_lo >> c) & 1u ? x[c] : -INFINITY;
#pragma unroll
            for (int c = 0; c < 32; ++c) x[32 + c] = (m_hi >> c) & 1u ? x[32 + c] : -INFINITY;
          }
          float mx[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) mx[q] = max3(x[2 * q], x[2 * q + 1], x[16 + 2 * q]);
#pragma unroll
          for (int c = 32; c < HALF; c += 16)
#pragma unroll
            for (int q = 0; q < 8; ++q) mx[q] = max3(mx[q], x[c + 2 * q], x[c + 2 * q + 1]);
#pragma unroll
          for (int q = 0; q < 8; ++q) mx[q] = fmaxf(mx[q], x[16 + 2 * q + 1]);
          mt = max3(max3(mx[0], mx[1], mx[2]), max3(mx[3], mx[4], mx[5]), fmaxf(mx[6], mx[7]));
          if (!lmk) mt *= sl2;
        }
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
        if (!all_out) {
          const float ms = (m == -INFINITY) ? 0.f : m;
          float sm8[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) sm8[q] = 0.f;
#pragma unroll
          for (int c = 0; c < HALF; ++c) {
            x[c] = fast_exp2(fmaf(x[c], xs, -ms));
            sm8[c & 7] += x[c];
          }
          const float sum = ((sm8[0] + sm8[1]) + (sm8[2] + sm8[3])) + ((sm8[4] + sm8[5]) + (sm8[6] + sm8[7]));
          l = l * factor + sum;
        } else {
          l = l * factor;
        }

        // this half's P chunk and O_h are free once its previous P·V has completed
        if (g >= 1) {
          ok = mbar_wait(bar[O_DONE + half], (g - 1) & 1, abort_flag, p.status);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
          tc_fence_after();
        }
        if (t == 0) {
          // the P buffer also stages the previous item's fp32 O: free once the TMA
          // stores that thread 0 issued have read it (thread 0 releases it here)
          if (tid == 0) {
            bulk_wait_read0();
            mbar_arrive(bar[STAGE_FREE]);
          }
          ok = mbar_wait(bar[STAGE_FREE], li & 1, abort_flag, p.status);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        }
        if (all_out) {
          const uint4 z = make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
          for (int c8 = 0; c8 < HALF / 8; ++c8) *reinterpret_cast<uint4*>(sp + sw128_offset(r, c8 * 8)) = z;
        } else {
#pragma unroll
          for (int c8 = 0; c8 < HALF / 8; ++c8) {
            const int c = c8 * 8;
            uint4 u;
            u.x = pack2(x[c + 0], x[c + 1], kBF16);
            u.y = pack2(x[c + 2], x[c + 3], kBF16);
            u.z = pack2(x[c + 4], x[c + 5], kBF16);
            u.w = pack2(x[c + 6], x[c + 7], kBF16);
            *reinterpret_cast<uint4*>(sp + sw128_offset(r, c)) = u;
          }
        }
        if (!lmk && !all_out && ne > 0) {
          // soft window edge on this row's edge keys in this thread's columns:
          // p *= σ((w̃ − d)/τ); the key at distance d_e0 + e sits in column ce0 − e.
          // Each lane walks only its own entries (a row's edge is a few keys), the
          // factors past the precomputed ones computed by the same expression.
          const int ce0 = i - d_e0 - n0 - c0;
          const int rx = r & 7;
          uint8_t* rowp = sp + r * 128;
          for (int e = max(0, ce0 - (HALF - 1)); e < ne && ce0 - e >= 0; ++e) {
            const int c = ce0 - e;
            T* ep = reinterpret_cast<T*>(rowp + ((((c >> 3) ^ rx) << 4) | ((c & 7) << 1)));
            const float pv = to_f32<T>(*ep);
            const float sg = e < kMaxEdge ? in.row_eg[e][r]
                                          : 1.0f / (1.0f + expf(-((wt - (float)(d_e0 + e)) * inv_tau)));
            *ep = from_f32<T>(pv * sg);
            l -= pv * (1.0f - sg);
          }
        }
        // rescale O_h once P is out of registers; a finite running max implies an
        // earlier tile of this item had valid keys in this half, so O_h has been
        // written (and holds this item's sums) whenever a rescale happens
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int ch = 0; ch < D / 32; ++ch) {
            float o[32];
            tmem_ld32(tOh + lane_addr + ch * 32, o);
            tmem_wait_ld();
            const float f = rescale ? factor : 1.0f;
#pragma unroll
            for (int j = 0; j < 32; ++j) o[j] *= f;
            tmem_st32(tOh + lane_addr + ch * 32, o);
          }
          tmem_wait_st();
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(bar[P_FULL + half]);
      }
      if (!ok) break;
      // ---- epilogue: merge the two halves of each row, O / l, LSE
      sm.m_half[ib][half][r] = m;
      sm.l_half[ib][half][r] = l;
      if (!(ok = epi_sync())) break;
      const float mh0 = sm.m_half[ib][0][r], mh1 = sm.m_half[ib][1][r];
      const float lh0 = sm.l_half[ib][0][r], lh1 = sm.l_half[ib][1][r];
      const float mm = fmaxf(mh0, mh1);
      // a half with l = 0 never had a valid key and its O_h may hold an earlier item's sums
      const float f0 = lh0 > 0.f ? exp2f(mh0 - mm) : 0.f;
      const float f1 = lh1 > 0.f ? exp2f(mh1 - mm) : 0.f;
      const float lt = lh0 * f0 + lh1 * f1;
      const bool nonempty = lt > 1e-9f;
      const float inv_l = nonempty ? 1.0f / lt : 0.f;
      const bool use0 = nonempty && lh0 > 0.f, use1 = nonempty && lh1 > 0.f;
      if (row_ok && half == 0) p.lse[(s0 + i) * p.H + h] = nonempty ? (mm + log2f(lt)) * kLn2 : -INFINITY;
      // both halves' last P·V have completed: O_0 and O_1 are final
      const int gl = gt + n_tiles - 1;  // the item's last tile
      ok = mbar_wait(bar[O_DONE], gl & 1, abort_flag, p.status) &&
           mbar_wait(bar[O_DONE + 1], gl & 1, abort_flag, p.status);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) break;
      tc_fence_after();
      const int rows = min(BM, L - m0);
      const int64_t HD = (int64_t)p.H * D;
      uint8_t* stage = sm.p;
      if (p.o_f32 != nullptr) {
        // fp32 O in rounds of 64 output columns: half h merges columns 64·rd + 32·h + [0, 32)
        // of its row into box h of the staging area (128 rows x 128 B, 16-byte units
        // XOR-swizzled by row % 8: the SWIZZLE_128B image of one 32-column box of tm_o)
        const bool tma = a.o_tma != 0 && rows == BM;
        uint8_t* box = stage + half * (BM * 128);
        for (int rd = 0; rd < D / 64; ++rd) {
          float v[32];
#pragma unroll
          for (int c16 = 0; c16 < 2; ++c16) {
            const int col = 64 * rd + 32 * half + 16 * c16;
            float o1[16];
            tmem_ld16(tO + lane_addr + col, v + 16 * c16);
            tmem_ld16(tO + D + lane_addr + col, o1);
            tmem_wait_ld();
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float a0 = use0 ? v[16 * c16 + j] * f0 : 0.f;
              const float a1 = use1 ? o1[j] * f1 : 0.f;
              v[16 * c16 + j] = round_to<T>((a0 + a1) * inv_l);
            }
          }
          if (rd == D / 64 - 1) {
            tc_fence_before();
            mbar_arrive(bar[O_FREE]);  // O is read: the next item's P·V may overwrite it
          }
          if (rd > 0) {
            // the previous round's boxes have been read by its TMA stores (while this
            // round's columns came out of TMEM) or copied by the threads
            if (tma && tid == 0) bulk_wait_read0();
            if (!(ok = epi_sync())) break;
          }
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<float4*>(box + r * 128 + ((u ^ (r & 7)) << 4)) =
                make_float4(v[4 * u], v[4 * u + 1], v[4 * u + 2], v[4 * u + 3]);
          if (tma) fence_async_smem();  // the staged rows, visible to the TMA stores
          if (!(ok = epi_sync())) break;
          if (tma) {
            if (tid == 0) {
              tma_store_3d(&a.tm_o, smem_u32(stage), 64 * rd, h, (int)(s0 + m0));
              tma_store_3d(&a.tm_o, smem_u32(stage + BM * 128), 64 * rd + 32, h, (int)(s0 + m0));
              bulk_commit();
            }
          } else {
            // a block cut by its sequence end: the rows that exist, row-contiguously
            uint8_t* dst = reinterpret_cast<uint8_t*>(p.o_f32) + ((s0 + m0) * HD + (int64_t)h * D + rd * 64) * 4;
            const int64_t row_bytes = HD * 4;
            for (int un = r + BM * half; un < rows * 16; un += kRowThreads) {
              const int rr = un >> 4, uu = un & 15;
              const uint8_t* src = stage + (uu >> 3) * (BM * 128) + rr * 128 + (((uu & 7) ^ (rr & 7)) << 4);
              *reinterpret_cast<uint4*>(dst + rr * row_bytes + uu * 16) = *reinterpret_cast<const uint4*>(src);
            }
          }
        }
        // the threads' copies are done before the next item writes P (TMA stores:
        // released through STAGE_FREE at the next item's first P)
        if (ok && !tma) ok = epi_sync();
      } else {
        // input-dtype O: 128 rows x D·2 bytes staged with 16-byte units XOR-swizzled
        // by row % 8, then stored row-contiguously
#pragma unroll
        for (int ch = 0; ch < D / 32; ++ch) {  // this thread's D/2 output columns, 16 at a time
          const int col = half * (D / 2) + ch * 16;
          float o0[16], o1[16];
          tmem_ld16(tO + lane_addr + col, o0);
          tmem_ld16(tO + D + lane_addr + col, o1);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float a0 = use0 ? o0[j] * f0 : 0.f;
            const float a1 = use1 ? o1[j] * f1 : 0.f;
            o0[j] = (a0 + a1) * inv_l;
          }
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int un = col / 8 + u;
            *reinterpret_cast<uint4*>(stage + r * 256 + ((un ^ (r & 7)) << 4)) =
                make_uint4(pack2(o0[8 * u + 0], o0[8 * u + 1], kBF16), pack2(o0[8 * u + 2], o0[8 * u + 3], kBF16),
                           pack2(o0[8 * u + 4], o0[8 * u + 5], kBF16), pack2(o0[8 * u + 6], o0[8 * u + 7], kBF16));
          }
        }
        tc_fence_before();
        mbar_arrive(bar[O_FREE]);  // O is read: the next item's P·V may overwrite it
        if (!(ok = epi_sync())) break;
        uint8_t* dst = reinterpret_cast<uint8_t*>(p.o) + ((s0 + m0) * HD + (int64_t)h * D) * 2;
        const int64_t row_bytes = HD * 2;
        constexpr int units = D / 8;  // 16-byte units per staged row
        for (int un = r + BM * half; un < rows * units; un += kRowThreads) {
          const int rr = un / units, uu = un % units;
          *reinterpret_cast<uint4*>(dst + rr * row_bytes + uu * 16) =
              *reinterpret_cast<const uint4*>(stage + rr * 256 + ((uu ^ (rr & 7)) << 4));
        }
        if (!(ok = epi_sync())) break;  // the staging area is reused by the next item's P
      }
      if (!ok) break;
      gt += n_tiles;
      __syncwarp();
      if (lane == 0) mbar_arrive(bar[INFO_EMPTY + ib]);
    }
  }
  if (tid == 0) bulk_wait_all();  // the fp32 O stores this thread issued have completed
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
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
  // k, v: [T, H_kv, D] (grouped kv heads read in place)
  const uint64_t hkv = (uint64_t)attn_kv_heads(p), kvrow = hkv * D * 2;
  if (encode_3d(&a.tm_k, dt, p.k, D, hkv, p.T, row, kvrow, 64, 1, BN) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  if (encode_3d(&a.tm_v, dt, p.v, D, hkv, p.T, row, kvrow, 64, 1, BN) != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const int kp = p.kp > 0 ? p.kp : 16;
  a.lmk_box = kp < BN ? kp : BN;
  const void* lk = p.kp > 0 ? p.lmk_k : p.k;  // any valid address when there are no landmarks
  const void* lv = p.kp > 0 ? p.lmk_v : p.v;
  const uint64_t hs = p.kp > 0 ? (uint64_t)p.H * p.S : 1;
  if (encode_3d(&a.tm_lk, dt, lk, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  if (encode_3d(&a.tm_lv, dt, lv, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  // fp32 O: [T, H, D] in boxes of 32 columns (128 B, the swizzle span) x 128 rows
  a.o_tma = p.o_f32 != nullptr && ((uintptr_t)p.o_f32 & 15u) == 0 &&
            encode_3d(&a.tm_o, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.o_f32, D, p.H, p.T, (uint64_t)D * 4,
                      (uint64_t)p.H * D * 4, 32, 1, BM) == CUDA_SUCCESS;
  // at least ~116 KB so that one CTA (and its 512 TMEM columns) owns the SM
  const size_t smem = std::max(sizeof(FwdSmem<D>) + 1024, (size_t)(116 * 1024));
  cudaError_t e = ensure_smem((const void*)tc_fwd_kernel<T, D>, smem);
  if (e != cudaSuccess) return e;
  // persistent: one CTA per SM walks the (head, query block) items round-robin
  static int sms[64] = {};
  int dev = 0;
  e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (sms[dev] <= 0) {
    e = cudaDeviceGetAttribute(&sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  const long long items = (long long)p.max_blocks * p.H;
  const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>(items, sms[dev]));
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
