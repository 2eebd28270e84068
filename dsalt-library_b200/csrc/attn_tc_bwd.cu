// tcgen05 / TMEM / TMA dK/dV kernel of the DSALT attention backward for sm_100a
// (key-parallel, atomic-free for dK/dV; reference _train_bwd_dkdv_kernel
// dsalt/kernels/dsalt_triton_train.py:386-481 and the landmark atomics of
// _train_bwd_kernel :302-333).
//
//   rows = 128 keys; tiles = 64 queries.  Sᵀ = K·Qᵀ, dPᵀ = V·dOᵀ (TMEM) ->
//   Pᵀ, dSᵀ (bf16, written back into the TMEM columns of Sᵀ, dPᵀ they came
//   from, with the soft-edge factor) ->
//   dV += Pᵀ·dO, dK += dSᵀ·Q (TMEM, A operand read from TMEM).  Landmark items (the sorted landmark slots
//   of one (head, sequence) as the keys, every later query as columns) write
//   fp32 dK/dV per slot and d_lw (a row sum: no atomics); band items (128
//   consecutive keys) add those slot rows into their own before the single
//   store.  dK/dV and d_lw are deterministic.
//
// Every finished dSᵀ tile is also written to one of two shared buffers (the
// 128B-swizzled image of a 128 × 64 K-major tile) and bulk-copied from there to
// the ds_tiles scratch (16 KB per tile), where the dQ stage (attn_tc_dq.cu) reads
// it: dQ = scale·Σ dS·K without a second computation of S, dP and the
// exponentials.
// ∂loss/∂w̃ = Σ_edge dS·(1 − σ)/τ of each query (the reference's D_w, :371-383)
// is formed by the dQ stage from the stored, σ-scaled dSᵀ entries.
//
// All waits are bounded (sm100::mbar_wait); see attn_tc.cu.
#include <mutex>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {

cudaError_t simt_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st);
cudaError_t tc_bwd_dq_stage(const DsaltAttnParams& p, cudaStream_t st);

namespace bwd {

constexpr int kMaxEdge = kQRecEdge;  // soft-edge keys per query handled with precomputed factors
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ int round16(int n) { return (n + 15) & ~15; }

// the 16-bit element in the low half of b as float, and a float rounded to the
// 16-bit type's bits
template <typename T>
__device__ __forceinline__ float bits_to_f32(uint32_t b) {
  const unsigned short u = (unsigned short)(b & 0xffffu);
  if constexpr (std::is_same<T, __half>::value) return __half2float(__ushort_as_half(u));
  else return __bfloat162float(__ushort_as_bfloat16(u));
}
template <typename T>
__device__ __forceinline__ uint32_t f32_to_bits(float v) {
  if constexpr (std::is_same<T, __half>::value) return (uint32_t)__half_as_ushort(__float2half_rn(v));
  else return (uint32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
}

struct alignas(64) BwdArgs {
  CUtensorMap tm_q, tm_do, tm_k, tm_v, tm_lk, tm_lv;
  DsaltAttnParams p;
  float* dk_lmk;   // [DSALT_LMK_SPLIT,H,S,kp,D] fp32 scratch: partial landmark-slot dK / dV
  float* dv_lmk;
  float* dlw_lmk;  // [DSALT_LMK_SPLIT,H,S,kp] fp32 scratch: partial landmark-slot d_lw
  float* band_lmk;  // [2,H,S,kp,D] fp32 scratch: band-pass dK / dV of keys holding landmark slots
  int64_t part_stride;  // H·S·kp: slots per partial
  int lmk_box;    // rows of one landmark TMA box
};

// store 32 values of one row as four 16-byte bf16/fp16 units of a 128B-swizzled tile
template <bool BF16>
__device__ __forceinline__ void store_row32(uint8_t* base, int row, int col0, const float* v) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    uint4 u;
    u.x = sm100::pack2(v[8 * g + 0], v[8 * g + 1], BF16);
    u.y = sm100::pack2(v[8 * g + 2], v[8 * g + 3], BF16);
    u.z = sm100::pack2(v[8 * g + 4], v[8 * g + 5], BF16);
    u.w = sm100::pack2(v[8 * g + 6], v[8 * g + 7], BF16);
    *reinterpret_cast<uint4*>(base + sm100::sw128_offset(row, col0 + 8 * g)) = u;
  }
}

// store 32 packed bf16/fp16 values (16 words) of one row into a 128B-swizzled tile
__device__ __forceinline__ void store_row32_packed(uint8_t* base, int row, int col0, const uint32_t* pk) {
#pragma unroll
  for (int g = 0; g < 4; ++g)
    *reinterpret_cast<uint4*>(base + sm100::sw128_offset(row, col0 + 8 * g)) =
        make_uint4(pk[4 * g], pk[4 * g + 1], pk[4 * g + 2], pk[4 * g + 3]);
}


// ==================================================================== dK / dV
namespace dkv {
constexpr int BM = 128, BN = 64;  // BM keys (TMEM lanes), BN queries per tile
constexpr int kQStages = 3;       // Q / dO tile ring
constexpr int kColStages = 4;     // per-tile column data ring
// 16 row warps: warp w reads TMEM lanes 32·(w % 4)… and owns the 16-column
// quarter w / 4 of every tile (four warps per scheduler hide the latencies of
// the element-wise work); a quarter is one K = 16 step of the dV / dK MMAs, so
// it writes its packed Pᵀ / dSᵀ over its own (already read) Sᵀ / dPᵀ columns.
// Then the TMA warp, MMA warp A (TMEM owner: Sᵀ, dV), the column warp and MMA
// warp B (dPᵀ, dK).
constexpr int kRowWarps = 16;
constexpr int kRowThreads = 32 * kRowWarps;
constexpr int kProducerWarp = 16;
constexpr int kMmaWarp = 17;
constexpr int kColWarp = 18;
constexpr int kMmaWarpB = 19;
constexpr int kThreadsKV = 640;
constexpr int kQuarter = BN / 4;  // tile columns per row thread
enum { KV_FULL = 0, KV_EMPTY = 1, Q_FULL = 2, DO_FULL = Q_FULL + kQStages, QDO_EMPTY = DO_FULL + kQStages,
       REC_FULL = QDO_EMPTY + kQStages, COL_FULL = REC_FULL + kColStages, COL_EMPTY = COL_FULL + kColStages,
       SD_FULL = COL_EMPTY + kColStages, PDS_FULL = SD_FULL + 2, DONE_A = PDS_FULL + 2, DONE_B = DONE_A + 2,
       DS_EMPTY = DONE_B + 2, KV_DONE = DS_EMPTY + 2, ACC_EMPTY = KV_DONE + 1, FINAL = ACC_EMPTY + 1, EPI = FINAL + 2,
       NB = EPI + 1 };

// per-tile summary of the query records, written by the column warp
struct alignas(16) ColStats {
  int lo_max[4], lo_min[4], qi_min[4], qi_max[4];  // per 16-column quarter: mask skipping
  float wlo_min[4];
  int elo_min[4], ehi_max[4];  // per quarter: the soft-edge keys of its columns lie in [elo_min, ehi_max]
};

template <int D>
struct alignas(1024) Smem {
  uint8_t k[BM * D * 2];
  uint8_t v[BM * D * 2];
  uint8_t q[kQStages][BN * D * 2];
  uint8_t dO[kQStages][BN * D * 2];
  // the two dSᵀ tile buffers of the scratch stores; in the band epilogue the
  // staging area of one dK or dV block (D ≤ 128)
  uint8_t stage[2 * BM * BN * 2];
  uint64_t bars[NB];
  uint32_t tmem_base;
  int abort_flag;
  QRec rec[kColStages][BN];  // the tile's query records (bulk-copied, then fixed up)
  ColStats stats[kColStages];
  float dlw_part[4][BM];  // landmark items: d_lw partial sums of the four column quarters
};
static_assert(2 * BM * BN * 2 >= BM * 128 * 2, "the dSᵀ buffers hold one staged dK or dV block (D ≤ 128)");

// One work item: 128 keys (a band block, or a chunk of sorted landmark slots with
// one part of its query range) of one (sequence, head), and its query tiles.
// Every role of the persistent CTA decodes the same items in the same order.
struct Item {
  int h, s, key0, nkeys, q_start, n_tiles, part, L;
  int blk, chunk, u0;  // band: block_map index; landmark: 128-slot chunk and its first query tile
  int64_t s0, lbase;
};

template <bool LMK>
__device__ __forceinline__ int num_items(const DsaltAttnParams& p) {
  if (LMK) return p.S * ((p.kp + BM - 1) / BM) * DSALT_LMK_SPLIT * p.H;
  return __ldg(p.num_blocks) * p.H;
}

// Decode item idx (any single thread may call it).
template <bool LMK>
__device__ __forceinline__ Item decode_item(const DsaltAttnParams& p, int idx) {
  Item it;
  it.part = 0;
  if (LMK) {
    const int nch = (p.kp + BM - 1) / BM;
    const int per_h = p.S * nch * DSALT_LMK_SPLIT;
    it.h = idx / per_h;
    const int x = idx % per_h;
    it.part = x % DSALT_LMK_SPLIT;
    it.s = x / DSALT_LMK_SPLIT / nch;
    const int chunk = x / DSALT_LMK_SPLIT % nch;
    it.s0 = __ldg(p.cu_seqlens + it.s);
    it.L = (int)(__ldg(p.cu_seqlens + it.s + 1) - it.s0);
    it.lbase = ((int64_t)it.h * p.S + it.s) * p.kp;
    it.key0 = chunk * BM;
    // valid slots are a prefix of the sorted list: the chunk's first invalid slot by bisection
    int lo_c = it.key0, hi_c = min(it.key0 + BM, p.kp);
    while (lo_c < hi_c) {
      const int mid = (lo_c + hi_c) >> 1;
      if (__ldg(p.pos_sorted + it.lbase + mid) >= 0) lo_c = mid + 1; else hi_c = mid;
    }
    const int nv = lo_c - it.key0;
    it.nkeys = nv;
    it.chunk = chunk;
    it.blk = 0;
    // query tiles from the 128-query block of the first slot's position to the
    // sequence end (aligned to the dQ stage's query blocks; the columns before
    // the first slot attend nothing), split into DSALT_LMK_SPLIT parts of whole
    // tile pairs
    const int first = nv > 0 ? __ldg(p.pos_sorted + it.lbase + it.key0) : 0;
    const int qs = (first / BM) * BM;
    const int n = nv > 0 ? (it.L - qs + BN - 1) / BN : 0;
    const int per = ((n + DSALT_LMK_SPLIT - 1) / DSALT_LMK_SPLIT + 1) & ~1;
    const int u0 = per * it.part;
    it.n_tiles = max(0, min(n, u0 + per) - u0);
    it.u0 = u0;
    it.q_start = qs + BN * u0;
  } else {
    const int nb = __ldg(p.num_blocks);
    const int blk = idx % nb;
    it.h = idx / nb;
    it.blk = blk;
    it.chunk = 0;
    it.u0 = 0;
    it.s = __ldg(p.block_map + 2 * blk);
    it.s0 = __ldg(p.cu_seqlens + it.s);
    it.L = (int)(__ldg(p.cu_seqlens + it.s + 1) - it.s0);
    it.key0 = __ldg(p.block_map + 2 * blk + 1) * BM;
    it.nkeys = min(BM, it.L - it.key0);
    it.q_start = it.key0;
    it.lbase = ((int64_t)it.h * p.S + it.s) * p.kp;
    const int q_end = min(it.L - 1, it.key0 + BM - 1 + max(__ldg(p.seq_wmax + it.s), 0));
    it.n_tiles = q_end >= it.q_start ? (q_end - it.q_start + BN) / BN : 0;
  }
  return it;
}

// Index of tile u of an item in the ds_tiles scratch (the dQ stage's layout,
// attn_tc_dq.cu): band tiles per (head, block_map index), landmark tiles per
// (head, sequence, chunk) counted from the chunk's first query block; -1 when
// the caller's ds_band_tiles / ds_lmk_tiles leave no room for it.
template <bool LMK>
__device__ __forceinline__ int64_t ds_tile_index(const DsaltAttnParams& p, const Item& it, int u) {
  if (LMK) {
    const int ul = it.u0 + u;
    if (ul >= p.ds_lmk_tiles) return -1;
    const int nch = (p.kp + BM - 1) / BM;
    return (int64_t)p.H * p.max_blocks * p.ds_band_tiles +
           (((int64_t)it.h * p.S + it.s) * nch + it.chunk) * p.ds_lmk_tiles + ul;
  }
  if (u >= p.ds_band_tiles) return -1;
  return ((int64_t)it.h * p.max_blocks + it.blk) * p.ds_band_tiles + u;
}

template <bool LMK, typename T, int D>
__global__ void __launch_bounds__(kThreadsKV, 1) tc_bwd_dkdv_kernel(const __grid_constant__ BwdArgs a) {
  using namespace sm100;
  const DsaltAttnParams& p = a.p;
  // persistent CTA: items blockIdx.x, blockIdx.x + gridDim.x, …
  const int n_items = num_items<LMK>(p);
  if ((int)blockIdx.x >= n_items) return;  // CTA-uniform, before any barrier or TMEM use

  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBF16 = !std::is_same<T, __half>::value;
  const BarArray bar{smem_u32(&sm.bars[0])};
  if (tid == 0) {
    // barriers completed by tcgen05.commit get one arrival from each MMA warp
    mbar_init(bar[KV_FULL], 1);
    mbar_init(bar[KV_EMPTY], 2);
    for (int st = 0; st < kQStages; ++st) {
      mbar_init(bar[Q_FULL + st], 1);
      mbar_init(bar[DO_FULL + st], 1);
      mbar_init(bar[QDO_EMPTY + st], 2);
    }
    for (int st = 0; st < kColStages; ++st) {
      mbar_init(bar[REC_FULL + st], 1);
      mbar_init(bar[COL_FULL + st], 32);
      mbar_init(bar[COL_EMPTY + st], kRowThreads);
    }
    for (int st = 0; st < 2; ++st) {
      mbar_init(bar[SD_FULL + st], 2);
      mbar_init(bar[PDS_FULL + st], kRowThreads);
      mbar_init(bar[DONE_A + st], 1);    // dV of the buffer's tile completed (its Pᵀ is read)
      mbar_init(bar[DONE_B + st], 1);    // dK of the buffer's tile completed (its dSᵀ is read)
      mbar_init(bar[DS_EMPTY + st], 1);  // the store lane's copy has read the shared dSᵀ buffer
    }
    mbar_init(bar[KV_DONE], 3);  // both MMA warps, and the store warp (the item's last tile copied)
    mbar_init(bar[ACC_EMPTY], kRowThreads);
    mbar_init(bar[FINAL], 1);
    mbar_init(bar[FINAL + 1], 1);
    mbar_init(bar[EPI], kRowThreads);
    fence_mbar_init();
    sm.abort_flag = 0;
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&sm.tmem_base), 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  const uint32_t tS = tmem, tdP = tmem + 2 * BN, tdK = tmem + 4 * BN, tdV = tmem + 4 * BN + D;
  const float inv_tau = 1.0f / p.tau_win;
  const int stride = gridDim.x;

  if (warp == kProducerWarp && lane == 0) {
    // ---------------------------------------------------- TMA lane: per item K/V, then the global Q/dO ring
    int gt = 0, gi = 0, g_issued = 0, kv_issued = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride) {
      const Item it = decode_item<LMK>(p, idx);
      if (it.n_tiles == 0) continue;
      if (gi >= 1) ok = mbar_wait(bar[KV_EMPTY], (gi - 1) & 1, abort_flag, p.status);
      if (ok) {
        const uint32_t kv_bytes = (LMK ? a.lmk_box : BM) * D * 2;
        mbar_expect_tx(bar[KV_FULL], 2 * kv_bytes);
#pragma unroll
        for (int c = 0; c < D / 64; ++c) {
          if (LMK) {
            tma_load_3d(smem_u32(sm.k + c * (BM * 128)), &a.tm_lk, bar[KV_FULL], c * 64, it.key0, it.h * p.S + it.s);
            tma_load_3d(smem_u32(sm.v + c * (BM * 128)), &a.tm_lv, bar[KV_FULL], c * 64, it.key0, it.h * p.S + it.s);
          } else {
            tma_load_3d(smem_u32(sm.k + c * (BM * 128)), &a.tm_k, bar[KV_FULL], c * 64, attn_kv_head(p, it.h),
                        (int)(it.s0 + it.key0));
            tma_load_3d(smem_u32(sm.v + c * (BM * 128)), &a.tm_v, bar[KV_FULL], c * 64, attn_kv_head(p, it.h),
                        (int)(it.s0 + it.key0));
          }
        }
        kv_issued = gi + 1;
      }
      for (int u = 0; ok && u < it.n_tiles; ++u) {
        const int g = gt + u, st = g % kQStages;
        if (g >= kQStages && !mbar_wait(bar[QDO_EMPTY + st], (g / kQStages - 1) & 1, abort_flag, p.status)) {
          ok = false;
          break;
        }
        const int q0 = it.q_start + BN * u;
        mbar_expect_tx(bar[Q_FULL + st], BN * D * 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(smem_u32(sm.q[st] + c * (BN * 128)), &a.tm_q, bar[Q_FULL + st], c * 64, it.h,
                      (int)(it.s0 + q0));
        mbar_expect_tx(bar[DO_FULL + st], BN * D * 2);
#pragma unroll
        for (int c = 0; c < D / 64; ++c)
          tma_load_3d(smem_u32(sm.dO[st] + c * (BN * 128)), &a.tm_do, bar[DO_FULL + st], c * 64, it.h,
                      (int)(it.s0 + q0));
        g_issued = g + 1;
      }
      gt += it.n_tiles;
      ++gi;
    }
    // never leave a TMA write in flight into shared memory
    for (int g = max(0, g_issued - kQStages); g < g_issued; ++g) {
      mbar_drain(bar[Q_FULL + g % kQStages], (g / kQStages) & 1);
      mbar_drain(bar[DO_FULL + g % kQStages], (g / kQStages) & 1);
    }
    if (kv_issued > 0) mbar_drain(bar[KV_FULL], (kv_issued - 1) & 1);
  } else if (warp == kProducerWarp && lane == 1) {
    // ---------------------------------------------------- store lane: dSᵀ tiles to the scratch
    // Bulk-copies each finished dSᵀ tile from its shared buffer (tile g in buffer
    // g % 2) to the ds_tiles scratch that the dQ stage reads, and releases the
    // buffer (DS_EMPTY) once the copy has read it; after an item's last tile it
    // also completes KV_DONE, so that the epilogue's staging never overwrites a
    // tile that is still being copied.
    int gt = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride) {
      const Item it = decode_item<LMK>(p, idx);
      const int n = it.n_tiles;
      if (n == 0) continue;
      for (int u = 0; ok && u < n; ++u) {
        const int g = gt + u, st = g & 1;
        ok = mbar_wait(bar[PDS_FULL + st], (g >> 1) & 1, abort_flag, p.status);
        if (!ok) break;
        bool stored = false;
        if (p.ds_tiles) {
          const int64_t ti = ds_tile_index<LMK>(p, it, u);
          if (ti >= 0) {
            bulk_store(reinterpret_cast<uint8_t*>(p.ds_tiles) + ti * DSALT_DS_TILE_BYTES,
                       smem_u32(sm.stage + st * (BM * BN * 2)), DSALT_DS_TILE_BYTES);
            bulk_commit();
            stored = true;
          } else {
            flag_status(p.status, DSALT_DEV_BAD_INDEX);
          }
        }
        if (stored) bulk_wait_read0();  // the buffer is read: the rows may overwrite it
        mbar_arrive(bar[DS_EMPTY + st]);
      }
      if (ok) mbar_arrive(bar[KV_DONE]);
      gt += n;
    }
    bulk_wait_all();  // every tile store completes before the exit
  } else if (warp == kColWarp) {
    // ---------------------------------------------------- column warp: per-tile query records
    // Lane 0 bulk-copies each tile's records (written by the preprocess stage)
    // kColStages − 1 tiles ahead, across items; the warp then masks the columns
    // past the sequence end and summarises the tile for the row warps.
    struct Cur {
      int idx, u;
      Item it;
    };
    auto seek = [&](Cur& c) {  // first item with tiles at or after c.idx
      while (c.idx < n_items) {
        c.it = decode_item<LMK>(p, c.idx);
        if (c.it.n_tiles > 0) return;
        c.idx += stride;
      }
    };
    auto advance = [&](Cur& c) {
      if (++c.u < c.it.n_tiles) return;
      c.u = 0;
      c.idx += stride;
      seek(c);
    };
    auto issue = [&](const Cur& c, int g) {
      const int st = g % kColStages;
      const int q0 = c.it.q_start + BN * c.u;
      const QRec* recg = reinterpret_cast<const QRec*>(p.qrec) + (int64_t)c.it.h * p.T + c.it.s0;
      const int nrec = (int)min((int64_t)BN, p.T - (c.it.s0 + q0));  // never read past the array
      mbar_expect_tx(bar[REC_FULL + st], nrec * (uint32_t)sizeof(QRec));
      bulk_load(smem_u32(&sm.rec[st][0]), recg + q0, nrec * (uint32_t)sizeof(QRec), bar[REC_FULL + st]);
    };
    Cur ci{(int)blockIdx.x, 0, Item{}}, cp{(int)blockIdx.x, 0, Item{}};
    seek(ci);
    seek(cp);
    int g_issued = 0;
    for (; ci.idx < n_items && g_issued < kColStages - 1; ++g_issued, advance(ci))
      if (lane == 0) issue(ci, g_issued);
    for (int g = 0; cp.idx < n_items; ++g, advance(cp)) {
      const int st = g % kColStages;
      if (!__all_sync(0xffffffffu, mbar_wait(bar[REC_FULL + st], (g / kColStages) & 1, abort_flag, p.status)))
        break;
      const int q0 = cp.it.q_start + BN * cp.u;
      // per lane: columns lane (quarter lane/16) and lane + 32 (quarter 2 + lane/16)
      int st_lo_max[2], st_lo_min[2], st_qi_min[2], st_qi_max[2], st_elo_min[2], st_ehi_max[2];
      float st_wlo_min[2];
#pragma unroll
      for (int k2 = 0; k2 < 2; ++k2) {
        const int c = lane + 32 * k2;
        QRec& rc = sm.rec[st][c];
        if (q0 + c >= cp.it.L) {  // another sequence's query (or past the array): no pairs
          rc.nlse2 = 0.f; rc.delta = 0.f; rc.lo = INT_MAX; rc.qi = INT_MIN;
          rc.wlo = -INFINITY; rc.ehi = INT_MIN; rc.elo = INT_MAX;
        }
        const int clo = rc.lo, ci_ = rc.qi;
        st_lo_max[k2] = clo; st_lo_min[k2] = clo; st_qi_min[k2] = ci_; st_qi_max[k2] = ci_; st_wlo_min[k2] = rc.wlo;
        st_elo_min[k2] = rc.elo; st_ehi_max[k2] = rc.ehi;
      }
#pragma unroll
      for (int off = 8; off > 0; off >>= 1) {  // within 16-lane groups
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          st_lo_max[k2] = max(st_lo_max[k2], __shfl_xor_sync(0xffffffffu, st_lo_max[k2], off));
          st_lo_min[k2] = min(st_lo_min[k2], __shfl_xor_sync(0xffffffffu, st_lo_min[k2], off));
          st_qi_min[k2] = min(st_qi_min[k2], __shfl_xor_sync(0xffffffffu, st_qi_min[k2], off));
          st_qi_max[k2] = max(st_qi_max[k2], __shfl_xor_sync(0xffffffffu, st_qi_max[k2], off));
          st_wlo_min[k2] = fminf(st_wlo_min[k2], __shfl_xor_sync(0xffffffffu, st_wlo_min[k2], off));
          st_elo_min[k2] = min(st_elo_min[k2], __shfl_xor_sync(0xffffffffu, st_elo_min[k2], off));
          st_ehi_max[k2] = max(st_ehi_max[k2], __shfl_xor_sync(0xffffffffu, st_ehi_max[k2], off));
        }
      }
      if ((lane & 15) == 0) {
        ColStats& cs = sm.stats[st];
#pragma unroll
        for (int k2 = 0; k2 < 2; ++k2) {
          const int qq = 2 * k2 + (lane >> 4);
          cs.lo_max[qq] = st_lo_max[k2]; cs.lo_min[qq] = st_lo_min[k2];
          cs.qi_min[qq] = st_qi_min[k2]; cs.qi_max[qq] = st_qi_max[k2]; cs.wlo_min[qq] = st_wlo_min[k2];
          cs.elo_min[qq] = st_elo_min[k2]; cs.ehi_max[qq] = st_ehi_max[k2];
        }
      }
      mbar_arrive(bar[COL_FULL + st]);
      // refill the stage of tile g − 1 with the next tile once the rows released it
      if (ci.idx < n_items) {
        const int ng = g_issued;  // == g + kColStages − 1
        if (ng >= kColStages &&
            !__all_sync(0xffffffffu,
                        mbar_wait(bar[COL_EMPTY + ng % kColStages], (ng / kColStages - 1) & 1, abort_flag, p.status)))
          break;
        if (lane == 0) issue(ci, ng);
        ++g_issued;
        advance(ci);
      }
    }
    if (lane == 0)
      for (int g = max(0, g_issued - kColStages); g < g_issued; ++g)
        mbar_drain(bar[REC_FULL + g % kColStages], (g / kColStages) & 1);
  } else if (warp == kMmaWarp || warp == kMmaWarpB) {
    // ---------------------------------------------------- MMA issuers
    // Two warps issue so that their MMAs overlap (one issuing thread sustains
    // only about one MMA per 110 cycles): warp A issues Sᵀ = K·Qᵀ and
    // dV += Pᵀ·dO, warp B dPᵀ = V·dOᵀ and dK += dSᵀ·Q.  Barriers they both
    // complete count two arrivals.  Pᵀ / dSᵀ of tile g sit in the TMEM buffer
    // g % 2 of Sᵀ / dPᵀ, so a warp issues Sᵀ / dPᵀ of tile g + 2 into that buffer
    // only after its own dV / dK MMA of tile g completed (DONE_A / DONE_B).  An
    // item's first two Sᵀ / dPᵀ run while the row warps still store the previous
    // item (its accumulators are only overwritten after the epilogue released
    // them: ACC_EMPTY).
    const bool is_a = warp == kMmaWarp;
    const uint32_t id_s = idesc_f16(kBF16, BM, BN, false, false);
    const uint32_t id_kv = idesc_f16(kBF16, BM, D, false, true);
    const uint32_t kv_addr = smem_u32(is_a ? sm.k : sm.v);
    const uint32_t t_sd = is_a ? tS : tdP, t_acc = is_a ? tdV : tdK;
    const int done = is_a ? DONE_A : DONE_B;
    // operand tiles: Sᵀ reads Q, dPᵀ reads dO; dV reads dO, dK reads Q
    auto tile_sd = [&](int qs) { return smem_u32(is_a ? sm.q[qs] : sm.dO[qs]); };
    auto tile_acc = [&](int qs) { return smem_u32(is_a ? sm.dO[qs] : sm.q[qs]); };
    auto issue_sd = [&](int g) -> bool {
      const int st = g & 1, qs = g % kQStages;
      if (!mbar_wait(bar[(is_a ? Q_FULL : DO_FULL) + qs], (g / kQStages) & 1, abort_flag, p.status)) return false;
      if (g >= 2 && !mbar_wait(bar[done + st], ((g >> 1) - 1) & 1, abort_flag, p.status)) return false;
      tc_fence_after();
      const uint32_t ba = tile_sd(qs);
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const uint32_t aoff = (kk >> 2) * (BM * 128) + (kk & 3) * 32;
        const uint32_t boff = (kk >> 2) * (BN * 128) + (kk & 3) * 32;
        mma_f16(t_sd + st * BN, sdesc_sw128(kv_addr + aoff, 16, 1024), sdesc_sw128(ba + boff, 16, 1024), id_s,
                kk > 0 ? 1u : 0u);
      }
      mma_commit(bar[SD_FULL + st]);
      return true;
    };
    int gt = 0, gi = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride) {
      const Item it = decode_item<LMK>(p, idx);
      const int n = it.n_tiles;
      if (n == 0) continue;
      if (lane == 0) {
        ok = mbar_wait(bar[KV_FULL], gi & 1, abort_flag, p.status);
        if (ok) ok = issue_sd(gt);
        if (ok && n > 1) ok = issue_sd(gt + 1);
        if (ok && n <= 2) mma_commit(bar[KV_EMPTY]);  // every Sᵀ / dPᵀ of the item is issued
        for (int u = 0; ok && u < n; ++u) {
          const int g = gt + u, qs = g % kQStages;
          ok = mbar_wait(bar[PDS_FULL + (g & 1)], (g >> 1) & 1, abort_flag, p.status) &&
               mbar_wait(bar[(is_a ? DO_FULL : Q_FULL) + qs], (g / kQStages) & 1, abort_flag, p.status) &&
               (u > 0 || gi == 0 || mbar_wait(bar[ACC_EMPTY], (gi - 1) & 1, abort_flag, p.status));
          if (!ok) break;
          tc_fence_after();
          const uint32_t ba = tile_acc(qs);
          // A = Pᵀ / dSᵀ in TMEM: K step kk (queries 16·kk …) in columns 16·kk … 16·kk + 7
          // of the buffer, where the row warps of quarter kk wrote them
#pragma unroll
          for (int kk = 0; kk < BN / 16; ++kk)
            mma_f16_tmem_a(t_acc, t_sd + (g & 1) * BN + kQuarter * kk, sdesc_sw128(ba + kk * 2048, BN * 128, 1024),
                           id_kv, (u > 0 || kk > 0) ? 1u : 0u);
          mma_commit(bar[done + (g & 1)]);
          mma_commit(bar[QDO_EMPTY + qs]);
          if (u + 2 < n) {
            ok = issue_sd(g + 2);
            if (ok && u + 2 == n - 1) mma_commit(bar[KV_EMPTY]);
          }
        }
        if (ok) mma_commit(bar[KV_DONE]);
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
      gt += n;
      ++gi;
    }
    if (lane == 0) {
      // every issued MMA completes before TMEM is released
      mma_commit(bar[FINAL + (is_a ? 0 : 1)]);
      mbar_drain(bar[FINAL + (is_a ? 0 : 1)], 0);
    }
  } else if (warp < kRowWarps) {
    // ---------------------------------------------------- key-row warps (Pᵀ, dSᵀ)
    const int r = 32 * (warp & 3) + lane;  // key row / TMEM lane
    const int quarter = warp >> 2;
    const int c0 = kQuarter * quarter;     // this thread's first column of a tile
    const uint32_t lane_addr = ((uint32_t)(32 * (warp & 3)) << 16);
    const float sl2 = p.scale * kLog2e;
    int gt = 0, gi = 0, epi_phase = 0;
    bool ok = true;
    // all row threads meet (bounded wait on the EPI barrier)
    auto rows_sync = [&]() -> bool {
      mbar_arrive(bar[EPI]);
      const bool w = mbar_wait(bar[EPI], epi_phase & 1, abort_flag, p.status);
      ++epi_phase;
      return __all_sync(0xffffffffu, w);
    };
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride) {
      const Item it = decode_item<LMK>(p, idx);
      const int n = it.n_tiles, key0 = it.key0, nkeys = it.nkeys, h = it.h;
      const int64_t s0 = it.s0, lbase = it.lbase;
      const bool key_ok = r < nkeys;
      const int j = LMK ? (key_ok ? __ldg(p.pos_sorted + lbase + key0 + r) : INT_MAX) : key0 + r;
      if (n == 0) {
        // a landmark part without queries: its partial sums are zero
        if (LMK && key_ok) {
          const int64_t slot = it.part * a.part_stride + lbase + key0 + r;
          const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
          for (int e = 0; e < D / 4; e += 4) {
            *reinterpret_cast<float4*>(a.dk_lmk + slot * D + quarter * (D / 4) + e) = z;
            *reinterpret_cast<float4*>(a.dv_lmk + slot * D + quarter * (D / 4) + e) = z;
          }
          if (quarter == 0) a.dlw_lmk[slot] = 0.f;
        }
        continue;
      }
      const float lw2 = (LMK && key_ok) ? __ldg(p.w_sorted + lbase + key0 + r) * kLog2e : 0.f;
      // first landmark slot at this key (band items; -1: none), used by the epilogue
      const int cl_first = (!LMK && key_ok && p.lmk_slot) ? __ldg(p.lmk_slot + (s0 + j) * p.H + h) : -1;
      // key range of this warp's 32 rows (band: consecutive; landmarks: sorted positions)
      const int jf = LMK ? __shfl_sync(0xffffffffu, j, 0) : key0 + 32 * (warp & 3);
      const int jl = LMK ? __reduce_max_sync(0xffffffffu, key_ok ? j : INT_MIN) : jf + 31;
      const bool warp_keys_ok = __all_sync(0xffffffffu, key_ok);
      const float jfl = (float)j;
      float dlw = 0.f;
      for (int u = 0; u < n; ++u) {
        const int g = gt + u, st = g & 1, cs = g % kColStages;
        ok = mbar_wait(bar[SD_FULL + st], (g >> 1) & 1, abort_flag, p.status) &&
             mbar_wait(bar[COL_FULL + cs], (g / kColStages) & 1, abort_flag, p.status);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
        const QRec* rec = &sm.rec[cs][c0];
        const ColStats& cst = sm.stats[cs];
        bool all_in, all_out;
        if (LMK) {
          all_in = warp_keys_ok && cst.qi_min[quarter] >= jl && cst.wlo_min[quarter] > (float)jl;
          all_out = false;
        } else {
          all_in = cst.lo_max[quarter] <= jf && cst.qi_min[quarter] >= jl;
          all_out = cst.lo_min[quarter] > jl || cst.qi_max[quarter] < jf;
        }
        // band items: bit c of emask is set when column c0 + c has soft-edge keys
        // among this warp's 32 keys (warp-uniform; a column's edge is a few keys,
        // so few bits are set)
        uint32_t emask = 0u;
        if (!LMK) {
          bool hit = false;
          if (lane < kQuarter) {
            const int2 eb = *reinterpret_cast<const int2*>(&rec[lane].ehi);  // ehi, elo
            hit = eb.y <= eb.x && eb.y <= jl && eb.x >= jf;
          }
          emask = __ballot_sync(0xffffffffu, hit);
        }
        // Pᵀ and dSᵀ of this thread's 16 columns, packed to the input dtype
        uint32_t pk_p[8], pk_d[8];
        if (all_out) {
#pragma unroll
          for (int q = 0; q < 8; ++q) { pk_p[q] = 0u; pk_d[q] = 0u; }
        } else {
          float sv[16], dpv[16];
          tmem_ld16(tS + lane_addr + st * BN + c0, sv);
          tmem_ld16(tdP + lane_addr + st * BN + c0, dpv);
          tmem_wait_ld();
          // the all-valid case (warp-uniform) runs without the per-element test
          auto body = [&](auto kAllIn) {
            constexpr bool kIn = decltype(kAllIn)::value;
#pragma unroll
            for (int c = 0; c < 16; c += 2) {
              float pr2[2], ds2[2];
#pragma unroll
              for (int e = 0; e < 2; ++e) {
                const QRec& rq = rec[c + e];
                // nlse2, delta (and lo, qi only where a column can be invalid)
                float4 r0;
                if (kIn) {
                  const float2 h2 = *reinterpret_cast<const float2*>(&rq.nlse2);
                  r0 = make_float4(h2.x, h2.y, 0.f, 0.f);
                } else {
                  r0 = *reinterpret_cast<const float4*>(&rq.nlse2);
                }
                bool valid;
                float pr;
                if (LMK) {
                  pr = fast_exp2(fmaf(sv[c + e], sl2, lw2 + r0.x));
                  valid = kIn || (key_ok && j <= __float_as_int(r0.w) && jfl < rq.wlo);
                } else {
                  pr = fast_exp2(fmaf(sv[c + e], sl2, r0.x));
                  valid = kIn || (j >= __float_as_int(r0.z) && j <= __float_as_int(r0.w));
                }
                const float dsv = pr * (dpv[c + e] - r0.y);
                pr2[e] = valid ? pr : 0.f;
                ds2[e] = valid ? dsv : 0.f;
                if (LMK) dlw += ds2[e];
              }
              pk_p[c / 2] = pack2(pr2[0], pr2[1], kBF16);
              pk_d[c / 2] = pack2(ds2[0], ds2[1], kBF16);
            }
          };
          if (all_in) body(std::true_type{}); else body(std::false_type{});
        }
        // soft window edge (band items, the columns of emask only, after the
        // straight-line pass above): Pᵀ, dSᵀ *= σ((w̃ − d)/τ) on the column's edge
        // keys elo … ehi, applied to the rounded entries (factor ehi − j of the
        // record, or computed past the stored ones)
        // (branch-free per column: lanes outside the edge multiply by 1, which leaves
        // an entry's bits unchanged)
        for (uint32_t m = emask; m != 0u; m &= m - 1u) {  // warp-uniform
          const int c = __ffs(m) - 1;
          const QRec& rq = rec[c];
          const int2 eb = *reinterpret_cast<const int2*>(&rq.ehi);  // ehi, elo
          const bool ed = j >= eb.y && j <= eb.x;
          float gf;
          if (eb.x - eb.y < kMaxEdge) {  // warp-uniform: every factor stored
            const float f = rq.eg[(uint32_t)(eb.x - j) & (uint32_t)(kMaxEdge - 1)];
            gf = ed ? f : 1.0f;
          } else {
            const int ei = eb.x - j;
            gf = !ed ? 1.0f : ei < kMaxEdge ? rq.eg[ei] : qrec_edge_factor(rq.wt, rq.qi - j, inv_tau);
          }
          const int w2 = c >> 1, sh = (c & 1) * 16;
          uint32_t wp = 0u, wd = 0u;
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (i == w2) { wp = pk_p[i]; wd = pk_d[i]; }
          wp = (wp & ~(0xffffu << sh)) | (f32_to_bits<T>(bits_to_f32<T>(wp >> sh) * gf) << sh);
          wd = (wd & ~(0xffffu << sh)) | (f32_to_bits<T>(bits_to_f32<T>(wd >> sh) * gf) << sh);
#pragma unroll
          for (int i = 0; i < 8; ++i)
            if (i == w2) { pk_p[i] = wp; pk_d[i] = wd; }
        }
        // the shared dSᵀ buffer g % 2 is free once the store lane has read its
        // previous tile
        if (g >= 2) {
          ok = mbar_wait(bar[DS_EMPTY + st], ((g >> 1) - 1) & 1, abort_flag, p.status);
          if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        }
        // Pᵀ, dSᵀ over this quarter's own (already read) Sᵀ, dPᵀ columns: the
        // A operand of K step `quarter` of the dV / dK MMAs
        tmem_st8u(tS + lane_addr + st * BN + c0, pk_p);
        tmem_st8u(tdP + lane_addr + st * BN + c0, pk_d);
        // the dSᵀ tile for the dQ stage: row r, columns c0 … c0 + 15 of the
        // 128B-swizzled shared buffer
        {
          uint8_t* dsb = sm.stage + st * (BM * BN * 2);
          *reinterpret_cast<uint4*>(dsb + sw128_offset(r, c0)) = make_uint4(pk_d[0], pk_d[1], pk_d[2], pk_d[3]);
          *reinterpret_cast<uint4*>(dsb + sw128_offset(r, c0 + 8)) = make_uint4(pk_d[4], pk_d[5], pk_d[6], pk_d[7]);
        }
        tmem_wait_st();
        tc_fence_before();
        fence_async_smem();  // the store lane's bulk copy reads the buffer
        mbar_arrive(bar[PDS_FULL + st]);
        mbar_arrive(bar[COL_EMPTY + cs]);
      }
      if (!ok) break;
      ok = __all_sync(0xffffffffu, mbar_wait(bar[KV_DONE], gi & 1, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      // this thread handles dK/dV columns [quarter·D/4, (quarter+1)·D/4) of key row r
      if (LMK) {
        const int64_t slot = it.part * a.part_stride + lbase + key0 + r;
        float* dkl = a.dk_lmk + slot * D;
        float* dvl = a.dv_lmk + slot * D;
#pragma unroll
        for (int ch = 0; ch < D / 64; ++ch) {
          const int col = quarter * (D / 4) + ch * 16;
          float kk_[16], vv[16];
          tmem_ld16(tdK + lane_addr + col, kk_);
          tmem_ld16(tdV + lane_addr + col, vv);
          tmem_wait_ld();
          if (key_ok) {
#pragma unroll
            for (int e = 0; e < 16; e += 4) {
              *reinterpret_cast<float4*>(dkl + col + e) =
                  make_float4(kk_[e] * p.scale, kk_[e + 1] * p.scale, kk_[e + 2] * p.scale, kk_[e + 3] * p.scale);
              *reinterpret_cast<float4*>(dvl + col + e) = make_float4(vv[e], vv[e + 1], vv[e + 2], vv[e + 3]);
            }
          }
        }
        tc_fence_before();
        mbar_arrive(bar[ACC_EMPTY]);
        // d_lw of the slot: sum of the four column quarters, in quarter order
        sm.dlw_part[quarter][r] = dlw;
        ok = rows_sync();
        if (quarter == 0 && key_ok)
          a.dlw_lmk[slot] = ok ? ((sm.dlw_part[0][r] + sm.dlw_part[1][r]) + (sm.dlw_part[2][r] + sm.dlw_part[3][r]))
                               : 0.f;
        ok = ok && rows_sync();  // dlw_part is reused by the next item
      } else {
        // dK, then dV: the rows are staged in shared memory, 16-byte units
        // XOR-swizzled by row % 8, and stored row-contiguously.  A key that
        // holds landmark slots (first slot cl_first) also leaves its fp32 rows in
        // the band scratch: lmk_fixup_kernel adds the landmark pass's parts to them
        // and rounds once.
        constexpr int kUnits = D * 2 / 16;
        uint8_t* stage = sm.stage;
        const int64_t HD = (int64_t)p.H * D;
#pragma unroll 1
        for (int m = 0; ok && m < 2; ++m) {
          const uint32_t tacc = m == 0 ? tdK : tdV;
          const float mul = m == 0 ? p.scale : 1.0f;
          float* bl = cl_first >= 0 ? a.band_lmk + (m == 0 ? 0 : a.part_stride * D) + (lbase + cl_first) * D
                                    : nullptr;
#pragma unroll 1
          for (int ch = 0; ch < D / 64; ++ch) {  // 16 columns at a time
            const int col = quarter * (D / 4) + ch * 16;
            float x[16];
            tmem_ld16(tacc + lane_addr + col, x);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) x[e] *= mul;
            if (bl) {
#pragma unroll
              for (int e = 0; e < 16; e += 4)
                *reinterpret_cast<float4*>(bl + col + e) = make_float4(x[e], x[e + 1], x[e + 2], x[e + 3]);
            }
#pragma unroll
            for (int e = 0; e < 16; e += 8) {
              const int un = (col + e) / 8;
              uint4 u0;
              u0.x = pack2(x[e], x[e + 1], kBF16); u0.y = pack2(x[e + 2], x[e + 3], kBF16);
              u0.z = pack2(x[e + 4], x[e + 5], kBF16); u0.w = pack2(x[e + 6], x[e + 7], kBF16);
              *reinterpret_cast<uint4*>(stage + r * (kUnits * 16) + ((un ^ (r & 7)) << 4)) = u0;
            }
          }
          if (m == 1) {
            tc_fence_before();
            mbar_arrive(bar[ACC_EMPTY]);  // both accumulators are read
          }
          ok = rows_sync();
          if (!ok) break;
          uint8_t* dst = reinterpret_cast<uint8_t*>(m == 0 ? p.dk : p.dv) + ((s0 + key0) * HD + (int64_t)h * D) * 2;
          for (int un = tid; un < nkeys * kUnits; un += kRowThreads) {
            const int rr = un / kUnits, uu = un % kUnits;
            *reinterpret_cast<uint4*>(dst + rr * HD * 2 + uu * 16) =
                *reinterpret_cast<const uint4*>(stage + rr * (kUnits * 16) + ((uu ^ (rr & 7)) << 4));
          }
          ok = rows_sync();  // the staging area is reused (dV, or the next item's dSᵀ tiles)
        }
      }
      gt += n;
      ++gi;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 512);
}

// Keys holding landmark slots: dK / dV = round(band rows + Σ over the key's slots
// (duplicates are adjacent) and over the landmark pass's query-range parts, in
// that fixed order); d_lw of every slot = Σ over its parts (0 for an empty slot).  One warp per
// (slot, sequence, head): blockIdx.x = s·ceil(kp/4) + slot/4; D/32 columns per lane.
template <typename T, int D>
__global__ void __launch_bounds__(128) lmk_fixup_kernel(const BwdArgs a) {
  const DsaltAttnParams& p = a.p;
  const int nq = (p.kp + 3) / 4;
  const int s = blockIdx.x / nq, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = 4 * (blockIdx.x % nq) + warp;
  if (c >= p.kp) return;
  const int64_t lbase = ((int64_t)h * p.S + s) * p.kp;
  const int64_t s0 = __ldg(p.cu_seqlens + s);
  constexpr int kCols = D / 32;
  const float* band_v = a.band_lmk + a.part_stride * D;
  {
    const int pos = __ldg(p.pos_sorted + lbase + c);
    // every caller slot sits at one sorted position (empty ones last): its d_lw,
    // 0 for an empty slot, is written here
    if (lane == 0 && p.d_lw) {
      const int slot_c = __ldg(p.perm + lbase + c);
      if (slot_c >= 0) {
        float g = 0.f;
        if (pos >= 0)
          for (int pp = 0; pp < DSALT_LMK_SPLIT; ++pp) g += __ldg(a.dlw_lmk + pp * a.part_stride + lbase + c);
        p.d_lw[((int64_t)h * p.S + s) * p.k_lmk + slot_c] = p.grad_round ? round_to<T>(g) : g;
      }
    }
    if (pos < 0) return;  // an invalid slot
    if (c > 0 && __ldg(p.pos_sorted + lbase + c - 1) == pos) return;  // not the first slot of its key
    float kk[kCols], vv[kCols];
    const int col0 = lane * kCols;
#pragma unroll
    for (int e = 0; e < kCols; ++e) {
      kk[e] = __ldg(a.band_lmk + (lbase + c) * D + col0 + e);
      vv[e] = __ldg(band_v + (lbase + c) * D + col0 + e);
    }
    for (int cc = c; cc < p.kp && __ldg(p.pos_sorted + lbase + cc) == pos; ++cc)
      for (int pp = 0; pp < DSALT_LMK_SPLIT; ++pp) {
        const float* lk = a.dk_lmk + (pp * a.part_stride + lbase + cc) * D + col0;
        const float* lv = a.dv_lmk + (pp * a.part_stride + lbase + cc) * D + col0;
#pragma unroll
        for (int e = 0; e < kCols; ++e) { kk[e] += __ldg(lk + e); vv[e] += __ldg(lv + e); }
      }
    const int64_t row = ((s0 + pos) * p.H + h) * D + col0;
    T* dk = reinterpret_cast<T*>(p.dk) + row;
    T* dv = reinterpret_cast<T*>(p.dv) + row;
#pragma unroll
    for (int e = 0; e < kCols; ++e) { dk[e] = from_f32<T>(kk[e]); dv[e] = from_f32<T>(vv[e]); }
  }
}
}  // namespace dkv

// ---------------------------------------------------------------- host side
CUresult encode_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1, uint64_t d2,
                   uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0, uint32_t box1, uint32_t box2) {
  return encode_tensor_map_3d(m, dt, base, d0, d1, d2, stride1_bytes, stride2_bytes, box0, box1, box2);
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
  // k, v: [T, H_kv, D] (grouped kv heads read in place; dk, dv stay per query head)
  const uint64_t hkv = (uint64_t)attn_kv_heads(p), kvrow = hkv * D * 2;
  if (encode_3d(&a.tm_k, dt, p.k, D, hkv, p.T, row, kvrow, 64, 1, rows_k) != CUDA_SUCCESS) return false;
  if (encode_3d(&a.tm_v, dt, p.v, D, hkv, p.T, row, kvrow, 64, 1, rows_k) != CUDA_SUCCESS) return false;
  const int kp = p.kp > 0 ? p.kp : 16;
  a.lmk_box = kp < rows_l ? kp : rows_l;
  const void* lk = p.kp > 0 ? p.lmk_k : p.k;
  const void* lv = p.kp > 0 ? p.lmk_v : p.v;
  const uint64_t hs = p.kp > 0 ? (uint64_t)p.H * p.S : 1;
  if (encode_3d(&a.tm_lk, dt, lk, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS) return false;
  if (encode_3d(&a.tm_lv, dt, lv, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS) return false;
  return true;
}

// Non-blocking stream per device on which the landmark pass runs next to the band
// pass, and the two events that fork it from and join it back into the caller's
// stream; created once per device and reused (a wait uses the event's latest
// record), so the entry point is meant for one host thread per device.
static cudaError_t side_stream(cudaStream_t* out, cudaEvent_t* fork, cudaEvent_t* join) {
  static std::mutex mu;
  static cudaStream_t streams[64] = {};
  static cudaEvent_t forks[64] = {}, joins[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!streams[dev]) {
    e = cudaStreamCreateWithFlags(&streams[dev], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&forks[dev], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&joins[dev], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      streams[dev] = nullptr;
      return e;
    }
  }
  *out = streams[dev];
  *fork = forks[dev];
  *join = joins[dev];
  return cudaSuccess;
}

// multiprocessor count of the current device (cached)
static cudaError_t sm_count(int* out) {
  static int counts[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (counts[dev] <= 0) {
    e = cudaDeviceGetAttribute(&counts[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
  }
  *out = counts[dev];
  return cudaSuccess;
}

template <typename T, int D>
cudaError_t launch_dkdv(const DsaltAttnParams& p, float* lmk_scratch, cudaStream_t st) {
  BwdArgs a;
  if (!make_args<T, D>(a, p, dkv::BN, dkv::BM, dkv::BM)) return cudaErrorInvalidValue;
  a.part_stride = (int64_t)p.H * p.S * p.kp;
  const int64_t part_floats = DSALT_LMK_SPLIT * a.part_stride * D;
  a.dk_lmk = lmk_scratch;
  a.dv_lmk = lmk_scratch ? lmk_scratch + part_floats : nullptr;
  a.dlw_lmk = lmk_scratch ? lmk_scratch + 2 * part_floats : nullptr;
  a.band_lmk = lmk_scratch ? a.dlw_lmk + DSALT_LMK_SPLIT * a.part_stride : nullptr;
  const size_t smem = std::max(sizeof(dkv::Smem<D>) + 1024, (size_t)(116 * 1024));
  cudaError_t e;
  if (p.ds_tiles) {
    // the all-zero tile the dQ stage reads in place of a tile that was never stored
    const int64_t zero = DSALT_DS_TILES(p.H, p.max_blocks, p.S, p.kp, p.ds_band_tiles, p.ds_lmk_tiles) - 1;
    e = cudaMemsetAsync(reinterpret_cast<uint8_t*>(p.ds_tiles) + zero * DSALT_DS_TILE_BYTES, 0,
                        DSALT_DS_TILE_BYTES, st);
    if (e != cudaSuccess) return e;
  }
  const bool lmk = p.kp > 0 && p.S > 0;
  // the landmark pass (under-filled grid) runs on a side stream next to the band pass
  cudaEvent_t fork = nullptr, join = nullptr;
  if (lmk) {
    cudaStream_t side;
    e = side_stream(&side, &fork, &join);
    if (e == cudaSuccess) e = cudaEventRecord(fork, st);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(side, fork, 0);
    if (e == cudaSuccess)
      e = ensure_smem((const void*)dkv::tc_bwd_dkdv_kernel<true, T, D>, smem);
    if (e == cudaSuccess) {
      const int nch = (p.kp + dkv::BM - 1) / dkv::BM;
      const unsigned items = (unsigned)(p.S * nch * DSALT_LMK_SPLIT * p.H);  // one item per CTA
      dkv::tc_bwd_dkdv_kernel<true, T, D><<<items, dkv::kThreadsKV, smem, side>>>(a);
      e = cudaGetLastError();
    }
    if (e == cudaSuccess) e = cudaEventRecord(join, side);
    if (e != cudaSuccess) return e;
  }
  e = ensure_smem((const void*)dkv::tc_bwd_dkdv_kernel<false, T, D>, smem);
  if (e == cudaSuccess) {
    // persistent: one CTA per SM walks the band items (block, head) round-robin
    int sms = 0;
    e = sm_count(&sms);
    if (e == cudaSuccess) {
      const long long items = (long long)p.max_blocks * p.H;
      const unsigned grid = (unsigned)std::min<long long>(items, sms);
      dkv::tc_bwd_dkdv_kernel<false, T, D><<<grid, dkv::kThreadsKV, smem, st>>>(a);
      e = cudaGetLastError();
    }
  }
  if (lmk) {
    // join before anything can fail past this point, so the caller's stream never runs ahead of the side work
    const cudaError_t ej = cudaStreamWaitEvent(st, join, 0);
    if (e == cudaSuccess) e = ej;
    if (e == cudaSuccess) {
      dkv::lmk_fixup_kernel<T, D><<<dim3((unsigned)(p.S * ((p.kp + 3) / 4)), (unsigned)p.H), 128, 0, st>>>(a);
      e = cudaGetLastError();
    }
  }
  return e;
}

}  // namespace bwd

// lmk_scratch: the caller's fp32 buffer (((2·D + 1)·DSALT_LMK_SPLIT + 2·D)·H·S·kp
// floats) for the partial landmark-slot dK / dV / d_lw of the landmark pass and
// the band pass's fp32 rows of the keys that hold landmark slots.
cudaError_t tc_bwd_stage(int stage, const DsaltAttnParams& p, float* lmk_scratch, cudaStream_t st) {
  const bool bf = p.dtype == DSALT_BF16;
  if (stage == 3) return tc_bwd_dq_stage(p, st);
  if (stage == 2) {
    if (p.kp > 0 && !lmk_scratch) return cudaErrorInvalidValue;
    if (bf) return p.D == 64 ? bwd::launch_dkdv<__nv_bfloat16, 64>(p, lmk_scratch, st)
                             : bwd::launch_dkdv<__nv_bfloat16, 128>(p, lmk_scratch, st);
    return p.D == 64 ? bwd::launch_dkdv<__half, 64>(p, lmk_scratch, st)
                     : bwd::launch_dkdv<__half, 128>(p, lmk_scratch, st);
  }
  return simt_attention_stage(stage, p, st);
}

}  // namespace dsalt
