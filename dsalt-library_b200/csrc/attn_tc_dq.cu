// dQ stage of the tensor-core backward for sm_100a: dQ = scale · Σ dS·K over the
// dSᵀ tiles that the dK/dV stage stored.
//
// The dK/dV stage (attn_tc_bwd.cu) computes every dSᵀ tile of the band and the
// landmark pass once, applies the soft window edge and stores the tile (128 keys
// × 64 queries, 16-bit, in the 128-byte-swizzled layout of a K-major shared-memory
// operand tile) to the ds_tiles scratch.  Here each work item is one 128-query block of
// one head: for every key block (and landmark chunk) whose dK/dV item covered
// the block, the two stored 64-query tiles and the 128-row K tile are loaded
// (bulk copy and TMA) and one tcgen05.mma chain accumulates dQ in TMEM:
//   A = dS   (M = 128 queries, K = 16 keys per MMA): the stored dSᵀ tiles read
//            MN-major (queries contiguous), the two tiles at 16 KB apart;
//   B = K    (K = 16 keys, N = D): the TMA-loaded key tile, MN-major.
// No exponentials and no S/dP recomputation: this replaces the query-parallel
// recompute of the reference's _train_bwd_kernel (dsalt/kernels/
// dsalt_triton_train.py:240-383, dQ at :335-368; landmark part :302-333).
// ∂loss/∂w̃ of each query row is formed here too, by the epilogue thread of the
// row: Σ over the row's soft-edge keys, in a fixed order, of dS·(1 − σ)/τ, read
// back from the stored σ-scaled dSᵀ entries (reference :371-383), one store per
// (token, head), no atomics.
//
// Persistent CTAs (one per SM), items (head, query block) round-robin, two TMEM
// accumulators so that one item's epilogue overlaps the next item's MMAs.
//   warp 0      producer: bulk copies of the dSᵀ tile pairs, TMA of the K tiles
//   warp 1      TMEM owner, single-thread MMA issuer
//   warps 2-5   epilogue: TMEM lane quadrant warp % 4, dQ rows scaled, rounded,
//               staged in shared memory and stored row-contiguously
// Every wait is bounded (sm100::mbar_wait).
#include <algorithm>

#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {

cudaError_t simt_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st);

namespace dq2 {

constexpr int BM = 128;                 // queries per item (TMEM lanes)
constexpr int KB = 128;                 // keys per band work unit (one dK/dV key block)
constexpr int kTile = DSALT_DS_TILE_BYTES;
constexpr int kStages = 3;
constexpr int kThreads = 192;
constexpr int kProducerWarp = 0, kMmaWarp = 1, kEpiWarp0 = 2;
constexpr int kEpiThreads = 128;
enum { FULL = 0, EMPTY = FULL + kStages, ACC_FULL = EMPTY + kStages, ACC_EMPTY = ACC_FULL + 2, EPI = ACC_EMPTY + 2,
       FINAL = EPI + 1, NB = FINAL + 1 };

template <int D>
struct alignas(1024) Smem {
  uint8_t ds[kStages][2 * kTile];   // the item's two 64-query dSᵀ tiles of one key block
  uint8_t k[kStages][KB * D * 2];   // key tile: D/64 chunks of [rows × 128 B]
  uint8_t stage[BM * D * 2];        // epilogue staging of the 16-bit dQ rows
  uint64_t bars[NB];
  uint32_t tmem_base;
  int abort_flag;
};

struct alignas(64) DqArgs {
  CUtensorMap tm_k, tm_lk;
  DsaltAttnParams p;
  int lmk_box;  // rows of one landmark TMA box: min(kp, 128)
};

// One work item: 128 queries of one (sequence, head).
struct Item {
  int h, blk, s, qb, L, nvalid;
  int64_t s0, lbase;
};

__device__ __forceinline__ Item decode(const DsaltAttnParams& p, int idx, int nb) {
  Item it;
  it.blk = idx % nb;
  it.h = idx / nb;
  it.s = __ldg(p.block_map + 2 * it.blk);
  it.qb = __ldg(p.block_map + 2 * it.blk + 1);
  it.s0 = __ldg(p.cu_seqlens + it.s);
  it.L = (int)(__ldg(p.cu_seqlens + it.s + 1) - it.s0);
  it.lbase = ((int64_t)it.h * p.S + it.s) * p.kp;
  it.nvalid = 0;
  return it;
}

// valid landmark slots of (head, sequence): a prefix of the sorted list (whole warp)
__device__ __forceinline__ int count_valid(const DsaltAttnParams& p, int64_t lbase) {
  const int lane = threadIdx.x & 31;
  int nv = 0;
  for (int c0 = 0; c0 < p.kp; c0 += 32) {
    const int c = c0 + lane;
    nv += __popc(__ballot_sync(0xffffffffu, c < p.kp && __ldg(p.pos_sorted + lbase + c) >= 0));
  }
  return nv;
}

// A work unit: the global indices of its two dSᵀ tiles (-1: the zero tile) and its K rows.
struct Unit {
  int64_t t0, t1;  // tile indices into ds_tiles
  bool lmk;
  int krow;        // band: first key (in the sequence); landmark: first slot of the chunk
  int nk;          // MMA K extent (multiple of 16)
};

// Units of an item, in a fixed order: landmark chunks, then key blocks ascending.
// Mirrors the tiles the dK/dV stage stored (decode_item in attn_tc_bwd.cu):
//   band key block kb: query tiles from 128·kb, n = ceil((min(L − 1, 128·kb + 127 + wmax) − 128·kb + 1) / 64);
//   landmark chunk c: query tiles from 128·floor(first slot position / 128) to L − 1.
// Calls f(const Unit&) for each; returns the number of units.
template <typename F>
__device__ __forceinline__ int for_units(const DsaltAttnParams& p, const Item& it, F&& f) {
  const int m0 = it.qb * BM;
  int n = 0;
  const int nch = (p.kp + 127) / 128;
  const int64_t band_total = (int64_t)p.H * p.max_blocks * p.ds_band_tiles;
  for (int c = 0; c < nch; ++c) {
    const int nv = min(max(it.nvalid - 128 * c, 0), 128);
    if (nv == 0) break;
    const int first = __ldg(p.pos_sorted + it.lbase + 128 * c);
    const int qs = (first / BM) * BM;
    if (m0 < qs) continue;
    const int ntile = (it.L - qs + 63) / 64;
    const int u = (m0 - qs) / 64;
    if (u >= ntile || u >= p.ds_lmk_tiles) continue;
    const int64_t base = band_total + (((int64_t)it.h * p.S + it.s) * nch + c) * p.ds_lmk_tiles;
    Unit un;
    un.t0 = base + u;
    un.t1 = (u + 1 < ntile && u + 1 < p.ds_lmk_tiles) ? base + u + 1 : -1;
    un.lmk = true;
    un.krow = 128 * c;
    un.nk = (nv + 15) & ~15;
    f(un);
    ++n;
  }
  const int wmax = max(__ldg(p.seq_wmax + it.s), 0);
  const int kb_lo = max(0, it.qb - (p.ds_band_tiles + 1) / 2);
  for (int kb = kb_lo; kb <= it.qb; ++kb) {
    const int key0 = kb * KB;
    const int q_end = min(it.L - 1, key0 + KB - 1 + wmax);
    const int ntile = min(q_end >= key0 ? (q_end - key0 + 64) / 64 : 0, p.ds_band_tiles);
    const int u = 2 * (it.qb - kb);
    if (u >= ntile) continue;
    const int64_t base = ((int64_t)it.h * p.max_blocks + (it.blk - (it.qb - kb))) * p.ds_band_tiles;
    Unit un;
    un.t0 = base + u;
    un.t1 = u + 1 < ntile ? base + u + 1 : -1;
    un.lmk = false;
    un.krow = key0;
    un.nk = KB;
    f(un);
    ++n;
  }
  return n;
}

template <typename T, int D>
__global__ void __launch_bounds__(kThreads, 1) tc_bwd_dq_kernel(const __grid_constant__ DqArgs a) {
  using namespace sm100;
  const DsaltAttnParams& p = a.p;
  const int nb = __ldg(p.num_blocks);
  const int n_items = nb * p.H;
  if ((int)blockIdx.x >= n_items) return;  // CTA-uniform, before any barrier or TMEM use

  extern __shared__ uint8_t smem_raw[];
  Smem<D>& sm = *reinterpret_cast<Smem<D>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr bool kBF16 = !std::is_same<T, __half>::value;
  const BarArray bar{smem_u32(&sm.bars[0])};
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(bar[FULL + st], 1);
      mbar_init(bar[EMPTY + st], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar[ACC_FULL + b], 1);
      mbar_init(bar[ACC_EMPTY + b], kEpiThreads);
    }
    mbar_init(bar[EPI], kEpiThreads);
    mbar_init(bar[FINAL], 1);
    fence_mbar_init();
    sm.abort_flag = 0;
  }
  if (warp == kMmaWarp) tmem_alloc(smem_u32(&sm.tmem_base), 2 * D);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  volatile int* abort_flag = &sm.abort_flag;
  const int stride = gridDim.x;
  const uint8_t* ds_base = reinterpret_cast<const uint8_t*>(p.ds_tiles);
  const int64_t zero_tile = (int64_t)p.H * p.max_blocks * p.ds_band_tiles +
                            (int64_t)p.H * p.S * ((p.kp + 127) / 128) * p.ds_lmk_tiles;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ loads
    int g = 0, g_issued = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride) {
      Item it = decode(p, idx, nb);
      it.nvalid = p.kp > 0 ? count_valid(p, it.lbase) : 0;
      if (lane == 0) {
        for_units(p, it, [&](const Unit& un) {
          if (!ok) return;
          const int st = g % kStages;
          if (g >= kStages && !mbar_wait(bar[EMPTY + st], (g / kStages - 1) & 1, abort_flag, p.status)) {
            ok = false;
            return;
          }
          const int krows = un.lmk ? a.lmk_box : KB;
          mbar_expect_tx(bar[FULL + st], 2 * kTile + krows * D * 2);
          bulk_load(smem_u32(sm.ds[st]), ds_base + un.t0 * kTile, kTile, bar[FULL + st]);
          bulk_load(smem_u32(sm.ds[st] + kTile), ds_base + (un.t1 >= 0 ? un.t1 : zero_tile) * kTile, kTile,
                    bar[FULL + st]);
#pragma unroll
          for (int c = 0; c < D / 64; ++c) {
            if (un.lmk)
              tma_load_3d(smem_u32(sm.k[st] + c * (krows * 128)), &a.tm_lk, bar[FULL + st], c * 64, un.krow,
                          it.h * p.S + it.s);
            else
              tma_load_3d(smem_u32(sm.k[st] + c * (KB * 128)), &a.tm_k, bar[FULL + st], c * 64,
                          attn_kv_head(p, it.h), (int)(it.s0 + un.krow));
          }
          ++g;
          g_issued = g;
        });
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0)  // never leave a copy in flight into shared memory
      for (int gg = max(0, g_issued - kStages); gg < g_issued; ++gg)
        mbar_drain(bar[FULL + gg % kStages], (gg / kStages) & 1);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    const uint32_t idesc = idesc_f16(kBF16, BM, D, true, true);
    int g = 0, li = 0;
    bool ok = true;
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride, ++li) {
      Item it = decode(p, idx, nb);
      it.nvalid = p.kp > 0 ? count_valid(p, it.lbase) : 0;
      if (lane == 0) {
        const int acc = li & 1;
        const uint32_t tacc = tmem + acc * D;
        if (li >= 2) ok = mbar_wait(bar[ACC_EMPTY + acc], ((li >> 1) - 1) & 1, abort_flag, p.status);
        bool first = true;
        if (ok) {
          for_units(p, it, [&](const Unit& un) {
            if (!ok) return;
            const int st = g % kStages;
            if (!mbar_wait(bar[FULL + st], (g / kStages) & 1, abort_flag, p.status)) {
              ok = false;
              return;
            }
            tc_fence_after();
            const uint32_t a_addr = smem_u32(sm.ds[st]), b_addr = smem_u32(sm.k[st]);
            const uint32_t b_lbo = (un.lmk ? a.lmk_box : KB) * 128;
            for (int kk = 0; kk < un.nk / 16; ++kk) {
              mma_f16(tacc, sdesc_sw128(a_addr + kk * 2048, kTile, 1024), sdesc_sw128(b_addr + kk * 2048, b_lbo, 1024),
                      idesc, first ? 0u : 1u);
              first = false;
            }
            mma_commit(bar[EMPTY + st]);
            ++g;
          });
        }
        if (ok) mma_commit(bar[ACC_FULL + acc]);  // also for an item without units (nothing accumulated)
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) {
      mma_commit(bar[FINAL]);
      mbar_drain(bar[FINAL], 0);
    }
  } else {
    // ------------------------------------------------------------ epilogue (128 threads)
    const int q4 = warp & 3;                  // TMEM lane quadrant of this warp
    const int r = 32 * q4 + lane;             // query row of the item
    const int et = tid - 32 * kEpiWarp0;      // 0..127
    const uint32_t lane_addr = (uint32_t)(32 * q4) << 16;
    constexpr int kUnits = D * 2 / 16;        // 16-byte units per dQ row
    const float inv_tau = 1.0f / p.tau_win;
    int li = 0, epi_phase = 0;
    bool ok = true;
    auto epi_sync = [&]() -> bool {
      mbar_arrive(bar[EPI]);
      const bool w = mbar_wait(bar[EPI], epi_phase & 1, abort_flag, p.status);
      ++epi_phase;
      return __all_sync(0xffffffffu, w);
    };
    for (int idx = blockIdx.x; ok && idx < n_items; idx += stride, ++li) {
      Item it = decode(p, idx, nb);
      it.nvalid = p.kp > 0 ? count_valid(p, it.lbase) : 0;
      const int n_units = for_units(p, it, [](const Unit&) {});
      const int acc = li & 1;
      const int m0 = it.qb * BM;
      const int rows = min(BM, it.L - m0);
      // ∂loss/∂w̃ of query row r, its loads issued before the wait for the
      // accumulator: edge key j = ehi − e (summed in the order of e) sits in key
      // block kb = j / 128, query tile u = (q − 128·kb) / 64 of that block's band
      // tiles, entry (j − 128·kb, q − 128·kb − 64·u) of the tile image
      const bool dw_row = p.dw_head != nullptr && r < rows;
      QRec rc;
      rc.elo = INT_MAX;
      rc.ehi = INT_MIN;
      if (dw_row) {
        const float4* rp = reinterpret_cast<const float4*>(p.qrec + ((int64_t)it.h * p.T + it.s0 + m0 + r) *
                                                                        DSALT_QREC_FLOATS);
        float4* rcv = reinterpret_cast<float4*>(&rc);
#pragma unroll
        for (int k = 0; k < DSALT_QREC_FLOATS / 4; ++k) rcv[k] = __ldg(rp + k);
      }
      const int ne = qrec_ne(rc);
      auto edge_entry = [&](int e) -> float {  // the stored dS·σ of edge key ehi − e (0 past the scratch)
        const int q = m0 + r, j = rc.ehi - e;
        const int kb = j / KB, u = (q - kb * KB) / 64;
        if (u >= p.ds_band_tiles) return 0.f;
        const int64_t tile = ((int64_t)it.h * p.max_blocks + (it.blk - (it.qb - kb))) * p.ds_band_tiles + u;
        return to_f32<T>(*reinterpret_cast<const T*>(ds_base + tile * kTile +
                                                      sm100::sw128_offset(j - kb * KB, q - kb * KB - 64 * u)));
      };
      float dwv[kQRecEdge];
#pragma unroll
      for (int e = 0; e < kQRecEdge; ++e) dwv[e] = e < ne ? edge_entry(e) : 0.f;
      ok = __all_sync(0xffffffffu, mbar_wait(bar[ACC_FULL + acc], (li >> 1) & 1, abort_flag, p.status));
      if (!ok) break;
      tc_fence_after();
      // dQ row r → staging (16-byte units XOR-swizzled by row % 8)
#pragma unroll 1
      for (int ch = 0; ch < D / 32; ++ch) {
        float x[32];
        if (n_units > 0) {
          tmem_ld32(tmem + acc * D + lane_addr + ch * 32, x);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) x[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          const int un = (ch * 32 + j) / 8;
          uint4 u;
          u.x = pack2(x[j + 0] * p.scale, x[j + 1] * p.scale, kBF16);
          u.y = pack2(x[j + 2] * p.scale, x[j + 3] * p.scale, kBF16);
          u.z = pack2(x[j + 4] * p.scale, x[j + 5] * p.scale, kBF16);
          u.w = pack2(x[j + 6] * p.scale, x[j + 7] * p.scale, kBF16);
          *reinterpret_cast<uint4*>(sm.stage + r * (kUnits * 16) + ((un ^ (r & 7)) << 4)) = u;
        }
      }
      tc_fence_before();
      mbar_arrive(bar[ACC_EMPTY + acc]);  // this accumulator is read: the MMA warp may reuse it
      if (!(ok = epi_sync())) break;
      const int64_t HD = (int64_t)p.H * D;
      uint8_t* dqg = reinterpret_cast<uint8_t*>(p.dq) + ((it.s0 + m0) * HD + (int64_t)it.h * D) * 2;
      for (int un = et; un < rows * kUnits; un += kEpiThreads) {
        const int rr = un / kUnits, uu = un % kUnits;
        *reinterpret_cast<uint4*>(dqg + rr * HD * 2 + uu * 16) =
            *reinterpret_cast<const uint4*>(sm.stage + rr * (kUnits * 16) + ((uu ^ (rr & 7)) << 4));
      }
      if (dw_row) {
        float dw = 0.f;
#pragma unroll
        for (int e = 0; e < kQRecEdge; ++e) dw += dwv[e] * (1.0f - rc.eg[e]) * inv_tau;
        for (int e = kQRecEdge; e < ne; ++e)
          dw += edge_entry(e) * (1.0f - qrec_edge_factor(rc.wt, rc.qi - (rc.ehi - e), inv_tau)) * inv_tau;
        p.dw_head[(it.s0 + m0 + r) * p.H + it.h] = dw;
      }
      if (!(ok = epi_sync())) break;  // the staging area is reused by the next item
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, 2 * D);
}

}  // namespace dq2

CUresult encode_tensor_map_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                              uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                              uint32_t box1, uint32_t box2);

namespace {
// multiprocessor count of the current device (cached)
cudaError_t sm_count_dq(int* out) {
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
cudaError_t launch_dq2(const DsaltAttnParams& p, cudaStream_t st) {
  dq2::DqArgs a;
  memset(&a, 0, sizeof(a));
  a.p = p;
  const CUtensorMapDataType dt = std::is_same<T, __half>::value ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                                 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  const uint64_t row = (uint64_t)D * 2;
  const uint64_t hkv = (uint64_t)attn_kv_heads(p);  // k: [T, H_kv, D]
  if (encode_tensor_map_3d(&a.tm_k, dt, p.k, D, hkv, p.T, row, hkv * D * 2, 64, 1, dq2::KB) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const int kp = p.kp > 0 ? p.kp : 16;
  a.lmk_box = kp < 128 ? kp : 128;
  const void* lk = p.kp > 0 ? p.lmk_k : p.k;
  const uint64_t hs = p.kp > 0 ? (uint64_t)p.H * p.S : 1;
  if (encode_tensor_map_3d(&a.tm_lk, dt, lk, D, kp, hs, row, (uint64_t)kp * row, 64, a.lmk_box, 1) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const size_t smem = sizeof(dq2::Smem<D>) + 1024;
  cudaError_t e = ensure_smem((const void*)dq2::tc_bwd_dq_kernel<T, D>, smem);
  if (e != cudaSuccess) return e;
  int sms = 0;
  e = sm_count_dq(&sms);
  if (e != cudaSuccess) return e;
  const long long items = (long long)p.max_blocks * p.H;
  const unsigned grid = (unsigned)std::max<long long>(1, std::min<long long>(items, sms));
  dq2::tc_bwd_dq_kernel<T, D><<<grid, dq2::kThreads, smem, st>>>(a);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  if (p.dw && p.dw_head) return simt_attention_stage(4, p, st);  // dw = Σ_h dw_head
  return cudaSuccess;
}
}  // namespace

// dQ from the stored dSᵀ tiles (stage 3 of the tensor-core family)
cudaError_t tc_bwd_dq_stage(const DsaltAttnParams& p, cudaStream_t st) {
  if (!p.ds_tiles || p.ds_band_tiles <= 0 || (p.kp > 0 && p.ds_lmk_tiles <= 0)) return cudaErrorInvalidValue;
  if (p.dtype == DSALT_BF16)
    return p.D == 64 ? launch_dq2<__nv_bfloat16, 64>(p, st) : launch_dq2<__nv_bfloat16, 128>(p, st);
  return p.D == 64 ? launch_dq2<__half, 64>(p, st) : launch_dq2<__half, 128>(p, st);
}

}  // namespace dsalt
