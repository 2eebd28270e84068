// Packed-batch scheduling and landmark gathering.
//
// build_schedule replaces the host-side, (total, num_seqs)-keyed caches of the
// reference (dsalt/kernels/selectors.py:15-67): the (sequence, block) table is
// rebuilt on the device from the actual cu_seqlens every call, so batches with
// equal totals but different lengths can never share a stale table, and no
// device-to-host copy is needed.
//
// gather_landmarks replaces _build_landmark_kv (selectors.py:137-159) and the
// landmark padding (dsalt_triton_train.py:44-68); it also sorts the landmarks
// of each (head, sequence) by position so that the attended landmark set of
// every query is a prefix of the sorted list.
#include "common.cuh"

namespace dsalt {

// One CTA: per-sequence block counts, exclusive scan, table fill; also clears
// the band maxima that seq_meta_kernel (launched after it) raises.
__global__ void __launch_bounds__(1024) build_block_map_kernel(DsaltScheduleParams p) {
  __shared__ int32_t warp_tot[32];
  __shared__ int32_t carry;
  const int tid = threadIdx.x;
  if (tid == 0) carry = 0;
  if (p.seq_wmax) {
    for (int b = tid; b < p.S; b += 1024) p.seq_wmax[b] = 0;
    if (tid == 0 && p.seq_wmax_batch) *p.seq_wmax_batch = 0;
  }
  __syncthreads();
  for (int base = 0; base < p.S; base += 1024) {
    const int b = base + tid;
    int nb = 0;
    if (b < p.S) {
      const int len = p.cu_seqlens[b + 1] - p.cu_seqlens[b];
      nb = len > 0 ? (len + p.block - 1) / p.block : 0;
    }
    // block-wide inclusive scan
    int v = nb;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xffffffffu, v, o);
      if ((tid & 31) >= o) v += n;
    }
    if ((tid & 31) == 31) warp_tot[tid >> 5] = v;
    __syncthreads();
    if (tid < 32) {
      int wv = warp_tot[tid];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, wv, o);
        if (tid >= o) wv += n;
      }
      warp_tot[tid] = wv;
    }
    __syncthreads();
    const int excl = carry + v - nb + ((tid >> 5) ? warp_tot[(tid >> 5) - 1] : 0);
    if (b < p.S) {
      for (int k = 0; k < nb; ++k) {
        const int e = excl + k;
        if (e < p.max_blocks) {
          p.block_map[2 * e] = b;
          p.block_map[2 * e + 1] = k;
        }
      }
    }
    __syncthreads();
    if (tid == 1023) carry = excl + nb;
    __syncthreads();
  }
  if (tid == 0) *p.num_blocks = min(carry, p.max_blocks);
}

// Per token: its sequence id and the running per-sequence max band length.  A
// warp whose 32 tokens lie in one sequence (the common case) reduces its maximum
// first and issues one atomic; a warp across a boundary issues one per token.
// The batch maximum is raised only by a value that raised its sequence's: every
// final seq_wmax[s] reaches it, with a few atomics per sequence on one word.
__global__ void seq_meta_kernel(DsaltScheduleParams p) {
  const int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const bool valid = t < p.T;
  int s = -1, W = 0;
  if (valid) {
    s = find_seq(p.cu_seqlens, p.S, t);
    if (p.seq_id) p.seq_id[t] = s;
    const int i = (int)(t - p.cu_seqlens[s]);
    const RowWindow rw = row_window(p.w[t], i, p.semantics, 0.0f);
    W = max(min(rw.W, i), 0);
  }
  if (!p.seq_wmax) return;  // uniform over the grid
  const int s0 = __shfl_sync(0xffffffffu, s, 0);
  if (__all_sync(0xffffffffu, s == s0)) {
    const int m = __reduce_max_sync(0xffffffffu, W);
    if ((threadIdx.x & 31) == 0 && s0 >= 0 && m > 0 && atomicMax(p.seq_wmax + s0, m) < m && p.seq_wmax_batch)
      atomicMax(p.seq_wmax_batch, m);
  } else if (valid && W > 0) {
    if (atomicMax(p.seq_wmax + s, W) < W && p.seq_wmax_batch) atomicMax(p.seq_wmax_batch, W);
  }
}

cudaError_t launch_schedule(const DsaltScheduleParams& p, cudaStream_t st) {
  build_block_map_kernel<<<1, 1024, 0, st>>>(p);
  if (p.T > 0 && (p.seq_wmax || p.seq_id))
    seq_meta_kernel<<<(unsigned)((p.T + 255) / 256), 256, 0, st>>>(p);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ gather
// gridDim.x = H·S CTAs groups, one per (head, sequence); gridDim.y CTAs share
// the group's row copies.  Each CTA ranks the k slots itself (k <= 1024, in
// shared memory); the y = 0 CTA writes the sorted metadata.
template <typename T>
__global__ void __launch_bounds__(256) gather_landmarks_kernel(DsaltGatherParams p) {
  extern __shared__ int64_t sm_keys[];  // [k] sort keys, then [kp] sorted positions (int32)
  int32_t* spos = reinterpret_cast<int32_t*>(sm_keys + p.k_lmk);
  const int h = blockIdx.x / p.S;
  const int s = blockIdx.x % p.S;
  const bool meta = blockIdx.y == 0;
  const int64_t s0 = p.cu_seqlens[s];
  const int L = (int)(p.cu_seqlens[s + 1] - s0);
  const int64_t in_base = ((int64_t)h * p.S + s) * p.k_lmk;
  const int64_t out_base = ((int64_t)h * p.S + s) * p.kp;

  for (int c = threadIdx.x; c < p.k_lmk; c += blockDim.x) {
    const int64_t pos = p.lmk_pos[in_base + c];
    const bool valid = pos >= 0 && pos < L;
    if (meta && pos >= L) flag_status(p.status, DSALT_DEV_BAD_INDEX);
    sm_keys[c] = valid ? pos : (int64_t)1 << 40;
  }
  __syncthreads();
  // rank = number of entries before this one in (position, slot) order
  for (int c = threadIdx.x; c < p.k_lmk; c += blockDim.x) {
    const int64_t key = sm_keys[c];
    int rank = 0;
    for (int c2 = 0; c2 < p.k_lmk; ++c2) {
      const int64_t k2 = sm_keys[c2];
      rank += (k2 < key) || (k2 == key && c2 < c);
    }
    const bool valid = key < ((int64_t)1 << 40);
    spos[rank] = valid ? (int32_t)key : -1;
    if (!meta) continue;
    p.pos_sorted[out_base + rank] = valid ? (int32_t)key : -1;
    p.w_sorted[out_base + rank] = p.lmk_w[in_base + c];
    p.perm[out_base + rank] = c;
    if (valid) {
      // first of a run of equal positions owns the reverse-map entry
      bool first = true;
      for (int c2 = 0; c2 < p.k_lmk; ++c2) {
        const int64_t k2 = sm_keys[c2];
        if (k2 == key && c2 < c) { first = false; break; }
      }
      if (first) p.lmk_slot[(s0 + key) * p.H + h] = rank;
    }
  }
  for (int c = p.k_lmk + threadIdx.x; c < p.kp; c += blockDim.x) {
    spos[c] = -1;
    if (!meta) continue;
    p.pos_sorted[out_base + c] = -1;
    p.w_sorted[out_base + c] = 0.f;
    p.perm[out_base + c] = -1;
  }
  __syncthreads();
  // gather rows (16-byte vectors): sorted slot r copies token spos[r]; this CTA
  // takes rows [r0, r1) of the group
  const int vec = 16 / (int)sizeof(T);
  const int nvec = p.D / vec;
  const int per = (p.kp + gridDim.y - 1) / gridDim.y;
  const int r0 = blockIdx.y * per, r1 = min(p.kp, r0 + per);
  // k, v: [T, H_kv, D]; query head h reads kv head h / (H / H_kv)
  const int hkv = p.H_kv > 0 ? p.H_kv : p.H;
  const int64_t HD = (int64_t)hkv * p.D;
  const int g = h / (p.H / hkv);
  const uint4* ksrc = reinterpret_cast<const uint4*>(p.k);
  const uint4* vsrc = reinterpret_cast<const uint4*>(p.v);
  uint4* kdst = reinterpret_cast<uint4*>(p.lmk_k);
  uint4* vdst = reinterpret_cast<uint4*>(p.lmk_v);
  for (int e = r0 * nvec + threadIdx.x; e < r1 * nvec; e += blockDim.x) {
    const int r = e / nvec, c = e % nvec;
    const int pos = spos[r];
    uint4 kv = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
    if (pos >= 0) {
      const int64_t src = ((s0 + pos) * HD + (int64_t)g * p.D) / vec + c;
      kv = ksrc[src];
      vv = vsrc[src];
    }
    const int64_t dst = ((out_base + r) * p.D) / vec + c;
    kdst[dst] = kv;
    vdst[dst] = vv;
  }
}

cudaError_t launch_gather(const DsaltGatherParams& p, cudaStream_t st) {
  if (p.H * p.S == 0) return cudaSuccess;
  const size_t smem = sizeof(int64_t) * (size_t)max(p.k_lmk, 1) + sizeof(int32_t) * (size_t)max(p.kp, 1);
  // about two CTAs per SM in all, at least 8 rows per CTA
  const int groups = p.H * p.S;
  const int ny = max(1, min((p.kp + 7) / 8, (2 * 148 + groups - 1) / groups));
  const dim3 grid((unsigned)groups, (unsigned)ny);
  switch (p.dtype) {
    case DSALT_F16: gather_landmarks_kernel<__half><<<grid, 256, smem, st>>>(p); break;
    case DSALT_BF16: gather_landmarks_kernel<__nv_bfloat16><<<grid, 256, smem, st>>>(p); break;
    case DSALT_F32: gather_landmarks_kernel<float><<<grid, 256, smem, st>>>(p); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace dsalt
