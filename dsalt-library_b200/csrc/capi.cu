// extern "C" entry points of libdsalt_b200.so: argument checks, then launches.
// No entry point allocates device memory; every buffer belongs to the caller.
#include <cudaTypedefs.h>
#include <mutex>

#include "common.cuh"
#include "sm100.cuh"

namespace dsalt {
CUresult encode_tensor_map_3d(CUtensorMap* m, CUtensorMapDataType dt, const void* base, uint64_t d0, uint64_t d1,
                              uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t box0,
                              uint32_t box1, uint32_t box2) {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  if (!fn) return CUDA_ERROR_NOT_FOUND;
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  cuuint32_t box[3] = {box0, box1, box2};
  cuuint32_t es[3] = {1, 1, 1};
  return fn(m, dt, 3, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}
}  // namespace dsalt

namespace dsalt {
cudaError_t launch_schedule(const DsaltScheduleParams& p, cudaStream_t st);
cudaError_t launch_gather(const DsaltGatherParams& p, cudaStream_t st);
cudaError_t simt_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st);
cudaError_t launch_win_gate(const DsaltWinGateParams& p, cudaStream_t st);
cudaError_t launch_rope_gqa(const DsaltRopeParams& p, bool bwd, cudaStream_t st);
bool rope_gqa_fits(const DsaltRopeParams& p);
cudaError_t launch_rmsnorm(const DsaltRmsNormParams& p, bool bwd, cudaStream_t st);
bool rmsnorm_supported(int d);
cudaError_t launch_scale_rows(const DsaltScaleRowsParams& p, cudaStream_t st);
cudaError_t launch_xent(const DsaltXentParams& p, cudaStream_t st);
cudaError_t launch_swiglu(const DsaltSwigluParams& p, bool bwd, cudaStream_t st);
cudaError_t launch_win_gate_bwd(const DsaltWinGateBwdParams& p, cudaStream_t st);
cudaError_t launch_hybrid_scores_bwd(const DsaltScoreBwdParams& p, cudaStream_t st);
cudaError_t launch_gqa_reduce(const DsaltGqaReduceParams& p, cudaStream_t st);
cudaError_t launch_wait_timeout_probe(int32_t* status, cudaStream_t st);
cudaError_t launch_hybrid_scores(const DsaltScoreParams& p, cudaStream_t st);
cudaError_t launch_topk(const DsaltTopkParams& p, cudaStream_t st);
cudaError_t noalloc_score_scratch(float** out);
// tcgen05 path (attn_tc.cu); returns cudaErrorNotSupported when the shape is
// outside what the tensor-core kernels cover, so the caller can report it.
cudaError_t tc_attention_stage(int stage, const DsaltAttnParams& p, cudaStream_t st);
bool tc_supported(const DsaltAttnParams& p);
}  // namespace dsalt

using namespace dsalt;

static int status_of(cudaError_t e) {
  if (e == cudaSuccess) return DSALT_OK;
  if (e == cudaErrorInvalidValue) return DSALT_ERR_ARG;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver || e == cudaErrorNoKernelImageForDevice)
    return DSALT_ERR_NO_DEVICE;
  return DSALT_ERR_LAUNCH;
}

static bool aligned16(const void* p) { return ((uintptr_t)p & 15u) == 0; }

static int check_attn(const DsaltAttnParams* p, int stage) {
  if (!p) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (p->D <= 0 || p->D > 256 || p->D % 8 != 0) return DSALT_ERR_HEAD_DIM;
  if (p->T < 0 || p->H <= 0 || p->S < 0 || p->k_lmk < 0 || p->kp < p->k_lmk) return DSALT_ERR_ARG;
  // grouped kv heads: H a multiple of H_kv (0 = H)
  if (p->H_kv < 0 || p->H_kv > p->H || (p->H_kv > 0 && p->H % p->H_kv != 0)) return DSALT_ERR_ARG;
  if (p->semantics != DSALT_TRAIN && p->semantics != DSALT_INFER) return DSALT_ERR_ARG;
  if (!(p->tau_win > 0.f)) return DSALT_ERR_ARG;
  if (p->impl < DSALT_IMPL_AUTO || p->impl > DSALT_IMPL_TCGEN05) return DSALT_ERR_ARG;
  if (p->grad_round != 0 && p->grad_round != 1) return DSALT_ERR_ARG;
  if (p->T == 0) return DSALT_OK;
  if (!p->q || !p->k || !p->v || !p->w || !p->cu_seqlens) return DSALT_ERR_ARG;
  if (p->kp > 0 && (!p->lmk_k || !p->lmk_v || !p->pos_sorted || !p->w_sorted)) return DSALT_ERR_ARG;
  if (!aligned16(p->q) || !aligned16(p->k) || !aligned16(p->v)) return DSALT_ERR_ALIGN;
  switch (stage) {
    case 0: if ((!p->o && !p->o_f32) || !p->lse) return DSALT_ERR_ARG; break;
    case 1: if ((!p->o && !p->o_f32) || !p->dout || !p->delta) return DSALT_ERR_ARG; break;
    case 2: if (!p->dout || !p->lse || !p->delta || !p->dk || !p->dv || !p->seq_wmax) return DSALT_ERR_ARG;
            if (p->kp > 0 && (!p->lmk_slot || !p->perm)) return DSALT_ERR_ARG;
            break;
    case 3: if (!p->dout || !p->lse || !p->delta || !p->dq) return DSALT_ERR_ARG; break;
  }
  return DSALT_OK;
}

static int run_attn(const DsaltAttnParams* p, int stage, void* stream) {
  int st = check_attn(p, stage);
  if (st != DSALT_OK) return st;
  if (p->T == 0) {
    // no tokens: every landmark slot is empty and its gradient is 0
    const size_t n_lw = (size_t)p->H * p->S * p->k_lmk;
    if (stage == 2 && p->d_lw && n_lw)
      return status_of(cudaMemsetAsync(p->d_lw, 0, n_lw * sizeof(float), (cudaStream_t)stream));
    return DSALT_OK;
  }
  cudaStream_t s = (cudaStream_t)stream;
  bool use_tc = false;
  if (p->impl == DSALT_IMPL_TCGEN05) {
    if (p->dtype == DSALT_F32 || !tc_supported(*p)) return DSALT_ERR_DTYPE;
    use_tc = true;
  } else if (p->impl == DSALT_IMPL_AUTO) {
    use_tc = p->dtype != DSALT_F32 && tc_supported(*p);
  }
  if (use_tc && (stage == 2 || stage == 3)) {
    // the dSᵀ tile scratch that the dK/dV stage fills and the dQ stage reads
    if (!p->ds_tiles || p->ds_band_tiles <= 0 || (p->kp > 0 && p->ds_lmk_tiles <= 0)) return DSALT_ERR_ARG;
    if (((uintptr_t)p->ds_tiles & 1023u) != 0) return DSALT_ERR_ALIGN;
  }
  cudaError_t e = use_tc ? tc_attention_stage(stage, *p, s) : simt_attention_stage(stage, *p, s);
  return status_of(e);
}

extern "C" {

int dsalt_b200_abi_version(void) { return DSALT_B200_ABI_VERSION; }

const char* dsalt_b200_status_string(int status) {
  switch (status) {
    case DSALT_OK: return "ok";
    case DSALT_ERR_ARG: return "invalid argument";
    case DSALT_ERR_DTYPE: return "unsupported dtype for this kernel family";
    case DSALT_ERR_HEAD_DIM: return "unsupported head_dim (multiples of 8 up to 256)";
    case DSALT_ERR_LAUNCH: return "CUDA launch or API error";
    case DSALT_ERR_NO_DEVICE: return "no usable sm_100 device";
    case DSALT_ERR_ALIGN: return "pointer not 16-byte aligned";
    case DSALT_ERR_TOO_LARGE: return "size beyond a documented limit";
  }
  return "unknown status";
}

int dsalt_b200_params_sizeof(int which) {
  switch (which) {
    case 0: return (int)sizeof(DsaltScheduleParams);
    case 1: return (int)sizeof(DsaltGatherParams);
    case 2: return (int)sizeof(DsaltAttnParams);
    case 3: return (int)sizeof(DsaltScoreParams);
    case 4: return (int)sizeof(DsaltTopkParams);
    case 5: return (int)sizeof(DsaltWinGateParams);
    case 6: return (int)sizeof(DsaltRopeParams);
    case 7: return (int)sizeof(DsaltRmsNormParams);
    case 8: return (int)sizeof(DsaltScaleRowsParams);
    case 9: return (int)sizeof(DsaltXentParams);
    case 10: return (int)sizeof(DsaltSwigluParams);
    case 11: return (int)sizeof(DsaltWinGateBwdParams);
    case 12: return (int)sizeof(DsaltScoreBwdParams);
    case 13: return (int)sizeof(DsaltGqaReduceParams);
  }
  return -1;
}

int dsalt_build_schedule(const DsaltScheduleParams* p, void* stream) {
  if (!p || p->S < 0 || p->T < 0 || p->block <= 0 || p->max_blocks < 0) return DSALT_ERR_ARG;
  if (!p->cu_seqlens || !p->block_map || !p->num_blocks) return DSALT_ERR_ARG;
  if ((p->seq_wmax || p->seq_id) && p->T > 0 && !p->w) return DSALT_ERR_ARG;
  if (p->seq_wmax_batch && !p->seq_wmax) return DSALT_ERR_ARG;
  if (p->S == 0) {
    cudaError_t e = cudaMemsetAsync(p->num_blocks, 0, sizeof(int32_t), (cudaStream_t)stream);
    if (e == cudaSuccess && p->seq_wmax_batch)
      e = cudaMemsetAsync(p->seq_wmax_batch, 0, sizeof(int32_t), (cudaStream_t)stream);
    return status_of(e);
  }
  return status_of(launch_schedule(*p, (cudaStream_t)stream));
}

int dsalt_gather_landmarks(const DsaltGatherParams* p, void* stream) {
  if (!p || p->H <= 0 || p->S < 0 || p->k_lmk < 0 || p->kp < p->k_lmk || p->k_lmk > 1024 || p->kp > 2048)
    return DSALT_ERR_ARG;
  if (p->H_kv < 0 || p->H_kv > p->H || (p->H_kv > 0 && p->H % p->H_kv != 0)) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if ((p->D * (p->dtype == DSALT_F32 ? 4 : 2)) % 16 != 0) return DSALT_ERR_HEAD_DIM;
  if (p->kp == 0 || p->S == 0) return DSALT_OK;
  if (!p->k || !p->v || !p->lmk_k || !p->lmk_v || !p->pos_sorted || !p->w_sorted || !p->perm ||
      !p->lmk_slot || !p->cu_seqlens || (p->k_lmk > 0 && (!p->lmk_pos || !p->lmk_w)))
    return DSALT_ERR_ARG;
  if (!aligned16(p->k) || !aligned16(p->v) || !aligned16(p->lmk_k) || !aligned16(p->lmk_v)) return DSALT_ERR_ALIGN;
  cudaStream_t s = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(p->lmk_slot, 0xFF, sizeof(int32_t) * (size_t)p->T * p->H, s);
  if (e != cudaSuccess) return status_of(e);
  return status_of(launch_gather(*p, s));
}

int dsalt_attn_fwd(const DsaltAttnParams* p, void* stream) { return run_attn(p, 0, stream); }
int dsalt_attn_bwd_preprocess(const DsaltAttnParams* p, void* stream) { return run_attn(p, 1, stream); }
int dsalt_attn_bwd_dkdv(const DsaltAttnParams* p, void* stream) { return run_attn(p, 2, stream); }
int dsalt_attn_bwd_dq(const DsaltAttnParams* p, void* stream) { return run_attn(p, 3, stream); }

int dsalt_hybrid_scores(const DsaltScoreParams* p, void* stream) {
  if (!p || p->T < 0 || p->H <= 0 || p->n_kv <= 0 || p->H % p->n_kv != 0 || p->dh <= 0 || p->d_model <= 0)
    return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (p->T == 0) return DSALT_OK;
  if (!p->x || !p->xwv || !p->alpha || !p->scores || !p->stats || !p->norms) return DSALT_ERR_ARG;
  return status_of(launch_hybrid_scores(*p, (cudaStream_t)stream));
}

// See dsalt_b200.h: the same pipeline as dsalt_hybrid_scores with its scratch in
// the library's fixed device array (select.cu); nothing is allocated here.
int dsalt_hybrid_scores_noalloc(const DsaltScoreParams* p, void* stream) {
  if (!p || p->T < 0 || p->H <= 0 || p->n_kv <= 0 || p->H % p->n_kv != 0 || p->dh <= 0 || p->d_model <= 0)
    return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  const int64_t need = p->T * (int64_t)(1 + p->n_kv) + 2 + 2 * (int64_t)p->n_kv;
  if (need > (int64_t)DSALT_NOALLOC_SCORE_MAX_FLOATS) return DSALT_ERR_TOO_LARGE;
  if (p->T == 0) return DSALT_OK;
  if (!p->x || !p->xwv || !p->alpha || !p->scores) return DSALT_ERR_ARG;
  float* scratch = nullptr;
  cudaError_t e = noalloc_score_scratch(&scratch);
  if (e != cudaSuccess) return status_of(e);
  DsaltScoreParams q = *p;
  q.stats = scratch;                      // [2 + 2*n_kv]
  q.norms = scratch + 2 + 2 * p->n_kv;    // [(1 + n_kv), T], column-major
  return status_of(launch_hybrid_scores(q, (cudaStream_t)stream));
}

int dsalt_select_topk(const DsaltTopkParams* p, void* stream) {
  if (!p || p->T < 0 || p->H <= 0 || p->S < 0 || p->k < 0 || p->max_len < 0) return DSALT_ERR_ARG;
  if (p->k > 1024 || p->max_len > 49152) return DSALT_ERR_TOO_LARGE;
  if (p->S == 0 || p->k == 0) return DSALT_OK;
  if (!p->scores || !p->w_sizes || !p->cu_seqlens || !p->idx) return DSALT_ERR_ARG;
  return status_of(launch_topk(*p, (cudaStream_t)stream));
}

int dsalt_win_gate(const DsaltWinGateParams* p, void* stream) {
  if (!p || p->T < 0 || p->d_model <= 0) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (p->T == 0) return DSALT_OK;
  if (!p->x || !p->weight || !p->bias || !p->w_cont) return DSALT_ERR_ARG;
  return status_of(launch_win_gate(*p, (cudaStream_t)stream));
}

static int check_rope(const DsaltRopeParams* p, bool bwd) {
  if (!p || p->T < 0 || p->H <= 0 || p->Hkv <= 0 || p->H % p->Hkv != 0) return DSALT_ERR_ARG;
  if (p->kv_out_heads != 0 && p->kv_out_heads != p->H && p->kv_out_heads != p->Hkv) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (p->D <= 0 || p->D > 256 || p->D % 16 != 0) return DSALT_ERR_HEAD_DIM;
  if (p->ld != 0 && (p->ld < (int64_t)p->H * p->D || p->ld % (p->dtype == DSALT_F32 ? 4 : 8) != 0))
    return DSALT_ERR_ARG;
  if (p->T == 0) return DSALT_OK;
  if (!rope_gqa_fits(*p)) return DSALT_ERR_TOO_LARGE;
  if (!p->cos || !p->sin) return DSALT_ERR_ARG;
  if (!aligned16(p->cos) || !aligned16(p->sin)) return DSALT_ERR_ALIGN;
  const void* need[] = {bwd ? p->dq_out : p->q, bwd ? p->dk_out : p->k, bwd ? p->dq : p->q_out, bwd ? p->dk : p->k_out};
  for (const void* ptr : need) {
    if (!ptr) return DSALT_ERR_ARG;
    if (!aligned16(ptr)) return DSALT_ERR_ALIGN;
  }
  const void* opt[] = {bwd ? p->dv_out : p->v_out, bwd ? p->dv : p->v};
  if ((opt[0] != nullptr) != (opt[1] != nullptr)) return DSALT_ERR_ARG;  // both or neither
  for (const void* ptr : opt)
    if (ptr && !aligned16(ptr)) return DSALT_ERR_ALIGN;
  return DSALT_OK;
}

int dsalt_rope_gqa_fwd(const DsaltRopeParams* p, void* stream) {
  const int st = check_rope(p, false);
  if (st != DSALT_OK || p->T == 0) return st;
  return status_of(launch_rope_gqa(*p, false, (cudaStream_t)stream));
}

int dsalt_rope_gqa_bwd(const DsaltRopeParams* p, void* stream) {
  const int st = check_rope(p, true);
  if (st != DSALT_OK || p->T == 0) return st;
  return status_of(launch_rope_gqa(*p, true, (cudaStream_t)stream));
}

static int check_rmsnorm(const DsaltRmsNormParams* p, bool bwd) {
  if (!p || p->T < 0) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (!rmsnorm_supported(p->d)) return DSALT_ERR_HEAD_DIM;
  if (!(p->eps >= 0.f)) return DSALT_ERR_ARG;
  if (p->T == 0) return DSALT_OK;
  const void* need[] = {p->x, bwd ? p->dy : p->y, bwd ? p->dx : p->x, p->w};
  for (const void* ptr : need) {
    if (!ptr) return DSALT_ERR_ARG;
    if (!aligned16(ptr)) return DSALT_ERR_ALIGN;
  }
  if (bwd && (!p->rstd || !p->dw_part)) return DSALT_ERR_ARG;
  if (!bwd && p->res && (!p->x_sum || !aligned16(p->res) || !aligned16(p->x_sum)))
    return p->x_sum ? DSALT_ERR_ALIGN : DSALT_ERR_ARG;
  if (bwd && p->dres && !aligned16(p->dres)) return DSALT_ERR_ALIGN;
  if ((p->T + DSALT_RMSNORM_ROWS_PER_PART - 1) / DSALT_RMSNORM_ROWS_PER_PART > INT32_MAX) return DSALT_ERR_TOO_LARGE;
  return DSALT_OK;
}

int dsalt_rmsnorm_fwd(const DsaltRmsNormParams* p, void* stream) {
  const int st = check_rmsnorm(p, false);
  if (st != DSALT_OK || p->T == 0) return st;
  return status_of(launch_rmsnorm(*p, false, (cudaStream_t)stream));
}

int dsalt_rmsnorm_bwd(const DsaltRmsNormParams* p, void* stream) {
  const int st = check_rmsnorm(p, true);
  if (st != DSALT_OK || p->T == 0) return st;
  return status_of(launch_rmsnorm(*p, true, (cudaStream_t)stream));
}

int dsalt_scale_rows(const DsaltScaleRowsParams* p, void* stream) {
  if (!p || p->T < 0 || p->groups <= 0 || p->width <= 0 || p->width % 8 != 0) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (p->T == 0) return DSALT_OK;
  if (!p->x || !p->coef || !p->out) return DSALT_ERR_ARG;
  if (!aligned16(p->x) || !aligned16(p->out)) return DSALT_ERR_ALIGN;
  return status_of(launch_scale_rows(*p, (cudaStream_t)stream));
}

int dsalt_xent_fwd_grad(const DsaltXentParams* p, void* stream) {
  if (!p || p->rows < 0 || p->vocab <= 0 || p->rows > INT32_MAX) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16) return DSALT_ERR_DTYPE;
  if (p->rows == 0) return DSALT_OK;
  if (!p->logits || !p->labels || !p->row_loss || !p->scale) return DSALT_ERR_ARG;
  if (!aligned16(p->logits)) return DSALT_ERR_ALIGN;
  return status_of(launch_xent(*p, (cudaStream_t)stream));
}

static int check_swiglu(const DsaltSwigluParams* p, bool bwd) {
  if (!p || p->T < 0 || p->F <= 0 || p->F % 8 != 0) return DSALT_ERR_ARG;
  if (p->ld_in < p->F || p->ld_in % 8 != 0) return DSALT_ERR_ARG;
  if (bwd && (p->ld_out < p->F || p->ld_out % 8 != 0)) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16) return DSALT_ERR_DTYPE;
  if (p->T == 0) return DSALT_OK;
  if (p->T > INT64_MAX / p->ld_in || (p->T + 7) / 8 > (int64_t)UINT32_MAX || p->F / 8 > INT32_MAX)
    return DSALT_ERR_TOO_LARGE;
  const void* fwd_ptrs[] = {p->g, p->u, p->h};
  const void* bwd_ptrs[] = {p->g, p->u, p->dh, p->dg, p->du};
  const void* const* need = bwd ? bwd_ptrs : fwd_ptrs;
  const int n = bwd ? 5 : 3;
  for (int i = 0; i < n; ++i) {
    if (!need[i]) return DSALT_ERR_ARG;
    if (!aligned16(need[i])) return DSALT_ERR_ALIGN;
  }
  return DSALT_OK;
}

int dsalt_selftest_wait_timeout(int32_t* status, void* stream) {
  if (!status) return DSALT_ERR_ARG;
  return status_of(launch_wait_timeout_probe(status, (cudaStream_t)stream));
}

int dsalt_hybrid_scores_bwd(const DsaltScoreBwdParams* p, void* stream) {
  if (!p || p->T < 0 || p->H <= 0 || p->n_kv <= 0 || p->H % p->n_kv != 0 || p->H > 4096) return DSALT_ERR_ARG;
  if (!p->g_s || !p->alpha || !p->z_x || !p->z_v || !p->stats || !p->sums || !p->d_alpha) return DSALT_ERR_ARG;
  if (p->T > 0 && !p->partials) return DSALT_ERR_ARG;
  // one partial-sum block keeps 128 tokens × (2·(1+n_kv) + H) floats in shared memory
  if (2 * (1 + p->n_kv) + p->H > DSALT_SCORE_BWD_MAX_SUMS) return DSALT_ERR_TOO_LARGE;
  if (p->T > 0 && (!p->norms || !p->coef_x || !p->coef_v)) return DSALT_ERR_ARG;
  return status_of(launch_hybrid_scores_bwd(*p, (cudaStream_t)stream));
}

int dsalt_win_gate_bwd(const DsaltWinGateBwdParams* p, void* stream) {
  if (!p || p->T < 0 || p->d_model <= 0 || p->d_model % 8 != 0) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16) return DSALT_ERR_DTYPE;
  if (p->T == 0 || (!p->dx && !p->dw_part)) return DSALT_OK;
  if ((p->T + DSALT_WIN_GATE_ROWS_PER_PART - 1) / DSALT_WIN_GATE_ROWS_PER_PART > (int64_t)UINT32_MAX)
    return DSALT_ERR_TOO_LARGE;
  if (!p->weight || !p->dl || (p->dw_part && !p->x)) return DSALT_ERR_ARG;
  if (!aligned16(p->weight) || (p->dw_part && (!aligned16(p->x) || !aligned16(p->dw_part))) ||
      (p->dx && !aligned16(p->dx)))
    return DSALT_ERR_ALIGN;
  return status_of(launch_win_gate_bwd(*p, (cudaStream_t)stream));
}

int dsalt_swiglu_fwd(const DsaltSwigluParams* p, void* stream) {
  const int st = check_swiglu(p, false);
  if (st != DSALT_OK || p->T == 0) return st;
  return status_of(launch_swiglu(*p, false, (cudaStream_t)stream));
}

int dsalt_swiglu_bwd(const DsaltSwigluParams* p, void* stream) {
  const int st = check_swiglu(p, true);
  if (st != DSALT_OK || p->T == 0) return st;
  return status_of(launch_swiglu(*p, true, (cudaStream_t)stream));
}

int dsalt_gqa_reduce(const DsaltGqaReduceParams* p, void* stream) {
  if (!p || p->T < 0 || p->H <= 0 || p->H_kv <= 0 || p->H_kv > p->H || p->H % p->H_kv != 0) return DSALT_ERR_ARG;
  if (p->dtype != DSALT_F16 && p->dtype != DSALT_BF16 && p->dtype != DSALT_F32) return DSALT_ERR_DTYPE;
  if (p->D <= 0 || (p->D * (p->dtype == DSALT_F32 ? 4 : 2)) % 16 != 0) return DSALT_ERR_HEAD_DIM;
  if (p->T == 0) return DSALT_OK;
  if (!p->x || !p->y) return DSALT_ERR_ARG;
  if (!aligned16(p->x) || !aligned16(p->y)) return DSALT_ERR_ALIGN;
  return status_of(launch_gqa_reduce(*p, (cudaStream_t)stream));
}

}  // extern "C"
