/*
 * dsalt_b200.h — C ABI of the B200 (sm_100a) DSALT sparse-attention library.
 *
 * Every entry point takes caller-owned device buffers (plain pointers and
 * sizes), launches on the caller's CUDA stream (`stream` is a CUstream /
 * cudaStream_t handle passed as void*), allocates no device memory and returns
 * a status code (DSALT_OK == 0).  Argument errors are reported before any
 * launch; a device-side fault report (a bounded wait that gave up, an index
 * outside its range) is written to the optional device status word
 * `status` (int32, caller-zeroed) instead of trapping.
 *
 * Reference interfaces replaced (paths relative to the reference project,
 * LeonardoCofone/dsalt-library v1.0.0) are cited beside each entry point.
 * The Python host package `dsalt` (same module paths as the reference) binds
 * these with ctypes (dsalt/kernels/_ext.py).
 */
#ifndef DSALT_B200_H
#define DSALT_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DSALT_API __attribute__((visibility("default")))
#else
#define DSALT_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DSALT_B200_ABI_VERSION 8

/* The tensor-core dK/dV stage splits each landmark chunk's query range into
 * this many parts that run as separate CTAs; their fp32 partial sums are added
 * in a fixed order (deterministic) by the band pass. */
#define DSALT_LMK_SPLIT 4

/* fp32 words per query record of the backward (DsaltAttnParams.qrec) */
#define DSALT_QREC_FLOATS 16
/* dSᵀ tiles of the tensor-core backward (ds_tiles below): 128 x 64 16-bit
 * elements; band tiles per (head, key block), landmark tiles per (head,
 * sequence, 128-slot chunk), and one all-zero tile at the end.              */
#define DSALT_DS_TILE_BYTES 16384
#define DSALT_DS_TILES(H, max_blocks, S, kp, band_tiles, lmk_tiles)                        \
  ((int64_t)(H) * (max_blocks) * (band_tiles) +                                             \
   (int64_t)(H) * (S) * (((kp) + 127) / 128) * (lmk_tiles) + 1)

/* ---- status codes ------------------------------------------------------ */
enum {
  DSALT_OK = 0,
  DSALT_ERR_ARG = 1,          /* invalid argument (shape, pointer, range)      */
  DSALT_ERR_DTYPE = 2,        /* unsupported dtype                             */
  DSALT_ERR_HEAD_DIM = 3,     /* unsupported head_dim                          */
  DSALT_ERR_LAUNCH = 4,       /* CUDA launch / API error                       */
  DSALT_ERR_NO_DEVICE = 5,    /* no sm_100 device / driver entry point missing */
  DSALT_ERR_ALIGN = 6,        /* pointer not 16-byte aligned                   */
  DSALT_ERR_TOO_LARGE = 7     /* size beyond a documented limit                */
};

/* device status word bits (written by kernels, never a trap) */
enum {
  DSALT_DEV_WAIT_TIMEOUT = 1, /* an mbarrier wait exceeded its time limit      */
  DSALT_DEV_BAD_INDEX = 2     /* an index (landmark position, seq id) was out of range */
};

/* dtype codes */
enum { DSALT_F16 = 0, DSALT_BF16 = 1, DSALT_F32 = 2 };

/* attention semantics */
enum {
  DSALT_TRAIN = 0,  /* continuous window w̃, soft edge, lmk bias = log-weight    */
  DSALT_INFER = 1   /* integer window w, no edge, additive lmk bias             */
};

/* kernel family selection */
enum {
  DSALT_IMPL_AUTO = 0,    /* tcgen05 for f16/bf16, exact-fp32 SIMT for f32     */
  DSALT_IMPL_SIMT = 1,    /* exact SIMT kernels for every dtype                */
  DSALT_IMPL_TCGEN05 = 2  /* tcgen05/TMEM/TMA kernels (f16/bf16 only)          */
};

/* ---- packed-batch schedule ---------------------------------------------
 * Replaces selectors._build_seq_block_map (dsalt/kernels/selectors.py:37-67)
 * and selectors._seq_meta (:15-34).  Built on the device from cu_seqlens and
 * the window, keyed by content (no host cache), no device-to-host copy.
 *   block_map [max_blocks][2] int32 = (sequence, block-in-sequence) for
 *     blocks of `block` query rows; rows past num_blocks are untouched;
 *   num_blocks [1] int32; seq_wmax [S] int32 = max over the sequence's rows of
 *     the number of band keys before the diagonal (floor(w̃) train, w-1 infer);
 *   seq_wmax_batch [1] int32 = max over s of seq_wmax[s] (optional, may be
 *     NULL; needs seq_wmax) — the widest band of the batch, ready to copy to
 *     the host without a reduction launch;
 *   seq_id [T] int32 = sequence of every packed token (optional, may be NULL).
 * max_blocks must be >= ceil(T/block) + S.                                    */
typedef struct DsaltScheduleParams {
  const int32_t* cu_seqlens;  /* [S+1] */
  const float* w;             /* [T] window, fp32 */
  int32_t* block_map;         /* [max_blocks*2] */
  int32_t* num_blocks;        /* [1] */
  int32_t* seq_wmax;          /* [S] */
  int32_t* seq_id;            /* [T] or NULL */
  int64_t T;
  int32_t S;
  int32_t block;
  int32_t max_blocks;
  int32_t semantics;
  int32_t* seq_wmax_batch;    /* [1] or NULL */
} DsaltScheduleParams;
DSALT_API int dsalt_build_schedule(const DsaltScheduleParams* p, void* stream);

/* ---- landmark gather ----------------------------------------------------
 * Replaces selectors._build_landmark_kv (dsalt/kernels/selectors.py:137-159)
 * and _pad_landmarks (dsalt/kernels/dsalt_triton_train.py:44-68).  Per
 * (head, sequence): sorts the k landmark slots by position (invalid slots,
 * pos < 0 or pos >= len, last), pads to kp, gathers K/V rows into
 * [H,S,kp,D] (zeros for invalid), copies the log-weight / bias in sorted
 * order, records the caller's slot of every sorted entry (perm) and writes
 * the reverse map lmk_slot[T,H] (sorted slot of the first landmark at that
 * token, else -1; the caller pre-fills it with -1).  k_lmk <= 1024,
 * kp <= 2048.                                                               */
typedef struct DsaltGatherParams {
  const void* k;              /* [T,H_kv,D] dtype (H_kv = H without grouped kv heads) */
  const void* v;              /* [T,H_kv,D] dtype */
  const int64_t* lmk_pos;     /* [H,S,k_lmk] caller order, relative positions */
  const float* lmk_w;         /* [H,S,k] log-weight (train) / bias (infer), fp32 */
  const int32_t* cu_seqlens;  /* [S+1] */
  void* lmk_k;                /* [H,S,kp,D] dtype */
  void* lmk_v;                /* [H,S,kp,D] dtype */
  int32_t* pos_sorted;        /* [H,S,kp] (-1 = invalid) */
  float* w_sorted;            /* [H,S,kp] */
  int32_t* perm;              /* [H,S,kp] caller slot (-1 for padding) */
  int32_t* lmk_slot;          /* [T,H] */
  int32_t* status;            /* device status word or NULL */
  int64_t T;
  int32_t H, D, S, k_lmk, kp;
  int32_t dtype;
  int32_t H_kv;               /* kv heads (0: H); query head h gathers from kv head
                                 h / (H / H_kv); H must be a multiple of H_kv */
} DsaltGatherParams;
DSALT_API int dsalt_gather_landmarks(const DsaltGatherParams* p, void* stream);

/* ---- attention ------------------------------------------------------------
 * One parameter block for the forward and the three backward stages.
 * Layouts: q,o,dout,dq,dk,dv [T,H,D] and k,v [T,H_kv,D] contiguous; lse,
 * delta, dw_head [T,H] fp32; landmark buffers from dsalt_gather_landmarks.
 * Grouped kv heads (H_kv < H, the reference's n_kv_heads): query head h reads
 * kv head h / (H / H_kv) in every kernel, so K/V are never expanded; dk and dv
 * are then per query head ([T,H,D], the gradients of the expanded K/V), and
 * dsalt_gqa_reduce sums each group into the [T,H_kv,D] gradient.            */
typedef struct DsaltAttnParams {
  /* inputs */
  const void* q; const void* k; const void* v;
  const float* w;             /* [T] w̃ (train) or w (infer), fp32 */
  const int32_t* cu_seqlens;  /* [S+1] */
  const int32_t* block_map;   /* from dsalt_build_schedule (block = 128) */
  const int32_t* num_blocks;
  const int32_t* seq_wmax;    /* [S] */
  const void* lmk_k; const void* lmk_v;
  const int32_t* pos_sorted; const float* w_sorted; const int32_t* perm;
  const int32_t* lmk_slot;
  /* forward outputs */
  void* o;                    /* [T,H,D] dtype, or NULL when o_f32 is given for 16-bit
                                 inputs (then only the fp32 O is written, and the
                                 backward stages read that one) */
  float* o_f32;               /* [T,H,D] fp32 O holding the bf16/f16-rounded values
                                 (the reference op's output), or NULL */
  float* lse;                 /* [T,H] natural-log LSE, -inf for empty rows */
  /* backward */
  const void* dout;           /* [T,H,D] dtype (written by the preprocess stage when
                                 dout_f32 is given) */
  const float* dout_f32;      /* [T,H,D] fp32 upstream gradient, or NULL */
  float* delta;               /* [T,H] scratch */
  void* dq; void* dk; void* dv;       /* [T,H,D] dtype */
  float* dw_head;             /* [T,H] scratch (train) */
  float* dw;                  /* [T] fp32: Σ_h ∂loss/∂w̃ (train) or NULL */
  float* d_lw;                /* [H,S,k_lmk] fp32, caller slot order: ∂loss/∂lmk_w;
                                 every slot is written (0 for an empty slot) */
  float* lmk_grad;            /* fp32 scratch of the tensor-core dK/dV stage:
                                 ((2·D + 1)·DSALT_LMK_SPLIT + 2·D)·H·S·kp floats
                                 (partial landmark-slot dK, dV, d_lw and the band
                                 rows of landmark keys); unused by the SIMT family */
  float* qrec;                /* [H,T,DSALT_QREC_FLOATS] fp32 scratch: per-query records
                                 (LSE, Delta, window, soft-edge factors) written by the
                                 preprocess stage and read by the tensor-core dK/dV
                                 stage; unused by the SIMT family */
  void* ds_tiles;             /* scratch of the tensor-core backward, 1024-byte aligned:
                                 the dK/dV stage stores every dSᵀ tile it computes
                                 (dtype, 128 keys x 64 queries, DSALT_DS_TILE_BYTES each,
                                 after the soft edge) and the dQ stage multiplies them
                                 with K, so dQ needs no recomputation of S and dP.
                                 DSALT_DS_TILES(H, max_blocks, S, kp, ds_band_tiles,
                                 ds_lmk_tiles) tiles; unused by the SIMT family */
  int32_t* status;            /* device status word or NULL */
  /* sizes */
  int64_t T;
  int32_t H, D, S, k_lmk, kp;
  int32_t max_blocks;
  int32_t ds_band_tiles;      /* 64-query tiles stored per key block: at least
                                 ceil((128 + max_s seq_wmax[s]) / 64) (the widest band
                                 item); a key block that needs more flags
                                 DSALT_DEV_BAD_INDEX */
  int32_t ds_lmk_tiles;       /* 64-query tiles stored per landmark chunk: at least
                                 ceil(longest sequence / 64) + 1 */
  float scale;                /* 1/sqrt(D) */
  float tau_win, win_edge;
  int32_t semantics;          /* DSALT_TRAIN / DSALT_INFER */
  int32_t dtype;              /* DSALT_F16 / DSALT_BF16 / DSALT_F32 */
  int32_t impl;               /* DSALT_IMPL_* */
  int32_t H_kv;               /* kv heads of k and v (0: H); H must be a multiple */
  int32_t grad_round;         /* 1: dw and d_lw hold their fp32 sums rounded to the
                                 input dtype (the values the reference's autograd
                                 functions return, .to(out_dtype), widened back to
                                 fp32 exactly); 0: the fp32 sums */
} DsaltAttnParams;

/* Replaces _train_fwd_kernel (dsalt/kernels/dsalt_triton_train.py:74-214) and
 * _dsalt_fwd_kernel (dsalt/kernels/dsalt_triton_attn.py:27-169).             */
DSALT_API int dsalt_attn_fwd(const DsaltAttnParams* p, void* stream);
/* Replaces _train_bwd_preprocess (dsalt_triton_train.py:220-237) and
 * _dsalt_bwd_preprocess (dsalt/kernels/dsalt_triton_bwd.py:17-49).           */
DSALT_API int dsalt_attn_bwd_preprocess(const DsaltAttnParams* p, void* stream);
/* Replaces _train_bwd_dkdv_kernel (dsalt_triton_train.py:386-481) plus the
 * landmark dK/dV/d_logw atomics of _train_bwd_kernel (:302-333) and of
 * _dsalt_bwd_kernel (dsalt_triton_bwd.py:121-162, 198-207): key-parallel,
 * atomic-free, deterministic.                                               */
DSALT_API int dsalt_attn_bwd_dkdv(const DsaltAttnParams* p, void* stream);
/* Replaces the dQ / d_w̃ part of _train_bwd_kernel (dsalt_triton_train.py:
 * 335-383) and the dQ of _dsalt_bwd_kernel; writes dq, dw_head (from the
 * σ-scaled dSᵀ entries dsalt_attn_bwd_dkdv stored) and dw.                  */
DSALT_API int dsalt_attn_bwd_dq(const DsaltAttnParams* p, void* stream);

/* Grouped kv heads: y[t, g, :] = Σ_{r < H/H_kv} x[t, g·(H/H_kv) + r, :], summed in
 * fp32 and rounded once to the dtype.  Replaces the backward of the reference's
 * K/V expansion _repeat_kv (dsalt/modules/dsalt_attention.py:254-268), whose
 * autograd sums the expanded heads' gradients; x is dk or dv of the attention
 * backward with H_kv < H.                                                   */
typedef struct DsaltGqaReduceParams {
  const void* x;              /* [T,H,D] dtype, 16-byte aligned */
  void* y;                    /* [T,H_kv,D] dtype, 16-byte aligned */
  int64_t T;
  int32_t H, H_kv, D;
  int32_t dtype;
} DsaltGqaReduceParams;
DSALT_API int dsalt_gqa_reduce(const DsaltGqaReduceParams* p, void* stream);

/* ---- selection ------------------------------------------------------------
 * Replaces the norm / z-standardisation / mix of hybrid_scores_per_head
 * (dsalt/kernels/landmark_tokens_ker.py:19-61).  xwv is the caller's
 * x @ W_V^T GEMM output [T, n_kv*dh] (any library GEMM).                    */
typedef struct DsaltScoreParams {
  const void* x;              /* [T, d_model] dtype */
  const void* xwv;            /* [T, n_kv*dh] dtype */
  const float* alpha;         /* [H] */
  float* scores;              /* [T,H] fp32 */
  float* z_x;                 /* [T] fp32 */
  float* z_v;                 /* [T,H] fp32 */
  float* stats;               /* scratch [2 + 2*n_kv] fp32 */
  float* norms;               /* scratch [(1+n_kv), T] fp32, column-major */
  int64_t T;
  int32_t d_model, H, n_kv, dh;
  int32_t dtype;
} DsaltScoreParams;
DSALT_API int dsalt_hybrid_scores(const DsaltScoreParams* p, void* stream);

/* No counterpart in the reference.  Same result as dsalt_hybrid_scores for
 * callers that may not allocate device memory (for example a host runtime that
 * owns and plans every device buffer and hands a plugin only its inputs and
 * outputs): p->stats and p->norms are ignored, and the scratch lives in a
 * fixed array inside the library, DSALT_NOALLOC_SCORE_MAX_FLOATS floats (8 MiB)
 * held on every GPU that loads the library until the process exits.  Sizes
 * with T*(1+n_kv) + 2 + 2*n_kv > DSALT_NOALLOC_SCORE_MAX_FLOATS return
 * DSALT_ERR_TOO_LARGE.  The first call on a device looks up the array's device
 * address (cudaGetSymbolAddress, with that device current) and caches it;
 * make that first call before any stream capture.  All calls on a device share
 * the array, so calls that overlap on the GPU race.  Nothing is allocated.
 * Forward only: the statistics and norms stay in the shared array (the next
 * call on the device overwrites them), so they cannot feed
 * dsalt_hybrid_scores_bwd; a caller that needs the backward uses
 * dsalt_hybrid_scores with its own stats and norms buffers.                 */
#define DSALT_NOALLOC_SCORE_MAX_FLOATS (1 << 21)
DSALT_API int dsalt_hybrid_scores_noalloc(const DsaltScoreParams* p, void* stream);

/* Backward of dsalt_hybrid_scores through the z-scores to the norms, the
 * gradient of landmark_tokens_ker.py:47-60 (unbiased std, clamp at 1e-6):
 *   dz[t,0] = Σ_h g_s[t,h]·(1 − α_h), dz[t,1+g] = Σ_{h in group g} g_s[t,h]·α_h,
 *   dn[t,c] = (dz[t,c] − mean_t dz[·,c]) / sd_c
 *             − [sd_c > 1e-6]·z[t,c]·Σ_t dz[·,c]·z[·,c] / ((T − 1)·sd_c),
 *   coef_x[t] = dn[t,0] / ‖x_t‖, coef_v[t,g] = dn[t,1+g] / ‖(x·W_Vᵀ)_t,g‖
 *   (a zero norm divides by 1), d_alpha[h] = Σ_t g_s[t,h]·(z_v[t,h] − z_x[t]),
 * with z, sd, the norms taken from the forward's outputs and scratch.  The
 * input gradients are then coef · x and coef · x·W_Vᵀ row by row
 * (dsalt_scale_rows).  Sums in a fixed order (deterministic).               */
typedef struct DsaltScoreBwdParams {
  const float* g_s;           /* [T,H] gradient of the scores */
  const float* alpha;         /* [H] */
  const float* z_x;           /* [T]   (forward output) */
  const float* z_v;           /* [T,H] (forward output) */
  const float* norms;         /* [(1+n_kv), T] column-major (forward scratch) */
  const float* stats;         /* [2 + 2*n_kv] (forward scratch: mean, clamped std) */
  float* sums;                /* scratch [2*(1+n_kv)] */
  float* partials;            /* scratch [ceil(T / DSALT_SCORE_BWD_TOKENS), 2*(1+n_kv) + H]:
                                 per-block partial sums, added in block order */
  float* d_alpha;             /* [H] */
  float* coef_x;              /* [T] */
  float* coef_v;              /* [T, n_kv] */
  int64_t T;
  int32_t H, n_kv;
} DsaltScoreBwdParams;
#define DSALT_SCORE_BWD_TOKENS 128
/* limit on 2·(1+n_kv) + H (the sums one partial block holds in shared memory);
 * larger head counts return DSALT_ERR_TOO_LARGE                             */
#define DSALT_SCORE_BWD_MAX_SUMS 400
DSALT_API int dsalt_hybrid_scores_bwd(const DsaltScoreBwdParams* p, void* stream);

/* Replaces the exclusion + top-k of _compute_landmark_indices
 * (dsalt/kernels/selectors.py:103-134): per (head, sequence) the k largest
 * scores among tokens with seq_off >= w_sizes (own window), -1 when fewer are
 * finite.  Ties go to the lower position.  idx is written sorted by
 * descending score.                                                         */
typedef struct DsaltTopkParams {
  const float* scores;        /* [T,H] */
  const float* w_sizes;       /* [T] (floored window, any float) */
  const int32_t* cu_seqlens;  /* [S+1] */
  int64_t* idx;               /* [H,S,k] */
  int64_t T;
  int32_t H, S, k;
  int32_t max_len;            /* upper bound on sequence length (<= 1<<20) */
} DsaltTopkParams;
DSALT_API int dsalt_select_topk(const DsaltTopkParams* p, void* stream);

/* Replaces DSALTAttention._window_continuous / _window_sizes
 * (dsalt/modules/dsalt_attention.py:270-284): w̃ = n_min + σ(x·W + b)·(n_max −
 * n_min), with torch's autocast rounding when dtype is bf16/f16 (logit,
 * sigmoid, product and sum each rounded), plus w_disc = max(floor(w̃), 1).   */
typedef struct DsaltWinGateParams {
  const void* x;              /* [T, d_model] dtype */
  const void* weight;         /* [d_model] dtype */
  const void* bias;           /* [1] dtype */
  void* w_cont;               /* [T] dtype */
  float* w_f32;               /* [T] fp32 copy of w_cont, or NULL */
  float* w_disc;              /* [T] fp32, or NULL */
  float* logits;              /* [T] fp32 (pre-rounding), or NULL */
  int64_t T;
  int32_t d_model;
  float n_min, n_max;
  int32_t dtype;
} DsaltWinGateParams;
DSALT_API int dsalt_win_gate(const DsaltWinGateParams* p, void* stream);

/* Backward of the window gate's Linear, d_model a multiple of 8, f16 / bf16:
 * given dl[t] = d loss / d logit[t] (fp32), dx[t, j] = dl[t]·w[j] rounded once to
 * dtype, and the weight gradient Σ_t dl[t]·x[t, j] as ceil(T /
 * DSALT_WIN_GATE_ROWS_PER_PART) fp32 partial rows (each summed in row order; the
 * caller adds them).  dx or dw_part may be NULL to skip that output.          */
#define DSALT_WIN_GATE_ROWS_PER_PART 32
typedef struct DsaltWinGateBwdParams {
  const void* x;              /* [T, d_model] dtype */
  const void* weight;         /* [d_model] dtype */
  const float* dl;            /* [T] fp32 */
  void* dx;                   /* [T, d_model] dtype, or NULL */
  float* dw_part;             /* [ceil(T / DSALT_WIN_GATE_ROWS_PER_PART), d_model] fp32, or NULL */
  int64_t T;
  int32_t d_model;
  int32_t dtype;
} DsaltWinGateBwdParams;
DSALT_API int dsalt_win_gate_bwd(const DsaltWinGateBwdParams* p, void* stream);

/* Backward of hybrid_scores_per_head's norms (landmark_tokens_ker.py:47,52):
 * out[t, g·width + j] = coef[t·groups + g] · x[t, g·width + j], fp32 product
 * rounded once to dtype (width a multiple of 8; x, out 16-byte aligned).      */
typedef struct DsaltScaleRowsParams {
  const void* x;              /* [T, groups·width] dtype */
  const float* coef;          /* [T, groups] fp32 */
  void* out;                  /* [T, groups·width] dtype */
  int64_t T;
  int32_t groups, width;
  int32_t dtype;
} DsaltScaleRowsParams;
DSALT_API int dsalt_scale_rows(const DsaltScaleRowsParams* p, void* stream);

/* ---- attention prologue ---------------------------------------------------
 * Replaces apply_rotary_emb (dsalt/kernels/window_utils.py:73-88) on q and k
 * plus _repeat_kv (dsalt/modules/dsalt_attention.py:254-268) on k and v, as
 * DSALTAttention._packed calls them, in one pass:
 *   q_out = q·cos + rot(q)·sin, k_out[:, h] = (k·cos + rot(k)·sin)[:, h / n_rep],
 *   v_out[:, h] = v[:, h / n_rep],  rot(x) = cat(−x[D/2:], x[:D/2])
 * with the reference's rounding: each product, and the sum, rounded to dtype.
 * The backward stage maps dq_out, dk_out, dv_out back: the sum over the n_rep
 * copies of a kv head (rounded once), then the transposed rotation.         */
typedef struct DsaltRopeParams {
  const void* q;              /* [T, H, D] dtype                 (forward) */
  const void* k;              /* [T, Hkv, D]                               */
  const void* v;              /* [T, Hkv, D]                               */
  const void* cos;            /* [T, D] dtype: the row of each token's position */
  const void* sin;            /* [T, D] dtype                              */
  void* q_out;                /* [T, H, D]                                 */
  void* k_out;                /* [T, H, D]                                 */
  void* v_out;                /* [T, H, D], or NULL (v not expanded)       */
  const void* dq_out;         /* [T, H, D]                      (backward) */
  const void* dk_out;         /* [T, H, D]                                 */
  const void* dv_out;         /* [T, H, D], or NULL                        */
  void* dq;                   /* [T, H, D]                                 */
  void* dk;                   /* [T, Hkv, D]                               */
  void* dv;                   /* [T, Hkv, D], or NULL                      */
  int64_t T;
  int64_t ld;                 /* 0: q, k, v, dq, dk, dv dense as above; else
                                 the row stride (elements) of all six, column
                                 blocks of one [T, ld] buffer (a multiple of 8,
                                 fp32: 4, and at least H·D)                */
  int32_t H, Hkv, D;          /* D a multiple of 16 up to 256; H a multiple of Hkv */
  int32_t dtype;
  int32_t kv_out_heads;       /* heads of k_out (and v_out, dk_out, dv_out): 0 or H
                                 = k expanded to the query heads; Hkv = not expanded
                                 (the attention kernels then read the kv head in
                                 place), with v_out / dv_out NULL (v passes through) */
} DsaltRopeParams;
DSALT_API int dsalt_rope_gqa_fwd(const DsaltRopeParams* p, void* stream);
DSALT_API int dsalt_rope_gqa_bwd(const DsaltRopeParams* p, void* stream);

/* ---- model helpers --------------------------------------------------------
 * RMSNorm of the model blocks (dsalt/kernels/RMSENorm.py: F.rms_norm, fp32 math
 * under autocast, result in the input dtype), forward and backward, for
 * d = 256, 512, 768 or 1024:
 *   y = x·r·w, r = 1/sqrt(mean(x²) + eps);  dx = r·(g − x·r²·mean(g·x)), g = dy·w.
 * With res set, the forward first forms x_sum = R(x + res) (the block's residual
 * add, rounded to dtype), writes it and normalises it; the backward then takes
 * x = x_sum and, with dres set, returns dx = R(R(dx) + dres), dres being the
 * gradient reaching x_sum from its other consumers.  The backward writes dw as
 * ceil(T / DSALT_RMSNORM_ROWS_PER_PART) partial rows (each the fixed-order sum
 * over its rows) and, with dw set, their fixed-order column sums.           */
#define DSALT_RMSNORM_ROWS_PER_PART 64
typedef struct DsaltRmsNormParams {
  const void* x;              /* [T, d] dtype (backward: the normalised input) */
  const void* res;            /* [T, d] dtype, or NULL                    (forward) */
  void* x_sum;                /* [T, d] dtype, written when res is set    (forward) */
  const float* w;             /* [d] fp32, 16-byte aligned */
  void* y;                    /* [T, d] dtype                             (forward) */
  float* rstd;                /* [T] fp32: written by the forward, read by the backward */
  const void* dy;             /* [T, d] dtype                            (backward) */
  const void* dres;           /* [T, d] dtype, or NULL                   (backward) */
  void* dx;                   /* [T, d] dtype */
  float* dw_part;             /* [ceil(T / DSALT_RMSNORM_ROWS_PER_PART), d] fp32 */
  float* dw;                  /* [d] fp32, or NULL: the partials summed */
  int64_t T;
  int32_t d;
  float eps;
  int32_t dtype;
} DsaltRmsNormParams;
DSALT_API int dsalt_rmsnorm_fwd(const DsaltRmsNormParams* p, void* stream);
DSALT_API int dsalt_rmsnorm_bwd(const DsaltRmsNormParams* p, void* stream);

/* Cross-entropy of one chunk of LM-head logits (dsalt/model/dsalt_lm.py:19-39:
 * F.cross_entropy, fp32 math, sum reduction) with its gradient written over
 * the logits: row_loss[r] = logsumexp(l_r) − l_r[y_r] (0 when y_r is
 * ignore_index), l_r := (softmax(l_r) − onehot(y_r)) · *scale (0 for ignored
 * rows), rounded to dtype (f16 / bf16).  *scale is typically 1 / #valid labels. */
typedef struct DsaltXentParams {
  void* logits;               /* [rows, vocab] dtype, 16-byte aligned; overwritten */
  const int64_t* labels;      /* [rows] */
  float* row_loss;            /* [rows] fp32 */
  const float* scale;         /* device scalar */
  int64_t rows;
  int32_t vocab;
  int32_t ignore_index;
  int32_t dtype;
} DsaltXentParams;
DSALT_API int dsalt_xent_fwd_grad(const DsaltXentParams* p, void* stream);

/* SwiGLU activation of the feed-forward blocks (dsalt/modules/dsalt_transformer.py:
 * 10-21, silu(gate(x)) * up(x) under autocast), f16 / bf16, fp32 math with the
 * rounding of the torch ops it replaces:
 *   forward   s = R(g / (1 + exp(-g))), h = R(s·u)
 *   backward  du = R(dh·s), dg = R(R(dh·u)·σ·(1 + g·(1 − σ))), σ = sigmoid(g)
 * g and u are [T, F] with row stride ld_in (the two halves of a [T, 2F] GEMM
 * output when ld_in = 2F); dg and du use row stride ld_out; h and dh are dense
 * [T, F].  F, ld_in and ld_out are multiples of 8; pointers 16-byte aligned. */
typedef struct DsaltSwigluParams {
  const void* g;              /* [T, F] stride ld_in */
  const void* u;              /* [T, F] stride ld_in */
  void* h;                    /* [T, F]                          (forward) */
  const void* dh;             /* [T, F]                         (backward) */
  void* dg;                   /* [T, F] stride ld_out           (backward) */
  void* du;                   /* [T, F] stride ld_out           (backward) */
  int64_t T;
  int64_t F;
  int64_t ld_in;
  int64_t ld_out;
  int32_t dtype;
} DsaltSwigluParams;
DSALT_API int dsalt_swiglu_fwd(const DsaltSwigluParams* p, void* stream);
DSALT_API int dsalt_swiglu_bwd(const DsaltSwigluParams* p, void* stream);

/* ---- self-test of the failure path ---------------------------------------
 * Launches one CTA whose mbarrier wait can never complete.  The bounded wait
 * every tensor-core kernel uses gives up after its limit (about 2 s), ORs
 * DSALT_DEV_WAIT_TIMEOUT into *status (a device int32) and the kernel returns
 * normally: the stream and the context stay usable.                          */
DSALT_API int dsalt_selftest_wait_timeout(int32_t* status, void* stream);

/* ---- introspection ------------------------------------------------------- */
DSALT_API int dsalt_b200_abi_version(void);
DSALT_API const char* dsalt_b200_status_string(int status);
/* sizeof of the parameter structs, for bindings to check their mirrors:
 * which = 0 schedule, 1 gather, 2 attn, 3 score, 4 topk, 5 win_gate, 6 rope,
 * 7 rmsnorm, 8 scale_rows, 9 xent, 10 swiglu, 11 win_gate_bwd,
 * 12 score_bwd                                                              */
DSALT_API int dsalt_b200_params_sizeof(int which);

#ifdef __cplusplus
}
#endif
#endif /* DSALT_B200_H */
