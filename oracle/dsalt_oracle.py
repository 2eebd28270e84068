"""CPU oracle for the DSALT sparse-attention hot path (test infrastructure only).

This module is a numpy restatement of the reference library's algorithm
(LeonardoCofone/dsalt-library, ``dsalt`` v1.0.0).  It is the checker the CUDA
path is compared with; nothing in the shipped package imports it.  Only
``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / reference
arm of ``bench.py`` may call it.

Pinning: ``tests/golden/make_golden.py`` runs the reference's own code (its
dense SDPA training path, its selectors and its Triton kernels under the Triton
interpreter) on seeded inputs and stores the results in ``tests/golden/``;
``tests/test_oracle_golden.py`` checks every function below against them.

Every function cites the reference file:line it restates (paths relative to the
reference project root).

Numerics: the attention math runs in float64 by default (``dtype`` argument),
with the comparisons that decide set membership (band, landmark validity,
window exclusion) done in float32 exactly as the reference kernels do, so the
attended sets are identical to the reference's.
"""

from __future__ import annotations

import math

import numpy as np

LOG2E = 1.4426950408889634


# --------------------------------------------------------------------------- #
#  bf16 emulation
# --------------------------------------------------------------------------- #
def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), as float32.

    Matches ``torch.Tensor.to(torch.bfloat16)`` for finite inputs.
    """
    f = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    bits = f.view(np.uint32).astype(np.uint64)
    rounding = ((bits >> 16) & 1) + 0x7FFF
    out = ((bits + rounding) & 0xFFFF0000).astype(np.uint32)
    res = out.view(np.float32).copy()
    nan = np.isnan(f)
    res[nan] = np.nan
    return res


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    """Widen raw bfloat16 bit patterns (uint16) to float32."""
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(a) -> np.ndarray:
    """Raw bfloat16 bit patterns of ``bf16_round(a)``."""
    return (bf16_round(a).view(np.uint32) >> 16).astype(np.uint16)


# --------------------------------------------------------------------------- #
#  window gate  (dsalt/modules/dsalt_attention.py:270-284)
# --------------------------------------------------------------------------- #
def _sigmoid32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def window_from_logits(logits, n_min: int, n_max: int, dtype: str = "fp32") -> np.ndarray:
    """``w̃ = n_min + σ(logit)·(n_max − n_min)`` (dsalt_attention.py:274-275).

    ``dtype="bf16"`` reproduces autocast: the Linear output is bf16 and every
    elementwise op rounds its result to bf16 (sigmoid, the product with the
    Python int, the sum with the Python int).
    """
    lg = np.asarray(logits, dtype=np.float32)
    span = np.float32(n_max - n_min)
    if dtype == "bf16":
        lg = bf16_round(lg)
        s = bf16_round(_sigmoid32(lg))
        t = bf16_round(s * span)
        return bf16_round(np.float32(n_min) + t)
    s = _sigmoid32(lg)
    return (np.float32(n_min) + s * span).astype(np.float32)


def window_logits(x, weight, bias) -> np.ndarray:
    """``win_gate(x)`` logits in float64 (``nn.Linear(d_model, 1)``, dsalt_attention.py:223,274)."""
    x = np.asarray(x, dtype=np.float64)
    return x @ np.asarray(weight, dtype=np.float64).reshape(-1) + float(np.asarray(bias).reshape(-1)[0])


def window_discrete(w_cont) -> np.ndarray:
    """``floor(w̃).clamp(min=1)`` used by the selection (dsalt_attention.py:471)."""
    return np.maximum(np.floor(np.asarray(w_cont, dtype=np.float32)), np.float32(1.0))


# --------------------------------------------------------------------------- #
#  hybrid landmark score  (dsalt/kernels/landmark_tokens_ker.py:19-61)
# --------------------------------------------------------------------------- #
def hybrid_scores(x, W_V, alpha, n_heads: int, dh: int):
    """``s = α·z(‖x W_Vᵀ‖) + (1−α)·z(‖x‖)`` per head.

    z standardises over ALL packed tokens with the unbiased std clamped at 1e-6
    (landmark_tokens_ker.py:47-55); under GQA the kv-head value norm is repeated
    to its query heads (:56-58).  Returns ``(scores [T,H], z_x [T], z_v [T,H])``
    as float64.
    """
    x = np.asarray(x, dtype=np.float64)
    W_V = np.asarray(W_V, dtype=np.float64)
    alpha = np.asarray(alpha, dtype=np.float64).reshape(-1)
    T = x.shape[0]
    x_norm = np.linalg.norm(x, axis=-1)
    sd = x_norm.std(ddof=1) if T > 1 else float("nan")
    z_x = (x_norm - x_norm.mean()) / max(sd, 1e-6) if T > 1 else np.full(T, np.nan)
    n_kv = W_V.shape[0] // dh
    xwv = np.linalg.norm((x @ W_V.T).reshape(T, n_kv, dh), axis=-1)
    mu_v = xwv.mean(0, keepdims=True)
    sd_v = np.maximum(xwv.std(0, ddof=1, keepdims=True), 1e-6) if T > 1 else np.full((1, n_kv), np.nan)
    z_v = (xwv - mu_v) / sd_v
    if n_kv != n_heads:
        z_v = np.repeat(z_v, n_heads // n_kv, axis=1)
    scores = alpha[None, :] * z_v + (1.0 - alpha[None, :]) * z_x[:, None]
    return scores, z_x, z_v


# --------------------------------------------------------------------------- #
#  landmark top-k  (dsalt/kernels/selectors.py:75-134)
# --------------------------------------------------------------------------- #
def seq_offsets(cu) -> np.ndarray:
    """Position of every packed token inside its own sequence (selectors.py:24-27)."""
    cu = np.asarray(cu, dtype=np.int64)
    out = np.empty(int(cu[-1]), dtype=np.int64)
    for b in range(len(cu) - 1):
        out[cu[b]:cu[b + 1]] = np.arange(cu[b + 1] - cu[b])
    return out


def landmark_indices(scores, w_sizes, cu, k_lmk: int) -> np.ndarray:
    """Top-``k_lmk`` landmark positions per (head, sequence).

    Tokens with ``seq_off < w_sizes.long()`` are excluded (selectors.py:105-107,
    the token's OWN window), the top-k runs over every position of the sequence
    (:117-133), and slots whose score is not finite hold -1.  The reference's
    ``torch.topk(sorted=False)`` leaves the slot order unspecified; this oracle
    returns the selected positions ordered by descending score with ties
    broken by the lower position, and the tests compare sets.
    Returns ``int64 [H, S, k_lmk]`` (positions relative to the sequence start).
    """
    scores = np.asarray(scores, dtype=np.float64)
    cu = np.asarray(cu, dtype=np.int64)
    T, H = scores.shape
    S = len(cu) - 1
    off = seq_offsets(cu)
    covered = off < np.asarray(w_sizes).astype(np.int64)
    out = np.full((H, S, k_lmk), -1, dtype=np.int64)
    lens = cu[1:] - cu[:-1]
    max_len = int(lens.max()) if S > 0 else 0
    k_eff = min(k_lmk, max_len)
    for b in range(S):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        for h in range(H):
            sc = scores[s0:s1, h].copy()
            sc[covered[s0:s1]] = -np.inf
            # torch.topk ranks NaN above +inf above every finite score (the
            # non-finite winners then become -1 slots, selectors.py:131-132)
            rank_key = np.where(np.isnan(sc), 2.0, np.where(sc == np.inf, 1.0, 0.0))
            finite_sc = np.where(np.isfinite(sc), sc, np.where(sc == -np.inf, -np.inf, 0.0))
            order = np.lexsort((np.arange(s1 - s0), -finite_sc, -rank_key))  # score desc, position asc
            sel = order[:k_eff]
            sel = [int(p) for p in sel if np.isfinite(sc[p])]
            out[h, b, :len(sel)] = sel
    return out


def landmark_logw(scores, lmk_pos, cu, tau_lmk: float = 2.0) -> np.ndarray:
    """``log σ(s_sel/τ_lmk)`` clamped at 1e-20, −inf on empty slots (dsalt_attention.py:480-486)."""
    scores = np.asarray(scores, dtype=np.float64)
    cu = np.asarray(cu, dtype=np.int64)
    H, S, k = lmk_pos.shape
    abs_pos = cu[:-1][None, :, None] + np.maximum(lmk_pos, 0)
    s_sel = scores[abs_pos, np.arange(H)[:, None, None]]
    sig = 1.0 / (1.0 + np.exp(-s_sel / tau_lmk))
    lw = np.log(np.maximum(sig, 1e-20))
    return np.where(lmk_pos >= 0, lw, -np.inf)


def landmark_logw_grad_alpha(d_logw, scores, z_x, z_v, lmk_pos, cu, tau_lmk: float = 2.0) -> np.ndarray:
    """∂loss/∂α per head from ``d_logw`` through ``log σ(s/τ)`` and ``s = α z_v + (1−α) z_x``.

    Restates the autograd chain the reference builds in dsalt_attention.py:477-486
    and landmark_tokens_ker.py:60.  Returns ``[H]``.
    """
    cu = np.asarray(cu, dtype=np.int64)
    H, S, k = lmk_pos.shape
    abs_pos = cu[:-1][None, :, None] + np.maximum(lmk_pos, 0)
    hix = np.arange(H)[:, None, None]
    s_sel = np.asarray(scores, dtype=np.float64)[abs_pos, hix]
    sig = 1.0 / (1.0 + np.exp(-s_sel / tau_lmk))
    dlw_ds = (1.0 - sig) / tau_lmk
    ds_dalpha = np.asarray(z_v, dtype=np.float64)[abs_pos, hix] - np.asarray(z_x, dtype=np.float64)[abs_pos]
    g = np.where(lmk_pos >= 0, np.asarray(d_logw, dtype=np.float64) * dlw_ds * ds_dalpha, 0.0)
    return g.sum(axis=(1, 2))


# --------------------------------------------------------------------------- #
#  attention: attended set and log-bias
# --------------------------------------------------------------------------- #
def _band_bias(L, w_seq, tau_win, win_edge, semantics):
    """Dense ``[L, L]`` band log-bias of one sequence, d(bias)/d(w̃) and the landmark threshold.

    Training semantics (dsalt/kernels/dsalt_triton_train.py:145-156; dense twin
    dsalt/modules/dsalt_attention.py:534-541): band ``0 ≤ d ≤ w̃`` with ``d = i − j``,
    bias 0 in the core ``d ≤ w̃ − win_edge`` and ``log σ((w̃ − d)/τ_win)`` on the edge.
    Inference semantics (dsalt/kernels/dsalt_triton_attn.py:102-105): band
    ``i − w + 1 ≤ j ≤ i`` with ``w = max(int(w), 1)`` and no bias.
    Also returns, per query, the bound ``win_lo`` of the landmark rule
    (train: ``float32(i) − w̃``, :183; infer: ``i − w + 1``, dsalt_triton_attn.py:133).
    """
    i = np.arange(L)
    d = (i[:, None] - i[None, :]).astype(np.float32)
    dbias_dw = np.zeros((L, L))
    if semantics == "train":
        w32 = np.asarray(w_seq, dtype=np.float32)[:, None]
        band = (d >= 0) & (d <= w32)
        core = d <= (w32 - np.float32(win_edge))
        z = (w32.astype(np.float64) - d.astype(np.float64)) / tau_win
        with np.errstate(over="ignore"):
            logedge = -np.log1p(np.exp(-z))
            sig = 1.0 / (1.0 + np.exp(-z))
        bias = np.where(band, np.where(core, 0.0, logedge), -np.inf)
        dbias_dw = np.where(band & ~core, (1.0 - sig) / tau_win, 0.0)
        win_lo = i.astype(np.float32) - np.asarray(w_seq, dtype=np.float32)   # float32, as the kernel
    else:
        w_int = np.maximum(np.asarray(w_seq).astype(np.int64), 1)[:, None]
        jj = i[None, :]
        band = (jj >= i[:, None] - w_int + 1) & (jj <= i[:, None])
        bias = np.where(band, 0.0, -np.inf)
        win_lo = (i - w_int[:, 0] + 1)
    return bias, dbias_dw, win_lo


def _landmark_bias(L, pos_h, lw_h, win_lo, semantics):
    """``[L, k]`` log-bias of the landmark slots of one (sequence, head).

    Slot ``c`` at position ``p`` is a separate key column (as in the reference
    kernels, dsalt_triton_train.py:168-198, where each landmark slot is a column
    of the landmark tile), valid for query ``i`` iff ``0 ≤ p < len``, ``p ≤ i`` and
    ``p < win_lo(i)`` (train: compared in float32), with bias ``lmk_logw[c]``.
    Band and landmark keys are disjoint for every query.
    """
    i = np.arange(L)
    k = len(pos_h)
    bias = np.full((L, k), -np.inf)
    for c, (p, lw) in enumerate(zip(pos_h, lw_h)):
        p = int(p)
        if p < 0 or p >= L:
            continue
        if semantics == "train":
            ok = (p <= i) & (np.float32(p) < win_lo)
        else:
            ok = (p <= i) & (p < win_lo)
        bias[ok, c] = float(lw)
    return bias


def _rows_softmax(logits):
    m = logits.max(axis=1, keepdims=True)
    empty = ~np.isfinite(m[:, 0])
    m = np.where(np.isfinite(m), m, 0.0)
    e = np.exp(logits - m)
    l = e.sum(axis=1, keepdims=True)
    P = np.where(empty[:, None], 0.0, e / np.where(l > 0, l, 1.0))
    lse = np.where(empty, -np.inf, m[:, 0] + np.log(np.where(l[:, 0] > 0, l[:, 0], 1.0)))
    return P, lse


def attention_fwd(q, k, v, lmk_pos, lmk_logw, w, cu, tau_win=1.0, win_edge=4.0,
                  semantics="train", dtype=np.float64):
    """Forward ``O [T,H,D]`` and ``LSE [T,H]`` of the DSALT attention.

    Restates ``_train_fwd_kernel`` (dsalt/kernels/dsalt_triton_train.py:74-214) for
    ``semantics="train"`` and ``_dsalt_fwd_kernel`` (dsalt/kernels/dsalt_triton_attn.py:27-169)
    for ``"infer"`` (then ``lmk_logw`` is the additive ``lmk_bias``).  Scale ``1/√D``;
    rows with an empty attended set give ``O = 0`` and ``LSE = −inf``.
    """
    out = _attention(q, k, v, None, lmk_pos, lmk_logw, w, cu, tau_win, win_edge, semantics, dtype)
    return out["o"], out["lse"]


def attention_bwd(q, k, v, do, lmk_pos, lmk_logw, w, cu, tau_win=1.0, win_edge=4.0,
                  semantics="train", dtype=np.float64):
    """Gradients of the DSALT attention.

    Restates the backward of ``DSALTTrainFunction`` (dsalt/kernels/dsalt_triton_train.py:665-760:
    ``_train_bwd_preprocess`` :220-237, ``_train_bwd_dkdv_kernel`` :386-481, ``_train_bwd_kernel``
    :240-383).  Returns a dict with ``dq, dk, dv [T,H,D]``, ``d_logw [H,S,k]`` (the landmark
    log-weight / inference ``d_bias`` gradient), ``d_w [T]`` (∂loss/∂w̃ summed over heads, train
    only) and the forward ``o``, ``lse``.
    """
    return _attention(q, k, v, do, lmk_pos, lmk_logw, w, cu, tau_win, win_edge, semantics, dtype)


def _attention(q, k, v, do, lmk_pos, lmk_logw, w, cu, tau_win, win_edge, semantics, dtype):
    q = np.asarray(q, dtype=dtype)
    k = np.asarray(k, dtype=dtype)
    v = np.asarray(v, dtype=dtype)
    cu = np.asarray(cu, dtype=np.int64)
    lmk_pos = np.asarray(lmk_pos, dtype=np.int64)
    lmk_logw = np.asarray(lmk_logw, dtype=np.float64)
    T, H, D = q.shape
    S = len(cu) - 1
    scale = 1.0 / math.sqrt(D)
    o = np.zeros((T, H, D), dtype=dtype)
    lse = np.full((T, H), -np.inf)
    want_bwd = do is not None
    if want_bwd:
        do = np.asarray(do, dtype=dtype)
        dq = np.zeros_like(q)
        dk = np.zeros_like(k)
        dv = np.zeros_like(v)
        d_logw = np.zeros(lmk_pos.shape, dtype=np.float64)
        d_w = np.zeros((T, H), dtype=np.float64)
    for b in range(S):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        L = s1 - s0
        if L == 0:
            continue
        w_seq = np.asarray(w)[s0:s1]
        band_bias, dbias_dw, win_lo = _band_bias(L, w_seq, tau_win, win_edge, semantics)
        for h in range(H):
            pos = lmk_pos[h, b]
            lmk_bias = _landmark_bias(L, pos, lmk_logw[h, b], win_lo, semantics)
            pc = np.clip(pos, 0, L - 1)
            qs, ks, vs = q[s0:s1, h], k[s0:s1, h], v[s0:s1, h]
            kl, vl = ks[pc], vs[pc]                       # landmark slot keys / values [k, D]
            logits = np.concatenate([(qs @ ks.T) * scale + band_bias,
                                     (qs @ kl.T) * scale + lmk_bias], axis=1)
            P, lse_h = _rows_softmax(logits)
            Pb, Pl = P[:, :L], P[:, L:]
            oh = Pb @ vs + Pl @ vl
            o[s0:s1, h] = oh
            lse[s0:s1, h] = lse_h
            if not want_bwd:
                continue
            dos = do[s0:s1, h]
            delta = (dos * oh).sum(axis=1, keepdims=True)
            dSb = Pb * (dos @ vs.T - delta)
            dSl = Pl * (dos @ vl.T - delta)
            dq[s0:s1, h] += (dSb @ ks + dSl @ kl) * scale
            dkh = (dSb.T @ qs) * scale
            dvh = Pb.T @ dos
            np.add.at(dkh, pc, (dSl.T @ qs) * scale)
            np.add.at(dvh, pc, Pl.T @ dos)
            dk[s0:s1, h] += dkh
            dv[s0:s1, h] += dvh
            d_w[s0:s1, h] = (dSb * dbias_dw).sum(axis=1)
            d_logw[h, b] = dSl.sum(axis=0)
    res = {"o": o, "lse": lse}
    if want_bwd:
        res.update(dq=dq, dk=dk, dv=dv, d_logw=d_logw, d_w=d_w.sum(axis=1), d_w_head=d_w)
    return res


def attention_fwd_rows(q, k, v, lmk_pos, lmk_logw, w, cu, rows, tau_win=1.0, win_edge=4.0,
                       semantics="train", dtype=np.float64):
    """``O`` and ``LSE`` of selected ``(token, head)`` rows only, for sequences too long
    for the dense per-sequence matrices of ``attention_fwd``.  Same definitions as
    ``_band_bias`` / ``_landmark_bias`` (dsalt/kernels/dsalt_triton_train.py:145-198,
    dsalt/kernels/dsalt_triton_attn.py:102-135), one row at a time.  Returns
    ``(o [n, D], lse [n])``.
    """
    cu = np.asarray(cu, dtype=np.int64)
    lmk_pos = np.asarray(lmk_pos, dtype=np.int64)
    lmk_logw = np.asarray(lmk_logw, dtype=np.float64)
    w = np.asarray(w)
    D = q.shape[2]
    scale = 1.0 / math.sqrt(D)
    out_o = np.zeros((len(rows), D))
    out_lse = np.full(len(rows), -np.inf)
    for n, (t, h) in enumerate(rows):
        b = int(np.searchsorted(cu, t, side="right") - 1)
        s0, L = int(cu[b]), int(cu[b + 1] - cu[b])
        i = t - s0
        j = np.arange(i + 1)
        d = (i - j).astype(np.float32)
        if semantics == "train":
            w32 = np.float32(w[t])
            band = (d >= 0) & (d <= w32)
            core = d <= (w32 - np.float32(win_edge))
            z = (np.float64(w32) - d.astype(np.float64)) / tau_win
            with np.errstate(over="ignore"):
                logedge = -np.log1p(np.exp(-z))
            bb = np.where(band, np.where(core, 0.0, logedge), -np.inf)
            win_lo = np.float32(i) - w32
        else:
            w_int = max(int(np.int64(w[t])), 1)
            bb = np.where(j >= i - w_int + 1, 0.0, -np.inf)
            win_lo = i - w_int + 1
        qi = np.asarray(q[t, h], dtype=dtype)
        ks = np.asarray(k[s0:s0 + i + 1, h], dtype=dtype)
        vs = np.asarray(v[s0:s0 + i + 1, h], dtype=dtype)
        logits = [(ks @ qi) * scale + bb]
        vals = [vs]
        pos = lmk_pos[h, b]
        lb = np.full(len(pos), -np.inf)
        for c, p in enumerate(pos):
            p = int(p)
            if p < 0 or p >= L:
                continue
            ok = p <= i and ((np.float32(p) < win_lo) if semantics == "train" else (p < win_lo))
            if ok:
                lb[c] = lmk_logw[h, b, c]
        pc = np.clip(pos, 0, L - 1) + s0
        logits.append((np.asarray(k[pc, h], dtype=dtype) @ qi) * scale + lb)
        vals.append(np.asarray(v[pc, h], dtype=dtype))
        lg = np.concatenate(logits)
        m = lg.max()
        if not np.isfinite(m):
            continue
        e = np.exp(lg - m)
        out_o[n] = (e[:, None] * np.concatenate(vals)).sum(axis=0) / e.sum()
        out_lse[n] = m + np.log(e.sum())
    return out_o, out_lse


# --------------------------------------------------------------------------- #
#  work accounting (roofline denominator)
# --------------------------------------------------------------------------- #
def attended_pairs(w, lmk_pos, cu, semantics="train") -> int:
    """``P = Σ_(seq,h,i) |W(i)| + |L(i)|`` for the FLOP count ``4·D·P`` (fwd) / ``14·D·P`` (fwd+bwd)."""
    cu = np.asarray(cu, dtype=np.int64)
    lmk_pos = np.asarray(lmk_pos, dtype=np.int64)
    H, S, _ = lmk_pos.shape
    total = 0
    for b in range(S):
        s0, s1 = int(cu[b]), int(cu[b + 1])
        L = s1 - s0
        if L == 0:
            continue
        i = np.arange(L)
        w_seq = np.asarray(w)[s0:s1]
        if semantics == "train":
            w32 = np.asarray(w_seq, dtype=np.float32)
            nw = np.where(w32 >= 0, np.minimum(np.floor(w32), i) + 1, 0).astype(np.int64)
            win_lo = i.astype(np.float32) - w32
        else:
            wi = np.maximum(w_seq.astype(np.int64), 1)
            nw = np.minimum(wi, i + 1)
            win_lo = i - wi + 1
        for h in range(H):
            total += int(nw.sum())
            for p in lmk_pos[h, b]:
                p = int(p)
                if 0 <= p < L:
                    if semantics == "train":
                        total += int(((p <= i) & (np.float32(p) < win_lo)).sum())
                    else:
                        total += int(((p <= i) & (p < win_lo)).sum())
    return total
