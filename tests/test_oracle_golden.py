"""The numpy oracle against golden vectors produced by the reference's own code.

Fixtures come from ``tests/golden/make_golden.py`` (reference dense SDPA path,
reference selectors, reference Triton kernels under the Triton interpreter).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import dsalt_oracle as O


def _np(t):
    return t.detach().float().numpy() if torch.is_tensor(t) else np.asarray(t)


# ----------------------------------------------------------------- selectors
@pytest.mark.parametrize("case", ["varlen", "uniform", "gqa"])
def test_hybrid_scores_match_reference(golden_selectors, case):
    g = golden_selectors[case]
    H = g["alpha"].shape[0]
    s, zx, zv = O.hybrid_scores(_np(g["x"]), _np(g["W_V"]), _np(g["alpha"]), H, int(g["dh"]))
    np.testing.assert_allclose(s, _np(g["scores"]), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(zx, _np(g["z_x"]), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(zv, _np(g["z_v"]), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("case", ["varlen", "uniform", "gqa"])
def test_landmark_sets_match_reference(golden_selectors, case):
    g = golden_selectors[case]
    idx = O.landmark_indices(_np(g["scores"]), _np(g["w_disc"]), _np(g["cu"]), int(g["k"]))
    ref = g["idx"].numpy()
    assert idx.shape == ref.shape
    for h in range(ref.shape[0]):
        for b in range(ref.shape[1]):
            assert sorted(idx[h, b].tolist()) == sorted(ref[h, b].tolist()), (h, b)


def test_window_bf16_bit_exact():
    g = load_golden("window.pt")
    w = O.window_from_logits(_np(g["logits"]), int(g["n_min"]), int(g["n_max"]), "bf16")
    assert np.array_equal(w, _np(g["w_bf16"]))


def test_window_fp32_close():
    g = load_golden("window.pt")
    w = O.window_from_logits(_np(g["logits"]), int(g["n_min"]), int(g["n_max"]), "fp32")
    ref = _np(g["w_fp32"])
    # numpy's and torch's float32 exp may differ in the last ulp
    assert np.max(np.abs(w - ref) / np.spacing(ref)) <= 2
    assert np.array_equal(O.window_discrete(w), O.window_discrete(ref))


# ----------------------------------------------------------------- attention
TRAIN_CASES = ["train_small", "train_d128", "train_ragged", "train_intw"]


def _run_oracle(g, semantics="train"):
    i = g["inputs"]
    return O.attention_bwd(_np(i["q"]), _np(i["k"]), _np(i["v"]), _np(i["do"]), i["pos"].numpy(),
                           _np(i["logw"] if semantics == "train" else i["bias"]), _np(i["w"]),
                           i["cu"].numpy(), 1.0, 4.0, semantics)


@pytest.mark.parametrize("case", TRAIN_CASES)
def test_oracle_matches_reference_dense_fp32(golden_ops, case):
    g = golden_ops[case]
    r = _run_oracle(g)
    d = g["dense"]
    for key in ("o", "dq", "dk", "dv"):
        np.testing.assert_allclose(r[key], _np(d[key]), atol=1e-4, rtol=1e-4, err_msg=key)
    np.testing.assert_allclose(r["d_w"], _np(d["d_w"]), atol=1e-4, rtol=1e-4, err_msg="d_w")
    np.testing.assert_allclose(r["d_logw"], _np(d["d_logw"]), atol=1e-4, rtol=1e-4, err_msg="d_logw")


@pytest.mark.parametrize("case", TRAIN_CASES)
def test_oracle_matches_reference_triton_fp16(golden_ops, case):
    g = golden_ops[case]
    r = _run_oracle(g)
    t = g["triton"]
    for key in ("o", "dq", "dk", "dv", "d_w", "d_logw"):
        ref = _np(t[key])
        got = r[key]
        np.testing.assert_allclose(got, ref, atol=2e-2, rtol=1e-2, err_msg=key)


def test_oracle_matches_reference_triton_infer(golden_ops):
    g = golden_ops["infer_small"]
    r = _run_oracle(g, "infer")
    t = g["triton"]
    for key, rk in (("o", "o"), ("dq", "dq"), ("dk", "dk"), ("dv", "dv"), ("d_bias", "d_logw")):
        np.testing.assert_allclose(r[rk], _np(t[key]), atol=2e-2, rtol=1e-2, err_msg=key)


def test_attended_pairs_small():
    # one sequence of 5 tokens, w̃ = 1.5 everywhere, one landmark at 0
    w = np.full(5, 1.5, dtype=np.float32)
    pos = np.array([[[0]]])
    # band sizes min(floor(1.5), i)+1 = 1,2,2,2,2 ; landmark 0 valid for i with 0 < i-1.5 → i ≥ 2
    assert O.attended_pairs(w, pos, [0, 5]) == 9 + 3


@pytest.mark.parametrize("semantics", ["train", "infer"])
def test_rowwise_oracle_matches_dense(semantics):
    """The row-at-a-time restatement used for long sequences equals the dense one."""
    rng = np.random.default_rng(5)
    lens = [70, 33]
    T, H, D, k = sum(lens), 2, 16, 6
    q, kk, v = (rng.standard_normal((T, H, D)) for _ in range(3))
    w = rng.uniform(1.0, 40.0, T)
    cu = np.array([0, 70, 103])
    pos = np.full((H, 2, k), -1)
    for h in range(H):
        for b, L in enumerate(lens):
            pos[h, b, :4] = rng.choice(L, 4, replace=False)
    lw = np.where(pos >= 0, np.log(1 / (1 + np.exp(-rng.standard_normal((H, 2, k))))), -np.inf)
    o, lse = O.attention_fwd(q, kk, v, pos, lw, w, cu, semantics=semantics)
    rows = [(t, h) for t in range(T) for h in range(H)]
    o_r, lse_r = O.attention_fwd_rows(q, kk, v, pos, lw, w, cu, rows, semantics=semantics)
    np.testing.assert_allclose(o_r, np.array([o[t, h] for t, h in rows]), rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(lse_r, np.array([lse[t, h] for t, h in rows]), rtol=1e-12, atol=1e-12)
