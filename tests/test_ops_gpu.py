"""GPU parity tests of the DSALT attention op against the oracle and the reference goldens.

Tolerances (north_star): bf16/fp16 outputs within max-abs 2e-2 / rel 1e-2,
fp32 within 1e-4, on O, dQ, dK, dV, d_w̃ and d_logw.
"""

from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import dsalt_oracle as O

pytestmark = pytest.mark.gpu

TOL = {torch.float32: (1e-4, 1e-4), torch.float16: (2e-2, 1e-2), torch.bfloat16: (2e-2, 1e-2)}
TRAIN_CASES = ["train_small", "train_d128", "train_ragged", "train_intw"]


def _close(got, ref, dtype, what):
    atol, rtol = TOL[dtype]
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    err = np.abs(got - ref) - (atol + rtol * np.abs(ref))
    bad = err > 0
    assert not bad.any(), f"{what}: {bad.sum()} / {bad.size} outside tol, max abs err " \
                          f"{np.abs(got - ref).max():.3e}"


def run_train(inp, dtype, impl=None, tau=1.0, edge=4.0, n_max=256, semantics="train"):
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    from dsalt.kernels.dsalt_triton_attn import dsalt_triton_attention
    if impl is not None:
        os.environ["DSALT_IMPL"] = impl
    try:
        dev = torch.device("cuda")
        q = inp["q"].to(dev, dtype).requires_grad_(True)
        k = inp["k"].to(dev, dtype).requires_grad_(True)
        v = inp["v"].to(dev, dtype).requires_grad_(True)
        cu = inp["cu"].to(dev)
        pos = inp["pos"].to(dev)
        if semantics == "train":
            w = inp["w"].to(dev).float().requires_grad_(True)
            lw = inp["logw"].to(dev).float().requires_grad_(True)
            o = dsalt_triton_train_attention(q, k, v, pos, lw, w, cu, tau, edge, n_max)
        else:
            w = inp["w"].to(dev).float()
            lw = inp["bias"].to(dev).float().requires_grad_(True)
            o = dsalt_triton_attention(q, k, v, pos, lw, w, cu)
        o.backward(inp["do"].to(dev, torch.float32))
        torch.cuda.synchronize()
        from dsalt.kernels.dsalt_cuda import check_device_status
        check_device_status(dev)
        res = dict(o=o.detach(), dq=q.grad, dk=k.grad, dv=v.grad, d_logw=lw.grad)
        if semantics == "train":
            res["d_w"] = w.grad
        return {kk: vv.float().cpu().numpy() for kk, vv in res.items()}
    finally:
        if impl is not None:
            os.environ.pop("DSALT_IMPL", None)


def oracle_train(inp, dtype, semantics="train", tau=1.0, edge=4.0):
    def rd(t):
        return t.to(dtype).float().numpy()
    return O.attention_bwd(rd(inp["q"]), rd(inp["k"]), rd(inp["v"]), rd(inp["do"]),
                           inp["pos"].numpy(),
                           (inp["logw"] if semantics == "train" else inp["bias"]).float().numpy(),
                           inp["w"].float().numpy(), inp["cu"].numpy(), tau, edge, semantics)


def _compare(res, ref, dtype, keys=("o", "dq", "dk", "dv", "d_w", "d_logw")):
    for key in keys:
        if key in ref and key in res:
            _close(res[key], ref[key], dtype, key)


# ------------------------------------------------------------ golden pins
@pytest.mark.parametrize("case", TRAIN_CASES)
def test_train_fp32_matches_reference_dense(golden_ops, case):
    g = golden_ops[case]
    res = run_train(g["inputs"], torch.float32, n_max=int(g["n_max"]))
    d = {k: v.float().numpy() for k, v in g["dense"].items()}
    _compare(res, d, torch.float32)


@pytest.mark.parametrize("case", TRAIN_CASES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_train_half_matches_reference_triton(golden_ops, case, dtype):
    g = golden_ops[case]
    res = run_train(g["inputs"], dtype, n_max=int(g["n_max"]))
    if dtype == torch.float16:
        ref = {k: v.float().numpy() for k, v in g["triton"].items()}
    else:
        ref = oracle_train(g["inputs"], dtype)
    _compare(res, ref, dtype)


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_infer_matches_reference_triton(golden_ops, dtype):
    g = golden_ops["infer_small"]
    res = run_train(g["inputs"], dtype, semantics="infer")
    if dtype == torch.float16:
        t = g["triton"]
        ref = dict(o=t["o"], dq=t["dq"], dk=t["dk"], dv=t["dv"], d_logw=t["d_bias"])
        ref = {k: v.float().numpy() for k, v in ref.items()}
    else:
        ref = oracle_train(g["inputs"], torch.float32, semantics="infer")
    _compare(res, ref, dtype, keys=("o", "dq", "dk", "dv", "d_logw"))


# ------------------------------------------------------------ seeded cases
def make_inputs(lens, H, D, k, w_lo, w_hi, seed, empty_slots=1, dup=False):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q, kk, v, do = (torch.randn(T, H, D, generator=g) for _ in range(4))
    w = w_lo + torch.rand(T, generator=g) * (w_hi - w_lo)
    S = len(lens)
    pos = torch.full((H, S, k), -1, dtype=torch.long)
    for h in range(H):
        for b, L in enumerate(lens):
            n = max(0, min(k - empty_slots, L))
            if n:
                pos[h, b, :n] = torch.randperm(L, generator=g)[:n]
            if dup and n >= 2:
                pos[h, b, 1] = pos[h, b, 0]
    lw = torch.log(torch.sigmoid(torch.randn(H, S, k, generator=g) / 2)).where(pos >= 0,
                                                                               torch.tensor(float("-inf")))
    cu = torch.tensor([0] + np.cumsum(lens).tolist(), dtype=torch.int32)
    return dict(q=q, k=kk, v=v, do=do, w=w, pos=pos, logw=lw, cu=cu)


SEEDED = {
    # name: (lens, H, D, k, w_lo, w_hi)
    "d128_long": ([700, 300], 2, 128, 64, 32.0, 512.0),
    "d64_multi": ([129, 128, 1, 255, 0, 77], 3, 64, 16, 1.0, 90.0),
    "tiny_windows": ([200], 2, 64, 8, -2.0, 5.0),      # w̃ < edge and w̃ < 0 rows
    "k_gt_len": ([10, 5], 2, 64, 32, 1.0, 4.0),          # more slots than tokens
    "no_landmarks": ([300], 1, 128, 0, 10.0, 60.0),
}


@pytest.mark.parametrize("case", list(SEEDED))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_train_seeded_vs_oracle(case, dtype):
    lens, H, D, k, wlo, whi = SEEDED[case]
    inp = make_inputs(lens, H, D, k, wlo, whi, seed=sum(map(ord, case)))
    res = run_train(inp, dtype)
    ref = oracle_train(inp, dtype)
    _compare(res, ref, dtype)


def test_wide_soft_edge():
    """A soft edge wider than the precomputed factors (win_edge 20 > 8 keys): the
    key-by-key fix-up paths of the dQ and dK/dV kernels."""
    inp = make_inputs([400, 150], 2, 128, 16, 24.0, 120.0, seed=31)
    res = run_train(inp, torch.bfloat16, edge=20.0)
    _compare(res, oracle_train(inp, torch.bfloat16, edge=20.0), torch.bfloat16)


def test_duplicate_landmark_positions():
    inp = make_inputs([150, 90], 2, 64, 8, 4.0, 40.0, seed=5, dup=True)
    _compare(run_train(inp, torch.float32), oracle_train(inp, torch.float32), torch.float32)


def test_backward_is_deterministic():
    inp = make_inputs([513, 260], 2, 128, 64, 16.0, 300.0, seed=9)
    a = run_train(inp, torch.bfloat16)
    b = run_train(inp, torch.bfloat16)
    for key in a:
        assert np.array_equal(a[key], b[key]), key


def test_simt_and_default_paths_agree():
    inp = make_inputs([640, 384], 2, 128, 64, 32.0, 400.0, seed=13)
    a = run_train(inp, torch.bfloat16, impl="simt")
    b = run_train(inp, torch.bfloat16)
    for key in a:
        _close(b[key], a[key], torch.bfloat16, key)


def test_bad_cu_seqlens_rejected_before_launch():
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    q = torch.randn(16, 1, 64, device="cuda")
    pos = torch.zeros(1, 2, 1, dtype=torch.long, device="cuda")
    with pytest.raises(ValueError):
        dsalt_triton_train_attention(q, q, q, pos, torch.zeros(1, 2, 1, device="cuda"),
                                     torch.ones(16, device="cuda"),
                                     torch.tensor([0, 9, 8], dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError):
        dsalt_triton_train_attention(q, q, q, pos, torch.zeros(1, 2, 1, device="cuda"),
                                     torch.ones(16, device="cuda"),
                                     torch.tensor([0, 4, 12], dtype=torch.int32, device="cuda"))


@pytest.mark.parametrize("semantics", ["infer", "train"])
def test_config5_long_context_rows_vs_oracle(semantics):
    """Config-5 shapes (one sequence of 32,768, D=128, k=256, windows 128…2048; 4 of
    the 32 heads, which are independent): sampled rows against the row-wise oracle."""
    from dsalt.kernels.dsalt_triton_attn import dsalt_triton_attention
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    from dsalt.kernels.selectors import select_topk
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(21)
    N, H, D, k = 32768, 4, 128, 256
    q, kk, v = (torch.randn(N, H, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3))
    w = 128.0 + torch.sigmoid(torch.randn(N, generator=g, device=dev)) * (2048.0 - 128.0)
    cu = torch.tensor([0, N], dtype=torch.int32, device=dev)
    scores = torch.randn(N, H, generator=g, device=dev)
    pos = select_topk(scores, w.floor().clamp(min=1), cu, k, N)
    if semantics == "infer":
        w_in = w.floor()
        bias = torch.zeros(H, 1, k, device=dev)
        o = dsalt_triton_attention(q, kk, v, pos, bias, w_in, cu)
        lw = bias
    else:
        w_in = w
        lw = torch.log(torch.sigmoid(torch.randn(H, 1, k, generator=g, device=dev) / 2))
        lw = torch.where(pos >= 0, lw, torch.full_like(lw, float("-inf")))
        o = dsalt_triton_train_attention(q, kk, v, pos, lw, w_in, cu, 1.0, 4.0, 2048)
    torch.cuda.synchronize()
    rng = np.random.default_rng(0)
    rows = [(int(t), int(h)) for t, h in zip(rng.integers(0, N, 48), rng.integers(0, H, 48))]
    rows += [(0, 0), (1, 1), (N - 1, 3), (2047, 2), (2048, 0)]
    qf, kf, vf = (x.float().cpu().numpy() for x in (q, kk, v))
    ref, _ = O.attention_fwd_rows(qf, kf, vf, pos.cpu().numpy(), lw.float().cpu().numpy(),
                                  w_in.float().cpu().numpy(), cu.cpu().numpy(), rows, semantics=semantics)
    got = np.stack([o[t, h].float().cpu().numpy() for t, h in rows])
    _close(got, ref, torch.bfloat16, f"o ({semantics})")
