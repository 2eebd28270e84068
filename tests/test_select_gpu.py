"""GPU tests of the selection and gating kernels against reference goldens."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle import dsalt_oracle as O

pytestmark = pytest.mark.gpu


def _win_gate(x, weight, bias, n_min, n_max):
    from dsalt.kernels import _ext
    T, d = x.shape
    w_cont = torch.empty(T, dtype=x.dtype, device=x.device)
    w_f32 = torch.empty(T, dtype=torch.float32, device=x.device)
    w_disc = torch.empty(T, dtype=torch.float32, device=x.device)
    p = _ext.WinGateParams(x=_ext.ptr(x), weight=_ext.ptr(weight), bias=_ext.ptr(bias),
                           w_cont=_ext.ptr(w_cont), w_f32=_ext.ptr(w_f32), w_disc=_ext.ptr(w_disc),
                           logits=0, T=T, d_model=d, n_min=float(n_min), n_max=float(n_max),
                           dtype=_ext.dtype_code(x.dtype))
    _ext.call("dsalt_win_gate", p)
    torch.cuda.synchronize()
    return w_cont, w_f32, w_disc


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_win_gate_bit_exact_at_fixed_logits(dtype):
    g = load_golden("window.pt")
    logits = g["logits"]
    T, d = logits.shape[0], 8
    x = torch.zeros(T, d)
    x[:, 0] = logits
    weight = torch.zeros(d)
    weight[0] = 1.0
    dev = torch.device("cuda")
    xd = x.to(dev, dtype).contiguous()
    w_cont, w_f32, w_disc = _win_gate(xd, weight.to(dev, dtype), torch.zeros(1, device=dev, dtype=dtype),
                                      int(g["n_min"]), int(g["n_max"]))
    ref = g["w_bf16"] if dtype == torch.bfloat16 else g["w_fp32"]
    got = w_cont.float().cpu()
    if dtype == torch.bfloat16:
        assert torch.equal(got, ref.float())
    else:
        # the golden comes from the reference on the host (torch's CPU sigmoid): within
        # 2 ulp; the same expression on this GPU (torch's CUDA sigmoid, which the
        # reference's _window_continuous runs on a CUDA device) bit-exactly
        ulp = (got - ref).abs() / torch.from_numpy(np.spacing(ref.numpy()))
        assert ulp.max() <= 2
        lg = logits.to(dev, torch.float32)
        on_gpu = float(g["n_min"]) + torch.sigmoid(lg) * (float(g["n_max"]) - float(g["n_min"]))
        assert torch.equal(w_cont, on_gpu)
    # the discrete window sizes against the reference's own floor(w̃).clamp(min=1)
    # (dsalt_attention.py:471), not against this kernel's output
    assert torch.equal(w_disc.cpu(), ref.float().floor().clamp(min=1))


@pytest.mark.parametrize("noalloc", [False, True])
def test_hybrid_scores_single_token_is_nan(noalloc):
    """One packed token: torch's unbiased std of one element is NaN and
    clamp(min=1e-6) keeps it, so the reference's z-scores and scores are NaN
    (landmark_tokens_ker.py:47-55) and its top-k leaves every slot at -1."""
    from dsalt.kernels import _ext
    from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
    from dsalt.kernels.selectors import select_topk
    dev = torch.device("cuda")
    g = torch.Generator().manual_seed(1)
    H, dh, dm = 4, 16, 64
    x = torch.randn(1, dm, generator=g)
    W = torch.randn(H * dh, dm, generator=g) * 0.2
    a = torch.rand(H, generator=g)
    ref, _, _ = O.hybrid_scores(x.numpy(), W.numpy(), a.numpy(), H, dh)
    assert np.isnan(ref).all()
    if noalloc:
        xd, Wd, ad = x.to(dev), W.to(dev), a.to(dev)
        xwv = xd @ Wd.T
        s = torch.empty(1, H, device=dev)
        p = _ext.ScoreParams(x=_ext.ptr(xd), xwv=_ext.ptr(xwv), alpha=_ext.ptr(ad), scores=_ext.ptr(s),
                             z_x=0, z_v=0, norms=0, stats=0, T=1, d_model=dm, H=H, n_kv=H, dh=dh,
                             dtype=_ext.dtype_code(torch.float32))
        _ext.call("dsalt_hybrid_scores_noalloc", p)
    else:
        s, _, _ = hybrid_scores_per_head(x.to(dev), W.to(dev), a.to(dev), H, dh)
    torch.cuda.synchronize()
    assert torch.isnan(s).all()
    cu = torch.tensor([0, 1], dtype=torch.int32, device=dev)
    idx = select_topk(s, torch.ones(1, device=dev), cu, 4, 1)
    assert (idx == -1).all()
    ref_idx = O.landmark_indices(ref, np.ones(1, dtype=np.float32), np.array([0, 1]), 4)
    assert (ref_idx == -1).all()


@pytest.mark.parametrize("case", ["varlen", "uniform", "gqa"])
def test_hybrid_scores_match_reference(golden_selectors, case):
    from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
    g = golden_selectors[case]
    dev = torch.device("cuda")
    H = g["alpha"].shape[0]
    s, zx, zv = hybrid_scores_per_head(g["x"].to(dev), g["W_V"].to(dev), g["alpha"].to(dev), H, int(g["dh"]))
    torch.testing.assert_close(s.cpu(), g["scores"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(zx.cpu(), g["z_x"], rtol=1e-5, atol=1e-5)
    torch.testing.assert_close(zv.cpu(), g["z_v"], rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("shape", [(97, 32, 4, 2, 8), (4096, 256, 16, 16, 16), (2, 32, 4, 4, 8)])
def test_hybrid_scores_alpha_and_x_gradients(shape):
    """The analytic backward (dsalt_hybrid_scores_bwd + row scaling) matches autograd
    through the reference formula: GQA, an MHA shape with many tokens, two tokens."""
    from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
    torch.manual_seed(0)
    dev = torch.device("cuda")
    T, dm, H, n_kv, dh = shape
    x = torch.randn(T, dm, device=dev, dtype=torch.float64).float().requires_grad_(True)
    W = (torch.randn(n_kv * dh, dm, device=dev) * 0.3).requires_grad_(True)
    a = torch.rand(H, device=dev).requires_grad_(True)
    gs = torch.randn(T, H, device=dev)
    s, _, _ = hybrid_scores_per_head(x, W, a, H, dh)
    (s * gs).sum().backward()
    x2 = x.detach().clone().requires_grad_(True)
    W2 = W.detach().clone().requires_grad_(True)
    a2 = a.detach().clone().requires_grad_(True)
    xn = x2.norm(dim=-1)
    zx = (xn - xn.mean()) / xn.std().clamp(min=1e-6)
    xv = (x2 @ W2.T).view(T, n_kv, dh).norm(dim=-1)
    zv = ((xv - xv.mean(0, keepdim=True)) / xv.std(0, keepdim=True).clamp(min=1e-6)).repeat_interleave(H // n_kv, 1)
    s2 = a2 * zv + (1 - a2) * zx[:, None]
    (s2 * gs).sum().backward()
    torch.testing.assert_close(a.grad, a2.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(x.grad, x2.grad, rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(W.grad, W2.grad, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("case", ["varlen", "uniform", "gqa"])
def test_landmark_sets_match_reference(golden_selectors, case):
    from dsalt.kernels.selectors import _compute_landmark_indices
    g = golden_selectors[case]
    dev = torch.device("cuda")
    H = g["alpha"].shape[0]
    cu = g["cu"]
    idx, _, _ = _compute_landmark_indices(g["x"].to(dev), g["W_V"].to(dev), g["alpha"].to(dev),
                                          g["w_disc"].to(dev), cu.to(dev), int(g["k"]), 4,
                                          int(cu[-1]), cu.tolist(), head_dim=int(g["dh"]))
    idx = idx.cpu().numpy()
    ref = g["idx"].numpy()
    for h in range(ref.shape[0]):
        for b in range(ref.shape[1]):
            assert sorted(idx[h, b].tolist()) == sorted(ref[h, b].tolist()), (h, b)


@pytest.mark.parametrize("L,k", [(4096, 64), (32768, 256), (37, 64), (5000, 1)])
def test_topk_full_size_vs_oracle(L, k):
    """Bit-exact index sets at the BASELINE sizes (scores given), ties to the lower position."""
    from dsalt.kernels.selectors import select_topk
    g = torch.Generator().manual_seed(L + k)
    lens = [L, max(L // 3, 1)]
    T, H = sum(lens), 2
    scores = torch.randn(T, H, generator=g)
    scores[5, 0] = scores[6, 0] = scores[7, 0] = 3.5   # ties
    w = (32 + torch.rand(T, generator=g) * 480).floor()
    cu = torch.tensor([0, lens[0], T], dtype=torch.int32)
    idx = select_topk(scores.cuda(), w.cuda(), cu.cuda(), k, max(lens)).cpu().numpy()
    ref = O.landmark_indices(scores.numpy(), w.numpy(), cu.numpy(), k)
    assert np.array_equal(idx, ref)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_hybrid_scores_from_value_projection(dtype):
    """Scoring from the module's value projection (no bias: v = x·W_Vᵀ) gives the
    same scores and gradients as the scorer's own GEMM."""
    from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
    g = torch.Generator(device="cuda").manual_seed(3)
    T, d, H, n_kv, dh = 777, 256, 8, 4, 32
    x = torch.randn(T, d, generator=g, device="cuda").to(dtype).requires_grad_(True)
    W = (torch.randn(n_kv * dh, d, generator=g, device="cuda") / d ** 0.5).requires_grad_(True)
    alpha = torch.rand(H, generator=g, device="cuda").requires_grad_(True)
    with torch.autocast("cuda", dtype=torch.bfloat16, enabled=dtype == torch.bfloat16):
        s_ref, _, _ = hybrid_scores_per_head(x, W, alpha, H, dh)
        v = torch.nn.functional.linear(x, W)
        s_v, _, _ = hybrid_scores_per_head(x, W, alpha, H, dh, xwv=v)
    assert torch.equal(s_ref, s_v)
    go = torch.randn_like(s_ref)
    ga = torch.autograd.grad(s_ref, (x, W, alpha), go)
    gb = torch.autograd.grad(s_v, (x, W, alpha), go)
    for a, b in zip(ga, gb):
        torch.testing.assert_close(a.float(), b.float(), rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_win_gate_backward(dtype):
    """``window_continuous`` gradients (the rank-one CUDA backward): against the same
    formulas in fp64 (dl = g·span·σ(1−σ); dx = dl ⊗ w, one rounding; dW = Σ_t dl·x), and
    against autograd of the reference expression ``n_min + sigmoid(win_gate(x)) *
    (n_max - n_min)`` under autocast, which rounds dl and dW to the dtype on the way."""
    from dsalt.kernels.window_gate import window_continuous
    torch.manual_seed(3)
    lin = torch.nn.Linear(256, 1).cuda()
    x = torch.randn(1000, 256, device="cuda").to(dtype)
    gw = torch.randn(1000, device="cuda")
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=dtype):
        wa = window_continuous(xa, lin, 32, 512)
        wb = 32 + torch.sigmoid(lin(xb).squeeze(-1)) * (512 - 32)
    ga = torch.autograd.grad(wa, [xa, lin.weight, lin.bias], gw)
    gb = torch.autograd.grad(wb, [xb, lin.weight, lin.bias], gw)
    w16 = lin.weight.detach().reshape(-1).to(dtype).double()
    logit = x.double() @ w16 + lin.bias.detach().to(dtype).double()
    sg = torch.sigmoid(logit)
    dl = gw.to(dtype).double() * 480 * sg * (1 - sg)  # autograd rounds gw to the output's dtype
    exp = (dl[:, None] * w16[None, :], (dl[None, :] @ x.double()), dl.sum().reshape(1))
    for name, a, e in zip(("x", "weight", "bias"), ga, exp):
        torch.testing.assert_close(a.double(), e, rtol=1e-2, atol=1e-3 * e.abs().max().item())
    for name, a, b in zip(("x", "weight", "bias"), ga, gb):
        assert a.shape == b.shape and a.dtype == b.dtype, name
        torch.testing.assert_close(a.float(), b.float(), rtol=5e-2, atol=2e-2 * b.abs().max().item())
