"""GPU parity of the fused attention prologue (RoPE on q/k + GQA expansion of k/v).

The reference is the torch expression the reference module evaluates
(``apply_rotary_emb`` then ``_repeat_kv``, dsalt/kernels/window_utils.py:73-88 and
dsalt/modules/dsalt_attention.py:254-268), run in the same dtype: the forward must
be bitwise equal, the backward equal to autograd of that expression.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(q, k, v, cos, sin, n_rep):
    from dsalt.kernels.window_utils import apply_rotary_emb
    qr, kr = apply_rotary_emb(q, k, cos.unsqueeze(1), sin.unsqueeze(1))
    if n_rep > 1:
        T, Hkv, D = kr.shape
        kr = kr.unsqueeze(2).expand(T, Hkv, n_rep, D).reshape(T, Hkv * n_rep, D)
        v = v.unsqueeze(2).expand(T, Hkv, n_rep, D).reshape(T, Hkv * n_rep, D)
    return qr, kr, v


def _inputs(T, H, Hkv, D, dtype, seed):
    from dsalt.kernels.window_utils import build_rope_cache
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(T, H, D, generator=g, device="cuda").to(dtype)
    k = torch.randn(T, Hkv, D, generator=g, device="cuda").to(dtype)
    v = torch.randn(T, Hkv, D, generator=g, device="cuda").to(dtype)
    cos, sin = build_rope_cache(4096, D, torch.device("cuda"))
    pos = torch.randint(0, 4096, (T,), generator=g, device="cuda")
    return q, k, v, cos[pos].to(dtype), sin[pos].to(dtype)


CASES = [(257, 8, 8, 64), (300, 8, 2, 128), (129, 4, 1, 64), (64, 16, 4, 256)]


@pytest.mark.parametrize("shape", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
def test_forward_bitwise(shape, dtype):
    from dsalt.kernels.rope_gqa import rope_gqa
    T, H, Hkv, D = shape
    q, k, v, cos, sin = _inputs(T, H, Hkv, D, dtype, seed=T + H)
    got = rope_gqa(q, k, v, cos, sin)
    ref = _reference(q, k, v, cos, sin, H // Hkv)
    for name, a, b in zip(("q", "k", "v"), got, ref):
        assert a.shape == b.shape, name
        assert torch.equal(a, b), f"{name}: max |diff| {(a.float() - b.float()).abs().max().item():.3e}"


@pytest.mark.parametrize("shape", CASES)
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_backward_matches_autograd(shape, dtype):
    from dsalt.kernels.rope_gqa import rope_gqa
    T, H, Hkv, D = shape
    q, k, v, cos, sin = _inputs(T, H, Hkv, D, dtype, seed=7 * T + H)
    g = torch.Generator(device="cuda").manual_seed(3)
    grads = [torch.randn(T, H, D, generator=g, device="cuda").to(dtype) for _ in range(3)]
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    torch.autograd.backward(rope_gqa(*leaves, cos, sin), grads)
    ref_leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    torch.autograd.backward(_reference(*ref_leaves, cos, sin, H // Hkv), grads)
    for name, a, b in zip(("dq", "dk", "dv"), leaves, ref_leaves):
        ga, gb = a.grad.float(), b.grad.float()
        if dtype == torch.float32:
            torch.testing.assert_close(ga, gb, rtol=1e-6, atol=1e-6, msg=name)
        elif H // Hkv <= 2:
            # the reference's rounding order is reproduced: bitwise equal
            assert torch.equal(a.grad, b.grad), f"{name}: max |diff| {(ga - gb).abs().max().item():.3e}"
        else:
            # the sum over more than two copies may round in another order: one ulp
            torch.testing.assert_close(ga, gb, rtol=8e-3, atol=1e-2, msg=name)


@pytest.mark.parametrize("shape", [(300, 8, 2, 128), (129, 4, 1, 64)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_unexpanded_kv_heads(shape, dtype):
    """``expand=False`` (the attention op reads the kv heads in place): k rotated per kv
    head, v passed through; bitwise equal forward, the backward of the same
    expression (no sum over copies)."""
    from dsalt.kernels.rope_gqa import rope_gqa
    T, H, Hkv, D = shape
    q, k, v, cos, sin = _inputs(T, H, Hkv, D, dtype, seed=5 * T + H)
    got = rope_gqa(q, k, v, cos, sin, expand=False)
    ref = _reference(q, k, v, cos, sin, 1)
    for name, a, b in zip(("q", "k", "v"), got, ref):
        assert a.shape == b.shape, name
        assert torch.equal(a, b), name
    g = torch.Generator(device="cuda").manual_seed(4)
    grads = [torch.randn(t.shape, generator=g, device="cuda").to(dtype) for t in ref]
    leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    torch.autograd.backward(rope_gqa(*leaves, cos, sin, expand=False), grads)
    ref_leaves = [t.clone().requires_grad_(True) for t in (q, k, v)]
    torch.autograd.backward(_reference(*ref_leaves, cos, sin, 1), grads)
    for name, a, b in zip(("dq", "dk", "dv"), leaves, ref_leaves):
        if dtype == torch.float32:
            torch.testing.assert_close(a.grad, b.grad, rtol=1e-6, atol=1e-6, msg=name)
        else:
            assert torch.equal(a.grad, b.grad), name


def test_module_uses_fused_prologue_with_gqa():
    """A GQA DSALTAttention forward+backward runs through the fused prologue."""
    from dsalt.modules.dsalt_attention import DSALTAttention
    torch.manual_seed(0)
    m = DSALTAttention(d_model=256, n_heads=8, n_kv_heads=2, n_min=8, n_max=64, k_lmk=8,
                       max_seq_len=512).cuda()
    x = torch.randn(384, 256, device="cuda", requires_grad=True)
    cu = torch.tensor([0, 200, 384], dtype=torch.int32, device="cuda")
    out, aux = m(x, cu_seqlens=cu, max_seqlen=200)
    (out.float().square().mean() + aux.float()).backward()
    assert torch.isfinite(out).all() and torch.isfinite(x.grad).all()
    assert m.k_proj.weight.grad is not None and torch.isfinite(m.k_proj.weight.grad).all()


@pytest.mark.parametrize("heads", [(8, 8), (8, 2)])
def test_qkv_rope_matches_separate_projections(heads):
    """The stacked q|k|v GEMM feeding the strided prologue against the three
    projections + ``rope_gqa`` under bf16 autocast: outputs, the value projection
    for the scorer, and the gradients of x and the three weights."""
    from dsalt.kernels.rope_gqa import qkv_rope, rope_gqa
    from dsalt.kernels.window_utils import build_rope_cache
    H, Hkv = heads
    D, d, T = 64, 256, 300
    torch.manual_seed(H + Hkv)
    lin = [torch.nn.Linear(d, n * D, bias=False).cuda() for n in (H, Hkv, Hkv)]
    x = torch.randn(T, d, device="cuda")
    cos, sin = build_rope_cache(512, D, torch.device("cuda"))
    pos = torch.randint(0, 512, (T,), device="cuda")
    cos, sin = cos[pos], sin[pos]
    grads = [torch.randn(T, H, D, device="cuda").to(torch.bfloat16) for _ in range(3)]
    g_xwv = torch.randn(T, Hkv * D, device="cuda").to(torch.bfloat16)
    res = []
    for fused in (True, False):
        xa = x.clone().requires_grad_(True)
        for m in lin:
            m.weight.grad = None
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                q, k, v, xwv = qkv_rope(xa, *(m.weight for m in lin), cos, sin, H, Hkv, D, torch.bfloat16)
            else:
                q0, k0, v0 = (m(xa).view(T, -1, D) for m in lin)
                xwv = v0.view(T, Hkv * D)
                q, k, v = rope_gqa(q0, k0, v0, cos.to(torch.bfloat16), sin.to(torch.bfloat16))
        torch.autograd.backward([q, k, v, xwv], grads + [g_xwv])
        res.append(([t.detach().float() for t in (q, k, v, xwv)], [xa.grad] + [m.weight.grad for m in lin]))
    (fa, ga), (fb, gb) = res
    for a, b in zip(fa, fb):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-2)
    for a, b in zip(ga, gb):
        assert a.dtype == b.dtype
        torch.testing.assert_close(a, b, rtol=2e-2, atol=1e-2 * b.abs().max().item())
