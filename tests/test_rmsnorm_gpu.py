"""GPU parity of the CUDA RMSNorm against F.rms_norm (the reference RMSENorm's op)."""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("d", [256, 512, 768, 1024])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_rmsnorm_matches_torch(d, dtype):
    from dsalt.kernels.rmsnorm_cuda import rms_norm
    g = torch.Generator(device="cuda").manual_seed(d)
    T = 1000  # not a multiple of the 64-row partials
    x = (torch.randn(T, d, generator=g, device="cuda") * 3).to(dtype)
    w = torch.randn(d, generator=g, device="cuda") * 0.5 + 1
    dy = torch.randn(T, d, generator=g, device="cuda").to(dtype)
    xa, wa = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    y = rms_norm(xa, wa, 1e-6)
    y.backward(dy)
    xb, wb = x.clone().float().requires_grad_(True), w.clone().requires_grad_(True)
    yb = F.rms_norm(xb, (d,), wb, 1e-6)
    yb.to(dtype).float().backward(dy.float())
    tol = dict(rtol=1e-2, atol=1e-2) if dtype != torch.float32 else dict(rtol=2e-5, atol=2e-5)
    assert y.dtype == dtype
    torch.testing.assert_close(y.float(), yb.detach().to(dtype).float(), **tol)
    torch.testing.assert_close(xa.grad.float(), xb.grad.to(dtype).float(), **tol)
    torch.testing.assert_close(wa.grad, wb.grad, rtol=2e-3 if dtype != torch.float32 else 2e-5,
                               atol=2e-2 if dtype != torch.float32 else 1e-4)


def test_rmsenorm_module_dispatch_and_determinism():
    from dsalt.kernels.RMSENorm import RMSENorm
    m = RMSENorm(512).cuda()
    x = torch.randn(777, 512, device="cuda", dtype=torch.bfloat16, requires_grad=True)
    outs = []
    for _ in range(2):
        m.zero_grad(set_to_none=True)
        x.grad = None
        y = m(x)
        y.float().square().sum().backward()
        outs.append((y.detach().clone(), x.grad.clone(), m.weight.grad.clone()))
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("d", [512, 1024])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_add_rmsnorm_matches_torch(d, dtype):
    """The residual add fused in front of the norm: x + res rounded like torch's add, the
    norm of that sum, and in the backward the residual gradient added to the norm's."""
    from dsalt.kernels.rmsnorm_cuda import add_rms_norm
    g = torch.Generator(device="cuda").manual_seed(d + 1)
    T = 1000
    x = (torch.randn(T, d, generator=g, device="cuda") * 2).to(dtype)
    res = torch.randn(T, d, generator=g, device="cuda").to(dtype)
    w = torch.randn(d, generator=g, device="cuda") * 0.5 + 1
    d_sum = torch.randn(T, d, generator=g, device="cuda").to(dtype)
    dy = torch.randn(T, d, generator=g, device="cuda").to(dtype)
    xa, ra, wa = (t.clone().requires_grad_(True) for t in (x, res, w))
    s_a, y_a = add_rms_norm(xa, ra, wa, 1e-6)
    torch.autograd.backward([s_a, y_a], [d_sum, dy])
    xb, rb, wb = (t.clone().requires_grad_(True) for t in (x, res, w))
    s_b = xb + rb
    y_b = F.rms_norm(s_b.float(), (d,), wb, 1e-6).to(dtype)
    torch.autograd.backward([s_b, y_b], [d_sum, dy])
    assert torch.equal(s_a, s_b)
    tol = dict(rtol=1e-2, atol=1e-2) if dtype != torch.float32 else dict(rtol=2e-5, atol=2e-5)
    torch.testing.assert_close(y_a.float(), y_b.float(), **tol)
    torch.testing.assert_close(xa.grad.float(), xb.grad.float(), **tol)
    assert torch.equal(xa.grad, ra.grad)
    torch.testing.assert_close(ra.grad.float(), rb.grad.float(), **tol)
    torch.testing.assert_close(wa.grad, wb.grad, rtol=2e-3 if dtype != torch.float32 else 2e-5,
                               atol=2e-2 if dtype != torch.float32 else 1e-4)


def test_block_fused_residual_matches_unfused():
    """A transformer block run with the residual adds fused into its norms gives the
    reference block's output and gradients (the unfused torch adds, same kernels otherwise)."""
    from dsalt.modules.dsalt_transformer import DSALTTransformerBlock
    torch.manual_seed(0)
    blk = DSALTTransformerBlock(d_model=256, n_heads=4, n_min=8, n_max=64, k_lmk=8, max_seq_len=512,
                                d_ff=768).cuda()
    x = torch.randn(384, 256, device="cuda")
    cu = torch.tensor([0, 200, 384], dtype=torch.int32, device="cuda")
    outs = []
    for fused in (True, False):
        xa = x.clone().requires_grad_(True)
        blk.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            if fused:
                y, aux, f = blk(xa.to(torch.bfloat16), cu_seqlens=cu, max_seqlen=200, cu_list=[0, 200, 384],
                                defer=True)
                y = y + f
            else:
                h = xa.to(torch.bfloat16)
                x_attn, aux = blk.attn(blk.attn_norm(h), cu_seqlens=cu, max_seqlen=200, cu_list=[0, 200, 384])
                h = h + x_attn
                y = h + blk.ffn(blk.ffn_norm(h))
        y.float().square().mean().backward()
        outs.append((y.detach().float(), xa.grad.clone(), blk.ffn_norm.weight.grad.clone()))
    (ya, ga, wa), (yb, gb, wb) = outs
    torch.testing.assert_close(ya, yb, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(ga, gb, rtol=2e-2, atol=2e-2 * gb.abs().max().item())
    torch.testing.assert_close(wa, wb, rtol=2e-2, atol=2e-2 * wb.abs().max().item())
