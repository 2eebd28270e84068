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
