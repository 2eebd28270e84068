"""GPU parity of the fused chunked cross-entropy against the reference's chunked loss."""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("vocab", [32000, 1003])  # 16-byte rows, and the scalar path
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_fused_ce_matches_chunked_torch(vocab, dtype):
    from dsalt.kernels.fused_ce import fused_chunked_cross_entropy
    from dsalt.model.dsalt_lm import _chunked_cross_entropy
    g = torch.Generator(device="cuda").manual_seed(vocab)
    N, d, chunk = 1500, 256, 512
    x = torch.randn(N, d, generator=g, device="cuda")
    w = torch.randn(vocab, d, generator=g, device="cuda") * 0.05
    labels = torch.randint(0, vocab, (N,), generator=g, device="cuda")
    labels[::7] = -100
    xa, wa = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=dtype):
        la = fused_chunked_cross_entropy(xa, wa, labels, chunk, dtype)
    la.backward()
    xb, wb = x.clone().requires_grad_(True), w.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=dtype):
        lb = _chunked_cross_entropy(xb, wb, labels, chunk)
    lb.backward()
    torch.testing.assert_close(la, lb, rtol=1e-4, atol=1e-4)
    # both paths round the logits gradient to the 16-bit dtype before the GEMMs and
    # accumulate in fp32 in different orders: 2 % of the element, or 0.5 % of the
    # largest gradient where the sum cancels to near zero
    for a, b in ((xa.grad, xb.grad), (wa.grad, wb.grad)):
        torch.testing.assert_close(a, b, rtol=2e-2, atol=5e-3 * b.abs().max().item())


def test_model_uses_fused_loss_under_autocast():
    from dsalt.model.dsalt_lm import DSALTLMHeadModel, _fused_ce_dtype
    x = torch.zeros(4, 8, device="cuda")
    w = torch.zeros(16, 8, device="cuda")
    assert _fused_ce_dtype(x, w) is None
    with torch.autocast("cuda", dtype=torch.bfloat16):
        assert _fused_ce_dtype(x, w) == torch.bfloat16
    assert _fused_ce_dtype(x.cpu(), w.cpu()) is None


def test_fused_ce_no_grad_loss_only():
    """Under no_grad (evaluation) only the loss is computed, and it equals the
    training path's loss bit for bit (same GEMM, same kernel, same sum)."""
    from dsalt.kernels.fused_ce import fused_chunked_cross_entropy
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn(700, 128, generator=g, device="cuda")
    w = torch.randn(5000, 128, generator=g, device="cuda") * 0.05
    labels = torch.randint(0, 5000, (700,), generator=g, device="cuda")
    labels[::5] = -100
    with torch.no_grad():
        l0 = fused_chunked_cross_entropy(x, w, labels, 256, torch.bfloat16)
    assert not l0.requires_grad
    l1 = fused_chunked_cross_entropy(x.requires_grad_(True), w, labels, 256, torch.bfloat16)
    assert torch.equal(l0, l1.detach())
