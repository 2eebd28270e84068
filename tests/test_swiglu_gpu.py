"""GPU parity of the SwiGLU feed-forward path against the reference's torch ops.

The activation (``dsalt_swiglu_fwd``) must equal ``F.silu(g) * u`` on 16-bit tensors
bitwise; its backward must equal autograd of that expression (``du`` bitwise,
``dg`` within one rounding of the dtype, since torch's ``silu_backward`` may contract
its fp32 expression differently).  The fused block (one gate+up GEMM) is compared
with the reference block ``down(silu(gate(x)) * up(x))`` under autocast.
"""

from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(1, 8), (257, 2816), (64, 1032)])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_activation_forward_bitwise(shape, dtype):
    from dsalt.kernels.swiglu import swiglu
    g_ = torch.Generator(device="cuda").manual_seed(shape[0])
    g = (torch.randn(*shape, generator=g_, device="cuda") * 4).to(dtype)
    u = torch.randn(*shape, generator=g_, device="cuda").to(dtype)
    g[0, :4] = torch.tensor([0.0, -30.0, 30.0, -90.0], dtype=dtype)
    got = swiglu(g, u)
    ref = F.silu(g) * u
    assert torch.equal(got, ref), f"max |diff| {(got.float() - ref.float()).abs().max().item():.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_activation_backward(dtype):
    from dsalt.kernels.swiglu import _act_bwd
    T, Fd = 300, 1024
    g_ = torch.Generator(device="cuda").manual_seed(5)
    g = (torch.randn(T, Fd, generator=g_, device="cuda") * 3).to(dtype)
    u = torch.randn(T, Fd, generator=g_, device="cuda").to(dtype)
    dh = torch.randn(T, Fd, generator=g_, device="cuda").to(dtype)
    dgu = _act_bwd(torch.cat([g, u], dim=1), dh, Fd)
    gl, ul = g.clone().requires_grad_(True), u.clone().requires_grad_(True)
    (F.silu(gl) * ul).backward(dh)
    assert torch.equal(dgu[:, Fd:], ul.grad)
    torch.testing.assert_close(dgu[:, :Fd].float(), gl.grad.float(), rtol=1e-2, atol=1e-6)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_ffn_block_matches_reference_ops(dtype):
    from dsalt.modules.dsalt_transformer import SwiGLUFFN
    from dsalt.kernels.swiglu import swiglu_ffn
    torch.manual_seed(0)
    m = SwiGLUFFN(256, 768).cuda()
    for p in m.parameters():
        p.data.normal_(0, 0.05)
    x = torch.randn(2, 200, 256, device="cuda")
    xa, xb = x.clone().requires_grad_(True), x.clone().requires_grad_(True)
    with torch.autocast("cuda", dtype=dtype):
        ya = swiglu_ffn(xa, m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight, dtype)
        yb = m.down_proj(F.silu(m.gate_proj(xb)) * m.up_proj(xb))
    assert ya.dtype == yb.dtype == dtype and ya.shape == yb.shape
    torch.testing.assert_close(ya.float(), yb.float(), rtol=2e-2, atol=2e-3)
    gy = torch.randn_like(ya)
    ga = torch.autograd.grad(ya, [xa, m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight], gy)
    gb = torch.autograd.grad(yb, [xb, m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight], gy)
    for name, a, b in zip(("x", "gate", "up", "down"), ga, gb):
        assert a.dtype == b.dtype, name
        torch.testing.assert_close(a.float(), b.float(), rtol=3e-2, atol=3e-3 * b.abs().max().item(), msg=name)


def test_module_dispatch():
    """Under autocast the module output equals the fused function's; in fp32 the torch ops run."""
    from dsalt.modules.dsalt_transformer import SwiGLUFFN
    from dsalt.kernels.swiglu import swiglu_ffn
    torch.manual_seed(1)
    m = SwiGLUFFN(256, 768).cuda()
    x = torch.randn(100, 256, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        y = m(x)
        ref = swiglu_ffn(x, m.gate_proj.weight, m.up_proj.weight, m.down_proj.weight, torch.bfloat16)
    assert torch.equal(y, ref)
    y32 = m(x)
    assert y32.dtype == torch.float32
    torch.testing.assert_close(y32, m.down_proj(F.silu(m.gate_proj(x)) * m.up_proj(x)))
