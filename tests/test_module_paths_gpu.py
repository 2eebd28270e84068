"""The module-level shortcuts give the reference module's results bit for bit.

Under bf16 autocast DSALTAttention asks the op for O in bf16 (the values of the
reference's fp32 output, which out_proj casts back at once) instead of fp32:
outputs and every gradient must be identical to the fp32-output path.
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _run(m, x, cu, native: bool):
    saved = m._op_out_dtype
    if not native:
        m._op_out_dtype = lambda q: None
    try:
        m.zero_grad(set_to_none=True)
        xx = x.clone().requires_grad_(True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out, aux = m(xx, cu_seqlens=cu, max_seqlen=int((cu[1:] - cu[:-1]).max()))
        out.float().square().mean().backward()
        grads = {n: p.grad.clone() for n, p in m.named_parameters() if p.grad is not None}
        return out.detach().clone(), xx.grad.clone(), grads
    finally:
        m._op_out_dtype = saved


def test_bf16_output_path_matches_fp32_output_path():
    from dsalt.modules.dsalt_attention import DSALTAttention
    torch.manual_seed(0)
    m = DSALTAttention(d_model=512, n_heads=8, n_min=16, n_max=128, k_lmk=16, max_seq_len=1024).cuda()
    m.train()
    x = torch.randn(900, 512, device="cuda")
    cu = torch.tensor([0, 500, 900], dtype=torch.int32, device="cuda")
    a = _run(m, x, cu, native=True)
    b = _run(m, x, cu, native=False)
    assert m._op_out_dtype(torch.empty(1, dtype=torch.bfloat16, device="cuda")) is None  # outside autocast
    assert torch.equal(a[0], b[0])
    assert torch.equal(a[1], b[1])
    assert a[2].keys() == b[2].keys()
    for n in a[2]:
        assert torch.equal(a[2][n], b[2][n]), n
