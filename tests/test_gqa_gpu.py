"""Grouped kv heads read in place (the reference's n_kv_heads, whose _repeat_kv
expands K/V ×n_rep before the op, dsalt/modules/dsalt_attention.py:254-268).

The op takes k, v with H_kv heads; every kernel reads kv head h / (H / H_kv), the
backward writes dK/dV per query head and dsalt_gqa_reduce sums each group.  The
references: the oracle on the expanded K/V with its dK/dV summed per group, and
this build's own op on explicitly expanded K/V (O and dQ bit-identical).
Tolerances as in test_ops_gpu (bf16 2e-2 / 1e-2, fp32 1e-4).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import dsalt_oracle as O
from test_ops_gpu import TOL, _close, make_inputs, run_train

pytestmark = pytest.mark.gpu

N_REP = 4


def _gqa_inputs(lens, H, D, k, wlo, whi, seed, semantics="train"):
    inp = make_inputs(lens, H, D, k, wlo, whi, seed)
    T = inp["k"].shape[0]
    inp["k"] = inp["k"][:, ::N_REP].contiguous()   # H / N_REP kv heads
    inp["v"] = inp["v"][:, ::N_REP].contiguous()
    if semantics == "infer":
        inp["bias"] = torch.randn(inp["pos"].shape, generator=torch.Generator().manual_seed(seed)) \
            .where(inp["pos"] >= 0, torch.tensor(0.0))
    assert inp["k"].shape == (T, H // N_REP, D)
    return inp


def _expand(t):
    return t.repeat_interleave(N_REP, dim=1)


def _oracle(inp, dtype, semantics="train"):
    def rd(t):
        return t.to(dtype).float().numpy()
    ref = O.attention_bwd(rd(inp["q"]), rd(_expand(inp["k"])), rd(_expand(inp["v"])), rd(inp["do"]),
                          inp["pos"].numpy(),
                          (inp["logw"] if semantics == "train" else inp["bias"]).float().numpy(),
                          inp["w"].float().numpy(), inp["cu"].numpy(), 1.0, 4.0, semantics)
    T, H, D = ref["dk"].shape
    for key in ("dk", "dv"):   # the autograd of the expansion: the sum over each group
        ref[key] = ref[key].reshape(T, H // N_REP, N_REP, D).sum(axis=2)
    return ref


CASES = {
    # name: (lens, H, D, k, w_lo, w_hi)
    "d128": ([700, 300], 8, 128, 64, 32.0, 300.0),
    "d64": ([129, 255, 1, 77], 8, 64, 16, 1.0, 90.0),
}


@pytest.mark.parametrize("case", list(CASES))
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_train_gqa_vs_oracle(case, dtype):
    lens, H, D, k, wlo, whi = CASES[case]
    inp = _gqa_inputs(lens, H, D, k, wlo, whi, seed=sum(map(ord, case)))
    res = run_train(inp, dtype)
    assert res["dk"].shape == tuple(inp["k"].shape) and res["dv"].shape == tuple(inp["v"].shape)
    ref = _oracle(inp, dtype)
    for key in ("o", "dq", "dk", "dv", "d_w", "d_logw"):
        _close(res[key], ref[key], dtype, key)


def test_infer_gqa_vs_oracle():
    lens, H, D, k, wlo, whi = CASES["d128"]
    inp = _gqa_inputs(lens, H, D, k, wlo, whi, seed=11, semantics="infer")
    res = run_train(inp, torch.bfloat16, semantics="infer")
    ref = _oracle(inp, torch.bfloat16, semantics="infer")
    for key in ("o", "dq", "dk", "dv", "d_logw"):
        _close(res[key], ref[key], torch.bfloat16, key)


def test_gqa_matches_expanded_kv():
    """In-place kv heads against the same op on K/V expanded ×n_rep: O and dQ bit for
    bit (the kernels see the same keys and values), dK/dV as the fp32 group sums of
    the expanded op's per-head gradients, rounded once."""
    lens, H, D, k, wlo, whi = CASES["d128"]
    inp = _gqa_inputs(lens, H, D, k, wlo, whi, seed=3)
    exp = dict(inp, k=_expand(inp["k"]), v=_expand(inp["v"]))
    a = run_train(inp, torch.bfloat16)
    b = run_train(exp, torch.bfloat16)
    for key in ("o", "dq", "d_w", "d_logw"):
        assert np.array_equal(a[key], b[key]), key
    T = b["dk"].shape[0]
    for key in ("dk", "dv"):
        want = torch.from_numpy(b[key]).view(T, H // N_REP, N_REP, D).sum(2).to(torch.bfloat16).float().numpy()
        assert np.max(np.abs(a[key] - want) / (np.abs(want) + 1e-3)) <= 2 ** -7, key


def test_gqa_reduce_entry_point():
    """dsalt_gqa_reduce alone: fp32 sums of each group, rounded once."""
    from dsalt.kernels.dsalt_cuda import gqa_reduce
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randn(333, 12, 64, generator=g, device="cuda").to(torch.bfloat16)
    y = gqa_reduce(x, 3)
    want = x.float().view(333, 3, 4, 64).sum(2).to(torch.bfloat16)
    assert torch.equal(y, want)


def test_module_gqa_matches_expanded_path():
    """DSALTAttention with n_kv_heads < n_heads: the in-place kv-head path against the
    same module with K/V expanded before the op (the reference's _repeat_kv)."""
    from dsalt.modules.dsalt_attention import DSALTAttention
    torch.manual_seed(0)
    m = DSALTAttention(d_model=512, n_heads=8, n_kv_heads=2, n_min=8, n_max=64, k_lmk=16,
                       max_seq_len=512).cuda().train()
    x = torch.randn(2, 200, 512, device="cuda")

    def run(expand):
        orig = m._project_qkv
        if expand:
            def proj(*args):
                q, k, v, xwv = orig(*args)
                return q, m._repeat_kv(k), m._repeat_kv(v), xwv
            m._project_qkv = proj
        try:
            m.zero_grad(set_to_none=True)
            xx = x.clone().requires_grad_(True)
            with torch.autocast("cuda", dtype=torch.bfloat16):
                out, _ = m(xx)
            out.float().square().mean().backward()
            return out.detach().float(), xx.grad.detach(), {n: p.grad.detach().clone() for n, p in m.named_parameters()
                                                           if p.grad is not None}
        finally:
            m._project_qkv = orig

    oa, xa, ga = run(False)
    ob, xb, gb = run(True)
    assert torch.equal(oa, ob)
    torch.testing.assert_close(xa, xb, rtol=2e-2, atol=2e-2 * xb.abs().max().item())
    assert ga.keys() == gb.keys()
    for n in ga:
        torch.testing.assert_close(ga[n], gb[n], rtol=2e-2, atol=2e-2 * gb[n].abs().max().item() + 1e-8, msg=n)
