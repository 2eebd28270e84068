"""GPU checks of what the backward hands to autograd for the landmark weights and
the window: fp32 tensors holding the input-dtype-rounded values (the reference's
``.to(out_dtype)`` casts, dsalt_triton_train.py:750-757 and
dsalt_triton_attn.py:325-328), every landmark slot written (0 for an empty one),
the unrounded fp32 d_bias of ``dsalt_triton_backward`` (dsalt_triton_bwd.py),
and the batch's widest band that the schedule kernels write for the host.
"""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest
import torch

from test_ops_gpu import make_inputs, oracle_train, _close

pytestmark = pytest.mark.gpu


def _rounded(x: torch.Tensor, dtype) -> bool:
    return bool(torch.equal(x, x.to(dtype).float()))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_train_grads_of_fp32_params_hold_rounded_values(dtype):
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    inp = make_inputs([300, 0, 190], 2, 128, 16, 8.0, 120.0, seed=41, empty_slots=3)
    dev = torch.device("cuda")
    q, k, v = (inp[n].to(dev, dtype).requires_grad_(True) for n in ("q", "k", "v"))
    w = inp["w"].to(dev).float().requires_grad_(True)
    lw = inp["logw"].to(dev).float().requires_grad_(True)
    o = dsalt_triton_train_attention(q, k, v, inp["pos"].to(dev), lw, w, inp["cu"].to(dev), 1.0, 4.0, 256)
    o.backward(inp["do"].to(dev))
    assert lw.grad.dtype == torch.float32 and w.grad.dtype == torch.float32
    assert _rounded(lw.grad, dtype) and _rounded(w.grad, dtype)
    # empty slots (the last three of every row, and every slot of the empty sequence)
    empty = inp["pos"].to(dev) < 0
    assert empty.any() and torch.equal(lw.grad[empty], torch.zeros_like(lw.grad[empty]))
    ref = oracle_train(inp, dtype)
    _close(lw.grad.cpu().numpy(), ref["d_logw"], dtype, "d_logw")
    _close(w.grad.cpu().numpy(), ref["d_w"], dtype, "d_w")


def test_infer_autograd_rounds_and_backward_api_does_not():
    """DSALTAttentionFunction returns d_bias.to(out_dtype) (held in fp32);
    dsalt_triton_backward returns the fp32 sums themselves."""
    from dsalt.kernels import _ext
    from dsalt.kernels import dsalt_cuda as C
    from dsalt.kernels.dsalt_triton_attn import dsalt_triton_attention
    from dsalt.kernels.dsalt_triton_bwd import dsalt_triton_backward
    inp = make_inputs([700, 333], 2, 128, 64, 16.0, 200.0, seed=43)
    dev = torch.device("cuda")
    q, k, v = (inp[n].to(dev, torch.bfloat16) for n in ("q", "k", "v"))
    pos, cu = inp["pos"].to(dev), inp["cu"].to(dev)
    w = inp["w"].to(dev).floor().clamp(min=1)
    bias = torch.randn(inp["pos"].shape, generator=torch.Generator().manual_seed(3)).to(dev)
    bias_p = bias.clone().requires_grad_(True)
    qa = q.clone().requires_grad_(True)
    o = dsalt_triton_attention(qa, k, v, pos, bias_p, w, cu)
    do = inp["do"].to(dev)
    o.backward(do)
    d_auto = bias_p.grad
    assert d_auto.dtype == torch.float32 and _rounded(d_auto, torch.bfloat16)

    prep = C.prepare(k, v, pos, bias, w, cu, _ext.INFER, for_backward=True)
    o_in, _, lse = C.forward(q, k, v, prep, 1.0, 0.0, _ext.default_impl(), f32_out=False)
    dq, dk, dv, d_bias = dsalt_triton_backward(do, q, k, v, o_in, lse, None, None, pos, bias, w, cu,
                                               1.0 / math.sqrt(q.shape[-1]))
    torch.cuda.synchronize()
    assert d_bias.dtype == torch.float32
    assert not _rounded(d_bias, torch.bfloat16)  # 252 fp32 sums: not all of them bf16 values
    assert torch.allclose(d_bias.to(torch.bfloat16).float(), d_auto, rtol=2 ** -7, atol=1e-6)
    ref = oracle_train(dict(inp, bias=bias.cpu(), w=w.cpu()), torch.bfloat16, semantics="infer")
    _close(d_bias.cpu().numpy(), ref["d_logw"], torch.bfloat16, "d_bias")


def test_schedule_batch_widest_band():
    """seq_wmax_batch = max over s of seq_wmax[s], also after a wider batch used
    the same memory (the schedule kernels clear both)."""
    from dsalt.kernels import _ext
    from dsalt.kernels import dsalt_cuda as C
    dev = torch.device("cuda")
    for lens, lo, hi, seed in (([900, 40, 0, 513], 50.0, 700.0, 1), ([64, 300, 5], 1.0, 30.0, 2),
                               ([4096], 100.0, 2000.0, 3), ([128, 128], 1.0, 2.0, 4)):
        inp = make_inputs(lens, 1, 64, 8, lo, hi, seed=seed)
        k = inp["k"].to(dev, torch.bfloat16)
        prep = C.prepare(k, k, inp["pos"].to(dev), inp["logw"].to(dev), inp["w"].to(dev), inp["cu"].to(dev),
                         _ext.TRAIN, for_backward=True)
        torch.cuda.synchronize()
        assert int(prep.seq_wmax_batch.item()) == int(prep.seq_wmax.max().item())
        # the per-sequence maxima themselves, from the window rule on the host
        wf = inp["w"].numpy().astype(np.float32)
        cu = inp["cu"].numpy()
        for s in range(len(lens)):
            i = np.arange(lens[s])
            want = int(np.maximum(np.minimum(np.floor(wf[cu[s]:cu[s + 1]]), i), 0).max(initial=0))
            assert int(prep.seq_wmax[s].item()) == want, (lens, s)
        del prep


def test_dkdv_stage_zeroes_d_lw_of_an_empty_batch():
    """No tokens (every sequence empty): the dK/dV stage still writes d_lw = 0."""
    from dsalt.kernels import _ext
    from dsalt.kernels.dsalt_cuda import padded_landmarks
    lib = _ext.load()
    H, S, k_lmk = 2, 3, 5
    d_lw = torch.full((H, S, k_lmk), float("nan"), device="cuda")
    cu = torch.zeros(S + 1, dtype=torch.int32, device="cuda")
    p = _ext.AttnParams(cu_seqlens=_ext.ptr(cu), d_lw=_ext.ptr(d_lw), T=0, H=H, D=64, S=S, k_lmk=k_lmk,
                        kp=padded_landmarks(k_lmk),
                        scale=0.125, tau_win=1.0, win_edge=4.0, semantics=_ext.TRAIN, dtype=_ext.BF16,
                        impl=0, grad_round=1)
    assert lib.dsalt_attn_bwd_dkdv(ctypes.byref(p), None) == 0
    torch.cuda.synchronize()
    assert torch.equal(d_lw, torch.zeros_like(d_lw))
