"""Module / model level parity against the reference's own CPU path (fp32 goldens).

In fp32 the op runs the exact SIMT kernels, so the drop-in module and model
must match the reference's dense SDPA path at 1e-4.
"""

from __future__ import annotations

import pytest
import torch

from conftest import load_golden

pytestmark = pytest.mark.gpu


def test_attention_module_matches_reference():
    from dsalt.modules import DSALTAttention
    g = load_golden("module.pt")
    dev = torch.device("cuda")
    mod = DSALTAttention(**g["cfg"]).to(dev)
    missing, unexpected = mod.load_state_dict(g["state"], strict=True), None
    mod.train()
    x = g["x"].to(dev).requires_grad_(True)
    cu = g["cu"].to(dev)
    out, aux = mod(x, cu_seqlens=cu, max_seqlen=64, cu_list=g["cu"].tolist())
    out.backward(g["g"].to(dev))
    torch.testing.assert_close(out.detach().cpu(), g["out"], atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(x.grad.cpu(), g["x_grad"], atol=1e-4, rtol=1e-4)
    for name, p in mod.named_parameters():
        torch.testing.assert_close(p.grad.cpu(), g["grads"][name], atol=1e-4, rtol=1e-4, msg=name)


def test_small_model_loss_and_grads_match_reference():
    from dsalt.model import DSALTConfig, DSALTLMHeadModel
    g = load_golden("model_small.pt")
    dev = torch.device("cuda")
    model = DSALTLMHeadModel.from_config(DSALTConfig.from_dict(g["cfg"])).to(dev)
    model.load_state_dict(g["state"], strict=True)
    model.train()
    ids, labels = g["ids"].to(dev), g["labels"].to(dev)
    res = model(ids, cu_seqlens=torch.tensor([0, ids.shape[0]], dtype=torch.int32, device=dev), labels=labels)
    res["loss"].backward()
    torch.testing.assert_close(res["loss"].detach().cpu(), g["loss"], atol=1e-4, rtol=1e-4)
    for name, p in model.named_parameters():
        if name in g["grads"]:
            torch.testing.assert_close(p.grad.cpu(), g["grads"][name], atol=1e-4, rtol=1e-3, msg=name)


def test_config1_seeded_loss_matches_reference():
    """BASELINE config 1 (vocab 50257, 6 layers, fp32, seed 0): same weights from the
    same seeded construction, same packed ids, loss within 1e-4 of the reference CPU path."""
    from dsalt.model import DSALTConfig, DSALTLMHeadModel
    g = load_golden("config1_pin.pt")
    torch.manual_seed(0)
    model = DSALTLMHeadModel.from_config(DSALTConfig.from_dict(g["cfg"]))
    model = model.cuda().train()
    dev = torch.device("cuda")
    cu = torch.tensor([0, 1024, 2048], dtype=torch.int32, device=dev)
    with torch.no_grad():
        res = model(g["ids"].reshape(-1).to(dev), cu_seqlens=cu, labels=g["labels"].reshape(-1).to(dev))
    assert abs(float(res["loss"]) - float(g["loss"])) < 1e-4


def test_model_bf16_autocast_train_step_runs():
    """bf16 autocast fwd+bwd of a small model through the tensor-core kernels: finite loss and grads."""
    from dsalt.model import DSALTConfig, DSALTLMHeadModel
    torch.manual_seed(0)
    cfg = DSALTConfig(vocab_size=512, d_model=256, n_layers=2, n_heads=4, n_min=16, n_max=96, k_lmk=16,
                      max_seq_len=512)
    model = DSALTLMHeadModel.from_config(cfg).cuda().train()
    T = 3 * 300
    ids = torch.randint(0, 512, (T,), device="cuda")
    cu = torch.tensor([0, 300, 600, 900], dtype=torch.int32, device="cuda")
    with torch.autocast("cuda", dtype=torch.bfloat16):
        res = model(ids, cu_seqlens=cu, labels=ids)
    res["loss"].backward()
    assert torch.isfinite(res["loss"])
    for name, p in model.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), name
    assert model.layers[0].attn.alpha_w.grad.abs().sum() > 0
    assert model.layers[0].attn.win_gate.weight.grad.abs().sum() > 0


@pytest.mark.parametrize("autocast", [False, True])
def test_gradient_checkpointing_matches_plain_step(autocast):
    """The checkpointed block path (reference's torch.utils.checkpoint form, residual adds
    unfused) gives the loss and gradients of the plain path (fused residual adds)."""
    from dsalt.model import DSALTLMHeadModel
    torch.manual_seed(0)
    model = DSALTLMHeadModel(vocab_size=300, d_model=256, n_layers=2, n_heads=4, n_min=8, n_max=64, k_lmk=8,
                             max_seq_len=512).cuda().train()
    # non-uniform norm weights: with the initial all-ones weights every normed token has
    # the same ‖x‖ up to rounding, and the landmark score's 1/std(‖x‖) would turn
    # rounding-order differences of the two paths into large gradient differences
    with torch.no_grad():
        for n, p in model.named_parameters():
            if n.endswith("norm.weight"):
                p.normal_(1.0, 0.3)
    g = torch.Generator(device="cuda").manual_seed(1)
    ids = torch.randint(0, 300, (2 * 256 + 1,), generator=g, device="cuda")
    cu = torch.tensor([0, 256, 512], dtype=torch.int32, device="cuda")
    res = []
    for ckpt in (False, True):
        model.zero_grad(set_to_none=True)
        with torch.autocast("cuda", dtype=torch.bfloat16, enabled=autocast):
            out = model(ids[:-1], cu_seqlens=cu, max_seqlen=256, labels=ids[1:], gradient_checkpointing=ckpt)
        out["loss"].backward()
        res.append((out["loss"].detach().float(), {n: p.grad.detach().float().clone()
                                                   for n, p in model.named_parameters()}))
    (la, ga), (lb, gb) = res
    tol = 2e-2 if autocast else 1e-4
    torch.testing.assert_close(la, lb, rtol=tol, atol=tol)
    for n in ga:
        torch.testing.assert_close(ga[n], gb[n], rtol=5e-2 if autocast else 1e-3,
                                   atol=(5e-2 if autocast else 1e-4) * gb[n].abs().max().item() + 1e-8, msg=n)
