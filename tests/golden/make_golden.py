"""Generate the golden fixtures in this directory by running the REFERENCE's own code.

Run once, in a container where the reference checkout is importable::

    DSALT_REFERENCE=/path/to/dsalt-library python tests/golden/make_golden.py

The fixtures pin (1) the numpy oracle in ``oracle/`` and (2) the CUDA path, so
that neither is checked only against itself.  Sources of truth, all from the
reference project (paths relative to its root):

* selectors: ``dsalt/kernels/landmark_tokens_ker.py:19-61`` (hybrid score),
  ``dsalt/kernels/selectors.py:75-134`` (landmark top-k), the window gate of
  ``dsalt/modules/dsalt_attention.py:270-275`` (fp32 and bf16 autocast);
* training op, dense path: ``DSALTAttention._dense_logbias_from_kernel``
  (``dsalt_attention.py:520-563``) + ``F.scaled_dot_product_attention`` in fp32,
  differentiated by autograd, one call per sequence (the dense path only takes
  uniform lengths, ``:497-504``);
* training op, Triton path: ``dsalt_triton_train_attention``
  (``dsalt/kernels/dsalt_triton_train.py:770-782``) run by the Triton interpreter
  (``TRITON_INTERPRET=1``) in fp16, with its autotune pre-seeded;
* inference op, Triton path: ``dsalt_triton_attention``
  (``dsalt/kernels/dsalt_triton_attn.py:337-349``) under the interpreter in fp16;
* module / model: ``DSALTAttention`` train-mode dense path and a small
  ``DSALTLMHeadModel`` forward+loss+backward in fp32 on CPU, plus the config-1
  loss of BASELINE.json (seed 0).

Versions of the third-party arithmetic the reference depends on are recorded in
``meta.json`` (torch, triton, numpy).
"""

from __future__ import annotations

import json
import math
import os
import sys
from pathlib import Path

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
os.environ.setdefault("TRITON_INTERPRET", "1")
os.environ.setdefault("PYTHONDONTWRITEBYTECODE", "1")

REF = os.environ.get("DSALT_REFERENCE")
if not REF:
    raise SystemExit("set DSALT_REFERENCE to the reference checkout (see the module docstring)")
OUT = Path(__file__).resolve().parent
sys.path.insert(0, REF)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

torch.cuda.get_device_capability = lambda *a, **k: (10, 0)  # the interpreter has no device

from dsalt.kernels import selectors as ref_sel  # noqa: E402
from dsalt.kernels import autotune as ref_at  # noqa: E402
from dsalt.kernels import dsalt_triton_train as ref_train  # noqa: E402
from dsalt.kernels import dsalt_triton_attn as ref_attn  # noqa: E402
from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head  # noqa: E402
from dsalt.modules.dsalt_attention import DSALTAttention  # noqa: E402
from dsalt.model import DSALTConfig, DSALTLMHeadModel  # noqa: E402


def _seed_triton_cfg(head_dim: int) -> None:
    cfg = {"BLOCK_M": 32, "BLOCK_N": 32, "num_warps": 2, "num_stages": 2, "BLOCK_N_BWD": 32}
    ref_train._TRAIN_TUNED[(head_dim, 10, 0)] = dict(cfg)
    ref_at._TUNED_CONFIG[(head_dim, 10, 0)] = dict(cfg)


def _clear_ref_caches() -> None:
    # The reference keys these caches by (total, num_seqs[, block]) only, so a
    # batch with equal totals but different lengths would reuse stale maps.
    ref_sel._SEQ_META_CACHE.clear()
    ref_sel._SEQ_BLOCK_MAP_CACHE.clear()


def _cu(lens):
    return [0] + list(np.cumsum(lens).astype(int))


# --------------------------------------------------------------------------- #
def make_selectors():
    g = torch.Generator().manual_seed(11)
    out = {}
    for name, lens, H, n_kv in (("varlen", [60, 100, 140], 4, 4),
                                ("uniform", [128, 128], 4, 4),
                                ("gqa", [90, 70], 4, 2)):
        _clear_ref_caches()
        d_model, dh, k = 64, 16, 8
        T = sum(lens)
        x = torch.randn(T, d_model, generator=g)
        W_V = torch.randn(n_kv * dh, d_model, generator=g) * 0.1
        alpha = torch.rand(H, generator=g)
        w_cont = 4 + torch.rand(T, generator=g) * 30
        w_disc = w_cont.floor().clamp(min=1)
        cu = torch.tensor(_cu(lens), dtype=torch.int32)
        scores, z_x, z_v = hybrid_scores_per_head(x, W_V, alpha, H, dh)
        idx, _, _ = ref_sel._compute_landmark_indices(x, W_V, alpha, w_disc, cu, k, 4, T,
                                                      _cu(lens), head_dim=dh)
        out[name] = dict(x=x, W_V=W_V, alpha=alpha, w_disc=w_disc, cu=cu, k=torch.tensor(k),
                         dh=torch.tensor(dh), scores=scores, z_x=z_x, z_v=z_v, idx=idx)
    torch.save(out, OUT / "selectors.pt")


def make_window():
    g = torch.Generator().manual_seed(12)
    n_min, n_max = 32, 512
    logits = torch.randn(4096, generator=g) * 2.0
    m = DSALTAttention(d_model=8, n_heads=1, n_min=n_min, n_max=n_max, k_lmk=4, max_seq_len=16)
    with torch.no_grad():
        m.win_gate.weight.zero_()
        m.win_gate.weight[0, 0] = 1.0
        m.win_gate.bias.zero_()
    x = torch.zeros(4096, 8)
    x[:, 0] = logits
    w32 = m._window_continuous(x).detach()
    with torch.autocast("cpu", dtype=torch.bfloat16):
        w16 = m._window_continuous(x).detach()
    torch.save(dict(logits=logits, n_min=torch.tensor(n_min), n_max=torch.tensor(n_max),
                    w_fp32=w32, w_bf16=w16.float(), w_bf16_dtype=str(w16.dtype)),
               OUT / "window.pt")


# --------------------------------------------------------------------------- #
def _op_inputs(lens, H, D, k, w_lo, w_hi, seed, n_empty_slots=1, int_windows=False):
    g = torch.Generator().manual_seed(seed)
    T = sum(lens)
    q = torch.randn(T, H, D, generator=g)
    kk = torch.randn(T, H, D, generator=g)
    v = torch.randn(T, H, D, generator=g)
    do = torch.randn(T, H, D, generator=g)
    w = w_lo + torch.rand(T, generator=g) * (w_hi - w_lo)
    if int_windows:
        w = w.floor()
    S = len(lens)
    pos = torch.full((H, S, k), -1, dtype=torch.long)
    for h in range(H):
        for b, L in enumerate(lens):
            n = max(0, min(k - n_empty_slots, L))
            if n:
                pos[h, b, :n] = torch.randperm(L, generator=g)[:n]
    s_sel = torch.randn(H, S, k, generator=g)
    logw = torch.log(torch.sigmoid(s_sel / 2.0).clamp(min=1e-20))
    logw = torch.where(pos >= 0, logw, torch.full_like(logw, float("-inf")))
    return dict(q=q, k=kk, v=v, do=do, w=w, pos=pos, logw=logw,
                cu=torch.tensor(_cu(lens), dtype=torch.int32))


def _compact(inp):
    """Store the fp16-exact activations as fp16 to keep the fixture small."""
    return {kk: (vv.half() if kk in ("q", "k", "v", "do") else vv) for kk, vv in inp.items()}


def _dense_train_reference(inp, H, D, tau_win=1.0, win_edge=4.0):
    """Reference dense path, fp32, one sequence at a time."""
    mod = DSALTAttention(d_model=H * D, n_heads=H, n_min=1, n_max=2, k_lmk=1, max_seq_len=8)
    mod.tau_win, mod.win_edge = tau_win, win_edge
    q = inp["q"].clone().requires_grad_(True)
    k = inp["k"].clone().requires_grad_(True)
    v = inp["v"].clone().requires_grad_(True)
    w = inp["w"].clone().requires_grad_(True)
    logw = inp["logw"].clone().requires_grad_(True)
    cu = inp["cu"].tolist()
    outs = []
    for b in range(len(cu) - 1):
        s0, s1 = cu[b], cu[b + 1]
        L = s1 - s0
        if L == 0:
            continue
        lb = mod._dense_logbias_from_kernel(w[s0:s1], inp["pos"][:, b:b + 1], logw[:, b:b + 1],
                                            1, L, torch.device("cpu"))
        qb = q[s0:s1].transpose(0, 1).unsqueeze(0)
        kb = k[s0:s1].transpose(0, 1).unsqueeze(0)
        vb = v[s0:s1].transpose(0, 1).unsqueeze(0)
        ob = F.scaled_dot_product_attention(qb, kb, vb, attn_mask=lb)
        outs.append((s0, s1, ob[0].transpose(0, 1)))
    o = torch.zeros_like(inp["q"])
    o_parts = []
    for s0, s1, ob in outs:
        o_parts.append(ob)
    o = torch.cat(o_parts, 0) if o_parts else o
    o.backward(inp["do"])
    return dict(o=o.detach(), dq=q.grad, dk=k.grad, dv=v.grad, d_w=w.grad, d_logw=logw.grad)


def _triton_train_reference(inp, H, D, n_max, tau_win=1.0, win_edge=4.0):
    _seed_triton_cfg(D)
    _clear_ref_caches()
    q = inp["q"].half().requires_grad_(True)
    k = inp["k"].half().requires_grad_(True)
    v = inp["v"].half().requires_grad_(True)
    w = inp["w"].clone().requires_grad_(True)
    logw = inp["logw"].clone().requires_grad_(True)
    cu = inp["cu"]
    o = ref_train.dsalt_triton_train_attention(q, k, v, inp["pos"], logw, w, cu, tau_win, win_edge,
                                               n_max, cu.tolist())
    o.backward(inp["do"])
    return dict(o=o.detach(), dq=q.grad.float(), dk=k.grad.float(), dv=v.grad.float(),
                d_w=w.grad.float(), d_logw=logw.grad.float())


def _triton_infer_reference(inp, H, D, w_int, bias):
    _seed_triton_cfg(D)
    _clear_ref_caches()
    q = inp["q"].half().requires_grad_(True)
    k = inp["k"].half().requires_grad_(True)
    v = inp["v"].half().requires_grad_(True)
    b = bias.clone().requires_grad_(True)
    o = ref_attn.dsalt_triton_attention(q, k, v, inp["pos"], b, w_int, inp["cu"])
    o.backward(inp["do"])
    return dict(o=o.detach(), dq=q.grad.float(), dk=k.grad.float(), dv=v.grad.float(),
                d_bias=b.grad.float())


def make_ops():
    cases = {
        # name: (lens, H, D, k, w_lo, w_hi, n_max, seed, int_windows)
        "train_small": ([48, 80], 2, 64, 8, 2.0, 40.0, 40, 21, False),
        "train_d128": ([100, 28], 1, 128, 16, 6.0, 100.0, 100, 22, False),
        "train_ragged": ([0, 37, 1, 90], 2, 64, 4, 0.5, 30.0, 30, 23, False),
        "train_intw": ([130], 1, 64, 8, 3.0, 60.0, 60, 24, True),
    }
    out = {}
    for name, (lens, H, D, k, wlo, whi, n_max, seed, intw) in cases.items():
        inp = _op_inputs(lens, H, D, k, wlo, whi, seed, int_windows=intw)
        # Inputs rounded to fp16 so that the fp32 dense reference and the fp16 Triton
        # reference see identical values (fp16 values are exact in fp32).
        for key in ("q", "k", "v", "do"):
            inp[key] = inp[key].half().float()
        dense = _dense_train_reference(inp, H, D)
        trit = _triton_train_reference(inp, H, D, n_max)
        out[name] = dict(inputs=_compact(inp), n_max=torch.tensor(n_max), dense=dense,
                         triton={kk: vv.half() for kk, vv in trit.items()})
    # inference semantics
    lens, H, D, k = [100, 60], 2, 64, 8
    inp = _op_inputs(lens, H, D, k, 1.0, 30.0, 31)
    for key in ("q", "k", "v", "do"):
        inp[key] = inp[key].half().float()
    w_int = inp["w"].floor().clamp(min=1)
    bias = torch.randn(H, len(lens), k, generator=torch.Generator().manual_seed(32)) * 0.5
    inp["w"] = w_int
    inp["bias"] = bias
    trit = _triton_infer_reference(inp, H, D, w_int, bias)
    out["infer_small"] = dict(inputs=_compact(inp), triton={kk: vv.half() for kk, vv in trit.items()})
    torch.save(out, OUT / "ops.pt")


# --------------------------------------------------------------------------- #
def make_module():
    torch.manual_seed(5)
    _clear_ref_caches()
    mod = DSALTAttention(d_model=64, n_heads=4, n_min=4, n_max=24, k_lmk=4, max_seq_len=256)
    with torch.no_grad():
        mod.alpha_w.copy_(torch.randn(4) * 0.5)
        mod.win_gate.weight.mul_(4.0)
    mod.train()
    lens = [64, 64]
    T = sum(lens)
    x = torch.randn(T, 64).requires_grad_(True)
    cu = torch.tensor(_cu(lens), dtype=torch.int32)
    out, _ = mod(x, cu_seqlens=cu, max_seqlen=64, cu_list=_cu(lens))
    g = torch.randn_like(out)
    out.backward(g)
    grads = {n: p.grad.clone() for n, p in mod.named_parameters()}
    torch.save(dict(state=mod.state_dict(), cfg=dict(d_model=64, n_heads=4, n_min=4, n_max=24,
                                                     k_lmk=4, max_seq_len=256),
                    x=x.detach(), cu=cu, out=out.detach(), g=g, grads=grads, x_grad=x.grad),
               OUT / "module.pt")


def make_model_small():
    torch.manual_seed(7)
    _clear_ref_caches()
    cfg = DSALTConfig(vocab_size=97, d_model=64, n_layers=2, n_heads=4, n_min=4, n_max=24,
                      k_lmk=4, max_seq_len=128, d_ff=64)
    model = DSALTLMHeadModel.from_config(cfg)
    model.train()
    lens = [64, 48, 16]
    T = sum(lens)
    ids = torch.randint(0, 97, (T,))
    labels = torch.randint(0, 97, (T,))
    cu = torch.tensor(_cu(lens), dtype=torch.int32)
    # The dense fallback needs uniform lengths; run one sequence per forward.
    res = model(ids[:64], cu_seqlens=torch.tensor([0, 64], dtype=torch.int32), labels=labels[:64])
    res["loss"].backward()
    grads = {n: p.grad.clone() for n, p in model.named_parameters() if p.grad is not None}
    torch.save(dict(cfg=cfg.to_dict(), state=model.state_dict(), ids=ids[:64], labels=labels[:64],
                    loss=res["loss"].detach(), grads=grads), OUT / "model_small.pt")


def make_config1_pin():
    """CPU SDPA-fallback forward+loss, seed 0, packed [2048]."""
    torch.manual_seed(0)
    _clear_ref_caches()
    cfg = DSALTConfig(vocab_size=50257, d_model=512, n_layers=6, n_heads=8, n_min=64,
                      n_max=256, k_lmk=16, max_seq_len=1024)
    model = DSALTLMHeadModel.from_config(cfg)
    model.train()
    ids = torch.randint(0, 50257, (2, 1024))
    labels = torch.randint(0, 50257, (2, 1024))
    cu = torch.tensor([0, 1024, 2048], dtype=torch.int32)
    with torch.no_grad():
        res = model(ids.reshape(-1), cu_seqlens=cu, labels=labels.reshape(-1))
    torch.save(dict(cfg=cfg.to_dict(), ids=ids, labels=labels, loss=res["loss"]),
               OUT / "config1_pin.pt")
    return float(res["loss"])


def main():
    torch.set_num_threads(os.cpu_count() or 1)
    make_selectors()
    make_window()
    make_ops()
    make_module()
    make_model_small()
    l1 = make_config1_pin() if os.environ.get("GOLDEN_SKIP_CONFIG1") != "1" else None
    import triton
    meta = dict(torch=torch.__version__, triton=triton.__version__, numpy=np.__version__,
                reference="LeonardoCofone/dsalt-library v1.0.0", config1_loss=l1)
    (OUT / "meta.json").write_text(json.dumps(meta, indent=2))
    print(json.dumps(meta))


if __name__ == "__main__":
    main()
