"""The reference's own Triton training op, run in a process of its own.

Test and measurement infrastructure, like the rest of ``oracle/``: only
``tests/`` and ``bench.py`` start it, as a checker (GPU parity against the
reference's kernels) and as the B200 speed bar (the reference's Triton path
after its one-shot autotune).  Nothing in the product imports it.

The reference is installed, unmodified, under ``baseline/_ref`` (``pip install
--target baseline/_ref`` of the reference project).  Its package is also named
``dsalt``, so it cannot share a process with this build's package: this script
runs with ``baseline/_ref`` alone on ``sys.path`` and exchanges tensors through
a ``torch.save`` file.

    python oracle/ref_triton.py train  IN.pt OUT.pt [--steps K --warmup W] [--tuned-cache F]
    python oracle/ref_triton.py select IN.pt OUT.pt

``train``: ``dsalt_triton_train_attention`` (dsalt/kernels/dsalt_triton_train.py:770-782)
forward + backward on the inputs, as ``bench.step_fn`` runs this build's op; the first
call runs the reference's autotune (:512-582) unless ``--tuned-cache`` holds the
configuration an earlier run on this machine picked.  Writes the outputs and
gradients, the autotuned configuration and the CUDA-event time per step.

``select``: the reference's selectors on given x / weights: ``hybrid_scores_per_head``
(dsalt/kernels/landmark_tokens_ker.py:19-61), ``_compute_landmark_indices``
(dsalt/kernels/selectors.py:75-134) and the window gate expression of
``DSALTAttention._window_continuous`` (dsalt/modules/dsalt_attention.py:270-284).
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
REF = ROOT / "baseline" / "_ref"


def available() -> str | None:
    """None when the reference install and Triton are present, else the reason."""
    if not (REF / "dsalt" / "kernels" / "dsalt_triton_train.py").exists():
        return "reference not installed under baseline/_ref"
    try:
        import triton  # noqa: F401
    except Exception as e:  # pragma: no cover - depends on the image
        return f"triton not importable: {e}"
    return None


def run(mode: str, inp: dict, timeout: int = 1500, **opts) -> dict:
    """Run this script in a child process on ``inp`` and return what it wrote."""
    import subprocess
    import tempfile

    import torch
    with tempfile.TemporaryDirectory() as tmp:
        fi, fo = Path(tmp) / "in.pt", Path(tmp) / "out.pt"
        torch.save({k: (v.detach().cpu() if torch.is_tensor(v) else v) for k, v in inp.items()}, fi)
        cmd = [sys.executable, str(Path(__file__).resolve()), mode, str(fi), str(fo)]
        for k, v in opts.items():
            if v is not None:
                cmd += [f"--{k.replace('_', '-')}", str(v)]
        env = dict(os.environ, TORCHDYNAMO_DISABLE="1", PYTHONPATH="")
        res = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
        if res.returncode != 0:
            raise RuntimeError(f"reference Triton run failed (rc {res.returncode}):\n"
                               f"{res.stdout[-2000:]}\n{res.stderr[-4000:]}")
        out = torch.load(fo, weights_only=False)
        out["log"] = res.stdout[-4000:]
        return out


# ----------------------------------------------------------------- child side
def _child_train(d: dict, steps: int, warmup: int, tuned_cache: str | None) -> dict:
    import torch
    from dsalt.kernels import dsalt_triton_train as RT
    dev = torch.device("cuda")
    t = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in d.items()}
    q, k, v = (t[n].requires_grad_(True) for n in ("q", "k", "v"))
    w = t["w"].float().requires_grad_(True)
    lw = t["lmk_logw"].float().requires_grad_(True)
    D = q.shape[2]
    major, minor = torch.cuda.get_device_capability(dev)
    key = (int(D), int(major), int(minor))
    cache = Path(tuned_cache) if tuned_cache else None
    if cache is not None and cache.exists():
        saved = json.loads(cache.read_text())
        if saved.get("key") == list(key):
            RT._TRAIN_TUNED[key] = saved["cfg"]

    def step():
        o = RT.dsalt_triton_train_attention(q, k, v, t["lmk_pos"], lw, w, t["cu"], 1.0, 4.0, int(t["n_max"]),
                                            t.get("cu_list"))
        return o, torch.autograd.grad(o, (q, k, v, w, lw), t["do"])

    o, grads = step()  # the first call autotunes (unless pre-seeded)
    torch.cuda.synchronize()
    cfg = RT._TRAIN_TUNED.get(key)
    if cache is not None and cfg is not None:
        cache.write_text(json.dumps({"key": list(key), "cfg": cfg}))
    out = {"o": o.detach().cpu(), "dq": grads[0].cpu(), "dk": grads[1].cpu(), "dv": grads[2].cpu(),
           "d_w": grads[3].cpu(), "d_logw": grads[4].cpu(), "cfg": cfg, "device": torch.cuda.get_device_name(dev)}
    del o, grads
    if steps > 0:
        for _ in range(max(warmup, 1)):
            step()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(steps):
            step()
        b.record()
        torch.cuda.synchronize()
        out["ms_per_step"] = a.elapsed_time(b) / steps
        out["steps"] = steps
    return out


def _child_select(d: dict) -> dict:
    import torch
    from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
    from dsalt.kernels.selectors import _compute_landmark_indices
    import dsalt.kernels.selectors as sel
    dev = torch.device("cuda")
    t = {k: (v.to(dev) if torch.is_tensor(v) else v) for k, v in d.items()}
    H, dh = int(t["H"]), int(t["dh"])
    x = t["x"]
    scores, z_x, z_v = hybrid_scores_per_head(x, t["W_V"], t["alpha"], H, dh)
    # the window gate, as DSALTAttention._window_continuous computes it
    logit = torch.nn.functional.linear(x, t["gate_w"], t["gate_b"]).squeeze(-1)
    w_cont = float(t["n_min"]) + torch.sigmoid(logit) * (float(t["n_max"]) - float(t["n_min"]))
    w_disc = w_cont.detach().float().floor().clamp(min=1)
    sel._SEQ_META_CACHE.clear()
    sel._SEQ_BLOCK_MAP_CACHE.clear()
    idx, _, _ = _compute_landmark_indices(x, t["W_V"], t["alpha"], w_disc, t["cu"], int(t["k"]), int(t["n_min"]),
                                          int(x.shape[0]), t.get("cu_list"), head_dim=dh)
    return {"scores": scores.cpu(), "z_x": z_x.cpu(), "z_v": z_v.cpu(), "w_cont": w_cont.detach().cpu(),
            "w_disc": w_disc.cpu(), "idx": idx.cpu()}


def _main(argv: list[str]) -> None:
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("mode", choices=["train", "select"])
    ap.add_argument("inp")
    ap.add_argument("out")
    ap.add_argument("--steps", type=int, default=0)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--tuned-cache", default=None)
    a = ap.parse_args(argv)
    # the reference alone: drop this build's package paths
    here = {str(ROOT), str(ROOT / "dsalt-library_b200"), str(Path(__file__).resolve().parent)}
    sys.path[:] = [p for p in sys.path if p not in here and p != ""]
    sys.path.insert(0, str(REF))
    import torch
    d = torch.load(a.inp, weights_only=False)
    out = _child_train(d, a.steps, a.warmup, a.tuned_cache) if a.mode == "train" else _child_select(d)
    torch.save(out, a.out)


if __name__ == "__main__":
    _main(sys.argv[1:])
