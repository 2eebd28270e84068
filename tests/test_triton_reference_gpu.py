"""GPU parity against the reference's own kernels, run on the same B200.

The reference (installed unmodified under ``baseline/_ref``) runs in a child
process (``oracle/ref_triton.py``): its Triton training op
``dsalt_triton_train_attention`` after its autotune, and its torch selectors.
Both sides get the same seeded inputs at the benchmarked size (config 2: 4 ×
4,096 tokens, H=16, D=128, k=64).  Outputs and gradients must agree within the
north_star tolerance for 16-bit inputs (max-abs 2e-2 + rel 1e-2); window sizes
and landmark index sets bit-exactly.  Skipped where the reference install or
Triton is absent.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

import bench
from oracle import ref_triton

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(ref_triton.available() is not None,
                                 reason=str(ref_triton.available()))]

ATOL, RTOL = 2e-2, 1e-2
TUNED = "/tmp/dsalt_ref_triton_tuned.json"


def _close(got, ref, what):
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (what, got.shape, ref.shape)
    bad = np.abs(got - ref) > ATOL + RTOL * np.abs(ref)
    assert not bad.any(), f"{what}: {int(bad.sum())} / {bad.size} outside tol, max abs err " \
                          f"{np.abs(got - ref).max():.3e}"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_op_matches_reference_triton_at_config2(dtype):
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    dev = torch.device("cuda")
    d = bench.make_workload(bench.WORKLOADS["config2"], seed=0, device=dev)
    for n in ("q", "k", "v"):
        d[n] = d[n].to(dtype)
    inp = {n: d[n] for n in ("q", "k", "v", "do", "w", "lmk_pos", "lmk_logw", "cu")}
    inp.update(cu_list=d["cu_list"], n_max=d["n_max"])
    ref = ref_triton.run("train", inp, tuned_cache=TUNED)
    q, k, v = (d[n].detach().clone().requires_grad_(True) for n in ("q", "k", "v"))
    w = d["w"].detach().clone().requires_grad_(True)
    lw = d["lmk_logw"].detach().clone().requires_grad_(True)
    o = dsalt_triton_train_attention(q, k, v, d["lmk_pos"], lw, w, d["cu"], 1.0, 4.0, d["n_max"], d["cu_list"])
    grads = torch.autograd.grad(o, (q, k, v, w, lw), d["do"])
    got = {"o": o, "dq": grads[0], "dk": grads[1], "dv": grads[2], "d_w": grads[3], "d_logw": grads[4]}
    for key, t in got.items():
        assert t.dtype == ref[key].dtype, (key, t.dtype, ref[key].dtype)
        _close(t.detach().float().cpu().numpy(), ref[key].float().numpy(), f"{dtype} {key}")


def test_selection_matches_reference_at_config2():
    """Window gate, hybrid scores and top-k against the reference's torch selectors on
    the GPU: T = 16,384 packed tokens (4 × 4,096), d_model 2,048, H = 16, dh = 128,
    k = 64, n 32…512, fp32."""
    from dsalt.kernels.landmark_tokens_ker import hybrid_scores_per_head
    from dsalt.kernels.selectors import select_topk
    from dsalt.kernels.window_gate import window_continuous
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(7)
    T, dm, H, dh, k = 16384, 2048, 16, 128, 64
    x = torch.randn(T, dm, generator=g, device=dev)
    W_V = torch.randn(H * dh, dm, generator=g, device=dev) / dm ** 0.5
    alpha = torch.rand(H, generator=g, device=dev)
    gate = torch.nn.Linear(dm, 1).to(dev)
    cu_list = [0, 4096, 8192, 12288, 16384]
    cu = torch.tensor(cu_list, dtype=torch.int32, device=dev)
    ref = ref_triton.run("select", {"x": x, "W_V": W_V, "alpha": alpha, "gate_w": gate.weight.detach(),
                                    "gate_b": gate.bias.detach(), "cu": cu, "cu_list": cu_list, "H": H, "dh": dh,
                                    "k": k, "n_min": 32, "n_max": 512})
    with torch.no_grad():
        w_cont = window_continuous(x, gate, 32, 512)
        scores, z_x, z_v = hybrid_scores_per_head(x, W_V, alpha, H, dh)
    # The gate's Linear is a 2,048-long dot product per token: cuBLAS (the reference's
    # nn.Linear) and this build's warp reduction add the products in different orders,
    # so w̃ agrees to a few ulp (at equal logits the window chain is bit-exact:
    # test_select_gpu.py::test_win_gate_bit_exact_at_fixed_logits).  The window sizes
    # floor(w̃) must then agree bit for bit at every token whose w̃ is not within that
    # rounding distance of an integer.
    got_w, ref_w = w_cont.float().cpu(), ref["w_cont"].float()
    ulp = torch.from_numpy(np.spacing(ref_w.numpy()))
    diff_ulp = ((got_w - ref_w).abs() / ulp)
    assert diff_ulp.max() <= 64, f"w̃ differs by {diff_ulp.max():.0f} ulp"
    margin = (diff_ulp.max() + 1) * ulp
    frac = ref_w - ref_w.floor()
    clear = (frac > margin) & (1 - frac > margin)
    assert clear.float().mean() > 0.999
    w_disc = got_w.floor().clamp(min=1)
    assert torch.equal(w_disc[clear], ref["w_disc"][clear])
    # z-scores: this build accumulates the mean and the std in fp64, torch in fp32
    torch.testing.assert_close(scores.cpu(), ref["scores"], rtol=1e-4, atol=1e-4)
    torch.testing.assert_close(z_x.cpu(), ref["z_x"], rtol=1e-4, atol=1e-4)
    # landmark index sets: bit-exact given the reference's scores and windows
    idx = select_topk(ref["scores"].to(dev), ref["w_disc"].to(dev), cu, k, 4096).cpu()
    ri = ref["idx"]
    assert idx.shape == ri.shape
    a = np.sort(idx.numpy(), axis=-1)
    b = np.sort(ri.numpy(), axis=-1)
    assert np.array_equal(a, b), f"{int((a != b).any(-1).sum())} (head, sequence) sets differ"
