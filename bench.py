#!/usr/bin/env python
"""Benchmark of the DSALT sparse-attention op on B200.

Headline (BASELINE.json metric, config 2): attended-pair TFLOP/s of one
forward+backward of the training op, B=4 packed sequences of N=4096, H=16,
D=128, bf16, k_lmk=64, w̃ = 32 + σ(g)·480.  A "step" is one call of the public
op ``dsalt_triton_train_attention`` plus its backward over the whole batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload config2|config3]
    python bench.py --impl reference        # the CPU restatement on the host cores

Multi-GPU (torchrun, one rank per GPU): the one global batch is split by heads
(rank r runs heads [r·H/N, (r+1)·H/N) of every sequence: config 2's 64 (sequence,
head) units become 8 per GPU at N=8), no collective in the timed region (strong
scaling); ``value`` sums the attended FLOPs of all ranks over the slowest rank's
time.  The NCCL all-gather that reassembles O along heads is timed apart
(``allgather_o``).  ``--workload config5`` (inference, heads sharded) and
``config4`` (model training step, DDP) are the other BASELINE configs.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "dsalt-library_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "attended-pair TFLOP/s fwd+bwd (N=4096, D=128)"
UNIT = "TFLOP/s"

WORKLOADS = {
    "config2": dict(lens=[4096] * 4, H=16, D=128, k=64, n_min=32, n_max=512,
                    desc="config2: B=4 packed x N=4096, H=16, D=128, bf16, k_lmk=64, w=32+sigmoid(g)*480"),
    "config3": dict(lens=None, H=16, D=128, k=64, n_min=64, n_max=1024,
                    desc="config3: 16 varlen seqs (randint(256,4097) seed 0), H=16, D=128, bf16, k_lmk=64, "
                         "w=64+sigmoid(g)*960"),
}

# per attended pair, algorithmic FLOPs of each kernel (fwd 4D; bwd 10D = dK/dV kernel: S, dP, dV, dK
# = 8D; dQ kernel: dQ = 2D, its S/dP recompute is not algorithmic work)
FLOPS_PER_PAIR = {"dsalt_attn_fwd": 4, "dsalt_attn_bwd_dkdv": 8, "dsalt_attn_bwd_dq": 2}
# kernels launched by each C-ABI entry point
KERNELS_PER_CALL = {"dsalt_build_schedule": 2, "dsalt_gather_landmarks": 1, "dsalt_attn_fwd": 1,
                    "dsalt_attn_bwd_preprocess": 1, "dsalt_attn_bwd_dkdv": 3, "dsalt_attn_bwd_dq": 2}
# (dsalt_attn_bwd_dkdv: landmark pass, band pass, landmark fix-up; dsalt_attn_bwd_dq: dQ, Σ_h d_w̃)
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) per launch of each entry point's main
# kernel: the median over the ten config-2 launches of one ncu capture of those two metrics
# (profiles/dram_traffic_config2.txt; for dsalt_attn_bwd_dkdv the band pass, which the landmark
# pass and the fix-up kernel accompany)
NCU_TRAFFIC_BYTES = {"config2": {"dsalt_attn_fwd": 301239808, "dsalt_attn_bwd_dkdv": 687554688,
                                 "dsalt_attn_bwd_dq": 515452800}}
# digest of csrc/ (kernel_source_digest) when that capture was taken; other sources -> traffic null
NCU_TRAFFIC_SRC = "232497833c0a8d95"
CLOCK_REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap",
                 0x8: "hw_slowdown", 0x10: "sync_boost", 0x20: "sw_thermal_slowdown",
                 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown", 0x100: "display_clock_setting"}


def seq_lens(wl) -> list[int]:
    if wl["lens"] is not None:
        return list(wl["lens"])
    import torch
    g = torch.Generator().manual_seed(0)
    return [int(x) for x in torch.randint(256, 4097, (16,), generator=g)]


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), float(d["hbm_gbs"]), "measured"
    return 1590.0, 1400.0, 6650.0, "fallback"


# ------------------------------------------------------------- multi-rank
def job_totals(ms: float, work: float, world: int, device) -> tuple[float, float]:
    """(max over the ranks of the timed milliseconds, sum over the ranks of the work):
    every rank calls it, two all-reduces in a fixed order (MAX, then SUM)."""
    if world <= 1:
        return float(ms), float(work)
    import torch
    import torch.distributed as dist
    tm = torch.tensor([ms], dtype=torch.float64, device=device)
    tw = torch.tensor([work], dtype=torch.float64, device=device)
    dist.all_reduce(tm, op=dist.ReduceOp.MAX)
    dist.all_reduce(tw, op=dist.ReduceOp.SUM)
    return float(tm.item()), float(tw.item())


def config5_shard(world: int) -> int:
    """Heads per rank of config 5 (its 32 heads split evenly, no collective in the op)."""
    if world <= 0 or CONFIG5["H"] % world:
        raise SystemExit("config5 shards 32 heads: --gpus must divide 32")
    return CONFIG5["H"] // world


# ----------------------------------------------------------------- workload
def make_workload(wl, seed, device):
    import torch
    from dsalt.kernels.selectors import select_topk
    lens = seq_lens(wl)
    T, H, D, k = sum(lens), wl["H"], wl["D"], wl["k"]
    g = torch.Generator(device=device).manual_seed(seed)
    q, kk, v, do = (torch.randn(T, H, D, generator=g, device=device).to(torch.bfloat16) for _ in range(4))
    do = do.float()  # the op returns fp32, so its upstream gradient arrives in fp32
    gate = torch.randn(T, generator=g, device=device)
    w = wl["n_min"] + torch.sigmoid(gate) * (wl["n_max"] - wl["n_min"])
    scores = torch.randn(T, H, generator=g, device=device)
    cu = torch.tensor([0] + list(__import__("itertools").accumulate(lens)), dtype=torch.int32, device=device)
    w_disc = w.floor().clamp(min=1)
    lmk_pos = select_topk(scores, w_disc, cu, k, max(lens))
    starts = cu[:-1].long()
    s_sel = scores[starts[None, :, None] + lmk_pos.clamp(min=0), torch.arange(H, device=device)[:, None, None]]
    lmk_logw = torch.log(torch.sigmoid(s_sel / 2.0).clamp(min=1e-20))
    lmk_logw = torch.where(lmk_pos >= 0, lmk_logw, torch.full_like(lmk_logw, float("-inf")))
    cu_list = [0] + list(__import__("itertools").accumulate(lens))
    return dict(q=q, k=kk, v=v, do=do, w=w, lmk_pos=lmk_pos, lmk_logw=lmk_logw, cu=cu, cu_list=cu_list,
                lens=lens, T=T, H=H, D=D, n_max=wl["n_max"])


def step_fn(d):
    import torch
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    q = d["q"].requires_grad_(True)
    k = d["k"].requires_grad_(True)
    v = d["v"].requires_grad_(True)
    w = d["w"].requires_grad_(True)
    lw = d["lmk_logw"].requires_grad_(True)

    def step():
        o = dsalt_triton_train_attention(q, k, v, d["lmk_pos"], lw, w, d["cu"], 1.0, 4.0, d["n_max"],
                                         d["cu_list"])
        return torch.autograd.grad(o, (q, k, v, w, lw), d["do"])
    return step


# ------------------------------------------------------------------- clocks
class ClockSampler:
    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index),
                 "--query-gpu=clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active",
                 "--format=csv,noheader,nounits", "-lms", "100"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self):
        if self.proc is None:
            return None
        sm, mx, reasons = [], [], 0
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 4:
                continue
            try:
                sm.append(float(parts[0]))
                mx.append(float(parts[1]))
                reasons |= int(parts[3], 16) if parts[3].startswith("0x") else int(parts[3])
            except ValueError:
                continue
        os.unlink(self.path)
        if not sm:
            return None
        names = [n for b, n in CLOCK_REASONS.items() if reasons & b and n != "gpu_idle"]
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": names,
                "samples": len(sm)}


# ------------------------------------------------------------- cpu baseline
def cpu_unit(wl, seed=0):
    """One (sequence, head) unit of the workload, built on the host (numpy)."""
    import numpy as np
    import torch
    from oracle import dsalt_oracle as O
    L, D, k = seq_lens(wl)[0], wl["D"], wl["k"]
    g = torch.Generator().manual_seed(1000 + seed)
    q, kk, v, do = (torch.randn(L, 1, D, generator=g).to(torch.bfloat16).float().numpy() for _ in range(4))
    gate = torch.randn(L, generator=g)
    w = (wl["n_min"] + torch.sigmoid(gate) * (wl["n_max"] - wl["n_min"])).numpy().astype(np.float32)
    scores = torch.randn(L, 1, generator=g).numpy()
    cu = np.array([0, L])
    pos = O.landmark_indices(scores, O.window_discrete(w), cu, k)
    lw = O.landmark_logw(scores, pos, cu)
    pairs = O.attended_pairs(w, pos, cu)
    return dict(q=q, k=kk, v=v, do=do, w=w, pos=pos, lw=lw, cu=cu, pairs=pairs, D=D, L=L)


def cpu_time_unit(u):
    import numpy as np
    from oracle import dsalt_oracle as O
    t0 = time.perf_counter()
    O.attention_bwd(u["q"], u["k"], u["v"], u["do"], u["pos"], u["lw"], u["w"], u["cu"], 1.0, 4.0, "train",
                    dtype=np.float32)
    return time.perf_counter() - t0


def prologue_bench(dev, hbm_gbs, reps=20):
    """The fused attention prologue (RoPE on q/k + GQA expansion, forward and
    backward) on config 4's per-GPU attention shape (8 x 2048 tokens, 16 heads,
    head_dim 64, bf16), and with 4 kv heads; timed with CUDA events against the
    torch expression it replaces.  Bytes are the algorithmic HBM bytes of the
    fused kernels (each tensor read or written once)."""
    import torch
    from dsalt.kernels.rope_gqa import rope_gqa
    from dsalt.kernels.window_utils import apply_rotary_emb, build_rope_cache
    T, H, D = 8 * 2048, 16, 64
    out = {"workload": "config4 attention prologue: T=16384 (8 x 2048), H=16, D=64, bf16, fwd+bwd"}
    cos_c, sin_c = build_rope_cache(2048, D, dev)
    pos = torch.arange(T, device=dev) % 2048
    cos, sin = cos_c[pos].to(torch.bfloat16), sin_c[pos].to(torch.bfloat16)
    for hkv in (16, 4):
        g = torch.Generator(device=dev).manual_seed(hkv)
        q = torch.randn(T, H, D, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
        k = torch.randn(T, hkv, D, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
        v = torch.randn(T, hkv, D, generator=g, device=dev).to(torch.bfloat16).requires_grad_(True)
        grads = [torch.randn(T, H, D, generator=g, device=dev).to(torch.bfloat16) for _ in range(3)]
        n_rep = H // hkv

        def torch_path():
            qr, kr = apply_rotary_emb(q, k, cos.unsqueeze(1), sin.unsqueeze(1))
            vr = v
            if n_rep > 1:
                kr = kr.unsqueeze(2).expand(T, hkv, n_rep, D).reshape(T, H, D)
                vr = v.unsqueeze(2).expand(T, hkv, n_rep, D).reshape(T, H, D)
            return qr, kr, vr

        def run(fn):
            outs = fn()
            torch.autograd.backward(outs, grads)

        # the two kernels alone through the C ABI (buffers allocated once)
        from dsalt.kernels import _ext
        from dsalt.kernels.rope_gqa import _params
        qo, ko = torch.empty_like(grads[0]), torch.empty_like(grads[0])
        vo = torch.empty_like(grads[0]) if n_rep > 1 else None
        dq, dk = torch.empty_like(q), torch.empty_like(k)
        dvv = torch.empty_like(v) if n_rep > 1 else None
        pf = _params(q, k, cos, sin, q=q, k=k, v=v if n_rep > 1 else None, q_out=qo, k_out=ko, v_out=vo)
        pb = _params(grads[0], k, cos, sin, dq_out=grads[0], dk_out=grads[1], dv_out=grads[2] if n_rep > 1 else None,
                     dq=dq, dk=dk, dv=dvv)
        for _ in range(3):
            _ext.call("dsalt_rope_gqa_fwd", pf)
            _ext.call("dsalt_rope_gqa_bwd", pb)
        ka, kb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        ka.record()
        for _ in range(reps):
            _ext.call("dsalt_rope_gqa_fwd", pf)
            _ext.call("dsalt_rope_gqa_bwd", pb)
        kb.record()
        torch.cuda.synchronize()
        res = {"kernels": ka.elapsed_time(kb) / reps * 1e3}
        for name, fn in (("fused", lambda: rope_gqa(q, k, v, cos, sin)), ("torch", torch_path)):
            for _ in range(3):
                run(fn)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            torch.cuda.synchronize()
            a.record()
            for _ in range(reps):
                run(fn)
            b.record()
            torch.cuda.synchronize()
            res[name] = a.elapsed_time(b) / reps * 1e3  # us per fwd+bwd
        e = 2  # bytes per element
        th, tkv, cs = T * H * D * e, T * hkv * D * e, 2 * T * D * e
        exp = n_rep > 1  # v is expanded (else it passes through untouched)
        fwd = th + th + tkv + th + cs + ((tkv + th) if exp else 0)   # q, q_out, k, k_out, cos/sin, v, v_out
        bwd = th + th + cs + th + tkv + ((th + tkv) if exp else 0)   # dq_out, dk_out, cos/sin, dq, dk, dv_out, dv
        gbs = (fwd + bwd) / (res["kernels"] * 1e-6) / 1e9
        out[f"hkv{hkv}"] = {"kernels_us": round(res["kernels"], 2), "bytes": int(fwd + bwd),
                            "achieved_gbs": round(gbs, 1), "frac_of_hbm": round(gbs / hbm_gbs, 3),
                            "op_fused_us": round(res["fused"], 2), "op_torch_us": round(res["torch"], 2)}
    out["note"] = ("kernels_us: the forward and backward kernels through the C ABI; op_*_us: forward + "
                   "autograd backward through the fused op and through the torch expression it replaces")
    return out


def cpu_baseline(wl, units=8):
    """The oracle on ``units`` (sequence, head) units of the workload: about 10 s of host work."""
    us = [cpu_unit(wl, s) for s in range(units)]
    cpu_time_unit(us[0])  # warm-up (BLAS threads, page faults)
    secs = sum(cpu_time_unit(u) for u in us)
    flops = sum(14 * u["D"] * u["pairs"] for u in us)
    return {"value": flops / secs / 1e12, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{units} (sequence, head) units of N={us[0]['L']}, D={us[0]['D']}, fwd+bwd, numpy float32 "
                      f"dense masked oracle, {secs:.1f} s"}


def run_reference(args, wl):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    u = [cpu_unit(wl, s) for s in range(max(args.steps, 1))]
    for s in range(args.warmup):
        cpu_time_unit(u[s % len(u)])
    secs = [cpu_time_unit(x) for x in u[:args.steps]]
    flops = sum(14 * x["D"] * x["pairs"] for x in u[:args.steps])
    val = flops / sum(secs) / 1e12
    line = {"metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": 1e3 * sum(secs) / len(secs), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": wl["desc"] + " (one (sequence, head) unit per step)", "seq_len": u[0]["L"]},
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
                             "sample": "one (sequence, head) unit per step, numpy float32 dense masked oracle "
                                       "(the reference is pure Python: its CPU path is restated in oracle/)"},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ config 4: LM training step
CONFIG4 = dict(vocab_size=32000, d_model=1024, n_layers=24, n_heads=16, n_min=32, n_max=512, k_lmk=64,
               max_seq_len=2048)
CONFIG4_BATCH, CONFIG4_SEQ = 8, 2048


def run_config4(args):
    """a full training step of DSALTLMHeadModel (forward, backward, AdamW) in bf16
    autocast on 8 x 2048 packed tokens per GPU, random init, seeded synthetic token ids; DDP with
    NCCL all-reduce of the gradients for N > 1 (weak scaling).  value = tokens/s of the whole job."""
    import datetime
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    from dsalt.model.dsalt_lm import DSALTLMHeadModel
    torch.manual_seed(0)
    model = DSALTLMHeadModel(**CONFIG4).to(dev)
    n_params = model.num_parameters()
    ddp = model
    if world > 1:
        from torch.nn.parallel import DistributedDataParallel as DDP
        # the model's only buffers are the constant RoPE tables: no per-step broadcast
        ddp = DDP(model, device_ids=[local], bucket_cap_mb=args.bucket_mb, gradient_as_bucket_view=True,
                  static_graph=True, broadcast_buffers=False)
        if args.ddp_bf16_grads:
            # all-reduce the gradient buckets in bf16 (half the NVLink bytes; rounds the summed gradients)
            from torch.distributed.algorithms.ddp_comm_hooks.default_hooks import bf16_compress_hook
            ddp.register_comm_hook(None, bf16_compress_hook)
    opt = torch.optim.AdamW(model.parameters(), lr=3e-4, betas=(0.9, 0.95), weight_decay=0.1, fused=True)
    T = CONFIG4_BATCH * CONFIG4_SEQ
    g = torch.Generator().manual_seed(1000 + rank)
    ids_host = torch.randint(0, CONFIG4["vocab_size"], (2, T + 1), generator=g).pin_memory()
    cu = torch.arange(0, T + 1, CONFIG4_SEQ, dtype=torch.int32, device=dev)
    ids_dev = [torch.empty(T + 1, dtype=torch.int64, device=dev) for _ in range(2)]
    loss_host = torch.empty(1, dtype=torch.float32).pin_memory()

    def step(n, e2e=False):
        buf = ids_dev[n % 2]
        if e2e:
            buf.copy_(ids_host[n % 2], non_blocking=True)
        with torch.autocast("cuda", dtype=torch.bfloat16):
            out = ddp(buf[:-1], cu_seqlens=cu, max_seqlen=CONFIG4_SEQ, labels=buf[1:])
        out["loss"].backward()
        opt.step()
        opt.zero_grad(set_to_none=True)
        if e2e:
            loss_host.copy_(out["loss"].detach().float().reshape(1), non_blocking=True)
        return out["loss"]

    for b in ids_dev:
        b.copy_(ids_host[0])

    def barrier():
        if world > 1:
            dist.barrier()

    def timed(k, e2e):
        barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for n in range(k):
            step(n, e2e)
        b.record()
        torch.cuda.synchronize()
        t = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for n in range(max(args.warmup, 3)):
        step(n)
    with ClockSampler(local) as clk:
        ms = timed(args.steps, False)
    ms_e2e = timed(args.steps, True)
    loss = float(step(0).detach().float().item())
    if rank == 0:
        tokens = world * T * args.steps
        line = {"metric": "train tokens/s (DSALTLMHeadModel config 4 training step)", "value": tokens / (ms / 1e3),
                "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": max(args.warmup, 3),
                "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                "dtype": "bf16", "data": "synthetic (seeded uniform token ids, random init)",
                "config": {"workload": "config4: DSALTLMHeadModel vocab 32000, d_model 1024, 24 layers, 16 heads, "
                                       "n_min 32, n_max 512, k_lmk 64; 8 x 2048 packed tokens per GPU, bf16 autocast, "
                                       "AdamW, chunked cross-entropy",
                           "global_batch": CONFIG4_BATCH * world, "seq_len": CONFIG4_SEQ, "tokens_per_gpu": T,
                           "parameters": n_params,
                           "parallelism": (f"dp{world} (DDP, NCCL all-reduce of gradients, {args.bucket_mb} MB buckets"
                                           + (", bf16 hook)" if args.ddp_bf16_grads else ")")) if world > 1 else "dp1",
                           "l2": "activations and weights far larger than L2, no flush"},
                "e2e": {"value": tokens / (ms_e2e / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": int((T + 1) * 8), "d2h_bytes_per_step": 4},
                "final_loss": loss,
                "clocks": clk.summary()}
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


# ------------------------------------------------------ selection and gating kernels
SEL_SHAPES = {
    # the standalone op's shapes (d_model = H·D, as in a DSALT layer of that width)
    "config2": dict(lens=[4096] * 4, H=16, D=128, d_model=2048, k=64, n_min=32, n_max=512),
    "config5": dict(lens=[32768], H=32, D=128, d_model=4096, k=256, n_min=128, n_max=2048),
}


def run_selection(args):
    """HBM throughput of the selection and gating kernels (window gate, hybrid score,
    top-k, and their backward passes) at the config-2 and config-5 shapes, bf16,
    each C-ABI entry point timed alone with CUDA events (``--steps`` launches after
    ``--warmup``).  Bytes are algorithmic: every input read once and every output
    written once (the hybrid score's internal norm / statistics scratch not counted).
    The x·W_Vᵀ GEMM feeding the score is cuBLAS and not part of these kernels."""
    import torch
    from dsalt.kernels import _ext
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", "0")))
    torch.cuda.set_device(dev)
    burst, sustained, hbm, src = peaks()
    out = {}
    shapes = [s for s in args.sel_shapes.split(",") if s]
    for name in shapes:
        c = SEL_SHAPES[name]
        lens, H, D, dm, k = c["lens"], c["H"], c["D"], c["d_model"], c["k"]
        T, S = sum(lens), len(lens)
        g = torch.Generator(device=dev).manual_seed(3)
        bf = torch.bfloat16
        x = torch.randn(T, dm, generator=g, device=dev).to(bf)
        W = (torch.randn(H * D, dm, generator=g, device=dev) / dm ** 0.5).to(bf)
        xwv = x @ W.t()
        gate_w = (torch.randn(dm, generator=g, device=dev) * 0.02).to(bf)
        gate_b = torch.zeros(1, device=dev, dtype=bf)
        alpha = torch.rand(H, generator=g, device=dev)
        cu = torch.tensor([0] + list(__import__("itertools").accumulate(lens)), dtype=torch.int32, device=dev)
        w_cont = torch.empty(T, dtype=bf, device=dev)
        w_disc = torch.empty(T, device=dev)
        logits = torch.empty(T, device=dev)
        scores, z_v = torch.empty(T, H, device=dev), torch.empty(T, H, device=dev)
        z_x = torch.empty(T, device=dev)
        stats, norms = torch.empty(2 + 2 * H, device=dev), torch.empty((1 + H) * T, device=dev)
        idx = torch.empty(H, S, k, dtype=torch.int64, device=dev)
        g_s = torch.randn(T, H, generator=g, device=dev)
        sums, d_alpha = torch.empty(2 * (1 + H), device=dev), torch.empty(H, device=dev)
        sparts = torch.empty((T + _ext.SCORE_BWD_TOKENS - 1) // _ext.SCORE_BWD_TOKENS, 2 * (1 + H) + H, device=dev)
        coef_x, coef_v = torch.empty(T, device=dev), torch.empty(T, H, device=dev)
        dl = torch.randn(T, generator=g, device=dev)
        dx = torch.empty_like(x)
        parts = torch.empty((T + _ext.WIN_GATE_ROWS_PER_PART - 1) // _ext.WIN_GATE_ROWS_PER_PART, dm, device=dev)
        sx, sv = torch.empty_like(x), torch.empty_like(xwv)
        P = _ext
        wg = P.WinGateParams(x=P.ptr(x), weight=P.ptr(gate_w), bias=P.ptr(gate_b), w_cont=P.ptr(w_cont), w_f32=0,
                             w_disc=P.ptr(w_disc), logits=P.ptr(logits), T=T, d_model=dm,
                             n_min=float(c["n_min"]), n_max=float(c["n_max"]), dtype=P.BF16)
        sc = P.ScoreParams(x=P.ptr(x), xwv=P.ptr(xwv), alpha=P.ptr(alpha), scores=P.ptr(scores), z_x=P.ptr(z_x),
                           z_v=P.ptr(z_v), stats=P.ptr(stats), norms=P.ptr(norms), T=T, d_model=dm, H=H, n_kv=H,
                           dh=D, dtype=P.BF16)
        tk = P.TopkParams(scores=P.ptr(scores), w_sizes=P.ptr(w_disc), cu_seqlens=P.ptr(cu), idx=P.ptr(idx), T=T,
                          H=H, S=S, k=k, max_len=max(lens))
        wgb = P.WinGateBwdParams(x=P.ptr(x), weight=P.ptr(gate_w), dl=P.ptr(dl), dx=P.ptr(dx), dw_part=P.ptr(parts),
                                 T=T, d_model=dm, dtype=P.BF16)
        scb = P.ScoreBwdParams(g_s=P.ptr(g_s), alpha=P.ptr(alpha), z_x=P.ptr(z_x), z_v=P.ptr(z_v),
                               norms=P.ptr(norms), stats=P.ptr(stats), sums=P.ptr(sums), partials=P.ptr(sparts),
                               d_alpha=P.ptr(d_alpha),
                               coef_x=P.ptr(coef_x), coef_v=P.ptr(coef_v), T=T, H=H, n_kv=H)
        srx = P.ScaleRowsParams(x=P.ptr(x), coef=P.ptr(coef_x), out=P.ptr(sx), T=T, groups=1, width=dm, dtype=P.BF16)
        srv = P.ScaleRowsParams(x=P.ptr(xwv), coef=P.ptr(coef_v), out=P.ptr(sv), T=T, groups=H, width=D,
                                dtype=P.BF16)
        e2, e4, e8 = 2, 4, 8
        kernels = [  # (entry point, params, algorithmic bytes)
            ("dsalt_win_gate", wg, T * dm * e2 + dm * e2 + T * (e2 + e4 + e4)),
            ("dsalt_hybrid_scores", sc, T * dm * e2 + T * H * D * e2 + T * H * e4 * 2 + T * e4),
            ("dsalt_select_topk", tk, T * H * e4 + T * e4 + H * S * k * e8),
            ("dsalt_win_gate_bwd", wgb, T * dm * e2 + dm * e2 + T * e4 + T * dm * e2 + parts.numel() * e4),
            ("dsalt_hybrid_scores_bwd", scb, T * H * e4 * 2 + T * e4 + (1 + H) * T * e4 + T * (1 + H) * e4),
            ("dsalt_scale_rows:x", srx, 2 * T * dm * e2 + T * e4),
            ("dsalt_scale_rows:xwv", srv, 2 * T * H * D * e2 + T * H * e4),
        ]
        res = {}
        for kname, prm, nbytes in kernels:
            entry = kname.split(":")[0]
            for _ in range(max(args.warmup, 1)):
                P.call(entry, prm)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            for _ in range(args.steps):
                P.call(entry, prm)
            b.record()
            torch.cuda.synchronize()
            us = a.elapsed_time(b) / args.steps * 1e3
            gbs = nbytes / (us * 1e-6) / 1e9
            res[kname] = {"us": round(us, 2), "bytes": int(nbytes), "gbs": round(gbs, 1),
                          "frac_of_hbm": round(gbs / hbm, 3)}
        out[name] = {"shape": f"T={T} ({S} x {lens[0]}), H={H}, D={D}, d_model={dm}, k={k}, bf16", "kernels": res}
    tot_b = sum(v["bytes"] for o in out.values() for v in o["kernels"].values())
    tot_us = sum(v["us"] for o in out.values() for v in o["kernels"].values())
    line = {"metric": "HBM GB/s of the selection and gating kernels", "value": tot_b / (tot_us * 1e-6) / 1e9,
            "unit": "GB/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": "selection/gating kernels at " + ", ".join(shapes) + " shapes"},
            "hbm_peak_gbs": hbm, "peak_source": src, "shapes": out}
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------- main
CONFIG5 = dict(N=32768, H=32, D=128, k=256, n_min=128, n_max=2048)
METRIC5 = "attended-pair TFLOP/s inference fwd (N=32768, D=128, H=32)"


def config5_inputs(heads, seed, device):
    """Config-5 inputs for ``heads`` of the 32 heads: q, k, v bf16 N(0,1), the per-token
    integer windows floor(128 + sigmoid(g)·1920) (one draw for all heads: the window
    gate is head-independent), hybrid scores N(0,1) and their top-256 landmarks."""
    import torch
    from dsalt.kernels.selectors import select_topk
    c = CONFIG5
    N, D, k = c["N"], c["D"], c["k"]
    gw = torch.Generator(device=device).manual_seed(5)
    w = (c["n_min"] + torch.sigmoid(torch.randn(N, generator=gw, device=device)) * (c["n_max"] - c["n_min"])).floor()
    g = torch.Generator(device=device).manual_seed(500 + seed)
    q, kk, v = (torch.randn(N, heads, D, generator=g, device=device).to(torch.bfloat16) for _ in range(3))
    scores = torch.randn(N, heads, generator=g, device=device)
    cu = torch.tensor([0, N], dtype=torch.int32, device=device)
    lmk = select_topk(scores, w.clamp(min=1), cu, k, N)
    bias = torch.zeros(heads, 1, k, device=device)
    return dict(q=q, k=kk, v=v, w=w, cu=cu, lmk=lmk, bias=bias, N=N, D=D)


def config5_cpu(rows_n=512, seed=0):
    """The oracle's row-wise inference forward on a bounded sample of (token, head) rows of
    one config-5 head (inputs drawn on the host with the same distributions)."""
    import numpy as np
    import torch
    from oracle import dsalt_oracle as O
    c = CONFIG5
    N, D, k = c["N"], c["D"], c["k"]
    g = torch.Generator().manual_seed(700 + seed)
    q, kk, v = (torch.randn(N, 1, D, generator=g).to(torch.bfloat16).float().numpy() for _ in range(3))
    w = (c["n_min"] + torch.sigmoid(torch.randn(N, generator=g)) * (c["n_max"] - c["n_min"])).floor().numpy()
    scores = torch.randn(N, 1, generator=g).numpy()
    cu = np.array([0, N])
    pos = O.landmark_indices(scores, O.window_discrete(w), cu, k)
    lw = np.zeros(pos.shape, dtype=np.float32)
    rng = np.random.default_rng(seed)
    rows = [(int(t), 0) for t in rng.integers(0, N, rows_n)]
    O.attention_fwd_rows(q, kk, v, pos, lw, w, cu, rows[:8], semantics="infer", dtype=np.float32)  # warm-up
    t0 = time.perf_counter()
    O.attention_fwd_rows(q, kk, v, pos, lw, w, cu, rows, semantics="infer", dtype=np.float32)
    secs = time.perf_counter() - t0
    # attended pairs of the sampled rows: the window min(w, i + 1) plus the landmarks before it
    p0 = pos[0, 0]
    pairs = 0
    for t, _ in rows:
        wi = max(int(w[t]), 1)
        pairs += min(wi, t + 1) + int(((p0 >= 0) & (p0 <= t) & (p0 < t - wi + 1)).sum())
    return {"value": 4 * D * pairs / secs / 1e12, "unit": UNIT, "cores": os.cpu_count(), "kind": "port",
            "sample": f"{rows_n} random (token, head) rows of one head, N=32768, D=128, numpy float32 row-wise "
                      f"inference oracle, {secs:.1f} s"}


def run_config5(args):
    """long-context inference forward of the op (B=1, H=32, N=32,768, D=128,
    bf16, n_min 128, n_max 2048, k_lmk 256) through dsalt_triton_attention; the 32 heads are
    sharded over the ranks (32/N per GPU, no collective in the op: strong scaling).  value =
    4·D·P over all heads (attended pairs, inference semantics) / max-over-ranks time."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        if rank == 0:
            vals = [config5_cpu(rows_n=256, seed=s) for s in range(max(args.steps, 1))]
            val = statistics.mean(v["value"] for v in vals)
            line = {"metric": METRIC5, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
                    "warmup": args.warmup, "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
                    "dtype": "f32", "data": "synthetic", "impl": "reference",
                    "config": {"workload": "config5 (CPU oracle on sampled rows)"},
                    "cpu_baseline": dict(vals[0], value=val),
                    "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
            print(json.dumps(line), flush=True)
        return
    heads = config5_shard(world)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from dsalt.kernels import _ext
    from dsalt.kernels.dsalt_triton_attn import dsalt_triton_attention
    from dsalt.kernels.flops import attended_pairs
    d = config5_inputs(heads, rank, dev)
    pairs = attended_pairs(d["w"], d["lmk"], d["cu"], semantics="infer")

    def step():
        return dsalt_triton_attention(d["q"], d["k"], d["v"], d["lmk"], d["bias"], d["w"], d["cu"])
    with torch.no_grad():
        for _ in range(max(args.warmup, 3)):
            step()
        torch.cuda.synchronize()
        barrier()
        with ClockSampler(local) as clk:
            _ext.RECORD = []
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            barrier()
            torch.cuda.synchronize()
            e0.record()
            for _ in range(args.steps):
                step()
            e1.record()
            torch.cuda.synchronize()
            rec, _ext.RECORD = _ext.RECORD, None
            barrier()
        ms = e0.elapsed_time(e1)
        launches = sum(KERNELS_PER_CALL.get(n, 1) for n, _, _ in rec)
        fwd = [a.elapsed_time(b) for n, a, b in rec if n == "dsalt_attn_fwd"]
        flops = 4.0 * d["D"] * pairs
        ms_max, flops_all = job_totals(ms, flops, world, dev)
        value = flops_all * args.steps / (ms_max / 1e3) / 1e12
        # end to end: q, k, v and the selection inputs copied from pinned host memory and O
        # (fp32) read back every step, copies on their own streams pipelined with the compute
        names = ("q", "k", "v", "w", "lmk", "bias")
        host = {kk: d[kk].cpu().pin_memory() for kk in names}
        dbuf = [{kk: torch.empty_like(d[kk]) for kk in names} for _ in range(2)]
        obuf = [torch.empty(d["q"].shape, dtype=torch.float32).pin_memory() for _ in range(2)]
        h2d = sum(x.numel() * x.element_size() for x in host.values())
        d2h = obuf[0].numel() * 4
        main = torch.cuda.current_stream(dev)
        cs, os_ = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
        ev_in, ev_used = [torch.cuda.Event() for _ in range(2)], [torch.cuda.Event() for _ in range(2)]

        def run(nsteps):
            cs.wait_stream(main)

            def h2d_step(n):
                if n >= 2:
                    cs.wait_event(ev_used[n % 2])
                with torch.cuda.stream(cs):
                    for kk in names:
                        dbuf[n % 2][kk].copy_(host[kk], non_blocking=True)
                ev_in[n % 2].record(cs)
            h2d_step(0)
            for n in range(nsteps):
                if n + 1 < nsteps:
                    h2d_step(n + 1)
                main.wait_event(ev_in[n % 2])
                x = dbuf[n % 2]
                o = dsalt_triton_attention(x["q"], x["k"], x["v"], x["lmk"], x["bias"], x["w"], d["cu"])
                ev_used[n % 2].record(main)
                os_.wait_stream(main)
                with torch.cuda.stream(os_):
                    o.record_stream(os_)
                    obuf[n % 2].copy_(o, non_blocking=True)
            main.wait_stream(os_)
            main.wait_stream(cs)
        run(2)
        torch.cuda.synchronize()
        barrier()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(main)
        run(args.steps)
        b.record(main)
        torch.cuda.synchronize()
        ems = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    if rank == 0:
        burst, sustained, hbm, src = peaks()
        kt = statistics.mean(fwd) if fwd else None
        roof = None
        if kt:
            ach = flops / (kt / 1e3) / 1e12
            roof = {"bound": "tensor", "kernel": "dsalt_attn_fwd", "achieved": ach, "peak": burst, "unit": UNIT,
                    "frac": ach / burst, "traffic": None,
                    "peak_source": f"{src} bf16_tflops (burst: the forward is timed alone)"}
        line = {"metric": METRIC5, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": "config5: B=1, N=32768, H=32, D=128, bf16, n_min 128, n_max 2048, "
                                       "k_lmk 256, inference forward (integer windows, zero landmark bias)",
                           "heads_per_gpu": heads, "parallelism": f"heads sharded {heads} per GPU, no collective",
                           "l2": "inputs larger than L2 (q,k,v bf16 = 805 MB at 32 heads), no flush"},
                "roofline": roof, "attended_pairs_per_gpu": pairs, "gpu_launches": launches,
                "e2e": {"value": flops_all * args.steps / (float(ems.item()) / 1e3) / 1e12, "unit": UNIT,
                        "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
                        "note": "host<->device copies on their own streams, pipelined with the neighbouring steps"},
                "clocks": clk.summary()}
        if not args.no_cpu_baseline and world == 1:  # the host baseline is timed at N = 1 only
            line["cpu_baseline"] = config5_cpu(rows_n=2048)  # about 10 s of host work
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="config2", choices=list(WORKLOADS) + ["config4", "config5", "selection"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-triton-ref", action="store_true", help="skip timing the reference's Triton op")
    ap.add_argument("--no-graph", action="store_true", help="time the eager step only (no CUDA graph)")
    ap.add_argument("--sel-shapes", default="config2,config5", help="selection: shapes to run")
    ap.add_argument("--bucket-mb", type=int, default=100, help="config4: DDP bucket size (MB)")
    ap.add_argument("--ddp-bf16-grads", action="store_true", help="config4: bf16 gradient all-reduce hook")
    args = ap.parse_args()
    if args.workload == "config4":
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the config-4 training step on the host "
                                  "cores takes far longer than the benchmark's time bound; the op workloads carry "
                                  "the CPU reference arm"}), flush=True)
            return
        run_config4(args)
        return
    if args.workload == "config5":
        run_config5(args)
        return
    if args.workload == "selection":
        if args.impl == "reference":
            print(json.dumps({"impl": "reference", "unavailable": "the selection kernels have no CPU arm; the op "
                              "workloads carry the CPU reference arm"}), flush=True)
            return
        run_selection(args)
        return
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
        return
    run_op(args, wl)


def run_op(args, wl):
    """Configs 2 and 3: forward + backward of the public training op.  With N ranks the
    one global batch is split by heads (``dsalt.kernels.head_shard``): rank r runs
    heads [h0, h1) of every sequence, no collective in the timed region (strong
    scaling: the whole job's work is fixed).  ``value`` = 14·D·P over all heads /
    the slowest rank's time."""
    import torch
    import torch.distributed as dist
    from dsalt.kernels import _ext
    from dsalt.kernels.head_shard import shard_op_inputs
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    from dsalt.kernels.flops import attended_pairs, scanned_pairs_fwd
    d = make_workload(wl, seed=0, device=dev)   # the same global batch on every rank
    H_all = d["H"]
    sh = shard_op_inputs(d["q"], d["k"], d["v"], d["lmk_pos"], d["lmk_logw"], rank, world, extra={"do": d["do"]})
    d.update(sh)
    d["H"] = sh["heads"][1] - sh["heads"][0]
    torch.cuda.empty_cache()
    pairs = attended_pairs(d["w"], d["lmk_pos"], d["cu"])
    scanned = scanned_pairs_fwd(d["w"], d["lmk_pos"], d["cu"])
    step = step_fn(d)
    for _ in range(max(args.warmup, 3)):
        step()
    torch.cuda.synchronize()
    barrier()

    def timed(fn):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record()
        for _ in range(args.steps):
            fn()
        e1.record()
        torch.cuda.synchronize()
        barrier()
        return e0.elapsed_time(e1)

    # the eager step: the public op called from Python every step
    ms_eager = timed(step)
    # the same step captured once as a CUDA graph and replayed: every kernel of the
    # forward and backward runs each step, without the per-call host work (at N > 1
    # the per-GPU problem is small enough for that host work to dominate)
    graph, graph_note = None, "eager"
    if not args.no_graph:
        try:
            cs = torch.cuda.Stream(device=dev)
            cs.wait_stream(torch.cuda.current_stream(dev))
            with torch.cuda.stream(cs):
                for _ in range(3):
                    step()
            torch.cuda.current_stream(dev).wait_stream(cs)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                step()
            for _ in range(3):
                graph.replay()
            torch.cuda.synchronize()
            graph_note = "CUDA graph of the whole forward + backward step, replayed"
        except Exception as e:  # keep the eager number
            graph, graph_note = None, f"eager (graph capture failed: {str(e)[:200]})"
    graph_ok = graph is not None
    if world > 1:  # every rank takes the same path
        flag = torch.tensor([1 if graph_ok else 0], device=dev)
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if not bool(flag.item()):
            graph, graph_ok = None, False
            graph_note = graph_note if graph_note.startswith("eager") else "eager (capture failed on another rank)"
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("timed_steps")
        ms = timed(graph.replay if graph_ok else step)
        torch.cuda.nvtx.range_pop()
    # per-entry-point durations for the roofline and the launch count: the same steps
    # again with CUDA events recorded around each C-ABI call (the stages run one after
    # the other on the caller's stream), outside the timed region
    _ext.RECORD = []
    n_rec = max(3, min(args.steps, 10))
    for _ in range(n_rec):
        step()
    torch.cuda.synchronize()
    rec, _ext.RECORD = _ext.RECORD, None
    launches = sum(KERNELS_PER_CALL.get(n, 1) for n, _, _ in rec) * args.steps // n_rec
    per_kernel = {}
    for name, a, b in rec:
        per_kernel.setdefault(name, []).append(a.elapsed_time(b))

    ms_max, flops_all = job_totals(ms, 14.0 * d["D"] * pairs, world, dev)
    ms_eager_max, _ = job_totals(ms_eager, 0.0, world, dev)
    _, scanned_all = job_totals(0.0, float(scanned), world, dev)
    _, pairs_all = job_totals(0.0, float(pairs), world, dev)
    value = flops_all * args.steps / (ms_max / 1e3) / 1e12

    # the optional reassembly of O along heads (one NCCL all-gather), timed apart
    gather = None
    if world > 1:
        from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
        from dsalt.kernels.head_shard import gather_heads
        with torch.no_grad():
            o_sh = dsalt_triton_train_attention(d["q"], d["k"], d["v"], d["lmk_pos"], d["lmk_logw"], d["w"],
                                                d["cu"], 1.0, 4.0, d["n_max"], d["cu_list"])
        for _ in range(3):
            gather_heads(o_sh, H_all)
        torch.cuda.synchronize()
        barrier()
        ga, gb = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 10
        ga.record()
        for _ in range(reps):
            gather_heads(o_sh, H_all)
        gb.record()
        torch.cuda.synchronize()
        gms, _ = job_totals(ga.elapsed_time(gb) / reps, 0.0, world, dev)
        gather = {"ms": gms, "bytes_out_per_rank": int(o_sh.numel() * 4), "dtype": "f32",
                  "note": "NCCL all_gather_into_tensor of the fp32 O shards along heads, outside the timed op"}
        del o_sh

    e2e = None
    if not args.no_e2e:
        e2e = e2e_op(args, d, dev, world, flops_all)

    if rank == 0:
        burst, sustained, hbm, src = peaks()
        kern = {n: (sum(v) / len(v), sum(v)) for n, v in per_kernel.items()}
        dom = max((n for n in kern if n in FLOPS_PER_PAIR), key=lambda n: kern[n][1])
        ach = FLOPS_PER_PAIR[dom] * d["D"] * pairs / (kern[dom][0] / 1e3) / 1e12
        traffic, traffic_note = ncu_traffic(args.workload, dom, world)
        roof = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": burst, "unit": UNIT,
                "frac": ach / burst, "traffic": traffic, "traffic_unit": "bytes per call (ncu dram read+write)",
                "traffic_note": traffic_note,
                "peak_source": f"{src} bf16_tflops (burst: each entry point is timed by its own events)"}
        units = len(d["lens"]) * d["H"]
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": max(args.warmup, 3), "ms_per_step": ms_max / args.steps, "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": wl["desc"], "global_batch": len(d["lens"]),
                           "seq_len": max(d["lens"]), "tokens": d["T"], "heads": H_all,
                           "heads_per_gpu": d["H"], "units_per_gpu": units,
                           "parallelism": (f"heads sharded {d['H']} per GPU ({units} (sequence, head) units), "
                                           "no collective in the op") if world > 1 else "single GPU, all 16 heads",
                           "l2": "inputs larger than L2 (q,k,v bf16 + dO fp32 = 320 MiB per step at N=1), no flush"},
                "roofline": roof,
                "kernels_ms": {n: round(v[0], 4) for n, v in kern.items()},
                "kernels_ms_note": "CUDA events around each C-ABI call, in steps run after the timed ones",
                "step": graph_note,
                "eager": {"value": flops_all * args.steps / (ms_eager_max / 1e3) / 1e12,
                          "ms_per_step": ms_eager_max / args.steps,
                          "note": "the public op called from Python every step (host launch work included)"},
                "attended_pairs": int(pairs_all), "scanned_pairs_fwd": int(scanned_all),
                "attended_over_scanned": pairs_all / max(scanned_all, 1.0),
                "gpu_launches": launches,
                "clocks": clk.summary()}
        if gather is not None:
            line["allgather_o"] = gather
        if e2e is not None:
            line["e2e"] = e2e
        if world == 1:
            line["prologue"] = prologue_bench(dev, hbm)
            if not args.no_triton_ref:
                line["triton_reference"] = triton_reference(args, d, flops_all, value)
        if not args.no_cpu_baseline and world == 1:  # the host baseline is timed at N = 1 only
            line["cpu_baseline"] = cpu_baseline(wl)
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()


def e2e_op(args, d, dev, world, flops_all):
    """The same op end to end through the public API with host buffers: every step
    copies its inputs (q, k, v bf16, the fp32 upstream gradient dO, w̃, landmark
    positions and weights) from pinned host memory and its results (O fp32, dQ, dK,
    dV, d_w̃, d_logw) back.  The copies run on their own streams, pipelined with the
    neighbouring steps' compute (inputs double-buffered on the device, outputs
    double-buffered on the host)."""
    import torch
    import torch.distributed as dist
    from dsalt.kernels.dsalt_triton_train import dsalt_triton_train_attention
    names = ("q", "k", "v", "w", "lmk_logw", "lmk_pos", "do")
    host = {kk: d[kk].detach().cpu().pin_memory() for kk in names}
    T = d["q"].shape[0]
    obuf = [[torch.empty(d["q"].shape, dtype=torch.float32).pin_memory()]
            + [torch.empty(d["q"].shape, dtype=torch.bfloat16).pin_memory() for _ in range(3)]
            + [torch.empty(T, dtype=torch.float32).pin_memory(),
               torch.empty(d["lmk_logw"].shape, dtype=torch.float32).pin_memory()] for _ in range(2)]
    dbuf = [{kk: torch.empty(host[kk].shape, dtype=host[kk].dtype, device=dev) for kk in names}
            for _ in range(2)]
    h2d = sum(x.numel() * x.element_size() for x in host.values())
    d2h = sum(x.numel() * x.element_size() for x in obuf[0])
    main = torch.cuda.current_stream(dev)
    copy_s, out_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    ev_in = [torch.cuda.Event() for _ in range(2)]
    ev_used = [torch.cuda.Event() for _ in range(2)]

    def h2d_step(n):
        bi = n % 2
        if n >= 2:
            copy_s.wait_event(ev_used[bi])  # the step that last read this buffer is done with it
        with torch.cuda.stream(copy_s):
            for kk in names:
                dbuf[bi][kk].copy_(host[kk], non_blocking=True)
        ev_in[bi].record(copy_s)

    def compute_step(n):
        bi = n % 2
        main.wait_event(ev_in[bi])
        x = dbuf[bi]
        q = x["q"].detach().requires_grad_(True)
        k = x["k"].detach().requires_grad_(True)
        v = x["v"].detach().requires_grad_(True)
        w = x["w"].detach().requires_grad_(True)
        lw = x["lmk_logw"].detach().requires_grad_(True)
        o = dsalt_triton_train_attention(q, k, v, x["lmk_pos"], lw, w, d["cu"], 1.0, 4.0, d["n_max"],
                                         d["cu_list"])
        grads = torch.autograd.grad(o, (q, k, v, w, lw), x["do"])
        ev_used[bi].record(main)
        return (o.detach(),) + tuple(grads)

    def d2h_step(n, outs):
        out_s.wait_stream(main)
        with torch.cuda.stream(out_s):
            for dst, g in zip(obuf[n % 2], outs):
                g.record_stream(out_s)
                dst.copy_(g, non_blocking=True)

    def run(nsteps):
        copy_s.wait_stream(main)
        h2d_step(0)
        for n in range(nsteps):
            if n + 1 < nsteps:
                h2d_step(n + 1)
            d2h_step(n, compute_step(n))
        main.wait_stream(out_s)
        main.wait_stream(copy_s)

    run(3)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(main)
    run(args.steps)
    b.record(main)
    torch.cuda.synchronize()
    ems = torch.tensor([a.elapsed_time(b)], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ems, op=dist.ReduceOp.MAX)
    return {"value": flops_all * args.steps / (float(ems.item()) / 1e3) / 1e12, "unit": UNIT,
            "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h),
            "note": "host<->device copies on their own streams, pipelined with the neighbouring steps; "
                    "dO shipped in fp32 (the op's output dtype), O and every gradient copied back"}


def triton_reference(args, d, flops_all, value):
    """The reference's own Triton training op on this GPU (the B200 speed bar): the
    unmodified package under baseline/_ref, run in a child process after its
    one-shot autotune, on the same inputs; forward + backward per step, CUDA events."""
    from oracle import ref_triton
    why = ref_triton.available()
    if why is not None:
        return {"unavailable": why}
    inp = {n: d[n] for n in ("q", "k", "v", "do", "w", "lmk_pos", "lmk_logw", "cu")}
    inp.update(cu_list=d["cu_list"], n_max=d["n_max"])
    try:
        r = ref_triton.run("train", inp, steps=max(3, min(args.steps, 10)), warmup=max(args.warmup, 3),
                           tuned_cache="/tmp/dsalt_ref_triton_tuned.json")
    except Exception as e:  # report, do not fail the benchmark line
        return {"unavailable": f"reference Triton run failed: {str(e)[-300:]}"}
    ref_val = flops_all * 1.0 / (r["ms_per_step"] / 1e3) / 1e12
    return {"value": ref_val, "unit": UNIT, "ms_per_step": r["ms_per_step"], "steps": r["steps"],
            "autotuned_config": r["cfg"], "this_build_over_reference": value / ref_val,
            "note": "dsalt_triton_train_attention from the unmodified reference (baseline/_ref) after its "
                    "autotune, same inputs, same attended-pair FLOP count"}


def ncu_traffic(workload, kernel, world):
    """DRAM bytes per call of ``kernel`` from the committed ncu capture, or None when the
    kernel sources changed since that capture (then the figure would be stale)."""
    rec = NCU_TRAFFIC_BYTES.get(workload, {})
    if world != 1 or kernel not in rec:
        return None, "no ncu capture for this workload / shard"
    if NCU_TRAFFIC_SRC != kernel_source_digest():
        return None, "stale: the kernel sources changed since the ncu capture"
    return rec[kernel], f"ncu capture of the same sources (digest {NCU_TRAFFIC_SRC})"


def kernel_source_digest() -> str:
    import hashlib
    h = hashlib.sha256()
    for f in sorted((ROOT / "dsalt-library_b200" / "csrc").glob("*.cu*")):
        h.update(f.name.encode())
        h.update(f.read_bytes())
    return h.hexdigest()[:16]


if __name__ == "__main__":
    main()
