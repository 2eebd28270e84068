"""CPU checks of host-side logic of the model path: the compute-dtype choice that
routes layers to the CUDA kernels, the cached host copy of ``cu_seqlens`` and the
argument checks of the model-step entry points (no kernel is launched)."""

from __future__ import annotations

import ctypes

import pytest
import torch


def test_half_compute_dtype_rules():
    from dsalt.kernels import _ext
    x32, w32 = torch.zeros(4, 8), torch.zeros(16, 8)
    assert _ext.half_compute_dtype(x32, w32) is None  # CPU tensors never take the CUDA path
    assert _ext.half_compute_dtype(x32.bfloat16(), w32.bfloat16()) is None


def test_host_cu_copy_is_reused_until_the_tensor_changes():
    from dsalt.model.dsalt_lm import DSALTLMHeadModel
    m = DSALTLMHeadModel(vocab_size=64, d_model=256, n_layers=1, n_heads=4, n_min=8, n_max=32, k_lmk=4,
                         max_seq_len=256)
    cu = torch.tensor([0, 100, 256], dtype=torch.int32)
    first = m._host_cu(cu)
    assert first == [0, 100, 256]
    assert m._host_cu(cu) is first                      # same tensor, unmodified: no new copy
    cu[1] = 120                                         # in-place write bumps the version counter
    assert m._host_cu(cu) == [0, 120, 256]
    other = torch.tensor([0, 120, 256], dtype=torch.int32)
    assert m._host_cu(other) == [0, 120, 256]            # another tensor object: copied again
    assert m._cu_host[0] is other


def test_fused_ce_falls_back_on_cpu():
    from dsalt.model.dsalt_lm import _fused_ce_dtype
    assert _fused_ce_dtype(torch.zeros(2, 8), torch.zeros(10, 8)) is None


def _rc(name, p):
    from dsalt.kernels import _ext
    lib = _ext.load()
    return getattr(lib, name)(ctypes.byref(p), ctypes.c_void_p(0))


def test_model_step_entry_points_reject_bad_arguments():
    """Argument checks run before any launch: bad sizes, strides and dtypes come back
    as status codes (null device pointers are never dereferenced)."""
    from dsalt.kernels import _ext
    ARG, DT, HD = 1, 2, 3  # DSALT_ERR_ARG, DSALT_ERR_DTYPE, DSALT_ERR_HEAD_DIM of include/dsalt_b200.h
    # SwiGLU: F must split into 16-byte pieces, the row strides must cover F
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=4, F=12, ld_in=24, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=4, F=16, ld_in=8, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_swiglu_bwd", _ext.SwigluParams(T=4, F=16, ld_in=32, ld_out=8, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=4, F=16, ld_in=32, dtype=_ext.F32)) == DT
    assert _rc("dsalt_swiglu_fwd", _ext.SwigluParams(T=0, F=16, ld_in=32, dtype=_ext.BF16)) == _ext.OK
    # RMSNorm: supported widths only
    assert _rc("dsalt_rmsnorm_fwd", _ext.RmsNormParams(T=4, d=300, eps=1e-6, dtype=_ext.BF16)) == HD
    # window-gate backward: d_model a multiple of 8, 16-bit only
    assert _rc("dsalt_win_gate_bwd", _ext.WinGateBwdParams(T=4, d_model=12, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_win_gate_bwd", _ext.WinGateBwdParams(T=4, d_model=16, dtype=_ext.F32)) == DT
    # the prologue's row stride: a multiple of 8 elements and at least H·D
    assert _rc("dsalt_rope_gqa_fwd", _ext.RopeParams(T=4, ld=100, H=2, Hkv=2, D=64, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_rope_gqa_fwd", _ext.RopeParams(T=4, ld=130, H=2, Hkv=2, D=64, dtype=_ext.BF16)) == ARG
    # cross-entropy: 16-bit logits only
    assert _rc("dsalt_xent_fwd_grad", _ext.XentParams(rows=4, vocab=10, dtype=_ext.F32)) == DT


def test_grouped_kv_head_arguments_checked():
    """Grouped kv heads: H must be a multiple of H_kv (0 meaning H) in the attention,
    gather, prologue and group-sum entry points; checked before any launch."""
    from dsalt.kernels import _ext
    ARG, HD, OK = 1, 3, _ext.OK  # DSALT_ERR_ARG, DSALT_ERR_HEAD_DIM, DSALT_OK of include/dsalt_b200.h
    p = _ext.AttnParams(T=4, H=6, D=64, S=1, dtype=_ext.BF16, tau_win=1.0, H_kv=4)
    assert _rc("dsalt_attn_fwd", p) == ARG          # 6 query heads over 4 kv heads
    p.H_kv = 8
    assert _rc("dsalt_attn_fwd", p) == ARG          # more kv heads than query heads
    p.H_kv = -1
    assert _rc("dsalt_attn_fwd", p) == ARG
    g = _ext.GatherParams(T=4, H=6, D=64, S=1, dtype=_ext.BF16, H_kv=4)
    assert _rc("dsalt_gather_landmarks", g) == ARG
    assert _rc("dsalt_gqa_reduce", _ext.GqaReduceParams(T=4, H=6, H_kv=4, D=64, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_gqa_reduce", _ext.GqaReduceParams(T=4, H=8, H_kv=0, D=64, dtype=_ext.BF16)) == ARG
    assert _rc("dsalt_gqa_reduce", _ext.GqaReduceParams(T=0, H=8, H_kv=2, D=64, dtype=_ext.BF16)) == OK
    assert _rc("dsalt_gqa_reduce", _ext.GqaReduceParams(T=4, H=8, H_kv=2, D=12, dtype=_ext.BF16)) == HD
    # the prologue's k output: expanded (0 or H) or per kv head (Hkv), nothing else
    assert _rc("dsalt_rope_gqa_fwd", _ext.RopeParams(T=0, H=8, Hkv=2, D=64, dtype=_ext.BF16,
                                                     kv_out_heads=4)) == ARG
    assert _rc("dsalt_rope_gqa_fwd", _ext.RopeParams(T=0, H=8, Hkv=2, D=64, dtype=_ext.BF16,
                                                     kv_out_heads=2)) == OK


def test_gqa_head_sharding_keeps_groups():
    """head_shard with grouped kv heads: each rank takes whole kv-head groups and the
    query heads that read them."""
    import torch
    from dsalt.kernels.head_shard import shard_op_inputs
    T, H, Hkv, D = 5, 8, 2, 4
    q = torch.arange(T * H * D, dtype=torch.float32).view(T, H, D)
    k = torch.arange(T * Hkv * D, dtype=torch.float32).view(T, Hkv, D)
    pos = torch.zeros(H, 1, 3, dtype=torch.long)
    lw = torch.zeros(H, 1, 3)
    got = [shard_op_inputs(q, k, k, pos, lw, r, 2) for r in range(2)]
    assert [g["heads"] for g in got] == [(0, 4), (4, 8)]
    assert torch.equal(got[1]["k"], k[:, 1:2]) and torch.equal(got[1]["q"], q[:, 4:8])


def test_model_step_functions_refuse_cpu_tensors():
    """The CUDA model-step functions have no CPU path: called directly on CPU tensors
    they raise (the modules route CPU tensors to the reference's torch ops instead)."""
    from dsalt.kernels.fused_ce import fused_chunked_cross_entropy
    from dsalt.kernels.rmsnorm_cuda import add_rms_norm, rms_norm
    from dsalt.kernels.rope_gqa import qkv_rope
    from dsalt.kernels.swiglu import swiglu_ffn
    x = torch.randn(4, 256)
    w = torch.ones(256)
    with pytest.raises(RuntimeError, match="CUDA"):
        rms_norm(x, w, 1e-6)
    with pytest.raises(RuntimeError, match="CUDA"):
        add_rms_norm(x, x, w, 1e-6)
    with pytest.raises(RuntimeError, match="CUDA"):
        swiglu_ffn(x, torch.randn(512, 256), torch.randn(512, 256), torch.randn(256, 512), torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        fused_chunked_cross_entropy(x, torch.randn(10, 256), torch.zeros(4, dtype=torch.long), 2, torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        qkv_rope(x, torch.randn(128, 256), torch.randn(128, 256), torch.randn(128, 256), torch.ones(4, 64),
                 torch.zeros(4, 64), 2, 2, 64, torch.bfloat16)


def test_modules_keep_reference_ops_on_cpu():
    """On CPU the norm and FFN modules compute with the reference's torch ops."""
    import torch.nn.functional as F
    from dsalt.kernels.RMSENorm import RMSENorm
    from dsalt.modules.dsalt_transformer import SwiGLUFFN
    torch.manual_seed(0)
    n, ffn = RMSENorm(256), SwiGLUFFN(256, 512)
    x, r = torch.randn(5, 256), torch.randn(5, 256)
    s, y = n.add_forward(x, r)
    torch.testing.assert_close(s, x + r)
    torch.testing.assert_close(y, F.rms_norm(x + r, (256,), n.weight, n.eps))
    torch.testing.assert_close(ffn(x), ffn.down_proj(F.silu(ffn.gate_proj(x)) * ffn.up_proj(x)))


@pytest.mark.parametrize("loss_fn", ["chunked", "liger", "auto"])
def test_every_loss_fn_gives_the_chunked_loss_on_cpu(loss_fn):
    """All three reference loss options build and, on CPU, give the reference's chunked loss."""
    from dsalt.model.dsalt_lm import DSALTLMHeadModel, _chunked_cross_entropy
    torch.manual_seed(0)
    m = DSALTLMHeadModel(vocab_size=50, d_model=256, n_layers=1, n_heads=4, n_min=8, n_max=32, k_lmk=4,
                         max_seq_len=256, loss_fn=loss_fn, lm_head_chunk_size=7)
    x = torch.randn(2, 10, 256)
    labels = torch.randint(0, 50, (2, 10))
    labels[0, :3] = -100
    ref = _chunked_cross_entropy(x.reshape(-1, 256), m.lm_head.weight, labels.reshape(-1), 7)
    torch.testing.assert_close(m._compute_loss(x, labels), ref)


def test_tile_table_states_the_kernels_shapes():
    """The fixed tile table (autotune.py, the reference tuner's replacement) gives the
    shapes the CUDA sources compile: threads, rows, tiles and stages of each kernel."""
    import re
    from conftest import PKG
    from dsalt.kernels.autotune import get_tuned_config

    def const(fname, name):
        txt = (PKG / "csrc" / fname).read_text()
        m = re.search(rf"constexpr int {name} = (\d+);", txt)
        assert m, (fname, name)
        return int(m.group(1))
    for D in (64, 128):
        c = get_tuned_config(D)
        assert c["fwd"]["threads"] == const("attn_tc.cu", "kThreads")
        assert c["BLOCK_M"] == c["fwd"]["query_rows"] == const("attn_tc.cu", "BM")
        assert c["BLOCK_N"] == c["fwd"]["key_tile"] == const("attn_tc.cu", "BN")
        assert c["num_warps"] * 32 == c["fwd"]["threads"]
        assert c["bwd_dkdv"]["threads"] == const("attn_tc_bwd.cu", "kThreadsKV")
        assert c["BLOCK_N_BWD"] == c["bwd_dkdv"]["key_rows"]
        assert c["bwd_dkdv"]["q_do_stages"] == const("attn_tc_bwd.cu", "kQStages")
        assert c["bwd_dkdv"]["record_stages"] == const("attn_tc_bwd.cu", "kColStages")
        assert c["bwd_dq"]["threads"] == const("attn_tc_dq.cu", "kThreads")
        assert c["bwd_dq"]["stages"] == const("attn_tc_dq.cu", "kStages")
        assert sum(c["fwd"]["warps"].values()) * 32 == c["fwd"]["threads"]
        assert sum(c["bwd_dkdv"]["warps"].values()) * 32 == c["bwd_dkdv"]["threads"]
        assert sum(c["bwd_dq"]["warps"].values()) * 32 == c["bwd_dq"]["threads"]


def test_gradient_rounding_and_batch_band_arguments():
    """grad_round is 0 or 1; the batch's widest band needs the per-sequence maxima
    (both checked before any launch)."""
    from dsalt.kernels import _ext
    ARG = 1  # DSALT_ERR_ARG
    base = dict(T=0, H=2, D=64, S=1, k_lmk=0, kp=0, scale=0.125, tau_win=1.0, win_edge=4.0,
                semantics=_ext.TRAIN, dtype=_ext.BF16, impl=0)
    assert _rc("dsalt_attn_bwd_dkdv", _ext.AttnParams(**base, grad_round=2)) == ARG
    assert _rc("dsalt_attn_bwd_dq", _ext.AttnParams(**base, grad_round=-1)) == ARG
    assert _rc("dsalt_attn_bwd_dkdv", _ext.AttnParams(**base, grad_round=1)) == _ext.OK  # no tokens, no slots
    cu = ctypes.c_int32(0)
    sp = _ext.ScheduleParams(cu_seqlens=ctypes.addressof(cu), block_map=1, num_blocks=1, seq_wmax=0,
                             seq_wmax_batch=1, T=0, S=1, block=128, max_blocks=1, semantics=_ext.TRAIN)
    assert _rc("dsalt_build_schedule", sp) == ARG


def test_reduce_window_grad_single_process_rounds_once():
    """Without a process group the shard sum is the local one; with out_dtype it is
    rounded once to that dtype and kept in fp32."""
    from dsalt.kernels.head_shard import reduce_window_grad
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1000, generator=g, dtype=torch.float64)
    assert torch.equal(reduce_window_grad(x), x.float())
    r = reduce_window_grad(x, torch.bfloat16)
    assert r.dtype == torch.float32 and torch.equal(r, x.float().bfloat16().float())
