"""The entry point that allocates nothing: dsalt_hybrid_scores_noalloc.

Some callers may not allocate device memory, for example a host runtime that
plans and owns every device buffer and passes a plugin only its inputs and
outputs.  For them the library offers dsalt_hybrid_scores_noalloc, which keeps
the scratch of the hybrid-score pipeline (per-token norms and their mean/std)
in a fixed array inside the library instead of in caller buffers.

These tests call it through the C ABI and check it against the allocating
entry point dsalt_hybrid_scores.  The file is named to be collected last, so a
run that stops at the first failure has run every other test before it; each
test also passes alone in a fresh process (the first call on a device sets up
the array's address).
"""

from __future__ import annotations

import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _call(name, x, xwv, alpha, H, n_kv, dh, scratch):
    from dsalt.kernels import _ext
    T, d = x.shape
    dev = x.device
    scores = torch.full((T, H), float("nan"), dtype=torch.float32, device=dev)
    z_x = torch.full((T,), float("nan"), dtype=torch.float32, device=dev)
    z_v = torch.full((T, H), float("nan"), dtype=torch.float32, device=dev)
    stats = torch.empty(2 + 2 * n_kv, dtype=torch.float32, device=dev) if scratch else None
    norms = torch.empty(T * (1 + n_kv), dtype=torch.float32, device=dev) if scratch else None
    p = _ext.ScoreParams(x=_ext.ptr(x), xwv=_ext.ptr(xwv), alpha=_ext.ptr(alpha), scores=_ext.ptr(scores),
                         z_x=_ext.ptr(z_x), z_v=_ext.ptr(z_v), stats=_ext.ptr(stats), norms=_ext.ptr(norms),
                         T=T, d_model=d, H=H, n_kv=n_kv, dh=dh, dtype=_ext.dtype_code(x.dtype))
    lib = _ext.load()
    rc = getattr(lib, name)(ctypes.byref(p), ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, _ext.status_string(rc)
    return scores, z_x, z_v


def _inputs(seed, T, d_model, H, n_kv, dh, dtype):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(T, d_model, generator=g, device="cuda").to(dtype)
    xwv = torch.randn(T, n_kv * dh, generator=g, device="cuda").to(dtype)
    alpha = torch.rand(H, generator=g, device="cuda")
    return x, xwv, alpha


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_noalloc_matches_allocating_entry_point_two_calls(dtype):
    shapes = [(4096 + 37, 256, 16, 16, 16), (1500, 128, 8, 4, 32)]   # second call: other sizes, GQA
    ins = [_inputs(100 + i, T, dm, H, nkv, dh, dtype) for i, (T, dm, H, nkv, dh) in enumerate(shapes)]
    refs = [_call("dsalt_hybrid_scores", *inp, H, nkv, dh, True)
            for inp, (T, dm, H, nkv, dh) in zip(ins, shapes)]
    # two no-allocation calls in a row, sharing the library's fixed scratch
    gots = [_call("dsalt_hybrid_scores_noalloc", *inp, H, nkv, dh, False)
            for inp, (T, dm, H, nkv, dh) in zip(ins, shapes)]
    torch.cuda.synchronize()
    for ref, got in zip(refs, gots):
        for r, g_ in zip(ref, got):
            torch.testing.assert_close(g_, r, rtol=1e-5, atol=1e-5)


def test_noalloc_rejects_sizes_beyond_its_limit():
    from dsalt.kernels import _ext
    lib = _ext.load()
    limit = 1 << 21  # DSALT_NOALLOC_SCORE_MAX_FLOATS
    n_kv = 16
    T = limit // (1 + n_kv) + 1
    p = _ext.ScoreParams(x=16, xwv=16, alpha=16, scores=16, T=T, d_model=64, H=16, n_kv=n_kv, dh=8,
                         dtype=_ext.BF16)
    assert lib.dsalt_hybrid_scores_noalloc(ctypes.byref(p), None) == 7  # DSALT_ERR_TOO_LARGE
