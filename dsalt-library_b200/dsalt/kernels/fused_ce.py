"""Chunked LM-head cross-entropy with the gradient computed in the forward pass.

The reference's chunked loss (``dsalt/model/dsalt_lm.py:19-39``) runs, per chunk
of tokens, the LM-head GEMM, ``F.cross_entropy`` on fp32 copies of the logits
and, in the backward, the log-softmax backward and casts, keeping every chunk's
logits alive.  Here each chunk's logits (input dtype, cuBLAS GEMM) are turned in
place into their gradient by one CUDA kernel (``dsalt_xent_fwd_grad``) and
consumed at once by the two gradient GEMMs: dx (input dtype) and dW, summed
over the chunks in fp32 by the GEMM epilogue (autograd sums the reference's
per-chunk weight gradients in the compute dtype, which rounds more).  Only dx and dW are kept for the
backward, which scales them by the incoming gradient.
"""

from __future__ import annotations

import torch

from . import _ext


class FusedChunkedCE(torch.autograd.Function):
    """``(x [N, d], weight [V, d], labels [N], chunk) -> mean CE over labels != -100``."""

    @staticmethod
    def forward(ctx, x, weight, labels, chunk: int, dtype: torch.dtype):
        _ext.require_cuda(x, "x")
        N, d = x.shape
        V = weight.shape[0]
        dev = x.device
        chunk = max(int(chunk), 1)
        labels = labels.contiguous().long()
        x_c = x.to(dtype).contiguous()
        w_c = weight.to(dtype).contiguous()
        n_valid = (labels != -100).sum()
        scale = (1.0 / n_valid.clamp(min=1).float()).reshape(1)
        row_loss = torch.empty(N, dtype=torch.float32, device=dev)
        dx = torch.empty_like(x_c)
        dw = None
        for s in range(0, N, chunk):
            e = min(s + chunk, N)
            logits = torch.mm(x_c[s:e], w_c.t())
            p = _ext.XentParams(logits=_ext.ptr(logits), labels=_ext.ptr(labels[s:e]), row_loss=_ext.ptr(row_loss[s:e]),
                                scale=_ext.ptr(scale), rows=e - s, vocab=V, ignore_index=-100,
                                dtype=_ext.dtype_code(dtype))
            _ext.call("dsalt_xent_fwd_grad", p)
            torch.mm(logits, w_c, out=dx[s:e])
            # dW accumulated in fp32 by the GEMM epilogue
            if dw is None:
                dw = torch.mm(logits.t(), x_c[s:e], out_dtype=torch.float32)
            else:
                torch.addmm(dw, logits.t(), x_c[s:e], out_dtype=torch.float32, out=dw)
        if dw is None:
            dw = torch.zeros(V, d, dtype=torch.float32, device=dev)
        ctx.save_for_backward(dx, dw)
        ctx.x_dtype, ctx.w_dtype = x.dtype, weight.dtype
        return row_loss.sum() * scale[0]

    @staticmethod
    def backward(ctx, g):
        dx, dw = ctx.saved_tensors
        return (dx * g).to(ctx.x_dtype), (dw * g).to(ctx.w_dtype), None, None, None


def fused_chunked_cross_entropy(x: torch.Tensor, weight: torch.Tensor, labels: torch.Tensor,
                                chunk: int, dtype: torch.dtype) -> torch.Tensor:
    """Mean CE of ``x @ weightᵀ`` against ``labels`` in ``dtype`` (f16 / bf16) chunk by chunk."""
    return FusedChunkedCE.apply(x, weight, labels, chunk, dtype)
