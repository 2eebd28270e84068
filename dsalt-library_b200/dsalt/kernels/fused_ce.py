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


def _prepare(x, weight, labels, dtype):
    labels = labels.contiguous().long()
    V = weight.shape[0]
    # the kernel scores a label only inside [0, V): count exactly those, so the mean is
    # taken over the rows that carry a loss (ignore_index -100 and out-of-range labels
    # add nothing to either sum)
    n_valid = ((labels >= 0) & (labels < V)).sum()
    scale = (1.0 / n_valid.clamp(min=1).float()).reshape(1)
    row_loss = torch.empty(x.shape[0], dtype=torch.float32, device=x.device)
    return labels, x.to(dtype).contiguous(), weight.to(dtype).contiguous(), scale, row_loss


def _chunk_loss(x_c, w_c, labels, scale, row_loss, s, e, dtype):
    """Rows ``s:e``: logits GEMM, then the kernel's row losses; returns the logits
    buffer, which the kernel has overwritten with their gradient."""
    logits = torch.mm(x_c[s:e], w_c.t())
    p = _ext.XentParams(logits=_ext.ptr(logits), labels=_ext.ptr(labels[s:e]), row_loss=_ext.ptr(row_loss[s:e]),
                        scale=_ext.ptr(scale), rows=e - s, vocab=w_c.shape[0], ignore_index=-100,
                        dtype=_ext.dtype_code(dtype))
    _ext.call("dsalt_xent_fwd_grad", p)
    return logits


def _loss_only(x, weight, labels, chunk: int, dtype: torch.dtype) -> torch.Tensor:
    """Evaluation path (no gradient wanted): the per-chunk logits GEMM and row losses
    only; neither gradient GEMM runs and nothing is kept."""
    _ext.require_cuda(x, "x")
    labels, x_c, w_c, scale, row_loss = _prepare(x, weight, labels, dtype)
    chunk = max(int(chunk), 1)
    for s in range(0, x.shape[0], chunk):
        _chunk_loss(x_c, w_c, labels, scale, row_loss, s, min(s + chunk, x.shape[0]), dtype)
    return row_loss.sum() * scale[0]


class FusedChunkedCE(torch.autograd.Function):
    """``(x [N, d], weight [V, d], labels [N], chunk) -> mean CE over labels != -100``."""

    @staticmethod
    def forward(ctx, x, weight, labels, chunk: int, dtype: torch.dtype):
        _ext.require_cuda(x, "x")
        N, d = x.shape
        V = weight.shape[0]
        dev = x.device
        chunk = max(int(chunk), 1)
        labels, x_c, w_c, scale, row_loss = _prepare(x, weight, labels, dtype)
        dx = torch.empty_like(x_c)
        dw = None
        for s in range(0, N, chunk):
            e = min(s + chunk, N)
            logits = _chunk_loss(x_c, w_c, labels, scale, row_loss, s, e, dtype)
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
    if not (torch.is_grad_enabled() and (x.requires_grad or weight.requires_grad)):
        return _loss_only(x, weight, labels, chunk, dtype)
    return FusedChunkedCE.apply(x, weight, labels, chunk, dtype)
