"""Linear layers of the Whisper train step with the bias gradient on the
tau_column_sum kernel.

Autograd's linear backward forms the bias gradient as grad_output.sum(0)
through torch's generic reduction, which runs bf16 column sums at ~1.6 TB/s
(4 ms per Whisper-small step). ``LinearFunction`` keeps the forward (F.linear
under autocast's bf16 policy) and the dX / dW GEMMs, and sums the columns
with one HBM sweep instead. ``patch_linears(model)`` routes every nn.Linear
of a CUDA model through it; ``linear`` is the function form.

``cross_entropy`` is the train step's loss on bf16 logits: autocast runs
F.cross_entropy in fp32, which first copies the [tokens, vocab] logits to
fp32 (1.5 GB per Whisper-small step) and casts the gradient back; the fused
kernels read the bf16 logits directly (fp32 math) and write a bf16 gradient.
"""
from __future__ import annotations

import types

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _capi as C


def column_sum(g: torch.Tensor, out_dtype=None) -> torch.Tensor:
    """sum over rows of a [M, N] bf16 / fp32 CUDA matrix (fixed order)."""
    M, N = g.shape
    out = torch.empty(N, dtype=out_dtype or g.dtype, device=g.device)
    lib = C.lib()
    ws = torch.empty(max(lib.tau_column_sum_workspace_bytes(M, N), 4), dtype=torch.uint8, device=g.device)
    rc = lib.tau_column_sum(g.data_ptr(), C.dtype_code(g.dtype), M, N, out.data_ptr(), C.dtype_code(out.dtype),
                            ws.data_ptr(), ws.numel(), C.stream_ptr(g.device))
    C.check("tau_column_sum", rc)
    return out


def _kernel_ok(g: torch.Tensor) -> bool:
    return g.is_cuda and g.dtype in (torch.bfloat16, torch.float32) and g.shape[-1] % 8 == 0 \
        and g.is_contiguous() and g.data_ptr() % 16 == 0


class LinearFunction(torch.autograd.Function):
    """y = x W^T + b, as F.linear under autocast (inputs cast to bf16)."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.bfloat16)
    def forward(ctx, x, weight, bias):
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        return F.linear(x, weight, bias)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, gy):
        x, w = ctx.saved_tensors
        g2 = gy.reshape(-1, gy.shape[-1])
        dx = dw = db = None
        if ctx.needs_input_grad[0]:
            dx = (g2 @ w).view(*gy.shape[:-1], w.shape[1])
        if ctx.needs_input_grad[1]:
            dw = g2.t() @ x.reshape(-1, x.shape[-1])
        if ctx.has_bias and ctx.needs_input_grad[2]:
            g2c = g2.contiguous()
            db = column_sum(g2c) if _kernel_ok(g2c) else g2c.sum(0)
        return dx, dw, db


def linear(x, weight, bias=None):
    """F.linear whose backward sums the bias gradient on the column-sum kernel."""
    if not x.is_cuda:
        return F.linear(x, weight, bias)
    return LinearFunction.apply(x, weight, bias)


def _forward(self, x):
    return linear(x, self.weight, self.bias)


def patch_linears(model) -> int:
    """Route every nn.Linear of the model through ``linear``; returns the count."""
    n = 0
    for m in model.modules():
        if isinstance(m, nn.Linear):
            m.forward = types.MethodType(_forward, m)
            n += 1
    return n


class CrossEntropyFunction(torch.autograd.Function):
    """Mean cross-entropy of bf16 logits [M, V] against int64 labels [M]
    (ignore_index rows not counted), fp32 math, no fp32 copy of the logits."""

    @staticmethod
    def forward(ctx, logits, labels, ignore_index):
        M, V = logits.shape
        loss_row = torch.empty(M, dtype=torch.float32, device=logits.device)
        lse = torch.empty_like(loss_row)
        rc = C.lib().tau_cross_entropy_fwd(logits.data_ptr(), M, V, labels.data_ptr(), int(ignore_index),
                                           loss_row.data_ptr(), lse.data_ptr(), C.stream_ptr(logits.device))
        C.check("tau_cross_entropy_fwd", rc)
        counted = (labels != ignore_index).sum().to(torch.float32)
        ctx.save_for_backward(logits, labels, lse, counted)
        ctx.ignore_index = int(ignore_index)
        return loss_row.sum() / counted

    @staticmethod
    def backward(ctx, g):
        logits, labels, lse, counted = ctx.saved_tensors
        M, V = logits.shape
        scale = (g.float() / counted).reshape(1).contiguous()
        dlogits = torch.empty_like(logits)
        rc = C.lib().tau_cross_entropy_bwd(logits.data_ptr(), M, V, labels.data_ptr(), ctx.ignore_index,
                                           lse.data_ptr(), scale.data_ptr(), dlogits.data_ptr(),
                                           C.stream_ptr(logits.device))
        C.check("tau_cross_entropy_bwd", rc)
        return dlogits, None, None


def cross_entropy(logits, labels, ignore_index: int = -100):
    """F.cross_entropy(logits, labels) (mean, ignore_index) -- on the fused
    kernels for contiguous bf16 CUDA logits with a width that is a multiple
    of 8, else F.cross_entropy itself."""
    if logits.is_cuda and logits.dtype == torch.bfloat16 and logits.dim() == 2 and logits.shape[1] % 8 == 0 \
            and labels.dtype == torch.int64:
        lg = logits.contiguous()
        if lg.data_ptr() % 16 == 0:
            return CrossEntropyFunction.apply(lg, labels.contiguous(), ignore_index)
    return F.cross_entropy(logits, labels, ignore_index=ignore_index)

