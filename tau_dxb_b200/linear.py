"""Linear layers of the Whisper train step with the bias gradient on the
tau_column_sum kernel.

Autograd's linear backward forms the bias gradient as grad_output.sum(0)
through torch's generic reduction, which runs bf16 column sums at ~1.6 TB/s
(4 ms per Whisper-small step). ``LinearFunction`` keeps the forward (F.linear
under autocast's bf16 policy) and the dX / dW GEMMs, and sums the columns
with one HBM sweep instead. ``patch_linears(model)`` routes every nn.Linear
of a CUDA model through it; ``linear`` is the function form.
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
