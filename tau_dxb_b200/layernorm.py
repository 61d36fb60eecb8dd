"""fp32 LayerNorm of the Whisper train step on the tau_layer_norm_* kernels.

transformers' Whisper layers use nn.LayerNorm over d_model = 768, which
autocast runs in fp32. Its stock CUDA backward reduces dgamma / dbeta in a
separate, slow pass (~200 us per encoder norm at batch 16); the kernels here
compute dx and the dgamma / dbeta partials in one sweep over dy and x.
``patch_layer_norms(model)`` swaps the forward of every nn.LayerNorm whose
width the kernels take (a multiple of 128 up to 1024) for ``fused_layer_norm``;
others are left as they are.

A norm whose output feeds exactly one GEMM (``bf16_out=True``) writes that
output in bf16 under autocast: the value autocast would have cast the fp32
output to, and its gradient comes back in bf16 and is read as such. This
drops one cast forward and one (strided, slow) cast back per norm and step.
A norm with several consumers keeps fp32 output, so that their gradients
still add in fp32.
"""
from __future__ import annotations

import types

import torch
import torch.nn as nn

from . import _capi as C


def supported(d: int) -> bool:
    return d % 128 == 0 and 0 < d <= 1024


class FusedLayerNormFunction(torch.autograd.Function):
    """y = layer_norm(x, (d,), weight, bias, eps) in fp32 on CUDA tensors."""

    @staticmethod
    @torch.amp.custom_fwd(device_type="cuda", cast_inputs=torch.float32)
    def forward(ctx, x, weight, bias, eps, out_bf16=False):
        d = x.shape[-1]
        x2 = x.reshape(-1, d).contiguous()
        M = x2.shape[0]
        y = torch.empty(M, d, dtype=torch.bfloat16 if out_bf16 else torch.float32, device=x.device)
        mean = torch.empty(M, dtype=torch.float32, device=x.device)
        rstd = torch.empty_like(mean)
        w = weight.contiguous()
        b = bias.contiguous()
        rc = C.lib().tau_layer_norm_fwd(x2.data_ptr(), M, d, w.data_ptr(), b.data_ptr(), float(eps),
                                        y.data_ptr(), C.BF16 if out_bf16 else C.F32, mean.data_ptr(),
                                        rstd.data_ptr(), C.stream_ptr(x.device))
        C.check("tau_layer_norm_fwd", rc)
        ctx.save_for_backward(x2, w, mean, rstd)
        ctx.shape = x.shape
        return y.view(x.shape)

    @staticmethod
    @torch.amp.custom_bwd(device_type="cuda")
    def backward(ctx, dy):
        x2, w, mean, rstd = ctx.saved_tensors
        M, d = x2.shape
        g = dy.reshape(M, d)
        if g.dtype not in (torch.float32, torch.bfloat16):
            g = g.float()
        g = g.contiguous()
        dx = torch.empty_like(x2)
        dw = torch.empty(d, dtype=torch.float32, device=x2.device)
        db = torch.empty_like(dw)
        lib = C.lib()
        ws = torch.empty(max(lib.tau_layer_norm_bwd_workspace_bytes(M, d), 16), dtype=torch.uint8,
                         device=x2.device)
        rc = lib.tau_layer_norm_bwd(g.data_ptr(), C.BF16 if g.dtype == torch.bfloat16 else C.F32,
                                    x2.data_ptr(), mean.data_ptr(), rstd.data_ptr(), w.data_ptr(),
                                    M, d, dx.data_ptr(), dw.data_ptr(), db.data_ptr(), ws.data_ptr(), ws.numel(),
                                    C.stream_ptr(x2.device))
        C.check("tau_layer_norm_bwd", rc)
        return dx.view(ctx.shape), dw, db, None, None


def fused_layer_norm(x, weight, bias, eps=1e-5, out_bf16=False):
    """fp32 layer norm; out_bf16 returns y in bf16 (rounded to nearest even)."""
    if not x.is_cuda:
        raise RuntimeError("tau_dxb_b200: fused_layer_norm runs on CUDA tensors only "
                           "(this build has no CPU implementation)")
    return FusedLayerNormFunction.apply(x, weight, bias, eps, bool(out_bf16))


def _forward(self, x):
    # the kernels take fp32 CUDA tensors (the model's master dtype, which
    # autocast keeps for layer norms); CPU models and other dtypes keep
    # torch's own norm
    fp32 = (x.dtype == torch.float32 or torch.is_autocast_enabled("cuda")) and self.weight.dtype == torch.float32
    if not (x.is_cuda and fp32):
        return nn.functional.layer_norm(x, self.normalized_shape, self.weight, self.bias, self.eps)
    bf16 = getattr(self, "_tau_dxb_bf16_out", False) and torch.is_autocast_enabled("cuda") \
        and torch.get_autocast_dtype("cuda") == torch.bfloat16
    return fused_layer_norm(x, self.weight, self.bias, self.eps, out_bf16=bf16)


def patch_layer_norms(model, bf16_out=None) -> int:
    """Route every affine nn.LayerNorm over one supported width to the fused
    kernels; returns how many were patched. bf16_out(name) -> bool names the
    norms whose output is the input of a single bf16 GEMM."""
    n = 0
    for name, m in model.named_modules():
        if isinstance(m, nn.LayerNorm) and len(m.normalized_shape) == 1 and m.elementwise_affine \
                and m.bias is not None and supported(m.normalized_shape[0]):
            m.forward = types.MethodType(_forward, m)
            m._tau_dxb_bf16_out = bool(bf16_out(name)) if bf16_out is not None else False
            n += 1
    return n


def unpatch_layer_norms(model) -> None:
    for m in model.modules():
        if isinstance(m, nn.LayerNorm):
            m.__dict__.pop("forward", None)
