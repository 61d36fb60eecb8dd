"""Torch autograd wrappers around the numpy oracle (test infrastructure only).

They let a Whisper model run the reference semantics on CPU, so model-level
tests can compare a model patched with the B200 kernels against the same
model patched with the oracle. Never imported by the product.
"""
import numpy as np
import torch

from oracle import stau_attention as OA
from oracle import wta as OW


def _np(t):
    return t.detach().float().cpu().numpy()


class OracleAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, log_tau, log_alpha, sigma_name, attn_mask=None, scale=None):
        out, c = OA.forward(_np(Q), _np(K), _np(V), _np(log_tau), _np(log_alpha), sigma_name,
                            None if attn_mask is None else _np(attn_mask), scale)
        ctx.c = c
        ctx.meta = (Q.dtype, Q.device, log_tau.dtype)
        return torch.from_numpy(out).to(Q.device, Q.dtype), None

    @staticmethod
    def backward(ctx, g, _unused=None):
        dt, dev, pdt = ctx.meta
        dQ, dK, dV, dlt, dla = OA.backward(ctx.c, _np(g))
        t = lambda a, d=dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev, d)
        return t(dQ), t(dK), t(dV), t(dlt, pdt), t(dla, pdt), None, None, None


class OracleCausalAttention(torch.autograd.Function):
    @staticmethod
    def forward(ctx, Q, K, V, log_tau, log_alpha, sigma_name, scale=None):
        mask = OA.causal_mask(Q.shape[2], K.shape[2])
        out, c = OA.forward(_np(Q), _np(K), _np(V), _np(log_tau), _np(log_alpha), sigma_name,
                            mask, scale)
        ctx.c = c
        ctx.meta = (Q.dtype, Q.device, log_tau.dtype)
        return torch.from_numpy(out).to(Q.device, Q.dtype)

    @staticmethod
    def backward(ctx, g):
        dt, dev, pdt = ctx.meta
        dQ, dK, dV, dlt, dla = OA.backward(ctx.c, _np(g))
        t = lambda a, d=dt: torch.from_numpy(np.ascontiguousarray(a)).to(dev, d)
        return t(dQ), t(dK), t(dV), t(dlt, pdt), t(dla, pdt), None, None


def _k_int(k, d):
    if isinstance(k, torch.Tensor):
        k = int(k.reshape(-1)[0].item())
    return OW.clamp_k(k, d)


class OracleSparseGrad(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, k):
        ctx.mask = torch.from_numpy(OW.threshold_mask(_np(x), _k_int(k, x.shape[-1]))).to(x.device)
        return x

    @staticmethod
    def backward(ctx, g):
        return g * ctx.mask.to(g.dtype), None


class OracleWTA(torch.autograd.Function):
    """Threshold WTA with an optional win-count buffer (the fused counting op)."""

    @staticmethod
    def forward(ctx, x, k, win=None):
        m = OW.threshold_mask(_np(x), _k_int(k, x.shape[-1]))
        mask = torch.from_numpy(m).to(x.device)
        if win is not None:
            win += mask.reshape(-1, x.shape[-1]).sum(0).to(win.dtype)
        ctx.mask = mask
        return torch.where(mask, x, torch.zeros_like(x))

    @staticmethod
    def backward(ctx, g):
        return g * ctx.mask.to(g.dtype), None, None


def use_oracle_ops(monkeypatch):
    """Route the patch modules' operators to the oracle (for CPU / reference runs)."""
    from tau_dxb_b200 import patch_whisper_sparse_grad as SG
    from tau_dxb_b200 import patch_whisper_stau as ST
    monkeypatch.setattr(ST, "STauOpusAttentionFunction", OracleAttention)
    monkeypatch.setattr(ST, "STauOpusCausalFunction", OracleCausalAttention)
    monkeypatch.setattr(SG, "SparseGradWTA_Function", OracleSparseGrad)
    monkeypatch.setattr(SG, "_WTAFusedCounting", OracleWTA)
