"""Oracle for tau-opus attention in torch on the host (TEST INFRASTRUCTURE ONLY).

The same restatement as ``oracle.stau_attention`` (the reference's eager
operator, echo/stau_opus_operator.py:66-166), written with torch CPU ops in
the order the eager operator runs them: fp32 matmuls and full-size
elementwise passes over the [B,H,Lq,Lk] score tensor. It is the CPU arm that
bench.py times as the reference's eager path on the host cores, and it is
pinned to the same golden vectors as the numpy oracle
(tests/test_oracle_golden.py). The product never imports it.

Math per (b, h, row i), reference line numbers:
  s = scale Q K^T + mask; m = max_j s; x = s - m            (:82-88)
  sig = max(sigma(alpha x), 1e-8); q = max(sig^tau, 1e-8)   (:93-95)
  Z = max(sum q, 1e-8); P = q / Z; out = P V                (:96-99)
  dP = dO V^T; dV = P^T dO; D = sum P dP                     (:124-139)
  F = tau P (dP - D) sigma'(alpha x)/sig alpha; F[i, argmax_i] -= sum_j F
  dQ = scale F K; dK = scale F^T Q                           (:140-146)
  dtau = sum P (dP - D) max(log sig, -30)                    (:148-156)
  dalpha = sum tau P (dP - D) clip(sigma'/sig x, -30, 30)    (:158-162)
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

CLAMP_MIN = 1e-8


def _sigma(name, x):
    if name == "softplus":
        v = F.softplus(x)
    elif name == "sigmoid":
        v = torch.sigmoid(x)
    elif name == "exp":
        v = torch.exp(x.clamp(max=20))
    elif name == "relu":
        v = F.relu(x)
    else:
        raise KeyError(name)
    return v.clamp(min=CLAMP_MIN)


def _sigma_prime(name, x):
    if name == "softplus":
        return torch.sigmoid(x)
    if name == "sigmoid":
        s = torch.sigmoid(x)
        return s * (1 - s)
    if name == "exp":
        return torch.exp(x.clamp(max=15))
    if name == "relu":
        return (x > 0).to(x.dtype)
    raise KeyError(name)


@torch.no_grad()
def forward_backward(Q, K, V, log_tau, log_alpha, sigma_name, dO, attn_mask=None, scale=None):
    """Forward and backward of the eager operator on host tensors (fp32).

    Returns (out, (dQ, dK, dV, dlog_tau, dlog_alpha)) as torch tensors."""
    Q, K, V, dO = (torch.as_tensor(t, dtype=torch.float32) for t in (Q, K, V, dO))
    log_tau = torch.as_tensor(log_tau, dtype=torch.float32)
    log_alpha = torch.as_tensor(log_alpha, dtype=torch.float32)
    B, H, Lq, D = Q.shape
    if scale is None:
        scale = D ** -0.5
    s = torch.matmul(Q, K.transpose(-2, -1)) * scale
    if attn_mask is not None:
        s = s + torch.as_tensor(attn_mask, dtype=torch.float32)
    m = s.max(dim=-1, keepdim=True).values
    amax = s.argmax(dim=-1, keepdim=True)
    x = s - m
    del s
    tau = (F.softplus(log_tau) + 1.0).view(1, H, 1, 1)
    alpha = torch.exp(log_alpha).view(1, H, 1, 1)
    ax = x * alpha
    sig = _sigma(sigma_name, ax)
    q = sig.pow(tau).clamp(min=CLAMP_MIN)
    Z = q.sum(dim=-1, keepdim=True).clamp(min=CLAMP_MIN)
    P = q / Z
    del q
    out = torch.matmul(P, V)

    dP = torch.matmul(dO, V.transpose(-2, -1))
    dV = torch.matmul(P.transpose(-2, -1), dO)
    r = _sigma_prime(sigma_name, ax).clamp(min=CLAMP_MIN) / sig
    Dr = (dP * P).sum(dim=-1, keepdim=True)
    t = P * (dP - Dr)
    del dP, P
    Fs = tau * t * r * alpha
    Fs.scatter_add_(-1, amax, -Fs.sum(dim=-1, keepdim=True))
    dQ = torch.matmul(Fs, K) * scale
    dK = torch.matmul(Fs.transpose(-2, -1), Q) * scale
    del Fs
    dtau = (t * sig.log().clamp(min=-30)).sum(dim=(0, 2, 3))
    dalpha = (tau * t * (r * x).clamp(-30, 30)).sum(dim=(0, 2, 3))
    dlog_tau = dtau * torch.sigmoid(log_tau)
    dlog_alpha = dalpha * torch.exp(log_alpha)
    return out, (dQ, dK, dV, dlog_tau, dlog_alpha)
