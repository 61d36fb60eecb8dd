"""Oracle for the tau* solver (TEST INFRASTRUCTURE ONLY).

numpy restatement of solve_tau_star (tau_star/tau_star_solver.py:60-128), the
batched Newton iteration for

    tau* = argmin_tau KL(softmax(s) || softmax(tau * log sigma(s)))

per row of attention scores s: log sigma per tau_star_solver.py:25-43
(softplus: log(max(softplus, 1e-30)); sigmoid: -softplus(-s); exp: min(s, 20);
relu: log(max(relu, 1e-30))), e_ref = E_softmax(s)[log sigma], then n_iter
steps tau <- clip(tau - (E_p[log sigma] - e_ref) / (Var_p[log sigma] + eps),
tau_min, tau_max) with p = softmax(tau log sigma); the returned KL is
sum ref * log(max(ref / p, 1e-30)); non-finite tau -> tau_init, non-finite
KL -> 0; rows of one key return (tau_init, 0). fp32 throughout, as the
reference. The product never imports this module.
"""
from __future__ import annotations

import numpy as np


def _softplus(x):
    return np.where(x > 20.0, x, np.log1p(np.exp(np.minimum(x, 20.0)))).astype(np.float32)


def log_sigma(name: str, s: np.ndarray) -> np.ndarray:
    s = s.astype(np.float32)
    with np.errstate(divide="ignore", over="ignore"):
        if name == "softplus":
            return np.log(np.maximum(_softplus(s), np.float32(1e-30))).astype(np.float32)
        if name == "sigmoid":
            return (-_softplus(-s)).astype(np.float32)
        if name == "exp":
            return np.minimum(s, np.float32(20.0))
        if name == "relu":
            return np.log(np.maximum(np.maximum(s, 0.0), np.float32(1e-30))).astype(np.float32)
    raise KeyError(name)


def _softmax(x):
    m = x.max(axis=-1, keepdims=True)
    e = np.exp(x - m)
    return (e / e.sum(axis=-1, keepdims=True)).astype(np.float32)


def solve_tau_star(scores, sigma="softplus", n_iter=30, tau_init=2.0, tau_min=0.1, tau_max=10.0, eps=1e-6):
    s = np.asarray(scores, dtype=np.float32)
    shape = s.shape[:-1]
    if s.shape[-1] <= 1:
        return np.full(shape, tau_init, np.float32), np.zeros(shape, np.float32)
    ls = log_sigma(sigma, s)
    ref = _softmax(s)
    e_ref = (ref * ls).sum(-1)
    tau = np.full(shape, tau_init, np.float32)
    with np.errstate(all="ignore"):
        for _ in range(n_iter):
            p = _softmax(tau[..., None] * ls)
            e_p = (p * ls).sum(-1)
            var = (p * (ls - e_p[..., None]) ** 2).sum(-1)
            tau = np.clip(tau - (e_p - e_ref) / (var + np.float32(eps)), tau_min, tau_max).astype(np.float32)
        p = _softmax(tau[..., None] * ls)
        kl = (ref * np.log(np.maximum(ref / p, np.float32(1e-30)))).sum(-1).astype(np.float32)
    tau = np.where(np.isfinite(tau), tau, np.float32(tau_init)).astype(np.float32)
    kl = np.where(np.isfinite(kl), kl, np.float32(0.0)).astype(np.float32)
    return tau, kl


def solve_tau_star_analytic(scores, sigma="softplus"):
    """tau_star/tau_star_solver.py:131-151: clamp(cov_ref(s, ls) / (var_ref(ls)
    + 1e-6), 0.1, 10) with ref = softmax(s); NaN is kept (no sanitising)."""
    s = np.asarray(scores, dtype=np.float32)
    with np.errstate(all="ignore"):
        ls = log_sigma(sigma, s)
        ref = _softmax(s)
        mu_s = (ref * s).sum(-1, keepdims=True)
        mu_l = (ref * ls).sum(-1, keepdims=True)
        cov = (ref * (s - mu_s) * (ls - mu_l)).sum(-1)
        var = (ref * (ls - mu_l) ** 2).sum(-1)
        return np.clip(cov / (var + np.float32(1e-6)), 0.1, 10.0).astype(np.float32)

