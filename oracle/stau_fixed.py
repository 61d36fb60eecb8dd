"""Oracle for the fixed-tau attention weights (TEST INFRASTRUCTURE ONLY).

A numpy restatement of ``STauOpusMaxStableFn`` of the fixed-tau patch
(echo/patch_whisper_stau.py:74-112): attention weights from materialised
scores with a fixed per-head tau, and their gradient with respect to the
scores. Pinned to tests/golden/maxstable.npz (made by running the
reference's function, tests/golden/make_golden.py). The product never
imports it.

Per row of scores s (reference line numbers):
  x = s - max(s)                                   (:78)
  sig = sigma(x), every sigma clamped at 1e-8      (:79, :40-45)
  q = max(sig, 1e-8) ** tau                        (:80; no clamp on q)
  S = max(sum q, 1e-8); attn = q / S               (:81-82)
Backward with upstream g = dL/dattn (:89-112):
  A = tau max(sig, 1e-8)**(tau - 1) sigma'(x)      (sigma' unclamped)
  wda = sum g q; da = sum g A; sA = sum A
  ds = A (g / S - wda / S^2); ds[argmax s] -= da / S - wda sA / S^2
"""
from __future__ import annotations

import numpy as np

CLAMP_MIN = 1e-8
SIGMAS = ("softplus", "sigmoid", "exp", "relu", "tanh_shift")


def _sigmoid(x):
    with np.errstate(over="ignore"):
        return 1.0 / (1.0 + np.exp(-x))


def sigma(name, x):
    """The fixed-tau module's sigma registry (echo/patch_whisper_stau.py:40-53)."""
    with np.errstate(over="ignore"):
        if name == "softplus":
            v = np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, 20))))
        elif name == "sigmoid":
            v = _sigmoid(x)
        elif name == "exp":
            v = np.exp(np.minimum(x, 20))
        elif name == "relu":
            v = np.maximum(x, 0)
        elif name == "tanh_shift":
            v = np.tanh(x) + 1
        else:
            raise KeyError(name)
    return np.maximum(v, x.dtype.type(CLAMP_MIN))


def sigma_prime(name, x):
    """sigma' registry of the same module (echo/patch_whisper_stau.py:56-71); a
    name without an entry has sigma' = 1."""
    with np.errstate(over="ignore"):
        if name == "softplus":
            return _sigmoid(x)
        if name == "sigmoid":
            s = _sigmoid(x)
            return s * (1 - s)
        if name == "exp":
            return np.exp(np.minimum(x, 15))
        if name == "tanh_shift":
            return 1 - np.tanh(x) ** 2
        if name == "relu":
            return (x > 0).astype(x.dtype)
    return np.ones_like(x)


def _tau_rows(tau, shape):
    """tau as a scalar or a per-head vector broadcast over [B, H, Lq, Lk] rows."""
    t = np.asarray(tau, dtype=np.float32).reshape(-1)
    if t.size == 1:
        return t.reshape(())
    H = shape[1]
    return t.reshape(1, H, 1, 1)


def forward(scores, tau, sigma_name, dtype=np.float32):
    s = np.asarray(scores, dtype=dtype)
    x = s - s.max(axis=-1, keepdims=True)
    sig = sigma(sigma_name, x)
    tr = _tau_rows(tau, s.shape).astype(dtype)
    with np.errstate(under="ignore"):
        q = np.power(np.maximum(sig, dtype(CLAMP_MIN)), tr)
    S = np.maximum(q.sum(axis=-1, keepdims=True), dtype(CLAMP_MIN))
    return q / S


def backward(scores, tau, sigma_name, g, dtype=np.float32):
    s = np.asarray(scores, dtype=dtype)
    g = np.asarray(g, dtype=dtype)
    x = s - s.max(axis=-1, keepdims=True)
    sig = np.maximum(sigma(sigma_name, x), dtype(CLAMP_MIN))
    tr = _tau_rows(tau, s.shape).astype(dtype)
    with np.errstate(under="ignore", over="ignore"):
        A = tr * np.power(sig, tr - 1) * sigma_prime(sigma_name, x)
        q = np.power(sig, tr)
    S = np.maximum(q.sum(axis=-1, keepdims=True), dtype(CLAMP_MIN))
    wda = (g * q).sum(axis=-1, keepdims=True)
    da = (g * A).sum(axis=-1, keepdims=True)
    sA = A.sum(axis=-1, keepdims=True)
    ds = A * (g / S - wda / S ** 2)
    t2 = (da / S - wda * sA / S ** 2)[..., 0]
    idx = s.argmax(axis=-1)
    np.put_along_axis(ds, idx[..., None], np.take_along_axis(ds, idx[..., None], -1) - t2[..., None], -1)
    return ds
