"""Oracle for WTA top-k sparsity (TEST INFRASTRUCTURE ONLY).

numpy restatements of the reference's selection rules; the product never
imports this module.

* threshold semantics -- the reference's GPU path and sparse_grad:
    thr_i = k-th largest of row i;  keep_ij = x_ij >= thr_i
  echo/triton_wta.py:81-83 (topk(k).values[:, -1]) with the compare at
  echo/triton_wta.py:46-47, and echo/patch_whisper_sparse_grad.py:52-53
  (kthvalue(D-k+1), the same value). Ties at the threshold keep more than k.
* exact-k semantics -- echo/triton_wta.py:117-123 (topk indices + scatter):
  exactly k kept. Among elements equal to the threshold the lowest indices
  are kept here; torch.topk's tie order is implementation-defined, so tests
  compare this mode exactly only on rows without a tie at the threshold.
* k from the learnable logit -- echo/patch_whisper_sparse_grad.py:159-161:
  k = clamp(int(round(sigmoid_f32(logit) * d_ff)), 1, d_ff), Python's
  round-half-even on the float64 value of the fp32 sigmoid.
* forward output: threshold mode y = where(keep, x, +0) (echo/triton_wta.py:48);
  exact-k mode y = x * keep (echo/triton_wta.py:122), i.e. a dropped
  negative value becomes -0. Backward dx = dy * keep (echo/triton_wta.py:66-67;
  patch_whisper_sparse_grad.py:58-60).

bf16 inputs are handled as float32 arrays holding bf16-representable values
(exact), or as raw uint16 bit patterns via ``bf16_bits_to_f32``.
"""
from __future__ import annotations

import math

import numpy as np


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (NaN kept as NaN)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    rounding = ((u >> 16) & 1) + 0x7FFF
    out = ((u + rounding) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    out[nan] = 0x7FC0
    return out


def clamp_k(k: int, d: int) -> int:
    return max(1, min(d, int(k)))


def threshold_values(x: np.ndarray, k: int) -> np.ndarray:
    """k-th largest value of every row (float comparisons)."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    k = clamp_k(k, d)
    part = np.partition(x, d - k, axis=-1)
    return part[..., d - k]


def threshold_mask(x: np.ndarray, k: int) -> np.ndarray:
    x = np.asarray(x, dtype=np.float32)
    thr = threshold_values(x, k)
    return x >= thr[..., None]


def exact_k_mask(x: np.ndarray, k: int) -> np.ndarray:
    """Exactly k per row: all values > thr, then ties at thr by lowest index."""
    x = np.asarray(x, dtype=np.float32)
    d = x.shape[-1]
    k = clamp_k(k, d)
    thr = threshold_values(x, k)[..., None]
    gt = x > thr
    eq = x == thr
    need = k - gt.sum(axis=-1, keepdims=True)
    rank = np.cumsum(eq, axis=-1) - 1
    return gt | (eq & (rank < need))


def tie_rows(x: np.ndarray, k: int) -> np.ndarray:
    """Rows where the threshold value occurs so often that >= keeps more than k."""
    return threshold_mask(x, k).sum(axis=-1) > clamp_k(k, np.asarray(x).shape[-1])


def wta_forward(x: np.ndarray, k: int, mode: str = "threshold"):
    x = np.asarray(x, dtype=np.float32)
    if mode == "threshold":
        mask = threshold_mask(x, k)
        y = np.where(mask, x, np.float32(0.0))
    else:
        mask = exact_k_mask(x, k)
        y = x * mask.astype(np.float32)
    return y, mask


def wta_backward(dy: np.ndarray, mask: np.ndarray) -> np.ndarray:
    dy = np.asarray(dy, dtype=np.float32)
    return dy * mask.astype(np.float32)


def pack_mask_bits(mask: np.ndarray) -> np.ndarray:
    """Row-major bitmask, bit (j % 8) of byte j // 8 is element j (LSB first)."""
    return np.packbits(np.asarray(mask, dtype=bool), axis=-1, bitorder="little")


def k_from_logit(logit_k: float, d_ff: int) -> int:
    """LearnableKRatio.get_k (echo/patch_whisper_sparse_grad.py:159-161)."""
    lk = np.float32(logit_k)
    s = np.float32(1.0) / (np.float32(1.0) + np.exp(-lk, dtype=np.float32))
    k = int(round(float(s) * d_ff))
    return max(1, min(d_ff, k))


def logit_for_ratio(init_k_ratio: float) -> float:
    """LearnableKRatio._reset (echo/patch_whisper_sparse_grad.py:150-153)."""
    r = max(0.1, min(0.9, init_k_ratio))
    return float(np.float32(math.log(r / (1.0 - r + 1e-8))))
