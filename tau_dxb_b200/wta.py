"""WTA top-k sparsity on B200: autograd Functions over libtau_dxb.

Public surface (reference names and semantics):
  wta_fused_forward(x, k) -> y              echo/triton_wta.py:142-154
      threshold semantics (keep x >= k-th largest; the reference's CUDA path),
      straight-through backward dx = dy * keep.
  wta_fused_forward_with_mask(x, k) -> (y, bool mask)   echo/triton_wta.py:157-161
  SparseGradWTA_Function.apply(x, k) -> x   echo/patch_whisper_sparse_grad.py:38-60
      identity forward, dx = dy * (x >= k-th largest).
  WTA_Activation_Function.apply(x, k) -> y  echo/patch_whisper_sparse_grad.py:63-82
      exactly-k forward (ties by lowest index), same-mask backward.

The mask is kept as packed bits ([..., ceil(d/8)] uint8, 1/16 of the bf16
activation) between forward and backward. `k` may be a Python int or a
0-dim int32 CUDA tensor (read by the kernel: no host synchronisation).
CUDA tensors only: CPU inputs raise (there is no CPU implementation).
"""
from __future__ import annotations

import torch

from . import _capi as C

THRESHOLD = C.WTA_THRESHOLD
EXACT_K = C.WTA_EXACT_K


def _require_cuda(x):
    if not x.is_cuda:
        raise RuntimeError("tau_dxb_b200: WTA kernels run on CUDA tensors only "
                           "(this build has no CPU implementation)")


def _k_args(k, d):
    if isinstance(k, torch.Tensor):
        if k.dtype != torch.int32 or not k.is_cuda or k.numel() != 1:
            raise TypeError("tau_dxb_b200: a tensor k must be a 1-element int32 CUDA tensor")
        return 1, k.data_ptr()
    k = int(k)
    return max(1, min(d, k)), None


def wta_select(x: torch.Tensor, k, mode: int = THRESHOLD, write_y: bool = True,
               win_counts: torch.Tensor | None = None):
    """Run the fused selection kernel. Returns (y or None, packed bitmask)."""
    _require_cuda(x)
    d = x.shape[-1]
    x2 = x.reshape(-1, d)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    n = x2.shape[0]
    bits = torch.empty(x.shape[:-1] + ((d + 7) // 8,), dtype=torch.uint8, device=x.device)
    y = torch.empty_like(x, memory_format=torch.contiguous_format) if write_y else None
    kh, kd = _k_args(k, d)
    if win_counts is not None and (win_counts.dtype != torch.int32 or win_counts.numel() != d):
        raise TypeError("win_counts must be an int32 tensor with d elements")
    rc = C.lib().wta_fwd(x2.data_ptr(), C.dtype_code(x.dtype), n, d, x2.stride(0) if n else d,
                         kh, kd, mode, y.data_ptr() if y is not None else None, bits.data_ptr(),
                         win_counts.data_ptr() if win_counts is not None else None,
                         C.stream_ptr(x.device))
    C.check("wta_fwd", rc)
    return y, bits


def wta_backward_gelu(grad: torch.Tensor, x_pre: torch.Tensor, bits: torch.Tensor) -> torch.Tensor:
    """dx = gelu'(x_pre) * (dy * keep) for a selection run on gelu(x_pre)
    (wta_select(..., mode=THRESHOLD | C.WTA_GELU_INPUT)); bf16."""
    _require_cuda(grad)
    d = grad.shape[-1]
    g = grad.contiguous()
    xp = x_pre.contiguous()
    dx = torch.empty_like(g)
    n = g.numel() // d if d else 0
    rc = C.lib().wta_bwd_gelu(g.data_ptr(), xp.data_ptr(), bits.data_ptr(), n, d, dx.data_ptr(),
                              C.stream_ptr(g.device))
    C.check("wta_bwd_gelu", rc)
    return dx


def wta_backward(grad: torch.Tensor, bits: torch.Tensor) -> torch.Tensor:
    """dx = dy * keep for a packed bitmask from wta_select."""
    _require_cuda(grad)
    d = grad.shape[-1]
    g = grad.contiguous()
    dx = torch.empty_like(g)
    n = g.numel() // d if d else 0
    rc = C.lib().wta_bwd(g.data_ptr(), C.dtype_code(g.dtype), bits.data_ptr(), n, d,
                         dx.data_ptr(), C.stream_ptr(g.device))
    C.check("wta_bwd", rc)
    return dx


def unpack_mask(bits: torch.Tensor, d: int) -> torch.Tensor:
    """Packed bitmask -> bool mask [..., d]."""
    shifts = torch.arange(8, device=bits.device, dtype=torch.uint8)
    m = (bits.unsqueeze(-1) >> shifts) & 1
    return m.reshape(*bits.shape[:-1], -1)[..., :d].bool()


def k_from_logits(logits: torch.Tensor, d_ff: int) -> torch.Tensor:
    """k for every layer on device (LearnableKRatio.get_k without .item())."""
    _require_cuda(logits)
    lg = logits.detach().float().contiguous()
    out = torch.empty(lg.numel(), dtype=torch.int32, device=lg.device)
    rc = C.lib().wta_k_from_logits(lg.data_ptr(), lg.numel(), d_ff, out.data_ptr(),
                                   C.stream_ptr(lg.device))
    C.check("wta_k_from_logits", rc)
    return out


class _WTAFusedSTE(torch.autograd.Function):
    """Threshold WTA + straight-through backward (echo/triton_wta.py:94-114)."""

    @staticmethod
    def forward(ctx, x, k):
        y, bits = wta_select(x, k, THRESHOLD, write_y=True)
        ctx.save_for_backward(bits)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        (bits,) = ctx.saved_tensors
        return wta_backward(grad_y, bits), None


class WTA_Activation_Function(torch.autograd.Function):
    """Exactly-k WTA forward, same-mask backward (patch_whisper_sparse_grad.py:63-82)."""

    @staticmethod
    def forward(ctx, x, k):
        if not isinstance(k, torch.Tensor) and k < 1:
            k = max(1, int(x.shape[-1] * 0.3))
        y, bits = wta_select(x, k, EXACT_K, write_y=True)
        ctx.save_for_backward(bits)
        return y

    @staticmethod
    def backward(ctx, grad_output):
        (bits,) = ctx.saved_tensors
        return wta_backward(grad_output, bits), None


class SparseGradWTA_Function(torch.autograd.Function):
    """Identity forward; backward keeps the top-k positions of x
    (echo/patch_whisper_sparse_grad.py:38-60)."""

    @staticmethod
    def forward(ctx, x, k):
        if not isinstance(k, torch.Tensor) and k < 1:
            k = max(1, int(x.shape[-1] * 0.3))
        _, bits = wta_select(x, k, THRESHOLD, write_y=False)
        ctx.save_for_backward(bits)
        return x

    @staticmethod
    def backward(ctx, grad_output):
        (bits,) = ctx.saved_tensors
        return wta_backward(grad_output, bits), None


def wta_fused_forward(x: torch.Tensor, k) -> torch.Tensor:
    """Top-k per row, zero the rest; straight-through backward."""
    return _WTAFusedSTE.apply(x, k)


def wta_fused_forward_with_mask(x: torch.Tensor, k):
    """Like wta_fused_forward (no autograd) but also returns the bool mask."""
    y, bits = wta_select(x, k, THRESHOLD, write_y=True)
    return y, unpack_mask(bits, x.shape[-1])


def has_fused_kernels() -> bool:
    """True when libtau_dxb loads (the reference's has_triton() question)."""
    try:
        C.lib()
        return True
    except ImportError:
        return False
