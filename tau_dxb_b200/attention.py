"""tau-opus attention on B200: autograd Function and modules over libtau_dxb.

Public surface (same names, arguments and return values as the reference):
  STauOpusAttentionFunction.apply(Q, K, V, log_tau, log_alpha, sigma_name,
                                  attn_mask=None, scale=None) -> (out, None)
      echo/stau_opus_operator.py:48-166. The second output -- the
      materialised [B,H,Lq,Lk] attention matrix in the eager operator -- is
      None, as in echo/stau_opus_flash_v2.py:463; no caller on the training
      path reads it (echo/patch_whisper_stau.py:130-133).
  STauOpusAttentionModule(n_heads, sigma_name)   echo/stau_opus_operator.py:169-185
  init_log_tau_from_values, _log_tau_for_init    echo/stau_opus_operator.py:188-195

Differences from the eager operator, by design:
  * CUDA tensors only. There is no CPU path: CPU inputs raise.
  * Unknown sigma names raise KeyError, as the eager registry lookup does.
  * The output is a [B,H,Lq,D] view of a [B,Lq,H,D] buffer, so the
    attention-interface transpose(1,2).contiguous() that follows in the
    Whisper patch is free. Gradients dQ/dK/dV come back in the same layout.
  * bf16/f16 inputs run on the tcgen05 tensor-core kernels (D = 64); fp32
    inputs run on the precise fp32 kernels. set_attention_path() overrides.
"""
from __future__ import annotations

import contextlib
import math
import threading

import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _capi as C

CLAMP_MIN = 1e-8
SIGMA_NAMES = tuple(C.SIGMA_IDS)

_PATHS = {"auto": C.PATH_AUTO, "precise": C.PATH_PRECISE, "tensor": C.PATH_TENSOR}
_state = threading.local()


def _path() -> int:
    return getattr(_state, "path", C.PATH_AUTO)


def set_attention_path(name: str) -> None:
    """Select the kernel family for this thread: 'auto', 'precise' or 'tensor'."""
    _state.path = _PATHS[name]


@contextlib.contextmanager
def attention_path(name: str):
    old = _path()
    set_attention_path(name)
    try:
        yield
    finally:
        _state.path = old


def _require_cuda(*ts):
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("tau_dxb_b200: tau-opus attention runs on CUDA tensors only "
                               "(this build has no CPU implementation)")


def _per_head_values(log_tau, log_alpha):
    # echo/stau_opus_operator.py:90-91, evaluated in the parameters' dtype
    tau = F.softplus(log_tau) + 1.0
    alpha = torch.exp(log_alpha)
    return tau.float().contiguous(), alpha.float().contiguous()


def _mask_args(attn_mask, B, H, Lq, Lk, device):
    if attn_mask is None:
        return None, 0, None, None
    m = attn_mask
    if m.dtype == torch.bool:
        m = m.to(torch.float32)
    if m.device != device:
        m = m.to(device)
    while m.dim() < 4:
        m = m.unsqueeze(0)
    m = m.expand(B, H, Lq, Lk)
    return m, C.dtype_code(m.dtype), C.strides4(m), m


def _bhld_buffer(B, H, L, D, dtype, device):
    """[B,H,L,D] view of a contiguous [B,L,H,D] buffer."""
    return torch.empty(B, L, H, D, dtype=dtype, device=device).permute(0, 2, 1, 3)


class STauOpusAttentionFunction(torch.autograd.Function):
    """Fused tau-opus attention: out = softmax_sigma^tau(Q K^T * scale + mask) V."""

    @staticmethod
    def forward(ctx, Q, K, V, log_tau, log_alpha, sigma_name, attn_mask=None, scale=None):
        sigma_id = C.SIGMA_IDS[sigma_name]
        _require_cuda(Q, K, V, log_tau, log_alpha)
        B, H, Lq, D = Q.shape
        Lk = K.shape[2]
        if V.shape[-1] != D or K.shape[-1] != D:
            raise ValueError("tau_dxb_b200: Q, K and V must share the head dimension")
        if scale is None:
            scale = D ** -0.5
        dt = Q.dtype
        K = K if K.dtype == dt else K.to(dt)
        V = V if V.dtype == dt else V.to(dt)
        tau, alpha = _per_head_values(log_tau.detach(), log_alpha.detach())
        out = _bhld_buffer(B, H, Lq, D, dt, Q.device)
        row_max = torch.empty(B, H, Lq, dtype=torch.float32, device=Q.device)
        row_z = torch.empty_like(row_max)
        row_amax = torch.empty(B, H, Lq, dtype=torch.int32, device=Q.device)
        mptr, mdt, mst, mkeep = _mask_args(attn_mask, B, H, Lq, Lk, Q.device)
        path = _path()
        lib = C.lib()
        st = C.stream_ptr(Q.device)
        rc = lib.tau_attn_fwd(
            Q.data_ptr(), C.strides4(Q), K.data_ptr(), C.strides4(K), V.data_ptr(), C.strides4(V),
            C.dtype_code(dt), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(), sigma_id,
            float(scale), mptr.data_ptr() if mptr is not None else None, mdt, mst, 0,
            out.data_ptr(), C.strides4(out), row_max.data_ptr(), row_z.data_ptr(),
            row_amax.data_ptr(), path, st)
        C.check("tau_attn_fwd", rc)
        ctx.save_for_backward(Q, K, V, out, row_max, row_z, row_amax, tau, alpha,
                              log_tau, log_alpha, mkeep)
        ctx.sigma_id = sigma_id
        ctx.scale = float(scale)
        ctx.path = path
        return out, None

    @staticmethod
    def backward(ctx, grad_out, grad_attn_unused=None):
        (Q, K, V, out, row_max, row_z, row_amax, tau, alpha, log_tau, log_alpha,
         mkeep) = ctx.saved_tensors
        B, H, Lq, D = Q.shape
        Lk = K.shape[2]
        dt = Q.dtype
        g = grad_out if grad_out.dtype == dt else grad_out.to(dt)
        dQ = _bhld_buffer(B, H, Lq, D, dt, Q.device)
        dK = _bhld_buffer(B, H, Lk, D, dt, Q.device)
        dV = _bhld_buffer(B, H, Lk, D, dt, Q.device)
        dtau = torch.empty(H, dtype=torch.float32, device=Q.device)
        dalpha = torch.empty_like(dtau)
        lib = C.lib()
        ws_bytes = lib.tau_attn_bwd_workspace_bytes(B, H, Lq, Lk, D)
        ws = torch.empty(max(ws_bytes, 256), dtype=torch.uint8, device=Q.device)
        if mkeep is not None:
            mptr, mdt, mst = mkeep, C.dtype_code(mkeep.dtype), C.strides4(mkeep)
        else:
            mptr, mdt, mst = None, 0, None
        rc = lib.tau_attn_bwd(
            Q.data_ptr(), C.strides4(Q), K.data_ptr(), C.strides4(K), V.data_ptr(), C.strides4(V),
            out.data_ptr(), C.strides4(out), g.data_ptr(), C.strides4(g),
            C.dtype_code(dt), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(), ctx.sigma_id,
            ctx.scale, mptr.data_ptr() if mptr is not None else None, mdt, mst, 0,
            row_max.data_ptr(), row_z.data_ptr(), row_amax.data_ptr(),
            dQ.data_ptr(), C.strides4(dQ), dK.data_ptr(), C.strides4(dK),
            dV.data_ptr(), C.strides4(dV), dtau.data_ptr(), dalpha.data_ptr(),
            ws.data_ptr(), ws.numel(), ctx.path, C.stream_ptr(Q.device))
        C.check("tau_attn_bwd", rc)
        # echo/stau_opus_operator.py:154-155, 161
        grad_log_tau = dtau * torch.sigmoid(log_tau)
        grad_log_alpha = dalpha * torch.exp(log_alpha)
        return dQ, dK, dV, grad_log_tau, grad_log_alpha, None, None, None


class STauOpusCausalFunction(torch.autograd.Function):
    """tau-opus attention with a built-in causal mask (no mask tensor read).

    Equivalent to STauOpusAttentionFunction with the additive causal mask
    transformers builds for the Whisper decoder (finfo(float32).min where
    key j > query i + Lk - Lq) and no padding. The kernels apply it from the
    indices instead of loading a [B,1,Lq,Lk] tensor.
    """

    @staticmethod
    def forward(ctx, Q, K, V, log_tau, log_alpha, sigma_name, scale=None):
        sigma_id = C.SIGMA_IDS[sigma_name]
        _require_cuda(Q, K, V, log_tau, log_alpha)
        B, H, Lq, D = Q.shape
        Lk = K.shape[2]
        if scale is None:
            scale = D ** -0.5
        dt = Q.dtype
        K = K if K.dtype == dt else K.to(dt)
        V = V if V.dtype == dt else V.to(dt)
        tau, alpha = _per_head_values(log_tau.detach(), log_alpha.detach())
        out = _bhld_buffer(B, H, Lq, D, dt, Q.device)
        row_max = torch.empty(B, H, Lq, dtype=torch.float32, device=Q.device)
        row_z = torch.empty_like(row_max)
        row_amax = torch.empty(B, H, Lq, dtype=torch.int32, device=Q.device)
        path = _path()
        rc = C.lib().tau_attn_fwd(
            Q.data_ptr(), C.strides4(Q), K.data_ptr(), C.strides4(K), V.data_ptr(), C.strides4(V),
            C.dtype_code(dt), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(), sigma_id,
            float(scale), None, 0, None, 1, out.data_ptr(), C.strides4(out), row_max.data_ptr(),
            row_z.data_ptr(), row_amax.data_ptr(), path, C.stream_ptr(Q.device))
        C.check("tau_attn_fwd", rc)
        ctx.save_for_backward(Q, K, V, out, row_max, row_z, row_amax, tau, alpha, log_tau, log_alpha)
        ctx.sigma_id = sigma_id
        ctx.scale = float(scale)
        ctx.path = path
        return out

    @staticmethod
    def backward(ctx, grad_out):
        Q, K, V, out, row_max, row_z, row_amax, tau, alpha, log_tau, log_alpha = ctx.saved_tensors
        B, H, Lq, D = Q.shape
        Lk = K.shape[2]
        dt = Q.dtype
        g = grad_out if grad_out.dtype == dt else grad_out.to(dt)
        dQ = _bhld_buffer(B, H, Lq, D, dt, Q.device)
        dK = _bhld_buffer(B, H, Lk, D, dt, Q.device)
        dV = _bhld_buffer(B, H, Lk, D, dt, Q.device)
        dtau = torch.empty(H, dtype=torch.float32, device=Q.device)
        dalpha = torch.empty_like(dtau)
        lib = C.lib()
        ws = torch.empty(max(lib.tau_attn_bwd_workspace_bytes(B, H, Lq, Lk, D), 256),
                         dtype=torch.uint8, device=Q.device)
        rc = lib.tau_attn_bwd(
            Q.data_ptr(), C.strides4(Q), K.data_ptr(), C.strides4(K), V.data_ptr(), C.strides4(V),
            out.data_ptr(), C.strides4(out), g.data_ptr(), C.strides4(g),
            C.dtype_code(dt), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(), ctx.sigma_id,
            ctx.scale, None, 0, None, 1, row_max.data_ptr(), row_z.data_ptr(), row_amax.data_ptr(),
            dQ.data_ptr(), C.strides4(dQ), dK.data_ptr(), C.strides4(dK),
            dV.data_ptr(), C.strides4(dV), dtau.data_ptr(), dalpha.data_ptr(),
            ws.data_ptr(), ws.numel(), ctx.path, C.stream_ptr(Q.device))
        C.check("tau_attn_bwd", rc)
        return (dQ, dK, dV, dtau * torch.sigmoid(log_tau), dalpha * torch.exp(log_alpha),
                None, None)


class STauOpusAttentionModule(nn.Module):
    """Per-site module owning log_tau and log_alpha (echo/stau_opus_operator.py:169-185)."""

    def __init__(self, n_heads, sigma_name="softplus"):
        super().__init__()
        self.n_heads = n_heads
        self.log_tau = nn.Parameter(torch.zeros(n_heads))
        self.log_alpha = nn.Parameter(torch.zeros(n_heads))
        self.sigma_name = sigma_name

    def forward(self, Q, K, V, attn_mask=None, scale=None, is_causal=False):
        if is_causal and attn_mask is None:
            return STauOpusCausalFunction.apply(Q, K, V, self.log_tau, self.log_alpha,
                                                self.sigma_name, scale)
        out, _ = STauOpusAttentionFunction.apply(Q, K, V, self.log_tau, self.log_alpha,
                                                 self.sigma_name, attn_mask, scale)
        return out


def _log_tau_for_init(tau: float) -> float:
    """log_tau with softplus(log_tau) + 1 = tau (echo/stau_opus_operator.py:188-191)."""
    if tau <= 1.001:
        return -8.0
    return math.log(math.exp(tau - 1.0) - 1.0)


def init_log_tau_from_values(tau_list):
    return torch.tensor([_log_tau_for_init(t) for t in tau_list], dtype=torch.float32)
