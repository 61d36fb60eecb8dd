"""Attach learnable tau-opus attention to HuggingFace Whisper (B200 kernels).

Same public functions as the reference module echo/patch_whisper_stau.py:
  apply_learnable_stau(model, tau_init, alpha_init, sigma_name, default_tau_json,
                       use_flash)                       (:325-405)
  remove_stau(model)                                    (:408-415)
  load_tau_dict(json_path)                              (:150-183)
  STauOpusLearnable(n_heads, sigma_name)                (:115-133)
  apply_fixed_stau(model, tau_source, sigma_name)       (:279-322)
  STauOpusMaxStableFn.apply(scores, tau, sigma_name)    (:74-112)
  _classify_attn, _parse_layer_idx, _log_tau_for_init   (:140-147, :274-276, :267-271)

Every WhisperAttention module gets a `_stau_opus` submodule owning per-head
`log_tau` and `log_alpha` (state_dict keys `...self_attn._stau_opus.log_tau`
as in the reference), and transformers' module-global
`eager_attention_forward` is swapped for one that runs the fused operator.
`use_flash` is accepted for signature compatibility; there is one operator.

Each patched WhisperAttention also gets a forward that hands the operator
the q/k/v projections as strided [B,H,L,D] views, with the 1/sqrt(d) scale
passed to the kernel, instead of transformers' `.transpose(1, 2).contiguous()`
copies and its separate `q * scaling` pass (three activation-sized copies and
one multiply per call). The scale is 2^-3 for Whisper's head size, so scaling
q in bf16 and scaling inside the kernel give the same bits. Calls with a KV
cache (generation) go through transformers' own forward.

`fuse_qkv=True` computes q, k and v with one GEMM over the concatenated
projection weights (k and v for cross-attention): the shared input is cast to
bf16 once and its gradient is one tensor, instead of three casts, three casts
back and two adds. Parameters stay separate; values change at the level of
rounding (one fp32 accumulation over 3 x d instead of three).

`assume_causal_decoder=True` tells the decoder self-attention
sites that their additive mask is the plain causal mask (true in training
with labels and no decoder padding mask); the kernels then apply causality
from indices instead of reading the [B,1,L,L] mask tensor. Results are the
same as with the mask tensor.
"""
from __future__ import annotations

import json
import math
import re
import types
from pathlib import Path
from typing import Dict, Union

import torch
import torch.nn as nn
import torch.nn.functional as F
from transformers.models.whisper import modeling_whisper as whisper_module

from .attention import STauOpusAttentionFunction, STauOpusCausalFunction

_ORIGINAL_EAGER_FORWARD = whisper_module.eager_attention_forward
SITE_KINDS = ("encoder_self", "decoder_self", "decoder_cross")


class STauOpusLearnable(nn.Module):
    """tau-opus with learnable per-head tau = softplus(log_tau) + 1 and
    alpha = exp(log_alpha) (echo/patch_whisper_stau.py:115-133)."""

    def __init__(self, n_heads, sigma_name="softplus"):
        super().__init__()
        self.log_tau = nn.Parameter(torch.zeros(n_heads))
        self.log_alpha = nn.Parameter(torch.zeros(n_heads))
        self.sigma_name = sigma_name
        self.assume_causal = False

    def forward(self, Q, K, V, attn_mask=None, scale=None):
        if self.assume_causal and attn_mask is not None and Q.shape[2] > 1:
            return STauOpusCausalFunction.apply(Q, K, V, self.log_tau, self.log_alpha,
                                                self.sigma_name, scale)
        out, _ = STauOpusAttentionFunction.apply(Q, K, V, self.log_tau, self.log_alpha,
                                                 self.sigma_name, attn_mask, scale)
        return out


def _classify_attn(name: str, module) -> str:
    """encoder_self / decoder_self / decoder_cross (echo/patch_whisper_stau.py:140-147)."""
    if not getattr(module, "is_decoder", False):
        return "encoder_self"
    if "encoder_attn" in name:
        return "decoder_cross"
    return "decoder_self"


def _parse_layer_idx(name: str) -> int:
    m = re.search(r"layers\.(\d+)", name)
    return int(m.group(1)) if m else 0


def load_tau_dict(json_path: Union[str, Path]) -> Dict[str, Dict[int, list]]:
    """Read a tau* JSON (either record format of echo/patch_whisper_stau.py:150-183)
    into {"encoder_self": {layer: [H taus]}, ...}."""
    with open(json_path, "r", encoding="utf-8") as f:
        data = json.load(f)
    out = {k: {} for k in SITE_KINDS}
    for item in data:
        if "module_name" in item:
            name = item["module_name"]
            if "encoder_attn" in name:
                key = "decoder_cross"
            elif "decoder" in name and "self_attn" in name:
                key = "decoder_self"
            else:
                key = "encoder_self"
            layer = _parse_layer_idx(name)
        else:
            kind = item.get("attention_type")
            if kind in out:
                key = kind
            elif item.get("cross_attention"):
                key = "decoder_cross"
            else:
                key = "decoder_self" if item.get("is_decoder") else "encoder_self"
            layer = item.get("layer_idx")
            if layer is None:
                layer = 0
        out[key][layer] = item["tau_per_head"]
    return out


def _log_tau_for_init(tau: float) -> float:
    """log_tau with softplus(log_tau) + 1 = tau; -8 for tau <= 1.001."""
    if tau <= 1.001:
        return -8.0
    return math.log(math.exp(tau - 1.0) - 1.0)


class STauOpusMaxStableFn(torch.autograd.Function):
    """Fixed-tau attention weights from materialised scores
    (echo/patch_whisper_stau.py:74-112): x = s - max(s), q = max(sigma(x),
    1e-8)^tau, attn = q / max(sum q, 1e-8), and the score gradient with the
    max shift's correction at the row's first argmax. The operator of the
    fixed-tau patch. Runs on tau_opus_fixed_fwd / tau_opus_fixed_bwd (one warp
    per row, fp32). tau: a number or a per-head tensor of shape (1, H, 1, 1)
    for [B, H, Lq, Lk] scores; sigma_name adds 'tanh_shift' to the four sigmas
    of the fused operator. CUDA tensors only."""

    @staticmethod
    def forward(ctx, scores, tau, sigma_name):
        from . import _capi as C
        sid = C.FIXED_SIGMA_IDS[sigma_name]
        if not scores.is_cuda:
            raise RuntimeError("tau_dxb_b200: STauOpusMaxStableFn runs on CUDA tensors only")
        s = scores.float().contiguous()
        L = s.shape[-1]
        rows = s.numel() // L if L else 0
        if torch.is_tensor(tau):
            tv = tau.detach().reshape(-1).to(device=s.device, dtype=torch.float32).contiguous()
        else:
            tv = torch.full((1,), float(tau), dtype=torch.float32, device=s.device)
        if tv.numel() == 1:
            rows_per_tau = 1
        elif s.dim() == 4 and tv.numel() == s.shape[1]:
            rows_per_tau = s.shape[2]          # [B, H, Lq, Lk] with a per-head tau
        else:
            raise ValueError(f"tau with {tv.numel()} values does not match scores of shape {tuple(s.shape)}")
        attn = torch.empty_like(s)
        rc = C.lib().tau_opus_fixed_fwd(s.data_ptr(), rows, L, L, tv.data_ptr(), tv.numel(), rows_per_tau, sid,
                                        attn.data_ptr(), C.stream_ptr(s.device))
        C.check("tau_opus_fixed_fwd", rc)
        ctx.save_for_backward(s, tv)
        ctx.meta = (sid, rows, L, rows_per_tau)
        return attn

    @staticmethod
    def backward(ctx, grad_attn):
        from . import _capi as C
        s, tv = ctx.saved_tensors
        sid, rows, L, rows_per_tau = ctx.meta
        g = grad_attn.float().contiguous()
        ds = torch.empty_like(s)
        rc = C.lib().tau_opus_fixed_bwd(s.data_ptr(), g.data_ptr(), rows, L, L, tv.data_ptr(), tv.numel(),
                                        rows_per_tau, sid, ds.data_ptr(), C.stream_ptr(s.device))
        C.check("tau_opus_fixed_bwd", rc)
        return ds, None, None


def _make_fixed_stau_forward():
    """transformers' eager attention with the fixed-tau weights
    (echo/patch_whisper_stau.py:190-214): scores = q k^T * scaling (+ mask) as
    the projections' dtype computes them, the weights in fp32 from the module's
    _stau_tau / _stau_sigma, dropout, then the weights (cast back) times v.
    Returns the weights as well, as the reference does."""
    def stau_eager_attention_forward(module, query, key, value, attention_mask, scaling=None,
                                     dropout=0.0, **kwargs):
        if scaling is None:
            scaling = query.size(-1) ** -0.5
        scores = torch.matmul(query, key.transpose(2, 3)) * scaling
        if attention_mask is not None:
            scores = scores + attention_mask
        tau = getattr(module, "_stau_tau", None)
        tau = 1.0 if tau is None else tau.to(scores.device)
        sigma_name = getattr(module, "_stau_sigma", "softplus")
        weights = STauOpusMaxStableFn.apply(scores.float(), tau, sigma_name)
        weights = F.dropout(weights, p=dropout, training=module.training)
        out = torch.matmul(weights.to(value.dtype), value)
        return out.transpose(1, 2).contiguous(), weights.to(value.dtype)
    return stau_eager_attention_forward


def apply_fixed_stau(model, tau_source, sigma_name="softplus"):
    """Give every WhisperAttention a fixed per-head tau
    (echo/patch_whisper_stau.py:279-322). tau_source: a number (every head), a
    dict {"encoder_self": {layer: [H taus]}, ...}, or the path of a tau* JSON;
    sigma_name: one name or a dict per site kind. Heads without an entry get
    tau = 1. Sets module._stau_tau ((1, H, 1, 1) fp32) and module._stau_sigma,
    and swaps transformers' eager attention for the fixed-tau one."""
    if isinstance(tau_source, (str, Path)):
        tau_dict = load_tau_dict(tau_source)
    elif isinstance(tau_source, dict):
        tau_dict = tau_source
    elif isinstance(tau_source, (float, int)):
        tau_dict = None
        scalar_tau = float(tau_source)
    else:
        raise TypeError(f"Unsupported tau_source type: {type(tau_source)}")
    sigma_map = _sigma_map(sigma_name)
    for name, module in model.named_modules():
        if module.__class__.__name__ != "WhisperAttention":
            continue
        h = module.num_heads
        kind = _classify_attn(name, module)
        if tau_dict is not None:
            tau_list = tau_dict.get(kind, {}).get(_parse_layer_idx(name), [1.0] * h)
            tau_tensor = torch.tensor(tau_list, dtype=torch.float32).view(1, h, 1, 1)
        else:
            tau_tensor = torch.full((1, h, 1, 1), scalar_tau, dtype=torch.float32)
        module._stau_tau = tau_tensor
        module._stau_sigma = sigma_map[kind]
        module.__dict__.pop("forward", None)      # transformers' own forward calls the eager function
    whisper_module.eager_attention_forward = _make_fixed_stau_forward()


def _make_learnable_stau_forward():
    def stau_eager_attention_forward(module, query, key, value, attention_mask, scaling=None,
                                     dropout=0.0, **kwargs):
        opus = getattr(module, "_stau_opus", None)
        if opus is None:
            raise RuntimeError("Module has no _stau_opus. Call apply_learnable_stau first.")
        if scaling is None:
            scaling = query.size(-1) ** -0.5
        out = opus(query, key, value, attn_mask=attention_mask, scale=scaling)
        out = F.dropout(out, p=dropout, training=module.training)
        # the operator's output is a [B,H,L,D] view of a [B,L,H,D] buffer: no copy here
        return out.transpose(1, 2).contiguous(), None
    return stau_eager_attention_forward


def stau_whisper_attention_forward(self, hidden_states, key_value_states=None, past_key_values=None,
                                   attention_mask=None, output_attentions=False, **kwargs):
    """WhisperAttention.forward for a module with `_stau_opus`, without layout
    copies: q, k and v stay [B,L,H,D] projections viewed as [B,H,L,D], the
    operator writes its output as a [B,H,L,D] view of a [B,L,H,D] buffer, and
    out_proj reads that buffer directly. Same values as transformers' forward
    followed by the operator (its q * scaling with scaling = 2^-3 is exact in
    bf16). With a KV cache it is transformers' forward unchanged."""
    if past_key_values is not None:
        return type(self).forward(self, hidden_states, key_value_states=key_value_states,
                                  past_key_values=past_key_values, attention_mask=attention_mask,
                                  output_attentions=output_attentions, **kwargs)
    bsz, tgt_len = hidden_states.shape[:-1]
    src = key_value_states if key_value_states is not None else hidden_states
    if getattr(self, "_stau_fused_qkv", False):
        q, k, v = _fused_projections(self, hidden_states, key_value_states)
    else:
        q = self.q_proj(hidden_states)
        k = self.k_proj(src)
        v = self.v_proj(src)
    q = q.view(bsz, tgt_len, -1, self.head_dim).transpose(1, 2)
    k = k.view(bsz, -1, self.num_heads, self.head_dim).transpose(1, 2)
    v = v.view(bsz, -1, self.num_heads, self.head_dim).transpose(1, 2)
    out = self._stau_opus(q, k, v, attn_mask=attention_mask, scale=self.scaling)
    out = F.dropout(out, p=self.dropout if self.training else 0.0, training=self.training)
    out = out.transpose(1, 2).reshape(bsz, tgt_len, -1)
    return self.out_proj(out), None


def _proj_bias(lin, like):
    return lin.bias if lin.bias is not None else torch.zeros(lin.out_features, dtype=like.dtype, device=like.device)


def _fused_projections(self, hidden_states, key_value_states):
    """q, k, v from one GEMM over the concatenated weights (k and v only for
    cross-attention, whose q reads the decoder stream): the shared input is
    cast to bf16 once under autocast, and its gradient comes back as one
    tensor instead of three cast back to fp32 and added. Parameters stay
    separate (same state_dict); the outputs are strided views of one buffer."""
    from .linear import linear
    wq, wk, wv = self.q_proj.weight, self.k_proj.weight, self.v_proj.weight
    if key_value_states is None:
        w = torch.cat([wq, wk, wv], 0)
        b = torch.cat([_proj_bias(self.q_proj, wq), _proj_bias(self.k_proj, wq), _proj_bias(self.v_proj, wq)])
        return linear(hidden_states, w, b).split([wq.shape[0], wk.shape[0], wv.shape[0]], dim=-1)
    q = self.q_proj(hidden_states)
    w = torch.cat([wk, wv], 0)
    b = torch.cat([_proj_bias(self.k_proj, wk), _proj_bias(self.v_proj, wk)])
    k, v = linear(key_value_states, w, b).split([wk.shape[0], wv.shape[0]], dim=-1)
    return q, k, v


def _sigma_map(sigma_name):
    if isinstance(sigma_name, str):
        return {k: sigma_name for k in SITE_KINDS}
    if isinstance(sigma_name, dict):
        return {k: sigma_name.get(k, "softplus") for k in SITE_KINDS}
    raise TypeError(f"Unsupported sigma_name type: {type(sigma_name)}")


def apply_learnable_stau(model, tau_init=1.0, alpha_init: float = 1.0, sigma_name="softplus",
                         default_tau_json=None, use_flash: bool = False,
                         assume_causal_decoder: bool = False, fuse_qkv: bool = False):
    """Attach a learnable tau-opus operator to every WhisperAttention module."""
    if isinstance(tau_init, (str, Path)):
        if str(tau_init).lower() == "tau_star":
            if default_tau_json is None:
                raise ValueError("tau_init='tau_star' needs default_tau_json")
            tau_dict = load_tau_dict(default_tau_json)
        else:
            tau_dict = load_tau_dict(tau_init)
    elif isinstance(tau_init, dict):
        tau_dict = tau_init
    elif isinstance(tau_init, (float, int)):
        tau_dict = None
        scalar_tau = float(tau_init)
    else:
        raise TypeError(f"Unsupported tau_init type: {type(tau_init)}")
    sigma_map = _sigma_map(sigma_name)

    n_attached = 0
    for name, module in model.named_modules():
        if module.__class__.__name__ != "WhisperAttention":
            continue
        h = module.num_heads
        kind = _classify_attn(name, module)
        opus = STauOpusLearnable(h, sigma_name=sigma_map[kind]).to(next(module.parameters()).dtype)
        opus = opus.to(next(module.parameters()).device)
        opus.log_alpha.data.fill_(math.log(alpha_init))
        if tau_dict is not None:
            tau_list = tau_dict.get(kind, {}).get(_parse_layer_idx(name), [1.0] * h)
        else:
            tau_list = [scalar_tau] * h
        tau_list = [max(1.0, float(t)) for t in tau_list[:h]]
        opus.log_tau.data = torch.tensor([_log_tau_for_init(t) for t in tau_list],
                                         dtype=opus.log_tau.dtype, device=opus.log_tau.device)
        opus.assume_causal = bool(assume_causal_decoder and kind == "decoder_self")
        module._stau_opus = opus
        module._stau_fused_qkv = bool(fuse_qkv)
        module.forward = types.MethodType(stau_whisper_attention_forward, module)
        n_attached += 1
    print(f"[tau-opus] Attached fused B200 STauOpus to {n_attached} attention modules")
    print(f"  sigma config: {sigma_map}")
    whisper_module.eager_attention_forward = _make_learnable_stau_forward()
    return n_attached


def remove_stau(model=None):
    """Restore transformers' eager attention and clear the attached operators."""
    whisper_module.eager_attention_forward = _ORIGINAL_EAGER_FORWARD
    if model is not None:
        for module in model.modules():
            if module.__class__.__name__ == "WhisperAttention":
                module._stau_tau = None
                if "_stau_opus" in module._modules:
                    del module._modules["_stau_opus"]
                module.__dict__.pop("forward", None)
