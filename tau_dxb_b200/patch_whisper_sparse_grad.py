"""SparseGrad / WTA top-k sparsity for the Whisper FFN (B200 kernels).

Same public surface as the reference module echo/patch_whisper_sparse_grad.py:
  SparseGradWTA_Function, WTA_Activation_Function           (:38-82)
  WinCountTracker                                           (:89-121)
  LearnableKRatio                                           (:139-164)
  apply_sparse_grad_wta(model, k_ratio, target, mode, encoder_mode, decoder_mode,
                        encoder_k_ratio, decoder_k_ratio, track_wins,
                        learnable_k, init_k_ratio)          (:233-330)
  set_sparse_grad_k_ratio, set_win_collection, get_win_tracker,
  prune_low_winners, unfreeze_all, reset_win_counts,
  get_sparsity_loss, remove_sparse_grad                     (:333-431)

Modes per layer type: "sparse_grad" (identity forward, top-k gradient mask),
"wta_activation" (top-k forward, straight-through backward), "none".

Differences from the reference, by design:
  * the learnable k is computed on the device (wta_k_from_logits) and read by
    the kernel, so the per-layer `.item()` host sync of the reference
    (echo/patch_whisper_sparse_grad.py:160,209) is gone; LearnableKRatio.get_k
    still returns the same Python int for callers that want it;
  * win counts come out of the WTA kernel itself (per-column counts of the
    kept positions, accumulated in an int32 device buffer) instead of an extra
    x.topk + .cpu() copy per layer (:218-221). On rows with ties at the
    threshold the kernel counts every kept tied element, the reference counts
    exactly k.
"""
from __future__ import annotations

import math
from collections import defaultdict
from typing import Dict, Optional

import torch
import torch.nn as nn

from .wta import (THRESHOLD, SparseGradWTA_Function, WTA_Activation_Function,  # noqa: F401
                  has_fused_kernels, k_from_logits, wta_backward, wta_backward_gelu, wta_fused_forward,
                  wta_select)

# The reference module's names for its fused WTA entry point and whether it
# loaded (echo/patch_whisper_sparse_grad.py:26-31); here the CUDA kernels.
_triton_wta_forward = wta_fused_forward
_HAS_TRITON_WTA = has_fused_kernels()


class _WTAFusedCounting(torch.autograd.Function):
    """Threshold WTA (the reference's CUDA semantics) whose kernel also adds
    the per-column win counts into `win` (int32 [d]) when given."""

    @staticmethod
    def forward(ctx, x, k, win):
        y, bits = wta_select(x, k, THRESHOLD, write_y=True, win_counts=win)
        ctx.save_for_backward(bits)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        (bits,) = ctx.saved_tensors
        return wta_backward(grad_y, bits), None, None


class _WTAGeluFusedCounting(torch.autograd.Function):
    """GELU then threshold WTA: x is the fc1 output (the GELU's input), y =
    WTA(gelu(x)) with the win counts; the backward applies the mask and the
    GELU gradient in one kernel (132 us against 51 + 114 us for the two
    backward passes at 24000 x 3072). The forward keeps torch's GELU kernel:
    the WTA kernel's GELU-input mode gives the same bits but measured slower
    (199 us against 85 + 71 us), the erf being issue-bound in a warp-per-row
    kernel."""

    @staticmethod
    def forward(ctx, x, k, win):
        y, bits = wta_select(torch.nn.functional.gelu(x), k, THRESHOLD, write_y=True, win_counts=win)
        ctx.save_for_backward(x, bits)
        return y

    @staticmethod
    def backward(ctx, grad_y):
        x, bits = ctx.saved_tensors
        return wta_backward_gelu(grad_y, x, bits), None, None


class WinCountTracker:
    """Per-FFN-neuron win counts (echo/patch_whisper_sparse_grad.py:89-121).

    Counts live on the device as int32 and are only brought to the host by
    win_rate() / prune_low_winners()."""

    def __init__(self):
        self.win_counts: Dict[str, torch.Tensor] = {}
        self.total_steps: Dict[str, int] = defaultdict(int)

    def buffer(self, module_name: str, d_ff: int, device) -> torch.Tensor:
        buf = self.win_counts.get(module_name)
        if buf is None or buf.device != torch.device(device) or buf.dtype != torch.int32:
            buf = torch.zeros(d_ff, dtype=torch.int32, device=device)
            self.win_counts[module_name] = buf
        return buf

    def record(self, module_name: str, topk_idx: torch.Tensor, d_ff: int):
        """Reference-compatible: add the wins of explicit top-k indices."""
        buf = self.buffer(module_name, d_ff, topk_idx.device)
        flat = topk_idx.reshape(-1).long()
        buf.scatter_add_(0, flat, torch.ones_like(flat, dtype=torch.int32))
        self.total_steps[module_name] += 1

    def step(self, module_name: str):
        self.total_steps[module_name] += 1

    def win_rate(self, module_name: str) -> Optional[torch.Tensor]:
        if module_name not in self.win_counts:
            return None
        counts = self.win_counts[module_name].float()
        return counts / counts.mean().clamp(min=1.0)

    def reset(self):
        self.win_counts.clear()
        self.total_steps.clear()


_HOOK_HANDLES = []
_K_RATIOS: Dict[str, float] = {"encoder": 0.5, "decoder": 0.5}
_MODES: Dict[str, str] = {"encoder": "sparse_grad", "decoder": "sparse_grad"}
_TRACKER: Optional[WinCountTracker] = None
_GRAD_MASKS: Dict[str, torch.Tensor] = {}
_COLLECT_WINS = False
_LEARNABLE_K: Dict[str, "LearnableKRatio"] = {}


class LearnableKRatio(nn.Module):
    """Per-layer learnable k ratio = sigmoid(logit_k) (echo/patch_whisper_sparse_grad.py:139-164)."""

    def __init__(self, init_k_ratio: float = 0.4):
        super().__init__()
        self.logit_k = nn.Parameter(torch.tensor(0.0))
        self._reset(init_k_ratio)

    def _reset(self, init_k_ratio: float):
        init_k_ratio = max(0.1, min(0.9, init_k_ratio))
        nn.init.constant_(self.logit_k, float(math.log(init_k_ratio / (1.0 - init_k_ratio + 1e-8))))

    @property
    def k_ratio(self) -> float:
        return torch.sigmoid(self.logit_k).item()

    def get_k(self, d_ff: int) -> int:
        k = int(round(torch.sigmoid(self.logit_k).item() * d_ff))
        return max(1, min(d_ff, k))

    def get_k_device(self, d_ff: int) -> torch.Tensor:
        """The same k as get_k, as a 1-element int32 device tensor (no host sync)."""
        return k_from_logits(self.logit_k.detach().reshape(1), d_ff)

    def extra_repr(self) -> str:
        return f"logit_k={float(self.logit_k.detach()):.4f}"


def masked_grad(grad: torch.Tensor, keep: torch.Tensor, axis: int) -> torch.Tensor:
    """grad * keep along `axis` (0: rows, 1: columns) as the reference's hooks
    compute it (echo/patch_whisper_sparse_grad.py:167-194). CUDA gradients run
    on tau_grad_mask (one pass, the bool keep mask read as bytes); host
    tensors use torch."""
    if not grad.is_cuda:
        m = keep.to(grad.device, grad.dtype)
        return grad * (m.unsqueeze(-1) if axis == 0 and grad.dim() > 1 else m)
    from . import _capi as C
    g = grad.contiguous()
    k = keep.to(device=g.device, dtype=torch.bool).contiguous()
    rows = g.shape[0] if g.dim() > 1 else 1
    cols = g.numel() // max(rows, 1) if g.dim() > 1 else g.numel()
    if g.dim() == 1:       # a bias: one row, keep along its columns
        axis = 1
    out = torch.empty_like(g)
    rc = C.lib().tau_grad_mask(g.data_ptr(), C.dtype_code(g.dtype), rows, cols, k.data_ptr(), axis,
                               out.data_ptr(), C.stream_ptr(g.device))
    C.check("tau_grad_mask", rc)
    return out


def _make_fc1_weight_grad_hook(module_name: str):
    def hook(grad):
        m = _GRAD_MASKS.get(module_name)
        return grad if m is None else masked_grad(grad, m, 0)     # fc1.weight [d_ff, d_model]: rows
    return hook


def _make_fc1_bias_grad_hook(module_name: str):
    def hook(grad):
        m = _GRAD_MASKS.get(module_name)
        return grad if m is None else masked_grad(grad, m, 1)     # fc1.bias [d_ff]
    return hook


def _make_fc2_weight_grad_hook(module_name: str):
    def hook(grad):
        m = _GRAD_MASKS.get(module_name)
        return grad if m is None else masked_grad(grad, m, 1)     # fc2.weight [d_model, d_ff]: columns
    return hook


def _layer_k(module_name: str, layer_type: str, d_ff: int, x: torch.Tensor):
    lk = _LEARNABLE_K.get(module_name)
    if lk is not None:
        return lk.get_k_device(d_ff) if x.is_cuda else lk.get_k(d_ff)
    return max(1, int(d_ff * _K_RATIOS.get(layer_type, 0.3)))


def _make_fc2_pre_hook(module_name: str, layer_type: str):
    """fc2 forward-pre-hook (echo/patch_whisper_sparse_grad.py:197-230): only
    when the input requires grad (inert at inference)."""
    def hook(module, input_):
        x = input_[0]
        # fuse_gelu_into_wta moved the layer's GELU here: x is then the fc1 output
        gelu_in = getattr(module, "_tau_dxb_gelu_in", False)
        mode = _MODES.get(layer_type, "sparse_grad")
        if not x.requires_grad or mode == "none":
            return (torch.nn.functional.gelu(x),) + tuple(input_[1:]) if gelu_in else input_
        d_ff = x.shape[-1]
        if gelu_in and mode != "wta_activation":
            x = torch.nn.functional.gelu(x)
            gelu_in = False
        k = _layer_k(module_name, layer_type, d_ff, x)
        if mode == "sparse_grad":
            x = SparseGradWTA_Function.apply(x, k)
        elif mode == "wta_activation":
            win = None
            if _COLLECT_WINS and _TRACKER is not None:
                win = _TRACKER.buffer(module_name, d_ff, x.device)
                _TRACKER.step(module_name)
            x = (_WTAGeluFusedCounting if gelu_in else _WTAFusedCounting).apply(x, k, win)
        return (x,) + tuple(input_[1:])
    return hook


def apply_sparse_grad_wta(model, k_ratio: float = 0.3, target: str = "encoder+decoder",
                          mode: str = "sparse_grad", encoder_mode: Optional[str] = None,
                          decoder_mode: Optional[str] = None,
                          encoder_k_ratio: Optional[float] = None,
                          decoder_k_ratio: Optional[float] = None, track_wins: bool = False,
                          learnable_k: bool = False, init_k_ratio: float = 0.4):
    """Install the fc2 pre-hooks (and fc1/fc2 gradient-mask hooks) on Whisper's FFNs."""
    global _K_RATIOS, _MODES, _TRACKER, _COLLECT_WINS, _LEARNABLE_K
    enc_mode = encoder_mode or mode
    dec_mode = decoder_mode or mode
    enc_k = encoder_k_ratio or k_ratio
    dec_k = decoder_k_ratio or k_ratio
    _K_RATIOS = {"encoder": enc_k, "decoder": dec_k}
    _MODES = {"encoder": enc_mode, "decoder": dec_mode}
    if track_wins:
        _TRACKER = WinCountTracker()
        _COLLECT_WINS = True
    else:
        _COLLECT_WINS = False
    remove_sparse_grad()
    _LEARNABLE_K = {}
    want = {"WhisperEncoderLayer": ("encoder", target in ("encoder", "encoder+decoder")),
            "WhisperDecoderLayer": ("decoder", target in ("decoder", "encoder+decoder"))}
    counts = {"encoder": 0, "decoder": 0}
    for name, module in model.named_modules():
        kind, on = want.get(module.__class__.__name__, (None, False))
        if not on or not hasattr(module, "fc2"):
            continue
        if learnable_k:
            lk = LearnableKRatio(init_k_ratio=init_k_ratio).to(module.fc2.weight.device)
            module.register_module("_learnable_k", lk)
            _LEARNABLE_K[name] = lk
        _HOOK_HANDLES.append(module.fc2.register_forward_pre_hook(_make_fc2_pre_hook(name, kind)))
        if not getattr(module, "_grad_hook_installed", False):
            module.fc1.weight.register_hook(_make_fc1_weight_grad_hook(name))
            if module.fc1.bias is not None:
                module.fc1.bias.register_hook(_make_fc1_bias_grad_hook(name))
            module.fc2.weight.register_hook(_make_fc2_weight_grad_hook(name))
            module._grad_hook_installed = True
        counts[kind] += 1
    print(f"[SparseGrad] encoder: {counts['encoder']} layers, mode={enc_mode}, k={enc_k}")
    print(f"[SparseGrad] decoder: {counts['decoder']} layers, mode={dec_mode}, k={dec_k}")
    if learnable_k:
        print(f"[SparseGrad] Learnable k_ratio ENABLED (init={init_k_ratio})")
    if track_wins:
        print("[SparseGrad] Win count tracking ENABLED")
    return counts


def set_sparse_grad_k_ratio(model, k_ratio: float, layer_type: Optional[str] = None):
    global _K_RATIOS
    if layer_type:
        _K_RATIOS[layer_type] = float(k_ratio)
    else:
        _K_RATIOS = {"encoder": float(k_ratio), "decoder": float(k_ratio)}


def set_win_collection(enabled: bool):
    global _COLLECT_WINS
    _COLLECT_WINS = enabled


def get_win_tracker() -> Optional[WinCountTracker]:
    return _TRACKER


def prune_low_winners(model, threshold: float = 0.05):
    """Soft prune: freeze the gradients of neurons whose win rate is below
    `threshold` (weights kept; echo/patch_whisper_sparse_grad.py:352-395)."""
    global _GRAD_MASKS
    if _TRACKER is None:
        print("[prune] No win tracker, skipping")
        return 0
    total_pruned = total = 0
    for name, module in model.named_modules():
        if module.__class__.__name__ not in ("WhisperEncoderLayer", "WhisperDecoderLayer"):
            continue
        rate = _TRACKER.win_rate(name)
        if rate is None:
            continue
        active = rate >= threshold
        _GRAD_MASKS[name] = active.to(module.fc1.weight.device)
        total_pruned += int((~active).sum().item())
        total += rate.shape[0]
    pct = total_pruned / max(1, total) * 100
    print(f"[prune] Soft-pruned {total_pruned}/{total} neurons ({pct:.1f}%) "
          "-- gradients frozen, weights preserved")
    return total_pruned


def unfreeze_all():
    global _GRAD_MASKS
    n = len(_GRAD_MASKS)
    _GRAD_MASKS = {}
    print(f"[prune] Cleared {n} grad masks -- all neurons back to training")


def reset_win_counts():
    if _TRACKER is not None:
        _TRACKER.reset()


def get_sparsity_loss() -> torch.Tensor:
    """mean over layers of sigmoid(logit_k) (echo/patch_whisper_sparse_grad.py:413-422)."""
    if not _LEARNABLE_K:
        return torch.tensor(0.0, requires_grad=False)
    return torch.stack([torch.sigmoid(lk.logit_k) for lk in _LEARNABLE_K.values()]).mean()


def remove_sparse_grad(model=None):
    global _HOOK_HANDLES, _GRAD_MASKS
    for h in _HOOK_HANDLES:
        h.remove()
    _HOOK_HANDLES = []
    _GRAD_MASKS = {}


def fuse_gelu_into_wta(model) -> int:
    """Move the GELU of every encoder MLP whose fc2 input goes through the
    wta_activation hook into that hook's kernel: the layer's activation_fn
    becomes the identity and the hook selects on gelu(fc1 output) directly,
    with the GELU gradient fused into the mask backward. Values are those of
    GELU followed by WTA (the kernels evaluate GELU as PyTorch's bf16 kernels
    do). Only for layers with the exact-erf GELU, no activation dropout and an
    MLP width the fused kernels take (256 x {3, 4, 6, 8, 12, 16}); returns how
    many layers were fused. unfuse_gelu_from_wta undoes it."""
    n = 0
    for name, m in model.named_modules():
        if m.__class__.__name__ != "WhisperEncoderLayer" or _MODES.get("encoder") != "wta_activation":
            continue
        act = getattr(m, "activation_fn", None)
        exact_gelu = act is not None and act.__class__.__name__ == "GELUActivation" \
            and getattr(act, "act", None) is torch.nn.functional.gelu
        d_ff = getattr(getattr(m, "fc1", None), "out_features", 0)
        fast_width = d_ff % 256 == 0 and d_ff // 256 in (3, 4, 6, 8, 12, 16)   # the kernels' row widths
        if not exact_gelu or not fast_width or getattr(m, "activation_dropout", 0.0) != 0.0:
            continue
        m._tau_dxb_saved_act = act
        m.activation_fn = torch.nn.Identity()
        m.fc2._tau_dxb_gelu_in = True
        n += 1
    return n


def unfuse_gelu_from_wta(model) -> None:
    for m in model.modules():
        if hasattr(m, "_tau_dxb_saved_act"):
            m.activation_fn = m._tau_dxb_saved_act
            del m._tau_dxb_saved_act
            m.fc2._tau_dxb_gelu_in = False

