"""Reference-named module: the drop-in for echo/stau_opus_flash_v2.py.

STauOpusFlashV2Function is the same fused operator as
STauOpusAttentionFunction (the reference's Triton version of it computes
wrong dQ/dK at scale != 1, wrong dlog_tau/dlog_alpha beyond 64 keys and
ignores the mask; this one does not). `_HAS_TRITON` keeps the name the
reference's patch module imports (echo/patch_whisper_stau.py:25); here it
means "the fused kernels are available".
"""
import torch.nn as nn
import torch

from . import _capi as C
from .attention import STauOpusAttentionFunction

STauOpusFlashV2Function = STauOpusAttentionFunction
_SIGMA_NAME_TO_ID = dict(C.SIGMA_IDS)


def _fused_available() -> bool:
    try:
        C.lib()
        return True
    except ImportError:
        return False


_HAS_TRITON = _fused_available()


class STauOpusFlashV2Module(nn.Module):
    """echo/stau_opus_flash_v2.py:558-570."""

    def __init__(self, n_heads, sigma_name="softplus"):
        super().__init__()
        self.log_tau = nn.Parameter(torch.zeros(n_heads))
        self.log_alpha = nn.Parameter(torch.zeros(n_heads))
        self.sigma_name = sigma_name

    def forward(self, Q, K, V, attn_mask=None, scale=None):
        out, _ = STauOpusFlashV2Function.apply(Q, K, V, self.log_tau, self.log_alpha,
                                               self.sigma_name, attn_mask, scale)
        return out


def get_best_stau_function():
    """echo/stau_opus_flash_v2.py:577-583 -- always the fused B200 operator."""
    return STauOpusFlashV2Function
