"""Reference-named module: the drop-in for echo/triton_wta.py.

The reference's patch module imports `wta_fused_forward` from a module of
this name (echo/patch_whisper_sparse_grad.py:27); the implementation is the
CUDA radix-select kernel family in tau_dxb_b200.wta (no Triton involved).
"""
from .wta import (_WTAFusedSTE, has_fused_kernels, wta_fused_forward,  # noqa: F401
                  wta_fused_forward_with_mask)


def has_triton() -> bool:
    """echo/triton_wta.py:164-165: whether the fused kernels are usable."""
    return has_fused_kernels()
