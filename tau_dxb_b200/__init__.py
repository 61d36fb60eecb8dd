"""tau_dxb_b200 -- B200-native (sm_100a) kernels for tau-dxb's training hot paths.

* tau-opus attention (forward + backward): ``attention``; reference-named
  modules ``stau_opus_operator`` and ``stau_opus_flash_v2``.
* WTA top-k sparsity (forward + backward): ``wta``; reference-named module
  ``triton_wta`` (the name the reference's patch module imports).
* Whisper patches: ``patch_whisper_stau``, ``patch_whisper_sparse_grad``.
* Data-parallel Whisper-small train step: ``train``.

All compute runs in libtau_dxb.so (C ABI: include/tau_dxb.h), built in-tree
by ``python -m tau_dxb_b200.build``. CUDA tensors only.
"""
__version__ = "0.1.0"

from . import _capi  # noqa: F401


def library_path() -> str:
    return _capi.LIB_PATH


def load_library():
    """Load libtau_dxb.so now (raises ImportError if it has not been built)."""
    return _capi.lib()
