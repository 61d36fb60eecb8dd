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


# The module names the reference's own code imports its operators under
# (echo/patch_whisper_stau.py:20-29, echo/patch_whisper_sparse_grad.py:26-31,
# echo/train_echo_opus1.py:39-43, echo/predict.py:58-59).
OPERATOR_MODULES = ("stau_opus_operator", "stau_opus_flash_v2", "triton_wta")
PATCH_MODULES = ("patch_whisper_stau", "patch_whisper_sparse_grad")


def install_reference_aliases(patch_modules: bool = False) -> dict:
    """Register this package's modules in ``sys.modules`` under the top-level
    names the reference imports, so that its unmodified files bind the B200
    kernels.

    The reference's patch modules put their own directory first on
    ``sys.path`` and then run ``from stau_opus_operator import ...``,
    ``from stau_opus_flash_v2 import ...`` and ``from triton_wta import ...``
    (echo/patch_whisper_stau.py:20-29, echo/patch_whisper_sparse_grad.py:26-31).
    Python resolves an import from ``sys.modules`` before it searches the
    path, so once this has run those statements bind
    ``tau_dxb_b200.stau_opus_operator`` (and the other two) whatever the path
    order. Call it before the reference's patch modules are imported.

    patch_modules=True also registers ``patch_whisper_stau`` and
    ``patch_whisper_sparse_grad``, so that the reference's training and
    prediction scripts (echo/train_echo_opus1.py:39-43, echo/predict.py:58-59)
    bind this package's patch modules as well: their decoder sparse-grad path
    and learnable k then run on the device kernels too.

    A name that is already bound to a different module raises RuntimeError
    (the reference's own module was imported first, and its functions would
    keep the objects they bound). Returns {name: module}.
    """
    import importlib
    import sys
    names = OPERATOR_MODULES + (PATCH_MODULES if patch_modules else ())
    mods = {n: importlib.import_module(f"{__name__}.{n}") for n in names}
    for n, m in mods.items():
        cur = sys.modules.get(n)
        if cur is not None and cur is not m:
            raise RuntimeError(
                f"tau_dxb_b200.install_reference_aliases: module {n!r} is already imported from "
                f"{getattr(cur, '__file__', '?')}; call this before the reference's modules are imported")
    for n, m in mods.items():
        sys.modules[n] = m
    return mods
