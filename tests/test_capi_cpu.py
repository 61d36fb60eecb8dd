"""The C-ABI library loads without a GPU and exports every declared symbol;
argument validation answers before any CUDA call."""
import ctypes
import os
import re

import pytest

from conftest import ROOT


def _declared_functions():
    text = open(os.path.join(ROOT, "include", "tau_dxb.h")).read()
    return sorted(set(re.findall(r"TAU_DXB_API\s+[\w\s\*]+?\b(\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def C():
    from tau_dxb_b200 import _capi
    return _capi


def test_header_declares_expected_entry_points():
    names = _declared_functions()
    for n in ("tau_attn_fwd", "tau_attn_bwd", "tau_attn_bwd_workspace_bytes", "wta_fwd",
              "wta_bwd", "wta_k_from_logits", "tau_dxb_strerror", "tau_dxb_last_error",
              "tau_dxb_version", "whisper_log_mel", "tau_star_solve", "tau_star_analytic"):
        assert n in names


def test_library_exports_every_declared_symbol(C):
    lib = C.lib()
    for name in _declared_functions():
        assert hasattr(lib, name), name
        assert name in C.SIGNATURES, f"{name} has no ctypes signature"
    raw = ctypes.CDLL(C.LIB_PATH)
    for name in _declared_functions():
        getattr(raw, name)


def test_version_and_strerror(C):
    lib = C.lib()
    assert lib.tau_dxb_version() >= 100
    assert C.strerror(0) == "ok"
    assert C.strerror(C.ERR_WORKSPACE) == "workspace too small"
    assert C.strerror(12345) == "unknown status"


def test_validation_without_gpu(C):
    lib = C.lib()
    # missing pointers -> invalid argument, before touching CUDA
    assert lib.wta_fwd(None, 1, 4, 3072, 3072, 5, None, 0, None, None, None, None) == C.ERR_INVALID_ARGUMENT
    assert "required" in C.last_error()
    assert lib.wta_bwd(None, 1, None, 4, 3072, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.wta_k_from_logits(None, 3, 3072, None, None) == C.ERR_INVALID_ARGUMENT
    s = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    rc = lib.tau_attn_fwd(None, s, None, s, None, s, 1, 1, 1, 8, 8, 64, None, None, 0, 1.0,
                          None, 0, None, 0, None, s, None, None, None, 0, None)
    assert rc == C.ERR_INVALID_ARGUMENT
    # tau* solver: key count, sigma id and pointers are checked first
    assert lib.tau_star_solve(None, 4, 0, 0, 0, 30, 2.0, 0.1, 10.0, 1e-6, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert lib.tau_star_solve(None, 4, C.TAU_STAR_MAX_KEYS + 1, C.TAU_STAR_MAX_KEYS + 1, 0, 30, 2.0, 0.1,
                              10.0, 1e-6, None, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_star_solve(None, 4, 64, 64, 7, 30, 2.0, 0.1, 10.0, 1e-6, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert lib.tau_star_solve(None, 4, 64, 32, 0, 30, 2.0, 0.1, 10.0, 1e-6, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert lib.tau_star_solve(None, 4, 64, 64, 0, 30, 2.0, 0.1, 10.0, 1e-6, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert "null pointer" in C.last_error()
    assert lib.tau_star_solve(None, 0, 64, 64, 0, 30, 2.0, 0.1, 10.0, 1e-6, None, None, None) == C.OK
    assert lib.tau_star_analytic(None, 4, 64, 64, 9, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_star_analytic(None, 4, 64, 64, 0, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_star_analytic(None, 0, 64, 64, 0, None, None) == C.OK
    assert lib.tau_layer_norm_fwd(None, 8, 100, None, None, 1e-5, None, C.F32, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert lib.tau_layer_norm_fwd(None, 8, 768, None, None, 1e-5, None, C.F32, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert lib.tau_layer_norm_fwd(None, 8, 768, None, None, 1e-5, None, C.F16, None, None, None) == \
        C.ERR_INVALID_ARGUMENT
    assert lib.tau_layer_norm_fwd(None, 0, 768, None, None, 1e-5, None, C.BF16, None, None, None) == C.OK
    assert lib.tau_layer_norm_bwd_workspace_bytes(24000, 768) >= 768 * 8
    assert lib.tau_column_sum(None, C.BF16, 8, 100, None, C.BF16, None, 0, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_column_sum(None, C.F16, 8, 128, None, C.BF16, None, 0, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_column_sum(None, C.BF16, 8, 128, None, C.BF16, None, 0, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_column_sum_workspace_bytes(24000, 3072) >= 3072 * 4
    assert lib.tau_cross_entropy_fwd(None, 4, 100, None, -100, None, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_cross_entropy_fwd(None, 4, 128, None, -100, None, None, None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_cross_entropy_bwd(None, 0, 128, None, -100, None, None, None, None) == C.OK


def test_workspace_size_formula(C):
    lib = C.lib()
    B, H, Lq, Lk, D = 16, 12, 1500, 1500, 64
    n = lib.tau_attn_bwd_workspace_bytes(B, H, Lq, Lk, D)
    up = lambda v: (v + 255) // 256 * 256
    assert n == up(B * H * Lq * D * 4) + up(B * H * Lk * D * 4) + 2 * up(B * H * Lq * 4)


def test_workspace_size_saturates_instead_of_wrapping(C):
    """Shapes whose workspace does not fit a size_t report SIZE_MAX, so no
    workspace (and not the no-allocation array) can look large enough."""
    lib = C.lib()
    size_max = 2 ** 64 - 1
    assert lib.tau_attn_bwd_workspace_bytes(65535, 65535, (1 << 24) - 1, (1 << 24) - 1, 128) == size_max
    assert lib.tau_attn_bwd_workspace_bytes(1 << 40, 1 << 40, 1, 1, 1) == size_max
    s = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    p = ctypes.c_void_p(256)       # never dereferenced: the size check answers first
    rc = lib.tau_attn_bwd_noalloc(p, s, p, s, p, s, p, s, p, s, C.BF16, 65535, 65535, (1 << 24) - 1,
                                  (1 << 24) - 1, 128, p, p, 0, 0.125, None, 0, None, 0, p, p, p, p, s, p,
                                  s, p, s, p, p, C.PATH_AUTO, None)
    assert rc == C.ERR_WORKSPACE and "16 MiB" in C.last_error()


def test_wait_selftest_validates_its_limit(C):
    lib = C.lib()
    st = ctypes.c_int32(0)
    assert lib.tau_dxb_selftest_wait_timeout(0, ctypes.byref(st), None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_dxb_selftest_wait_timeout(11 * 10 ** 9, ctypes.byref(st), None) == C.ERR_INVALID_ARGUMENT
    assert lib.tau_dxb_selftest_wait_timeout(10 ** 6, None, None) == C.ERR_INVALID_ARGUMENT
