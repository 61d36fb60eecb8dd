"""tau_attn_bwd_noalloc: the attention backward for callers that cannot
allocate device memory (hosts that own all device memory through their own
pool or budget, FFI callers without an allocator). Its scratch is a fixed
16 MiB array inside the library.

The file name sorts last so that a `-x` run reaches it only after every other
test; it also passes alone in a fresh process (the first call sets up the
array's address on the device).
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import rel_err

pytestmark = pytest.mark.gpu
DEV = "cuda"
TOL_BF16 = 2e-2


def _problem(seed=3, B=2, H=4, Lq=300, Lk=260):
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(seed)
    mk = lambda L: torch.randn(B, L, H, 64, generator=g).to(torch.bfloat16).to(DEV).transpose(1, 2)
    q, k, v, do = mk(Lq), mk(Lk), mk(Lk), mk(Lq)
    lt = torch.randn(H, generator=g) * 0.5
    tau = (F.softplus(lt) + 1).float().to(DEV)
    alpha = torch.ones(H, device=DEV)
    return q, k, v, do, tau, alpha


def _forward(C, q, k, v, tau, alpha):
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    out = torch.empty(B, Lq, H, D, dtype=q.dtype, device=DEV).transpose(1, 2)
    m = torch.empty(B, H, Lq, device=DEV)
    z = torch.empty_like(m)
    a = torch.empty(B, H, Lq, dtype=torch.int32, device=DEV)
    rc = C.lib().tau_attn_fwd(
        q.data_ptr(), C.strides4(q), k.data_ptr(), C.strides4(k), v.data_ptr(), C.strides4(v),
        C.BF16, B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(), C.SIGMA_IDS["softplus"], 0.125,
        None, 0, None, 0, out.data_ptr(), C.strides4(out), m.data_ptr(), z.data_ptr(),
        a.data_ptr(), C.PATH_AUTO, C.stream_ptr())
    C.check("tau_attn_fwd", rc)
    return out, m, z, a


def _grads(q, k, v):
    e = lambda t: torch.empty_like(t)
    return e(q), e(k), e(v), torch.empty(q.shape[1], device=DEV), torch.empty(q.shape[1], device=DEV)


def _backward(C, fn, q, k, v, out, do, tau, alpha, m, z, a, workspace=None):
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    dq, dk, dv, dtau, dalpha = _grads(q, k, v)
    args = [q.data_ptr(), C.strides4(q), k.data_ptr(), C.strides4(k), v.data_ptr(), C.strides4(v),
            out.data_ptr(), C.strides4(out), do.data_ptr(), C.strides4(do),
            C.BF16, B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(), C.SIGMA_IDS["softplus"],
            0.125, None, 0, None, 0, m.data_ptr(), z.data_ptr(), a.data_ptr(),
            dq.data_ptr(), C.strides4(dq), dk.data_ptr(), C.strides4(dk), dv.data_ptr(),
            C.strides4(dv), dtau.data_ptr(), dalpha.data_ptr()]
    if workspace is not None:
        args += [workspace.data_ptr(), workspace.numel()]
    args += [C.PATH_AUTO, C.stream_ptr()]
    rc = fn(*args)
    C.check(fn.__name__, rc)
    torch.cuda.synchronize()
    return [t.float().cpu().numpy() for t in (dq, dk, dv, dtau, dalpha)]


def test_noalloc_backward_matches_workspace_backward_twice():
    from tau_dxb_b200 import _capi as C
    lib = C.lib()
    q, k, v, do, tau, alpha = _problem()
    out, m, z, a = _forward(C, q, k, v, tau, alpha)
    B, H, Lq, D = q.shape
    ws = torch.empty(lib.tau_attn_bwd_workspace_bytes(B, H, Lq, k.shape[2], D), dtype=torch.uint8,
                     device=DEV)
    ref = _backward(C, lib.tau_attn_bwd, q, k, v, out, do, tau, alpha, m, z, a, workspace=ws)
    for call in range(2):   # the shared array keeps the previous call's contents
        got = _backward(C, lib.tau_attn_bwd_noalloc, q, k, v, out, do, tau, alpha, m, z, a)
        for name, x, y in zip(["dQ", "dK", "dV", "dtau", "dalpha"], got, ref):
            assert rel_err(x, y) < TOL_BF16, (call, name, rel_err(x, y))
    assert lib.tau_dxb_device_error(1) == 0


def test_noalloc_rejects_problems_beyond_its_scratch():
    from tau_dxb_b200 import _capi as C
    lib = C.lib()
    # B*H*(Lq+Lk)*D*4 bytes of accumulators alone exceed 16 MiB here
    B, H, Lq, Lk, D = 16, 12, 1500, 1500, 64
    assert lib.tau_attn_bwd_workspace_bytes(B, H, Lq, Lk, D) > (16 << 20)
    s = (ctypes.c_int64 * 4)(0, 0, 0, 1)
    t = torch.empty(H, device=DEV)
    rc = lib.tau_attn_bwd_noalloc(
        t.data_ptr(), s, t.data_ptr(), s, t.data_ptr(), s, t.data_ptr(), s, t.data_ptr(), s,
        C.BF16, B, H, Lq, Lk, D, t.data_ptr(), t.data_ptr(), 0, 0.125, None, 0, None, 0,
        t.data_ptr(), t.data_ptr(), t.data_ptr(), t.data_ptr(), s, t.data_ptr(), s, t.data_ptr(),
        s, t.data_ptr(), t.data_ptr(), C.PATH_AUTO, C.stream_ptr())
    assert rc == C.ERR_WORKSPACE
    assert "16 MiB" in C.last_error()
