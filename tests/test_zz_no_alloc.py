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


def _problem(seed=3, B=2, H=4, Lq=300, Lk=260, dtype=torch.bfloat16):
    import torch.nn.functional as F
    g = torch.Generator().manual_seed(seed)
    mk = lambda L: torch.randn(B, L, H, 64, generator=g).to(dtype).to(DEV).transpose(1, 2)
    q, k, v, do = mk(Lq), mk(Lk), mk(Lk), mk(Lq)
    lt = torch.randn(H, generator=g) * 0.5
    tau = (F.softplus(lt) + 1).float().to(DEV)
    alpha = torch.ones(H, device=DEV)
    return q, k, v, do, tau, alpha


def _forward(C, q, k, v, tau, alpha, causal=0, path=None):
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    out = torch.empty(B, Lq, H, D, dtype=q.dtype, device=DEV).transpose(1, 2)
    m = torch.empty(B, H, Lq, device=DEV)
    z = torch.empty_like(m)
    a = torch.empty(B, H, Lq, dtype=torch.int32, device=DEV)
    rc = C.lib().tau_attn_fwd(
        q.data_ptr(), C.strides4(q), k.data_ptr(), C.strides4(k), v.data_ptr(), C.strides4(v),
        C.dtype_code(q.dtype), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(),
        C.SIGMA_IDS["softplus"], 0.125, None, 0, None, causal, out.data_ptr(), C.strides4(out),
        m.data_ptr(), z.data_ptr(), a.data_ptr(), C.PATH_AUTO if path is None else path, C.stream_ptr())
    C.check("tau_attn_fwd", rc)
    return out, m, z, a


def _grads(q, k, v):
    e = lambda t: torch.empty_like(t)
    return e(q), e(k), e(v), torch.empty(q.shape[1], device=DEV), torch.empty(q.shape[1], device=DEV)


def _backward(C, fn, q, k, v, out, do, tau, alpha, m, z, a, workspace=None, causal=0, path=None):
    B, H, Lq, D = q.shape
    Lk = k.shape[2]
    dq, dk, dv, dtau, dalpha = _grads(q, k, v)
    args = [q.data_ptr(), C.strides4(q), k.data_ptr(), C.strides4(k), v.data_ptr(), C.strides4(v),
            out.data_ptr(), C.strides4(out), do.data_ptr(), C.strides4(do),
            C.dtype_code(q.dtype), B, H, Lq, Lk, D, tau.data_ptr(), alpha.data_ptr(),
            C.SIGMA_IDS["softplus"], 0.125, None, 0, None, causal, m.data_ptr(), z.data_ptr(),
            a.data_ptr(), dq.data_ptr(), C.strides4(dq), dk.data_ptr(), C.strides4(dk), dv.data_ptr(),
            C.strides4(dv), dtau.data_ptr(), dalpha.data_ptr()]
    if workspace is not None:
        args += [workspace.data_ptr(), workspace.numel()]
    args += [C.PATH_AUTO if path is None else path, C.stream_ptr()]
    rc = fn(*args)
    C.check(fn.__name__, rc)
    torch.cuda.synchronize()
    assert C.lib().tau_dxb_device_error(1) == 0
    return [t.float().cpu().numpy() for t in (dq, dk, dv, dtau, dalpha)]


def _reference_backward(C, problem, path=None):
    """The same backward through tau_attn_bwd with a caller-provided workspace."""
    q, k, v, do, tau, alpha = problem
    out, m, z, a = _forward(C, q, k, v, tau, alpha, path=path)
    B, H, Lq, D = q.shape
    ws = torch.empty(C.lib().tau_attn_bwd_workspace_bytes(B, H, Lq, k.shape[2], D), dtype=torch.uint8,
                     device=DEV)
    ref = _backward(C, C.lib().tau_attn_bwd, q, k, v, out, do, tau, alpha, m, z, a, workspace=ws, path=path)
    return (out, m, z, a), ref


def _dirty_the_array(C):
    """A different, larger causal problem through the no-allocation entry point:
    every region of the shared array the next call uses is left holding this
    call's values."""
    q, k, v, do, tau, alpha = _problem(seed=11, B=4, H=6, Lq=700, Lk=900)
    out, m, z, a = _forward(C, q, k, v, tau, alpha, causal=1)
    _backward(C, C.lib().tau_attn_bwd_noalloc, q, k, v, out, do, tau, alpha, m, z, a, causal=1)


def _assert_same_backward(got, ref, exact_dv, label):
    """dV and, on the tensor path, everything but the atomically accumulated
    sums are the same computation: dV bit for bit; dQ and dK (fp32 atomic
    sums cast to the output type) within one rounding step of that type,
    rarely even that; the per-head sums within fp32 summation-order rounding."""
    dq, dk, dv, dtau, dalpha = got
    rq, rk, rv, rtau, ralpha = ref
    if exact_dv:
        assert np.array_equal(dv, rv), label
    else:
        assert rel_err(dv, rv) < 1e-5, label
    for name, x, y in (("dQ", dq, rq), ("dK", dk, rk)):
        step = np.abs(y) * 2.0 ** -7 + 1e-6      # one bf16 rounding step (far looser than fp32's)
        assert np.all(np.abs(x - y) <= step), (label, name, float(np.abs(x - y).max()))
        assert np.mean(x != y) < 1e-3, (label, name, float(np.mean(x != y)))
    for name, x, y in (("dtau", dtau, rtau), ("dalpha", dalpha, ralpha)):
        assert rel_err(x, y) < 1e-5, (label, name, rel_err(x, y))


def test_noalloc_backward_matches_workspace_backward_twice():
    """Two calls in a row on the tensor-core path (bf16), each after the shared
    array was left holding another problem's values, against tau_attn_bwd with
    a caller workspace on the same inputs."""
    from tau_dxb_b200 import _capi as C
    lib = C.lib()
    problem = _problem()
    (out, m, z, a), ref = _reference_backward(C, problem)
    q, k, v, do, tau, alpha = problem
    _dirty_the_array(C)
    for call in range(2):   # the shared array keeps the previous call's contents
        got = _backward(C, lib.tau_attn_bwd_noalloc, q, k, v, out, do, tau, alpha, m, z, a)
        _assert_same_backward(got, ref, True, f"tensor path, call {call}")
    assert lib.tau_dxb_device_error(1) == 0


def test_noalloc_precise_path_fp32():
    """The fp32 precise path (whose prologue clears the array with memsets)
    through the no-allocation entry point, after a tensor-path call."""
    from tau_dxb_b200 import _capi as C
    lib = C.lib()
    problem = _problem(seed=5, B=1, H=3, Lq=130, Lk=200, dtype=torch.float32)
    (out, m, z, a), ref = _reference_backward(C, problem, path=C.PATH_PRECISE)
    q, k, v, do, tau, alpha = problem
    _dirty_the_array(C)
    for call in range(2):
        got = _backward(C, lib.tau_attn_bwd_noalloc, q, k, v, out, do, tau, alpha, m, z, a,
                        path=C.PATH_PRECISE)
        for name, x, y in zip(["dQ", "dK", "dV", "dtau", "dalpha"], got, ref):
            assert rel_err(x, y) < 1e-5, (call, name, rel_err(x, y))


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
