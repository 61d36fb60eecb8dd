"""Generate the golden vectors in this directory by running the REFERENCE.

Run once in a container that has the reference checkout (it reads
echo/stau_opus_operator.py, echo/triton_wta.py,
echo/patch_whisper_sparse_grad.py and the LR lambda of
echo/train_echo_opus1.py from it); the resulting .npz files are committed, so
tests never need the reference at run time.

    python tests/golden/make_golden.py /path/to/reference
    TAU_DXB_GOLDEN_ONLY=lr_table python tests/golden/make_golden.py /path/to/reference   # one table

Every case is seeded; attention inputs and the reference's outputs are
stored in fp32, WTA inputs/outputs as raw bf16 bit patterns (uint16) and
masks as little-endian packed bits.
"""
from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch
import torch.nn.functional as Fnn

HERE = os.path.dirname(os.path.abspath(__file__))


def _ref_path(argv):
    if len(argv) < 2:
        sys.exit("usage: python tests/golden/make_golden.py /path/to/reference-checkout")
    return argv[1]


def attn_cases():
    # (name, sigma, B, H, Lq, Lk, D, scale, mask kind, log_tau spec, seed)
    return [
        ("attn_softplus_l65", "softplus", 1, 2, 65, 65, 64, None, None, "normal", 11),
        ("attn_softplus_l200_s1", "softplus", 1, 2, 200, 200, 64, 1.0, None, "normal", 12),
        ("attn_sigmoid_causal_l70", "sigmoid", 2, 2, 70, 70, 64, 1.0, "causal", "normal", 13),
        ("attn_exp_cross_33x100", "exp", 1, 3, 33, 100, 64, 0.125, None, "normal", 14),
        ("attn_exp_tau1_softmax", "exp", 1, 2, 40, 90, 64, None, None, "tau1", 15),
        ("attn_softplus_alpha_l17", "softplus", 2, 2, 17, 17, 64, None, None, "alpha", 16),
        ("attn_sigmoid_l1", "sigmoid", 1, 2, 1, 1, 64, None, None, "normal", 17),
    ]


def make_attn(ref):
    from stau_opus_operator import STauOpusAttentionFunction as E
    for (name, sg, B, H, Lq, Lk, D, scale, mk, lt_spec, seed) in attn_cases():
        g = torch.Generator().manual_seed(seed)
        Q = torch.randn(B, H, Lq, D, generator=g)
        K = torch.randn(B, H, Lk, D, generator=g)
        V = torch.randn(B, H, Lk, D, generator=g)
        dO = torch.randn(B, H, Lq, D, generator=g)
        log_tau = torch.randn(H, generator=g) * 0.5
        log_alpha = torch.zeros(H)
        if lt_spec == "tau1":
            log_tau = torch.full((H,), -30.0)
        if lt_spec == "alpha":
            log_alpha = torch.randn(H, generator=g) * 0.3
        mask = None
        if mk == "causal":
            mask = torch.full((Lq, Lk), torch.finfo(torch.float32).min).triu(1)[None, None]
        q, k, v = (t.clone().requires_grad_() for t in (Q, K, V))
        lt = log_tau.clone().requires_grad_()
        la = log_alpha.clone().requires_grad_()
        out, _ = E.apply(q, k, v, lt, la, sg, mask, scale)
        out.backward(dO)
        rec = dict(Q=Q.numpy(), K=K.numpy(), V=V.numpy(), dO=dO.numpy(),
                   log_tau=log_tau.numpy(), log_alpha=log_alpha.numpy(),
                   out=out.detach().numpy(), dQ=q.grad.numpy(), dK=k.grad.numpy(),
                   dV=v.grad.numpy(), dlog_tau=lt.grad.numpy(), dlog_alpha=la.grad.numpy(),
                   sigma=np.array(sg), scale=np.array(np.nan if scale is None else scale,
                                                       dtype=np.float64))
        if mask is not None:
            rec["mask"] = mask.numpy()
        if lt_spec == "tau1":
            s = torch.matmul(Q, K.transpose(-1, -2)) * (D ** -0.5 if scale is None else scale)
            rec["softmax_out"] = torch.matmul(torch.softmax(s, -1), V).numpy()
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **rec)
        print("wrote", name)


def make_maxstable(ref):
    """STauOpusMaxStableFn of the fixed-tau patch (echo/patch_whisper_stau.py:74-112):
    attention weights from materialised scores and their gradient, every sigma
    of that module's registry, a per-head tau tensor and a scalar tau."""
    import patch_whisper_stau as P
    out = {}
    cases = [("softplus", "head"), ("sigmoid", "head"), ("exp", "head"), ("relu", "head"),
             ("tanh_shift", "head"), ("softplus", "scalar"), ("exp", "scalar")]
    for ci, (sg, tk) in enumerate(cases):
        g = torch.Generator().manual_seed(400 + ci)
        B, H, Lq, Lk = 2, 3, 17, 45
        scores = torch.randn(B, H, Lq, Lk, generator=g) * 3.0
        if ci == 0:       # a causal additive mask, as the decoder passes it
            scores = scores + torch.full((Lq, Lk), torch.finfo(torch.float32).min).triu(Lk - Lq + 1)
        if tk == "head":
            tau = (1.0 + torch.rand(H, generator=g) * 2.5).view(1, H, 1, 1)
        else:
            tau = 1.7
        dO = torch.randn(B, H, Lq, Lk, generator=g)
        sc = scores.clone().requires_grad_()
        attn = P.STauOpusMaxStableFn.apply(sc, tau, sg)
        attn.backward(dO)
        out[f"c{ci}_sigma"] = np.array(sg)
        out[f"c{ci}_scores"] = scores.numpy()
        out[f"c{ci}_tau"] = np.asarray(tau.reshape(-1).numpy() if torch.is_tensor(tau) else [tau], dtype=np.float32)
        out[f"c{ci}_tau_is_tensor"] = np.array(torch.is_tensor(tau))
        out[f"c{ci}_dO"] = dO.numpy()
        out[f"c{ci}_attn"] = attn.detach().numpy()
        out[f"c{ci}_dscores"] = sc.grad.numpy()
    out["n_cases"] = np.array(len(cases))
    np.savez_compressed(os.path.join(HERE, "maxstable.npz"), **out)
    print("wrote maxstable")


def make_wta(ref):
    import triton_wta as T
    import patch_whisper_sparse_grad as S
    g = torch.Generator().manual_seed(21)
    R, D = 48, 3072
    x = Fnn.gelu(torch.randn(R, D, generator=g)).to(torch.bfloat16)
    dy = torch.randn(R, D, generator=g).to(torch.bfloat16)
    bits = x.view(torch.int16).numpy().view(np.uint16)
    dybits = dy.view(torch.int16).numpy().view(np.uint16)
    rec = dict(x_bits=bits, dy_bits=dybits)
    ks = [1, 154, 306, 307, 768, 1536, 3072]
    rec["ks"] = np.array(ks)
    for k in ks:
        # threshold semantics: SparseGradWTA_Function (same rule as the GPU Triton path)
        xx = x.clone().requires_grad_()
        out = S.SparseGradWTA_Function.apply(xx, k)
        out.backward(dy)
        # the saved mask itself (the backward multiplies dy by it)
        thr = x.kthvalue(D - k + 1, dim=-1, keepdim=True).values
        thr_mask = (x >= thr)
        rec[f"thr_mask_k{k}"] = np.packbits(thr_mask.numpy(), axis=-1, bitorder="little")
        if k == 306:
            rec[f"sg_dx_bits_k{k}"] = xx.grad.view(torch.int16).numpy().view(np.uint16)
        rec[f"sg_out_is_x_k{k}"] = np.array(bool(torch.equal(out.detach(), x)))
        # exact-k semantics: the reference's CPU STE path
        y, m = T._torch_wta_forward(x, k)
        rec[f"exact_mask_k{k}"] = np.packbits(m.numpy(), axis=-1, bitorder="little")
        if k == 306:
            rec[f"exact_y_bits_k{k}"] = y.view(torch.int16).numpy().view(np.uint16)
    np.savez_compressed(os.path.join(HERE, "wta_gelu_48x3072.npz"), **rec)
    print("wrote wta")


def make_k_table(ref):
    import patch_whisper_sparse_grad as S
    logits = np.concatenate([np.linspace(-6, 6, 241), [-2.2, -2.1972246, 0.0,
                             -0.4054651, 2.0]]).astype(np.float32)
    rows = []
    for d_ff in (3072, 768, 100):
        for lg in logits:
            lk = S.LearnableKRatio(0.4)
            torch.nn.init.constant_(lk.logit_k, float(lg))
            rows.append((float(lg), d_ff, lk.get_k(d_ff)))
    inits = np.array([0.05, 0.1, 0.25, 0.4, 0.5, 0.9, 0.95])
    init_logits = []
    for r in inits:
        lk = S.LearnableKRatio(float(r))
        init_logits.append(float(lk.logit_k.item()))
    np.savez_compressed(os.path.join(HERE, "k_table.npz"),
                        logit=np.array([r[0] for r in rows], dtype=np.float32),
                        d_ff=np.array([r[1] for r in rows]),
                        k=np.array([r[2] for r in rows]),
                        init_ratio=inits, init_logit=np.array(init_logits, dtype=np.float32))
    print("wrote k_table")


def make_lr_table(ref):
    """The reference's LR lambda (echo/train_echo_opus1.py:230-244): its
    source is taken from the training script and executed alone (the script's
    top level needs the training data)."""
    import ast
    import math
    path = os.path.join(ref, "echo", "train_echo_opus1.py")
    tree = ast.parse(open(path).read())
    fn = next(n for n in tree.body if isinstance(n, ast.FunctionDef) and n.name == "make_lr_lambda")
    ns = {"math": math}
    exec(compile(ast.Module(body=[fn], type_ignores=[]), path, "exec"), ns)
    rows = []
    for warm, t0, tm in ((0, 10, 2), (5, 12, 2), (100, 400, 2), (7, 3, 1), (1, 1, 3)):
        f = ns["make_lr_lambda"](warm, t0, tm)
        for step in range(0, 4000, 7):
            rows.append((warm, t0, tm, step, f(step)))
    a = np.array(rows, dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, "lr_table.npz"), warmup=a[:, 0].astype(np.int64),
                        t0=a[:, 1].astype(np.int64), t_mult=a[:, 2].astype(np.int64),
                        step=a[:, 3].astype(np.int64), factor=a[:, 4])
    print("wrote lr_table")


def make_tau_star(ref):
    """solve_tau_star of tau_star/tau_star_solver.py:60-128 (imported from the
    reference) on seeded score rows, every sigma, with -1e9 key padding as its
    estimator adds."""
    sys.path.insert(0, os.path.join(ref, "tau_star"))
    import tau_star_solver as TS
    out = {}
    cases = [("softplus", 57, 30, 2.0, 1.5), ("sigmoid", 300, 30, 2.0, 2.0), ("exp", 120, 100, 1.0, 3.0),
             ("relu", 40, 20, 2.0, 1.0), ("softplus", 1, 30, 2.0, 1.0), ("softplus", 2, 50, 0.5, 4.0)]
    for ci, (sig, T, n_iter, tau_init, spread) in enumerate(cases):
        g = torch.Generator().manual_seed(500 + ci)
        scores = torch.randn(24, T, generator=g) * spread
        if T > 8:
            scores[3, T - 5:] = -1e9            # padded keys
        tau, kl = TS.solve_tau_star(scores, sigma=sig, n_iter=n_iter, tau_init=tau_init)
        key = f"c{ci}"
        out[key + "_scores"] = scores.numpy()
        out[key + "_tau"] = tau.numpy()
        out[key + "_kl"] = kl.numpy()
        out[key + "_meta"] = np.array([T, n_iter, tau_init])
        out[key + "_sigma"] = np.array(sig)
        # one-shot estimate cov_ref(s, ls) / var_ref(ls) (tau_star_solver.py:131-151)
        out[key + "_analytic"] = TS.solve_tau_star_analytic(scores, sigma=sig).numpy()
    # TauStarEstimator (tau_star_solver.py:180-275): two modules, calls of
    # different key lengths (padded with -1e9 to the longest), aggregated on the
    # host; per-"head" entries are tau[h].mean() over the flattened (N, H) rows
    est = TS.TauStarEstimator(n_iter=25)
    g = torch.Generator().manual_seed(640)
    calls = [("model.encoder.layers.0.self_attn", (2, 4, 6, 40)),
             ("model.encoder.layers.0.self_attn", (1, 4, 5, 33)),
             ("model.decoder.layers.1.encoder_attn", (3, 4, 2, 50)),
             ("model.decoder.layers.1.encoder_attn", (2, 4, 3, 50))]
    for ci, (name, shape) in enumerate(calls):
        sc = torch.randn(*shape, generator=g) * 2.0
        est.collect(name, sc)
        out[f"e{ci}_scores"] = sc.numpy()
        out[f"e{ci}_name"] = np.array(name)
    for mi, r in enumerate(est.aggregate(device="cpu")):
        out[f"m{mi}_name"] = np.array(r.module_name)
        out[f"m{mi}_tau"] = np.array(r.tau_per_head)
        out[f"m{mi}_kl"] = np.array(r.kl_per_head)
        out[f"m{mi}_dict"] = np.array(json.dumps(r.to_dict()))
    np.savez_compressed(os.path.join(HERE, "tau_star.npz"), **out)
    print("wrote tau_star")


def main(argv):
    ref = _ref_path(argv)
    sys.path.insert(0, os.path.join(ref, "echo"))
    torch.set_num_threads(4)
    only = os.environ.get("TAU_DXB_GOLDEN_ONLY")
    if only:
        globals()["make_" + only](ref)
        return
    make_attn(ref)
    make_wta(ref)
    make_k_table(ref)
    make_lr_table(ref)
    make_tau_star(ref)
    make_maxstable(ref)


if __name__ == "__main__":
    main(sys.argv)
