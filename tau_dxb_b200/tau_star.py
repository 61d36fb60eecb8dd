"""tau* estimation on the GPU: the reference's solve_tau_star operator.

``solve_tau_star`` keeps the signature and results of
tau_star/tau_star_solver.py:60-128 (the batched Newton solver for
tau* = argmin_tau KL(softmax(s) || softmax(tau log sigma(s))) over the last
dimension of ``scores``); ``solve_tau_star_analytic`` keeps its one-shot
estimate (:131-151); ``TauStarEstimator`` / ``ModuleResult`` keep the
collect / pad / solve / aggregate driver (:154-281); ``estimate_tau_per_head``
keeps tau_star/compute_tau_star_echo.py:116-136 (per-head means of tau* and
KL over all query rows of one attention call, n_iter = 100) without its host
copy of the scores. They run the ``tau_star_solve`` / ``tau_star_analytic``
kernels of libtau_dxb.so, which fuse every Newton step of a row on chip;
there is no CPU implementation.
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from typing import Dict, List, Tuple

import torch

from . import _capi as C


def _rows(scores: torch.Tensor) -> Tuple[torch.Tensor, int]:
    """[..., T] fp32 -> a [rows, T] view with unit key stride, and its row stride."""
    T = scores.shape[-1]
    x = scores.float()
    x2 = x.reshape(-1, T)
    if x2.shape[0] > 1 and (x2.stride(1) != 1 or x2.stride(0) < T):
        x2 = x2.contiguous()
    elif x2.stride(1) != 1:
        x2 = x2.contiguous()
    return x2, max(x2.stride(0), T)


def solve_tau_star(scores: torch.Tensor, sigma: str = "softplus", n_iter: int = 30, tau_init: float = 2.0,
                   tau_min: float = 0.1, tau_max: float = 10.0,
                   eps: float = 1e-6) -> Tuple[torch.Tensor, torch.Tensor]:
    """(tau, kl), each of shape scores.shape[:-1], fp32, on the scores' device.

    scores: [..., T] attention logits (any float dtype) on a CUDA device;
    sigma: "softplus", "sigmoid", "exp" or "relu". The reference also accepts
    a callable returning log sigma; this operator takes the named transfer
    functions only."""
    if not isinstance(sigma, str):
        raise TypeError("tau_dxb_b200.solve_tau_star: sigma must be one of "
                        f"{sorted(C.SIGMA_IDS)} (callables are not supported)")
    if sigma not in C.SIGMA_IDS:
        raise KeyError(sigma)
    if not scores.is_cuda:
        raise RuntimeError("tau_dxb_b200: solve_tau_star runs on CUDA tensors only "
                           "(this build has no CPU implementation)")
    shape = scores.shape[:-1]
    T = scores.shape[-1]
    tau = torch.empty(shape, dtype=torch.float32, device=scores.device)
    kl = torch.empty(shape, dtype=torch.float32, device=scores.device)
    n_rows = tau.numel()
    if n_rows == 0:
        return tau, kl
    if T <= 1:
        return tau.fill_(tau_init), kl.zero_()
    x2, stride = _rows(scores)
    rc = C.lib().tau_star_solve(x2.data_ptr(), n_rows, T, stride, C.SIGMA_IDS[sigma], int(n_iter),
                                float(tau_init), float(tau_min), float(tau_max), float(eps),
                                tau.data_ptr(), kl.data_ptr(), C.stream_ptr(scores.device))
    C.check("tau_star_solve", rc)
    return tau, kl


def tau_star_per_head(scores: torch.Tensor, sigma: str = "softplus", n_iter: int = 100,
                      **kw) -> Tuple[torch.Tensor, torch.Tensor]:
    """Device tensors [H] of the mean tau* and mean KL over the B * Lq rows of
    each head of scores [B, H, Lq, Lk]."""
    if scores.dim() != 4:
        raise ValueError(f"scores must be [B, H, Lq, Lk], got {tuple(scores.shape)}")
    tau, kl = solve_tau_star(scores, sigma=sigma, n_iter=n_iter, **kw)
    return tau.mean(dim=(0, 2)), kl.mean(dim=(0, 2))


def estimate_tau_per_head(scores_tensor: torch.Tensor, estimator=None,
                          sigma_name: str = "softplus") -> Tuple[List[float], List[float]]:
    """Per-head (tau list, KL list) of one attention call's scores
    [B, H, Lq, Lk], rounded to 4 and 6 decimals as the reference reports them;
    ``estimator`` is accepted for the reference's signature and not used (as
    there). One host read of 2 H floats replaces the per-head host loop."""
    taus, kls = tau_star_per_head(scores_tensor, sigma=sigma_name, n_iter=100)
    t = taus.cpu().tolist()
    k = kls.cpu().tolist()
    return [round(v, 4) for v in t], [round(v, 6) for v in k]


def solve_tau_star_analytic(scores: torch.Tensor, sigma: str = "softplus") -> torch.Tensor:
    """tau ~ Cov_ref(s, log sigma) / Var_ref(log sigma), clamped to [0.1, 10],
    shape scores.shape[:-1] (tau_star_solver.py:131-151)."""
    if not isinstance(sigma, str):
        raise TypeError("tau_dxb_b200.solve_tau_star_analytic: sigma must be one of "
                        f"{sorted(C.SIGMA_IDS)} (callables are not supported)")
    if sigma not in C.SIGMA_IDS:
        raise KeyError(sigma)
    if not scores.is_cuda:
        raise RuntimeError("tau_dxb_b200: solve_tau_star_analytic runs on CUDA tensors only "
                           "(this build has no CPU implementation)")
    tau = torch.empty(scores.shape[:-1], dtype=torch.float32, device=scores.device)
    if tau.numel() == 0:
        return tau
    x2, stride = _rows(scores)
    rc = C.lib().tau_star_analytic(x2.data_ptr(), tau.numel(), scores.shape[-1], stride, C.SIGMA_IDS[sigma],
                                   tau.data_ptr(), C.stream_ptr(scores.device))
    C.check("tau_star_analytic", rc)
    return tau


def _default_sigma_map() -> Dict[str, str]:
    return {
        "encoder.self_attn": "softplus",
        "decoder.self_attn": "sigmoid",
        "decoder.encoder_attn": "exp",
    }


@dataclass
class HeadTau:
    module_name: str
    head_index: int
    tau: float
    kl: float


def _std(xs: List[float]) -> float:
    """Population standard deviation (0 for an empty list)."""
    if not xs:
        return 0.0
    mean = sum(xs) / len(xs)
    return math.sqrt(sum((x - mean) ** 2 for x in xs) / max(1, len(xs)))


@dataclass
class ModuleResult:
    module_name: str
    num_heads: int
    tau_per_head: List[float] = field(default_factory=list)
    kl_per_head: List[float] = field(default_factory=list)

    def to_dict(self) -> dict:
        return {
            "module_name": self.module_name,
            "num_heads": self.num_heads,
            "tau_per_head": self.tau_per_head,
            "kl_per_head": self.kl_per_head,
            "tau_mean": float(sum(self.tau_per_head) / len(self.tau_per_head)) if self.tau_per_head else 0.0,
            "tau_std": _std(self.tau_per_head),
        }


class TauStarEstimator:
    """Collect score tensors per module and estimate tau* per head.

    collect(name, scores) keeps (B, H, ..., T) scores (the last dimension is
    the key length, dimension 1 the heads) on the host, as the reference does;
    aggregate() flattens each module's calls to (N, H, T), pads shorter key
    lengths with -1e9, solves all rows with tau_star_solve on ``device`` and
    reports entry h as round(tau[h].mean(), 4) — row h of the flattened
    (N, H) result averaged over heads, which is what the reference's
    ``tau[h].mean()`` computes (its result lists are indexed the same way).
    The sigma of a module is the first sigma_map key contained in its name,
    else softplus."""

    def __init__(self, n_iter: int = 30, tau_init: float = 2.0, tau_min: float = 0.1, tau_max: float = 10.0,
                 sigma_map: Dict[str, str] | None = None):
        self.n_iter = n_iter
        self.tau_init = tau_init
        self.tau_min = tau_min
        self.tau_max = tau_max
        self.sigma_map = sigma_map or _default_sigma_map()
        self.buffers: Dict[str, List[torch.Tensor]] = {}

    def _resolve_sigma(self, module_name: str) -> str:
        for key, val in self.sigma_map.items():
            if key in module_name:
                return val
        return "softplus"

    def collect(self, module_name: str, scores: torch.Tensor) -> None:
        if scores.numel() == 0:
            return
        self.buffers.setdefault(module_name, []).append(scores.detach().cpu())

    def _padded(self, tensors: List[torch.Tensor]) -> Tuple[torch.Tensor, int]:
        flat = [t.reshape(-1, t.shape[1], t.shape[-1]) for t in tensors]
        n_heads = flat[-1].shape[1]
        t_max = max(t.shape[2] for t in flat)
        padded = []
        for t in flat:
            if t.shape[2] < t_max:
                pad = torch.full((t.shape[0], n_heads, t_max - t.shape[2]), -1e9, dtype=torch.float32)
                t = torch.cat([t.float(), pad], dim=2)
            padded.append(t)
        return torch.cat(padded, dim=0).float(), n_heads

    def aggregate(self, device: str = "cuda") -> List[ModuleResult]:
        results = []
        for module_name, tensors in self.buffers.items():
            scores, n_heads = self._padded(tensors)
            tau, kl = solve_tau_star(scores.to(device), sigma=self._resolve_sigma(module_name), n_iter=self.n_iter,
                                     tau_init=self.tau_init, tau_min=self.tau_min, tau_max=self.tau_max)
            tau, kl = tau.cpu(), kl.cpu()
            res = ModuleResult(module_name=module_name, num_heads=n_heads)
            for h in range(n_heads):
                res.tau_per_head.append(round(float(tau[h].mean()), 4))
                res.kl_per_head.append(round(float(kl[h].mean()), 6))
            results.append(res)
        return results

    def save(self, path: str, results: List[ModuleResult] | None = None) -> None:
        if results is None:
            results = self.aggregate()
        with open(path, "w", encoding="utf-8") as f:
            json.dump([r.to_dict() for r in results], f, ensure_ascii=False, indent=2)

