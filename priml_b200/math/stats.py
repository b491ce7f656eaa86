"""Statistics helpers (``priml/math/stats.py:30-430``): covariance, entropies,
Jensen-Shannon divergence, PCA (eigh / SVD / power iteration), robust
normalization and throughput windows."""

from __future__ import annotations

from collections.abc import Callable, Sequence

import torch
from torch import Tensor

from priml_b200.math.custom_types import Tensorable, convert_to_tensor
from priml_b200.math.distributed import logmeanexp_all_to_all
from priml_b200.math.numeric import logmeanexp

__all__ = [
    "SlidingWindow",
    "cov",
    "ema_update",
    "entropy_logits",
    "entropy_logits_mean_all_to_all",
    "entropy_probs",
    "jsd",
    "pca",
    "pca_eigh",
    "pca_power",
    "pca_svd",
    "quantile_normalize",
]

PcaDecompose = Callable[[Tensor], tuple[Tensor, Tensor]]


def cov(x: Tensorable, y: Tensorable | None = None, bias: bool = True, rowvar: bool = False) -> Tensor:
    """Covariance (or cross-covariance with ``y``); columns are variables unless ``rowvar``.
    ``bias`` divides by N, otherwise by N - 1. A 1-D input gives its scalar variance."""
    x = convert_to_tensor(x)
    yt = None if y is None else convert_to_tensor(y, dtype=x.dtype)
    vector = x.ndim == 1
    if vector:
        x = x[None]
        yt = None if yt is None else yt[None]
        rowvar = True
    if not rowvar:
        x = x.transpose(-1, -2)
        yt = None if yt is None else yt.transpose(-1, -2)
    # now [..., variables, observations]
    xc = x - x.mean(dim=-1, keepdim=True)
    yc = xc if yt is None else yt - yt.mean(dim=-1, keepdim=True)
    n = x.shape[-1]
    denom = n if (bias or n <= 1) else n - 1
    out = xc @ yc.transpose(-1, -2) / denom
    return out.reshape(()) if vector else out


def entropy_logits(x: Tensorable, y: Tensorable | None = None, dim: int | Sequence[int] = -1,
                   keepdim: bool = False) -> Tensor:  # fmt: skip
    """Cross-entropy ``H(softmax x, softmax y)`` (entropy when ``y`` is None)."""
    x = convert_to_tensor(x)
    y = x if y is None else convert_to_tensor(y, dtype=x.dtype)
    return -(torch.softmax(x, dim=dim) * torch.log_softmax(y, dim=dim)).sum(dim=dim, keepdim=keepdim)


def entropy_probs(p: Tensorable, q: Tensorable | None = None, dim: int | Sequence[int] = -1,
                  keepdim: bool = False) -> Tensor:  # fmt: skip
    """Cross-entropy ``H(p, q)`` (entropy when ``q`` is None); terms with ``p == 0`` contribute 0."""
    p = convert_to_tensor(p)
    q = p if q is None else convert_to_tensor(q, dtype=p.dtype)
    logq = torch.log(q.clamp_min(torch.finfo(q.dtype).tiny))
    return -torch.where(p > 0, p * logq, 0.0).sum(dim=dim, keepdim=keepdim)


def jsd(logp: Tensorable, *, ensemble_dim: int | Sequence[int] = 0, event_dim: int | Sequence[int] = -1) -> Tensor:
    """Generalized Jensen-Shannon divergence ``H(mean_i p_i) - mean_i H(p_i)`` (Lin 1991)."""
    logp = convert_to_tensor(logp)
    ens = (ensemble_dim,) if isinstance(ensemble_dim, int) else tuple(ensemble_dim)
    ev = (event_dim,) if isinstance(event_dim, int) else tuple(event_dim)

    def h(lp: Tensor) -> Tensor:
        return -(lp.exp() * torch.where(torch.isneginf(lp), 0.0, lp)).sum(dim=ev, keepdim=True)

    mixture = h(logmeanexp(logp, dim=ens, keepdim=True))
    members = h(logp).mean(dim=ens, keepdim=True)
    return (mixture - members).squeeze(tuple(sorted({d % logp.ndim for d in (*ens, *ev)})))


def entropy_logits_mean_all_to_all(x: Tensorable, y: Tensorable | None = None, *, dim: int | Sequence[int] = -1,
                                   dim_mean: int | Sequence[int] | None = None, keepdim: bool = False,
                                   keepdim_mean: bool = False, world_size: int | None = None) -> Tensor:  # fmt: skip
    """``H(mean p, mean q)`` where ``p = softmax x`` is averaged locally over ``dim_mean``
    and ``log mean q`` is averaged over ``dim_mean`` AND all ranks (mean-teacher entropy)."""
    x = convert_to_tensor(x)
    y = x if y is None else convert_to_tensor(y, dtype=x.dtype)
    if dim_mean is None:
        event = {d % x.ndim for d in ((dim,) if isinstance(dim, int) else dim)}
        dim_mean = tuple(d for d in range(x.ndim) if d not in event)
    mean_p = torch.softmax(x, dim=dim).mean(dim=dim_mean, keepdim=keepdim_mean)
    log_mean_q = logmeanexp_all_to_all(torch.log_softmax(y, dim=dim), dim=dim_mean, keepdim=keepdim_mean,
                                       world_size=world_size)  # fmt: skip
    return -(mean_p * log_mean_q).sum(dim=dim, keepdim=keepdim)


# ------------------------------------------------------------------ PCA
def _population_cov(xc: Tensor) -> Tensor:
    return xc.T @ xc / xc.shape[0]


def pca_eigh(x_centered: Tensor) -> tuple[Tensor, Tensor]:
    """Ascending eigenvalues / eigenvector columns of the population covariance via ``eigh``."""
    return torch.linalg.eigh(_population_cov(x_centered))


def pca_svd(x_centered: Tensor) -> tuple[Tensor, Tensor]:
    """Same decomposition from the SVD of the data matrix (ascending order)."""
    _, s, vh = torch.linalg.svd(x_centered, full_matrices=False)
    return (s * s / x_centered.shape[0]).flip(0), vh.T.flip(1)


def pca_power(x_centered: Tensor, num_iters: int = 200, tol: float = 0.0) -> tuple[Tensor, Tensor]:
    """Orthogonal (subspace) iteration with QR re-orthonormalization; only matmuls and QR."""
    sigma = _population_cov(x_centered)
    d = sigma.shape[0]
    q, _ = torch.linalg.qr(torch.randn(d, d, dtype=sigma.dtype, device=sigma.device))
    rayleigh = (q * (sigma @ q)).sum(0)
    for _ in range(num_iters):
        q, r = torch.linalg.qr(sigma @ q)
        q = q * torch.sign(torch.diagonal(r)).where(torch.diagonal(r) != 0, torch.ones_like(torch.diagonal(r)))
        if tol > 0:
            new = (q * (sigma @ q)).sum(0)
            done = bool((new - rayleigh).abs().max() < tol)
            rayleigh = new
            if done:
                break
    rayleigh = (q * (sigma @ q)).sum(0)
    order = rayleigh.argsort()
    return rayleigh[order], q[:, order]


def pca(x: Tensorable, *, whiten: bool = False, eps: float = 0.0, decompose: PcaDecompose = pca_eigh
        ) -> tuple[Tensor, Tensor]:  # fmt: skip
    """Fit PCA on rows-as-observations ``x`` (fp32): ascending eigenvalues and eigenvector
    columns of the population covariance; ``whiten`` scales columns by ``1/sqrt(lambda + eps)``."""
    xt = convert_to_tensor(x).float()
    vals, vecs = decompose(xt - xt.mean(dim=0, keepdim=True))
    if whiten:
        vecs = vecs * torch.rsqrt(vals + eps)[None, :]
    return vals, vecs


def quantile_normalize(x: Tensorable, q: float = 1e-3) -> Tensor:
    """Map ``x`` to [0, 1] between its ``q`` and ``1 - q`` quantiles (clipped)."""
    x = convert_to_tensor(x)
    flat = x.detach().reshape(-1).float()
    lo = torch.quantile(flat, q)
    hi = torch.quantile(flat, 1.0 - q)
    return ((x - lo) / (hi - lo).clamp_min(torch.finfo(torch.float32).eps)).clamp(0.0, 1.0)


def ema_update(current: float, new_value: float, alpha: float = 0.3) -> float:
    """``alpha * new + (1 - alpha) * current``."""
    return alpha * new_value + (1.0 - alpha) * current


class SlidingWindow:
    """Rate of a cumulative counter over the last ``window_sec`` seconds, smoothed by
    ``pseudocount`` items over ``pseudotime`` seconds (Laplace smoothing)."""

    def __init__(self, window_sec: float = 30.0, pseudocount: float = 2.0, pseudotime: float = 0.1) -> None:
        self.window_sec = window_sec
        self.pseudocount = pseudocount
        self.pseudotime = pseudotime
        self.samples: list[tuple[float, float]] = []

    def add(self, timestamp: float, cumulative_count: float) -> None:
        self.samples.append((timestamp, cumulative_count))
        horizon = timestamp - self.window_sec
        while self.samples and self.samples[0][0] < horizon:
            self.samples.pop(0)

    def compute_rate(self, current_time: float, current_count: float) -> float:
        if len(self.samples) < 2:
            return 0.0
        t0, c0 = self.samples[0]
        return (current_count - c0 + self.pseudocount) / (current_time - t0 + self.pseudotime)
