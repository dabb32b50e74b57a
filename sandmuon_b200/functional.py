"""Module-level helpers with the reference's names and signatures.

The reference package exports these functions next to its optimizers
(sandmuon/optimizer.py:19-93) and its tests import them.  They are kept here
for API compatibility only: the optimizer's step never calls them (it runs the
fused CUDA pipeline of libsandmuon_b200.so).  The small vector/matrix helpers
are plain torch expressions of the same formulas.  `_s8_fp32` runs the
engine's S8 map on CUDA tensors and, like the reference helper, the FP32 map
in torch arithmetic on any other device.
"""
from __future__ import annotations

import math

import torch


def diagonal_inverse_sqrt(value: torch.Tensor) -> torch.Tensor:
    """rsqrt(max(max(v, mean*1e-6) / max(mean, tiny), 1e-6)) (sandmuon/optimizer.py:19-24)."""
    mean = value.mean()
    tiny = torch.finfo(value.dtype).tiny
    ratio = torch.maximum(value, mean * 1e-6) / torch.clamp(mean, min=tiny)
    return torch.clamp(ratio, min=1e-6).rsqrt()


def rank1_inverse_sqrt(second: torch.Tensor, mean: torch.Tensor):
    """(D^-1/2, z, c) of the rank-one whitener (sandmuon/optimizer.py:27-35)."""
    q = torch.clamp(second.mean(), min=torch.finfo(second.dtype).tiny)
    inverse = torch.clamp(torch.clamp(second - mean * mean, min=0.0) / q, min=1e-6).rsqrt()
    z = inverse * mean / q.sqrt()
    rho = (1.0 + (z * z).sum()).sqrt()
    return inverse, z, -1.0 / (rho * (rho + 1.0))


def rank1_whiten(matrix: torch.Tensor, left, right) -> torch.Tensor:
    """L M R^T with L = (I + c zz^T) diag(d) applied without dense factors
    (sandmuon/optimizer.py:38-45)."""
    (di, zi, ci), (dj, zj, cj) = left, right
    v = matrix * di.unsqueeze(-1) * dj.unsqueeze(-2)
    v = v + ci[..., None, None] * zi.unsqueeze(-1) * torch.matmul(zi.unsqueeze(-2), v)
    return v + cj[..., None, None] * torch.matmul(v, zj.unsqueeze(-1)) * zj.unsqueeze(-2)


def rank1_mapback(value: torch.Tensor, left, right) -> torch.Tensor:
    """Rank-one factors first, then the diagonals (sandmuon/optimizer.py:48-60)."""
    (di, zi, ci), (dj, zj, cj) = left, right
    v = value + ci * zi[:, None] * (zi[None, :] @ value)
    v = v + cj * (v @ zj[:, None]) * zj[None, :]
    return v * di[:, None] * dj[None, :]


def _graft_direction(value: torch.Tensor, output_rows: int) -> torch.Tensor:
    """value * sqrt(rows) / max(|value|_F, tiny) (sandmuon/optimizer.py:63-66)."""
    v = value.float()
    return v * (math.sqrt(float(output_rows)) / torch.clamp(v.norm(), min=torch.finfo(torch.float32).tiny))


def _s8_fp32(x: torch.Tensor) -> torch.Tensor:
    """The S8 polar map of a [.., rows, cols] tensor (sandmuon/optimizer.py:69-93).

    CUDA tensors: the engine's map (same orientation, normalisation, margin
    and coefficients, with stages 1-4 in compensated BF16 and stage 5 in BF16,
    FP32 accumulation, on tcgen05).  Tensors on other devices: the map in
    FP32 torch arithmetic, as the reference helper computes it anywhere.  The
    optimizer's step never calls this function."""
    if x.is_cuda:
        from .engine import s8_polar
        return s8_polar(x.float())
    return _s8_torch_fp32(x)


def _s8_torch_fp32(x: torch.Tensor) -> torch.Tensor:
    """Five polynomial stages X <- (a I + b X X^T + c (X X^T)^2) X on the
    orientation with rows <= cols, after normalising X to unit Frobenius
    norm; stage 1 first rescales the gram by s = 1.35 |G^2|_F^(1/4).  An
    all-zero batch maps to zeros."""
    from .coefficients import S8_COEFFICIENTS, S8_MARGIN, S8_MULTIPLIER
    flip = x.shape[-2] > x.shape[-1]
    y = (x.mT if flip else x).float()
    if not torch.count_nonzero(y):
        return torch.zeros_like(y.mT if flip else y)
    y = y / y.norm(dim=(-2, -1), keepdim=True).clamp_min(1e-30)
    eye = torch.eye(y.shape[-2], dtype=y.dtype, device=y.device)
    for stage, (a, b, c) in enumerate(S8_COEFFICIENTS):
        gram = y @ y.mT
        gram_sq = gram @ gram
        if stage == 0:
            s = (S8_MARGIN * gram_sq.norm(dim=(-2, -1), keepdim=True).pow(0.25)).clamp_min(1e-30)
            y = ((a * eye + b * gram / s.square() + c * gram_sq / s.pow(4)) @ y) / s
        else:
            y = (a * eye + b * gram + c * gram_sq) @ y
    return (y.mT if flip else y) * S8_MULTIPLIER
