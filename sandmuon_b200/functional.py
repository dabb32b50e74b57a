"""Module-level helpers with the reference's names and signatures.

The reference package exports these functions next to its optimizers
(sandmuon/optimizer.py:19-93) and its tests import them.  They are kept here
for API compatibility only: the optimizer's step never calls them (it runs the
fused CUDA pipeline of libsandmuon_b200.so).  The small vector/matrix helpers
are plain torch expressions of the same formulas; `_s8_fp32` dispatches to the
engine's S8 map and therefore needs a CUDA float32 tensor.
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
    """The S8 polar map of the engine for a CUDA float32 [.., rows, cols] tensor.

    Replaces the reference's eager FP32 map (sandmuon/optimizer.py:69-93): same
    orientation, normalisation, margin and coefficients, with stages 1-4 in
    compensated BF16 and stage 5 in BF16 (FP32 accumulation) on tcgen05."""
    from .engine import s8_polar
    return s8_polar(x.float())
