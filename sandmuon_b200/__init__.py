"""sandmuon_b200: the SandMuon optimizer on B200 (sm_100a) CUDA kernels.

Drop-in for the `sandmuon` package: `import sandmuon_b200 as sandmuon`.
"""

from .optimizer import DiagonalWeightedPE, RankOneAWeightedPE
from .coefficients import S8_COEFFICIENTS, S8_MARGIN, S8_MULTIPLIER

__all__ = ["DiagonalWeightedPE", "RankOneAWeightedPE", "S8_COEFFICIENTS", "S8_MARGIN", "S8_MULTIPLIER"]
