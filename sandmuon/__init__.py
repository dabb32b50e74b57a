"""The reference's import path, `sandmuon`, bound to the B200 engine.

Code written against pxike/SandMuon (`from sandmuon import RankOneAWeightedPE`,
`from sandmuon.optimizer import _s8_fp32`) runs unchanged on sandmuon_b200
when this directory is importable (the repository root on sys.path) and the
reference package is not: every name here is sandmuon_b200's own object.
"""
from sandmuon_b200 import (DiagonalWeightedPE, RankOneAWeightedPE, S8_COEFFICIENTS, S8_MARGIN,  # noqa: F401
                           S8_MULTIPLIER)

__all__ = ["DiagonalWeightedPE", "RankOneAWeightedPE", "S8_COEFFICIENTS", "S8_MARGIN", "S8_MULTIPLIER"]
