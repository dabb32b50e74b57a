"""`sandmuon.optimizer` of the reference, bound to sandmuon_b200.optimizer:
the optimizers and the module helpers the reference's tests import."""
from sandmuon_b200.optimizer import (DiagonalWeightedPE, RankOneAWeightedPE, _graft_direction,  # noqa: F401
                                     _s8_fp32, diagonal_inverse_sqrt, rank1_inverse_sqrt, rank1_mapback,
                                     rank1_whiten)
