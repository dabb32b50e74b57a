"""Drop-in surface that needs no GPU: the reference's import path and the
module helper `_s8_fp32` on CPU tensors, checked against the reference's own
outputs (golden fixtures made by running the reference package)."""
from pathlib import Path

import numpy as np
import pytest
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"


def test_reference_import_path_resolves_to_the_engine():
    import sandmuon
    import sandmuon_b200
    from sandmuon.coefficients import S8_COEFFICIENTS, S8_MARGIN
    from sandmuon.optimizer import (DiagonalWeightedPE, RankOneAWeightedPE, _graft_direction, _s8_fp32,
                                    diagonal_inverse_sqrt, rank1_inverse_sqrt, rank1_mapback, rank1_whiten)
    assert sandmuon.RankOneAWeightedPE is sandmuon_b200.RankOneAWeightedPE is RankOneAWeightedPE
    assert DiagonalWeightedPE is sandmuon_b200.DiagonalWeightedPE
    assert S8_COEFFICIENTS is sandmuon_b200.S8_COEFFICIENTS and S8_MARGIN == 1.35
    assert sandmuon.__all__ == sandmuon_b200.__all__
    for fn in (_graft_direction, _s8_fp32, diagonal_inverse_sqrt, rank1_inverse_sqrt, rank1_mapback, rank1_whiten):
        assert callable(fn)


@pytest.mark.parametrize("case", range(8))
def test_s8_helper_on_cpu_matches_reference(case):
    from sandmuon_b200.optimizer import _s8_fp32
    g = np.load(GOLDEN / "s8.npz")
    x = torch.from_numpy(g[f"s8_in_{case}"])
    got = _s8_fp32(x)
    want = torch.from_numpy(g[f"s8_out_{case}"])
    assert got.shape == want.shape and got.dtype == torch.float32 and got.device.type == "cpu"
    assert float((got.double() - want.double()).norm() / want.double().norm()) < 2e-5


def test_s8_helper_on_cpu_zero_batch_and_orientation():
    from sandmuon_b200.optimizer import _s8_fp32
    g = np.load(GOLDEN / "s8.npz")
    zero = _s8_fp32(torch.from_numpy(g["s8_zero_in"]))
    assert zero.shape == g["s8_zero_out"].shape and not zero.any()
    tall = torch.randn(2, 7, 3, generator=torch.Generator().manual_seed(0))
    out = _s8_fp32(tall)
    assert out.shape == (2, 7, 3)
    assert torch.allclose(out, _s8_fp32(tall.mT.contiguous()).mT, atol=1e-6)
