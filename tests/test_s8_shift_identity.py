"""The shifted-gram form of the S8 polynomial used by stages 2-5 on the GPU:
with beta = b / (2c), a I + b G + c G^2 = c (G + beta I)^2 + (a - c beta^2) I.
Checked in float64 for every stage's coefficients on random symmetric grams
(CPU; the GPU parity tests check the kernels that use it)."""
import numpy as np
import pytest

from sandmuon_b200.coefficients import S8_COEFFICIENTS


@pytest.mark.parametrize("stage", range(1, len(S8_COEFFICIENTS)))
def test_shifted_gram_polynomial_equals_direct_form(stage):
    a, b, c = (float(v) for v in S8_COEFFICIENTS[stage])
    rng = np.random.default_rng(stage)
    x = rng.standard_normal((48, 80))
    x /= np.linalg.norm(x)
    g = x @ x.T
    eye = np.eye(len(g))
    beta = b / (2.0 * c)
    direct = a * eye + b * g + c * g @ g
    shifted = c * (g + beta * eye) @ (g + beta * eye) + (a - c * beta * beta) * eye
    assert np.linalg.norm(shifted - direct) / np.linalg.norm(direct) < 1e-12
