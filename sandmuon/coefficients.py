"""`sandmuon.coefficients` of the reference, bound to sandmuon_b200.coefficients."""
from sandmuon_b200.coefficients import S8_COEFFICIENTS, S8_MARGIN, S8_MULTIPLIER  # noqa: F401
