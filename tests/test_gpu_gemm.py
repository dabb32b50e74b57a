"""The batched tcgen05 GEMM (sm_gemm_bf16) against torch FP32/FP64 products of
the same BF16 operands.  Accumulation is FP32 in both, so plain-mode results
agree to FP32 rounding; the compensated mode must beat plain BF16 by orders of
magnitude against an FP64 product of the unrounded FP32 operands."""
import pytest
import torch

from sandmuon_b200 import _lib, engine

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def rnd(*shape, seed=0, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(DEV)


def split(x):
    hi = x.to(torch.bfloat16)
    lo = (x - hi.float()).to(torch.bfloat16)
    return hi, lo


def rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("batch,m,n,k", [(1, 128, 256, 64), (2, 128, 128, 192), (3, 256, 512, 320),
                                         (2, 384, 768, 768)])
def test_plain_kmajor_f32(batch, m, n, k):
    a = rnd(batch, m, k, seed=1).to(torch.bfloat16)
    b = rnd(batch, n, k, seed=2).to(torch.bfloat16)
    out = torch.empty(batch, m, n, device=DEV)
    engine.gemm_bf16(a, b, b_kmajor=True, epilogue=_lib.SM_EPI_F32, out0=out)
    want = torch.bmm(a.float(), b.float().transpose(1, 2))
    assert rel(out, want) < 1e-5
    assert _lib.device_status(DEV) == 0


@pytest.mark.parametrize("batch,m,n,k", [(1, 128, 256, 64), (2, 256, 384, 128), (2, 128, 768, 256)])
def test_plain_mnmajor_f32(batch, m, n, k):
    a = rnd(batch, m, k, seed=3).to(torch.bfloat16)
    b = rnd(batch, k, n, seed=4).to(torch.bfloat16)
    out = torch.empty(batch, m, n, device=DEV)
    engine.gemm_bf16(a, b, b_kmajor=False, epilogue=_lib.SM_EPI_F32, out0=out)
    want = torch.bmm(a.float(), b.float())
    assert rel(out, want) < 1e-5


def test_alpha_and_bf16_epilogue():
    a = rnd(2, 128, 128, seed=5).to(torch.bfloat16)
    b = rnd(2, 256, 128, seed=6).to(torch.bfloat16)
    alpha = torch.tensor([0.5, -2.0], device=DEV)
    out = torch.empty(2, 128, 256, device=DEV, dtype=torch.bfloat16)
    engine.gemm_bf16(a, b, epilogue=_lib.SM_EPI_BF16, out0=out, alpha=alpha)
    want = torch.bmm(a.float(), b.float().transpose(1, 2)) * alpha[:, None, None]
    assert rel(out.float(), want) < 4e-3


@pytest.mark.parametrize("b_kmajor", [True, False])
def test_compensated_mode_is_near_fp32(b_kmajor):
    x = rnd(2, 256, 192, seed=7)
    y = rnd(2, 256, 192, seed=8) if b_kmajor else rnd(2, 192, 256, seed=8)
    xh, xl = split(x)
    yh, yl = split(y)
    out = torch.empty(2, 256, 256, device=DEV)
    engine.gemm_bf16(xh, yh, a_lo=xl, b_lo=yl, b_kmajor=b_kmajor, epilogue=_lib.SM_EPI_F32, out0=out)
    want = torch.bmm(x.double(), (y.transpose(1, 2) if b_kmajor else y).double())
    plain = torch.bmm(xh.float(), (yh.transpose(1, 2) if b_kmajor else yh).float())
    assert rel(out, want) < 2e-5
    assert rel(plain, want) > 100 * rel(out, want)


def test_hilo_epilogue_reconstructs_fp32():
    x = rnd(1, 128, 128, seed=9)
    xh, xl = split(x)
    hi = torch.empty(1, 128, 128, device=DEV, dtype=torch.bfloat16)
    lo = torch.empty_like(hi)
    engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, epilogue=_lib.SM_EPI_HILO, out0=hi, out1=lo)
    want = torch.bmm(x.double(), x.double().transpose(1, 2))
    assert rel(hi.float() + lo.float(), want) < 2e-5
    # the lo plane is what remains after rounding to BF16: at most half an ulp of hi
    assert ((lo.float().abs() <= hi.float().abs() * 2.0 ** -8) | (hi == 0)).all()


def test_norm_partials_sum_to_frobenius_square():
    x = rnd(3, 256, 256, seed=10)
    xh, xl = split(x)
    out = torch.empty(3, 256, 256, device=DEV)
    per_mat = (256 // 128) * (256 // 256) * _lib.SM_EPI_NORM_SLOTS
    partials = torch.empty(3, per_mat, device=DEV)
    engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, epilogue=_lib.SM_EPI_F32_NORM, out0=out, partials=partials)
    torch.testing.assert_close(partials.double().sum(1), out.double().square().sum((1, 2)), rtol=1e-5, atol=0)


def test_poly_epilogue():
    g = rnd(2, 256, 256, seed=11, scale=0.05)
    g = ((g + g.transpose(1, 2)) / 2).to(torch.bfloat16)
    out = torch.empty_like(g)
    a, b, c = 4.1, -2.9, 0.53
    engine.gemm_bf16(g, g, epilogue=_lib.SM_EPI_POLY, out0=out, aux=g, poly=(a, b, c))
    gf = g.float()
    want = a * torch.eye(256, device=DEV) + b * gf + c * torch.bmm(gf, gf.transpose(1, 2))
    assert rel(out.float(), want) < 4e-3


def test_poly_hilo_epilogue_is_near_fp32():
    g = rnd(2, 256, 256, seed=13, scale=0.05)
    g = (g + g.transpose(1, 2)) / 2
    gh, gl = split(g)
    ph = torch.empty_like(gh)
    pl = torch.empty_like(gh)
    a, b, c = 3.93, -2.87, 0.537
    engine.gemm_bf16(gh, gh, a_lo=gl, b_lo=gl, epilogue=_lib.SM_EPI_POLY_HILO, out0=ph, out1=pl, aux=gh,
                     aux_lo=gl, poly=(a, b, c))
    gd = g.double()
    want = a * torch.eye(256, device=DEV, dtype=torch.float64) + b * gd + c * torch.bmm(gd, gd.transpose(1, 2))
    assert rel(ph.float() + pl.float(), want) < 2e-5


def test_compensated_mnmajor_hilo_output():
    p = rnd(2, 128, 256, seed=14)
    x = rnd(2, 256, 512, seed=15)
    phi, plo = split(p)
    xh, xl = split(x)
    oh = torch.empty(2, 128, 512, device=DEV, dtype=torch.bfloat16)
    ol = torch.empty_like(oh)
    alpha = torch.tensor([0.25, 3.0], device=DEV)
    engine.gemm_bf16(phi, xh, a_lo=plo, b_lo=xl, b_kmajor=False, epilogue=_lib.SM_EPI_HILO, out0=oh, out1=ol,
                     alpha=alpha)
    want = torch.bmm(p.double(), x.double()) * alpha.double()[:, None, None]
    assert rel(oh.float() + ol.float(), want) < 2e-5


def test_rejects_unaligned_shapes():
    a = torch.zeros(1, 100, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="M%128"):
        engine.gemm_bf16(a, a, out0=torch.empty(1, 100, 100, device=DEV))


def test_gemm_is_deterministic():
    a = rnd(4, 256, 512, seed=12).to(torch.bfloat16)
    outs = []
    for _ in range(2):
        out = torch.empty(4, 256, 256, device=DEV)
        engine.gemm_bf16(a, a, out0=out)
        outs.append(out)
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("epi", ["f32", "hilo", "norm"])
def test_symmetric_mode_matches_full_product(epi):
    """Upper-triangular tiles + mirrored stores reproduce the full X X^T."""
    x = rnd(3, 384, 512, seed=16)
    xh, xl = split(x)
    want = torch.bmm(x.double(), x.double().transpose(1, 2))
    sym = _lib.SM_EPI_SYMMETRIC
    if epi == "f32":
        out = torch.full((3, 384, 384), float("nan"), device=DEV)
        engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, epilogue=_lib.SM_EPI_F32 | sym, out0=out)
        assert rel(out, want) < 2e-5
    elif epi == "hilo":
        hi = torch.full((3, 384, 384), float("nan"), device=DEV, dtype=torch.bfloat16)
        lo = torch.full_like(hi, float("nan"))
        engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, epilogue=_lib.SM_EPI_HILO | sym, out0=hi, out1=lo)
        assert rel(hi.float() + lo.float(), want) < 2e-5
    else:
        out = torch.empty(3, 384, 384, device=DEV)
        partials = torch.full((3, 3 * 3 * _lib.SM_EPI_NORM_SLOTS), float("nan"), device=DEV)
        engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, epilogue=_lib.SM_EPI_F32_NORM | sym, out0=out, partials=partials)
        torch.testing.assert_close(partials.double().sum(1), want.square().sum((1, 2)), rtol=1e-5, atol=0)


def test_symmetric_poly_epilogue():
    g = rnd(2, 256, 256, seed=17, scale=0.05)
    g = (g + g.transpose(1, 2)) / 2
    gh, gl = split(g)
    ph = torch.full_like(gh, float("nan"))
    pl = torch.full_like(gh, float("nan"))
    a, b, c = 3.28, -2.41, 0.486
    engine.gemm_bf16(gh, gh, a_lo=gl, b_lo=gl, epilogue=_lib.SM_EPI_POLY_HILO | _lib.SM_EPI_SYMMETRIC, out0=ph,
                     out1=pl, aux=gh, aux_lo=gl, poly=(a, b, c))
    gd = (gh.double() + gl.double())
    want = a * torch.eye(256, device=DEV, dtype=torch.float64) + b * gd + c * torch.bmm(gd, gd.transpose(1, 2))
    assert rel(ph.float() + pl.float(), want) < 2e-5


@pytest.mark.parametrize("comp", [False, True])
@pytest.mark.parametrize("n", [256, 384])
def test_mn_major_a_and_b(comp, n):
    """A read MN-major ([K, M] storage) with an MN-major B: the layout of the
    symmetric P and G in P X and G G (32-deep k-blocks)."""
    at = rnd(2, 192, 256, seed=18)    # [K, M]
    b = rnd(2, 192, n, seed=19)       # [K, N]
    ah, al = split(at)
    bh, bl = split(b)
    out = torch.empty(2, 256, n, device=DEV)
    engine.gemm_bf16(ah, bh, a_lo=al if comp else None, b_lo=bl if comp else None, b_kmajor=False, a_mnmajor=True,
                     epilogue=_lib.SM_EPI_F32, out0=out)
    if comp:
        want = torch.bmm(at.double().transpose(1, 2), b.double())
        assert rel(out, want) < 2e-5
    else:
        want = torch.bmm(ah.float().transpose(1, 2), bh.float())
        assert rel(out, want) < 1e-5


# ------------------------------------------------------------ CTA-pair mode
# 256-row tiles computed by two CTAs with tcgen05 cta_group::2: each CTA
# stages its own A rows and half of B; the leader issues the MMAs.

@pytest.mark.parametrize("batch,m,n,k", [(1, 256, 256, 64), (2, 512, 384, 192), (2, 768, 768, 768),
                                         (1, 256, 3072, 128)])
@pytest.mark.parametrize("b_kmajor", [True, False])
def test_pair_plain_f32(batch, m, n, k, b_kmajor):
    a = rnd(batch, m, k, seed=21).to(torch.bfloat16)
    b = rnd(batch, n, k, seed=22).to(torch.bfloat16) if b_kmajor else rnd(batch, k, n, seed=22).to(torch.bfloat16)
    out = torch.full((batch, m, n), float("nan"), device=DEV)
    engine.gemm_bf16(a, b, b_kmajor=b_kmajor, pair=True, epilogue=_lib.SM_EPI_F32, out0=out)
    want = torch.bmm(a.float(), b.float().transpose(1, 2) if b_kmajor else b.float())
    assert rel(out, want) < 1e-5
    assert _lib.device_status(DEV) == 0


@pytest.mark.parametrize("b_kmajor", [True, False])
def test_pair_compensated_hilo_with_alpha(b_kmajor):
    p = rnd(2, 512, 256, seed=23)
    x = rnd(2, 512, 256, seed=24) if b_kmajor else rnd(2, 256, 512, seed=24)
    ph, pl = split(p)
    xh, xl = split(x)
    oh = torch.full((2, 512, 512), float("nan"), device=DEV, dtype=torch.bfloat16)
    ol = torch.full_like(oh, float("nan"))
    alpha = torch.tensor([0.5, -3.0], device=DEV)
    engine.gemm_bf16(ph, xh, a_lo=pl, b_lo=xl, b_kmajor=b_kmajor, pair=True, epilogue=_lib.SM_EPI_HILO, out0=oh,
                     out1=ol, alpha=alpha)
    want = torch.bmm(p.double(), x.double().transpose(1, 2) if b_kmajor else x.double())
    want = want * alpha.double()[:, None, None]
    assert rel(oh.float() + ol.float(), want) < 2e-5


def test_pair_matches_single_cta_bitwise():
    """Same tiles' K order and the same FP32 accumulation: identical results."""
    x = rnd(3, 512, 768, seed=25)
    xh, xl = split(x)
    outs = []
    for pair in (False, True):
        out = torch.empty(3, 512, 512, device=DEV)
        engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, pair=pair, epilogue=_lib.SM_EPI_F32, out0=out)
        outs.append(out)
    assert rel(outs[1], outs[0]) < 1e-6


@pytest.mark.parametrize("bn128", [False, True])
@pytest.mark.parametrize("epi", ["f32", "hilo", "norm"])
def test_pair_symmetric_mode(epi, bn128):
    """256 x 256 pair tiles, or 256 x 128 block-row pair tiles (bn128) whose
    below-diagonal blocks are skipped: the full product either way."""
    x = rnd(3, 768, 512, seed=26)
    xh, xl = split(x)
    want = torch.bmm(x.double(), x.double().transpose(1, 2))
    sym = _lib.SM_EPI_SYMMETRIC
    kw = dict(a_lo=xl, b_lo=xl, pair=True, bn128=bn128)
    if epi == "f32":
        out = torch.full((3, 768, 768), float("nan"), device=DEV)
        engine.gemm_bf16(xh, xh, epilogue=_lib.SM_EPI_F32 | sym, out0=out, **kw)
        assert rel(out, want) < 2e-5
    elif epi == "hilo":
        hi = torch.full((3, 768, 768), float("nan"), device=DEV, dtype=torch.bfloat16)
        lo = torch.full_like(hi, float("nan"))
        engine.gemm_bf16(xh, xh, epilogue=_lib.SM_EPI_HILO | sym, out0=hi, out1=lo, **kw)
        assert rel(hi.float() + lo.float(), want) < 2e-5
    else:
        out = torch.empty(3, 768, 768, device=DEV)
        tiles = 3 * (6 if bn128 else 3)
        partials = torch.full((3, tiles * _lib.SM_EPI_NORM_SLOTS), float("nan"), device=DEV)
        engine.gemm_bf16(xh, xh, epilogue=_lib.SM_EPI_F32_NORM | sym, out0=out, partials=partials, **kw)
        torch.testing.assert_close(partials.double().sum(1), want.square().sum((1, 2)), rtol=1e-5, atol=0)
    assert _lib.device_status(DEV) == 0


@pytest.mark.parametrize("m", [256, 1024])
def test_pair_block_row_tiles_match_square_tiles(m):
    """Equal up to FP32 rounding: a mirrored block adds the two compensation
    products (hi*lo, lo*hi) in the other order than a directly computed one."""
    x = rnd(2, m, 384, seed=28)
    xh, xl = split(x)
    outs = []
    for bn128 in (False, True):
        out = torch.full((2, m, m), float("nan"), device=DEV)
        engine.gemm_bf16(xh, xh, a_lo=xl, b_lo=xl, pair=True, bn128=bn128,
                         epilogue=_lib.SM_EPI_F32 | _lib.SM_EPI_SYMMETRIC, out0=out)
        outs.append(out)
    assert rel(outs[1], outs[0]) < 1e-6


@pytest.mark.parametrize("bn128", [False, True])
@pytest.mark.parametrize("comp", [False, True])
def test_pair_symmetric_poly_epilogues(comp, bn128):
    g = rnd(2, 512, 512, seed=27, scale=0.05)
    g = (g + g.transpose(1, 2)) / 2
    gh, gl = split(g)
    a, b, c = 3.28, -2.41, 0.486
    out = torch.full_like(gh, float("nan"))
    if comp:
        out_lo = torch.full_like(gh, float("nan"))
        engine.gemm_bf16(gh, gh, a_lo=gl, b_lo=gl, pair=True, bn128=bn128,
                         epilogue=_lib.SM_EPI_POLY_HILO | _lib.SM_EPI_SYMMETRIC,
                         out0=out, out1=out_lo, aux=gh, aux_lo=gl, poly=(a, b, c))
        gd = gh.double() + gl.double()
        got, tol = out.float() + out_lo.float(), 2e-5
    else:
        engine.gemm_bf16(gh, gh, pair=True, bn128=bn128, epilogue=_lib.SM_EPI_POLY | _lib.SM_EPI_SYMMETRIC,
                         out0=out, aux=gh, poly=(a, b, c))
        gd = gh.double()
        got, tol = out.float(), 4e-3
    want = a * torch.eye(512, device=DEV, dtype=torch.float64) + b * gd + c * torch.bmm(gd, gd.transpose(1, 2))
    assert rel(got, want) < tol
    assert _lib.device_status(DEV) == 0


def test_pair_rejects_unaligned_rows():
    a = torch.zeros(1, 384, 64, device=DEV, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="M%256"):
        engine.gemm_bf16(a, a, pair=True, out0=torch.empty(1, 384, 384, device=DEV))


@pytest.mark.parametrize("comp", [False, True])
def test_pair_narrow_mn_major_b(comp):
    """P X on 256 x 128 pair tiles (each CTA stages one 64-column chunk of an
    MN-major B), the tiling a plan may pick for P X at small batches."""
    p = rnd(3, 512, 384, seed=31)
    x = rnd(3, 384, 640, seed=32)
    ph, pl = split(p)
    xh, xl = split(x)
    out = torch.full((3, 512, 640), float("nan"), device=DEV)
    kw = dict(a_lo=pl, b_lo=xl) if comp else {}
    engine.gemm_bf16(ph, xh, b_kmajor=False, pair=True, bn128=True, epilogue=_lib.SM_EPI_F32, out0=out, **kw)
    if comp:
        want = torch.bmm(p.double(), x.double())
        assert rel(out, want) < 2e-5
    else:
        want = torch.bmm(ph.float(), xh.float())
        assert rel(out, want) < 1e-5
    assert _lib.device_status(DEV) == 0
