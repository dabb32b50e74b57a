"""CUDA kernels against the numpy oracle: hook statistics (N1), the S8 map
(stage 1 compensated BF16, stages 2-5 BF16), and multi-tensor AdamW (N8).

Tolerances: statistics 1e-5 relative (north_star); S8 output 1e-2 relative
Frobenius error and cosine >= 0.999 against the FP32 oracle."""
from pathlib import Path

import numpy as np
import pytest
import torch

from oracle import sandmuon_oracle as orc
from sandmuon_b200 import _lib, engine

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLDEN = Path(__file__).resolve().parent / "golden"


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30)


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


# ----------------------------------------------------------------- statistics

@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16, torch.float64])
@pytest.mark.parametrize("shape", [(2048, 768), (16384, 3072), (37, 5), (1, 768), (3, 4), (1000, 123)])
def test_column_stats_match_oracle(dtype, shape):
    g = torch.Generator().manual_seed(hash(shape) % 1000)
    n, c = shape
    x = (torch.randn(n, c, generator=g) * torch.exp(torch.randn(c, generator=g) * .5) + .1).to(dtype)
    sq = torch.full((c,), 0.5, device=DEV)
    s1 = torch.full((c,), -0.25, device=DEV)
    engine.accumulate_column_stats(x.to(DEV), sq, s1)
    want_sq, want_s = orc.column_stats(x.float().numpy(), True)
    assert rel(sq.cpu().numpy() - 0.5, want_sq) < 1e-5
    assert rel(s1.cpu().numpy() + 0.25, want_s) < 1e-5


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("rows,cols,stride", [(16384, 768, 768), (300, 512, 520), (200000, 32, 40),
                                              (5, 100000, 100000), (16385, 776, 784), (2, 8, 8)])
def test_column_stats_cluster_path(dtype, rows, cols, stride):
    """Contiguous 16-byte-aligned rows below the TMA size take the one-launch
    cluster reduction: padded row strides, a slab wider than the columns,
    very tall and very wide inputs, odd row counts; twice in a row."""
    g = torch.Generator().manual_seed(rows * 7 + cols)
    base = (torch.randn(rows, stride, generator=g) * torch.exp(torch.randn(stride, generator=g) * .5) + .3).to(dtype)
    x = base.to(DEV)[:, :cols]
    sq = torch.zeros(cols, device=DEV)
    s1 = torch.zeros(cols, device=DEV)
    for _ in range(2):
        engine.accumulate_column_stats(x, sq, s1)
    want_sq, want_s = orc.column_stats(base[:, :cols].float().numpy(), True)
    assert rel(sq.cpu().numpy(), 2 * want_sq) < 1e-5
    assert rel(s1.cpu().numpy(), 2 * want_s) < 1e-5
    assert _lib.device_status(DEV) == 0


def test_column_stats_strided_and_transposed_views():
    base = torch.randn(300, 200, device=DEV)
    for view in (base[:, ::2], base.t(), base[10:250, 7:190]):
        sq = torch.zeros(view.shape[1], device=DEV)
        s1 = torch.zeros(view.shape[1], device=DEV)
        engine.accumulate_column_stats(view, sq, s1)
        want_sq, want_s = orc.column_stats(view.cpu().numpy(), True)
        assert rel(sq.cpu().numpy(), want_sq) < 1e-5
        assert rel(s1.cpu().numpy(), want_s) < 1e-5


def test_column_stats_empty_rows_is_noop_and_deterministic():
    sq = torch.ones(8, device=DEV)
    engine.accumulate_column_stats(torch.empty(0, 8, device=DEV), sq)
    assert torch.equal(sq, torch.ones(8, device=DEV))
    x = torch.randn(5000, 768, device=DEV)
    a, b = torch.zeros(768, device=DEV), torch.zeros(768, device=DEV)
    engine.accumulate_column_stats(x, a)
    engine.accumulate_column_stats(x, b)
    assert torch.equal(a, b)


def _stats_call(lib, x, sq, s1, ws):
    import ctypes
    return lib.sm_stats_accumulate(
        ctypes.c_void_p(x.data_ptr()), _lib.DTYPE_CODES[x.dtype], x.shape[0], x.shape[1], x.stride(0), x.stride(1),
        ctypes.c_void_p(sq.data_ptr()), ctypes.c_void_p(0 if s1 is None else s1.data_ptr()),
        ctypes.c_void_p(ws.data_ptr()), ws.numel(), ctypes.c_void_p(torch.cuda.current_stream(DEV).cuda_stream))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float64])
@pytest.mark.parametrize("cols,stride", [(700, 768), (776, 776), (1280, 1536), (3072, 3072)])
def test_column_stats_tma_path_any_workspace_contents(dtype, cols, stride):
    """Inputs of 128 MB and more with contiguous 16-byte-aligned rows take the
    single-reduction-launch TMA kernel: ragged row blocks and column groups,
    padded row strides, and a workspace of arbitrary bytes (the call zeroes
    its tickets), over three calls in a row on the same workspace."""
    lib = _lib.load()
    _lib.ensure_device(DEV)
    size = torch.tensor([], dtype=dtype).element_size()
    rows = (140 << 20) // (cols * size) + 7
    g = torch.Generator().manual_seed(rows + cols)
    base = (torch.randn(rows, stride, generator=g) * 1.5 + .2).to(dtype)
    x = base.to(DEV)[:, :cols]
    nbytes = lib.sm_stats_workspace_bytes(rows, cols)
    ws = torch.randint(0, 256, (nbytes,), dtype=torch.uint8, generator=g).to(DEV)
    sq = torch.zeros(cols, device=DEV)
    s1 = torch.zeros(cols, device=DEV)
    for _ in range(3):
        assert _stats_call(lib, x, sq, s1, ws) == 0
    want_sq, want_s = orc.column_stats(base[:, :cols].float().numpy(), True)
    assert rel(sq.cpu().numpy(), 3 * want_sq) < 1e-5
    assert rel(s1.cpu().numpy(), 3 * want_s) < 1e-5
    assert _lib.device_status(DEV) == 0


# ------------------------------------------------------------------------ S8

@pytest.mark.parametrize("case", range(8))
def test_s8_matches_reference_golden(case):
    g = dict(np.load(GOLDEN / "s8.npz"))
    x, want = g[f"s8_in_{case}"], g[f"s8_out_{case}"]
    got = engine.s8_polar(torch.from_numpy(x).to(DEV)).cpu().numpy()
    for b in range(x.shape[0]):
        assert rel(got[b], want[b]) < 1e-2, (case, b, rel(got[b], want[b]))
        assert cos(got[b], want[b]) > 0.999


def test_s8_zero_matrices_give_exact_zeros():
    x = torch.randn(3, 40, 24, device=DEV)
    x[1].zero_()
    got = engine.s8_polar(x)
    assert torch.equal(got[1], torch.zeros_like(got[1]))
    assert torch.isfinite(got).all()
    z = engine.s8_polar(torch.zeros(1, 4, 3, device=DEV))
    assert torch.equal(z, torch.zeros_like(z))


def spiked(batch, rows, cols, seed):
    """cfg3-style matrices: N(0,1) columns scaled by LogNormal(0,1), plus a
    rank-1 spike of norm 10 x sigma_max."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((batch, rows, cols)).astype(np.float32) * np.exp(rng.standard_normal(cols)).astype(np.float32)
    for b in range(batch):
        smax = np.linalg.norm(x[b], 2)
        u = rng.standard_normal(rows); v = rng.standard_normal(cols)
        x[b] += (10 * smax * np.outer(u / np.linalg.norm(u), v / np.linalg.norm(v))).astype(np.float32)
    return x


@pytest.mark.parametrize("shape", [(4, 256, 256), (2, 384, 1024), (2, 1024, 384), (2, 768, 768), (1, 300, 517)])
def test_s8_cfg3_style_matrices_match_oracle(shape):
    x = spiked(*shape, seed=sum(shape))
    got = engine.s8_polar(torch.from_numpy(x).to(DEV)).cpu().numpy()
    want = orc.s8_fp32(x)
    for b in range(shape[0]):
        assert rel(got[b], want[b]) < 1e-2, rel(got[b], want[b])
        assert cos(got[b], want[b]) > 0.999


# --------------------------------------------------------------------- AdamW

def test_adamw_matches_oracle_over_steps():
    rng = np.random.default_rng(5)
    shapes = [(50257 // 64, 64), (1024,), (3,), (768, 33)] + [(17,)] * 30  # > one launch batch
    opt = orc.OracleSandMuon({}, {}, [f"p{i}" for i in range(len(shapes))], rank_one_a=True, lr=3e-3)
    w_np = {f"p{i}": rng.standard_normal(s).astype(np.float32) for i, s in enumerate(shapes)}
    params = [torch.from_numpy(w_np[f"p{i}"].copy()).to(DEV) for i in range(len(shapes))]
    m1 = [torch.zeros_like(p) for p in params]
    m2 = [torch.zeros_like(p) for p in params]
    for step in range(1, 4):
        grads = {f"p{i}": rng.standard_normal(s).astype(np.float32) for i, s in enumerate(shapes)}
        opt.step(w_np, grads)
        items = [engine.AdamItem(p, torch.from_numpy(grads[f"p{i}"]).to(DEV), a, b, step)
                 for i, (p, a, b) in enumerate(zip(params, m1, m2))]
        engine.adamw_multi(items, lr=3e-3 * .1, beta1=.9, beta2=.999, eps=1e-8, weight_decay=.01)
        for i, p in enumerate(params):
            np.testing.assert_allclose(p.cpu().numpy(), w_np[f"p{i}"], rtol=2e-6, atol=2e-7)


def test_device_status_clean_after_kernels():
    assert _lib.device_status(DEV) == 0
