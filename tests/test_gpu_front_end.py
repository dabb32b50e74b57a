"""The one-pass whitening front end on shapes chosen for its edge cases.

From a plan's second step on, the front end is one pass: the untransposed
matrices (d_out <= d_in) stream their rows through teams of 1, 2, 4 or 8
warps (chosen by the row length), the transposed ones stream 16-row blocks
whose columns become 32-byte pieces of X rows.
These runs step several times, so every step after the first goes through
that pass, and compare every step's update direction, and the final momenta
and statistic EMAs, with the CPU oracle (bars: direction 1e-2 relative
Frobenius error and cosine >= 0.999; state 1e-5).

Shapes: row lengths whose float4 count sits just above a team-size boundary
(257, 513, 1025 float4 -> 2, 4, 8 warps with ragged last columns), a row of
6 float4 (most of a warp idle), several matrices of one shape (CTA row ranges
that cross matrix boundaries), transposed matrices whose row counts leave a
ragged last block and whose float4 counts leave idle lanes, and the widest
config-4 row (8192).
"""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import sandmuon_oracle as orc
from sandmuon_b200 import DiagonalWeightedPE, RankOneAWeightedPE, _lib

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
DIR_REL, DIR_COS, STAT_REL = 1e-2, 0.999, 1e-5


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def cos(a, b):
    a, b = np.asarray(a, np.float64).ravel(), np.asarray(b, np.float64).ravel()
    return float(a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300))


def npy(t):
    return t.detach().float().cpu().numpy()


def run_steps(shapes, rank1, steps, seed, count=4096):
    """`steps` optimizer steps of a Sequential of bias-free Linear layers of
    the given (d_out, d_in) shapes, each with fresh statistics and gradients,
    against the oracle; returns the worst direction errors per step."""
    from sandmuon_b200.workloads import synth_gpt_statistics
    torch.manual_seed(seed)
    model = nn.Sequential(*[nn.Linear(i, o, bias=False) for o, i in shapes]).to(DEV)
    opt = (RankOneAWeightedPE if rank1 else DiagonalWeightedPE)(model, lr=1e-2)
    names = list(opt.named_matrices)
    oracle = orc.OracleSandMuon({n: tuple(p.shape) for n, p in opt.named_matrices.items()}, {n: n for n in names},
                                rank_one_a=rank1, lr=1e-2)
    rng = np.random.default_rng(seed)
    weights = {n: npy(p) for n, p in opt.named_matrices.items()}
    worst = []
    for step in range(steps):
        stats = synth_gpt_statistics(opt, rng, count=count)
        grads = {}
        for n, p in opt.named_matrices.items():
            grads[n] = (rng.standard_normal(tuple(p.shape)) * 1e-4).astype(np.float32)
            p.grad = torch.from_numpy(grads[n]).to(DEV)
            oracle.inject(n, **stats[n])
        before = {n: npy(p) for n, p in opt.named_matrices.items()}
        ref_before = dict(weights)
        oracle.step(weights, grads)
        opt.step()
        w_rel, w_cos = 0.0, 1.0
        for n in names:
            d_gpu = (before[n] - npy(opt.named_matrices[n])) / 1e-2
            d_ref = (ref_before[n] - weights[n]) / 1e-2
            w_rel, w_cos = max(w_rel, rel(d_gpu, d_ref)), min(w_cos, cos(d_gpu, d_ref))
            assert rel(d_gpu, d_ref) < DIR_REL and cos(d_gpu, d_ref) > DIR_COS, (step, n, rel(d_gpu, d_ref))
        worst.append((w_rel, w_cos))
    for n in names:
        st = opt.state[opt.named_matrices[n]]
        assert rel(npy(st["momentum_buffer"]), oracle.state[n]["momentum_buffer"]) < STAT_REL, n
        assert rel(npy(st["b_ema"]), oracle.state[n]["b_ema"]) < STAT_REL, n
    assert _lib.device_status(DEV) == 0
    opt.close()
    return worst


@pytest.mark.parametrize("variant", ["rank1", "diag"])
def test_row_stream_team_sizes_follow_oracle(variant):
    shapes = [
        (16, 24),                  # 6 float4 per row: one warp, most lanes idle
        (100, 1028), (100, 1028),  # 257 float4: two warps; ranges cross the matrix boundary
        (1028, 100),               # transposed partner of the same shape group
        (60, 2052),                # 513 float4: four warps
        (40, 4100), (40, 4100),    # 1025 float4: eight warps
        (96, 96), (96, 96), (96, 96),
        (40, 12), (40, 12),        # transposed, 3 float4 per row: most of a half idle, ragged last block
    ]
    run_steps(shapes, variant == "rank1", steps=3, seed=11)


def test_row_stream_widest_config4_row_follows_oracle():
    """The config-4 c_proj row (8192 float32: eight warps, 8 float4 each)
    beside its transposed c_fc partner, two steps."""
    run_steps([(256, 8192), (8192, 256)], True, steps=2, seed=12)


def test_row_stream_many_rows_per_cta_follows_oracle():
    """More rows than the grid has CTAs (48 x 256 rows of 64 float4): each CTA
    walks a range of several rows, many of them across a matrix boundary."""
    run_steps([(256, 256)] * 48, True, steps=2, seed=13)
