"""The historical split_sides option (reproduction/odl/optim/diagonal_weighted_pe.py:
408-410, 500-543): the rank-one whitening and mapback act on the activation
side only (the cotangent side has no rank-one term), with the transposed
matrices of a shape group batched first.

CPU: the oracle's one-sided restatement gives the same step as its two-sided
path (the rank-one action with a zero vector is the identity).  GPU: the B200
optimizer's kernels always apply the rank-one action on the activation side
alone, so RankOneAWeightedPE(split_sides=True) and (split_sides=False) give
bitwise identical weights, within the parity bar of the oracle's one-sided
step (1e-2 relative Frobenius error, cosine >= 0.999)."""
import numpy as np
import pytest
import torch
from torch import nn

from oracle import sandmuon_oracle as orc

SHAPES = [(96, 64), (64, 96), (64, 96), (80, 80), (200, 64)]


def _inputs(seed=3):
    rng = np.random.default_rng(seed)
    names = [f"m{i}" for i in range(len(SHAPES))]
    weights = {n: (rng.standard_normal(s) * 0.02).astype(np.float32) for n, s in zip(names, SHAPES)}
    stats, grads = {}, {}
    for n, (d_out, d_in) in zip(names, SHAPES):
        rows = 512
        mean, std = rng.normal(.1, .05, d_in), np.exp(rng.normal(0, .5, d_in))
        stats[n] = dict(a_sum=(rows * (mean ** 2 + std ** 2)).astype(np.float32),
                        a_first_sum=(rows * mean).astype(np.float32), a_count=rows,
                        b_sum=(rows * (1e-3 * np.exp(rng.normal(0, .5, d_out))) ** 2).astype(np.float32),
                        b_count=rows)
        grads[n] = (rng.standard_normal((d_out, d_in)) * 1e-4).astype(np.float32)
    return names, weights, stats, grads


def _oracle_directions(split_sides, steps=2):
    names, weights, stats, grads = _inputs()
    oracle = orc.OracleSandMuon(dict(zip(names, SHAPES)), {n: n for n in names}, rank_one_a=True, lr=1e-2,
                                split_sides=split_sides)
    out = []
    for _ in range(steps):
        for n in names:
            oracle.inject(n, **stats[n])
        d = {}
        oracle.step(weights, grads, directions_out=d)
        out.append(d)
    return names, out


def test_oracle_one_sided_path_equals_two_sided():
    names, one = _oracle_directions(True)
    _, two = _oracle_directions(False)
    for step in range(2):
        for n in names:
            a, b = one[step][n].astype(np.float64), two[step][n].astype(np.float64)
            assert np.linalg.norm(a - b) / np.linalg.norm(b) < 1e-5, (step, n)


def test_split_sides_keyword_is_accepted_on_cpu_models():
    from sandmuon_b200 import RankOneAWeightedPE
    model = nn.Sequential(nn.Linear(8, 4, bias=False))
    opt = RankOneAWeightedPE(model, lr=1e-3, split_sides=True)
    assert opt.split_sides is True
    opt.close()


@pytest.mark.gpu
def test_engine_split_sides_matches_oracle_and_two_sided_run():
    from sandmuon_b200 import RankOneAWeightedPE, _lib
    from sandmuon_b200.workloads import inject_statistics
    dev = torch.device("cuda:0")
    names, weights, stats, grads = _inputs()
    _, want = _oracle_directions(True)
    results = []
    for split in (True, False):
        model = nn.Sequential(*[nn.Linear(i, o, bias=False) for o, i in SHAPES]).to(dev)
        opt = RankOneAWeightedPE(model, lr=1e-2, split_sides=split)
        params = list(opt.named_matrices.values())
        with torch.no_grad():
            for p, n in zip(params, names):
                p.copy_(torch.from_numpy(weights[n]))
        for step in range(2):
            for p, n in zip(params, names):
                p.grad = torch.from_numpy(grads[n]).to(dev)
            inject_statistics(opt, {pn: stats[n] for pn, n in zip(opt.named_matrices, names)})
            before = [p.detach().clone() for p in params]
            opt.step()
            if split:
                for p, b, n in zip(params, before, names):
                    d = ((b - p.detach()) / 1e-2).double().cpu().numpy()
                    ref = want[step][n].astype(np.float64)
                    rel = np.linalg.norm(d - ref) / np.linalg.norm(ref)
                    cos = float((d * ref).sum() / (np.linalg.norm(d) * np.linalg.norm(ref)))
                    assert rel < 1e-2 and cos > 0.999, (step, n, rel, cos)
        results.append([p.detach().cpu().clone() for p in params])
        assert _lib.device_status(dev) == 0
        opt.close()
    for a, b in zip(*results):
        assert torch.equal(a, b)
