"""Every rank's share of a sharded config-1 step, on one GPU, against the oracle.

A sharded optimizer on rank r of N runs the plan of the matrices r owns: its
own shape-group batches (at N = 8 with the LPT partition, 3 or 5 of the 768^2
group and 2 or 3 of the 768 x 3072 group, sizes N <= 4 never builds), GEMM
launch sets whose tile counts fall below the resident CTA pairs, and its own
tile schedules.  This test builds exactly those per-rank plans on one GPU.
It swaps the process group for a test-only single-process view, which owns
what rank r owns, leaves the statistics as they are (every rank holds the
group's summed statistics after the all-reduce), and exchanges nothing.
Every owned matrix's update direction is compared with the oracle's step on
the same inputs (1e-2 relative Frobenius error, cosine >= 0.999).  Matrices
the rank does not own stay untouched, and the all-gather send slot holds what
the exchange would ship: the updated FP32 weight, or the BF16 delta the owner
subtracted.
"""
import numpy as np
import pytest
import torch

from oracle import sandmuon_oracle as orc
from sandmuon_b200 import RankOneAWeightedPE, _lib
from sandmuon_b200.distributed import partition_matrices

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
LR = 1e-2
DIR_REL, DIR_COS = 1e-2, 0.999


class _RankView:
    """Test-only stand-in for MatrixSharding on rank `rank` of `world`: the
    same ownership and send slots, no collectives."""

    def __init__(self, opt, world, rank, partition, exchange):
        self.rank, self.world = rank, world
        self.exchange_mode = exchange
        shapes = {n: tuple(p.shape) for n, p in opt.named_matrices.items()}
        owner = partition_matrices(shapes, world, partition)
        self._owner = {id(opt.named_matrices[n]): r for n, r in owner.items()}
        dtype = torch.bfloat16 if exchange == "bf16_delta" else torch.float32
        self.slots = {id(p): torch.zeros(p.shape, dtype=dtype, device=DEV)
                      for p in opt.named_matrices.values() if self.owns(p)}

    def owns(self, p):
        return self._owner[id(p)] == self.rank

    @property
    def export_mode(self):
        return _lib.SM_EXPORT_BF16_DELTA if self.exchange_mode == "bf16_delta" else _lib.SM_EXPORT_WEIGHTS

    def send_slot(self, p):
        return self.slots[id(p)]

    def reduce_statistics(self, tensors, counts):
        return None

    def exchange(self, matrix_items):
        pass

    peer_bases = []  # no peer delivery: the step writes the send slots

    def close(self):
        pass


@pytest.fixture(scope="module")
def cfg1():
    """Config-1 weights, gradients and statistics, and the oracle's step."""
    from sandmuon_b200.workloads import gpt_matrix_model, synth_gpt_statistics
    torch.manual_seed(1337)
    model = gpt_matrix_model(9, 768, 3072)
    opt = RankOneAWeightedPE(model.to(DEV), lr=LR)
    rng = np.random.default_rng(1337)
    stats = synth_gpt_statistics(opt, rng, count=8 * 16384, inject=False)
    names = list(opt.named_matrices)
    weights = {n: (rng.standard_normal(tuple(p.shape)) * 0.02).astype(np.float32)
               for n, p in opt.named_matrices.items()}
    grads = {n: (rng.standard_normal(tuple(p.shape)) * 1e-4).astype(np.float32)
             for n, p in opt.named_matrices.items()}
    sources = {n: opt.parameter_names[id(opt.a_sources[id(p)])] for n, p in opt.named_matrices.items()}
    oracle = orc.OracleSandMuon({n: tuple(p.shape) for n, p in opt.named_matrices.items()}, sources,
                                rank_one_a=True, lr=LR)
    for n in names:
        oracle.inject(n, **stats[n])
    after = {n: w.copy() for n, w in weights.items()}
    oracle.step(after, grads)
    directions = {n: (weights[n].astype(np.float64) - after[n]) / LR for n in names}
    opt.close()
    del opt, model
    return stats, weights, grads, directions


def _rel_cos(d, ref):
    d, ref = d.ravel(), ref.ravel()
    rel = float(np.linalg.norm(d - ref) / np.linalg.norm(ref))
    cos = float(d @ ref / (np.linalg.norm(d) * np.linalg.norm(ref)))
    return rel, cos


@pytest.mark.parametrize("world,partition,exchange", [
    (8, "lpt", "weights"), (8, "layer", "weights"), (4, "lpt", "weights"), (4, "layer", "weights"),
    (8, "lpt", "bf16_delta"),
])
def test_each_rank_plan_matches_oracle(cfg1, world, partition, exchange):
    from sandmuon_b200.workloads import gpt_matrix_model, inject_statistics
    stats, weights, grads, directions = cfg1
    model = gpt_matrix_model(9, 768, 3072).to(DEV)
    opt = RankOneAWeightedPE(model, lr=LR)
    params = opt.named_matrices
    owned_total = 0
    for rank in range(world):
        view = _RankView(opt, world, rank, partition, exchange)
        opt._sharding = view
        opt.state.clear()
        for plan in opt._plans.values():
            plan.close()
        opt._plans.clear()
        with torch.no_grad():
            for n, p in params.items():
                p.copy_(torch.from_numpy(weights[n]))
                p.grad = torch.from_numpy(grads[n]).to(DEV)
        inject_statistics(opt, stats)
        opt.step()
        torch.cuda.synchronize(DEV)
        owned = [n for n, p in params.items() if view.owns(p)]
        assert owned, (world, partition, rank)
        owned_total += len(owned)
        for n, p in params.items():
            w_after = p.detach().cpu().numpy()
            if not view.owns(p):
                assert np.array_equal(w_after, weights[n]), (rank, n, "a matrix the rank does not own changed")
                continue
            rel, cos = _rel_cos((weights[n].astype(np.float64) - w_after) / LR, directions[n])
            assert rel < DIR_REL and cos > DIR_COS, (world, partition, rank, n, rel, cos)
            slot = view.slots[id(p)]
            if exchange == "weights":
                assert torch.equal(slot, p.detach()), (rank, n)
            else:
                expect = torch.from_numpy(weights[n]).to(DEV) - slot.float()
                assert torch.equal(expect, p.detach()), (rank, n)
        assert _lib.device_status(DEV) == 0, (world, partition, rank)
    assert owned_total == len(params)
    opt.close()
