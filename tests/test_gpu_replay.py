"""Graph replay of the optimizer step: from its second step on, a plan runs its
kernels as one captured CUDA graph.  Replayed steps must give bit-identical
weights, momenta and statistics to the same steps launched kernel by kernel,
including when the gradients' alignment changes between steps (the graph is
re-captured with the other kernel variants)."""
import numpy as np
import pytest
import torch

from sandmuon_b200 import RankOneAWeightedPE
from sandmuon_b200.workloads import gpt_matrix_model, synth_gpt_statistics

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


def run(replay: bool, steps: int = 5):
    torch.manual_seed(11)
    model = gpt_matrix_model(2, 256, 1024).to(DEV)
    opt = RankOneAWeightedPE(model, lr=1e-2)
    rng = np.random.default_rng(11)
    names = list(opt.named_matrices)
    total = sum(p.numel() for p in opt.named_matrices.values())
    # step 3 reads gradients 4 bytes past a 16-byte boundary: the scalar
    # (non-vectorised) kernel variants, so the graph is captured anew
    spare = torch.empty(total + 4, dtype=torch.float32, device=DEV)
    for step in range(steps):
        synth_gpt_statistics(opt, rng, count=2048)
        off = 1 if step == 3 else 0
        for n in names:
            p = opt.named_matrices[n]
            g = torch.from_numpy((rng.standard_normal(tuple(p.shape)) * 1e-4).astype(np.float32))
            if off:
                view = spare[off:off + p.numel()].view(p.shape)
                view.copy_(g)
                p.grad = view
                off += p.numel()
            else:
                p.grad = g.to(DEV)
        opt.step()
        if step == 0 and not replay:
            opt._last_plan.set_replay(False)
    torch.cuda.synchronize()
    out = {n: p.detach().cpu().clone() for n, p in opt.named_matrices.items()}
    for n, p in opt.named_matrices.items():
        st = opt.state[p]
        out[n + "/momentum"] = st["momentum_buffer"].cpu().clone()
        out[n + "/b_ema"] = st["b_ema"].cpu().clone()
        if "a_ema" in st:
            out[n + "/a_ema"] = st["a_ema"].cpu().clone()
    launches = opt._last_plan.launches_per_step()
    opt.close()
    return out, launches


def test_replayed_steps_match_eager_steps_bitwise():
    graph, n_graph = run(True)
    eager, n_eager = run(False)
    assert n_graph == n_eager > 0
    assert graph.keys() == eager.keys()
    for k in graph:
        assert torch.equal(graph[k], eager[k]), k
