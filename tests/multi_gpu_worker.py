"""Worker for tests/test_gpu_multi.py: one rank of a sharded optimizer step.

Launched by torch.distributed.run (one process per GPU, any world size) with
the output directory, the partition ("lpt" / "layer"), the exchange
("weights" / "bf16_delta") and optionally "reduce" and "nccl" (the weight
exchange by NCCL all-gather instead of peer stores from the update kernel).  Every rank builds the
same mini GPT-named model, injects the same statistics and gradients (with
"reduce": rank-dependent gradients averaging to them, which the optimizer
reduces itself), runs STEPS sharded steps (statistic all-reduce, owned-matrix
S8, exchange) and saves its weights and consolidated momentum buffers to
<out_dir>/rank<r>.pt (rank 0 also the initial weights to init.pt).

oracle_run() replays the same inputs through the CPU oracle (the numpy
restatement of the reference step): every rank injects the same sums, so the
all-reduced statistics normalise to the single-rank ones.
"""
import datetime
import os
import sys
from pathlib import Path

import numpy as np
import torch
import torch.distributed as dist

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

LAYERS, WIDTH, HIDDEN, COUNT, STEPS, SEED, LR = 3, 256, 1024, 4096, 2, 5, 1e-2


def _inputs(opt, model, rng):
    """One step's statistics (accumulated sums) and gradients, drawn in a
    fixed order from `rng`."""
    from sandmuon_b200.workloads import synth_gpt_statistics
    stats = synth_gpt_statistics(opt, rng, count=COUNT, inject=False)
    grads = {n: (rng.standard_normal(tuple(p.shape)) * 1e-4).astype(np.float32) for n, p in model.named_parameters()}
    return stats, grads


def oracle_run():
    """(initial weights, weights after STEPS oracle steps, the oracle's state)."""
    from oracle import sandmuon_oracle as orc
    from sandmuon_b200 import RankOneAWeightedPE
    from sandmuon_b200.workloads import gpt_matrix_model
    torch.manual_seed(SEED)
    model = gpt_matrix_model(LAYERS, WIDTH, HIDDEN)        # CPU: only names, shapes and the q/k/v rule
    opt = RankOneAWeightedPE(model, lr=LR)
    sources = {n: opt.parameter_names[id(opt.a_sources[id(p)])] for n, p in opt.named_matrices.items()}
    oracle = orc.OracleSandMuon({n: tuple(p.shape) for n, p in opt.named_matrices.items()}, sources,
                                rank_one_a=True, lr=LR)
    init = {n: p.detach().numpy().copy() for n, p in model.named_parameters()}
    weights = {n: w.copy() for n, w in init.items()}
    rng = np.random.default_rng(SEED)
    for _ in range(STEPS):
        stats, grads = _inputs(opt, model, rng)
        for n in opt.named_matrices:
            oracle.inject(n, **stats[n])
        oracle.step(weights, grads)
    opt.close()
    return init, weights, oracle.state


def main(out_dir: str, partition: str, exchange: str, reduce: bool, transport: str = "auto"):
    from sandmuon_b200 import RankOneAWeightedPE
    from sandmuon_b200.workloads import gpt_matrix_model, inject_statistics
    rank = int(os.environ["RANK"])
    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=device)
    try:
        torch.manual_seed(SEED)
        model = gpt_matrix_model(LAYERS, WIDTH, HIDDEN).to(device)
        if rank == 0:
            torch.save({n: p.detach().cpu() for n, p in model.named_parameters()}, Path(out_dir) / "init.pt")
        opt = RankOneAWeightedPE(model, lr=LR, process_group=dist.group.WORLD, partition=partition,
                                 exchange=exchange, reduce_gradients=reduce, transport=transport)
        rng = np.random.default_rng(SEED)
        world = dist.get_world_size()
        for _ in range(STEPS):
            stats, grads = _inputs(opt, model, rng)
            inject_statistics(opt, stats)
            for n, p in model.named_parameters():
                g = grads[n]
                if reduce:  # rank-dependent gradients whose average over the ranks is g
                    g = g * np.float32(2.0 * (rank + 1) / (world + 1))
                p.grad = torch.from_numpy(g).to(device)
            opt.step()
        torch.cuda.synchronize()
        from sandmuon_b200 import _lib
        out = {n: p.detach().cpu() for n, p in model.named_parameters()}
        state = opt.consolidated_state_dict()
        names = [n for n, _ in model.named_parameters()]
        for i, st in state["state"].items():
            if "momentum_buffer" in st:
                out[names[i] + "/momentum"] = st["momentum_buffer"].detach().cpu()
        out["/device_status"] = torch.tensor(_lib.device_status(device))
        out["/owned"] = torch.tensor(sum(opt.sharding.owns(p) for p in opt.named_matrices.values()))
        out["/peer"] = torch.tensor(1 if opt.sharding.peer_bases else 0)
        torch.save(out, Path(out_dir) / f"rank{rank}.pt")
        opt.close()
        dist.barrier()
    finally:
        dist.destroy_process_group()


if __name__ == "__main__":
    extra = sys.argv[4:]
    main(sys.argv[1], sys.argv[2] if len(sys.argv) > 2 else "lpt", sys.argv[3] if len(sys.argv) > 3 else "weights",
         "reduce" in extra, "nccl" if "nccl" in extra else "auto")
